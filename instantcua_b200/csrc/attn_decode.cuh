// Decode attention: per-head QK RMSNorm + RoPE + KV append fused with split-K GQA flash-decode.
//
// Replaces the tail of the reference k_attn_in (per-head RMSNorm(128), rotate-half RoPE from the
// cos/sin table, fp16 K/V write at `pos`, Shaders.swift:790-834) and k_attention (softmax over
// the whole context in threadgroup memory, context <= 2048, Shaders.swift:1219-1289).
//
// Design (B200): the context of each kv head is split over n_split CTAs grouped in thread-block
// clusters; each CTA handles the two query heads of its GQA group, so every K/V byte is read once.
// Each warp streams its own contiguous run of cache rows through a ring of shared-memory slots
// with 1-D bulk copies (the first slots are requested before griddepcontrol.wait: cache rows
// [0, pos) do not depend on the previous kernel) and runs an online softmax in registers.  Warp
// results meet in shared memory, CTA results meet across the cluster through distributed shared
// memory, and each cluster writes one (max, sum, output) part that the o-proj GEMV folds in while
// loading its input.  The new position is normalised, rotated and rounded to the cache type in the
// CTA (as the reference reads it back from the fp16 cache) and folded in by the last split.  No
// global atomics, fences or spin waits.  Context length is bounded only by the cache allocation.
#pragma once
#include "common.cuh"
#include "gemv.cuh"

namespace icua {

constexpr int ATT_SLOT = 16;   // cache rows per ring slot (one MMA block)
constexpr int ATT_NS = 2;      // ring slots per warp
constexpr int ATT_QKV_PARTS_MAX = 8;  // split-K slices of the projection the kernel can sum

// KV rows are stored with their sixteen 16-byte chunks permuted by the row's position:
// element d of position p lives at chunk (d / 8) ^ (p & 7).  Eight consecutive rows then cover
// eight different bank groups, so ldmatrix reads from bulk-copied rows are conflict-free.
__host__ __device__ __forceinline__ int kv_swz(int d, int pos) { return (((d >> 3) ^ (pos & 7)) << 3) | (d & 7); }

template <typename KVT>
struct AttnParams {
    const float* qkv;        // raw projection [4096]: q(2048) | k(1024) | v(1024)
    const float* q_norm;     // [128]
    const float* k_norm;     // [128]
    const float2* rope;      // [max_ctx][64] (cos, sin) per cache slot
    KVT* kc;                 // this layer: [NKV][max_ctx][128] (swizzled rows)
    KVT* vc;
    int max_ctx;
    int n_split;             // CTAs per kv head (multiple of the cluster size)
    int cluster;             // CTAs per cluster
    float* part;             // out: [NKV][n_split / cluster][ATT_PART]
    DevState* st;
    L2Plan l2;               // data of later kernels to prefetch into L2
    // batched decode (blockIdx.y = row): row r uses session rows_sess[r] (state st + session,
    // cache kc / vc + session * sess_kv_elems, projection qkv + r * qkv_stride) and writes its
    // normalised output to out16[r][2048] (one part per kv head: n_split == cluster)
    const int* rows_sess;
    long long sess_kv_elems;
    long long sess_rope_elems;  // float2 entries between sessions' RoPE tables
    int qkv_stride;
    __half* out16;
    // split-K projection: the qkv rows are the sum of qkv_parts partial products qkv_part_stride
    // floats apart, added here in slice order (0 or 1: qkv holds the projection itself)
    int qkv_parts;
    long long qkv_part_stride;
    int out16_hilo;  // out16 as fp16 hi / lo row pairs (the batched GEMMs' input)
    // o-projection folded in (attn_decode_kernel<KVT, false, true>): the q4s o-proj matrix and the
    // per-kv-head partial products [NKV][2048] the next kernels add to the residual
    const uint8_t* wo;
    float* o_part;
};

// NT: query tokens per pass the layout holds (2 in the grammar-commit kernels).  CLM: largest
// cluster (16 for the kernel with the o-projection folded in, one cluster per kv head).
template <typename KVT, int NT = 1, int CLM = 8>
struct AttnSmem {
    static constexpr int row_bytes = HD * (int)sizeof(KVT);
    static constexpr int slot_bytes = 2 * ATT_SLOT * row_bytes;   // K rows then V rows
    static constexpr int ring_warp = ATT_NS * slot_bytes;
    static constexpr int ring_off = 0;
    static constexpr int new_off = 8 * ring_warp;                 // K rows, then V rows, of the new positions
    static constexpr int q_off = new_off + 2 * NT * row_bytes;    // float q[NT][2][128] (scaled)
    static constexpr int wpart_off = q_off + NT * 2 * HD * 4;     // float [8 warps][NT][ATT_PART]
    static constexpr int cpart_off = wpart_off + 8 * NT * ATT_PART * 4;  // float [CLM cluster ranks][NT][ATT_PART]
    static constexpr int bars_off = cpart_off + CLM * NT * ATT_PART * 4;
    static constexpr int total = bars_off + 8 * ATT_NS * 8 + 8;  // + the o-proj tile barrier
};

// o-projection folded into the attention (one cluster of n_split = 8 or 16 CTAs per kv head):
// CTA j of kv head h multiplies the head pair's output (256 columns of the o-proj input) by output
// rows [R j, R j + R), R = 2048 / n_split: R / 16 tiles of 16 rows x 4 q4s units of 64 columns.
// In the GEMV layout (16 K slices of 2 units) those units are slices 2h and 2h+1, and a slice's
// R / 16 tiles are one contiguous run of R / 8 units.
__host__ __device__ constexpr int att_o_run_bytes(int rows) { return (rows / 16) * 2 * icua_layout::Q4_UNIT_BYTES; }

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Split cluster barrier: arrive early, wait where it is needed (here: before the first access to a
// peer's shared memory, which requires every CTA of the cluster to have started).
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Stores a float into cluster peer `rank`'s shared memory at the address `local_ptr` has here.
__device__ __forceinline__ void st_dsmem(float* local_ptr, uint32_t rank, float v) {
    uint32_t a = smem_u32(local_ptr), ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}

// Loads a float of cluster peer `rank`'s shared memory.  Ordering against the peer's writes
// comes from the cluster barrier (release / acquire) around the combine, so the loads carry no
// memory clobber and a thread's loads can be in flight together.
__device__ __forceinline__ float ld_dsmem(const float* local_ptr, uint32_t rank) {
    uint32_t a = smem_u32(local_ptr), ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra));
    return v;
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

template <typename KVT>
__device__ __forceinline__ void mma_kv(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma_kv<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    mma_16816(d, a, b0, b1);
}
template <>
__device__ __forceinline__ void mma_kv<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename KVT>
__device__ __forceinline__ uint32_t pack2(KVT lo, KVT hi);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(__half lo, __half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(__nv_bfloat16 lo, __nv_bfloat16 hi) {
    return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
}

// hi (part 0) or lo (part 1) of v in the cache type
template <typename KVT>
__device__ __forceinline__ KVT split_part(float v, int part) {
    const KVT hi = float_to_kv<KVT>(v);
    return part ? float_to_kv<KVT>(v - kv_to_float(hi)) : hi;
}

// Warp state of the online softmax: lane (g, t) tracks query head t & 1; o holds dims
// 16*db + g (o[db][0..1], hi/lo columns) and 16*db + g + 8 (o[db][2..3]).
struct AttnAcc {
    float m, l;
    float o[8][4];
};

// One block of up to 16 cache rows (rows [0, n) of a slot whose first row is position r0) with
// tensor-core QK^T and PV.  Row addresses past n are clamped to row n-1 (finite data, p = 0).
// Two-token passes (two = true): columns 4..7 are the second token's, which sees n1 >= n rows of
// the block (the causal mask of the pass's own new rows); lanes t = 2, 3 track it.
template <typename KVT>
__device__ __forceinline__ void attn_block(uint32_t kslot, uint32_t vslot, int r0, int n, const uint32_t (&qb)[8][2],
                                           AttnAcc& acc, int lane, bool two = false, int n1 = 0) {
    constexpr int RB = HD * (int)sizeof(KVT);
    const int g = lane >> 2, t = lane & 3;
    const int nv = (two && t >= 2) ? n1 : n;  // rows this lane's column may see
    const int nmax = two ? n1 : n;
    // ---- scores S[16 rows][cols: h0 hi, h0 lo, h1 hi, h1 lo, dup x4] ----
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    {
        const int row = min((lane & 7) + ((lane >> 3) & 1) * 8, nmax - 1);
        const int key = (r0 + row) & 7;
        const uint32_t rowaddr = kslot + row * RB;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const int chunk = 2 * kk + (lane >> 4);
            uint32_t a[4];
            ldsm_x4(a, rowaddr + ((chunk ^ key) << 4));
            mma_kv<KVT>(d, a, qb[kk][0], qb[kk][1]);
        }
    }
    const bool va = g < nv, vb = g + 8 < nv;
    const float sa = va ? d[0] + d[1] : -INFINITY;
    const float sb = vb ? d[2] + d[3] : -INFINITY;
    float mb = fmaxf(sa, sb);
    mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, 4));
    mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, 8));
    mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, 16));
    const float mn = fmaxf(acc.m, mb);
    const float corr = (acc.m == -INFINITY) ? 0.f : expf(acc.m - mn);
    const float pa = va ? expf(sa - mn) : 0.f;
    const float pb = vb ? expf(sb - mn) : 0.f;
    acc.m = mn;
    acc.l = fmaf(acc.l, corr, pa + pb);
    // ---- P as the B operand: lane (g, t) needs rows 2t, 2t+1, 2t+8, 2t+9 of column g ----
    const int hh = two ? g >> 1 : (g >> 1) & 1, part = g & 1;  // column g -> lane t' = hh holds its scores
    const int src0 = (2 * t) * 4 + hh, src1 = (2 * t + 1) * 4 + hh;
    const float p0 = __shfl_sync(0xffffffffu, pa, src0);
    const float p1 = __shfl_sync(0xffffffffu, pa, src1);
    const float p8 = __shfl_sync(0xffffffffu, pb, src0);
    const float p9 = __shfl_sync(0xffffffffu, pb, src1);
    const uint32_t pb0 = pack2<KVT>(split_part<KVT>(p0, part), split_part<KVT>(p1, part));
    const uint32_t pb1 = pack2<KVT>(split_part<KVT>(p8, part), split_part<KVT>(p9, part));
    // the O columns of this lane (2t, 2t+1) belong to head t & 1, whose running max this lane keeps
    const float c = corr;
    // ---- O[16 dims x 8 cols] += V^T[dims x rows] P[rows x cols], 8 blocks of 16 dims ----
    {
        const int row = min((lane & 7) + ((lane >> 4) & 1) * 8, nmax - 1);
        const int key = (r0 + row) & 7;
        const uint32_t rowaddr = vslot + row * RB;
#pragma unroll
        for (int db = 0; db < 8; ++db) {
            const int chunk = 2 * db + ((lane >> 3) & 1);
            uint32_t a[4];
            ldsm_x4_trans(a, rowaddr + ((chunk ^ key) << 4));
#pragma unroll
            for (int i = 0; i < 4; ++i) acc.o[db][i] *= c;
            mma_kv<KVT>(acc.o[db], a, pb0, pb1);
        }
    }
}

// DUAL: the kernel of the grammar-commit engines, whose passes may carry two tokens
// (DevState::n_tok) at positions pos and pos + 1: both are normalised, rotated and appended, the
// second token's queries take MMA columns 4..7 next to the first's, so every K/V byte is still read
// once, and each token writes its own parts (token 1 after token 0's).
// FO: the o-projection is folded in (one token, q4s o-proj, one cluster of n_split = 8 or 16 CTAs
// per kv head): the cluster leader's combined output of the head pair is read by every CTA of the
// cluster through distributed shared memory, and each CTA writes the products of its 2048 / n_split
// o-proj rows with it to o_part[h] (replaces the o-proj GEMV launch and its fold of the attention
// parts; the next kernels add the eight partial vectors to the residual).
template <typename KVT, bool DUAL = false, bool FO = false>
__global__ void __launch_bounds__(256, 2) attn_decode_kernel(const AttnParams<KVT> p) {
    static_assert(!(DUAL && FO), "the folded o-projection is a one-token kernel");
    extern __shared__ __align__(128) uint8_t smem[];
    using S = AttnSmem<KVT, DUAL ? 2 : 1, FO ? 16 : 8>;
    constexpr int CLM = FO ? 16 : 8;
    constexpr int NTK = DUAL ? 2 : 1;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NSP = p.n_split;
    const int h = blockIdx.x / NSP, j = blockIdx.x % NSP;
    const int row = blockIdx.y;
    const int sess = p.rows_sess != nullptr ? p.rows_sess[row] : 0;
    DevState* const st = p.st + sess;
    const float* const qkv = p.qkv + (size_t)row * p.qkv_stride;
    KVT* const kc = p.kc + sess * p.sess_kv_elems;
    KVT* const vc = p.vc + sess * p.sess_kv_elems;
    const float2* const rope = p.rope + sess * p.sess_rope_elems;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::bars_off) + warp * ATT_NS;
    uint8_t* ring = smem + S::ring_off + warp * S::ring_warp;
    float* qs = reinterpret_cast<float*>(smem + S::q_off);
    float* wpart = reinterpret_cast<float*>(smem + S::wpart_off);
    float* cpart = reinterpret_cast<float*>(smem + S::cpart_off);
    KVT* knew = reinterpret_cast<KVT*>(smem + S::new_off);  // [NTK][HD]
    KVT* vnew = knew + NTK * HD;                              // [NTK][HD]

    // The cache position (and the pass's token count) was written by a kernel at least two launches
    // earlier (the commit or the prompt cursor advance of the previous step), so it can be read
    // before the wait.
    const int pos = *(volatile int*)&st->pos;
    const int ntok = DUAL ? *(volatile int*)&st->n_tok : 1;
    const bool two = DUAL && ntok == 2;
    const long long Ls = pos;
    const int p0 = (int)(Ls * j / NSP), p1 = (int)(Ls * (j + 1) / NSP);
    const int a = p0 + (int)((long long)(p1 - p0) * warp / 8), b = p0 + (int)((long long)(p1 - p0) * (warp + 1) / 8);
    const int n_chunks = (b - a + ATT_SLOT - 1) / ATT_SLOT;
    const KVT* kbase = kc + (long long)h * p.max_ctx * HD;
    const KVT* vbase = vc + (long long)h * p.max_ctx * HD;

    auto issue = [&](int c) {
        const int r0 = a + c * ATT_SLOT;
        const int n = min(ATT_SLOT, b - r0);
        const uint32_t bytes = (uint32_t)(n * HD * sizeof(KVT));
        uint8_t* dst = ring + (c % ATT_NS) * S::slot_bytes;
        uint64_t* bar = &bars[c % ATT_NS];
        mbar_expect_tx(bar, 2 * bytes);
        bulk_g2s(dst, kbase + (long long)r0 * HD, bytes, bar);
        bulk_g2s(dst + ATT_SLOT * S::row_bytes, vbase + (long long)r0 * HD, bytes, bar);
    };
    uint64_t* wbar = reinterpret_cast<uint64_t*>(smem + S::bars_off) + 8 * ATT_NS;  // o-proj tiles (FO)
    if (lane == 0) {
        for (int s = 0; s < ATT_NS; ++s) mbar_init(&bars[s], 1);
        if (FO && warp == 0) mbar_init(wbar, 1);
        fence_mbar_init();
        for (int c = 0; c < min(ATT_NS, n_chunks); ++c) issue(c);
    }
    if (tid == 32) l2_prefetch_plan(p.l2, pos);
    // norm weights and this position's rotation are inputs that do not depend on the producer
    // warps 0..3 prepare token 0 (q heads 2h, 2h+1, k, v), warps 4..7 token 1 of a 2-token pass
    const int role = warp & 3, tk = warp >> 2;
    const bool prep = warp < 4 || two;
    float nw[4] = {1.f, 1.f, 1.f, 1.f};
    float2 cs4[4];
    if (prep && role < 3) {
        const float4 w4 = *reinterpret_cast<const float4*>((role < 2 ? p.q_norm : p.k_norm) + 4 * lane);
        nw[0] = w4.x; nw[1] = w4.y; nw[2] = w4.z; nw[3] = w4.w;
#pragma unroll
        for (int e = 0; e < 4; ++e) cs4[e] = rope[(long long)(pos + tk) * 64 + 4 * (lane & 15) + e];
    }
    __syncwarp();

    pdl_wait();
    // the projection values are loaded before the stop-flag read so neither waits on the other
    float4 x4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (prep) {
        const int base = role < 2 ? (2 * h + role) * HD : (role == 2 ? 2048 + h * HD : 3072 + h * HD);
        const float* src = qkv + tk * QKV_ROWS + base + 4 * lane;
        x4 = *reinterpret_cast<const float4*>(src);
        if (p.qkv_parts > 1) {  // the slices' loads first, then the sums in slice order
            float4 y[ATT_QKV_PARTS_MAX - 1];
#pragma unroll
            for (int z = 1; z < ATT_QKV_PARTS_MAX; ++z)
                if (z < p.qkv_parts) y[z - 1] = *reinterpret_cast<const float4*>(src + z * p.qkv_part_stride);
#pragma unroll
            for (int z = 1; z < ATT_QKV_PARTS_MAX; ++z) {
                if (z < p.qkv_parts) {
                    x4.x += y[z - 1].x;
                    x4.y += y[z - 1].y;
                    x4.z += y[z - 1].z;
                    x4.w += y[z - 1].w;
                }
            }
        }
    }

    if (*(volatile int*)&st->done) {  // uniform over the grid: no CTA reaches the cluster barriers
        pdl_launch_dependents();
        if (lane == 0)
            for (int c = 0; c < min(ATT_NS, n_chunks); ++c) mbar_wait_bounded(&bars[c], 0);
        return;
    }

    cluster_arrive_relaxed();  // every CTA of the cluster has started (waited on before the push)

    // ---- q/k norm + RoPE for the new position: warp 0/1 -> q heads 2h, 2h+1, warp 2 -> k, 3 -> v ----
    if (prep) {
        const int tpos = pos + tk;
        float x[4] = {x4.x, x4.y, x4.z, x4.w};
        if (role < 3) {
            const float ss = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
            const float r = 1.0f / sqrtf(ss / (float)HD + EPS);
            float y[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) x[e] = x[e] * r * nw[e];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
                const float2 cs = cs4[e];
                y[e] = lane < 16 ? x[e] * cs.x - partner * cs.y : x[e] * cs.x + partner * cs.y;
            }
            if (role < 2) {
                const float sc = 0.08838834764831845f;  // 1 / sqrt(128)
#pragma unroll
                for (int e = 0; e < 4; ++e) qs[(tk * 2 + role) * HD + 4 * lane + e] = y[e] * sc;
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) knew[tk * HD + kv_swz(4 * lane + e, tpos)] = float_to_kv<KVT>(y[e]);
            }
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) vnew[tk * HD + kv_swz(4 * lane + e, tpos)] = float_to_kv<KVT>(x[e]);
        }
    }
    __syncthreads();
    pdl_launch_dependents();  // after the latency-bound q/k/v loads
    if (j == 0 && tid < ntok * HD) {  // append the new row(s) (already in the swizzled order)
        const int r = tid >> 7, d = tid & 127;
        kc[((long long)h * p.max_ctx + pos + r) * HD + d] = knew[r * HD + d];
        vc[((long long)h * p.max_ctx + pos + r) * HD + d] = vnew[r * HD + d];
    }

    // ---- per-warp flash-decode over rows [a, b) ------------------------------------------------
    // B operand of QK^T: columns (h0 hi, h0 lo, h1 hi, h1 lo) repeated; lane (g, t) holds rows
    // (dims) 2t, 2t+1, 2t+8, 2t+9 of column g for each 16-dim step.
    uint32_t qb[8][2];
    {
        const int g = lane >> 2, t = lane & 3;
        const int hh = two ? g >> 1 : (g >> 1) & 1, part = g & 1;  // two tokens: (token, head) = (hh >> 1, hh & 1)
        const float* q = qs + hh * HD;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const int d0 = 16 * kk + 2 * t;
            qb[kk][0] = pack2<KVT>(split_part<KVT>(q[d0], part), split_part<KVT>(q[d0 + 1], part));
            qb[kk][1] = pack2<KVT>(split_part<KVT>(q[d0 + 8], part), split_part<KVT>(q[d0 + 9], part));
        }
    }
    AttnAcc acc;
    acc.m = -INFINITY;
    acc.l = 0.f;
#pragma unroll
    for (int db = 0; db < 8; ++db)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc.o[db][i] = 0.f;
    for (int c = 0; c < n_chunks; ++c) {
        const int slot = c % ATT_NS;
        if (!mbar_wait_bounded(&bars[slot], (uint32_t)((c / ATT_NS) & 1))) {
            if (lane == 0) atomicOr(&st->error, ERR_WAIT_ATTN);
            break;  // keep going to the cluster barriers with what we have
        }
        const uint32_t kslot = smem_u32(ring + slot * S::slot_bytes);
        const int r0 = a + c * ATT_SLOT;
        const int nr = min(ATT_SLOT, b - r0);
        attn_block<KVT>(kslot, kslot + ATT_SLOT * S::row_bytes, r0, nr, qb, acc, lane, two, nr);
        __syncwarp();
        if (lane == 0 && c + ATT_NS < n_chunks) {
            fence_proxy_async_smem();
            issue(c + ATT_NS);
        }
    }
    if (j == NSP - 1 && warp == 7) {  // the new row(s): token 0 sees row pos, token 1 rows pos, pos + 1
        const uint32_t kn = smem_u32(knew);
        attn_block<KVT>(kn, kn + NTK * S::row_bytes, pos, 1, qb, acc, lane, two, ntok);
    }

    // warp result: lanes with t = 0 / 1 own head 0 / 1 of token 0, t = 2 / 3 those of token 1
    {
        const int g = lane >> 2, t = lane & 3;
        float l = acc.l;
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        const int hw = t & 1;
        float* wp = wpart + (warp * NTK + (t >> 1)) * ATT_PART;
        if (t < 2 * ntok) {
#pragma unroll
            for (int db = 0; db < 8; ++db) {
                wp[4 + hw * HD + 16 * db + g] = acc.o[db][0] + acc.o[db][1];
                wp[4 + hw * HD + 16 * db + g + 8] = acc.o[db][2] + acc.o[db][3];
            }
            if (g == 0) {
                wp[hw] = acc.m;
                wp[2 + hw] = l;
            }
        }
    }
    __syncthreads();
    const int o_rows = H / NSP;                  // FO: o-proj rows of this CTA (128 or 256)
    const int o_run = att_o_run_bytes(o_rows);   // FO: bytes of one slice's run of them
    if (FO && tid == 0) {
        // every warp is done with its ring (all chunk copies waited for): the CTA's o-proj tiles go
        // to the start of the ring while the splits are combined
        fence_proxy_async_smem();
        mbar_expect_tx(wbar, 2 * o_run);
        const long long run0 = ((long long)(2 * h) * (H / 16) + (o_rows / 16) * j) * 2 * icua_layout::Q4_UNIT_BYTES;
        const long long run1 = ((long long)(2 * h + 1) * (H / 16) + (o_rows / 16) * j) * 2 * icua_layout::Q4_UNIT_BYTES;
        bulk_g2s(smem + S::ring_off, p.wo + run0, o_run, wbar);
        bulk_g2s(smem + S::ring_off + o_run, p.wo + run1, o_run, wbar);
    }
    // CTA combine of the 8 warps: thread (hh, d), per token
    const int hh = tid >> 7, d = tid & 127;
    float Mt[NTK], Lt[NTK], Ot[NTK];
#pragma unroll
    for (int q = 0; q < NTK; ++q) {
        Mt[q] = -INFINITY;
        Lt[q] = Ot[q] = 0.f;
        if (q >= ntok) continue;
#pragma unroll
        for (int w2 = 0; w2 < 8; ++w2) Mt[q] = fmaxf(Mt[q], wpart[(w2 * NTK + q) * ATT_PART + hh]);
#pragma unroll
        for (int w2 = 0; w2 < 8; ++w2) {
            const float* wq = wpart + (w2 * NTK + q) * ATT_PART;
            const float mw = wq[hh];
            const float f = (mw == -INFINITY) ? 0.f : expf(mw - Mt[q]);
            Lt[q] = fmaf(wq[2 + hh], f, Lt[q]);
            Ot[q] = fmaf(wq[4 + hh * HD + d], f, Ot[q]);
        }
    }
    // push this CTA's part(s) into slot `rank` of the cluster leader's (rank 0) shared memory
    cluster_wait();
    {
        const uint32_t rank = cluster_ctarank();
#pragma unroll
        for (int q = 0; q < NTK; ++q) {
            if (q >= ntok) continue;
            float* slot = cpart + (rank * NTK + q) * ATT_PART;
            st_dsmem(&slot[4 + hh * HD + d], 0, Ot[q]);
            if (d == 0) {
                st_dsmem(&slot[hh], 0, Mt[q]);
                st_dsmem(&slot[2 + hh], 0, Lt[q]);
            }
        }
    }
    // one cluster barrier: the pushes (release) are visible to the leader (acquire); the other
    // CTAs are done, since nobody reads their shared memory
    cluster_sync_all();
    const bool leader = cluster_ctarank() == 0;
    if (!FO && !leader) return;
    const int CL = p.cluster;
#pragma unroll
    for (int tq = 0; tq < NTK; ++tq) {
        if (tq >= ntok || !leader) continue;
        float M = -INFINITY;
#pragma unroll
        for (int q = 0; q < CLM; ++q)
            if (q < CL) M = fmaxf(M, cpart[(q * NTK + tq) * ATT_PART + hh]);
        float Lsum = 0.f, O = 0.f;
#pragma unroll
        for (int q = 0; q < CLM; ++q) {
            if (q < CL) {
                const float* cq = cpart + (q * NTK + tq) * ATT_PART;
                const float mq = cq[hh];
                const float f = (mq == -INFINITY) ? 0.f : expf(mq - M);
                Lsum = fmaf(cq[2 + hh], f, Lsum);
                O = fmaf(cq[4 + hh * HD + d], f, O);
            }
        }
        if (FO) {
            qs[tid] = O / Lsum;  // the head pair's output, element hh * 128 + d (q is in registers now)
        } else if (p.out16 != nullptr) {
            const float y = O / Lsum;
            const size_t col = (size_t)(2 * h + hh) * HD + d;
            if (p.out16_hilo) {  // fp16 hi / lo rows 2 row, 2 row + 1
                const __half hi = __float2half_rn(y);
                p.out16[(size_t)(2 * row) * H + col] = hi;
                p.out16[(size_t)(2 * row + 1) * H + col] = __float2half_rn(y - __half2float(hi));
            } else {
                p.out16[(size_t)row * H + col] = __float2half_rn(y);
            }
        } else {
            // token tq's parts follow token 0's ([NTK][NKV][parts][ATT_PART])
            float* out = p.part + ((long long)(tq * NKV + h) * (NSP / CL) + j / CL) * ATT_PART;
            out[4 + hh * HD + d] = O;
            if (d == 0) {
                out[hh] = M;
                out[2 + hh] = Lsum;
            }
        }
    }
    if constexpr (FO) {
        // every CTA reads the leader's output of the head pair, multiplies it by its 128 o-proj rows
        cluster_sync_all();  // the leader's qs is written (release / acquire)
        const float y = ld_dsmem(&qs[tid], 0);
        float* xv = wpart;  // the warp parts are consumed: [256] inputs, then fragments and group sums
        uint2* xfrag = reinterpret_cast<uint2*>(wpart + 256);
        float* xsum = wpart + 256 + 64 * 4;
        xv[tid] = y;
        cluster_arrive_relaxed();  // the leader may leave once every CTA has read its output
        __syncthreads();
        if (tid < 64) {  // pair q = tid: elements k0, k0 + 1, k0 + 8, k0 + 9 (the GEMV fragment order)
            const int q = tid, k0 = (q >> 2) * 16 + 2 * (q & 3);
            const int kk[4] = {k0, k0 + 1, k0 + 8, k0 + 9};
            __half hi[4], lo[4];
            float gsum = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float x = xv[kk[i]];
                hi[i] = __float2half_rn(x);
                lo[i] = __float2half_rn(x - __half2float(hi[i]));
                gsum += __half2float(hi[i]) + __half2float(lo[i]);
            }
            uint2 h2, l2;
            h2.x = (uint32_t)__half_as_ushort(hi[0]) | ((uint32_t)__half_as_ushort(hi[1]) << 16);
            h2.y = (uint32_t)__half_as_ushort(hi[2]) | ((uint32_t)__half_as_ushort(hi[3]) << 16);
            l2.x = (uint32_t)__half_as_ushort(lo[0]) | ((uint32_t)__half_as_ushort(lo[1]) << 16);
            l2.y = (uint32_t)__half_as_ushort(lo[2]) | ((uint32_t)__half_as_ushort(lo[3]) << 16);
            xfrag[q * 2 + 0] = h2;
            xfrag[q * 2 + 1] = l2;
            gsum += __shfl_xor_sync(0xffffffffu, gsum, 1);
            gsum += __shfl_xor_sync(0xffffffffu, gsum, 2);
            gsum += __shfl_xor_sync(0xffffffffu, gsum, 4);
            if ((q & 7) == 0) xsum[q >> 3] = gsum;
        }
        __syncthreads();
        if (!mbar_wait_bounded(wbar, 0)) {
            if (lane == 0) atomicOr(&st->error, ERR_WAIT_ATTN);
            mbar_wait_bounded(wbar, 0);  // the copy lands before this CTA reads or leaves
        }
        // warp w: tiles w, w + 8 of the CTA's o_rows / 16 (rows o_rows j + 16 tile ..), the 4 units
        // of the head pair
        UnitConst<FMT_Q4S> uc[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) load_unit_const<FMT_Q4S>(uc[u], u, xfrag, xsum, lane);
        for (int tile = warp; tile < o_rows / 16; tile += 8) {
            float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint8_t* ub = smem + S::ring_off + (u >> 1) * o_run + (tile * 2 + (u & 1)) * icua_layout::Q4_UNIT_BYTES;
                gemv_unit<FMT_Q4S>(ub, uc[u], lane, acc0, acc1);
            }
            if ((lane & 3) == 0) {
                const int g = lane >> 2, r = o_rows * j + 16 * tile + g;
                p.o_part[h * H + r] = acc0 * 16777216.0f;  // rows g in units of 2^-24, rows g + 8 of 2^-20
                p.o_part[h * H + r + 8] = acc1 * 1048576.0f;
            }
        }
        cluster_wait();
    }
}

}  // namespace icua
