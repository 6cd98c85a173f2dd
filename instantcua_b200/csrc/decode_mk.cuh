// Persistent decode step: every decoder layer of one token in one cooperative launch.
//
// Replaces, for q4s engines, the per-layer launch chain of the decode step (QKV GEMV -> attention ->
// o-proj -> gate/up -> down, 5 x 28 launches): the reference's k_attn_in, k_attention, k_o_proj,
// k_mlp_in and k_mlp_out (Shaders.swift:714-834, 1219-1448) for the whole stack.
//
// Design (B200):
// * One CTA per SM (cooperative launch: all CTAs resident), 16 compute warps + 1 producer warp.
// * Weights: each CTA owns fixed row tiles of every matrix (QKV, o, gate/up, down) and its tiles of
//   all layers are stored back to back ("CTA stream", 18 KB items = 16 rows x 2048 columns of q4s).
//   The producer warp streams the CTA's items -- and, for attention, its range of cache rows --
//   into a ring of shared-memory slots with 1-D bulk copies, as far ahead as the ring allows.  None
//   of these bytes depends on the token, so the HBM stream runs ahead of the dependency chain.
// * Activations cross CTAs through L2 as tagged 64-bit words (value | tag << 32, one atomic store
//   each): a consumer polls the words it needs until they carry this launch's tag for the layer.
//   No counters or fences on the GEMV path.  Each warp needs only its own K slice of the input
//   vector, so it stages its fragments itself; the RMSNorm scale comes from sums of squares that
//   the producers of the vector publish per 16-row tile.
// * The residual rows of o-proj / down tile j stay in CTA j's shared memory for the whole step.
// * Attention: 8 kv heads x S context splits; each split CTA writes its (max, sum, output) part and
//   the last CTA of the head (atomic counter) folds the S parts into the head's output.
// * Every wait is bounded.  A CTA that gives up sets the session's error flag and a global abort
//   flag; the others see it within a few polls, stop waiting and run the rest of the step without
//   waiting (so every named barrier is still reached by every warp), the producer stops issuing,
//   and copies already in flight are waited for before the CTA exits.
#pragma once
#include "attn_decode.cuh"
#include "common.cuh"
#include "gemm_tc.cuh"
#include "gemv.cuh"

namespace icua {


constexpr int MK_WARPS = 16;                        // compute warps
constexpr int MK_CTHREADS = MK_WARPS * 32;          // named barrier 1
constexpr int MK_THREADS = MK_CTHREADS + 32;        // + the producer warp
constexpr int MK_ITEM = 32 * Q4_UNIT_BYTES;         // ring slot: 16 rows x 2048 columns of q4s (18432 B)
constexpr int MK_NS = 10;                           // ring slots
constexpr int MK_KV_ROWS = 32;                      // cache positions per attention item (K then V rows)
constexpr int MK_MAX_LAYERS = 32;                   // tags: epoch * 32 + layer
constexpr int MK_MAX_S = 20;                        // attention splits per kv head (G <= 167)
constexpr uint32_t MK_POLL_LIMIT = 1u << 21;        // polls of one exchange word before giving up
constexpr int MK_QKV_TILES = QKV_ROWS / 16, MK_O_TILES = H / 16, MK_GU_TILES = GU_ROWS / 16;
constexpr int ERR_WAIT_MK = 16;

struct MkLayer {
    const float *attn_norm, *q_norm, *k_norm, *mlp_norm;
};

template <typename KVT>
struct MkParams {
    const uint8_t* stream;                 // CTA streams (mk_pack_kernel)
    const unsigned long long* cta_base;    // [G] byte offset of CTA c's stream
    const MkLayer* layers;                 // [n_layers]
    int n_layers;
    int S;                                 // attention CTAs per kv head (8 * S <= G)
    // session
    DevState* st;
    const int* prompt;
    const float* pooler;
    const float* deepstack[3];
    const float2* rope;                    // [max_ctx][64]
    KVT* kc;                               // [n_layers][NKV][max_ctx][HD] (swizzled rows)
    KVT* vc;
    int max_ctx;
    // embedding
    const uint8_t* embed;
    int embed_tiles, embed_fmt;
    // exchange words (value bits | tag << 32)
    unsigned long long* qkv;               // [4096]
    unsigned long long* att;               // [2048] head outputs, column order
    unsigned long long* xmid;              // [2048] residual after o-proj
    unsigned long long* xout;              // [2048] residual after down
    unsigned long long* hbuf;              // [6144] SwiGLU output
    unsigned long long* parts;             // [NKV][S][ATT_PART] attention split parts (exchange words)
    unsigned* fin;                         // CTAs done with this launch
    unsigned* epoch;                       // launch counter (tags)
    int* abort;                            // a CTA gave up a wait
    float* x_final;                        // [2048] residual after the last layer (the lm_head's input)
};

// Tiles [t0, t1) of a T-tile phase owned by CTA c of G.
__host__ __device__ inline void mk_range(int T, int c, int G, int& t0, int& t1) {
    t0 = (int)((long long)c * T / G);
    t1 = (int)((long long)(c + 1) * T / G);
}

// Ring items of CTA c per layer (bytes of its stream per layer / MK_ITEM).
__host__ __device__ inline int mk_items_per_layer(int c, int G) {
    int a, b, n = 0;
    mk_range(MK_QKV_TILES, c, G, a, b);
    n += b - a;
    mk_range(MK_O_TILES, c, G, a, b);
    n += 4 * (b - a);  // o tile + the 3 K-thirds of the down tile of the same rows
    mk_range(MK_GU_TILES, c, G, a, b);
    n += b - a;
    return n;
}

struct MkSmem {
    static constexpr int ring = 0;
    static constexpr int frag = MK_NS * MK_ITEM;                    // [16 warps][2 units][16 pairs][2] uint2
    static constexpr int frag_warp = 2 * 16 * 2 * 8;                // 512 B
    static constexpr int xsum = frag + MK_WARPS * frag_warp;        // [16][4] float
    // union: embedding row / attention warp parts / the split parts the combiner folds
    static constexpr int big = xsum + MK_WARPS * 4 * 4;
    static constexpr int big_bytes = (MK_MAX_S > MK_WARPS ? MK_MAX_S : MK_WARPS) * ATT_PART * 4;
    // GEMV parts [tile][16 warps][16 rows]: QKV / gate-up use tiles 0..5, o / down tile 6, so a
    // phase's partial sums never overwrite those the previous phase is still reducing
    static constexpr int part = big + big_bytes;
    static constexpr int qs = part + 7 * MK_WARPS * 16 * 4;         // float [2][128]
    static constexpr int knew = qs + 2 * HD * 4;                    // KVT [128] (swizzled), then vnew [128]
    static constexpr int resid = knew + 2 * HD * 4;                 // float [16]
    static constexpr int misc = resid + 16 * 4;                     // int [8]: abort, bcast, ...
    static constexpr int ssp = misc + 8 * 4;                        // float [2][16]: per-warp sums of squares
    static constexpr int bars = (ssp + 2 * MK_WARPS * 4 + 7) & ~7;  // full[NS], empty[NS], ssbar
    static constexpr int total = bars + (2 * MK_NS + 1) * 8;
};

// Exchange words are read and written with plain (weak) 64-bit accesses cached only in L2, the
// point where all SMs meet: an aligned 8-byte access moves value and tag together, so a word is
// either the old one or the new one, and the tag says which; no ordering between words is needed.
// Strong (.relaxed.gpu / .volatile) loads complete one at a time (about one L2 round trip each),
// which made a poll of N words cost N round trips; weak loads of one poll are in flight together.
// `volatile` keeps every poll iteration's load, and no memory clobber lets the loads of a poll
// issue back to back.
__device__ __forceinline__ unsigned long long ll_ld(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.global.cg.u64 %0, [%1];" : "=l"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ void ll_st(unsigned long long* p, float v, uint32_t tag) {
    const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
    asm volatile("st.global.cg.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ int ld_relaxed_int(const int* p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void named_sync() { asm volatile("bar.sync 1, %0;" ::"n"(MK_CTHREADS) : "memory"); }

// Bounded mbarrier wait that sleeps between polls, for waits that can last microseconds (the
// producer waiting for a free ring slot, warps waiting for the others of their CTA): a warp that
// spins on try_wait keeps taking issue slots from the warps of its scheduler that have work.
__device__ __forceinline__ bool mbar_wait_sleepy(uint64_t* bar, uint32_t parity, uint32_t limit = (1u << 22)) {
    for (uint32_t i = 0; i < limit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        __nanosleep(40);
    }
    return false;
}

// Control state of a CTA: the shared abort flag and what a give-up records.
struct MkCtl {
    volatile int* s_abort;
    int* g_abort;
    DevState* st;
    // Records a wait that gave up (once per CTA is enough; repeats are harmless).
    __device__ void give_up() const {
        *s_abort = 1;
        asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(g_abort), "r"(1) : "memory");
        atomicOr(&st->error, ERR_WAIT_MK);
    }
    __device__ bool aborted() const { return *s_abort != 0; }
};

// Polls N exchange words per lane until all lanes' words carry `tag` (warp-wide).  Returns false
// (values undefined) when the CTA is in abort mode or the wait gave up.  Thousands of warps wait
// on the same few hundred words, so a warp first polls one word with one lane (one L2 sector per
// round) and loads its whole slice only once that word is current: polling every word from every
// warp saturated the L2 slices that hold those lines, which slowed every access routed to them.
template <int N>
__device__ __forceinline__ bool ll_poll(const unsigned long long* const (&addr)[N], float (&v)[N], uint32_t tag,
                                        const MkCtl& ctl) {
    uint32_t polls = 0;
    const int lane = threadIdx.x & 31;
    auto check_abort = [&]() -> bool {  // true: stop waiting
        if (ctl.aborted()) return true;
        if ((++polls & 31) == 0) {
            const bool g = ld_relaxed_int(ctl.g_abort) != 0;
            if (g || polls >= MK_POLL_LIMIT) {
                if (lane == 0) {
                    if (g)
                        *ctl.s_abort = 1;
                    else
                        ctl.give_up();
                }
                __syncwarp();
                return true;
            }
        }
        return false;
    };
    while (true) {
        bool ok = true;
        if (lane == 0) ok = (uint32_t)(ll_ld(addr[N - 1]) >> 32) == tag;
        if (__shfl_sync(0xffffffffu, ok, 0)) break;
        if (check_abort()) return false;
        __nanosleep(64);
    }
    while (true) {
        bool ok = true;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const unsigned long long w = ll_ld(addr[i]);
            v[i] = __uint_as_float((uint32_t)w);
            ok &= (uint32_t)(w >> 32) == tag;
        }
        if (__all_sync(0xffffffffu, ok)) return true;
        if (check_abort()) return false;
        __nanosleep(64);
    }
}

// Consumer side of the ring.
struct MkRing {
    uint8_t* base;
    uint64_t* full;
    uint64_t* empty;
    uint32_t it;  // next item
    __device__ const uint8_t* wait(const MkCtl& ctl) {
        const int s = it % MK_NS;
        if (!ctl.aborted() && !mbar_wait_sleepy(&full[s], (it / MK_NS) & 1)) {
            if ((threadIdx.x & 31) == 0) ctl.give_up();
        }
        return base + s * MK_ITEM;
    }
    __device__ void release() {
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&empty[it % MK_NS]);
        ++it;
    }
};

// Sum of squares of a vector whose 16 warp slices are held by the 16 compute warps: each warp
// publishes its slice's sum in shared memory and arrives on `bar`; after the phase completes every
// warp adds the 16 sums in the same order.  `uses` counts the calls (phase parity, buffer).
__device__ __forceinline__ float mk_cta_sumsq(float ss_warp, float* ssp, uint64_t* bar, uint32_t& uses, int warp,
                                              const MkCtl& ctl) {
    float* buf = ssp + (uses & 1) * MK_WARPS;
    if ((threadIdx.x & 31) == 0) {
        buf[warp] = ss_warp;
        mbar_arrive(bar);
    }
    if (!ctl.aborted() && !mbar_wait_sleepy(bar, uses & 1) && (threadIdx.x & 31) == 0) ctl.give_up();
    ++uses;
    float tot = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < MK_WARPS; ++w2) tot += buf[w2];
    return tot;
}

// Writes a warp's input fragments for one pair of units from 4 values per lane (lane = unit-half u
// (lane >> 4), pair q = lane & 15: columns 16 (q >> 2) + 2 (q & 3) + {0, 1, 8, 9} of the unit), in
// the layout load_unit_const reads: fp16 hi / lo of each value and per-32-column sums.
__device__ __forceinline__ void mk_store_frag(const float (&x)[4], int unit_pair, uint2* xfrag, float* xsum, int lane) {
    const int u = unit_pair * 2 + (lane >> 4), q = lane & 15;
    __half hi[4], lo[4];
    float gsum = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        hi[i] = __float2half_rn(x[i]);
        lo[i] = __float2half_rn(x[i] - __half2float(hi[i]));
        gsum += __half2float(hi[i]) + __half2float(lo[i]);
    }
    uint2 h2, l2;
    h2.x = (uint32_t)__half_as_ushort(hi[0]) | ((uint32_t)__half_as_ushort(hi[1]) << 16);
    h2.y = (uint32_t)__half_as_ushort(hi[2]) | ((uint32_t)__half_as_ushort(hi[3]) << 16);
    l2.x = (uint32_t)__half_as_ushort(lo[0]) | ((uint32_t)__half_as_ushort(lo[1]) << 16);
    l2.y = (uint32_t)__half_as_ushort(lo[2]) | ((uint32_t)__half_as_ushort(lo[3]) << 16);
    xfrag[(u * 16 + q) * 2 + 0] = h2;
    xfrag[(u * 16 + q) * 2 + 1] = l2;
    gsum += __shfl_xor_sync(0xffffffffu, gsum, 1);
    gsum += __shfl_xor_sync(0xffffffffu, gsum, 2);
    gsum += __shfl_xor_sync(0xffffffffu, gsum, 4);
    if ((q & 7) == 0) xsum[u * 2 + (q >> 3)] = gsum;
}

// Global column of value i (0..3) of this lane for unit-pair `pair` whose first unit starts at
// column `col0` (the pair covers 128 columns).
__device__ __forceinline__ int mk_col(int col0, int lane, int i) {
    const int q = lane & 15;
    return col0 + (lane >> 4) * 64 + 16 * (q >> 2) + 2 * (q & 3) + (i & 1) + (i >> 1) * 8;
}

// One GEMV tile slice of this warp: units u0, u0+1 of the tile at `tile` (an 18 KB item whose
// units are in K order) with the constants `uc` of the same units.  Returns the row sums scaled
// to fp32 units in acc0 (rows g) and acc1 (rows g + 8).
__device__ __forceinline__ void mk_tile2(const uint8_t* item, int u0, const UnitConst<FMT_Q4S> (&uc)[2], int lane,
                                         float& acc0, float& acc1) {
    gemv_unit<FMT_Q4S>(item + (u0 + 0) * Q4_UNIT_BYTES, uc[0], lane, acc0, acc1);
    gemv_unit<FMT_Q4S>(item + (u0 + 1) * Q4_UNIT_BYTES, uc[1], lane, acc0, acc1);
}

__device__ __forceinline__ void mk_put_part(float* part, int tile, int warp, int lane, float acc0, float acc1) {
    const int g = lane >> 2, t = lane & 3;
    if (t == 0) {
        float* p = part + (tile * MK_WARPS + warp) * 16;
        p[g] = acc0 * 16777216.0f;
        p[g + 8] = acc1 * 1048576.0f;
    }
}

template <typename KVT>
__global__ void __launch_bounds__(MK_THREADS, 1) decode_mk_kernel(const MkParams<KVT> p) {
    extern __shared__ __align__(128) uint8_t smem[];
    using S = MkSmem;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    DevState* const st = p.st;
    if (*(volatile int*)&st->done) return;  // uniform: every CTA reads the same flag

    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::bars);
    uint64_t* empty = full + MK_NS;
    int* misc = reinterpret_cast<int*>(smem + S::misc);
    float* big = reinterpret_cast<float*>(smem + S::big);
    float* part = reinterpret_cast<float*>(smem + S::part);
    float* qs = reinterpret_cast<float*>(smem + S::qs);
    KVT* knew = reinterpret_cast<KVT*>(smem + S::knew);
    KVT* vnew = knew + HD;
    float* resid = reinterpret_cast<float*>(smem + S::resid);
    MkCtl ctl{reinterpret_cast<volatile int*>(misc), p.abort, st};

    const int pos = *(volatile int*)&st->pos;
    const int L = p.n_layers, NSPLIT = p.S;
    int q0, q1, o0, o1, g0, g1;
    mk_range(MK_QKV_TILES, c, G, q0, q1);
    mk_range(MK_O_TILES, c, G, o0, o1);
    mk_range(MK_GU_TILES, c, G, g0, g1);
    const int nq = q1 - q0, no = o1 - o0, ngu = g1 - g0;
    const bool att_cta = c < NKV * NSPLIT;
    const int ah = att_cta ? c / NSPLIT : 0, aj = att_cta ? c % NSPLIT : 0;
    const int ap0 = att_cta ? (int)((long long)pos * aj / NSPLIT) : 0;
    const int ap1 = att_cta ? (int)((long long)pos * (aj + 1) / NSPLIT) : 0;
    const int n_kv = (ap1 - ap0 + MK_KV_ROWS - 1) / MK_KV_ROWS;
    const bool att_last = att_cta && aj == NSPLIT - 1;  // this split also holds the new position
    const int per_layer = nq + 4 * no + ngu;
    const uint8_t* my_stream = p.stream + p.cta_base[c];
    constexpr int RB = HD * (int)sizeof(KVT);  // bytes per cache row

    if (tid == 0) {
        misc[0] = 0;  // abort
        misc[2] = (int)*(volatile unsigned*)p.epoch;
        for (int s = 0; s < MK_NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], MK_WARPS);
        }
        mbar_init(full + 2 * MK_NS, MK_WARPS);
        fence_mbar_init();
    }
    __syncthreads();
    const uint32_t ep = (uint32_t)misc[2];

    // ================================ producer warp ================================
    if (warp == MK_WARPS) {
        if (lane == 0) {
            uint32_t it = 0;
            bool stop = false;
            auto issue = [&](const void* src0, uint32_t b0, const void* src1, uint32_t b1) {
                const int s = it % MK_NS;
                if (it >= MK_NS && !mbar_wait_sleepy(&empty[s], ((it / MK_NS) - 1) & 1)) {
                    ctl.give_up();
                    stop = true;
                    return;
                }
                if (ctl.aborted()) {
                    stop = true;
                    return;
                }
                fence_proxy_async_smem();
                uint8_t* dst = smem + S::ring + s * MK_ITEM;
                mbar_expect_tx(&full[s], b0 + b1);
                bulk_g2s(dst, src0, b0, &full[s]);
                if (b1) bulk_g2s(dst + MK_KV_ROWS * RB, src1, b1, &full[s]);
                ++it;
            };
            // L2 prefetch one layer ahead of the ring: the ring holds about half a layer of this
            // CTA's bytes, so HBM would idle whenever the CTA waits on a dependency; the prefetched
            // layer (45 MB over all CTAs at 4K context) keeps the stream going and the ring refills
            // from L2.
            auto prefetch_layer = [&](int l) {
                if (l >= L) return;
                l2_prefetch_range(my_stream + (size_t)l * per_layer * MK_ITEM, 0, (uint64_t)per_layer * MK_ITEM);
                if (att_cta && ap1 > ap0) {
                    const size_t off = (((size_t)l * NKV + ah) * p.max_ctx + ap0) * HD;
                    l2_prefetch_range(reinterpret_cast<const uint8_t*>(p.kc + off), 0, (uint64_t)(ap1 - ap0) * RB);
                    l2_prefetch_range(reinterpret_cast<const uint8_t*>(p.vc + off), 0, (uint64_t)(ap1 - ap0) * RB);
                }
            };
            prefetch_layer(0);
            for (int l = 0; l < L && !stop; ++l) {
                prefetch_layer(l + 1);
                const uint8_t* ls = my_stream + (size_t)l * per_layer * MK_ITEM;
                int k = 0;
                for (int i = 0; i < nq && !stop; ++i) issue(ls + (size_t)(k++) * MK_ITEM, MK_ITEM, nullptr, 0);
                if (att_cta) {
                    const KVT* kb = p.kc + ((size_t)l * NKV + ah) * p.max_ctx * HD;
                    const KVT* vb = p.vc + ((size_t)l * NKV + ah) * p.max_ctx * HD;
                    for (int i = 0; i < n_kv && !stop; ++i) {
                        const int r0 = ap0 + i * MK_KV_ROWS, nr = min(MK_KV_ROWS, ap1 - r0);
                        issue(kb + (size_t)r0 * HD, (uint32_t)(nr * RB), vb + (size_t)r0 * HD, (uint32_t)(nr * RB));
                    }
                }
                for (int i = 0; i < no && !stop; ++i) issue(ls + (size_t)(k++) * MK_ITEM, MK_ITEM, nullptr, 0);
                for (int i = 0; i < ngu && !stop; ++i) issue(ls + (size_t)(k++) * MK_ITEM, MK_ITEM, nullptr, 0);
                for (int i = 0; i < 3 * no && !stop; ++i) issue(ls + (size_t)(k++) * MK_ITEM, MK_ITEM, nullptr, 0);
            }
            // drain: the copies still in flight land before the CTA exits
            const uint32_t first = it > MK_NS ? it - MK_NS : 0;
            for (uint32_t i = first; i < it; ++i) mbar_wait_bounded(&full[i % MK_NS], (i / MK_NS) & 1);
        }
        __syncwarp();
    } else {
        // ================================ compute warps ================================
        MkRing ring{smem + S::ring, full, empty, 0};
        uint2* xfrag = reinterpret_cast<uint2*>(smem + S::frag + warp * S::frag_warp);
        float* xsum = reinterpret_cast<float*>(smem + S::xsum) + warp * 4;
        float* ssp = reinterpret_cast<float*>(smem + S::ssp);
        uint64_t* ssbar = full + 2 * MK_NS;
        uint32_t ss_uses = 0;
        UnitConst<FMT_Q4S> uc[2];
        auto consts2 = [&](int pair) {  // constants of this warp's unit pair `pair` of the staged slice
            load_unit_const<FMT_Q4S>(uc[0], pair * 2 + 0, xfrag, xsum, lane);
            load_unit_const<FMT_Q4S>(uc[1], pair * 2 + 1, xfrag, xsum, lane);
        };

        // ---- the step's input row: prompt token, visual row or the last generated token --------
        int ds_vi = -1;
        {
            const int idx = st->prompt_idx;
            const float* vis_row = nullptr;
            int tok;
            if (idx < st->prompt_len) {
                tok = p.prompt[idx];
                const int v = idx - st->vis_offset;
                if (st->vis_offset >= 0 && v >= 0 && v < st->n_vis) {
                    ds_vi = v;
                    if (tok == IMAGE_PAD_ID && p.pooler != nullptr) vis_row = p.pooler + (long long)v * H;
                }
            } else {
                tok = st->cur_token;
            }
            float ss = 0.f;
            for (int k = tid; k < H; k += MK_CTHREADS) {
                const float v = vis_row ? vis_row[k] : embed_value(p.embed_fmt, p.embed, p.embed_tiles, tok, k);
                big[k] = v;
                ss = fmaf(v, v, ss);
            }
            ss = warp_sum(ss);
            if (lane == 0) part[warp] = ss;
            named_sync();
            if (tid < 16 && no > 0) resid[tid] = big[o0 * 16 + tid];
            float tot = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < MK_WARPS; ++w2) tot += part[w2];
            named_sync();
            if (tid == 0) misc[4] = __float_as_int(tot);  // sum of squares of the embedded row
        }
        named_sync();

        for (int l = 0; l < L; ++l) {
            const MkLayer ly = p.layers[l];
            const uint32_t tag = ep * MK_MAX_LAYERS + l;
            const uint32_t tag_prev = ep * MK_MAX_LAYERS + l - 1;

            // ======== QKV: RMSNorm(x) -> q | k | v rows of this CTA's tiles ========
            {
                float x[4];
                float scale;
                const int col0 = warp * 128;
                float nwq[4];  // norm weights first: they do not depend on the step
#pragma unroll
                for (int i = 0; i < 4; ++i) nwq[i] = __ldg(ly.attn_norm + mk_col(col0, lane, i));
                if (l == 0) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) x[i] = big[mk_col(col0, lane, i)];
                    scale = 1.0f / sqrtf(__int_as_float(misc[4]) / (float)H + EPS);
                } else {
                    const unsigned long long* a[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) a[i] = p.xout + mk_col(col0, lane, i);
                    ll_poll<4>(a, x, tag_prev, ctl);
                    const float ssw = warp_sum((x[0] * x[0] + x[1] * x[1]) + (x[2] * x[2] + x[3] * x[3]));
                    const float ss = mk_cta_sumsq(ssw, ssp, ssbar, ss_uses, warp, ctl);
                    scale = 1.0f / sqrtf(ss / (float)H + EPS);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) x[i] = x[i] * scale * nwq[i];
                mk_store_frag(x, 0, xfrag, xsum, lane);
                __syncwarp();
                consts2(0);
                for (int i = 0; i < nq; ++i) {
                    const uint8_t* item = ring.wait(ctl);
                    float a0 = 0.f, a1 = 0.f;
                    mk_tile2(item, 2 * warp, uc, lane, a0, a1);
                    ring.release();
                    mk_put_part(part, i, warp, lane, a0, a1);
                }
                named_sync();
                if (tid < nq * 16) {
                    const int i = tid >> 4, r = tid & 15;
                    float v = 0.f;
#pragma unroll
                    for (int w2 = 0; w2 < MK_WARPS; ++w2) v += part[(i * MK_WARPS + w2) * 16 + r];
                    ll_st(p.qkv + (q0 + i) * 16 + r, v, tag);
                }
            }

            // ======== attention of kv head ah over cache rows [ap0, ap1) (+ the new row) ========
            if (att_cta) {
                const int role = warp;  // warps 0, 1: q heads 2h, 2h + 1; 2: k; 3: v (new position)
                if (role < 2 || (att_last && role < 4)) {
                    const int base = role < 2 ? (2 * ah + role) * HD : (role == 2 ? 2048 + ah * HD : 3072 + ah * HD);
                    // the norm weights and this position's rotation do not depend on the step
                    float nw[4] = {1.f, 1.f, 1.f, 1.f};
                    float2 cs4[4];
                    if (role < 3) {
                        const float4 w4 = *reinterpret_cast<const float4*>((role < 2 ? ly.q_norm : ly.k_norm) + 4 * lane);
                        nw[0] = w4.x; nw[1] = w4.y; nw[2] = w4.z; nw[3] = w4.w;
#pragma unroll
                        for (int e = 0; e < 4; ++e) cs4[e] = p.rope[(long long)pos * 64 + 4 * (lane & 15) + e];
                    }
                    const unsigned long long* a[4];
                    float xv[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) a[e] = p.qkv + base + 4 * lane + e;
                    ll_poll<4>(a, xv, tag, ctl);
                    if (role < 3) {
                        const float ss = warp_sum(xv[0] * xv[0] + xv[1] * xv[1] + xv[2] * xv[2] + xv[3] * xv[3]);
                        const float r = 1.0f / sqrtf(ss / (float)HD + EPS);
                        float y[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) xv[e] = xv[e] * r * nw[e];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float partner = __shfl_xor_sync(0xffffffffu, xv[e], 16);
                            const float2 cs = cs4[e];
                            y[e] = lane < 16 ? xv[e] * cs.x - partner * cs.y : xv[e] * cs.x + partner * cs.y;
                        }
                        if (role < 2) {
#pragma unroll
                            for (int e = 0; e < 4; ++e) qs[role * HD + 4 * lane + e] = y[e] * 0.08838834764831845f;
                        } else {
#pragma unroll
                            for (int e = 0; e < 4; ++e) knew[kv_swz(4 * lane + e, pos)] = float_to_kv<KVT>(y[e]);
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e) vnew[kv_swz(4 * lane + e, pos)] = float_to_kv<KVT>(xv[e]);
                    }
                }
                named_sync();
                if (att_last && tid < HD) {  // append the new row (already in the swizzled order)
                    const size_t row = (((size_t)l * NKV + ah) * p.max_ctx + pos) * HD;
                    p.kc[row + tid] = knew[tid];
                    p.vc[row + tid] = vnew[tid];
                }
                uint32_t qb[8][2];
                {
                    const int g = lane >> 2, t = lane & 3;
                    const int hh = (g >> 1) & 1, prt = g & 1;
                    const float* q = qs + hh * HD;
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const int d0 = 16 * kk + 2 * t;
                        qb[kk][0] = pack2<KVT>(split_part<KVT>(q[d0], prt), split_part<KVT>(q[d0 + 1], prt));
                        qb[kk][1] = pack2<KVT>(split_part<KVT>(q[d0 + 8], prt), split_part<KVT>(q[d0 + 9], prt));
                    }
                }
                AttnAcc acc;
                acc.m = -INFINITY;
                acc.l = 0.f;
#pragma unroll
                for (int db = 0; db < 8; ++db)
#pragma unroll
                    for (int i = 0; i < 4; ++i) acc.o[db][i] = 0.f;
                for (int i = 0; i < n_kv; ++i) {
                    const uint8_t* item = ring.wait(ctl);
                    const int r0 = ap0 + i * MK_KV_ROWS, nr = min(MK_KV_ROWS, ap1 - r0);
#pragma unroll
                    for (int b = 0; b < 2; ++b) {
                        if (((2 * i + b) & (MK_WARPS - 1)) == warp && 16 * b < nr) {
                            const uint32_t ks = smem_u32(item) + 16 * b * RB;
                            attn_block<KVT>(ks, ks + MK_KV_ROWS * RB, r0 + 16 * b, min(16, nr - 16 * b), qb, acc, lane);
                        }
                    }
                    ring.release();
                }
                if (att_last && warp == MK_WARPS - 1) {
                    const uint32_t kn = smem_u32(knew);
                    attn_block<KVT>(kn, kn + RB, pos, 1, qb, acc, lane);
                }
                // warp result: lanes with t = 0 / 1 own head 0 / 1
                float* wpart = big;
                {
                    const int g = lane >> 2, t = lane & 3;
                    float lsum = acc.l;
                    lsum += __shfl_xor_sync(0xffffffffu, lsum, 4);
                    lsum += __shfl_xor_sync(0xffffffffu, lsum, 8);
                    lsum += __shfl_xor_sync(0xffffffffu, lsum, 16);
                    if (t < 2) {
                        float* wp = wpart + warp * ATT_PART;
#pragma unroll
                        for (int db = 0; db < 8; ++db) {
                            wp[4 + t * HD + 16 * db + g] = acc.o[db][0] + acc.o[db][1];
                            wp[4 + t * HD + 16 * db + g + 8] = acc.o[db][2] + acc.o[db][3];
                        }
                        if (g == 0) {
                            wp[t] = acc.m;
                            wp[2 + t] = lsum;
                        }
                    }
                }
                named_sync();
                // CTA combine of the 16 warps, thread (hh, d).  The other splits publish the CTA's part as
                // exchange words; the head's last split (att_last) keeps its own in shared memory and
                // folds all S parts.
                float* own = part;  // the GEMV parts region is free between QKV and o-proj
                float* fw = part + 2 * ATT_PART;  // [2 heads][MK_MAX_S] softmax weights, then weight x sum
                if (tid < 2 * MK_WARPS) {  // weight of warp w for head hh: exp(m_w - max_w m)
                    const int hh = tid / MK_WARPS, w2 = tid % MK_WARPS;
                    float M = -INFINITY;
#pragma unroll
                    for (int i = 0; i < MK_WARPS; ++i) M = fmaxf(M, wpart[i * ATT_PART + hh]);
                    const float m = wpart[w2 * ATT_PART + hh];
                    const float f = (m == -INFINITY) ? 0.f : expf(m - M);
                    fw[hh * MK_MAX_S + w2] = f;
                    fw[(2 + hh) * MK_MAX_S + w2] = f * wpart[w2 * ATT_PART + 2 + hh];
                    if (w2 == 0) fw[(4 + hh) * MK_MAX_S] = M;
                }
                named_sync();
                if (tid < 2 * HD) {
                    const int hh = tid >> 7, d = tid & 127;
                    const float M = fw[(4 + hh) * MK_MAX_S];
                    float Ls = 0.f, Os = 0.f;
#pragma unroll
                    for (int w2 = 0; w2 < MK_WARPS; ++w2) {
                        Ls += fw[(2 + hh) * MK_MAX_S + w2];
                        Os = fmaf(wpart[w2 * ATT_PART + 4 + hh * HD + d], fw[hh * MK_MAX_S + w2], Os);
                    }
                    if (att_last) {
                        own[4 + hh * HD + d] = Os;
                        if (d == 0) {
                            own[hh] = M;
                            own[2 + hh] = Ls;
                        }
                    } else {
                        unsigned long long* pw = p.parts + ((size_t)ah * NSPLIT + aj) * ATT_PART;
                        ll_st(pw + 4 + hh * HD + d, Os, tag);
                        if (d == 0) {
                            ll_st(pw + hh, M, tag);
                            ll_st(pw + 2 + hh, Ls, tag);
                        }
                    }
                }
                if (att_last) {
                    named_sync();  // wpart fully read before the parts land in the same buffer
                    // poll the other S - 1 parts into shared memory: every thread its words
                    const unsigned long long* src = p.parts + (size_t)ah * NSPLIT * ATT_PART;
                    const int nwords = (NSPLIT - 1) * ATT_PART;
                    constexpr int NPT = ((MK_MAX_S - 1) * ATT_PART + MK_CTHREADS - 1) / MK_CTHREADS;
                    uint32_t pending = 0;
#pragma unroll
                    for (int k = 0; k < NPT; ++k)
                        if (tid + k * MK_CTHREADS < nwords) pending |= 1u << k;
                    uint32_t polls = 0;
                    while (pending && !ctl.aborted()) {
                        unsigned long long w[NPT];
#pragma unroll
                        for (int k = 0; k < NPT; ++k)  // all loads first, so they are in flight together
                            w[k] = (pending & (1u << k)) ? ll_ld(src + tid + k * MK_CTHREADS) : 0ull;
#pragma unroll
                        for (int k = 0; k < NPT; ++k) {
                            if ((pending & (1u << k)) && (uint32_t)(w[k] >> 32) == tag) {
                                big[tid + k * MK_CTHREADS] = __uint_as_float((uint32_t)w[k]);
                                pending &= ~(1u << k);
                            }
                        }
                        if (!pending) break;
                        if ((++polls & 31) == 0) {
                            if (ld_relaxed_int(ctl.g_abort) != 0) {
                                *ctl.s_abort = 1;
                            } else if (polls >= MK_POLL_LIMIT) {
                                ctl.give_up();
                            }
                        }
                        __nanosleep(32);
                    }
                    named_sync();
                    if (tid < 2 * NSPLIT) {  // weight of split j for head hh
                        const int hh = tid / NSPLIT, j = tid % NSPLIT;
                        float M = own[hh];
                        for (int i = 0; i < NSPLIT - 1; ++i) M = fmaxf(M, big[i * ATT_PART + hh]);
                        const float* pj = j < NSPLIT - 1 ? big + j * ATT_PART : own;
                        const float f = (pj[hh] == -INFINITY) ? 0.f : expf(pj[hh] - M);
                        fw[hh * MK_MAX_S + j] = f;
                        fw[(2 + hh) * MK_MAX_S + j] = f * pj[2 + hh];
                    }
                    named_sync();
                    if (tid < 2 * HD) {
                        const int hh = tid >> 7, d = tid & 127;
                        float Ls = 0.f, Os = 0.f;
#pragma unroll
                        for (int j = 0; j < MK_MAX_S; ++j) {
                            if (j < NSPLIT) {
                                const float* pj = j < NSPLIT - 1 ? big + j * ATT_PART : own;
                                Ls += fw[(2 + hh) * MK_MAX_S + j];
                                Os = fmaf(pj[4 + hh * HD + d], fw[hh * MK_MAX_S + j], Os);
                            }
                        }
                        ll_st(p.att + (2 * ah + hh) * HD + d, Os / Ls, tag);
                    }
                }
            }

            // ======== o-proj + residual (tile o0 = the rows this CTA keeps) ========
            if (no > 0) {
                {
                    const unsigned long long* a[4];
                    float x[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) a[i] = p.att + mk_col(warp * 128, lane, i);
                    ll_poll<4>(a, x, tag, ctl);
                    mk_store_frag(x, 0, xfrag, xsum, lane);
                }
                __syncwarp();
                consts2(0);
                {
                    const uint8_t* item = ring.wait(ctl);
                    float a0 = 0.f, a1 = 0.f;
                    mk_tile2(item, 2 * warp, uc, lane, a0, a1);
                    ring.release();
                    mk_put_part(part, 6, warp, lane, a0, a1);
                }
                named_sync();
                if (tid < 16) {
                    float v = 0.f;
#pragma unroll
                    for (int w2 = 0; w2 < MK_WARPS; ++w2) v += part[(6 * MK_WARPS + w2) * 16 + tid];
                    const float xm = resid[tid] + v;
                    resid[tid] = xm;
                    ll_st(p.xmid + o0 * 16 + tid, xm, tag);
                }
            }

            // ======== RMSNorm -> gate/up -> SwiGLU ========
            {
                const int col0 = warp * 128;
                float nwm[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) nwm[i] = __ldg(ly.mlp_norm + mk_col(col0, lane, i));
                const unsigned long long* a[4];
                float v[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) a[i] = p.xmid + mk_col(col0, lane, i);
                ll_poll<4>(a, v, tag, ctl);
                const float ssw = warp_sum((v[0] * v[0] + v[1] * v[1]) + (v[2] * v[2] + v[3] * v[3]));
                const float ss = mk_cta_sumsq(ssw, ssp, ssbar, ss_uses, warp, ctl);
                const float scale = 1.0f / sqrtf(ss / (float)H + EPS);
                float x[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) x[i] = v[i] * scale * nwm[i];
                mk_store_frag(x, 0, xfrag, xsum, lane);
                __syncwarp();
                consts2(0);
                for (int i = 0; i < ngu; ++i) {
                    const uint8_t* item = ring.wait(ctl);
                    float a0 = 0.f, a1 = 0.f;
                    mk_tile2(item, 2 * warp, uc, lane, a0, a1);
                    ring.release();
                    mk_put_part(part, i, warp, lane, a0, a1);
                }
                named_sync();
                if (tid < ngu * 8) {  // tile rows 0..7 are gate units, rows 8..15 the matching up units
                    const int i = tid >> 3, r8 = tid & 7;
                    float gv = 0.f, uv = 0.f;
#pragma unroll
                    for (int w2 = 0; w2 < MK_WARPS; ++w2) {
                        gv += part[(i * MK_WARPS + w2) * 16 + r8];
                        uv += part[(i * MK_WARPS + w2) * 16 + 8 + r8];
                    }
                    ll_st(p.hbuf + (g0 + i) * 8 + r8, (gv / (1.0f + expf(-gv))) * uv, tag);
                }
            }

            // ======== down + residual (+ DeepStack rows after layers 0..2) ========
            if (no > 0) {
                // this warp's units of the tile: 2w, 2w + 1 of each K-third (columns 2048 t + 128 w ..)
                const unsigned long long* a[12];
                float x[12];
#pragma unroll
                for (int th = 0; th < 3; ++th)
#pragma unroll
                    for (int i = 0; i < 4; ++i) a[th * 4 + i] = p.hbuf + mk_col(th * 2048 + warp * 128, lane, i);
                ll_poll<12>(a, x, tag, ctl);
                float a0 = 0.f, a1 = 0.f;
#pragma unroll
                for (int th = 0; th < 3; ++th) {
                    const float xt[4] = {x[th * 4 + 0], x[th * 4 + 1], x[th * 4 + 2], x[th * 4 + 3]};
                    mk_store_frag(xt, 0, xfrag, xsum, lane);
                    __syncwarp();
                    consts2(0);
                    __syncwarp();  // the next third's fragments overwrite these
                    const uint8_t* item = ring.wait(ctl);
                    mk_tile2(item, 2 * warp, uc, lane, a0, a1);
                    ring.release();
                }
                mk_put_part(part, 6, warp, lane, a0, a1);
                named_sync();
                if (tid < 16) {
                    float v = 0.f;
#pragma unroll
                    for (int w2 = 0; w2 < MK_WARPS; ++w2) v += part[(6 * MK_WARPS + w2) * 16 + tid];
                    const int row = o0 * 16 + tid;
                    float ds = 0.f;
                    if (l < 3 && ds_vi >= 0 && p.deepstack[l] != nullptr) ds = p.deepstack[l][(long long)ds_vi * H + row];
                    const float xo = resid[tid] + (v + ds);
                    resid[tid] = xo;
                    ll_st(p.xout + row, xo, tag);
                    if (l == L - 1) p.x_final[row] = xo;
                }
            }
            named_sync();  // GEMV parts are reused by the next layer's QKV
        }
    }

    // ---- end of the launch: the last CTA resets the per-launch counters and advances the epoch ----
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned old = atomicAdd(p.fin, 1u);
        if (old == (unsigned)(G - 1)) {
            __threadfence();
            *p.fin = 0;
            *(volatile unsigned*)p.epoch = ep + 1;
            __threadfence();
        }
    }
}

// Builds the CTA streams from the slice-major q4s matrices of every layer: CTA c's items of layer
// l are its QKV tiles, its o tile, its gate/up tiles and the three K-thirds of its down tile, each
// tile's 64-column units in K order.  One CTA per (stream CTA, layer).
__global__ void mk_pack_kernel(uint8_t* dst, const unsigned long long* cta_base, const uint8_t* const* mats,
                               int n_layers, int G) {
    const int c = blockIdx.x % G, l = blockIdx.x / G;
    if (l >= n_layers) return;
    int q0, q1, o0, o1, g0, g1;
    mk_range(MK_QKV_TILES, c, G, q0, q1);
    mk_range(MK_O_TILES, c, G, o0, o1);
    mk_range(MK_GU_TILES, c, G, g0, g1);
    const int per_layer = (q1 - q0) + 4 * (o1 - o0) + (g1 - g0);
    uint8_t* out = dst + cta_base[c] + (size_t)l * per_layer * MK_ITEM;
    // (matrix, n_tiles, upt, first tile, tiles) in stream order
    const uint8_t* m[4] = {mats[l * 4 + 0], mats[l * 4 + 1], mats[l * 4 + 2], mats[l * 4 + 3]};
    const int nt[4] = {MK_QKV_TILES, MK_O_TILES, MK_GU_TILES, MK_O_TILES};
    const int upt[4] = {H / 64, H / 64, H / 64, FF / 64};
    const int t0[4] = {q0, o0, g0, o0};
    const int tn[4] = {q1 - q0, o1 - o0, g1 - g0, o1 - o0};
    size_t off = 0;
    for (int ph = 0; ph < 4; ++ph) {
        const int units = tn[ph] * upt[ph];
        const int chunks = units * (Q4_UNIT_BYTES / 16);
        for (int i = threadIdx.x; i < chunks; i += blockDim.x) {
            const int u = i / (Q4_UNIT_BYTES / 16), w = i % (Q4_UNIT_BYTES / 16);
            const int tile = t0[ph] + u / upt[ph], kk = u % upt[ph];
            const uint4* src = reinterpret_cast<const uint4*>(
                m[ph] + icua_layout::unit_offset(FMT_Q4S, nt[ph], upt[ph], tile, kk));
            reinterpret_cast<uint4*>(out + off + (size_t)u * Q4_UNIT_BYTES)[w] = src[w];
        }
        off += (size_t)units * Q4_UNIT_BYTES;
    }
}

}  // namespace icua
