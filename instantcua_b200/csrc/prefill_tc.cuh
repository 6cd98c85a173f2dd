// Causal GQA prefill attention on the 5th-generation tensor cores.
//
// Replaces the reference's k_prefill_attn (Shaders.swift:1101-1216: scores and probabilities of
// a row block in threadgroup memory) for the prompt rows of a prefill call, which attend every
// earlier cache slot of the session and themselves.
//
// Design (B200): one CTA = 128 prompt rows x one query head (head dim 128); the two query heads of
// a GQA group read the same K / V tiles (the second CTA from L2).  Q (the row kernel's rotated,
// 1/sqrt(128)-scaled q in the cache type) arrives once by TMA as two 64-dim swizzle atoms.  K
// tiles of 64 slots come straight from the cache: its rows store 16-byte chunk c at c ^ (slot & 7)
// within each 128-byte half, which is exactly the 128-byte swizzle of a tile whose first slot is a
// multiple of 8, so a 4-D TMA map (dims 64 x 2 halves x slots x heads, no TMA swizzle) lands each
// half as a ready K-major atom.  V enters the P V product as V^T [dims][slots] (K-major), written
// per call by vt kernels, always in fp16 (a bf16 cache's values convert to fp16 exactly within the
// fp16 range), so P is rounded to fp16 for both cache types: 11 significant bits instead of bf16's
// 8 in the probabilities.  S = Q K^T (M=128, N=64, K=128) and O_j = P_j V_j (M=128, N=128, K=64)
// run on tcgen05 with S, P and O double-buffered; four softmax warps own one row per thread (the
// tensor-memory lane), mask slots past the row's position on the diagonal blocks only, and fold
// O_j into fp32 registers after producing the next P.  Every wait is bounded.
#pragma once
#include <cuda.h>

#include <type_traits>

#include "attn_tc.cuh"
#include "common.cuh"
#include "gemm_tc.cuh"

namespace icua {

constexpr int PT_BQ = 128;         // prompt rows per CTA (UMMA M)
constexpr int PT_BK = 64;          // cache slots per block
constexpr int PT_THREADS = 192;    // warp 0 TMA, warp 1 tensor memory + MMA, warps 2-5 softmax
constexpr int PT_TMEM_COLS = 512;  // S [2][128 x 64] at 0, 64; O [2][128 x 128] at 128, 256
constexpr int PT_NS = 3;           // K / V^T ring stages

struct PrefillTcSmem {
    static constexpr int q_off = 0;                       // 2 atoms [128 rows][64 dims], 32 KB
    static constexpr int k_off = 32768;                   // PT_NS x 2 atoms [64 slots][64 dims], 16 KB each
    static constexpr int vt_off = k_off + PT_NS * 16384;  // PT_NS x [128 dims][64 slots], 16 KB each
    static constexpr int p_off = vt_off + PT_NS * 16384;  // 2 x [128 rows][64 slots], 16 KB each
    // q_full, kv_full[PT_NS], kv_empty[PT_NS], s_full[2], p_full[2], o_full[2], done
    static constexpr int bar_off = p_off + 2 * 16384;
    static constexpr int tmem_off = bar_off + (2 * PT_NS + 8) * 8;
    static constexpr int total = tmem_off + 16;
    static constexpr int alloc = total + 1024;
};

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
        : "memory");
}

// Instruction descriptor of kind::f16 for the cache type: fp16 or bf16 A and B (the same type),
// fp32 accumulator, both K-major.
template <typename KVT>
__host__ __device__ constexpr uint32_t umma_idesc_kv(int M, int N) {
    return umma_idesc_f16(M, N) | (std::is_same<KVT, __nv_bfloat16>::value ? ((1u << 7) | (1u << 10)) : 0u);
}

template <typename KVT>
__device__ __forceinline__ uint32_t pack_kv2(float a, float b) {
    const KVT x = float_to_kv<KVT>(a), y = float_to_kv<KVT>(b);
    return (uint32_t)(*reinterpret_cast<const uint16_t*>(&x)) | ((uint32_t)(*reinterpret_cast<const uint16_t*>(&y)) << 16);
}

// qmap: q [n][16][128] in the cache type (4-D: 64 dims x 2 halves x 16 heads x n rows, box 64 x 1 x 1 x 128,
// 128-byte swizzle); kmap: this layer's K cache (4-D: 64 x 2 x max_ctx x 8, box 64 x 1 x 64 x 1, no
// swizzle: the rows are stored swizzled); vtmap: V^T [8][128][vstride] (3-D: slots x 128 x 8, box
// 64 x 128 x 1, 128-byte swizzle).  out: fp16 [n][2048], head qh at 128 qh.  Rows r of the prompt
// sit at cache slot pos0 + r.  Grid (ceil(n / 128), 16), longest row blocks first.
template <typename KVT>
__global__ void __launch_bounds__(PT_THREADS, 1) prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                        const __grid_constant__ CUtensorMap kmap,
                                                                        const __grid_constant__ CUtensorMap vtmap,
                                                                        int n, int pos0, __half* out, int* err) {
    using S = PrefillTcSmem;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base_u = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((base_u + 1023u) & ~1023u) - base_u);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::bar_off);
    uint64_t* q_full = bars;
    uint64_t* kv_full = bars + 1;
    uint64_t* kv_empty = kv_full + PT_NS;
    uint64_t* s_full = kv_empty + PT_NS;
    uint64_t* p_full = s_full + 2;
    uint64_t* o_full = p_full + 2;
    uint64_t* done = o_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::tmem_off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qh = blockIdx.y, kvh = qh >> 1;
    const int r0 = (gridDim.x - 1 - blockIdx.x) * PT_BQ;  // longest (last) row blocks first
    const int kend = pos0 + min(r0 + PT_BQ, n);          // slots [0, kend) are read
    const int nblk = (kend + PT_BK - 1) / PT_BK;
    const int diag0 = pos0 + r0;                         // slots past this need the causal mask

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < PT_NS; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], 4);
            mbar_init(&o_full[b], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, PT_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto s_tm = [&](int b) { return tmem + (uint32_t)(64 * b); };
    auto o_tm = [&](int b) { return tmem + (uint32_t)(128 + 128 * b); };

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&qmap) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&kmap) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&vtmap) : "memory");
            mbar_expect_tx(q_full, 32768);
            tma_load_4d(smem + S::q_off, &qmap, 0, 0, qh, r0, q_full);
            tma_load_4d(smem + S::q_off + 16384, &qmap, 0, 1, qh, r0, q_full);
            int j = 0;
            for (; j < nblk; ++j) {
                const int s = j % PT_NS;
                if (j >= PT_NS && !mbar_wait_bounded(&kv_empty[s], (uint32_t)((j / PT_NS - 1) & 1))) {
                    atomicOr(err, ERR_WAIT_PREFILL);
                    break;
                }
                mbar_expect_tx(&kv_full[s], 32768);
                uint8_t* kd = smem + S::k_off + s * 16384;
                tma_load_4d(kd, &kmap, 0, 0, j * PT_BK, kvh, &kv_full[s]);
                tma_load_4d(kd + 8192, &kmap, 0, 1, j * PT_BK, kvh, &kv_full[s]);
                tma_load_3d(smem + S::vt_off + s * 16384, &vtmap, j * PT_BK, 0, kvh, &kv_full[s]);
            }
            mbar_wait_bounded(q_full, 0);
            for (int c = (j > PT_NS ? j - PT_NS : 0); c < j; ++c)
                mbar_wait_bounded(&kv_full[c % PT_NS], (uint32_t)((c / PT_NS) & 1));
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t id_s = umma_idesc_kv<KVT>(PT_BQ, PT_BK), id_o = umma_idesc_kv<__half>(PT_BQ, 128);
            const uint32_t q_sa = smem_u32(smem + S::q_off);
            bool ok = mbar_wait_bounded(q_full, 0);
            auto issue_s = [&](int j) -> bool {
                if (!mbar_wait_bounded(&kv_full[j % PT_NS], (uint32_t)((j / PT_NS) & 1))) return false;
                tc_fence_after();
                const uint32_t k_sa = smem_u32(smem + S::k_off + (j % PT_NS) * 16384);
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {  // K = 128 dims: two atoms of four K=16 steps
                    const uint64_t ad = umma_desc_sw128(q_sa + (ks >> 2) * 16384) + 2 * (ks & 3);
                    const uint64_t bd = umma_desc_sw128(k_sa + (ks >> 2) * 8192) + 2 * (ks & 3);
                    tc_mma_f16(s_tm(j & 1), ad, bd, id_s, ks != 0);
                }
                tc_commit(&s_full[j & 1]);
                return true;
            };
            if (ok) ok = issue_s(0);
            if (ok && nblk > 1) ok = issue_s(1);
            for (int j = 0; ok && j < nblk; ++j) {
                const int b = j & 1;
                if (!mbar_wait_bounded(&p_full[b], (uint32_t)((j >> 1) & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t pd = umma_desc_sw128(smem_u32(smem + S::p_off + b * 16384));
                const uint64_t vd = umma_desc_sw128(smem_u32(smem + S::vt_off + (j % PT_NS) * 16384));
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) tc_mma_f16(o_tm(b), pd + 2 * ks, vd + 2 * ks, id_o, ks != 0);
                tc_commit(&o_full[b]);
                tc_commit(&kv_empty[j % PT_NS]);
                if (j + 2 < nblk) ok = issue_s(j + 2);
            }
            if (!ok) atomicOr(err, ERR_WAIT_PREFILL);
            tc_commit(done);
            mbar_wait_bounded(done, 0);
        }
    } else {
        const int quarter = warp & 3, row = quarter * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        const int qpos = pos0 + min(r0 + row, n - 1);  // rows past n compute a copy of the last one
        const float l2e = 1.4426950408889634f;      // q is pre-scaled by 1/sqrt(128)
        float o[128];
#pragma unroll
        for (int d = 0; d < 128; ++d) o[d] = 0.f;
        float m = -INFINITY, l = 0.f, corr_prev = 0.f;
        bool ok = true;
        auto fold = [&](int i, float c) -> bool {
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&o_full[i & 1], (uint32_t)((i >> 1) & 1)))) return false;
            tc_fence_after();
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float a[64];
                tmem_ld64(o_tm(i & 1) + lane_off + 64 * half, a);
#pragma unroll
                for (int d = 0; d < 64; ++d) o[64 * half + d] = fmaf(o[64 * half + d], c, a[d]);
            }
            tc_fence_before();
            return true;
        };
        for (int j = 0; j < nblk; ++j) {
            const int b = j & 1;
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_full[b], (uint32_t)((j >> 1) & 1)))) {
                ok = false;
                break;
            }
            tc_fence_after();
            float v[64];
            tmem_ld64(s_tm(b) + lane_off, v);
            const int k0 = j * PT_BK;
            if (k0 + PT_BK - 1 > diag0) {  // a diagonal block: slots past this row's position are masked
#pragma unroll
                for (int i = 0; i < 64; ++i) v[i] = (k0 + i <= qpos) ? v[i] : -INFINITY;
            }
            float bm = v[0];
#pragma unroll
            for (int i = 1; i < 64; ++i) bm = fmaxf(bm, v[i]);
            const float mn = fmaxf(m, bm);
            const float corr = ex2_approx((m - mn) * l2e);
            m = mn;
            const float off = -mn * l2e;
            float sum = 0.f;
            uint8_t* P = smem + S::p_off + b * 16384;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float p0 = ex2_approx(fmaf(v[8 * c + 2 * e], l2e, off));
                    const float p1 = ex2_approx(fmaf(v[8 * c + 2 * e + 1], l2e, off));
                    sum += p0 + p1;
                    w[e] = pack_kv2<__half>(p0, p1);
                }
                *reinterpret_cast<uint4*>(P + row * 128 + ((c ^ (row & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
            l = l * corr + sum;
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[b]);
            if (j >= 1 && !fold(j - 1, corr_prev)) {
                ok = false;
                break;
            }
            corr_prev = corr;
        }
        if (ok && nblk >= 1) ok = fold(nblk - 1, corr_prev);
        if (!ok) {
            if (lane == 0) atomicOr(err, ERR_WAIT_PREFILL);
        } else if (r0 + row < n) {
            const float il = 1.0f / l;
            uint4* dst = reinterpret_cast<uint4*>(out + (size_t)(r0 + row) * H + qh * HD);
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const __half2 p2 = __floats2half2_rn(o[8 * c + 2 * e] * il, o[8 * c + 2 * e + 1] * il);
                    w[e] = *reinterpret_cast<const uint32_t*>(&p2);
                }
                dst[c] = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, PT_TMEM_COLS);
    }
}

// V^T of the prompt rows: vt[h][d][pos0 + i] = v of row i (qkv columns 3072 + 128 h + d) rounded to
// the cache type as the cache stores it, held in fp16; 32 x 32 tiles through shared memory.  Grid
// (ceil(n / 32), 1024 / 32), 32 x 8.
template <typename KVT>
__global__ void __launch_bounds__(256) prefill_vt_kernel(const float* qkv, int n, int pos0, __half* vt, int vstride) {
    __shared__ float tile[32][33];
    const int i0 = blockIdx.x * 32, c0 = blockIdx.y * 32;  // c = h * 128 + d
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int i = i0 + r;
        tile[r][threadIdx.x] = i < n ? qkv[(size_t)i * QKV_ROWS + 3072 + c0 + threadIdx.x] : 0.f;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int i = i0 + threadIdx.x;
        if (i < n) vt[(size_t)(c0 + r) * vstride + pos0 + i] = __float2half_rn(kv_to_float(float_to_kv<KVT>(tile[threadIdx.x][r])));
    }
}

// V^T of the cache slots [0, n_slots) written by earlier calls: vt[h][d][p] = vc[h][p][kv_swz(d, p)],
// in fp16.  Grid (ceil(n_slots / 32), 1024 / 32), 32 x 8.
template <typename KVT>
__global__ void __launch_bounds__(256) prefill_vt_gather_kernel(const KVT* vc, int max_ctx, int n_slots, __half* vt,
                                                                int vstride) {
    __shared__ KVT tile[32][34];
    const int p0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    const int h = c0 >> 7, d0 = c0 & 127;
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int p = p0 + r;
        tile[r][threadIdx.x] = p < n_slots ? vc[((size_t)h * max_ctx + p) * HD + kv_swz(d0 + threadIdx.x, p)]
                                           : float_to_kv<KVT>(0.f);
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int p = p0 + threadIdx.x;
        if (p < n_slots) vt[(size_t)(c0 + r) * vstride + p] = __float2half_rn(kv_to_float(tile[threadIdx.x][r]));
    }
}

}  // namespace icua
