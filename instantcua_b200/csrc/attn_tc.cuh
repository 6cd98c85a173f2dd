// Bidirectional multi-head attention on the 5th-generation tensor cores (vision encoder).
//
// Replaces the reference's k_vit_attn (Shaders.swift:292-395: scores, probabilities and output
// per 16-query threadgroup through threadgroup memory).
//
// Design (B200): one CTA = 128 queries x one head (head dim 64).  Q (once), K and V^T tiles of 64
// keys arrive by TMA (3-D maps per head, so rows past the image read as zeros) into 128-byte-
// swizzled K-major tiles; a single thread issues tcgen05.mma: S = Q K^T (M=128, N=64, K=64) into
// tensor memory, and after the softmax the block product O_j = P V_j (M=128, N=64, K=64, P from
// shared memory, V^T as the K-major B operand) into tensor memory.  Four softmax warps own one
// query row per thread (tensor-memory lane = row): they read the row's 64 scores with
// tcgen05.ld, keep the running max and sum, write P (fp16) into the swizzled tile, and fold O_j
// into the row's fp32 output registers with the rescale factor.  S, P and O are double-buffered
// so that products and softmax overlap; the K / V^T ring has three stages.  Every wait is bounded and reports through the error flag; tensor
// memory is freed on every path.
#pragma once
#include <cuda.h>

#include "gemm_tc.cuh"
#include "vision.cuh"

namespace icua {

constexpr int VT_BQ = 128;         // queries per CTA (UMMA M)
constexpr int VT_BK = 64;          // keys per block
constexpr int VT_THREADS = 192;    // warp 0 TMA, warp 1 tensor memory + MMA, warps 2-5 softmax
constexpr int VT_TMEM_COLS = 256;  // S [2][128 x 64] at columns 0, 64; O blocks [2][128 x 64] at 128, 192
constexpr int VT_NS = 3;           // K / V^T ring stages

struct VitAttnSmem {
    static constexpr int q_off = 0;                      // [128 queries][64] fp16, 16 KB
    static constexpr int k_off = 16384;                  // VT_NS x [64 keys][64 dims], 8 KB each
    static constexpr int vt_off = k_off + VT_NS * 8192;  // VT_NS x [64 dims][64 keys], 8 KB each
    static constexpr int p_off = vt_off + VT_NS * 8192;  // 2 x [128 queries][64 keys] fp16, 16 KB each
    // q_full, kv_full[VT_NS], kv_empty[VT_NS], s_full[2], p_full[2], o_full[2], done
    static constexpr int bar_off = p_off + 2 * 16384;
    static constexpr int tmem_off = bar_off + (2 * VT_NS + 8) * 8;
    static constexpr int total = tmem_off + 16;
    static constexpr int alloc = total + 1024;           // room to align the tiles to 1024 bytes
};

// 64 consecutive fp32 columns of this warp's 32 tensor-memory lanes (two x32 loads, one wait: the
// load latency is paid once).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
    uint32_t r[64];
#define ICUA_LD32(OFF, B)                                                                                              \
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"      \
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                             \
                 : "=r"(r[B + 0]), "=r"(r[B + 1]), "=r"(r[B + 2]), "=r"(r[B + 3]), "=r"(r[B + 4]), "=r"(r[B + 5]),        \
                   "=r"(r[B + 6]), "=r"(r[B + 7]), "=r"(r[B + 8]), "=r"(r[B + 9]), "=r"(r[B + 10]), "=r"(r[B + 11]),     \
                   "=r"(r[B + 12]), "=r"(r[B + 13]), "=r"(r[B + 14]), "=r"(r[B + 15]), "=r"(r[B + 16]),                 \
                   "=r"(r[B + 17]), "=r"(r[B + 18]), "=r"(r[B + 19]), "=r"(r[B + 20]), "=r"(r[B + 21]),                 \
                   "=r"(r[B + 22]), "=r"(r[B + 23]), "=r"(r[B + 24]), "=r"(r[B + 25]), "=r"(r[B + 26]),                 \
                   "=r"(r[B + 27]), "=r"(r[B + 28]), "=r"(r[B + 29]), "=r"(r[B + 30]), "=r"(r[B + 31])                  \
                 : "r"(taddr + OFF)                                                                                    \
                 : "memory")
    ICUA_LD32(0, 0);
    ICUA_LD32(32, 32);
#undef ICUA_LD32
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// 2^x by the hardware approximation (ex2.approx, flush-to-zero): the softmax probabilities are
// rounded to fp16 right after, well above its error.
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// qmap / kmap: fp16 [16 heads][n][64] (box 64 x 128 / 64 x 64 x 1); vtmap: fp16 [16][64][n]
// with rows of npad keys (box 64 keys x 64 dims x 1).  out: fp16 [n][1024], head h at 64 h.
// Grid (ceil(n / 128), 16).
//
// Block j: S_j = Q K_j^T into S buffer j % 2, P_j (fp16) into P buffer j % 2, O_j = P_j V_j into
// O buffer j % 2.  The MMA thread issues S_{j+2} as soon as the softmax has consumed S_j, so the
// next block's scores are ready when the softmax gets to them, and the softmax folds O_{j-1} into
// its registers only after it has produced P_j: neither waits on a round trip to the other.
__global__ void __launch_bounds__(VT_THREADS, 2) vit_attn_tc_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                    const __grid_constant__ CUtensorMap kmap,
                                                                    const __grid_constant__ CUtensorMap vtmap, int n,
                                                                    __half* out, int* err) {
    using S = VitAttnSmem;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base_u = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((base_u + 1023u) & ~1023u) - base_u);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::bar_off);
    uint64_t* q_full = bars;
    uint64_t* kv_full = bars + 1;
    uint64_t* kv_empty = kv_full + VT_NS;
    uint64_t* s_full = kv_empty + VT_NS;  // [2]
    uint64_t* p_full = s_full + 2;        // [2]
    uint64_t* o_full = p_full + 2;        // [2]
    uint64_t* done = o_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::tmem_off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y, q0 = blockIdx.x * VT_BQ;
    const int nblk = (n + VT_BK - 1) / VT_BK;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < VT_NS; ++s) {
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
        tmem_alloc(tmem_slot, VT_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto s_tm = [&](int b) { return tmem + (uint32_t)(64 * b); };
    auto o_tm = [&](int b) { return tmem + (uint32_t)(128 + 64 * b); };

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&qmap) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&kmap) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&vtmap) : "memory");
            mbar_expect_tx(q_full, 16384);
            tma_load_3d(smem + S::q_off, &qmap, 0, q0, h, q_full);
            int j = 0;
            for (; j < nblk; ++j) {
                const int s = j % VT_NS;
                if (j >= VT_NS && !mbar_wait_bounded(&kv_empty[s], (uint32_t)((j / VT_NS - 1) & 1))) {
                    atomicOr(err, ERR_WAIT_PREFILL);
                    break;
                }
                mbar_expect_tx(&kv_full[s], 16384);
                tma_load_3d(smem + S::k_off + s * 8192, &kmap, 0, j * VT_BK, h, &kv_full[s]);
                tma_load_3d(smem + S::vt_off + s * 8192, &vtmap, j * VT_BK, 0, h, &kv_full[s]);
            }
            // copies still landing complete before the CTA may exit (at once on success)
            mbar_wait_bounded(q_full, 0);
            for (int c = (j > VT_NS ? j - VT_NS : 0); c < j; ++c)
                mbar_wait_bounded(&kv_full[c % VT_NS], (uint32_t)((c / VT_NS) & 1));
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(VT_BQ, VT_BK);  // both products: M = 128, N = 64
            const uint64_t qd = umma_desc_sw128(smem_u32(smem + S::q_off));
            bool ok = mbar_wait_bounded(q_full, 0);
            // S_j = Q K_j^T into S buffer j % 2
            auto issue_s = [&](int j) -> bool {
                if (!mbar_wait_bounded(&kv_full[j % VT_NS], (uint32_t)((j / VT_NS) & 1))) return false;
                tc_fence_after();
                const uint64_t kd = umma_desc_sw128(smem_u32(smem + S::k_off + (j % VT_NS) * 8192));
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) tc_mma_f16(s_tm(j & 1), qd + 2 * ks, kd + 2 * ks, idesc, ks != 0);
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
                const uint64_t vd = umma_desc_sw128(smem_u32(smem + S::vt_off + (j % VT_NS) * 8192));
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) tc_mma_f16(o_tm(b), pd + 2 * ks, vd + 2 * ks, idesc, ks != 0);
                tc_commit(&o_full[b]);
                tc_commit(&kv_empty[j % VT_NS]);
                if (j + 2 < nblk) ok = issue_s(j + 2);  // S buffer b: S_j has been consumed
            }
            if (!ok) atomicOr(err, ERR_WAIT_PREFILL);
            // every product issued has completed before tensor memory is freed (error paths too)
            tc_commit(done);
            mbar_wait_bounded(done, 0);
        }
    } else {
        // softmax warps: warp w reads tensor-memory lanes 32 (w % 4) ..; thread = query row
        const int quarter = warp & 3, row = quarter * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        const float sl2 = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
        float o[64];
#pragma unroll
        for (int d = 0; d < 64; ++d) o[d] = 0.f;
        float m = -INFINITY, l = 0.f, corr_prev = 0.f;
        bool ok = true;
        // folds O_i (O buffer i % 2) into the registers: o = o * c + O_i
        auto fold = [&](int i, float c) -> bool {
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&o_full[i & 1], (uint32_t)((i >> 1) & 1)))) return false;
            tc_fence_after();
            float a[64];
            tmem_ld64(o_tm(i & 1) + lane_off, a);
#pragma unroll
            for (int d = 0; d < 64; ++d) o[d] = fmaf(o[d], c, a[d]);
            tc_fence_before();  // the O reads are ordered before the next product into this buffer
            return true;
        };
        for (int j = 0; j < nblk; ++j) {
            const int b = j & 1;
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_full[b], (uint32_t)((j >> 1) & 1)))) {
                ok = false;
                break;
            }
            tc_fence_after();
            // raw scores; the scale enters the exponent: p = 2^(s * sl2 - max * sl2)
            float v[64];
            tmem_ld64(s_tm(b) + lane_off, v);
            const int k0 = j * VT_BK;
            if (k0 + VT_BK > n) {  // the last block: keys past n take no weight
#pragma unroll
                for (int i = 0; i < 64; ++i) v[i] = (k0 + i < n) ? v[i] : -INFINITY;
            }
            float bm = v[0];
#pragma unroll
            for (int i = 1; i < 64; ++i) bm = fmaxf(bm, v[i]);
            const float mn = fmaxf(m, bm);
            const float corr = ex2_approx((m - mn) * sl2);  // 0 on the first block (m = -inf)
            m = mn;
            const float off = -mn * sl2;
            float sum = 0.f;
            uint8_t* P = smem + S::p_off + b * 16384;
#pragma unroll
            for (int c = 0; c < 8; ++c) {  // 16-byte chunks of 8 keys
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float p0 = ex2_approx(fmaf(v[8 * c + 2 * e], sl2, off));
                    const float p1 = ex2_approx(fmaf(v[8 * c + 2 * e + 1], sl2, off));
                    sum += p0 + p1;
                    const __half2 p2 = __floats2half2_rn(p0, p1);
                    w[e] = *reinterpret_cast<const uint32_t*>(&p2);
                }
                *reinterpret_cast<uint4*>(P + row * 128 + ((c ^ (row & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
            l = l * corr + sum;
            fence_proxy_async_smem();  // P (generic proxy) -> visible to the tensor core
            tc_fence_before();         // the S reads are ordered before the next product into this buffer
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[b]);
            // O_{j-1} ran while P_j was being produced
            if (j >= 1 && !fold(j - 1, corr_prev)) {
                ok = false;
                break;
            }
            corr_prev = corr;
        }
        if (ok && nblk >= 1) ok = fold(nblk - 1, corr_prev);
        if (!ok) {
            if (lane == 0) atomicOr(err, ERR_WAIT_PREFILL);
        } else if (q0 + row < n) {
            const float il = 1.0f / l;
            uint4* dst = reinterpret_cast<uint4*>(out + (size_t)(q0 + row) * VIT_HIDDEN + h * VIT_HD);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
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
        tmem_dealloc(tmem, VT_TMEM_COLS);
    }
}

// vT[h][d][p] = v of head h, dim d, patch p (fp16, rows of npad keys): the K-major B operand of
// the P V product.  32 x 32 tiles through shared memory.  Grid (ceil(n / 32), 1024 / 32), 32 x 8.
__global__ void __launch_bounds__(256) vit_vt_kernel(const float* qkv, int n, int npad, __half* vt) {
    __shared__ float tile[32][33];
    const int p0 = blockIdx.x * 32, c0 = blockIdx.y * 32;  // c = h * 64 + d
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int p = p0 + r;
        tile[r][threadIdx.x] = p < n ? qkv[(size_t)p * VIT_QKV + 2 * VIT_HIDDEN + c0 + threadIdx.x] : 0.f;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int p = p0 + threadIdx.x;
        if (p < n) vt[(size_t)(c0 + r) * npad + p] = __float2half_rn(tile[threadIdx.x][r]);
    }
}

}  // namespace icua
