// Row-parallel prefill kernels around the tensor-core GEMM: prompt embedding, RMSNorm into fp16
// GEMM inputs, per-head QK norm + M-RoPE + KV append, and causal GQA flash attention.
//
// Reference counterparts: k_embed_prompt (Shaders.swift:676-692), k_rmsnorm_rows_h (838-864),
// k_qk_norm_rope (871-923) and k_prefill_attn (1101-1216).  The reference materialises the score
// matrix in threadgroup memory; here attention is a flash (online-softmax) kernel on the tensor
// cores that never leaves registers, with K/V tiles bulk-copied from the swizzled cache rows.
// Each kernel starts with griddepcontrol.wait, so it may be launched as a programmatic dependent
// of the kernel before it (its launch then overlaps that kernel's tail).
#pragma once
#include "attn_decode.cuh"
#include "common.cuh"
#include "gemv.cuh"

namespace icua {

// x[i] = pooler row (IMAGE_PAD tokens inside the visual block) or the dequantised embedding row.
// One CTA of 256 threads per prompt row.
__global__ void prefill_embed_kernel(const int* prompt, int n, int vis_off, int n_vis, const float* pooler,
                                     const uint8_t* embed, int embed_tiles, int embed_fmt, float* x) {
    pdl_wait();
    pdl_launch_dependents();
    const int i = blockIdx.x;
    if (i >= n) return;
    const int tok = prompt[i];
    const int v = i - vis_off;
    const float* vis_row = (tok == IMAGE_PAD_ID && vis_off >= 0 && pooler != nullptr && v >= 0 && v < n_vis)
                               ? pooler + (size_t)v * H : nullptr;
    float* xr = x + (size_t)i * H;
    for (int k = threadIdx.x; k < H; k += blockDim.x)
        xr[k] = vis_row ? vis_row[k] : embed_value(embed_fmt, embed, embed_tiles, tok, k);
}

// out[i] = fp16(x[i] * rsqrt(mean(x[i]^2) + eps) * w): the fp16 GEMM input of a prompt row.
// One CTA of 256 threads per row of 2048.
__global__ void __launch_bounds__(256) rmsnorm_rows_f16_kernel(const float* x, const float* w, int n, __half* out) {
    __shared__ float red[8];
    pdl_wait();
    pdl_launch_dependents();
    const int i = blockIdx.x, tid = threadIdx.x;
    if (i >= n) return;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)i * H);
    const float4 a = xr[tid], b = xr[tid + 256];
    float ss = a.x * a.x;
    ss = fmaf(a.y, a.y, ss);
    ss = fmaf(a.z, a.z, ss);
    ss = fmaf(a.w, a.w, ss);
    ss = fmaf(b.x, b.x, ss);
    ss = fmaf(b.y, b.y, ss);
    ss = fmaf(b.z, b.z, ss);
    ss = fmaf(b.w, b.w, ss);
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < 8; ++w2) tot += red[w2];
    const float r = 1.0f / sqrtf(tot / (float)H + EPS);
    const float4 wa = reinterpret_cast<const float4*>(w)[tid], wb = reinterpret_cast<const float4*>(w)[tid + 256];
    __half2* o = reinterpret_cast<__half2*>(out + (size_t)i * H);
    o[2 * tid] = __floats2half2_rn(a.x * r * wa.x, a.y * r * wa.y);
    o[2 * tid + 1] = __floats2half2_rn(a.z * r * wa.z, a.w * r * wa.w);
    o[2 * (tid + 256)] = __floats2half2_rn(b.x * r * wb.x, b.y * r * wb.y);
    o[2 * (tid + 256) + 1] = __floats2half2_rn(b.z * r * wb.z, b.w * r * wb.w);
}

// Per prompt row: RMSNorm(128) of the 16 q and 8 k heads, rotate-half RoPE from the cache slot's
// (cos, sin) row, q scaled by 1/sqrt(128) into q_out [n][16][128] fp32, k and v rounded to the
// cache type and stored at slot pos0 + i in the swizzled row order.  One CTA (8 warps) per row,
// one warp per head vector (32 vectors: 16 q, 8 k, 8 v).
template <typename KVT>
__global__ void __launch_bounds__(256) qk_rope_kv_kernel(const float* qkv, int n, const float* q_norm,
                                                         const float* k_norm, const float2* rope, int pos0, KVT* kc,
                                                         KVT* vc, int max_ctx, float* q_out) {
    const int i = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (i >= n) return;
    const int pos = pos0 + i;
    const float* row = qkv + (size_t)i * QKV_ROWS;
    float2 cs4[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) cs4[e] = rope[(size_t)pos * 64 + 4 * (lane & 15) + e];
    const float4 qn = reinterpret_cast<const float4*>(q_norm)[lane];
    const float4 kn = reinterpret_cast<const float4*>(k_norm)[lane];
    pdl_wait();  // the norm weights and the RoPE table do not depend on the previous kernel
    pdl_launch_dependents();
#pragma unroll 1
    for (int vi = warp; vi < 32; vi += 8) {
        const float4 x4 = reinterpret_cast<const float4*>(row + vi * HD)[lane];
        float x[4] = {x4.x, x4.y, x4.z, x4.w};
        if (vi < 24) {
            const float4 nw = vi < 16 ? qn : kn;
            const float nwv[4] = {nw.x, nw.y, nw.z, nw.w};
            const float ss = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
            const float r = 1.0f / sqrtf(ss / (float)HD + EPS);
#pragma unroll
            for (int e = 0; e < 4; ++e) x[e] = x[e] * r * nwv[e];
            float y[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
                const float2 cs = cs4[e];
                y[e] = lane < 16 ? x[e] * cs.x - partner * cs.y : x[e] * cs.x + partner * cs.y;
            }
            if (vi < 16) {
                const float sc = 0.08838834764831845f;  // 1 / sqrt(128)
                reinterpret_cast<float4*>(q_out + ((size_t)i * NQ + vi) * HD)[lane] =
                    make_float4(y[0] * sc, y[1] * sc, y[2] * sc, y[3] * sc);
            } else {
                KVT* dst = kc + ((size_t)(vi - 16) * max_ctx + pos) * HD;
#pragma unroll
                for (int e = 0; e < 4; ++e) dst[kv_swz(4 * lane + e, pos)] = float_to_kv<KVT>(y[e]);
            }
        } else {
            KVT* dst = vc + ((size_t)(vi - 24) * max_ctx + pos) * HD;
#pragma unroll
            for (int e = 0; e < 4; ++e) dst[kv_swz(4 * lane + e, pos)] = float_to_kv<KVT>(x[e]);
        }
    }
}

// ---- causal GQA prefill attention ------------------------------------------------------------
constexpr int PA_BQ = 32;   // query rows per CTA and q head (2 warps x 16 rows)
constexpr int PA_BK = 64;   // cache rows per stage
constexpr int PA_NS = 2;    // stages
constexpr int PA_THREADS = 128;

template <typename KVT>
struct PrefillAttnSmem {
    static constexpr int row_bytes = HD * (int)sizeof(KVT);
    static constexpr int stage_bytes = 2 * PA_BK * row_bytes;  // K rows then V rows
    static constexpr int bars_off = PA_NS * stage_bytes;
    static constexpr int total = bars_off + PA_NS * 8;
};

// One CTA per (block of 32 prompt rows, kv head); warps 0-1 take q head 2h, warps 2-3 q head
// 2h+1, 16 rows each, so every K/V tile in shared memory serves both heads of the GQA group.
// Query row i sits at cache slot pos0 + i and attends slots [0, pos0 + i].  Scores and the
// softmax stay in registers (m16n8k16 accumulators, fp32); q and the probabilities enter the
// MMAs in the cache type, the precision of the reference prefill (fp16 operands, fp32
// accumulation).  Small row blocks keep the causal critical path (the last block reads every
// slot) short; blocks are scheduled longest first.
template <typename KVT>
__global__ void __launch_bounds__(PA_THREADS) prefill_attn_kernel(const float* q, const KVT* kc, const KVT* vc,
                                                                  int max_ctx, int n, int pos0, __half* out, int* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    using S = PrefillAttnSmem<KVT>;
    constexpr int RB = S::row_bytes;
    pdl_wait();
    pdl_launch_dependents();
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::bars_off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int h = blockIdx.y;
    const int qb = gridDim.x - 1 - blockIdx.x;   // longest blocks first
    const int r0 = qb * PA_BQ;
    const int hh = warp >> 1, qh = 2 * h + hh;
    const int wr0 = r0 + 16 * (warp & 1);        // first row of this warp
    const int kend = pos0 + min(r0 + PA_BQ, n);   // cache slots [0, kend) are read
    const int nblk = (kend + PA_BK - 1) / PA_BK;
    const KVT* kbase = kc + (size_t)h * max_ctx * HD;
    const KVT* vbase = vc + (size_t)h * max_ctx * HD;

    auto issue = [&](int b) {
        const int s0 = b * PA_BK, cnt = min(PA_BK, kend - s0);
        const uint32_t bytes = (uint32_t)(cnt * RB);
        uint8_t* dst = smem + (b % PA_NS) * S::stage_bytes;
        mbar_expect_tx(&bars[b % PA_NS], 2 * bytes);
        bulk_g2s(dst, kbase + (size_t)s0 * HD, bytes, &bars[b % PA_NS]);
        bulk_g2s(dst + PA_BK * RB, vbase + (size_t)s0 * HD, bytes, &bars[b % PA_NS]);
    };
    if (threadIdx.x == 0) {
        for (int s = 0; s < PA_NS; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        for (int b = 0; b < min(PA_NS, nblk); ++b) issue(b);
    }

    // q fragments (A operand, rows g / g+8, dims 16 kk + 2t (+1, +8, +9)), scaled by log2(e) so
    // that the softmax runs on exp2
    constexpr float LOG2E = 1.4426950408889634f;
    uint32_t qa[8][4];
    {
        const int ra = min(wr0 + g, n - 1), rb = min(wr0 + g + 8, n - 1);
        const float* qra = q + ((size_t)ra * NQ + qh) * HD;
        const float* qrb = q + ((size_t)rb * NQ + qh) * HD;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const int d0 = 16 * kk + 2 * t;
            const float2 a0 = *reinterpret_cast<const float2*>(qra + d0);
            const float2 a1 = *reinterpret_cast<const float2*>(qrb + d0);
            const float2 a2 = *reinterpret_cast<const float2*>(qra + d0 + 8);
            const float2 a3 = *reinterpret_cast<const float2*>(qrb + d0 + 8);
            qa[kk][0] = pack2<KVT>(float_to_kv<KVT>(a0.x * LOG2E), float_to_kv<KVT>(a0.y * LOG2E));
            qa[kk][1] = pack2<KVT>(float_to_kv<KVT>(a1.x * LOG2E), float_to_kv<KVT>(a1.y * LOG2E));
            qa[kk][2] = pack2<KVT>(float_to_kv<KVT>(a2.x * LOG2E), float_to_kv<KVT>(a2.y * LOG2E));
            qa[kk][3] = pack2<KVT>(float_to_kv<KVT>(a3.x * LOG2E), float_to_kv<KVT>(a3.y * LOG2E));
        }
    }
    float o[16][4];
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[nt][e] = 0.f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
    const int pa_pos = pos0 + min(wr0 + g, n - 1), pb_pos = pos0 + min(wr0 + g + 8, n - 1);
    const int warp_last = pos0 + min(wr0 + 15, n - 1);  // last slot any row of this warp attends
    __syncthreads();

    bool ok = true;
    for (int b = 0; b < nblk; ++b) {
        const int st = b % PA_NS;
        const bool got = __all_sync(0xffffffffu, mbar_wait_bounded(&bars[st], (uint32_t)((b / PA_NS) & 1)));
        if (!got) {
            if (lane == 0) atomicOr(err, ERR_WAIT_PREFILL);
            ok = false;
            break;
        }
        const int s0 = b * PA_BK, cnt = min(PA_BK, kend - s0);
        if (s0 <= warp_last) {
            const uint32_t kst = smem_u32(smem + st * S::stage_bytes), vst = kst + PA_BK * RB;
            // ---- S = Q K^T over 64 slots: 8 n-tiles of 8 slots (log2 units) ----
            float s[8][4];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) s[nt][e] = 0.f;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
                for (int np = 0; np < 4; ++np) {  // 16 slots per ldmatrix.x4
                    const int row = min(16 * np + (lane & 7) + ((lane >> 4) << 3), cnt - 1);
                    const int chunk = 2 * kk + ((lane >> 3) & 1);
                    uint32_t bf[4];
                    ldsm_x4(bf, kst + row * RB + ((chunk ^ (row & 7)) << 4));
                    mma_kv<KVT>(s[2 * np], qa[kk], bf[0], bf[1]);
                    mma_kv<KVT>(s[2 * np + 1], qa[kk], bf[2], bf[3]);
                }
            }
            // ---- causal mask + online softmax (rows g: e 0,1; g+8: e 2,3) ----
            float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int slot = s0 + 8 * nt + 2 * t + (e & 1);
                    const bool valid = slot < kend && slot <= ((e < 2) ? pa_pos : pb_pos);
                    s[nt][e] = valid ? s[nt][e] : -INFINITY;
                }
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                mxa = fmaxf(mxa, fmaxf(s[nt][0], s[nt][1]));
                mxb = fmaxf(mxb, fmaxf(s[nt][2], s[nt][3]));
            }
            mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
            mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
            mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
            mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
            const float mna = fmaxf(m_a, mxa), mnb = fmaxf(m_b, mxb);
            const float ca = (mna == -INFINITY) ? 1.f : exp2f(m_a - mna);
            const float cb = (mnb == -INFINITY) ? 1.f : exp2f(m_b - mnb);
            m_a = mna;
            m_b = mnb;
            float suma = 0.f, sumb = 0.f;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                s[nt][0] = (s[nt][0] == -INFINITY) ? 0.f : exp2f(s[nt][0] - mna);
                s[nt][1] = (s[nt][1] == -INFINITY) ? 0.f : exp2f(s[nt][1] - mna);
                s[nt][2] = (s[nt][2] == -INFINITY) ? 0.f : exp2f(s[nt][2] - mnb);
                s[nt][3] = (s[nt][3] == -INFINITY) ? 0.f : exp2f(s[nt][3] - mnb);
                suma += s[nt][0] + s[nt][1];
                sumb += s[nt][2] + s[nt][3];
            }
            l_a = l_a * ca + suma;
            l_b = l_b * cb + sumb;
#pragma unroll
            for (int nt = 0; nt < 16; ++nt) {
                o[nt][0] *= ca;
                o[nt][1] *= ca;
                o[nt][2] *= cb;
                o[nt][3] *= cb;
            }
            // ---- O += P V: P from the score registers (A operand), V^T by ldmatrix.trans ----
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {  // 16 slots per step
                uint32_t pa[4];
                pa[0] = pack2<KVT>(float_to_kv<KVT>(s[2 * kk][0]), float_to_kv<KVT>(s[2 * kk][1]));
                pa[1] = pack2<KVT>(float_to_kv<KVT>(s[2 * kk][2]), float_to_kv<KVT>(s[2 * kk][3]));
                pa[2] = pack2<KVT>(float_to_kv<KVT>(s[2 * kk + 1][0]), float_to_kv<KVT>(s[2 * kk + 1][1]));
                pa[3] = pack2<KVT>(float_to_kv<KVT>(s[2 * kk + 1][2]), float_to_kv<KVT>(s[2 * kk + 1][3]));
                const int row = min(16 * kk + (lane & 7) + (((lane >> 3) & 1) << 3), cnt - 1);
#pragma unroll
                for (int dp = 0; dp < 8; ++dp) {  // 16 dims per ldmatrix.x4.trans
                    const int chunk = 2 * dp + (lane >> 4);
                    uint32_t vf[4];
                    ldsm_x4_trans(vf, vst + row * RB + ((chunk ^ (row & 7)) << 4));
                    mma_kv<KVT>(o[2 * dp], pa, vf[0], vf[1]);
                    mma_kv<KVT>(o[2 * dp + 1], pa, vf[2], vf[3]);
                }
            }
        }
        __syncthreads();  // every warp is done with this stage
        if (threadIdx.x == 0 && b + PA_NS < nblk) {
            fence_proxy_async_smem();
            issue(b + PA_NS);
        }
    }
    if (!ok) {
        // drain copies that may still be landing before the CTA exits
        if (threadIdx.x == 0)
            for (int b = 0; b < nblk && b < PA_NS; ++b) mbar_wait_bounded(&bars[b], 0);
        return;
    }
    // ---- normalise and store fp16 rows (the o-proj GEMM input) ----
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
    const float ia = 1.0f / l_a, ib = 1.0f / l_b;
    const int ra = wr0 + g, rb = wr0 + g + 8;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
        const int d = 8 * nt + 2 * t;
        if (ra < n)
            *reinterpret_cast<__half2*>(out + (size_t)ra * H + qh * HD + d) = __floats2half2_rn(o[nt][0] * ia, o[nt][1] * ia);
        if (rb < n)
            *reinterpret_cast<__half2*>(out + (size_t)rb * H + qh * HD + d) = __floats2half2_rn(o[nt][2] * ib, o[nt][3] * ib);
    }
}

}  // namespace icua
