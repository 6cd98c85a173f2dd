// Row-parallel prefill kernels around the tensor-core GEMM: prompt embedding, RMSNorm into fp16
// GEMM inputs, and per-head QK norm + M-RoPE + KV append.  The causal attention runs on tcgen05
// (prefill_tc.cuh).
//
// Reference counterparts: k_embed_prompt (Shaders.swift:676-692), k_rmsnorm_rows_h (838-864) and
// k_qk_norm_rope (871-923).
// Each kernel starts with griddepcontrol.wait, so it may be launched as a programmatic dependent
// of the kernel before it (its launch then overlaps that kernel's tail).
#pragma once
#include "attn_decode.cuh"
#include "common.cuh"
#include "gemm_tc.cuh"
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
// hilo: the output rows are fp16 hi / lo pairs (store_norm_row).
template <bool HILO = false>
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
    store_norm_row(out, i, tid, a, b, r, wa, wb, HILO);
}

// Per prompt row: RMSNorm(128) of the 16 q and 8 k heads, rotate-half RoPE from the cache slot's
// (cos, sin) row, q scaled by 1/sqrt(128) and rounded to the cache type into q_out [n][16][128]
// (the A operand of the tensor-core attention), k and v rounded to the cache type and stored at
// slot pos0 + i in the swizzled row order.  One CTA (8 warps) per row, one warp per head vector
// (32 vectors: 16 q, 8 k, 8 v).
template <typename KVT>
__global__ void __launch_bounds__(256) qk_rope_kv_kernel(const float* qkv, int n, const float* q_norm,
                                                         const float* k_norm, const float2* rope, int pos0, KVT* kc,
                                                         KVT* vc, int max_ctx, KVT* q_out) {
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
                KVT* qd = q_out + ((size_t)i * NQ + vi) * HD + 4 * lane;
#pragma unroll
                for (int e = 0; e < 4; ++e) qd[e] = float_to_kv<KVT>(y[e] * sc);
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

}  // namespace icua
