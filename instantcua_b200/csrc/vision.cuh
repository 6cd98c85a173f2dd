// Vision encoder row kernels around the tensor-core GEMM (fp16 weights): patchify, position
// resampling, LayerNorm into fp16 GEMM inputs, and the split of q / k with 2-D RoPE into
// head-major fp16.
//
// Replaces the reference's k_vit_patchify_rgb (Shaders.swift:82-110), k_vit_ln1024 / k_vit_ln4096
// (112-200) and the epilogue of k_vit_qkv (202-290: bias, 2-D RoPE, head-major fp16 q / k / v);
// the GEMMs themselves (patch embedding, QKV, projection, MLP, mergers; k_vit_gemm_T 396-454) run
// on tc_gemm_kernel with fp16 weights and the store / residual / GELU epilogues, the attention
// (k_vit_attn 292-395) on vit_attn_tc_kernel (attn_tc.cuh).
//
// Design (B200): one CTA per row for the row kernels.  Patches are kept in the 2x2 merge-block
// order throughout, so the mergers' [n / 4, 4096] inputs are views of the [n, 1024] rows.
#pragma once
#include "common.cuh"

namespace icua {

constexpr int VIT_HIDDEN = 1024;
constexpr int VIT_FF = 4096;
constexpr int VIT_HEADS = 16;
constexpr int VIT_HD = 64;
constexpr int VIT_QKV = 3072;
constexpr int VIT_PATCH = 16;
constexpr int VIT_PATCH_DIM = 768;  // 3 x 16 x 16 (the two temporal frames folded into the weights)
constexpr int VIT_POS_SIDE = 48;
constexpr int VIT_LAYERS = 24;
constexpr int VIT_MERGED = 4096;    // 2 x 2 patches of 1024

// Patch p of the merge-block order -> (row, col) in the patch grid (gw columns).
__device__ __forceinline__ void vit_patch_rc(int p, int gw, int& r, int& c) {
    const int blk = p >> 2, in = p & 3, bw = gw >> 1;
    r = (blk / bw) * 2 + (in >> 1);
    c = (blk % bw) * 2 + (in & 1);
}

// RGB8 [gh * 16][gw * 16][3] -> fp16 patches [n][768], element (c, dy, dx) = 2 v / 255 - 1
// (qwen3vl_ref.py:25-38).  One CTA per patch.
__global__ void __launch_bounds__(256) vit_patchify_kernel(const uint8_t* rgb, int gh, int gw, __half* patches) {
    const int p = blockIdx.x;
    int r, c;
    vit_patch_rc(p, gw, r, c);
    const int img_w = gw * VIT_PATCH;
    for (int i = threadIdx.x; i < VIT_PATCH_DIM; i += blockDim.x) {
        const int ch = i >> 8, dy = (i >> 4) & 15, dx = i & 15;
        const int y = r * VIT_PATCH + dy, x = c * VIT_PATCH + dx;
        const float v = (float)rgb[((size_t)y * img_w + x) * 3 + ch];
        patches[(size_t)p * VIT_PATCH_DIM + i] = __float2half_rn(v * (2.0f / 255.0f) - 1.0f);
    }
}

// x[p] = bilinear (align_corners) resampling of the 48 x 48 position table at patch p's grid
// position (qwen3vl_ref.py:41-68); the patch-embedding GEMM then adds W patch + bias.  One CTA
// per patch.
__global__ void __launch_bounds__(256) vit_pos_init_kernel(const float* table, int gh, int gw, float* x) {
    const int p = blockIdx.x;
    int r, c;
    vit_patch_rc(p, gw, r, c);
    const float sh = (float)r * (float)(VIT_POS_SIDE - 1) / (float)max(gh - 1, 1);
    const float sw = (float)c * (float)(VIT_POS_SIDE - 1) / (float)max(gw - 1, 1);
    const int h0 = (int)floorf(sh), w0 = (int)floorf(sw);
    const int h1 = min(h0 + 1, VIT_POS_SIDE - 1), w1 = min(w0 + 1, VIT_POS_SIDE - 1);
    const float dh = sh - (float)h0, dw = sw - (float)w0;
    const float* t00 = table + ((size_t)h0 * VIT_POS_SIDE + w0) * VIT_HIDDEN;
    const float* t01 = table + ((size_t)h0 * VIT_POS_SIDE + w1) * VIT_HIDDEN;
    const float* t10 = table + ((size_t)h1 * VIT_POS_SIDE + w0) * VIT_HIDDEN;
    const float* t11 = table + ((size_t)h1 * VIT_POS_SIDE + w1) * VIT_HIDDEN;
    for (int k = threadIdx.x; k < VIT_HIDDEN; k += blockDim.x)
        x[(size_t)p * VIT_HIDDEN + k] =
            (1.0f - dh) * ((1.0f - dw) * t00[k] + dw * t01[k]) + dh * ((1.0f - dw) * t10[k] + dw * t11[k]);
}

// out[i] = fp16(LayerNorm(x[i]) * w + b) over rows of `width` (1024 or 4096) floats, eps 1e-6
// (qwen3vl_ref.py:142-146): mean, then the variance of the centred values.  One CTA of 256
// threads per row, the row held in registers.
__global__ void __launch_bounds__(256) vit_layernorm_kernel(const float* x, const float* w, const float* b, int width,
                                                            __half* out) {
    __shared__ float red[8];
    const int i = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)i * width);
    const int nv = width / 1024;  // float4 per thread: 1 or 4
    float4 v[4];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        if (j < nv) {
            v[j] = xr[tid + 256 * j];
            s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
        }
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot += red[k];
    const float mean = tot / (float)width;
    __syncthreads();
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        if (j < nv) {
            v[j].x -= mean; v[j].y -= mean; v[j].z -= mean; v[j].w -= mean;
            q += (v[j].x * v[j].x + v[j].y * v[j].y) + (v[j].z * v[j].z + v[j].w * v[j].w);
        }
    q = warp_sum(q);
    if (lane == 0) red[warp] = q;
    __syncthreads();
    tot = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot += red[k];
    const float inv = 1.0f / sqrtf(tot / (float)width + 1e-6f);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    const float4* b4 = reinterpret_cast<const float4*>(b);
    __half2* o2 = reinterpret_cast<__half2*>(out + (size_t)i * width);
#pragma unroll
    for (int j = 0; j < 4; ++j)
        if (j < nv) {
            const int e = tid + 256 * j;
            const float4 ww = w4[e], bb = b4[e];
            o2[2 * e] = __floats2half2_rn(v[j].x * inv * ww.x + bb.x, v[j].y * inv * ww.y + bb.y);
            o2[2 * e + 1] = __floats2half2_rn(v[j].z * inv * ww.z + bb.z, v[j].w * inv * ww.w + bb.w);
        }
}

// 2-D RoPE table of an image: rope[p][d] = (cos, sin) of angle d of patch p for the rotate-half
// pairs (d, d + 32), d < 32: frequencies 0..15 (1 / 10000^(2f/32)) times the patch row for
// d < 16, times the column for d >= 16 (qwen3vl_ref.py:71-84).  Computed once per image.
__global__ void __launch_bounds__(256) vit_rope_table_kernel(int n, int gw, float2* rope) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * 32) return;
    const int p = i >> 5, d = i & 31, f = d & 15;
    int r, c;
    vit_patch_rc(p, gw, r, c);
    const float inv = powf(10000.0f, -(float)(2 * f) / 32.0f);
    float sn, cs;
    sincosf((float)(d < 16 ? r : c) * inv, &sn, &cs);
    rope[i] = make_float2(cs, sn);
}

// qkv [n][3072] fp32 (bias added by the GEMM) -> head-major fp16 q, k [16][n][64] rotated by the
// 2-D RoPE table (qwen3vl_ref.py:184-186); v goes to V^T (vit_vt_kernel).  One CTA per patch,
// thread (head, pair).
__global__ void __launch_bounds__(256) vit_qkv_rope_kernel(const float* qkv, const float2* rope, int n, __half* q,
                                                           __half* k) {
    const int p = blockIdx.x;
    const float* row = qkv + (size_t)p * VIT_QKV;
    for (int i = threadIdx.x; i < 2 * VIT_HEADS * 32; i += blockDim.x) {
        const int which = i >> 9, h = (i >> 5) & 15, d = i & 31;  // which: 0 q, 1 k
        const float2 csn = rope[p * 32 + d];
        const float cs = csn.x, sn = csn.y;
        const float* src = row + which * VIT_HIDDEN + h * VIT_HD;
        const float a = src[d], b = src[d + 32];
        __half* dst = (which ? k : q) + ((size_t)h * n + p) * VIT_HD;
        dst[d] = __float2half_rn(a * cs - b * sn);
        dst[d + 32] = __float2half_rn(b * cs + a * sn);
    }
}

}  // namespace icua
