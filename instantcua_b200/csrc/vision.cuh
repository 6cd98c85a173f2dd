// Vision encoder row kernels around the tensor-core GEMM (fp16 weights): patchify, position
// resampling, LayerNorm into fp16 GEMM inputs, QKV bias-free split with 2-D RoPE into head-major
// fp16, and bidirectional multi-head attention.
//
// Replaces the reference's k_vit_patchify_rgb (Shaders.swift:82-110), k_vit_ln1024 / k_vit_ln4096
// (112-200), the epilogue of k_vit_qkv (202-290: bias, 2-D RoPE, head-major fp16 q / k / v) and
// k_vit_attn (292-395, scores and probabilities in threadgroup memory); the GEMMs themselves
// (patch embedding, QKV, projection, MLP, mergers; k_vit_gemm_T 396-454) run on tc_gemm_kernel
// with fp16 weights and the store / residual / GELU epilogues.
//
// Design (B200): one CTA per row for the row kernels; attention is a flash kernel on the tensor
// cores (mma.sync m16n8k16, fp16 operands, fp32 accumulation, online softmax in registers, K / V
// tiles double-buffered through cp.async), 64 queries x one head per CTA, the score matrix never
// leaves registers.  Patches are kept in the 2x2 merge-block order throughout, so the mergers'
// [n / 4, 4096] inputs are views of the [n, 1024] rows.
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

// qkv [n][3072] fp32 (bias added by the GEMM) -> head-major fp16 q, k, v [16][n][64], q and k
// rotated by the 2-D RoPE table (qwen3vl_ref.py:184-186).  One CTA per patch; thread
// (head, pair) for q and k, plain copies for v.
__global__ void __launch_bounds__(256) vit_qkv_rope_kernel(const float* qkv, const float2* rope, int n, __half* q,
                                                           __half* k, __half* v) {
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
    for (int i = threadIdx.x; i < VIT_HIDDEN; i += blockDim.x) {
        const int h = i >> 6, d = i & 63;
        v[((size_t)h * n + p) * VIT_HD + d] = __float2half_rn(row[2 * VIT_HIDDEN + i]);
    }
}

// ---- bidirectional attention ------------------------------------------------------------------
constexpr int VA_BQ = 64;       // queries per CTA (4 warps x 16; 128 measured 6% slower)
constexpr int VA_BK = 64;       // keys per block
constexpr int VA_THREADS = 128;

__device__ __forceinline__ void va_ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void va_ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void va_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void va_cp16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
// 16-byte chunk j of a 128-byte tile row r, XOR-swizzled so ldmatrix rows hit distinct banks
__device__ __forceinline__ int va_swz(int r, int j) { return r * 128 + ((j ^ (r & 7)) << 4); }

// Scaled dot-product attention over all n patches (no mask), softmax in fp32, probabilities
// rounded to fp16 for the PV product (as the reference's fp16 vprobs).  Grid (ceil(n / 64), 16).
__global__ void __launch_bounds__(VA_THREADS) vit_attn_kernel(const __half* q, const __half* k, const __half* v, int n,
                                                              __half* out) {
    __shared__ __align__(128) uint8_t sm[VA_BQ * 128 + 2 * 2 * VA_BK * 128];  // Q, then K / V double buffers
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int h = blockIdx.y, q0 = blockIdx.x * VA_BQ;
    const __half* qh = q + (size_t)h * n * VIT_HD;
    const __half* kh = k + (size_t)h * n * VIT_HD;
    const __half* vh = v + (size_t)h * n * VIT_HD;
    const uint32_t sq = smem_u32(sm), skv = sq + VA_BQ * 128;
    auto kbuf = [&](int b) { return skv + b * 2 * VA_BK * 128; };
    auto vbuf = [&](int b) { return skv + b * 2 * VA_BK * 128 + VA_BK * 128; };
    // Q tile (rows past n read as zeros)
    for (int i = threadIdx.x; i < VA_BQ * 8; i += VA_THREADS) {
        const int r = i >> 3, j = i & 7;
        const bool ok = q0 + r < n;
        va_cp16(sq + va_swz(r, j), qh + (size_t)(ok ? q0 + r : 0) * VIT_HD + j * 8, ok);
    }
    auto load_kv = [&](int blk, int b) {
        const int k0 = blk * VA_BK;
        for (int i = threadIdx.x; i < VA_BK * 8; i += VA_THREADS) {
            const int r = i >> 3, j = i & 7;
            const bool ok = k0 + r < n;
            const size_t off = (size_t)(ok ? k0 + r : 0) * VIT_HD + j * 8;
            va_cp16(kbuf(b) + va_swz(r, j), kh + off, ok);
            va_cp16(vbuf(b) + va_swz(r, j), vh + off, ok);
        }
    };
    const int nblk = (n + VA_BK - 1) / VA_BK;
    load_kv(0, 0);
    asm volatile("cp.async.commit_group;" ::: "memory");
    // Q fragments of this warp's 16 rows: 4 k-steps of 16 dims
    uint32_t qa[4][4];
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows g and g + 8
    const float sl2 = 0.125f * 1.4426950408889634f;             // 1/sqrt(64) * log2(e)
    for (int blk = 0; blk < nblk; ++blk) {
        const int b = blk & 1;
        if (blk + 1 < nblk) load_kv(blk + 1, b ^ 1);
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();
        if (blk == 0) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const int r = warp * 16 + (lane & 15), j = 2 * kk + (lane >> 4);
                va_ldsm_x4(qa[kk], sq + va_swz(r, j));
            }
        }
        // S = Q K^T for 64 keys: 8 n-tiles of 8 keys
        float s[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; nt += 2) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                // keys nt*8 .. nt*8+15 (two n-tiles), dims kk*16 .. +15
                uint32_t kb[4];
                const int r = nt * 8 + (lane & 7) + ((lane >> 4) << 3), j = 2 * kk + ((lane >> 3) & 1);
                va_ldsm_x4(kb, kbuf(b) + va_swz(r, j));
                va_mma(s[nt], qa[kk], kb[0], kb[1]);
                va_mma(s[nt + 1], qa[kk], kb[2], kb[3]);
            }
        }
        // mask keys past n, online softmax (base 2)
        const int k0 = blk * VA_BK;
        float bm0 = -INFINITY, bm1 = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = k0 + nt * 8 + 2 * t + (e & 1);
                s[nt][e] = key < n ? s[nt][e] * sl2 : -INFINITY;
            }
            bm0 = fmaxf(bm0, fmaxf(s[nt][0], s[nt][1]));
            bm1 = fmaxf(bm1, fmaxf(s[nt][2], s[nt][3]));
        }
        bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, 1));
        bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, 2));
        bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, 1));
        bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, 2));
        const float nm0 = fmaxf(m0, bm0), nm1 = fmaxf(m1, bm1);
        const float c0 = exp2f(m0 - nm0), c1 = exp2f(m1 - nm1);  // m = -inf at first: 0
        m0 = nm0;
        m1 = nm1;
        float rs0 = 0.f, rs1 = 0.f;
        uint32_t pa[4][4];  // P as the A operand: k-step kk covers keys kk*16 .. +15 (n-tiles 2kk, 2kk+1)
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const float p0 = exp2f(s[nt][0] - m0), p1 = exp2f(s[nt][1] - m0);
            const float p2 = exp2f(s[nt][2] - m1), p3 = exp2f(s[nt][3] - m1);
            const __half2 h01 = __floats2half2_rn(p0, p1), h23 = __floats2half2_rn(p2, p3);
            // the row sums use the fp16 probabilities that enter the PV product
            rs0 += __low2float(h01) + __high2float(h01);
            rs1 += __low2float(h23) + __high2float(h23);
            const int kk = nt >> 1, hi = nt & 1;
            pa[kk][hi * 2 + 0] = *reinterpret_cast<const uint32_t*>(&h01);
            pa[kk][hi * 2 + 1] = *reinterpret_cast<const uint32_t*>(&h23);
        }
        l0 = l0 * c0 + rs0;
        l1 = l1 * c1 + rs1;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            o[j][0] *= c0;
            o[j][1] *= c0;
            o[j][2] *= c1;
            o[j][3] *= c1;
        }
        // O += P V: 8 n-tiles of 8 dims, 4 k-steps of 16 keys; V^T fragments by ldmatrix.trans
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                uint32_t vb[4];
                const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), c = j + (lane >> 4);
                va_ldsm_x4_t(vb, vbuf(b) + va_swz(r, c));
                va_mma(o[j], pa[kk], vb[0], vb[1]);
                va_mma(o[j + 1], pa[kk], vb[2], vb[3]);
            }
        }
        __syncthreads();  // the buffer is refilled two blocks later
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    // row sums over the quad, normalise, store fp16 [n][1024] at column h * 64
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float i0 = 1.0f / l0, i1 = 1.0f / l1;
    const int ra = q0 + warp * 16 + g, rb = ra + 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int d = j * 8 + 2 * t;
        if (ra < n)
            *reinterpret_cast<__half2*>(out + (size_t)ra * VIT_HIDDEN + h * VIT_HD + d) =
                __floats2half2_rn(o[j][0] * i0, o[j][1] * i0);
        if (rb < n)
            *reinterpret_cast<__half2*>(out + (size_t)rb * VIT_HIDDEN + h * VIT_HD + d) =
                __floats2half2_rn(o[j][2] * i1, o[j][3] * i1);
    }
}

}  // namespace icua
