// Batch-1 dequant-GEMV for the decode step (q4s / q8 weights, fp32 activations).
//
// Replaces the reference's dot64_row / reduce8 / chunk64_norm GEMV family and the kernels built
// on it: k_attn_in's QKV projection (Shaders.swift:714-834), k_o_proj (1293-1337), k_mlp_in
// (1342-1393), k_mlp_out (1397-1448) and k_lm_head (1452-1495).
//
// Design (B200):
// * Weights live in a tile layout (16 rows x 64 columns per "unit") whose bytes are exactly the
//   A-operand registers of four mma.sync.m16n8k16 per warp.  int4 / int8 codes are unpacked by
//   masking into fp16 *subnormal* integers (u * 2^-24), so the tensor core multiplies exact
//   integers; the code offset enters through the MMA accumulator start value and the row scale
//   and the power of two are applied in fp32.
// * Activations are fp32 split into fp16 hi + lo parts that occupy two B columns, so the dot
//   product keeps ~22 bits of the activation and accumulates in fp32.
// * A CTA owns whole 16-row tiles; its NW warps split K into NW slices.  Units are stored
//   slice-major ([slice][tile][unit]), so one warp's share of all the CTA's tiles is one
//   contiguous 1-D bulk copy (cp.async.bulk + mbarrier) requested before griddepcontrol.wait:
//   the weight stream overlaps the previous kernel.  The activation fragments and code-offset
//   terms of the warp's slice are loaded into registers once and reused for every tile.
// * Decode projections (<= 8 tiles per CTA): per-tile sums stay in registers, the NW slices meet
//   in shared memory after one __syncthreads and the epilogue runs on all threads.  Long
//   matrices (the lm_head) stream through a per-warp ring and the last warp to finish a tile
//   (shared-memory counter) applies its epilogue.  No global atomics, fences or spin waits.
// * Everything that does not depend on the previous kernel (weights, norm weights, the old
//   residual rows) is requested before griddepcontrol.wait; after it, the input loads are issued
//   before anything that could serialise them.
#pragma once
#include "common.cuh"
#include "layout.h"

namespace icua {

using icua_layout::fmt_slices;
using icua_layout::unit_offset;

enum InMode : int { IN_F32 = 0, IN_BF16 = 1, IN_EMBED = 2, IN_ATTN = 3 };
enum Epi : int { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_LOGITS = 3 };

constexpr int ATT_PART = 4 + 2 * HD;  // per (kv head, part): m[2], l[2], o[2][128] (unnormalised)
constexpr int ATT_MAX_PARTS = 8;
constexpr int SMALL_MAX_TILES = 8;    // tiles per CTA of the register-accumulating path

// Poll limit of a GEMV's wait for its RMSNorm weight copy (icua_set_wait_limit).  0 makes that wait
// give up at once, which exercises the timeout report path (ERR_WAIT_GEMV -> ICUA_ERR_TIMEOUT)
// without leaving a copy in flight: the kernel then waits for the copy with the default bound.
__constant__ uint32_t c_norm_wait_polls = 1u << 22;

struct GemvParams {
    const uint8_t* w;        // tile-packed units, slice-major
    int n_rows, k, upt;      // upt = k / 64 units per tile
    int n_tiles;
    int n_slots, chunk;      // streaming path: per-warp ring of n_slots slots of `chunk` tiles
    // input vector
    int in_mode;
    const void* x;           // IN_F32 / IN_BF16 input [k]
    const float* norm_w;     // RMSNorm weight [k] or nullptr
    const uint8_t* embed;    // IN_EMBED: q8 packed embedding [vocab, 2048]
    int embed_tiles;         // IN_EMBED: vocab / 16
    int embed_fmt;           // IN_EMBED: FMT_Q8 or FMT_Q4A
    const int* prompt;       // IN_EMBED: prompt tokens of the session
    const float* pooler;     // IN_EMBED: visual rows [n_vis, 2048] or nullptr
    const float* att_part;   // IN_ATTN: [NKV][att_parts][ATT_PART]
    int att_parts;
    float* x_resid;          // residual stream; written by CTA 0 in IN_EMBED, updated by EPI_RESID
    // o-projection partial products [NKV][2048] of an attention kernel with the o-proj folded in, or
    // nullptr, added in head order: in_add to the IN_F32 input (k = 2048), resid_add to the
    // residual rows EPI_RESID updates
    const float* in_add;
    const float* resid_add;
    // epilogue
    float* out;              // EPI_STORE: y [n_rows]; EPI_SWIGLU: h [n_rows / 2]
    const float* deepstack;  // EPI_RESID: [n_vis, 2048] for this layer, or nullptr
    float* logits;           // EPI_LOGITS: [vocab]
    float* step_logits;      // EPI_LOGITS: optional per-step capture [steps][vocab]
    float* cta_best_v;       // EPI_LOGITS: per-CTA argmax partials [gridDim.x]
    int* cta_best_i;
    DevState* st;            // nullptr for standalone GEMV
    L2Plan l2;               // data of later kernels to prefetch into L2
};

__host__ __device__ inline int gemv_tiles_per_cta(int n_tiles, int grid) { return (n_tiles + grid - 1) / grid; }

struct GemvSmem {
    int k, nw, n_slots, chunk, ub, ku, tiles_per_cta, has_norm;
    int ntok = 1;  // input vectors held (2 in the kernels of the grammar-commit 2-token pass)
    __host__ __device__ int xfrag_tok() const { return (k / 16) * 4 * 2 * 8; }  // bytes per input vector
    __host__ __device__ int xfrag_bytes() const { return ntok * xfrag_tok(); }
    __host__ __device__ int xsum_off() const { return xfrag_bytes(); }                       // float[ntok][k / 32]
    __host__ __device__ int red_off() const { return xsum_off() + ntok * (k / 32) * 4; }     // float[64]
    __host__ __device__ int normw_off() const { return red_off() + 64 * 4; }                 // float[k] if has_norm
    __host__ __device__ int part_off() const { return normw_off() + (has_norm ? k * 4 : 0); }  // float[ntok][tpc][nw][16]
    __host__ __device__ int part_tok() const { return tiles_per_cta * nw * 16; }             // floats per vector
    __host__ __device__ int cnt_off() const { return part_off() + ntok * part_tok() * 4; }
    __host__ __device__ int bars_off() const { return (cnt_off() + tiles_per_cta * 4 + 15) & ~15; }  // + norm bar
    __host__ __device__ int ring_off() const { return ((bars_off() + (nw * n_slots + 1) * 8) + 127) & ~127; }
    __host__ __device__ int slot_bytes() const { return chunk * ku * ub; }
    __host__ __device__ int ring_warp_bytes() const { return n_slots * slot_bytes(); }
    __host__ __device__ int total() const { return ring_off() + nw * ring_warp_bytes(); }
};

// fp32 value of element (row, k) of a q8 packed [n_rows, K] matrix: float(scale) * (u - 128).
__device__ __forceinline__ float q8_tile_value(const uint8_t* tiles, int n_tiles, int K, int row, int k) {
    const uint8_t* ub = tiles + unit_offset(FMT_Q8, n_tiles, K / UNIT_K, row >> 4, k >> 6);
    const int rt = row & 15, gq = rt & 7, up = rt >> 3;
    const int kin = k & 63, step = kin >> 4, kk = kin & 15;
    const int t = (kk & 7) >> 1, odd = kk & 1, hi8 = kk >> 3;
    const uint8_t* wp = ub + (step >> 1) * 512 + (gq * 4 + t) * 16 + ((step & 1) * 2 + hi8) * 4;
    const int u = wp[odd * 2 + up];
    const __half2 s2 = *reinterpret_cast<const __half2*>(ub + 1024 + gq * 8 + (kin >> 5) * 4);
    const float s = up ? __high2float(s2) : __low2float(s2);
    return s * (float)(u - 128);
}

// fp32 value of element (row, k) of a q4s packed matrix: float(scale) * (u - 8).
__device__ __forceinline__ float q4s_tile_value(const uint8_t* tiles, int n_tiles, int K, int row, int k) {
    const uint8_t* ub = tiles + unit_offset(FMT_Q4S, n_tiles, K / UNIT_K, row >> 4, k >> 6);
    const int rt = row & 15, gq = rt & 7, up = rt >> 3;
    const int kin = k & 63, step = kin >> 4, kk = kin & 15;
    const int t = (kk & 7) >> 1, odd = kk & 1, hi8 = kk >> 3;
    const uint32_t w = *reinterpret_cast<const uint32_t*>(ub + (gq * 4 + t) * 16 + step * 4);
    const int u = (w >> (odd * 16 + hi8 * 8 + up * 4)) & 0xF;
    const __half2 s2 = *reinterpret_cast<const __half2*>(ub + 512 + gq * 8 + (kin >> 5) * 4);
    const float s = up ? __high2float(s2) : __low2float(s2);
    return s * (float)(u - 8);
}

// fp32 value of element (row, k) of a q4a (reference affine q4) packed matrix: scale * u + bias
// (Shaders.swift:471-476).
__device__ __forceinline__ float q4a_tile_value(const uint8_t* tiles, int n_tiles, int K, int row, int k) {
    const uint8_t* ub = tiles + unit_offset(FMT_Q4A, n_tiles, K / UNIT_K, row >> 4, k >> 6);
    const int rt = row & 15, gq = rt & 7, up = rt >> 3;
    const int kin = k & 63, step = kin >> 4, kk = kin & 15;
    const int t = (kk & 7) >> 1, odd = kk & 1, hi8 = kk >> 3;
    const uint32_t w = *reinterpret_cast<const uint32_t*>(ub + (gq * 4 + t) * 16 + step * 4);
    const int u = (w >> (odd * 16 + hi8 * 8 + up * 4)) & 0xF;
    const float2 sb = __half22float2(*reinterpret_cast<const __half2*>(ub + 512 + gq * 8 + up * 4));
    return fmaf(sb.x, (float)u, sb.y);
}

// Embedding row element for the engine's embedding format (q8; q4a for reference q4 files; the
// row-major fp16 matrix of reference f16 files).
__device__ __forceinline__ float embed_value(int fmt, const uint8_t* tiles, int n_tiles, int row, int k) {
    if (fmt == FMT_F16) return __half2float(reinterpret_cast<const __half*>(tiles)[(size_t)row * H + k]);
    return fmt == FMT_Q4A ? q4a_tile_value(tiles, n_tiles, H, row, k) : q8_tile_value(tiles, n_tiles, H, row, k);
}

// ---------------------------------------------------------------------------------------------
// Input vector: values held in registers, then hi/lo fp16 B fragments + per-32 group sums.

template <int KMAX, int NT>
struct InputRegs {
    static constexpr int PPT = (KMAX / 4 + NT - 1) / NT;  // (k16 step, t) pairs per thread
    float v[PPT][4];
};

// Issues the input loads (independent) into registers.  IN_ATTN folds the attention parts of
// the element's head (max, sum, output) with their softmax weights; IN_EMBED first reads the
// prompt cursor (one extra round trip, layer 0 only).  `row` selects the input vector of a
// 2-token pass (x row, attention parts or embedded token of that row).
template <int KMAX, int NT, int IN>
__device__ __forceinline__ void load_input(InputRegs<KMAX, NT>& r, const GemvParams& p, int row = 0) {
    const int npairs = p.k / 4;
    const float* vis_row = nullptr;
    int tok = 0;
    if (IN == IN_EMBED) {
        const DevState* st = p.st;
        const int idx = st->prompt_idx;
        if (row == 1) {
            tok = st->cur_token2;
        } else if (idx < st->prompt_len) {
            tok = p.prompt[idx];
            const int v = idx - st->vis_offset;
            if (tok == IMAGE_PAD_ID && st->vis_offset >= 0 && p.pooler != nullptr && v >= 0 && v < st->n_vis)
                vis_row = p.pooler + (long long)v * H;
        } else {
            tok = st->cur_token;
        }
    }
#pragma unroll
    for (int j = 0; j < InputRegs<KMAX, NT>::PPT; ++j) {
        const int q = threadIdx.x + j * NT;
        if (q >= npairs) continue;
        const int s = q >> 2, t = q & 3, k0 = s * 16 + 2 * t;
        if (IN == IN_F32) {
            const float* x = reinterpret_cast<const float*>(p.x) + (long long)row * p.k;
            const float2 a = *reinterpret_cast<const float2*>(x + k0);
            const float2 b = *reinterpret_cast<const float2*>(x + k0 + 8);
            r.v[j][0] = a.x;
            r.v[j][1] = a.y;
            r.v[j][2] = b.x;
            r.v[j][3] = b.y;
            if (p.in_add != nullptr) {  // x + o_part[0] + ... + o_part[7]: every load first, then the sums
                float2 pa[NKV], pb[NKV];
#pragma unroll
                for (int hq = 0; hq < NKV; ++hq) {
                    pa[hq] = *reinterpret_cast<const float2*>(p.in_add + hq * H + k0);
                    pb[hq] = *reinterpret_cast<const float2*>(p.in_add + hq * H + k0 + 8);
                }
#pragma unroll
                for (int hq = 0; hq < NKV; ++hq) {
                    r.v[j][0] += pa[hq].x;
                    r.v[j][1] += pa[hq].y;
                    r.v[j][2] += pb[hq].x;
                    r.v[j][3] += pb[hq].y;
                }
            }
        } else if (IN == IN_BF16) {
            const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(p.x);
            r.v[j][0] = __bfloat162float(x[k0]);
            r.v[j][1] = __bfloat162float(x[k0 + 1]);
            r.v[j][2] = __bfloat162float(x[k0 + 8]);
            r.v[j][3] = __bfloat162float(x[k0 + 9]);
        } else if (IN == IN_ATTN) {
            // the four elements belong to one query head: fold its parts with a running max
            const int qh = k0 >> 7, h = qh >> 1, hh = qh & 1, P = p.att_parts;
            const float* b = p.att_part + ((long long)row * NKV + h) * P * ATT_PART;
            float M = -INFINITY, Ls = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
            for (int q2 = 0; q2 < P; ++q2) {
                const float* bq = b + q2 * ATT_PART;
                const float m = bq[hh], l = bq[2 + hh];
                const float* oq = bq + 4 + hh * HD + (k0 & 127);
                const float2 o01 = *reinterpret_cast<const float2*>(oq);
                const float2 o89 = *reinterpret_cast<const float2*>(oq + 8);
                if (m == -INFINITY) continue;
                const float Mn = fmaxf(M, m);
                const float c = (M == -INFINITY) ? 0.f : expf(M - Mn), f = expf(m - Mn);
                M = Mn;
                Ls = fmaf(Ls, c, l * f);
                acc[0] = fmaf(acc[0], c, o01.x * f);
                acc[1] = fmaf(acc[1], c, o01.y * f);
                acc[2] = fmaf(acc[2], c, o89.x * f);
                acc[3] = fmaf(acc[3], c, o89.y * f);
            }
            const float inv = 1.0f / Ls;
#pragma unroll
            for (int i = 0; i < 4; ++i) r.v[j][i] = acc[i] * inv;
        } else {
            const int kk[4] = {k0, k0 + 1, k0 + 8, k0 + 9};
#pragma unroll
            for (int i = 0; i < 4; ++i)
                r.v[j][i] = vis_row ? vis_row[kk[i]] : embed_value(p.embed_fmt, p.embed, p.embed_tiles, tok, kk[i]);
        }
    }
}

// Normalises (optionally) and writes the fragments; all threads; ends with __syncthreads.
// The RMSNorm weights were bulk-copied to shared memory before griddepcontrol.wait (nbar).
template <int KMAX, int NT>
__device__ __forceinline__ void store_input(const InputRegs<KMAX, NT>& r, const GemvParams& p, uint8_t* smem,
                                            const GemvSmem& L, uint64_t* nbar, int row = 0) {
    const int tid = threadIdx.x, npairs = p.k / 4;
    uint2* xfrag = reinterpret_cast<uint2*>(smem + row * L.xfrag_tok());
    float* xsum = reinterpret_cast<float*>(smem + L.xsum_off()) + row * (p.k / 32);
    float* red = reinterpret_cast<float*>(smem + L.red_off());
    const float* nws = reinterpret_cast<const float*>(smem + L.normw_off());
    float scale = 1.0f;
    if (p.norm_w != nullptr) {
        if (!mbar_wait_bounded(nbar, 0, c_norm_wait_polls)) {
            // gave up: flag it, then still wait (default bound) so that the copy has landed before
            // this CTA reads the weights or exits
            if (tid == 0 && p.st) atomicOr(&p.st->error, ERR_WAIT_GEMV);
            mbar_wait_bounded(nbar, 0);
        }
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < InputRegs<KMAX, NT>::PPT; ++j)
            if (tid + j * NT < npairs)
#pragma unroll
                for (int i = 0; i < 4; ++i) ss = fmaf(r.v[j][i], r.v[j][i], ss);
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w2 = 0; w2 < NT / 32; ++w2) tot += red[w2];
        scale = 1.0f / sqrtf(tot / (float)p.k + EPS);
    }
#pragma unroll
    for (int j = 0; j < InputRegs<KMAX, NT>::PPT; ++j) {
        const int q = tid + j * NT;
        if (q >= npairs) continue;
        const int s = q >> 2, t = q & 3, k0 = s * 16 + 2 * t;
        const int kk[4] = {k0, k0 + 1, k0 + 8, k0 + 9};
        __half hi[4], lo[4];
        float gsum = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float x = r.v[j][i];
            if (p.in_mode == IN_EMBED && blockIdx.x == 0) p.x_resid[row * H + kk[i]] = x;  // layer 0 keeps the embedded row
            if (p.norm_w != nullptr) x = x * scale * nws[kk[i]];
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
        // the 8 pairs of a 32-column group are 8 consecutive threads
        gsum += __shfl_xor_sync(0xffffffffu, gsum, 1);
        gsum += __shfl_xor_sync(0xffffffffu, gsum, 2);
        gsum += __shfl_xor_sync(0xffffffffu, gsum, 4);
        if ((q & 7) == 0) xsum[q >> 3] = gsum;
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------------------------
// Per-warp constants of one 16x64 unit column slice: the B fragments (x hi / lo) of its four k16
// steps and, per 32-column group, the MMA accumulator start values that subtract the code offset:
// D = 2^-24 * sum(u * x) + C with C = -off * X * 2^-24 (rows g) and 16x that for q4s rows g+8, so
// D = 2^-24 * sum(q * x) (rows g+8 of q4s: 2^-20 * sum(q * x)); the power of two is applied once
// per tile.
template <int FMT>
struct UnitConst {
    uint32_t b[4][2];
    float c0[2], c1[2];
    float xu24;  // q4a: sum of the unit's 64 inputs x 2^-24 (the bias term)
};

template <int FMT>
__device__ __forceinline__ void load_unit_const(UnitConst<FMT>& uc, int kk, const uint2* xfrag, const float* xsum,
                                                int lane) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int step = 0; step < 4; ++step) {
        const uint2 b = xfrag[((kk * 4 + step) * 4 + t) * 2 + (g & 1)];
        uc.b[step][0] = b.x;
        uc.b[step][1] = b.y;
    }
    // q4s / q8 store offset-binary codes: the offset enters through the accumulator start; q4a
    // codes are plain 0..15 and its bias multiplies the unit's input sum instead
    const float off = (FMT == FMT_Q4S) ? 8.0f : (FMT == FMT_Q8) ? 128.0f : 0.0f;
#pragma unroll
    for (int grp = 0; grp < 2; ++grp) {
        const float c = -off * xsum[kk * 2 + grp] * 5.9604644775390625e-08f;  // 2^-24
        uc.c0[grp] = c;
        uc.c1[grp] = (FMT != FMT_Q8) ? 16.0f * c : c;
    }
    uc.xu24 = (xsum[kk * 2] + xsum[kk * 2 + 1]) * 5.9604644775390625e-08f;
}

__device__ __forceinline__ void mma_16816_c(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, float c0,
                                            float c2) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%11};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c0), "f"(0.0f), "f"(c2));
}

// One 16x64 unit: adds s * D to rows g (acc0) and g+8 (acc1) in units of 2^-24 (rows g+8 of q4s:
// 2^-20); the caller applies the power of two when the tile is done.
template <int FMT>
__device__ __forceinline__ void gemv_unit(const uint8_t* ub, const UnitConst<FMT>& uc, int lane, float& acc0,
                                          float& acc1) {
    const int g = lane >> 2;
    const uint2 sc = *reinterpret_cast<const uint2*>(ub + unit_wbytes(FMT) + g * 8);
    uint32_t wq[8];
    if (FMT != FMT_Q8) {
        const uint4 w = *reinterpret_cast<const uint4*>(ub + lane * 16);
        wq[0] = w.x; wq[1] = w.y; wq[2] = w.z; wq[3] = w.w;
    } else {
        const uint4 w0 = *reinterpret_cast<const uint4*>(ub + lane * 16);
        const uint4 w1 = *reinterpret_cast<const uint4*>(ub + 512 + lane * 16);
        wq[0] = w0.x; wq[1] = w0.y; wq[2] = w0.z; wq[3] = w0.w;
        wq[4] = w1.x; wq[5] = w1.y; wq[6] = w1.z; wq[7] = w1.w;
    }
    float d[2][4];
#pragma unroll
    for (int step = 0; step < 4; ++step) {
        uint32_t a[4];
        if (FMT != FMT_Q8) {
            const uint32_t w = wq[step];
            a[0] = w & 0x000F000Fu;
            a[1] = w & 0x00F000F0u;
            a[2] = (w >> 8) & 0x000F000Fu;
            a[3] = (w >> 8) & 0x00F000F0u;
        } else {
            const uint32_t w0 = wq[step * 2], w1 = wq[step * 2 + 1];
            a[0] = w0 & 0x00FF00FFu;
            a[1] = (w0 >> 8) & 0x00FF00FFu;
            a[2] = w1 & 0x00FF00FFu;
            a[3] = (w1 >> 8) & 0x00FF00FFu;
        }
        const int grp = step >> 1;
        if ((step & 1) == 0)
            mma_16816_c(d[grp], a, uc.b[step][0], uc.b[step][1], uc.c0[grp], uc.c1[grp]);
        else
            mma_16816(d[grp], a, uc.b[step][0], uc.b[step][1]);
    }
    if (FMT == FMT_Q4A) {
        // one 64-column group: (scale, bias) of row g in sc.x, of row g+8 in sc.y
        const float2 sa = __half22float2(*reinterpret_cast<const __half2*>(&sc.x));
        const float2 sb = __half22float2(*reinterpret_cast<const __half2*>(&sc.y));
        acc0 = fmaf(sa.x, (d[0][0] + d[0][1]) + (d[1][0] + d[1][1]), acc0);
        acc0 = fmaf(sa.y, uc.xu24, acc0);
        acc1 = fmaf(sb.x, (d[0][2] + d[0][3]) + (d[1][2] + d[1][3]), acc1);
        acc1 = fmaf(sb.y, 16.0f * uc.xu24, acc1);  // rows g+8 accumulate in units of 2^-20
    } else {
#pragma unroll
        for (int grp = 0; grp < 2; ++grp) {
            const float2 s = __half22float2(*reinterpret_cast<const __half2*>(grp == 0 ? &sc.x : &sc.y));
            acc0 = fmaf(s.x, d[grp][0] + d[grp][1], acc0);
            acc1 = fmaf(s.y, d[grp][2] + d[grp][3], acc1);
        }
    }
}

// Epilogue of one output row.  xold: the row's residual value prefetched before the wait.
template <int EPI>
__device__ __forceinline__ void gemv_row_epilogue(const GemvParams& p, int r, float v, float xold, float ds,
                                                  int write_logits, int step, float& best_v, int& best_i) {
    if (EPI == EPI_STORE) {
        p.out[r] = v;
    } else if (EPI == EPI_RESID) {
        p.x_resid[r] = xold + (v + ds);
    } else if (EPI == EPI_LOGITS) {
        if (write_logits) p.logits[r] = v;
        if (p.step_logits != nullptr) p.step_logits[(long long)step * p.n_rows + r] = v;
        argmax_merge(best_v, best_i, v, r);
    }
}

// ---------------------------------------------------------------------------------------------
// DUAL: the kernel of the grammar-commit engines.  A pass may carry two tokens (DevState::n_tok);
// their input vectors take the B columns (tok0 hi, tok0 lo, tok1 hi, tok1 lo) x 2 of the same
// MMAs, so both rows come out of one read of the weights (the reference's dot64_row2 branches,
// Shaders.swift:529-595).  Lane (g, t) accumulates token t & 1.  The lm_head (EPI_LOGITS) reads
// only the pass's last row.  With one token the columns repeat it and the arithmetic is that of
// the single-token kernel.
//
// 64 registers: the q4 kernels (512 threads) keep two CTAs per SM, the running one and the next
// launch prefetching its weights, without spilling the hoisted unit constants.
template <int FMT, int EPI, int KMAX, bool STREAM, int IN, bool DUAL = false>
__global__ void __maxnreg__(64) gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int NW = fmt_slices(FMT), NT = NW * 32;
    constexpr int KU = KMAX / 64 / NW;  // units of a tile per warp at K = KMAX
    constexpr bool TWO = DUAL && EPI != EPI_LOGITS;  // two output rows per pass possible
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tpc = gemv_tiles_per_cta(p.n_tiles, gridDim.x);
    const int ku = p.upt / NW;
    const int chunk = STREAM ? p.chunk : tpc;
    const int NS = STREAM ? p.n_slots : 1;
    const GemvSmem L{p.k, NW, NS, chunk, unit_bytes(FMT), ku, tpc, p.norm_w != nullptr, TWO ? 2 : 1};
    const int UB = L.ub;
    const uint2* xfrag = reinterpret_cast<const uint2*>(smem);
    const float* xsum = reinterpret_cast<const float*>(smem + L.xsum_off());
    float* part = reinterpret_cast<float*>(smem + L.part_off());
    unsigned* cnt = reinterpret_cast<unsigned*>(smem + L.cnt_off());
    uint64_t* nbar = reinterpret_cast<uint64_t*>(smem + L.bars_off());
    uint64_t* bars = nbar + 1 + warp * NS;
    uint8_t* ring = smem + L.ring_off() + warp * L.ring_warp_bytes();

    const int t_begin = (int)((long long)blockIdx.x * p.n_tiles / gridDim.x);
    const int t_end = (int)((long long)(blockIdx.x + 1) * p.n_tiles / gridDim.x);
    const int nt = t_end - t_begin;
    const int n_chunks = (nt + chunk - 1) / chunk;
    const uint8_t* wslice = p.w + ((long long)warp * p.n_tiles + t_begin) * ku * UB;

    auto issue = [&](int c) {
        const int tiles = min(chunk, nt - c * chunk);
        const uint32_t bytes = (uint32_t)(tiles * ku * UB);
        uint64_t* bar = &bars[c % NS];
        mbar_expect_tx(bar, bytes);
        bulk_g2s(ring + (c % NS) * L.slot_bytes(), wslice + (long long)c * chunk * ku * UB, bytes, bar);
    };

    // ---- prologue: everything that does not depend on the previous kernel -------------------
    if (lane == 0) {
        for (int s = 0; s < NS; ++s) mbar_init(&bars[s], 1);
        if (warp == 0) mbar_init(nbar, 1);
        fence_mbar_init();
        if (warp == 0 && p.norm_w != nullptr) {
            mbar_expect_tx(nbar, (uint32_t)(p.k * 4));
            bulk_g2s(smem + L.normw_off(), p.norm_w, (uint32_t)(p.k * 4), nbar);
        }
        for (int c = 0; c < min(NS, n_chunks); ++c) issue(c);
    }
    if (threadIdx.x == 32) l2_prefetch_plan(p.l2, p.st ? *(volatile int*)&p.st->pos : 0);
    if (STREAM)
        for (int i = threadIdx.x; i < tpc; i += NT) cnt[i] = 0;
    InputRegs<KMAX, NT> in;
    // the residual rows this thread finalises (non-streaming path: thread i -> row i of the CTA)
    float xold = 0.f;
    if (!STREAM && EPI == EPI_RESID && (int)threadIdx.x < nt * 16) {
        const int r = t_begin * 16 + threadIdx.x;
        xold = p.x_resid[r];
        // the o-proj partial products were written two launches ago (the attention kernel), so they
        // are complete and visible once this kernel runs; summed in the order the IN_F32 load uses
        if (p.resid_add != nullptr) {
            float pr[NKV];
#pragma unroll
            for (int hq = 0; hq < NKV; ++hq) pr[hq] = p.resid_add[hq * H + r];
#pragma unroll
            for (int hq = 0; hq < NKV; ++hq) xold += pr[hq];
        }
    }
    __syncwarp();

    // the lm_head of a 2-token pass reads its last row; n_tok was set by the previous step's commit
    const int head_row = (DUAL && EPI == EPI_LOGITS && p.st != nullptr) ? *(volatile int*)&p.st->n_tok - 1 : 0;
    pdl_wait();
    load_input<KMAX, NT, IN>(in, p, head_row);  // issued before the stop-flag read so neither waits on the other
    const bool skip = (p.st != nullptr) && (*(volatile int*)&p.st->done != 0);
    const int ntok = (TWO && p.st != nullptr) ? *(volatile int*)&p.st->n_tok : 1;
    if (skip) {
        pdl_launch_dependents();
        if (lane == 0)
            for (int c = 0; c < min(NS, n_chunks); ++c) mbar_wait_bounded(&bars[c], 0);
        if (threadIdx.x == 0 && p.norm_w != nullptr) mbar_wait_bounded(nbar, 0);
        return;
    }
    int write_logits = (p.logits != nullptr && p.st == nullptr) ? 1 : 0, step = 0;
    float ds = 0.f;
    int ds_vi = -1;  // DeepStack row of this prompt row (visual rows of layers 0..2), or -1
    if (p.st != nullptr && (EPI == EPI_LOGITS || (EPI == EPI_RESID && p.deepstack != nullptr))) {
        const DevState* st = p.st;
        write_logits = st->write_logits;
        step = st->step;
        if (EPI == EPI_RESID) {
            const int vi = st->prompt_idx - st->vis_offset;
            if (st->prompt_idx < st->prompt_len && st->vis_offset >= 0 && vi >= 0 && vi < st->n_vis) ds_vi = vi;
            if (!STREAM && ds_vi >= 0 && (int)threadIdx.x < nt * 16)
                ds = p.deepstack[(long long)ds_vi * H + t_begin * 16 + threadIdx.x];
        }
    }
    store_input<KMAX, NT>(in, p, smem, L, nbar);  // ends with __syncthreads (also publishes cnt[] = 0)
    if (TWO && ntok == 2) {
        load_input<KMAX, NT, IN>(in, p, 1);
        store_input<KMAX, NT>(in, p, smem, L, nbar, 1);
    }
    // The next kernel's weight prefetch starts only now, so that it does not queue ahead of the
    // latency-bound input loads above.
    pdl_launch_dependents();

    const int g = lane >> 2, t = lane & 3;
    if (TWO && ntok == 2) {
        // B column g holds token (g >> 1) & 1; this lane's accumulator columns 2t, 2t+1 token t & 1
        xfrag += ((g >> 1) & 1) * (L.xfrag_tok() / 8);
        xsum += (t & 1) * (p.k / 32);
    }
    // the warp's K slice is the same for every tile: keep its constants in registers when small
    constexpr bool HOIST = KU <= 2;
    UnitConst<FMT> uc[HOIST ? KU : 1];
    if (HOIST) {
#pragma unroll
        for (int u = 0; u < (HOIST ? KU : 1); ++u)
            if (u < ku) load_unit_const<FMT>(uc[u], warp * ku + u, xfrag, xsum, lane);
    }
    const float f1 = (FMT != FMT_Q8) ? 1048576.0f : 16777216.0f;
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;

    auto tile_sum = [&](const uint8_t* base, float& acc0, float& acc1) {
        acc0 = acc1 = 0.f;
        if (HOIST) {
#pragma unroll
            for (int u = 0; u < (HOIST ? KU : 1); ++u)
                if (u < ku) gemv_unit<FMT>(base + u * UB, uc[u], lane, acc0, acc1);
        } else {
            for (int u = 0; u < ku; ++u) {
                load_unit_const<FMT>(uc[0], warp * ku + u, xfrag, xsum, lane);
                gemv_unit<FMT>(base + u * UB, uc[0], lane, acc0, acc1);
            }
        }
    };

    if (!STREAM) {
        // all tiles of the CTA arrive in one copy; sums stay in registers until the end
        if (n_chunks > 0 && !mbar_wait_bounded(&bars[0], 0)) {
            if (lane == 0 && p.st) atomicOr(&p.st->error, ERR_WAIT_GEMV);
        }
        // two tiles in flight: their unit MMA chains are independent
#pragma unroll 2
        for (int j = 0; j < nt; ++j) {
            float acc0, acc1;
            tile_sum(ring + j * ku * UB, acc0, acc1);
            if (t < (TWO ? ntok : 1)) {  // lane t = 0 (and t = 1 for the second token)
                float* pt = part + (TWO ? t * L.part_tok() : 0) + (j * NW + warp) * 16;
                pt[g] = acc0 * 16777216.0f;
                pt[g + 8] = acc1 * f1;
            }
        }
        __syncthreads();
        // thread i finalises row i of the CTA: fixed-order sum over the K slices
        const int i = threadIdx.x;
        for (int tk = 0; tk < (TWO ? ntok : 1); ++tk) {
            const float* pk = part + tk * L.part_tok();
            if (EPI == EPI_SWIGLU) {
                if (i < nt * 8) {
                    const int j = i >> 3, r8 = i & 7;
                    float gv = 0.f, uv = 0.f;
#pragma unroll
                    for (int w2 = 0; w2 < NW; ++w2) {
                        gv += pk[(j * NW + w2) * 16 + r8];
                        uv += pk[(j * NW + w2) * 16 + 8 + r8];
                    }
                    // tile rows 0..7 are gate units, rows 8..15 the matching up units
                    p.out[tk * (p.n_rows / 2) + (t_begin + j) * 8 + r8] = (gv / (1.0f + expf(-gv))) * uv;
                }
            } else if (i < nt * 16) {
                const int j = i >> 4, r = i & 15;
                float v = 0.f;
#pragma unroll
                for (int w2 = 0; w2 < NW; ++w2) v += pk[(j * NW + w2) * 16 + r];
                const int row = (t_begin + j) * 16 + r;
                if (TWO && tk == 1) {
                    if (EPI == EPI_STORE) p.out[p.n_rows + row] = v;
                    if (EPI == EPI_RESID) p.x_resid[p.n_rows + row] += v;
                } else {
                    gemv_row_epilogue<EPI>(p, row, v, xold, ds, write_logits, step, best_v, best_i);
                }
            }
        }
    } else {
        for (int c = 0; c < n_chunks; ++c) {
            const int slot = c % NS;
            if (!mbar_wait_bounded(&bars[slot], (uint32_t)((c / NS) & 1))) {
                if (lane == 0 && p.st) atomicOr(&p.st->error, ERR_WAIT_GEMV);
                break;
            }
            const int tiles = min(chunk, nt - c * chunk);
            for (int jj = 0; jj < tiles; ++jj) {
                const int j = c * chunk + jj;
                float acc0, acc1;
                tile_sum(ring + slot * L.slot_bytes() + jj * ku * UB, acc0, acc1);
                if (t < (TWO ? ntok : 1)) {  // lane t = 0 (and t = 1 for the second token)
                    float* pt = part + (TWO ? t * L.part_tok() : 0) + (j * NW + warp) * 16;
                    pt[g] = acc0 * 16777216.0f;
                    pt[g + 8] = acc1 * f1;
                }
                __threadfence_block();
                __syncwarp();
                unsigned prev = 0;
                if (lane == 0) prev = atomicAdd(&cnt[j], 1u);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (prev == NW - 1) {  // this warp completed the tile: reduce the K slices in a fixed order
                    __threadfence_block();
                    // lanes 0..15: rows of token 0; lanes 16..31: the same rows of token 1 (two-token kernels)
                    const int r = lane & 15, tk = TWO ? lane >> 4 : 0;
                    const float* pk = part + tk * L.part_tok();
                    float v = 0.f;
#pragma unroll
                    for (int w2 = 0; w2 < NW; ++w2) v += *(volatile float*)&pk[(j * NW + w2) * 16 + r];
                    if (EPI == EPI_SWIGLU) {
                        // tile rows 0..7 are gate units, rows 8..15 the matching up units
                        const float uv = __shfl_down_sync(0xffffffffu, v, 8);
                        if (r < 8 && (TWO ? tk < ntok : lane < 8))
                            p.out[tk * (p.n_rows / 2) + (t_begin + j) * 8 + r] = (v / (1.0f + expf(-v))) * uv;
                    } else if (TWO ? tk < ntok : lane < 16) {
                        const int row = (t_begin + j) * 16 + r + tk * p.n_rows;
                        float xo = 0.f, dsv = 0.f;
                        if (EPI == EPI_RESID) {
                            xo = p.x_resid[row];
                            if (ds_vi >= 0 && tk == 0) dsv = p.deepstack[(long long)ds_vi * H + row];
                        }
                        gemv_row_epilogue<EPI>(p, row, v, xo, dsv, write_logits, step, best_v, best_i);
                    }
                }
            }
            __syncwarp();
            if (lane == 0 && c + NS < n_chunks) {
                fence_proxy_async_smem();
                issue(c + NS);
            }
        }
    }

    if (EPI == EPI_LOGITS) {
        __shared__ float bv_s[32];
        __shared__ int bi_s[32];
        warp_argmax(best_v, best_i);
        if (lane == 0) {
            bv_s[warp] = best_v;
            bi_s[warp] = best_i;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float bv = bv_s[0];
            int bi = bi_s[0];
            for (int w2 = 1; w2 < NW; ++w2) argmax_merge(bv, bi, bv_s[w2], bi_s[w2]);
            p.cta_best_v[blockIdx.x] = bv;
            p.cta_best_i[blockIdx.x] = bi;
        }
    }
}

// Reduces per-CTA argmax partials to one token id (standalone greedy head): one CTA; -1 when no
// partial holds a finite logit.
__global__ void __launch_bounds__(256) argmax_parts_kernel(const float* best_v, const int* best_i, int n_parts,
                                                           int* token) {
    pdl_wait();
    pdl_launch_dependents();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n_parts; i += blockDim.x) argmax_merge(bv, bi, best_v[i], best_i[i]);
    warp_argmax(bv, bi);
    __shared__ float sv[8];
    __shared__ int si[8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w2 = 1; w2 < (int)(blockDim.x >> 5); ++w2) argmax_merge(sv[0], si[0], sv[w2], si[w2]);
        // no finite logit (NaN activations or norm weights) leaves no winner: report -1, never an
        // id that a caller could use as an index
        *token = si[0] == 0x7fffffff ? -1 : si[0];
    }
}

// Reduces the lm_head's per-CTA argmax partials to the next token and commits it (reference
// k_commit, Shaders.swift:1501-1571): one CTA.  When the call has the grammar-guided commit
// (st->grammar, engines built with it), ')' ends the call like EOS and a forced syntax token is
// appended after ',' and after a first-output action word; the next pass then carries both tokens
// (n_tok = 2) and advances the position by two.
__global__ void __launch_bounds__(256) commit_kernel(const float* cta_best_v, const int* cta_best_i, int n_parts,
                                                     int* out_tokens, DevState* st, GrammarRule rule, int vocab) {
    pdl_wait();
    pdl_launch_dependents();
    if (st->done) return;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n_parts; i += blockDim.x) argmax_merge(bv, bi, cta_best_v[i], cta_best_i[i]);
    warp_argmax(bv, bi);
    __shared__ float sv[8];
    __shared__ int si[8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w2 = 1; w2 < (int)(blockDim.x >> 5); ++w2) argmax_merge(sv[0], si[0], sv[w2], si[w2]);
        const int tok = si[0];
        if ((unsigned)tok >= (unsigned)vocab) {
            atomicOr(&st->error, ERR_BAD_TOKEN);
            st->done = 1;
            return;
        }
        const bool gram = rule.n_action >= 0 && st->grammar;
        st->pos += gram ? st->n_tok : 1;
        if (st->prompt_idx < st->prompt_len) st->prompt_idx += 1;
        out_tokens[st->step] = tok;
        st->step += 1;
        st->cur_token = tok;
        const bool stop = (st->stop_on_eos && (tok == st->eos0 || tok == st->eos1)) || st->step >= st->max_steps ||
                          (gram && tok == rule.close);
        if (gram) st->n_tok = 1;
        if (stop) {
            st->done = 1;
        } else if (gram) {
            const int syn = grammar_syntax(rule, tok, st->step);
            if (syn >= 0) {
                out_tokens[st->step] = syn;
                st->step += 1;
                st->n_tok = 2;
                st->cur_token2 = syn;
                if (st->step >= st->max_steps) st->done = 1;  // the forced token was the last output
            }
        }
    }
}

}  // namespace icua
