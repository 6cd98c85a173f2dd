// Tensor-core dequant-GEMM for the dense cases (prefill rows, batched decode): tcgen05.mma with
// the accumulator in tensor memory, weights dequantised from the q4s / q8 device tile layout into
// shared memory by CUDA cores, activations brought in by TMA.
//
// Replaces the reference prefill GEMM (llm_gemm_tile + k_g3_*, Shaders.swift:927-1097): fp16
// activations X [m_tok, K], weights dequantised to fp16 as half(q) * half(scale) (one fp16
// rounding, the rule of Shaders.swift:958-959 applied to the symmetric int4 codes), fp32
// accumulation, fused epilogues (store, residual add, SwiGLU into fp16, argmax partials).
//
// Design (B200): one CTA computes D[MH x 128 weight rows][BN tokens] = W X^T as UMMA M=128,
// N=BN, K=16 steps (kind::f16, both operands K-major with the 128-byte swizzle), MH = 1 or 2
// accumulators of BN columns in tensor memory sharing every activation tile (MH = 2 halves the
// L2 traffic per FLOP).  BN (a multiple of 16 up to 256) is chosen per GEMM by the host so that
// the tile count fills whole waves of SMs.
//   warp 0      producer: 1-D bulk copies of the 8 x MH 16-row weight units of each 64-column
//               k-block, and a 2-D TMA tile load (box 64 x BN, SWIZZLE_128B) of the activations
//   warp 1      allocates tensor memory and issues the MMAs (one thread); each stage is released
//               with tcgen05.commit onto the stage's "empty" barrier
//   warps 2..9  dequantise each staged unit into the swizzled A tile (two warps per scheduler),
//               then run the epilogue: tcgen05.ld 32x32b (warp w reads TMEM lanes 32 (w % 4) ..),
//               one weight row per thread, tokens along the registers
// Every wait is bounded; a wait that gives up records an error flag, and the kernel still drains
// its copies and frees its tensor memory before it exits.
// Programmatic dependent launch: the weights do not depend on the previous kernel, so quantised
// weights of the first stages are copied (and dequantised) before griddepcontrol.wait; the
// activation loads and every global access of the epilogue come after it.
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "layout.h"

namespace icua {

constexpr int TC_BM = 128;      // weight rows per accumulator (UMMA M)
constexpr int TC_SPLITK_MAX = 8;  // K slices of a split GEMM (finish kernels unroll over them)
constexpr int TC_BK = 64;       // columns per stage: one 128-byte swizzle row of fp16
constexpr int TC_THREADS = 320; // producer warp, MMA warp, 8 dequant / epilogue warps
constexpr int TC_SMEM_BUDGET = 225 * 1024;

// TC_GELU (fp16 weights only): out_h[tok * ldh + row] = half(gelu(y)), tanh form or, with
// gelu_erf, the exact erf form (the vision MLP and mergers).
enum TcEpi { TC_STORE = 0, TC_RESID = 1, TC_SWIGLU = 2, TC_ARGMAX = 3, TC_GELU = 4 };

struct TcGemmParams {
    const uint8_t* w;          // weights in the device tile layout [n_rows, k] (q4s, q4a or q8)
    const uint8_t* wtc;        // the same weights in tensor-core row order (tc_order_rows_kernel,
                               //   tc_order_rows_q8_kernel), or nullptr: then each stage gathers
                               //   8 x MH units from `w`
    int n_rows, k, n_tiles, upt;
    int m_tok;                 // activation rows (tokens)
    int bn;                    // tokens per CTA tile (multiple of 16, <= 256; the TMA box height)
    float* out;                // TC_STORE: out[tok * ldo + row] = y; TC_RESID: out[...] += y
    int ldo;
    __half* out_h;             // TC_SWIGLU: out_h[tok * ldh + j] = silu(gate_j) * up_j
    int ldh;
    const float* deepstack;    // TC_RESID: optional rows added after the residual, [ds_rows][ldo]
    int ds_row0, ds_rows;      // token range [ds_row0, ds_row0 + ds_rows) that receives them
    float* best_v;             // TC_ARGMAX: per (row tile, token) maximum [row tiles][m_tok] and the
    int* best_i;               //   row of it (lowest row on ties); out, when set, also gets the values
    int* err;                  // error flags (bounded waits that gave up)
    long long out_zstride;     // split K (gridDim.z > 1, TC_STORE only): slice z covers k-blocks
                               //   [z nk / Z, (z+1) nk / Z) and stores to out + z * out_zstride
    const float* bias;         // fp16-weight GEMMs: per weight row, added to y before the epilogue
    int gelu_erf;              // TC_GELU: 1 = exact erf GELU, 0 = tanh approximation
    int max_stages;            // pipeline depth cap (TcLayout), set by the launcher
    int pdl;                   // launched as a programmatic dependent: all S stages' quantised
                               //   weights are requested before griddepcontrol.wait (else only the
                               //   first, so that the first activation tile is not queued behind S
                               //   weight tiles)
    int hilo;                  // activations as fp16 hi / lo row pairs (rows 2t, 2t + 1 of token
                               //   t: x = hi + lo to ~22 bits): B has 2 m_tok rows, the epilogue
                               //   adds the pair's accumulator columns (batched decode)
    int hilo_out;              // TC_SWIGLU: out_h written as hi / lo row pairs as well
};

// Stores the normalised fp16 values of row i for thread tid's eight elements (4 tid .. 4 tid + 3
// and 1024 + 4 tid ..): out[i] or, hilo, the fp16 hi / lo rows 2i and 2i + 1 (hi + lo = the fp32
// value to ~22 bits, the batched decode GEMMs' input).
__device__ __forceinline__ void store_norm_row(__half* out, int i, int tid, float4 a, float4 b, float r, float4 wa,
                                               float4 wb, bool hilo) {
    const float y[8] = {a.x * r * wa.x, a.y * r * wa.y, a.z * r * wa.z, a.w * r * wa.w,
                        b.x * r * wb.x, b.y * r * wb.y, b.z * r * wb.z, b.w * r * wb.w};
    if (!hilo) {
        __half2* o = reinterpret_cast<__half2*>(out + (size_t)i * H);
        o[2 * tid] = __floats2half2_rn(y[0], y[1]);
        o[2 * tid + 1] = __floats2half2_rn(y[2], y[3]);
        o[2 * (tid + 256)] = __floats2half2_rn(y[4], y[5]);
        o[2 * (tid + 256) + 1] = __floats2half2_rn(y[6], y[7]);
        return;
    }
    __half hi[8], lo[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        hi[e] = __float2half_rn(y[e]);
        lo[e] = __float2half_rn(y[e] - __half2float(hi[e]));
    }
    __half2* oh = reinterpret_cast<__half2*>(out + (size_t)(2 * i) * H);
    __half2* ol = reinterpret_cast<__half2*>(out + (size_t)(2 * i + 1) * H);
    oh[2 * tid] = __halves2half2(hi[0], hi[1]);
    oh[2 * tid + 1] = __halves2half2(hi[2], hi[3]);
    oh[2 * (tid + 256)] = __halves2half2(hi[4], hi[5]);
    oh[2 * (tid + 256) + 1] = __halves2half2(hi[6], hi[7]);
    ol[2 * tid] = __halves2half2(lo[0], lo[1]);
    ol[2 * tid + 1] = __halves2half2(lo[2], lo[3]);
    ol[2 * (tid + 256)] = __halves2half2(lo[4], lo[5]);
    ol[2 * (tid + 256) + 1] = __halves2half2(lo[6], lo[7]);
}

// fp16 hi / lo pair of x: hi = fp16(x), lo = fp16(x - hi).
__device__ __forceinline__ void split_hilo(float x, __half& hi, __half& lo) {
    hi = __float2half_rn(x);
    lo = __float2half_rn(x - __half2float(hi));
}

// Epilogue activations on the hardware approximations (tanh.approx, ex2.approx through __expf,
// __fdividef): their outputs are rounded to fp16 right after, well above the approximation error.
__device__ __forceinline__ float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// Shared-memory layout of one CTA for a (BN, MH, format) choice; the same arithmetic runs on the
// host (launch size) and the device (offsets).
// A operand in tensor memory: for the 4-bit formats in row order (the batched decode GEMMs) with one
// accumulator of at most 128 columns, the dequantising warps write each stage's A tile [128 rows][64]
// with tcgen05.st into TMEM columns after the accumulator (lane = weight row, two fp16 of
// consecutive k per 32-bit column), and the MMA reads it from there: the A tile never passes
// through shared memory, whose bandwidth (A written by the CUDA cores and read by the tensor core
// at 4 bytes per weight) bounded these GEMMs.  TMEM columns: the accumulator, then 32 per stage;
// 256 columns up to 128 activation rows, all 512 above (one such CTA per SM).
__host__ __device__ constexpr int tc_acc_cols(int bn) { return (bn + 31) & ~31; }
__host__ __device__ constexpr int tc_tmem_cols(int mh, int bn, bool a_tmem) {
    return (mh == 2 || (a_tmem && bn > 128)) ? 512 : 256;
}
__host__ __device__ constexpr int tc_tmem_a_slots(int bn) { return (tc_tmem_cols(1, bn, true) - tc_acc_cols(bn)) / 32; }
__host__ __device__ constexpr bool tc_a_in_tmem(int fmt, bool row_order, int mh, int bn) {
    return (fmt == 1 || fmt == 2 || fmt == 3) && row_order && mh == 1 && bn <= 256;  // FMT_Q8, FMT_Q4A, FMT_Q4S
}
// k-blocks per pipeline stage: two with the A tiles in tensor memory when every K slice has an even
// number of them (the MMA-issuing thread, which paces these GEMMs, then waits, commits and loops
// once per 128 columns), else one.
__host__ __device__ constexpr int tc_kb(bool a_tmem, int nk_all, int ksplit) {
    return (a_tmem && nk_all % (2 * ksplit) == 0) ? 2 : 1;
}

struct TcLayout {
    int S;                                   // pipeline stages
    int a_bytes, b_bytes, raw_bytes, stage_bytes;
    int a_off, b_off, raw_off, bar_off, tmem_off, red_off, total, alloc;
    // max_stages: 8 for throughput GEMMs; the batched-decode GEMMs take 3, which halves the
    // footprint so that the next kernel's CTA (programmatic launch) fits beside this one on an SM
    // (measured 2% faster per batched step than 4 to 7 stages, 6% faster than 2)
    // a_tmem: the dequantised A tiles live in tensor memory (tc_a_in_tmem), at most
    // tc_tmem_a_slots(bn) stages of them
    // kb: k-blocks per stage (tc_kb); a stage holds kb activation tiles and kb quantised blocks
    __host__ __device__ TcLayout(int bn, int mh, int fmt, bool argmax, int max_stages = 8, bool a_tmem = false,
                                 int kb = 1) {
        a_bytes = a_tmem ? 0 : mh * TC_BM * 128;  // fp16 [mh * 128][64], swizzled
        b_bytes = kb * bn * 128;             // kb x fp16 [bn][64], swizzled by TMA
        raw_bytes = kb * mh * 8 * unit_bytes(fmt);
        stage_bytes = a_bytes + b_bytes + raw_bytes;
        const int red = argmax ? 4 * mh * bn * 8 : 0;
        S = (TC_SMEM_BUDGET - red - 1024 - 512) / stage_bytes;
        if (S > max_stages) S = max_stages;
        if (a_tmem && S > tc_tmem_a_slots(bn) / kb) S = tc_tmem_a_slots(bn) / kb;
        a_off = 0;
        b_off = a_off + S * a_bytes;
        raw_off = b_off + S * b_bytes;
        bar_off = raw_off + S * raw_bytes;   // rawfull, bfull, afull, empty [S]; accfull
        tmem_off = bar_off + (4 * S + 1) * 8;
        red_off = (tmem_off + 16 + 15) & ~15;
        total = red_off + red;
        alloc = total + 1024;                // room to align the tiles to 1024 B
    }
};

// ---- tcgen05 / TMA helpers ------------------------------------------------------------------

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart
// (stride byte offset), descriptor version 1, layout type 2 (SWIZZLE_128B).  The leading byte
// offset is unused for swizzled K-major layouts and set to 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16: fp32 accumulator, fp16 A and B, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The same with A read from tensor memory at `tmem_a` (K-major, 128 lanes = rows).
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 16 consecutive 32-bit columns of this warp's 32 TMEM lanes from registers, then waits until the
// stores are done.
__device__ __forceinline__ void tmem_st16_wait(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Arrives on `bar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes: lane i of the warp gets lane
// (base lane + i), columns col .. col + 31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[32]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 2-D TMA tile load into this CTA's shared memory.  x (the contiguous dimension) is a multiple of 64 elements.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Byte offset of element (row, k) of a [rows][64] fp16 tile in the 128-byte swizzle: row r at
// r * 128, its 16-byte chunk c at position c ^ (r & 7) (the TMA SWIZZLE_128B pattern).
__device__ __forceinline__ int sw128_off(int row, int k) {
    return row * 128 + ((((k >> 3) ^ (row & 7))) << 4) + ((k & 7) << 1);
}

// Dequantises lane l's 16 bytes of one q4s unit (rows row0 .. row0 + 15, 64 columns) into the
// swizzled A tile.  The lane holds rows g = l / 4 and g + 8 at columns 16 s + 2t (+1, +8, +9)
// for s = 0..3; codes u in 0..15 mean q = u - 8.  fp16(1024 + u) is built by OR-ing u into the
// mantissa of 1024, 1032 is subtracted exactly and the scale applied with one fp16 rounding.
__device__ __forceinline__ void dequant_q4s_lane(const uint8_t* unit, int l, uint8_t* A, int row0) {
    const uint4 nib = *reinterpret_cast<const uint4*>(unit + l * 16);
    const int g = l >> 2, t = l & 3;
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(unit + 512 + g * 8);  // ra g0, rb g0, ra g1, rb g1
    const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032
    const int ra = row0 + g, rb = ra + 8;
    const uint32_t w[4] = {nib.x, nib.y, nib.z, nib.w};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const __half sa1 = __ushort_as_half(sc[(s >> 1) * 2]), sb1 = __ushort_as_half(sc[(s >> 1) * 2 + 1]);
        const __half2 sa = __halves2half2(sa1, sa1), sb = __halves2half2(sb1, sb1);
        const int k0 = 16 * s + 2 * t;
        const uint32_t v = w[s];
        uint32_t h[4];
        h[0] = (v & 0x000F000Fu) | 0x64006400u;          // row a, k0 / k0+1
        h[1] = ((v >> 4) & 0x000F000Fu) | 0x64006400u;   // row b, k0 / k0+1
        h[2] = ((v >> 8) & 0x000F000Fu) | 0x64006400u;   // row a, k0+8 / k0+9
        h[3] = ((v >> 12) & 0x000F000Fu) | 0x64006400u;  // row b, k0+8 / k0+9
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __half2 x = *reinterpret_cast<__half2*>(&h[i]);
            x = __hmul2(__hsub2(x, bias), (i & 1) ? sb : sa);
            h[i] = *reinterpret_cast<uint32_t*>(&x);
        }
        *reinterpret_cast<uint32_t*>(A + sw128_off(ra, k0)) = h[0];
        *reinterpret_cast<uint32_t*>(A + sw128_off(rb, k0)) = h[1];
        *reinterpret_cast<uint32_t*>(A + sw128_off(ra, k0 + 8)) = h[2];
        *reinterpret_cast<uint32_t*>(A + sw128_off(rb, k0 + 8)) = h[3];
    }
}

// q8 counterpart: lane l's bytes of one q8 unit (offset-binary codes u = q + 128).  For k16 step
// s the lane's 8 bytes sit at (s / 2) * 512 + l * 16 + (s % 2) * 8: rows a/b interleaved at
// columns k0, k0+1, then k0+8, k0+9.  fp16(1024 + u) - 1152 = q exactly, then one fp16 rounding
// of q * scale (the reference prefill rule half4(char4) * s, Shaders.swift:958-959).
__device__ __forceinline__ void dequant_q8_lane(const uint8_t* unit, int l, uint8_t* A, int row0) {
    const int g = l >> 2, t = l & 3;
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(unit + 1024 + g * 8);
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
    const int ra = row0 + g, rb = ra + 8;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const __half sa1 = __ushort_as_half(sc[(s >> 1) * 2]), sb1 = __ushort_as_half(sc[(s >> 1) * 2 + 1]);
        const __half2 sa = __halves2half2(sa1, sa1), sb = __halves2half2(sb1, sb1);
        const int k0 = 16 * s + 2 * t;
        const uint2 w = *reinterpret_cast<const uint2*>(unit + (s >> 1) * 512 + l * 16 + (s & 1) * 8);
        uint32_t h[4];
        h[0] = __byte_perm(w.x, 0x6464u, 0x5240);  // row a, k0 / k0+1
        h[1] = __byte_perm(w.x, 0x6464u, 0x5341);  // row b, k0 / k0+1
        h[2] = __byte_perm(w.y, 0x6464u, 0x5240);  // row a, k0+8 / k0+9
        h[3] = __byte_perm(w.y, 0x6464u, 0x5341);  // row b, k0+8 / k0+9
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __half2 x = *reinterpret_cast<__half2*>(&h[i]);
            x = __hmul2(__hsub2(x, bias), (i & 1) ? sb : sa);
            h[i] = *reinterpret_cast<uint32_t*>(&x);
        }
        *reinterpret_cast<uint32_t*>(A + sw128_off(ra, k0)) = h[0];
        *reinterpret_cast<uint32_t*>(A + sw128_off(rb, k0)) = h[1];
        *reinterpret_cast<uint32_t*>(A + sw128_off(ra, k0 + 8)) = h[2];
        *reinterpret_cast<uint32_t*>(A + sw128_off(rb, k0 + 8)) = h[3];
    }
}

// Reference affine q4 (codes 0..15, one fp16 (scale, bias) per row and 64-column unit):
// fp16(1024 + u) - 1024 = u exactly, then one fused rounding of u * scale + bias.
__device__ __forceinline__ void dequant_q4a_lane(const uint8_t* unit, int l, uint8_t* A, int row0) {
    const uint4 nib = *reinterpret_cast<const uint4*>(unit + l * 16);
    const int g = l >> 2, t = l & 3;
    const uint2 sbw = *reinterpret_cast<const uint2*>(unit + 512 + g * 8);  // (scale, bias) rows g, g+8
    const __half2 sba = *reinterpret_cast<const __half2*>(&sbw.x), sbb = *reinterpret_cast<const __half2*>(&sbw.y);
    const __half2 sa = __half2half2(__low2half(sba)), ba = __half2half2(__high2half(sba));
    const __half2 sb = __half2half2(__low2half(sbb)), bb = __half2half2(__high2half(sbb));
    const __half2 base = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));  // 1024
    const int ra = row0 + g, rb = ra + 8;
    const uint32_t w[4] = {nib.x, nib.y, nib.z, nib.w};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const int k0 = 16 * s + 2 * t;
        const uint32_t v = w[s];
        uint32_t h[4];
        h[0] = (v & 0x000F000Fu) | 0x64006400u;
        h[1] = ((v >> 4) & 0x000F000Fu) | 0x64006400u;
        h[2] = ((v >> 8) & 0x000F000Fu) | 0x64006400u;
        h[3] = ((v >> 12) & 0x000F000Fu) | 0x64006400u;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __half2 x = __hsub2(*reinterpret_cast<__half2*>(&h[i]), base);
            x = (i & 1) ? __hfma2(x, sb, bb) : __hfma2(x, sa, ba);
            h[i] = *reinterpret_cast<uint32_t*>(&x);
        }
        *reinterpret_cast<uint32_t*>(A + sw128_off(ra, k0)) = h[0];
        *reinterpret_cast<uint32_t*>(A + sw128_off(rb, k0)) = h[1];
        *reinterpret_cast<uint32_t*>(A + sw128_off(ra, k0 + 8)) = h[2];
        *reinterpret_cast<uint32_t*>(A + sw128_off(rb, k0 + 8)) = h[3];
    }
}

// Row order of the 4-bit formats (q4s, q4a) for the batched GEMMs: the 128-row block of one
// 64-column k-block sits at ((tile / 8) * upt + kk) * 4608 as in tc_order_kernel, but inside the
// block each row owns 32 contiguous bytes (row r at r * 32) whose 32-bit word j holds columns
// 8j .. 8j+7 with column 8j + 2i in bits 4i .. 4i+3 and 8j + 2i + 1 in bits 16 + 4i .. 19 + 4i, so
// that ((w >> 4i) & 0x000F000F) is the fp16 pair of two consecutive columns and one thread writes
// 8 consecutive columns of the A tile with one 16-byte store.  The 512 bytes after them hold per
// row the two 32-column group scales (q4s) or the unit's (scale, bias) pair (q4a), 4 bytes a row.
// One thread per output word (nibbles gathered from the device tile layout) and per row's scales.
constexpr int TC_ROWS_BLOCK = 4608;
__global__ void tc_order_rows_kernel(const uint8_t* src, int fmt, int n_tiles, int upt, uint8_t* dst) {
    const long long blocks = (long long)(n_tiles / 8) * upt;
    const long long words = blocks * 128 * 8, total = words + blocks * 128;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const bool is_word = i < words;
        const long long e = is_word ? i : i - words;
        const long long b = is_word ? e >> 10 : e >> 7;   // block index: (g8 * upt + kk)
        const int r = is_word ? (int)((e >> 3) & 127) : (int)(e & 127);
        const int g8 = (int)(b / upt), kk = (int)(b % upt);
        const int tile = g8 * 8 + (r >> 4), rt = r & 15, gq = rt & 7, up = rt >> 3;
        const uint8_t* ub = src + icua_layout::unit_offset(fmt, n_tiles, upt, tile, kk);
        uint8_t* blk = dst + b * TC_ROWS_BLOCK;
        if (is_word) {
            const int j = (int)(e & 7);
            uint32_t w = 0;
#pragma unroll
            for (int c8 = 0; c8 < 8; ++c8) {  // column 8j + c8 of the unit
                const int kin = 8 * j + c8, step = kin >> 4, k16 = kin & 15;
                const int t = (k16 & 7) >> 1, odd = k16 & 1, hi8 = k16 >> 3;
                const uint32_t sw = *reinterpret_cast<const uint32_t*>(ub + (gq * 4 + t) * 16 + step * 4);
                const uint32_t u = (sw >> (odd * 16 + hi8 * 8 + up * 4)) & 0xFu;
                w |= u << ((c8 & 1) * 16 + (c8 >> 1) * 4);
            }
            *reinterpret_cast<uint32_t*>(blk + r * 32 + j * 4) = w;
        } else {
            uint16_t v[2];
            if (fmt == FMT_Q4S) {  // group scales of rows g (low half) and g + 8 (high half)
                v[0] = *reinterpret_cast<const uint16_t*>(ub + 512 + gq * 8 + up * 2);
                v[1] = *reinterpret_cast<const uint16_t*>(ub + 512 + gq * 8 + 4 + up * 2);
            } else {  // q4a: (scale, bias) of row g at +0, of row g + 8 at +4
                v[0] = *reinterpret_cast<const uint16_t*>(ub + 512 + gq * 8 + up * 4);
                v[1] = *reinterpret_cast<const uint16_t*>(ub + 512 + gq * 8 + up * 4 + 2);
            }
            *reinterpret_cast<uint32_t*>(blk + 4096 + r * 4) = (uint32_t)v[0] | ((uint32_t)v[1] << 16);
        }
    }
}

// Row order of q8 (the tied embedding / lm_head of the batched step): the same blocks of 128 rows x
// 64 columns (8,704 bytes, as 8 q8 units) with row r's 64 code bytes in column order at r * 64 and
// its two 32-column group scales at 8192 + r * 4.  One thread per 16 code bytes and per row's scales.
constexpr int TC_ROWS_BLOCK_Q8 = 8704;
__global__ void tc_order_rows_q8_kernel(const uint8_t* src, int n_tiles, int upt, uint8_t* dst) {
    const long long blocks = (long long)(n_tiles / 8) * upt;
    const long long chunks = blocks * 128 * 4, total = chunks + blocks * 128;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const bool is_chunk = i < chunks;
        const long long e = is_chunk ? i : i - chunks;
        const long long b = is_chunk ? e >> 9 : e >> 7;  // block index: (g8 * upt + kk)
        const int r = is_chunk ? (int)((e >> 2) & 127) : (int)(e & 127);
        const int g8 = (int)(b / upt), kk = (int)(b % upt);
        const int tile = g8 * 8 + (r >> 4), rt = r & 15, gq = rt & 7, up = rt >> 3;
        const uint8_t* ub = src + icua_layout::unit_offset(FMT_Q8, n_tiles, upt, tile, kk);
        uint8_t* blk = dst + b * TC_ROWS_BLOCK_Q8;
        if (is_chunk) {
            const int j = (int)(e & 3);
            uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
            for (int c = 0; c < 16; ++c) {  // column 16 j + c of the unit
                const int kin = 16 * j + c, step = kin >> 4, k16 = kin & 15;
                const int t = (k16 & 7) >> 1, odd = k16 & 1, hi8 = k16 >> 3;
                const uint8_t* wp = ub + (step >> 1) * 512 + (gq * 4 + t) * 16 + ((step & 1) * 2 + hi8) * 4;
                w[c >> 2] |= (uint32_t)wp[odd * 2 + up] << ((c & 3) * 8);
            }
            *reinterpret_cast<uint4*>(blk + r * 64 + j * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        } else {
            const uint16_t v0 = *reinterpret_cast<const uint16_t*>(ub + 1024 + gq * 8 + up * 2);
            const uint16_t v1 = *reinterpret_cast<const uint16_t*>(ub + 1024 + gq * 8 + 4 + up * 2);
            *reinterpret_cast<uint32_t*>(blk + 8192 + r * 4) = (uint32_t)v0 | ((uint32_t)v1 << 16);
        }
    }
}

// Dequantises half of one row of a row-order block: row r, columns 32 half .. +31 (one scale
// group), as 16 fp16 pairs of consecutive columns, with the arithmetic of dequant_q4s_lane /
// dequant_q4a_lane / dequant_q8_lane (bit-identical values).
template <int FMT>
__device__ __forceinline__ void dequant_rows_regs(const uint8_t* blk, int r, int half, uint32_t (&h)[16]) {
    if constexpr (FMT == FMT_Q8) {
        // fp16(1024 + u) from the code byte, - 1152 = q exactly, then one rounding of q * scale
        const uint4 b0 = *reinterpret_cast<const uint4*>(blk + r * 64 + half * 32);
        const uint4 b1 = *reinterpret_cast<const uint4*>(blk + r * 64 + half * 32 + 16);
        const uint32_t sv = *reinterpret_cast<const uint32_t*>(blk + 8192 + r * 4);
        const __half s1 = __ushort_as_half((uint16_t)(half ? sv >> 16 : sv & 0xFFFFu));
        const __half2 mul = __halves2half2(s1, s1);
        const __half2 off = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
        const uint32_t w[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t lo = __byte_perm(w[k], 0x6464u, 0x5140), hi = __byte_perm(w[k], 0x6464u, 0x5342);
            __half2 x0 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&lo), off), mul);
            __half2 x1 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&hi), off), mul);
            h[2 * k] = *reinterpret_cast<uint32_t*>(&x0);
            h[2 * k + 1] = *reinterpret_cast<uint32_t*>(&x1);
        }
        return;
    }
    const uint4 nib = *reinterpret_cast<const uint4*>(blk + r * 32 + half * 16);
    const uint32_t sv = *reinterpret_cast<const uint32_t*>(blk + 4096 + r * 4);
    __half2 mul, add;
    if (FMT == FMT_Q4S) {
        const __half s1 = __ushort_as_half((uint16_t)(half ? sv >> 16 : sv & 0xFFFFu));
        mul = __halves2half2(s1, s1);
        add = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032: u - 8 - 1024
    } else {
        const __half2 sb = *reinterpret_cast<const __half2*>(&sv);
        mul = __half2half2(__low2half(sb));
        add = __half2half2(__high2half(sb));
    }
    const __half2 base = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));  // 1024
    const uint32_t w[4] = {nib.x, nib.y, nib.z, nib.w};
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t v = ((w[jj] >> (4 * i)) & 0x000F000Fu) | 0x64006400u;
            __half2 x = *reinterpret_cast<const __half2*>(&v);
            if (FMT == FMT_Q4S)
                x = __hmul2(__hsub2(x, add), mul);
            else
                x = __hfma2(__hsub2(x, base), mul, add);
            h[jj * 4 + i] = *reinterpret_cast<uint32_t*>(&x);
        }
    }
}

// The same into the swizzled shared-memory A tile: thread d takes row d / 2 and half d % 2, four
// 16-byte stores of 8 consecutive columns.
template <int FMT>
__device__ __forceinline__ void dequant_rows_half(const uint8_t* blk, int d, uint8_t* A, int row_base) {
    const int r = d >> 1, half = d & 1;
    uint32_t h[16];
    dequant_rows_regs<FMT>(blk, r, half, h);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj)
        *reinterpret_cast<uint4*>(A + sw128_off(row_base + r, 32 * half + 8 * jj)) =
            make_uint4(h[jj * 4], h[jj * 4 + 1], h[jj * 4 + 2], h[jj * 4 + 3]);
}

template <int EPI, int FMT, int MH>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_gemm_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                const __grid_constant__ CUtensorMap wmap,
                                                                const TcGemmParams p) {
    constexpr int UB = unit_bytes(FMT);
    constexpr int NU = 8 * MH;  // 16-row units per stage
    const int BN = p.bn;
    const bool ATM = tc_a_in_tmem(FMT, p.wtc != nullptr, MH, BN);  // A tiles in tensor memory
    const int KB = tc_kb(ATM, p.k / TC_BK, gridDim.z);           // k-blocks per stage
    const TcLayout SM(BN, MH, FMT, EPI == TC_ARGMAX, p.max_stages, ATM, KB);
    const int S = SM.S;
    const int b_tile = BN * 128;  // bytes of one activation tile (64 columns)
    const uint32_t a_col0 = (uint32_t)tc_acc_cols(BN);  // ATM: stage s's A tile at columns a_col0 + 32 s
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base_u = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((base_u + 1023u) & ~1023u) - base_u);
    uint64_t* rawfull = reinterpret_cast<uint64_t*>(smem + SM.bar_off);
    uint64_t* bfull = rawfull + S;
    uint64_t* afull = bfull + S;
    uint64_t* empty = afull + S;
    uint64_t* accfull = empty + S;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SM.tmem_off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // grid: x = token tile (fastest), y = weight-row tile, z = K slice; CTAs that share a weight
    // tile are launched together, so it comes from DRAM once and from L2 for the others
    const int rtile = blockIdx.y;
    const int tile0 = rtile * (MH * TC_BM / 16);
    const int row0 = rtile * (MH * TC_BM);
    const int tok0 = blockIdx.x * BN;
    const int nk_all = p.k / TC_BK;
    const int kb0 = (int)((long long)nk_all * blockIdx.z / gridDim.z);
    // stages of this K slice (KB k-blocks each)
    const int nk = ((int)((long long)nk_all * (blockIdx.z + 1) / gridDim.z) - kb0) / KB;
    // CTAs that share a weight tile start at different k-blocks (rotation by the token-tile
    // index), so they do not all request the same rows from L2 at the same moment
    const int krot = (int)((blockIdx.x * 5u) % (unsigned)nk);
    const uint32_t tmem_cols = (uint32_t)tc_tmem_cols(MH, BN, ATM);
    constexpr int half_cols = 256;  // column offset of the second accumulator

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&rawfull[s], 1);
            mbar_init(&bfull[s], 1);
            mbar_init(&afull[s], ATM ? 9 : 8);  // ATM: + the producer's arrival with the activation bytes
            mbar_init(&empty[s], 1);
        }
        mbar_init(accfull, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // the dependents may start their own weight prefetch on the SMs this grid leaves free
    pdl_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&xmap) : "memory");
            if (FMT == FMT_F16) asm volatile("prefetch.tensormap [%0];" ::"l"(&wmap) : "memory");
            // weights of stage kc: the quantised units by bulk copy onto rawfull[s], or fp16 boxes by
            // TMA onto bfull[s] with the stage's activation tile (one barrier: measured 5% faster on
            // the prefill GEMMs than a barrier per operand), which is why fp16 weights are never
            // requested ahead of griddepcontrol.wait
            auto issue_w = [&](int kc) {
                const int s = kc % S;
                const int kblk = kb0 + KB * ((kc + krot) % nk);
                if constexpr (FMT == FMT_F16) {
                    mbar_expect_tx(&bfull[s], (uint32_t)(SM.a_bytes + SM.b_bytes));
#pragma unroll
                    for (int h = 0; h < MH; ++h)
                        tma_load_2d(smem + SM.a_off + s * SM.a_bytes + h * TC_BM * 128, &wmap, kblk * TC_BK,
                                    row0 + h * TC_BM, &bfull[s]);
                } else {
                    uint8_t* raw = smem + SM.raw_off + s * SM.raw_bytes;
                    mbar_expect_tx(&rawfull[s], KB * NU * UB);
                    if (p.wtc != nullptr) {
                        // tensor-core order: a 128-row block of a k-block is contiguous, and so are the
                        // KB blocks of a stage (consecutive k-blocks of one row tile)
#pragma unroll
                        for (int h = 0; h < MH; ++h)
                            bulk_g2s(raw + h * KB * 8 * UB, p.wtc + ((size_t)(rtile * MH + h) * p.upt + kblk) * 8 * UB,
                                     KB * 8 * UB, &rawfull[s]);
                    } else {
#pragma unroll 1
                        for (int t = 0; t < NU; ++t)
                            bulk_g2s(raw + t * UB, p.w + icua_layout::unit_offset(FMT, p.n_tiles, p.upt, tile0 + t, kblk),
                                     UB, &rawfull[s]);
                    }
                }
            };
            const int pre = FMT == FMT_F16 ? 0 : min(p.pdl ? S : 1, nk);
            for (int kc = 0; kc < pre; ++kc) issue_w(kc);
            pdl_wait();  // the activations are the previous kernel's output
            int kc = 0;
            for (; kc < nk; ++kc) {
                const int s = kc % S;
                if (kc >= S && !(ATM ? mbar_wait_nap(&empty[s], (uint32_t)((kc / S - 1) & 1), 64)
                                     : mbar_wait_bounded(&empty[s], (uint32_t)((kc / S - 1) & 1)))) {
                    atomicOr(p.err, ERR_WAIT_PREFILL);
                    break;
                }
                if (kc >= pre) issue_w(kc);
                // ATM: the activation tile completes on afull[s] with the dequantised A tile, so that
                // the MMA thread waits on one barrier per stage
                uint64_t* xbar = ATM ? &afull[s] : &bfull[s];
                if (FMT != FMT_F16) mbar_expect_tx(xbar, (uint32_t)SM.b_bytes);
                for (int kb = 0; kb < KB; ++kb)
                    tma_load_2d(smem + SM.b_off + s * SM.b_bytes + kb * b_tile, &xmap,
                                (kb0 + KB * ((kc + krot) % nk) + kb) * TC_BK, tok0, xbar);
            }
            // the copies of the last stages complete before the CTA may exit (at once on success);
            // after a failed wait at kc >= S the stages issued are [0, kc), all within this range
            // or consumed already
            const int issued = kc < pre ? pre : kc;
            for (int c = (issued > S ? issued - S : 0); c < issued; ++c) {
                if (FMT != FMT_F16) mbar_wait_bounded(&rawfull[c % S], (uint32_t)((c / S) & 1));
                if (c < kc) mbar_wait_bounded(ATM ? &afull[c % S] : &bfull[c % S], (uint32_t)((c / S) & 1));
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(TC_BM, BN);
            if (ATM) {
                // this thread paces the GEMM: one barrier per stage (A tile and activation tile),
                // stage and phase as counters, the MMAs read the stage's A columns of TMEM
                const uint64_t bd0 = umma_desc_sw128(smem_u32(smem + SM.b_off));
                const uint32_t b_step = (uint32_t)b_tile >> 4;  // one activation tile, descriptor units
                int s = 0;
                uint32_t ph = 0;
                for (int kc = 0; kc < nk; ++kc) {
                    if (!mbar_wait_bounded(&afull[s], ph)) {
                        atomicOr(p.err, ERR_WAIT_PREFILL);
                        break;
                    }
                    tc_fence_after();
                    for (int kb = 0; kb < KB; ++kb) {
                        const uint32_t slot = (uint32_t)(s * KB + kb);
                        const uint64_t bd = bd0 + (uint64_t)(b_step * slot);
                        const uint32_t at = tmem + a_col0 + 32u * slot;
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks)  // K = 16 per MMA: 8 TMEM columns of fp16 pairs
                            tc_mma_f16_ts(tmem, at + 8u * (uint32_t)ks, bd + 2 * ks, idesc, (kc | kb | ks) != 0);
                    }
                    tc_commit(&empty[s]);
                    if (++s == S) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                tc_commit(accfull);  // also on the error path: tracks the MMAs already issued
            }
            for (int kc = 0; kc < (ATM ? 0 : nk); ++kc) {
                const int s = kc % S;
                const uint32_t ph = (uint32_t)((kc / S) & 1);
                // A operand: dequantised by the CUDA-core warps (afull), or fp16 weights by TMA (rawfull)
                if ((FMT != FMT_F16 && !mbar_wait_bounded(&afull[s], ph)) || !mbar_wait_bounded(&bfull[s], ph)) {
                    atomicOr(p.err, ERR_WAIT_PREFILL);
                    break;
                }
                tc_fence_after();
                const uint64_t bd = umma_desc_sw128(smem_u32(smem + SM.b_off + s * SM.b_bytes));
#pragma unroll
                for (int h = 0; h < MH; ++h) {
                    const uint64_t ad = umma_desc_sw128(smem_u32(smem + SM.a_off + s * SM.a_bytes + h * TC_BM * 128));
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)  // K = 16 per MMA: 32 bytes along the swizzled row
                        tc_mma_f16(tmem + h * half_cols, ad + 2 * ks, bd + 2 * ks, idesc, (kc | ks) != 0);
                }
                tc_commit(&empty[s]);
            }
            if (!ATM) tc_commit(accfull);  // also on the error path: tracks the MMAs already issued
        }
    } else {
        // ---- dequantisation: NU units x 32 lanes per stage over 256 threads ----
        const int d = threadIdx.x - 64;
        for (int kc = 0; kc < (FMT == FMT_F16 ? 0 : nk); ++kc) {
            const int s = kc % S;
            const bool got = __all_sync(0xffffffffu, ATM ? mbar_wait_nap(&rawfull[s], (uint32_t)((kc / S) & 1), 32)
                                                         : mbar_wait_bounded(&rawfull[s], (uint32_t)((kc / S) & 1)));
            if (!got) {
                if (lane == 0) atomicOr(p.err, ERR_WAIT_PREFILL);
                break;
            }
            const uint8_t* raw = smem + SM.raw_off + s * SM.raw_bytes;
            uint8_t* A = smem + SM.a_off + s * SM.a_bytes;
            if (ATM) {
                // warp w writes TMEM lanes 32 (w % 4) .. + 31 (its lane quarter): row 32 (w % 4) +
                // lane, columns 32 half .. + 31 with half = 0 for warps 2..5, 1 for warps 6..9.  The
                // slot was last read by the MMAs of stage kc - S, complete before this stage's copy
                // was issued.
                tc_fence_after();
                const int q = warp & 3, half = (warp - 2) >> 2;
                for (int kb = 0; kb < KB; ++kb) {
                    uint32_t h[16];
                    dequant_rows_regs<FMT>(raw + kb * 8 * UB, q * 32 + lane, half, h);
                    tmem_st16_wait(tmem + ((uint32_t)(q * 32) << 16) + a_col0 + 32u * (uint32_t)(s * KB + kb) +
                                       16u * (uint32_t)half,
                                   h);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&afull[s]);
                continue;
            }
            if (p.wtc != nullptr) {
                // row order (tc_order_rows_kernel / tc_order_rows_q8_kernel): 16-byte stores of 8
                // consecutive columns
#pragma unroll
                for (int i = 0; i < MH; ++i) dequant_rows_half<FMT>(raw + i * 8 * UB, d, A, i * TC_BM);
            } else {
#pragma unroll
                for (int i = 0; i < MH; ++i) {
                    const int pi = d + 256 * i, t = pi >> 5;
                    if constexpr (FMT == FMT_Q4S)
                        dequant_q4s_lane(raw + t * UB, pi & 31, A, t * 16);
                    else if constexpr (FMT == FMT_Q8)
                        dequant_q8_lane(raw + t * UB, pi & 31, A, t * 16);
                    else if constexpr (FMT == FMT_Q4A)
                        dequant_q4a_lane(raw + t * UB, pi & 31, A, t * 16);
                }
            }
            fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(&afull[s]);
        }
        // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) ..; wg = 0 / 1 picks the accumulator
        // (MH == 2) or every other 32-column chunk (MH == 1) ----
        const bool done = __all_sync(0xffffffffu, mbar_wait_bounded(accfull, 0));
        tc_fence_after();
        pdl_wait();  // (already satisfied: the MMAs consumed activations loaded after it)
        if (!done) {
            if (lane == 0) atomicOr(p.err, ERR_WAIT_PREFILL);
        } else {
            const int q = warp & 3, wg = (warp - 2) >> 2;
            const int h = MH == 2 ? wg : 0;
            const int row = row0 + h * TC_BM + q * 32 + lane;
            const int cstep = MH == 2 ? 1 : 2;
            const int HL = p.hilo ? 2 : 1;  // accumulator columns per token
#pragma unroll 1
            for (int c = (MH == 2 ? 0 : wg); c * 32 < BN; c += cstep) {
                if (tok0 + c * 32 >= p.m_tok * HL) break;
                float v[32];
                const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * half_cols + c * 32);
                const int ncol_b = min(32, BN - c * 32);  // 32 or 16 accumulator columns
                if (ncol_b == 32)
                    tmem_ld32(taddr, v);
                else
                    tmem_ld16(taddr, v);
                if (p.hilo) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = v[2 * j] + v[2 * j + 1];
                }
                // from here on: tokens ctok .. ctok + ncol - 1 of the chunk in v[0 .. ncol - 1]
                const int ctok = (tok0 + c * 32) / HL, ncol = ncol_b / HL;
                if (FMT == FMT_F16 && p.bias != nullptr) {
                    const float b = p.bias[row];
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] += b;
                }
                if (EPI == TC_GELU) {
                    // one weight row per thread, 32 tokens: fp16 stores strided by ldh
                    const int nj = min(ncol, p.m_tok - ctok);
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (j < nj) {
                            const float x = v[j];
                            const float g = p.gelu_erf ? 0.5f * x * (1.0f + erff(x * 0.70710678118654752f))
                                                       : 0.5f * x * (1.0f + tanh_approx(0.79788456080286536f *
                                                                                  (x + 0.044715f * x * x * x)));
                            p.out_h[(size_t)(ctok + j) * p.ldh + row] = __float2half_rn(g);
                        }
                    }
                    continue;
                }
                if (EPI == TC_RESID) {
                    // residual rows: the chunk's loads first (independent, in flight together),
                    // then the adds and stores; DeepStack rows (three layers of a visual prefill)
                    // are added after the residual, as the reference does
                    const int nj = min(ncol, p.m_tok - ctok);
                    float old[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        old[j] = j < nj ? p.out[(size_t)(ctok + j) * p.ldo + row] : 0.f;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int tok = ctok + j;
                        if (j < nj) {
                            float nv = old[j] + v[j];
                            if (p.deepstack != nullptr && tok >= p.ds_row0 && tok < p.ds_row0 + p.ds_rows)
                                nv += p.deepstack[(size_t)(tok - p.ds_row0) * p.ldo + row];
                            p.out[(size_t)tok * p.ldo + row] = nv;
                        }
                    }
                    continue;
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int tok = ctok + j;
                    if (j >= ncol || tok >= p.m_tok) break;
                    if (EPI == TC_STORE) {
                        p.out[blockIdx.z * p.out_zstride + (size_t)tok * p.ldo + row] = v[j];
                    } else if (EPI == TC_ARGMAX) {
                        if (p.out != nullptr) p.out[(size_t)tok * p.ldo + row] = v[j];
                        float bv = v[j];
                        int bi = row;
                        warp_argmax(bv, bi);
                        if (lane == 0) {
                            float2* red = reinterpret_cast<float2*>(smem + SM.red_off);
                            red[(h * 4 + q) * BN + (c * 32) / HL + j] = make_float2(bv, __int_as_float(bi));
                        }
                    } else {
                        // rows of a 16-row tile: 0..7 gate j, 8..15 up j (tile * 8 + r)
                        const float u = __shfl_xor_sync(0xffffffffu, v[j], 8);
                        if (!(lane & 8)) {
                            const float gv = v[j];
                            const float hv = silu_fast(gv) * u;
                            const size_t col = (size_t)(row >> 4) * 8 + (lane & 7);
                            if (p.hilo_out) {
                                __half hi, lo;
                                split_hilo(hv, hi, lo);
                                p.out_h[(size_t)(2 * tok) * p.ldh + col] = hi;
                                p.out_h[(size_t)(2 * tok + 1) * p.ldh + col] = lo;
                            } else {
                                p.out_h[(size_t)tok * p.ldh + col] = __float2half_rn(hv);
                            }
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (EPI == TC_ARGMAX) {
        // combine the 4 x MH row quarters of this tile per token (lower row on ties)
        const float2* red = reinterpret_cast<const float2*>(smem + SM.red_off);
        const int HL = p.hilo ? 2 : 1, ttok0 = tok0 / HL;
        for (int t = threadIdx.x; t < BN / HL && ttok0 + t < p.m_tok; t += blockDim.x) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int q = 0; q < 4 * MH; ++q) {
                const float2 e = red[q * BN + t];
                argmax_merge(bv, bi, e.x, __float_as_int(e.y));
            }
            p.best_v[(size_t)rtile * p.m_tok + ttok0 + t] = bv;
            p.best_i[(size_t)rtile * p.m_tok + ttok0 + t] = bi;
        }
    }
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, tmem_cols);
    }
}

// Dequantises a q4s matrix of the device tile layout into row-major fp16 [n_rows][k] with the
// GEMM's rule half(q) * half(scale) (computed as one rounding of the exact fp32 product, which
// is the same value): the operand of the prefill GEMMs, whose tiles then come in by TMA.  One
// thread per (row, 8 consecutive columns): four words of the unit, one 16-byte store.
__global__ void __launch_bounds__(256) dequant_q4s_f16_kernel(const uint8_t* tiles, int n_rows, int K, __half* out) {
    const long long n8 = (long long)n_rows * (K / 8);
    const int n_tiles = n_rows / 16, upt = K / 64;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(i / (K / 8)), j8 = (int)(i % (K / 8));
        const uint8_t* ub = tiles + icua_layout::unit_offset(FMT_Q4S, n_tiles, upt, row >> 4, j8 >> 3);
        const int rt = row & 15, g = rt & 7, up = rt >> 3;
        const int j = j8 & 7, step = j >> 1, hi8 = j & 1;
        const __half s = *reinterpret_cast<const __half*>(ub + 512 + g * 8 + (step >> 1) * 4 + up * 2);
        const float sf = __half2float(s);
        uint32_t o[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(ub + (g * 4 + t) * 16 + step * 4);
            const int sh = hi8 * 8 + up * 4;
            const float a = sf * (float)((int)((w >> sh) & 0xF) - 8);
            const float b = sf * (float)((int)((w >> (16 + sh)) & 0xF) - 8);
            const __half2 hv = __floats2half2_rn(a, b);
            o[t] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        *reinterpret_cast<uint4*>(out + (size_t)row * K + (size_t)j8 * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// q8 counterpart of dequant_q4s_f16_kernel (reference FMT 1 weights): one rounding of
// float(scale) * q, q = u - 128 from the offset-binary byte.
__global__ void __launch_bounds__(256) dequant_q8_f16_kernel(const uint8_t* tiles, int n_rows, int K, __half* out) {
    const long long n8 = (long long)n_rows * (K / 8);
    const int n_tiles = n_rows / 16, upt = K / 64;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(i / (K / 8)), j8 = (int)(i % (K / 8));
        const uint8_t* ub = tiles + icua_layout::unit_offset(FMT_Q8, n_tiles, upt, row >> 4, j8 >> 3);
        const int rt = row & 15, g = rt & 7, up = rt >> 3;
        const int j = j8 & 7, step = j >> 1, hi8 = j & 1;
        const float sf = __half2float(*reinterpret_cast<const __half*>(ub + 1024 + g * 8 + (step >> 1) * 4 + up * 2));
        uint32_t o[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(ub + (step >> 1) * 512 + (g * 4 + t) * 16 +
                                                                  (step & 1) * 8 + hi8 * 4);
            const float a = sf * (float)((int)((w >> (8 * up)) & 0xFF) - 128);
            const float b = sf * (float)((int)((w >> (16 + 8 * up)) & 0xFF) - 128);
            const __half2 hv = __floats2half2_rn(a, b);
            o[t] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        *reinterpret_cast<uint4*>(out + (size_t)row * K + (size_t)j8 * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// Affine q4 counterpart of dequant_q4s_f16_kernel: one rounding of scale * u + bias.
__global__ void __launch_bounds__(256) dequant_q4a_f16_kernel(const uint8_t* tiles, int n_rows, int K, __half* out) {
    const long long n8 = (long long)n_rows * (K / 8);
    const int n_tiles = n_rows / 16, upt = K / 64;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(i / (K / 8)), j8 = (int)(i % (K / 8));
        const uint8_t* ub = tiles + icua_layout::unit_offset(FMT_Q4A, n_tiles, upt, row >> 4, j8 >> 3);
        const int rt = row & 15, g = rt & 7, up = rt >> 3;
        const int j = j8 & 7, step = j >> 1, hi8 = j & 1;
        const __half2 sbh = *reinterpret_cast<const __half2*>(ub + 512 + g * 8 + up * 4);
        const __half2 sc = __half2half2(__low2half(sbh)), bi = __half2half2(__high2half(sbh));
        uint32_t o[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(ub + (g * 4 + t) * 16 + step * 4);
            const int sh = hi8 * 8 + up * 4;
            const __half2 u = __floats2half2_rn((float)((w >> sh) & 0xF), (float)((w >> (16 + sh)) & 0xF));
            const __half2 hv = __hfma2(u, sc, bi);  // the fused path's single rounding of u * scale + bias
            o[t] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        *reinterpret_cast<uint4*>(out + (size_t)row * K + (size_t)j8 * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// Tensor-core tile order: unit (tile, kk) of the slice-major layout moves to
// ((tile / 8) * upt + kk) * 8 + tile % 8, so that a GEMM stage (8 consecutive tiles, one k-block)
// is one contiguous run of 8 units: one bulk copy instead of eight small ones, whose per-request
// cost bounded the fused dequant-GEMM.  One thread per 16 bytes.
__global__ void tc_order_kernel(const uint8_t* src, int fmt, int n_tiles, int upt, uint8_t* dst) {
    const int ub = unit_bytes(fmt), v_per_unit = ub / 16;
    const long long total = (long long)n_tiles * upt * v_per_unit;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const long long unit = i / v_per_unit;
        const int v = (int)(i % v_per_unit);
        const int t8 = (int)(unit % 8);
        const long long rest = unit / 8;
        const int kk = (int)(rest % upt), g8 = (int)(rest / upt);
        const long long so = icua_layout::unit_offset(fmt, n_tiles, upt, g8 * 8 + t8, kk);
        reinterpret_cast<uint4*>(dst + unit * ub)[v] = reinterpret_cast<const uint4*>(src + so)[v];
    }
}

// Split-K finish: sums the Z partial products [Z][m][n] in slice order (deterministic) and applies
// the epilogue of the GEMM that was split: store, residual add, or SwiGLU (gate rows 0..7 and up
// rows 8..15 of each 16-row tile) into fp16.
template <int EPI>
__global__ void __launch_bounds__(256) splitk_finish_kernel(const float* part, int Z, int m, int n, float* out,
                                                            __half* out_h, int hilo_out) {
    pdl_wait();
    pdl_launch_dependents();
    const long long total = (long long)m * n;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        float pz[TC_SPLITK_MAX];
#pragma unroll
        for (int z = 0; z < TC_SPLITK_MAX; ++z) pz[z] = z < Z ? part[(long long)z * total + i] : 0.f;
        float acc = pz[0];
#pragma unroll
        for (int z = 1; z < TC_SPLITK_MAX; ++z)
            if (z < Z) acc += pz[z];
        if (EPI == TC_STORE) {
            out[i] = acc;
        } else if (EPI == TC_RESID) {
            out[i] = out[i] + acc;
        } else {
            const int row = (int)(i % n), r = row & 15;
            if (r < 8) {
                float up = part[i + 8];
                for (int z = 1; z < Z; ++z) up += part[(long long)z * total + i + 8];
                const long long tok = i / n;
                const float hv = (acc / (1.0f + expf(-acc))) * up;
                const long long col = (row >> 4) * 8 + r;
                if (hilo_out) {
                    __half hi, lo;
                    split_hilo(hv, hi, lo);
                    out_h[(2 * tok) * (n / 2) + col] = hi;
                    out_h[(2 * tok + 1) * (n / 2) + col] = lo;
                } else {
                    out_h[tok * (n / 2) + col] = __float2half_rn(hv);
                }
            }
        }
    }
}

// Split-K finish of a residual GEMM over rows of H = 2048 fused with the RMSNorm that follows it:
// one CTA per token row adds the Z partial products to the residual row in slice order (the sums
// of splitk_finish_kernel<TC_RESID>), then writes the normalised fp16 row with the arithmetic of
// rmsnorm_rows_f16_kernel (same element mapping and reduction order), so that the pair of kernels
// it replaces and this one give the same bits.
__global__ void __launch_bounds__(256) splitk_resid_norm_kernel(const float* part, int Z, int m, float* x,
                                                                const float* w, __half* out, int hilo) {
    __shared__ float red[8];
    pdl_wait();
    pdl_launch_dependents();
    const int i = blockIdx.x, tid = threadIdx.x;
    if (i >= m) return;
    const long long total = (long long)m * H;
    float4* xr = reinterpret_cast<float4*>(x + (size_t)i * H);
    const float4* pr = reinterpret_cast<const float4*>(part + (size_t)i * H);
    // every load first (independent, in flight together), then the sums in slice order
    float4 za[TC_SPLITK_MAX], zb[TC_SPLITK_MAX];
#pragma unroll
    for (int z = 0; z < TC_SPLITK_MAX; ++z) {
        if (z < Z) {
            const float4* pz = reinterpret_cast<const float4*>(part + z * total + (size_t)i * H);
            za[z] = pz[tid];
            zb[z] = pz[tid + 256];
        }
    }
    const float4 xa = xr[tid], xb = xr[tid + 256];
    float4 a = za[0], b = zb[0];
#pragma unroll
    for (int z = 1; z < TC_SPLITK_MAX; ++z) {
        if (z < Z) {
            a.x += za[z].x; a.y += za[z].y; a.z += za[z].z; a.w += za[z].w;
            b.x += zb[z].x; b.y += zb[z].y; b.z += zb[z].z; b.w += zb[z].w;
        }
    }
    a = make_float4(xa.x + a.x, xa.y + a.y, xa.z + a.z, xa.w + a.w);
    b = make_float4(xb.x + b.x, xb.y + b.y, xb.z + b.z, xb.w + b.w);
    xr[tid] = a;
    xr[tid + 256] = b;
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
    store_norm_row(out, i, tid, a, b, r, wa, wb, hilo != 0);
}

}  // namespace icua
