// Shared constants, device state and inline-PTX helpers for the sm_100a kernels.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace icua {

// Qwen3VLTextModel dimensions (reference Sources/Engine/ModelFile.swift:47-59).
constexpr int H = 2048;
constexpr int FF = 6144;
constexpr int NQ = 16;
constexpr int NKV = 8;
constexpr int HD = 128;
constexpr int QKV_ROWS = 4096;
constexpr int GU_ROWS = 12288;
constexpr int IMAGE_PAD_ID = 151655;
constexpr float EPS = 1e-6f;

// Device tile format.  A matrix [N, K] is cut into 16-row tiles and 64-column units; a unit is
// the operand of four m16n8k16 MMAs for one warp.  Units are stored tile-major.
constexpr int UNIT_K = 64;
constexpr int Q4_UNIT_BYTES = 576;   // 512 B nibbles (32 lanes x 16 B) + 64 B scales
constexpr int Q8_UNIT_BYTES = 1088;  // 1024 B bytes (32 lanes x 32 B) + 64 B scales
// FMT_F16: weights already dequantised (row-major fp16, the prefill GEMM operand);
// FMT_Q4A: the reference's affine q4 (codes 0..15, fp16 scale and bias per 64 columns)
enum Fmt { FMT_F16 = 0, FMT_Q8 = 1, FMT_Q4A = 2, FMT_Q4S = 3 };

__host__ __device__ constexpr int unit_bytes(int fmt) {
    return fmt == FMT_Q8 ? Q8_UNIT_BYTES : (fmt == FMT_Q4S || fmt == FMT_Q4A) ? Q4_UNIT_BYTES : 0;
}
__host__ __device__ constexpr int unit_wbytes(int fmt) { return fmt == FMT_Q8 ? 1024 : 512; }

// Device-resident loop state of one session (reference `State`, Shaders.swift:41-54, extended
// with the prompt cursor so that prefill runs through the same step kernels).
struct DevState {
    int pos;          // KV position of the token processed by the current step
    int step;         // tokens committed so far in this call
    int done;         // stop flag: every kernel returns at once when set
    int max_steps;
    int eos0, eos1;
    int stop_on_eos;
    int cur_token;    // input token of the next decode step
    int prompt_idx;   // next prompt row to process (< prompt_len while prefilling)
    int prompt_len;
    int vis_offset;   // prompt row of the first visual token, -1 when none
    int n_vis;
    int write_logits; // lm_head also stores fp32 logits when set
    int error;        // bit flags set by bounded waits that gave up
    int session;
    int n_tok;        // tokens of the current decode pass: 2 after a grammar-forced pair, else 1
    int cur_token2;   // second input token of a 2-token pass (the forced syntax token)
    int grammar;      // grammar-guided 2-token commit applies to this call's commits
};

// Grammar-guided 2-token commit (reference k_commit, Shaders.swift:1497-1571).  After the greedy
// token `tok` is committed as output number `step` (1-based), a deterministic syntax token follows
// it: `open` after one of the `action` tokens when it is the call's first output, `space` after
// `comma`; the next pass then runs both tokens through the model with one weight read.  `close`
// ends the call.  The reference's ids (its Qwen tokenizer: 7 '(', 8 ')', 11 ',', 220 ' ' and eight
// action words) are the defaults; tests substitute ids of a small vocabulary.
struct GrammarRule {
    int n_action;
    int action[8];
    int comma, space, open, close;
};

// The forced token after committing `tok` as output `step`, or -1.
__host__ __device__ inline int grammar_syntax(const GrammarRule& r, int tok, int step) {
    if (tok == r.comma) return r.space;
    if (step == 1)
        for (int i = 0; i < r.n_action && i < 8; ++i)
            if (tok == r.action[i]) return r.open;
    return -1;
}

// ---------------------------------------------------------------------------------------------
// inline PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// 1-D bulk copy global -> shared, completing `bytes` on `bar`.  16-byte aligned, size % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and the caller records an error) when the
// phase did not complete within `limit` polls; try_wait itself suspends for a short,
// hardware-chosen time per poll, so the bound is well above any legitimate copy latency.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t limit = (1u << 22)) {
    for (uint32_t i = 0; i < limit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
    }
    return false;
}

// Bounded wait that sleeps `ns` nanoseconds between polls after the first: for warps that are off
// the critical path, so that their polling does not take issue slots from the thread that is on it.
__device__ __forceinline__ bool mbar_wait_nap(uint64_t* bar, uint32_t parity, uint32_t ns, uint32_t limit = (1u << 22)) {
    if (mbar_try_wait(bar, parity)) return true;
    for (uint32_t i = 0; i < limit; ++i) {
        __nanosleep(ns);
        if (mbar_try_wait(bar, parity)) return true;
    }
    return false;
}

// L2 prefetch plan of a kernel: byte ranges that a later kernel of the step will read (weights,
// cache rows), split evenly over this kernel's CTAs and requested before griddepcontrol.wait, so
// HBM streams ahead of the dependency chain.  Ranges: `n` plain ranges, plus optionally the
// [0, pos) rows of every kv head of one layer's K and V cache.
struct L2Plan {
    const uint8_t* ptr[2];
    uint64_t bytes[2];
    int n;
    const uint8_t* kv_k;     // cache rows of the layer to prefetch, or nullptr
    const uint8_t* kv_v;
    uint64_t kv_head_stride;  // bytes between kv heads (max_ctx * 128 * elem)
    int kv_row_bytes;
};

__device__ __forceinline__ void l2_prefetch_range(const uint8_t* base, uint64_t begin, uint64_t end) {
    begin &= ~uint64_t(15);
    end = (end + 15) & ~uint64_t(15);
    while (begin < end) {
        const uint64_t n = min(end - begin, (uint64_t)(1u << 20));
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + begin), "r"((uint32_t)n) : "memory");
        begin += n;
    }
}

// Issues this CTA's share of the plan (one thread).  `pos` bounds the cache rows.
__device__ __forceinline__ void l2_prefetch_plan(const L2Plan& pl, int pos) {
    const uint64_t G = gridDim.x, c = blockIdx.x;
    for (int i = 0; i < pl.n; ++i) {
        const uint64_t b = pl.bytes[i];
        if (b) l2_prefetch_range(pl.ptr[i], b * c / G, b * (c + 1) / G);
    }
    if (pl.kv_k != nullptr && pos > 0) {
        // 16 ranges (8 kv heads x K, V) of pos rows each, concatenated and split over the CTAs
        const uint64_t per = (uint64_t)pos * pl.kv_row_bytes, total = 16 * per;
        uint64_t a = total * c / G, e = total * (c + 1) / G;
        while (a < e) {
            const uint64_t r = a / per, off = a - r * per, n = min(e - a, per - off);
            const uint8_t* base = (r < 8 ? pl.kv_k : pl.kv_v) + (r & 7) * pl.kv_head_stride;
            l2_prefetch_range(base, off, off + n);
            a += n;
        }
    }
}

// Programmatic dependent launch: wait for the producing grid, then let the next grid start.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// D = A(16x16, row) * B(16x8, col) + 0 with fp16 inputs and fp32 accumulation.
__device__ __forceinline__ void mma_16816_zero(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.0f));
}

__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Argmax combine with the reference tie-break: larger value wins, equal values keep the lower
// index (Shaders.swift:1481-1487, 1517).
__device__ __forceinline__ void argmax_merge(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

__device__ __forceinline__ void warp_argmax(float& bv, int& bi) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, ov, oi);
    }
}

template <typename T>
__device__ __forceinline__ float kv_to_float(T v);
template <>
__device__ __forceinline__ float kv_to_float<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float kv_to_float<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T float_to_kv(float v);
template <>
__device__ __forceinline__ __half float_to_kv<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 float_to_kv<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Error flags written to DevState::error.
// ERR_BAD_TOKEN: a commit found no finite logit (NaN rows leave the argmax without a winner); the
// session stops instead of embedding an id outside the vocabulary on its next step.
enum : int { ERR_WAIT_GEMV = 1, ERR_WAIT_ATTN = 2, ERR_WAIT_PREFILL = 4, ERR_BAD_TOKEN = 8 };

}  // namespace icua
