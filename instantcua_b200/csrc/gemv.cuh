// Batch-1 dequant-GEMV for the decode step (q4s / q8 weights, fp32 activations).
//
// Replaces the reference's dot64_row / reduce8 / chunk64_norm GEMV family and the kernels built
// on it: k_attn_in's QKV projection (Shaders.swift:714-834), k_o_proj (1293-1337), k_mlp_in
// (1342-1393), k_mlp_out (1397-1448) and k_lm_head + k_commit (1452-1571).
//
// Design (B200):
// * Weights live in a tile layout (16 rows x 64 columns per "unit") whose bytes are exactly the
//   A-operand registers of four mma.sync.m16n8k16 per warp.  int4 / int8 codes are unpacked by
//   masking into fp16 *subnormal* integers (u * 2^-24), so the tensor core multiplies exact
//   integers; the 2^24 factor, the row scale and the code offset are applied in fp32 per group.
// * Activations are fp32 split into fp16 hi + lo parts that occupy two B columns, so the dot
//   product keeps ~22 bits of the activation and accumulates in fp32.
// * Every warp is an independent worker over a contiguous range of units with its own ring of
//   shared-memory slots filled by 1-D bulk copies (cp.async.bulk + mbarrier).  The first slots are
//   requested before griddepcontrol.wait, so weight streaming overlaps the previous kernel.
// * Tiles split between workers are reduced by the last arriving worker in a fixed order
//   (deterministic), with an atomic counter per tile; no spin waits.
#pragma once
#include "common.cuh"

namespace icua {

enum InMode : int { IN_F32 = 0, IN_BF16 = 1, IN_EMBED = 2 };
enum Epi : int { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_LOGITS = 3 };

struct GemvParams {
    const uint8_t* w;        // tile-packed units
    long long n_units;       // (n_rows / 16) * upt
    int n_rows, k, upt;      // upt = k / 64
    int slot_units, n_slots; // per-warp ring geometry
    // input vector
    int in_mode;
    const void* x;           // IN_F32 / IN_BF16 input [k]
    const float* norm_w;     // RMSNorm weight [k] or nullptr
    // IN_EMBED sources
    const uint8_t* embed;    // q8 tile-packed embedding [vocab, 2048]
    const int* prompt;       // prompt tokens of the session
    const float* pooler;     // visual rows [n_vis, 2048] or nullptr
    float* x_resid;          // residual stream; written by CTA 0 in IN_EMBED, updated by EPI_RESID
    // epilogue
    float* out;              // EPI_STORE: y [n_rows]; EPI_SWIGLU: h [n_rows / 2]
    const float* deepstack;  // EPI_RESID: [n_vis, 2048] for this layer, or nullptr
    float* logits;           // EPI_LOGITS: [vocab]
    float* cta_best_v;       // EPI_LOGITS: [gridDim.x]
    int* cta_best_i;
    unsigned* cta_done;      // EPI_LOGITS: grid completion counter
    int* out_tokens;         // EPI_LOGITS: committed tokens of the call
    float* step_logits;      // EPI_LOGITS: optional per-step logits capture [max_steps][vocab]
    // scratch
    float* partials;         // [n_workers * 2 * 16]
    unsigned* tile_cnt;      // [n_tiles]
    DevState* st;            // nullptr for standalone GEMV
};

struct GemvSmem {
    int k, n_slots, slot_units, ub;
    __host__ __device__ int xfrag_bytes() const { return (k / 16) * 4 * 2 * 8; }
    __host__ __device__ int xsum_off() const { return xfrag_bytes(); }
    __host__ __device__ int red_off() const { return xsum_off() + (k / 32) * 4; }
    __host__ __device__ int bars_off() const { return ((red_off() + 64 * 4) + 15) & ~15; }
    __host__ __device__ int ring_off() const { return ((bars_off() + 8 * n_slots * 8) + 127) & ~127; }
    __host__ __device__ int ring_warp_bytes() const { return n_slots * slot_units * ub; }
    __host__ __device__ int total() const { return ring_off() + 8 * ring_warp_bytes(); }
};

// fp32 value of embedding element (row, k) from the q8 tile layout (same bytes the lm_head
// streams).  Exact: float(scale) * (u - 128).
__device__ __forceinline__ float q8_tile_value(const uint8_t* tiles, int row, int k) {
    const int upt = H / UNIT_K;
    const long long unit = (long long)(row >> 4) * upt + (k >> 6);
    const uint8_t* ub = tiles + unit * Q8_UNIT_BYTES;
    const int rt = row & 15, gq = rt & 7, up = rt >> 3;
    const int kin = k & 63, step = kin >> 4, kk = kin & 15;
    const int t = (kk & 7) >> 1, odd = kk & 1, hi8 = kk >> 3;
    const int lane = gq * 4 + t;
    const int word = (step & 1) * 2 + hi8;  // within the lane's 16 B group
    const uint8_t* wp = ub + (step >> 1) * 512 + lane * 16 + word * 4;
    const int u = wp[odd * 2 + up];
    const __half2 s2 = *reinterpret_cast<const __half2*>(ub + 1024 + gq * 8 + (kin >> 5) * 4);
    const float s = up ? __high2float(s2) : __low2float(s2);
    return s * (float)(u - 128);
}

// Writes the fp16 hi/lo B fragments of x (optionally RMS-normalised) and the per-32 group sums.
// All threads of the CTA take part; ends with __syncthreads.
__device__ void gemv_prepare_x(const GemvParams& p, uint8_t* smem, const GemvSmem& L) {
    const int K = p.k;
    const int tid = threadIdx.x;
    uint2* xfrag = reinterpret_cast<uint2*>(smem);
    float* xsum = reinterpret_cast<float*>(smem + L.xsum_off());
    float* red = reinterpret_cast<float*>(smem + L.red_off());

    // Source row for IN_EMBED (prompt token, visual row or the last generated token).
    const float* vis_row = nullptr;
    int tok = 0;
    if (p.in_mode == IN_EMBED) {
        const DevState* st = p.st;
        const int idx = st->prompt_idx;
        if (idx < st->prompt_len) {
            tok = p.prompt[idx];
            const int v = idx - st->vis_offset;
            if (tok == IMAGE_PAD_ID && st->vis_offset >= 0 && p.pooler != nullptr && v >= 0 && v < st->n_vis)
                vis_row = p.pooler + (long long)v * H;
        } else {
            tok = st->cur_token;
        }
    }
    auto load = [&](int k) -> float {
        if (p.in_mode == IN_F32) return reinterpret_cast<const float*>(p.x)[k];
        if (p.in_mode == IN_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.x)[k]);
        return vis_row ? vis_row[k] : q8_tile_value(p.embed, tok, k);
    };

    const int npairs = K / 4;  // (k16 step, t) pairs
    float scale = 1.0f;
    if (p.norm_w != nullptr) {
        float ss = 0.f;
        for (int q = tid; q < npairs; q += blockDim.x) {
            const int s = q >> 2, t = q & 3, k0 = s * 16 + 2 * t;
            const float a = load(k0), b = load(k0 + 1), c = load(k0 + 8), d = load(k0 + 9);
            ss += a * a + b * b + c * c + d * d;
        }
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        __syncthreads();
        if (tid < 32) {
            float v = tid < (int)(blockDim.x >> 5) ? red[tid] : 0.f;
            v = warp_sum(v);
            if (tid == 0) red[32] = 1.0f / sqrtf(v / (float)K + EPS);
        }
        __syncthreads();
        scale = red[32];
    }
    for (int q = tid; q < npairs; q += blockDim.x) {
        const int s = q >> 2, t = q & 3, k0 = s * 16 + 2 * t;
        const int kk[4] = {k0, k0 + 1, k0 + 8, k0 + 9};
        __half hi[4], lo[4];
        float gsum = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float v = load(kk[i]);
            if (p.in_mode == IN_EMBED && blockIdx.x == 0) p.x_resid[kk[i]] = v;
            if (p.norm_w != nullptr) v = v * scale * p.norm_w[kk[i]];
            hi[i] = __float2half_rn(v);
            lo[i] = __float2half_rn(v - __half2float(hi[i]));
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

// One 16x64 unit: accumulates rows g (acc0) and g+8 (acc1) of the current tile.
template <int FMT>
__device__ __forceinline__ void gemv_unit(const uint8_t* ub, int kk, const uint2* xfrag, const float* xsum, int lane,
                                          float& acc0, float& acc1) {
    const int g = lane >> 2, t = lane & 3;
    const uint2 sc = *reinterpret_cast<const uint2*>(ub + unit_wbytes(FMT) + g * 8);
    uint32_t wq[8];
    if (FMT == FMT_Q4S) {
        const uint4 w = *reinterpret_cast<const uint4*>(ub + lane * 16);
        wq[0] = w.x; wq[1] = w.y; wq[2] = w.z; wq[3] = w.w;
    } else {
        const uint4 w0 = *reinterpret_cast<const uint4*>(ub + lane * 16);
        const uint4 w1 = *reinterpret_cast<const uint4*>(ub + 512 + lane * 16);
        wq[0] = w0.x; wq[1] = w0.y; wq[2] = w0.z; wq[3] = w0.w;
        wq[4] = w1.x; wq[5] = w1.y; wq[6] = w1.z; wq[7] = w1.w;
    }
#pragma unroll
    for (int grp = 0; grp < 2; ++grp) {
        float d[4];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int step = grp * 2 + i;
            uint32_t a[4];
            if (FMT == FMT_Q4S) {
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
            const uint2 b = xfrag[((kk * 4 + step) * 4 + t) * 2 + (g & 1)];
            if (i == 0)
                mma_16816_zero(d, a, b.x, b.y);
            else
                mma_16816(d, a, b.x, b.y);
        }
        const __half2 s2 = *reinterpret_cast<const __half2*>(grp == 0 ? &sc.x : &sc.y);
        const float sg = __low2float(s2), sg8 = __high2float(s2);
        const float X = xsum[kk * 2 + grp];
        // q4s: rows g+8 carry an extra x16 from the nibble position; q8: none.
        const float f0 = 16777216.0f;                                   // 2^24
        const float f1 = (FMT == FMT_Q4S) ? 1048576.0f : 16777216.0f;  // 2^20 or 2^24
        const float off = (FMT == FMT_Q4S) ? 8.0f : 128.0f;
        acc0 = fmaf(sg * f0, d[0] + d[1], acc0);
        acc0 = fmaf(-off * sg, X, acc0);
        acc1 = fmaf(sg8 * f1, d[2] + d[3], acc1);
        acc1 = fmaf(-off * sg8, X, acc1);
    }
}

__device__ __forceinline__ long long worker_start(long long w, long long U, long long W) { return w * U / W; }
// Worker whose range contains unit x: the largest w with start(w) <= x.
__device__ __forceinline__ long long worker_of(long long x, long long U, long long W) {
    return ((x + 1) * W + U - 1) / U - 1;
}

template <int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvParams& p, long long tile, float v0, float v1, int lane,
                                              float& best_v, int& best_i) {
    const int g = lane >> 2, t = lane & 3;
    const int r0 = (int)(tile * 16) + g, r1 = r0 + 8;
    if (EPI == EPI_STORE) {
        if (t == 0) {
            p.out[r0] = v0;
            p.out[r1] = v1;
        }
    } else if (EPI == EPI_RESID) {
        if (t == 0) {
            float a0 = v0, a1 = v1;
            if (p.deepstack != nullptr) {
                const DevState* st = p.st;
                const int v = st->prompt_idx - st->vis_offset;
                if (st->prompt_idx < st->prompt_len && st->vis_offset >= 0 && v >= 0 && v < st->n_vis) {
                    a0 += p.deepstack[(long long)v * H + r0];
                    a1 += p.deepstack[(long long)v * H + r1];
                }
            }
            p.x_resid[r0] += a0;
            p.x_resid[r1] += a1;
        }
    } else if (EPI == EPI_SWIGLU) {
        // tile rows 0..7 are gate units, rows 8..15 the matching up units
        if (t == 0) p.out[tile * 8 + g] = (v0 / (1.0f + expf(-v0))) * v1;
    } else {  // EPI_LOGITS
        if (t == 0) {
            if (p.st->write_logits) {
                p.logits[r0] = v0;
                p.logits[r1] = v1;
            }
            if (p.step_logits != nullptr) {
                float* sl = p.step_logits + (long long)p.st->step * p.n_rows;
                sl[r0] = v0;
                sl[r1] = v1;
            }
        }
        argmax_merge(best_v, best_i, v0, r0);
        argmax_merge(best_v, best_i, v1, r1);
    }
}

template <int FMT, int EPI>
__global__ void __launch_bounds__(256, 2) gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const GemvSmem L{p.k, p.n_slots, p.slot_units, unit_bytes(FMT)};
    const int UB = L.ub;
    const uint2* xfrag = reinterpret_cast<const uint2*>(smem);
    const float* xsum = reinterpret_cast<const float*>(smem + L.xsum_off());
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars_off()) + warp * p.n_slots;
    uint8_t* ring = smem + L.ring_off() + warp * L.ring_warp_bytes();

    const long long U = p.n_units;
    const long long W = (long long)gridDim.x * 8;
    const long long wid = (long long)blockIdx.x * 8 + warp;
    const long long u_begin = worker_start(wid, U, W), u_end = worker_start(wid + 1, U, W);
    const int SU = p.slot_units, NS = p.n_slots;
    const int n_chunks = (int)((u_end - u_begin + SU - 1) / SU);

    auto issue = [&](int c) {
        const long long u0 = u_begin + (long long)c * SU;
        const long long n = min((long long)SU, u_end - u0);
        const uint32_t bytes = (uint32_t)(n * UB);
        uint64_t* bar = &bars[c % NS];
        mbar_expect_tx(bar, bytes);
        bulk_g2s(ring + (c % NS) * SU * UB, p.w + u0 * UB, bytes, bar);
    };

    // Prologue: weights do not depend on the previous kernel, request them before waiting.
    if (lane == 0) {
        for (int s = 0; s < NS; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        for (int c = 0; c < min(NS, n_chunks); ++c) issue(c);
    }
    __syncwarp();

    pdl_wait();
    pdl_launch_dependents();

    const bool skip = (p.st != nullptr) && (*(volatile int*)&p.st->done != 0);
    if (skip) {
        // drain the copies already requested before leaving
        for (int c = 0; c < min(NS, n_chunks); ++c) mbar_wait_bounded(&bars[c % NS], 0);
        return;
    }

    gemv_prepare_x(p, smem, L);

    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    float acc0 = 0.f, acc1 = 0.f;
    long long cur_tile = -1;
    const long long first_tile = u_begin / p.upt;
    bool failed = false;

    auto flush = [&](long long tile) {
        const bool whole = tile * p.upt >= u_begin && (tile + 1) * p.upt <= u_end;
        if (whole) {
            gemv_epilogue<EPI>(p, tile, acc0, acc1, lane, best_v, best_i);
            return;
        }
        const int g = lane >> 2, t = lane & 3;
        const int slot = (tile == first_tile) ? 0 : 1;
        if (t == 0) {
            p.partials[(wid * 2 + slot) * 16 + g] = acc0;
            p.partials[(wid * 2 + slot) * 16 + g + 8] = acc1;
            __threadfence();
        }
        __syncwarp();
        const long long wf = worker_of(tile * p.upt, U, W);
        const long long wl = worker_of((tile + 1) * p.upt - 1, U, W);
        unsigned old = 0;
        if (lane == 0) old = atomicAdd(&p.tile_cnt[tile], 1u);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == (unsigned)(wl - wf)) {
            __threadfence();
            float s0 = 0.f, s1 = 0.f;
            for (long long w2 = wf; w2 <= wl; ++w2) {
                const int sl = (tile == worker_start(w2, U, W) / p.upt) ? 0 : 1;
                s0 += __ldcg(&p.partials[(w2 * 2 + sl) * 16 + g]);
                s1 += __ldcg(&p.partials[(w2 * 2 + sl) * 16 + g + 8]);
            }
            if (lane == 0) p.tile_cnt[tile] = 0;
            gemv_epilogue<EPI>(p, tile, s0, s1, lane, best_v, best_i);
        }
    };

    for (int c = 0; c < n_chunks; ++c) {
        const int slot = c % NS;
        if (!mbar_wait_bounded(&bars[slot], (uint32_t)((c / NS) & 1))) {
            if (lane == 0 && p.st) atomicOr(&p.st->error, ERR_WAIT_GEMV);
            failed = true;
            break;
        }
        const uint8_t* base = ring + slot * SU * UB;
        const long long u0 = u_begin + (long long)c * SU;
        const int nu = (int)min((long long)SU, u_end - u0);
        for (int j = 0; j < nu; ++j) {
            const long long u = u0 + j;
            const long long tile = u / p.upt;
            const int kk = (int)(u - tile * p.upt);
            if (tile != cur_tile) {
                if (cur_tile >= 0) flush(cur_tile);
                cur_tile = tile;
                acc0 = acc1 = 0.f;
            }
            gemv_unit<FMT>(base + j * UB, kk, xfrag, xsum, lane, acc0, acc1);
        }
        __syncwarp();
        if (lane == 0 && c + NS < n_chunks) {
            fence_proxy_async_smem();
            issue(c + NS);
        }
    }
    if (!failed && cur_tile >= 0) flush(cur_tile);

    if (EPI == EPI_LOGITS) {
        __shared__ float bv_s[8];
        __shared__ int bi_s[8];
        __shared__ unsigned last_s;
        warp_argmax(best_v, best_i);
        if (lane == 0) {
            bv_s[warp] = best_v;
            bi_s[warp] = best_i;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float bv = bv_s[0];
            int bi = bi_s[0];
            for (int w2 = 1; w2 < 8; ++w2) argmax_merge(bv, bi, bv_s[w2], bi_s[w2]);
            p.cta_best_v[blockIdx.x] = bv;
            p.cta_best_i[blockIdx.x] = bi;
            __threadfence();
            last_s = atomicAdd(p.cta_done, 1u);
        }
        __syncthreads();
        if (last_s == gridDim.x - 1) {
            __threadfence();
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int c2 = threadIdx.x; c2 < (int)gridDim.x; c2 += blockDim.x)
                argmax_merge(bv, bi, __ldcg(&p.cta_best_v[c2]), __ldcg(&p.cta_best_i[c2]));
            warp_argmax(bv, bi);
            if (lane == 0) {
                bv_s[warp] = bv;
                bi_s[warp] = bi;
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                for (int w2 = 1; w2 < 8; ++w2) argmax_merge(bv_s[0], bi_s[0], bv_s[w2], bi_s[w2]);
                const int tok = bi_s[0];
                DevState* st = p.st;
                *p.cta_done = 0;
                // commit (reference k_commit, Shaders.swift:1536-1547, without the grammar pairs)
                st->pos += 1;
                if (st->prompt_idx < st->prompt_len) st->prompt_idx += 1;
                p.out_tokens[st->step] = tok;
                st->step += 1;
                st->cur_token = tok;
                const bool stop = (st->stop_on_eos && (tok == st->eos0 || tok == st->eos1)) || st->step >= st->max_steps;
                if (stop) st->done = 1;
            }
        }
    }
}

}  // namespace icua
