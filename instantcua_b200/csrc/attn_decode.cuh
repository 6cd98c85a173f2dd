// Decode attention: per-head QK RMSNorm + RoPE + KV append fused with split-K GQA flash-decode.
//
// Replaces the tail of the reference k_attn_in (per-head RMSNorm(128), rotate-half RoPE from the
// cos/sin table, fp16 K/V write at `pos`, Shaders.swift:790-834) and k_attention (softmax over
// the whole context in threadgroup memory, context <= 2048, Shaders.swift:1219-1289).
//
// Design (B200): one CTA per (kv head, split) pair, so the two query heads of a GQA group share
// every K/V byte read.  The static positions [0, pos) of a split are streamed into a ring of
// shared-memory stages with 1-D bulk copies; the first stages are requested before
// griddepcontrol.wait (the cache rows do not depend on the previous kernel).  The new position
// is computed in the CTA from the QKV projection output, rounded to the cache type exactly as it
// is stored, and the last split folds it in.  Split results (running max, sum, output) are
// combined by the last arriving CTA of each kv head in split order (deterministic); no spin
// waits.  Context length is bounded only by the cache allocation.
#pragma once
#include "common.cuh"

namespace icua {

constexpr int ATT_CH = 32;      // positions per stage
constexpr int ATT_STAGES = 4;
constexpr int ATT_PART = 4 + 2 * HD;  // m[2], l[2], o[2][128]

template <typename KVT>
struct AttnParams {
    const float* qkv;        // raw projection [4096]: q(2048) | k(1024) | v(1024)
    const float* q_norm;     // [128]
    const float* k_norm;     // [128]
    const float2* rope;      // [max_ctx][64] (cos, sin) per cache slot
    KVT* kc;                 // this layer: [NKV][max_ctx][128]
    KVT* vc;
    int max_ctx;
    int n_split;
    float* attn_out;         // [2048]
    float* part;             // scratch [NKV][n_split][ATT_PART]
    unsigned* cnt;           // scratch [NKV]
    DevState* st;
};

template <typename KVT>
struct AttnSmem {
    static constexpr int stage_bytes = 2 * ATT_CH * HD * (int)sizeof(KVT);
    static constexpr int ring_off = 0;
    static constexpr int new_off = ATT_STAGES * stage_bytes;                 // K,V of the new position
    static constexpr int q_off = new_off + 2 * HD * (int)sizeof(KVT);        // float q[2][128]
    static constexpr int kv_off = q_off + 2 * HD * 4;                        // float k[128], v[128] scratch
    static constexpr int sc_off = kv_off + 2 * HD * 4;                       // float sc[2][ATT_CH]
    static constexpr int ml_off = sc_off + 2 * ATT_CH * 4;                   // float m[2], l[2], corr[2], red[8]
    static constexpr int red_off = ml_off + 16 * 4;                          // float red[8][2][128]
    static constexpr int bars_off = red_off + 8 * 2 * HD * 4;
    static constexpr int total = bars_off + ATT_STAGES * 8 + 16;
};

// Processes `n` positions whose K rows start at Ks and V rows at Vs (row stride 128).
template <typename KVT>
__device__ __forceinline__ void attn_chunk(const KVT* Ks, const KVT* Vs, int n, const float (&qr)[2][16], float* sc,
                                           float* ml, float (&acc)[2][4]) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // scores: warp w covers positions 4w..4w+3; lane = (p_sub, dpart) with 16 dims per lane
    {
        const int pp = warp * 4 + (lane >> 3), dp = lane & 7;
        float s0 = 0.f, s1 = 0.f;
        if (pp < n) {
            const KVT* kr = Ks + pp * HD;
            const uint4 ka = *reinterpret_cast<const uint4*>(kr + 8 * dp);
            const uint4 kb = *reinterpret_cast<const uint4*>(kr + 64 + 8 * dp);
            const KVT* ea = reinterpret_cast<const KVT*>(&ka);
            const KVT* eb = reinterpret_cast<const KVT*>(&kb);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float k0 = kv_to_float(ea[i]), k1 = kv_to_float(eb[i]);
                s0 = fmaf(qr[0][i], k0, s0);
                s0 = fmaf(qr[0][8 + i], k1, s0);
                s1 = fmaf(qr[1][i], k0, s1);
                s1 = fmaf(qr[1][8 + i], k1, s1);
            }
        }
        s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
        s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
        s0 += __shfl_xor_sync(0xffffffffu, s0, 4);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 4);
        if (dp == 0) {
            sc[pp] = pp < n ? s0 : -INFINITY;
            sc[ATT_CH + pp] = pp < n ? s1 : -INFINITY;
        }
    }
    __syncthreads();
    // online softmax: warp h handles query head h
    if (warp < 2) {
        const float v = sc[warp * ATT_CH + lane];
        const float mc = warp_max(v);
        const float m_old = ml[warp];
        const float m_new = fmaxf(m_old, mc);
        const float corr = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
        const float pv = (v == -INFINITY) ? 0.f : expf(v - m_new);
        const float ps = warp_sum(pv);
        sc[warp * ATT_CH + lane] = pv;
        __syncwarp();
        if (lane == 0) {
            ml[warp] = m_new;
            ml[2 + warp] = ml[2 + warp] * corr + ps;
            ml[4 + warp] = corr;
        }
    }
    __syncthreads();
    // P.V: thread (dq = 4 dims, psub = position phase)
    {
        const int dq = tid & 31, ps = tid >> 5;
        const float c0 = ml[4], c1 = ml[5];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            acc[0][i] *= c0;
            acc[1][i] *= c1;
        }
        for (int pp = ps; pp < n; pp += 8) {
            const uint2 vv = *reinterpret_cast<const uint2*>(Vs + pp * HD + 4 * dq);
            const KVT* e = reinterpret_cast<const KVT*>(&vv);
            const float p0 = sc[pp], p1 = sc[ATT_CH + pp];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float vf = kv_to_float(e[i]);
                acc[0][i] = fmaf(p0, vf, acc[0][i]);
                acc[1][i] = fmaf(p1, vf, acc[1][i]);
            }
        }
    }
    __syncthreads();
}

template <typename KVT>
__global__ void __launch_bounds__(256, 2) attn_decode_kernel(const AttnParams<KVT> p) {
    extern __shared__ __align__(128) uint8_t smem[];
    using S = AttnSmem<KVT>;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S_ = p.n_split;
    const int h = blockIdx.x / S_, j = blockIdx.x % S_;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::bars_off);
    float* qs = reinterpret_cast<float*>(smem + S::q_off);
    float* kvs = reinterpret_cast<float*>(smem + S::kv_off);
    float* sc = reinterpret_cast<float*>(smem + S::sc_off);
    float* ml = reinterpret_cast<float*>(smem + S::ml_off);
    float* red = reinterpret_cast<float*>(smem + S::red_off);
    KVT* knew = reinterpret_cast<KVT*>(smem + S::new_off);
    KVT* vnew = knew + HD;

    // The cache position was written by a kernel at least two launches earlier (the commit of
    // the previous step), so it can be read before griddepcontrol.wait.
    const int pos = *(volatile int*)&p.st->pos;
    const long long Ls = pos;
    const int p0 = (int)(Ls * j / S_), p1 = (int)(Ls * (j + 1) / S_);
    const int n_chunks = (p1 - p0 + ATT_CH - 1) / ATT_CH;
    const KVT* kbase = p.kc + (long long)h * p.max_ctx * HD;
    const KVT* vbase = p.vc + (long long)h * p.max_ctx * HD;

    auto issue = [&](int c) {
        const int a = p0 + c * ATT_CH;
        const int n = min(ATT_CH, p1 - a);
        const uint32_t bytes = (uint32_t)(n * HD * sizeof(KVT));
        uint8_t* st = smem + S::ring_off + (c % ATT_STAGES) * S::stage_bytes;
        uint64_t* bar = &bars[c % ATT_STAGES];
        mbar_expect_tx(bar, 2 * bytes);
        bulk_g2s(st, kbase + (long long)a * HD, bytes, bar);
        bulk_g2s(st + ATT_CH * HD * sizeof(KVT), vbase + (long long)a * HD, bytes, bar);
    };
    if (tid == 0) {
        for (int s = 0; s < ATT_STAGES; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        for (int c = 0; c < min(ATT_STAGES, n_chunks); ++c) issue(c);
    }
    __syncthreads();

    pdl_wait();
    pdl_launch_dependents();

    if (*(volatile int*)&p.st->done) {
        for (int c = 0; c < min(ATT_STAGES, n_chunks); ++c) mbar_wait_bounded(&bars[c], 0);
        return;
    }

    // ---- q/k norm + RoPE for the new position (heads 2h, 2h+1 and kv head h) ----------------
    {
        // threads 0..127: element tid of q0, q1, k; threads 128..255: v
        float q0 = 0.f, q1 = 0.f, kk = 0.f;
        if (tid < HD) {
            q0 = p.qkv[(2 * h) * HD + tid];
            q1 = p.qkv[(2 * h + 1) * HD + tid];
            kk = p.qkv[2048 + h * HD + tid];
            float a = warp_sum(q0 * q0), b = warp_sum(q1 * q1), c = warp_sum(kk * kk);
            if (lane == 0) {
                red[warp * 3 + 0] = a;
                red[warp * 3 + 1] = b;
                red[warp * 3 + 2] = c;
            }
        } else {
            const float v = p.qkv[3072 + h * HD + (tid - HD)];
            const KVT vr = float_to_kv<KVT>(v);
            vnew[tid - HD] = vr;
        }
        __syncthreads();
        if (tid < HD) {
            float a = 0.f, b = 0.f, c = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < 4; ++w2) {
                a += red[w2 * 3 + 0];
                b += red[w2 * 3 + 1];
                c += red[w2 * 3 + 2];
            }
            const float ra = 1.0f / sqrtf(a / (float)HD + EPS);
            const float rb = 1.0f / sqrtf(b / (float)HD + EPS);
            const float rc = 1.0f / sqrtf(c / (float)HD + EPS);
            const float qn = p.q_norm[tid], kn = p.k_norm[tid];
            qs[tid] = q0 * ra * qn;
            qs[HD + tid] = q1 * rb * qn;
            kvs[tid] = kk * rc * kn;
        }
        __syncthreads();
        if (tid < 64) {
            const float2 cs = p.rope[(long long)pos * 64 + tid];
            const float scale = 0.08838834764831845f;  // 1 / sqrt(128)
            float a = qs[tid], b = qs[tid + 64];
            const float a0 = (a * cs.x - b * cs.y) * scale, b0 = (b * cs.x + a * cs.y) * scale;
            a = qs[HD + tid];
            b = qs[HD + tid + 64];
            const float a1 = (a * cs.x - b * cs.y) * scale, b1 = (b * cs.x + a * cs.y) * scale;
            a = kvs[tid];
            b = kvs[tid + 64];
            const KVT ka = float_to_kv<KVT>(a * cs.x - b * cs.y);
            const KVT kb = float_to_kv<KVT>(b * cs.x + a * cs.y);
            __syncwarp(0xffffffffu);
            qs[tid] = a0;
            qs[tid + 64] = b0;
            qs[HD + tid] = a1;
            qs[HD + tid + 64] = b1;
            knew[tid] = ka;
            knew[tid + 64] = kb;
        }
        if (tid < 2) {
            ml[tid] = -INFINITY;
            ml[2 + tid] = 0.f;
        }
        __syncthreads();
        if (j == 0 && tid < HD) {
            p.kc[((long long)h * p.max_ctx + pos) * HD + tid] = knew[tid];
            p.vc[((long long)h * p.max_ctx + pos) * HD + tid] = vnew[tid];
        }
    }

    // per-lane query registers for the score phase: dims {8dp..8dp+7} and {64+8dp..}
    float qr[2][16];
    {
        const int dp = lane & 7;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            qr[0][i] = qs[8 * dp + i];
            qr[0][8 + i] = qs[64 + 8 * dp + i];
            qr[1][i] = qs[HD + 8 * dp + i];
            qr[1][8 + i] = qs[HD + 64 + 8 * dp + i];
        }
    }
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    bool failed = false;
    for (int c = 0; c < n_chunks; ++c) {
        const int slot = c % ATT_STAGES;
        if (!mbar_wait_bounded(&bars[slot], (uint32_t)((c / ATT_STAGES) & 1))) {
            if (tid == 0) atomicOr(&p.st->error, ERR_WAIT_ATTN);
            failed = true;
        }
        if (__syncthreads_or(failed)) {
            failed = true;
            break;
        }
        const KVT* Ks = reinterpret_cast<const KVT*>(smem + S::ring_off + slot * S::stage_bytes);
        const KVT* Vs = Ks + ATT_CH * HD;
        const int n = min(ATT_CH, p1 - (p0 + c * ATT_CH));
        attn_chunk<KVT>(Ks, Vs, n, qr, sc, ml, acc);
        if (tid == 0 && c + ATT_STAGES < n_chunks) {
            fence_proxy_async_smem();
            issue(c + ATT_STAGES);
        }
    }
    if (failed) return;
    if (j == S_ - 1) attn_chunk<KVT>(knew, vnew, 1, qr, sc, ml, acc);

    // reduce the 8 position phases and write this split's partial
    {
        const int dq = tid & 31, ps = tid >> 5;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            red[(ps * 2 + 0) * HD + 4 * dq + i] = acc[0][i];
            red[(ps * 2 + 1) * HD + 4 * dq + i] = acc[1][i];
        }
    }
    __syncthreads();
    float* part = p.part + ((long long)h * S_ + j) * ATT_PART;
    {
        const int hh = tid >> 7, d = tid & 127;
        float o = 0.f;
#pragma unroll
        for (int s = 0; s < 8; ++s) o += red[(s * 2 + hh) * HD + d];
        part[4 + hh * HD + d] = o;
        if (tid < 4) part[tid] = ml[tid];
    }
    __threadfence();
    __syncthreads();
    __shared__ unsigned last_s;
    if (tid == 0) last_s = atomicAdd(&p.cnt[h], 1u);
    __syncthreads();
    if (last_s != (unsigned)(S_ - 1)) return;
    __threadfence();
    {
        const int hh = tid >> 7, d = tid & 127;
        const float* base = p.part + (long long)h * S_ * ATT_PART;
        float M = -INFINITY;
        for (int s = 0; s < S_; ++s) M = fmaxf(M, __ldcg(&base[s * ATT_PART + hh]));
        float Lsum = 0.f, O = 0.f;
        for (int s = 0; s < S_; ++s) {
            const float m = __ldcg(&base[s * ATT_PART + hh]);
            const float f = (m == -INFINITY) ? 0.f : expf(m - M);
            Lsum = fmaf(__ldcg(&base[s * ATT_PART + 2 + hh]), f, Lsum);
            O = fmaf(__ldcg(&base[s * ATT_PART + 4 + hh * HD + d]), f, O);
        }
        p.attn_out[(2 * h + hh) * HD + d] = O / Lsum;
        if (tid == 0) p.cnt[h] = 0;
    }
}

}  // namespace icua
