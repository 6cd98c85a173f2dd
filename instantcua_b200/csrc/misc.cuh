// Small kernels around the decode step: prompt cursor advance, bit-exact dequantisation of the
// tile layout, KV cache fill.
#pragma once
#include "common.cuh"
#include "gemv.cuh"

namespace icua {

// Moves the prompt cursor after a prompt row that needs no logits (prefill token), the
// counterpart of `st->pos += st->n` in the reference commit (Shaders.swift:1537).
__global__ void advance_kernel(DevState* st) {
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x == 0 && !st->done) {
        st->pos += 1;
        st->prompt_idx += 1;
    }
}

// Loop state of one host-driven decode step (icua_decode_step), written by one launch whose
// arguments carry the host values instead of one host-to-device copy per field: the input token,
// the step's output slot and a budget of one token, no prompt rows left, logits kept; passes of
// grammar-commit engines carry one token and force none.
__global__ void step_head_kernel(DevState* st, int step, int cur_token, int grammar) {
    if (threadIdx.x != 0) return;
    st->step = step;
    st->done = 0;
    st->max_steps = step + 1;
    st->cur_token = cur_token;
    st->prompt_idx = 1 << 30;
    st->write_logits = 1;
    if (grammar) {
        st->n_tok = 1;
        st->cur_token2 = 0;
        st->grammar = 0;
    }
}

template <int FMT>
__global__ void dequant_kernel(const uint8_t* tiles, int n_rows, int K, float* out) {
    const long long total = (long long)n_rows * K;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(i / K), k = (int)(i % K);
        out[i] = FMT == FMT_Q4S ? q4s_tile_value(tiles, n_rows / 16, K, row, k) : q8_tile_value(tiles, n_rows / 16, K, row, k);
    }
}

// Counter-based N(0,1) (splitmix64 hash + Box-Muller) for filling a long KV cache on the device.
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

template <typename KVT>
__global__ void kv_fill_random_kernel(KVT* kc, KVT* vc, int n_layers, int max_ctx, int n_pos, uint64_t seed) {
    const long long per_layer = (long long)NKV * n_pos * HD;
    const long long total = (long long)n_layers * per_layer;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int l = (int)(i / per_layer);
        long long r = i % per_layer;
        const int h = (int)(r / ((long long)n_pos * HD));
        r %= (long long)n_pos * HD;
        const int p = (int)(r / HD), d = (int)(r % HD);
        const long long dst = (((long long)l * NKV + h) * max_ctx + p) * HD + d;
        const uint64_t a = splitmix64(seed ^ (uint64_t)(2 * i)), b = splitmix64(seed ^ (uint64_t)(2 * i + 1));
        const float u1 = ((float)(a >> 40) + 1.0f) * (1.0f / 16777217.0f);
        const float u2 = (float)(b >> 40) * (1.0f / 16777216.0f);
        const float rad = sqrtf(-2.0f * logf(u1));
        kc[dst] = float_to_kv<KVT>(rad * cosf(6.283185307179586f * u2));
        vc[dst] = float_to_kv<KVT>(rad * sinf(6.283185307179586f * u2));
    }
}

}  // namespace icua
