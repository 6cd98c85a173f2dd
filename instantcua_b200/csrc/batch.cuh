// Batched decode (many sessions, one token each per step): the row kernels around the tensor-core
// GEMMs.  Row r of a step belongs to session rows_sess[r]; that session's loop state, output
// tokens and caches are reached by one stride from the engine's contiguous session arrays.
//
// The reference engine decodes one session at a time (Engine.swift:770-796); this is the serving
// path of BASELINE config 4 (64 concurrent sessions per GPU), built from the same step as the
// batch-1 loop: embedding of each session's current token, the 28 layers, the tied lm_head with a
// per-row argmax, and the commit of each row into its own session (reference k_commit,
// Shaders.swift:1501-1547).
#pragma once
#include "common.cuh"
#include "gemv.cuh"

namespace icua {

// x[r] = embedding row of session rows_sess[r]'s current token.  One CTA per row.
__global__ void batch_embed_kernel(const int* rows_sess, const DevState* st_all, const uint8_t* embed, int embed_tiles,
                                   int embed_fmt, float* x) {
    pdl_wait();
    pdl_launch_dependents();
    const int r = blockIdx.x;
    const int tok = st_all[rows_sess[r]].cur_token;
    float* xr = x + (size_t)r * H;
    for (int k = threadIdx.x; k < H; k += blockDim.x) xr[k] = embed_value(embed_fmt, embed, embed_tiles, tok, k);
}

// Reduces row r's lm_head partials (best value and vocabulary row per 128-row tile, lowest row on
// ties) and commits the token to its session exactly as the batch-1 commit does.  One CTA per row.
__global__ void __launch_bounds__(256) batch_commit_kernel(const float* best_v, const int* best_i, int n_tiles,
                                                           int n_rows, const int* rows_sess, DevState* st_all,
                                                           int* out_all, int out_stride, int vocab) {
    pdl_wait();
    pdl_launch_dependents();
    const int r = blockIdx.x;
    DevState* st = st_all + rows_sess[r];
    if (st->done) return;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n_tiles; i += blockDim.x)
        argmax_merge(bv, bi, best_v[(size_t)i * n_rows + r], best_i[(size_t)i * n_rows + r]);
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
        if ((unsigned)tok >= (unsigned)vocab) {  // no finite logit: stop this session
            atomicOr(&st->error, ERR_BAD_TOKEN);
            st->done = 1;
            return;
        }
        st->pos += 1;
        out_all[(size_t)rows_sess[r] * out_stride + st->step] = tok;
        st->step += 1;
        st->cur_token = tok;
        const bool stop = (st->stop_on_eos && (tok == st->eos0 || tok == st->eos1)) || st->step >= st->max_steps;
        if (stop) st->done = 1;
    }
}

}  // namespace icua
