// Engine host code and C ABI (include/icua.h): weights, KV caches, device loop state, CUDA graphs
// of PDL-chained kernels, prefill / decode drivers.
//
// Counterpart of the reference's Swift Engine (Sources/Engine/Engine.swift): init (54-185),
// prepareMRoPE (254-298), encodeLLMLayer / encodeLMHead / encodeCommit / encodePrefill /
// encodeDecodeStep (476-681) and generateVision's token loop (696-827).  Where the reference
// encodes 142 dispatches per token into a Metal command buffer and batches 8 steps per submit,
// this engine captures `steps_per_graph` decode steps into one CUDA graph whose kernels are
// chained with programmatic dependent launch, so each kernel streams its weights while the
// previous one finishes.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <type_traits>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include <cudaTypedefs.h>

#include "../../include/icua.h"
#include "attn_decode.cuh"
#include "batch.cuh"
#include "decode_mk.cuh"
#include "common.cuh"
#include "gemm_tc.cuh"
#include "gemv.cuh"
#include "misc.cuh"
#include "prefill.cuh"
#include "vision.cuh"
#include "attn_tc.cuh"
#include "prefill_tc.cuh"

namespace icua_host {
uint16_t f32_to_f16_bits(float f);
float f16_bits_to_f32(uint16_t h);
void pack_q4s(int n_rows, int k, const uint8_t* packed, const uint16_t* scales, const int* row_map, uint8_t* out);
void pack_q8(int n_rows, int k, const int8_t* codes, const uint16_t* scales, const int* row_map, uint8_t* out);
void pack_q4a(int n_rows, int k, const uint8_t* packed, const uint16_t* sb, const int* row_map, uint8_t* out);
}  // namespace icua_host

using namespace icua;

namespace {

thread_local std::string g_error;

struct Matrix {
    uint8_t* dev = nullptr;
    uint8_t* tc = nullptr;     // the same matrix in tensor-core tile order (tensor-core GEMMs)
    int fmt = 0, n_rows = 0, k = 0;
    int n_tiles = 0, grid = 0;
    bool stream = false;      // streaming (ring) path; otherwise all tiles of a CTA in one copy
    int n_slots = 1, chunk = 1;
    size_t smem = 0;
    int n_slots2 = 1;  // ring depth and shared memory of the two-token (grammar-commit) kernels
    size_t smem2 = 0;
};

struct Layer {
    Matrix qkv, o, gu, d;
    float *attn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr, *mlp_norm = nullptr;
};

struct Session {
    DevState* st = nullptr;       // device
    int* prompt = nullptr;        // device [max_pass]
    int* out_tokens = nullptr;    // device [max_steps + slack]
    float2* rope = nullptr;       // device [max_ctx][64]
    void* kc = nullptr;           // device [L][NKV][max_ctx][HD]
    void* vc = nullptr;
    // host mirror
    int pos = 0;
    int step = 0;
    int done = 0;
    int rope_delta = 0;
    cudaGraphExec_t g_prefill_tok = nullptr, g_step1 = nullptr, g_stepn = nullptr;
    // system-prompt prefix cache: the tokens before the visual block of the last icua_generate,
    // whose K/V rows [0, prefix.size()) are still in the cache
    std::vector<int> prefix;
    bool prefix_valid = false;
};

}  // namespace

struct icua_engine {
    icua_config cfg{};
    int n_sm = 0;
    int att_split = 16;   // CTAs per kv head in the decode attention
    int att_cluster = 8;  // CTAs per cluster (att_split / att_cluster parts per kv head)
    // batch-1 decode with the o-projection folded into the attention: one cluster of attn_o CTAs per
    // kv head (16 when eight non-portable clusters of 16 fit at once, else 8; 0 = off, the o-proj
    // GEMV launch); ICUA_ATTN_O=0 turns it off
    int attn_o = 0;
    float* o_part = nullptr;  // [NKV][2048] o-proj partial products of the head pairs
    int* host_tok = nullptr;  // pinned host word: the token icua_decode_step returns
    cudaStream_t stream = nullptr;
    std::string err;
    bool failed = false;
    bool uploaded = false;
    std::map<int, std::vector<uint8_t>> staged;
    std::vector<Layer> layers;
    Matrix embed;
    float* final_norm = nullptr;
    // activations
    float *x = nullptr, *qkv = nullptr, *attn = nullptr, *h = nullptr, *logits = nullptr;
    float* pooler = nullptr;
    float* deepstack[3] = {nullptr, nullptr, nullptr};
    float* step_logits = nullptr;
    float* step_logits_host = nullptr;
    int step_logits_cap = 0;
    // intermediate results passed between kernels of a step
    float* att_part = nullptr;    // attention (max, sum, output) parts per kv head
    float* cta_best_v = nullptr;  // lm_head per-CTA argmax partials
    int* cta_best_i = nullptr;
    std::vector<Session> sessions;
    std::vector<void*> allocations;
    unsigned long long device_bytes = 0;  // sum of the allocations' sizes
    int eos0 = 151645, eos1 = 151643, stop_on_eos = 1;
    int prefix_cache = 1;  // reference Engine.usePrefixCache (Engine.swift:40), on by default
    // grammar-guided 2-token commit (reference k_commit): off unless icua_set_grammar_commit
    bool grammar = false;
    GrammarRule rule{8, {3678, 7241, 12476, 10855, 11862, 1339, 1472, 24769}, 11, 220, 7, 8};
    icua_timing timing{};
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
    float inv_freq[64];
    // prefill rows through the tensor-core GEMM (max_pass rows each)
    float *px = nullptr, *pqkv = nullptr;
    void* pq = nullptr;   // prompt-row q in the cache type [max_pass][16][128]
    void* pvt = nullptr;  // V^T of the session's cache slots [8][128][pvt_stride], fp16
    int pvt_stride = 0;
    __half *pxn = nullptr, *pattn = nullptr, *ph = nullptr;
    int* gemm_err = nullptr;                     // error flags of the batched kernels
    float* splitk_part = nullptr;                // split-K partial products of the batched GEMMs
    // prefill: the layer matrices dequantised to fp16, two layers' sets (layer l in set l % 2),
    // filled by a side stream one matrix ahead of the GEMMs
    __half* wscr[2][4] = {{nullptr, nullptr, nullptr, nullptr}, {nullptr, nullptr, nullptr, nullptr}};
    cudaStream_t side = nullptr;
    cudaEvent_t ev_ready[8] = {}, ev_done[8] = {};  // per GEMM of the sequence, mod 8
    // batched step: row groups recorded as parallel chains (second group on `side`); 1 unless
    // ICUA_BATCH_GROUPS=2 (measured within the run-to-run spread at config 4, and each group reads
    // the weights once)
    int batch_groups = 1;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    // sessions (contiguous arrays; Session holds pointers into them)
    DevState* st_all = nullptr;
    int* out_all = nullptr;
    float2* rope_all = nullptr;
    void* kc_all = nullptr;
    void* vc_all = nullptr;
    size_t kv_elems = 0;  // cache elements of one session (all layers, K or V)
    int out_stride = 0;
    // batched decode: row -> session table, lm_head argmax partials, cached graphs
    int* batch_rows = nullptr;
    float* batch_best_v = nullptr;
    int* batch_best_i = nullptr;
    std::vector<int> batch_key;
    int batch_ctx = 0;  // mean cache position of the sessions the batch graphs are recorded for
    cudaGraphExec_t g_batch1 = nullptr, g_batchn = nullptr;
    float* batch_logits = nullptr;  // [rows][vocab] of the last batched step, when requested
    float* batch_logits_buf = nullptr;  // its allocation, kept across disable / enable
    int batch_logits_cap = 0;           // rows the allocation holds
    float* batch_logits_host = nullptr;
    int batch_logits_rows = 0;
    // vision encoder: weights by reference tensor id (fp16 matrices, fp32 vectors), activations
    // for up to vit_np_max patches (allocated at the first encode), the visual rows it left in
    // pooler / deepstack (vis_rows, -1 when none)
    void* vit[ICUA_VIT_TENSORS] = {};
    int vit_count = 0;
    int vit_np_max = 0;
    uint8_t* vrgb = nullptr;
    __half *vpatch = nullptr, *vxn = nullptr, *vq = nullptr, *vk = nullptr, *vattn = nullptr, *vh = nullptr;
    float *vx = nullptr, *vqkv = nullptr;
    float2* vrope = nullptr;
    __half* vvt = nullptr;  // V^T per head [16][64][vit_np_max + 8]
    int vis_rows = -1;
    bool tc_ready = false;  // tensor-core tile order copies made (ensure_tc_order)
    // persistent decode step (decode_mk.cuh): q4s engines run every layer of a step in one
    // cooperative launch; mk is false when the device or configuration cannot (launch chain)
    bool mk = false;
    int mk_S = 0;                                // attention CTAs per kv head
    uint8_t* mk_stream = nullptr;                // CTA weight streams
    unsigned long long* mk_cta_base = nullptr;   // [n_sm]
    MkLayer* mk_layers = nullptr;                // [n_layers]
    unsigned long long* mk_words = nullptr;      // exchange words
    unsigned long long* mk_parts = nullptr;      // attention split parts (exchange words)
    unsigned* mk_cnt = nullptr;                  // CTAs done with the launch, launch epoch
    int* mk_abort = nullptr;
};

namespace {

icua_status fail(icua_engine* e, icua_status s, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (e) e->err = buf;
    g_error = buf;
    return s;
}

#define CK(call)                                                                                   \
    do {                                                                                           \
        cudaError_t _e = (call);                                                                   \
        if (_e != cudaSuccess) return fail(eng, ICUA_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(_e)); \
    } while (0)

icua_status dalloc(icua_engine* eng, void** p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes < 16 ? 16 : bytes);
    if (e != cudaSuccess) return fail(eng, ICUA_ERR_OOM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    eng->allocations.push_back(*p);
    eng->device_bytes += bytes < 16 ? 16 : bytes;
    return ICUA_OK;
}

template <typename T>
icua_status dalloc_t(icua_engine* eng, T** p, size_t count) {
    return dalloc(eng, reinterpret_cast<void**>(p), count * sizeof(T));
}

// Grid, path and shared memory of a GEMV: CTAs own whole 16-row tiles, each warp one K slice of
// every tile.  Up to SMALL_MAX_TILES tiles per CTA the whole weight slice of a warp is one bulk
// copy requested before the kernel waits on its producer; longer matrices stream one tile per
// ring slot.
void setup_matrix(Matrix& m, int fmt, int n_rows, int k, int n_sm) {
    m.fmt = fmt;
    m.n_rows = n_rows;
    m.k = k;
    m.n_tiles = n_rows / 16;
    m.grid = std::min(n_sm, m.n_tiles);
    const int tpc = gemv_tiles_per_cta(m.n_tiles, m.grid);
    const int nw = fmt_slices(fmt), ku = k / 64 / nw;
    m.stream = fmt == FMT_Q8 || tpc > SMALL_MAX_TILES;  // q8 kernels are built for the streaming path only
    // streaming chunk: tiles per bulk copy.  Each copy request has a fixed cost in the copy engine,
    // so the q8 lm_head moves two tiles (8.7 KB) per request
    m.chunk = !m.stream ? tpc : (fmt == FMT_Q8 && k <= 2048 ? 2 : 1);
    // streaming ring depth: up to 4 tiles per warp in flight (~140 KB per SM for the q8 lm_head,
    // enough to cover HBM latency at full bandwidth), as many as fit next to the input vector and
    // the RMSNorm weights
    for (int ntok : {1, 2}) {
        int& slots = ntok == 1 ? m.n_slots : m.n_slots2;
        slots = 1;
        for (int ns : {4, 2, 1}) {
            if (!m.stream && ns > 1) continue;
            GemvSmem L{k, nw, ns, m.chunk, unit_bytes(fmt), ku, tpc, 0, ntok};
            if ((size_t)L.total() + (size_t)k * 4 <= 216 * 1024) {
                slots = ns;
                break;
            }
        }
        GemvSmem L{k, nw, slots, m.chunk, unit_bytes(fmt), ku, tpc, 0, ntok};
        (ntok == 1 ? m.smem : m.smem2) = (size_t)L.total();  // without the RMSNorm weight copy; launch_gemv adds it
    }
}

template <typename Kern, typename... A>
cudaError_t launch(Kern kernel, int grid, int block, size_t smem, cudaStream_t s, bool pdl, A... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <typename Kern, typename P>
cudaError_t launch_cluster(Kern kernel, int grid, int cluster, int block, size_t smem, cudaStream_t s, const P& params) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, params);
}

template <int FMT, int EPI, int KMAX, bool STREAM, int IN, bool DUAL = false>
cudaError_t launch_gemv(const Matrix& m, const GemvParams& p, cudaStream_t s, bool pdl = true) {
    const int nt = fmt_slices(FMT) * 32;
    constexpr bool two = DUAL && EPI != EPI_LOGITS;  // the lm_head of a 2-token pass reads one row
    const size_t smem = (two ? m.smem2 : m.smem) + (p.norm_w != nullptr ? (size_t)m.k * 4 : 0);
    if (m.stream != STREAM || p.in_mode != IN) return cudaErrorInvalidValue;
    GemvParams q = p;
    if (two) q.n_slots = m.n_slots2;
    return launch(gemv_kernel<FMT, EPI, KMAX, STREAM, IN, DUAL>, m.grid, nt, smem, s, pdl, q);
}

// ---- tensor-core GEMM launch ------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// TMA map of an fp16 activation matrix [rows, k] (k contiguous): boxes of 64 columns (128 bytes,
// the swizzle span) x box_rows rows, SWIZZLE_128B, rows past `rows` read as zeros.
bool make_act_map(CUtensorMap* map, const void* base, int rows, int k, int box_rows) {
    auto enc = tensor_map_encoder();
    if (!enc || ((uintptr_t)base & 15) || k % 64 || rows < 1) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)k * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

TcGemmParams tc_params(const Matrix& m, int m_tok, int* err) {
    TcGemmParams p{};
    p.w = m.dev;
    p.wtc = m.tc;
    p.n_rows = m.n_rows;
    p.k = m.k;
    p.n_tiles = m.n_tiles;
    p.upt = m.k / 64;
    p.m_tok = m_tok;
    p.err = err;
    return p;
}

// Tile shape of a GEMM: MH accumulators of 128 weight rows (MH = 2 shares each activation tile
// between 256 rows) and BN tokens per CTA, chosen so that the CTA count fills whole waves of SMs:
// cost = waves x (MMA columns per CTA, at least those of 64 tokens per accumulator since below
// that the weight stream and its dequantisation set the pace, + a fixed per-CTA overhead);
// MH = 1 is charged 10% for its doubled activation traffic; ties go to the wider tile.
struct TcTile {
    int mh, bn;
};

TcTile choose_tc_tile(int n_rows, int m_tok, int n_sm, bool allow_mh2) {
    TcTile best{1, 16};
    double best_cost = 1e30;
    const int bn_max = std::min(256, (m_tok + 15) / 16 * 16);
    for (int mh = 2; mh >= 1; --mh) {
        if ((mh == 2 && !allow_mh2) || n_rows % (TC_BM * mh)) continue;
        for (int bn = bn_max; bn >= 16; bn -= 16) {
            const long tiles = (long)(n_rows / (TC_BM * mh)) * ((m_tok + bn - 1) / bn);
            const long waves = (tiles + n_sm - 1) / n_sm;
            const double cost = (double)waves * (mh * std::max(bn, 64) + 48) * (mh == 1 ? 1.1 : 1.0);
            if (cost < best_cost - 1e-9) {
                best_cost = cost;
                best = TcTile{mh, bn};
            }
        }
    }
    return best;
}

// Tile shape of a GEMM whose A tiles go to tensor memory (one accumulator of up to 256 columns):
// each 64-column stage costs about the same up to 256 activation rows (the MMA-issuing thread, not
// the tensor core, paces it), so the shape minimises waves x (max(bn, 128) + 64).
TcTile choose_tc_tile_atm(int n_rows, int b_rows, int n_sm) {
    TcTile best{1, 16};
    double best_cost = 1e30;
    const int bn_max = std::min(256, (b_rows + 15) / 16 * 16);
    for (int bn = bn_max; bn >= 16; bn -= 16) {
        const long tiles = (long)(n_rows / TC_BM) * ((b_rows + bn - 1) / bn);
        const long waves = (tiles + n_sm - 1) / n_sm;
        const double cost = (double)waves * (std::max(bn, 128) + 64);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = TcTile{1, bn};
        }
    }
    return best;
}

int g_n_sm_cache = 0;

// Launches the GEMM over activations `x` ([rows_alloc, k] fp16) with a TMA map built for the
// chosen tile height.  FMT_F16: the weights are the row-major fp16 matrix w16 (dequantised by
// dequant_q4s_f16_kernel), brought in by TMA as well.
// one_tile: every activation row in one tile (MH = 1, BN = all B rows, at most 128), so that each
// weight tile is dequantised by exactly one CTA (the batched decode GEMMs, which read the weights
// once; the tile search below would trade that for fewer MMA columns).
template <int EPI, int FMT = FMT_Q4S>
cudaError_t launch_tc_gemm(const void* x, int rows_alloc, TcGemmParams p, cudaStream_t s, const __half* w16 = nullptr,
                           int ksplit = 1, bool pdl = false, int max_stages = 8, bool one_tile = false) {
    // rows_alloc: rows of the activation buffer x (B rows: 2 per token with p.hilo)
    const int b_rows = p.hilo ? 2 * p.m_tok : p.m_tok;
    if (p.n_rows % TC_BM || p.k % TC_BK || p.m_tok < 1 || b_rows > rows_alloc) return cudaErrorInvalidValue;
    if (!g_n_sm_cache) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_n_sm_cache, cudaDevAttrMultiProcessorCount, dev);
    }
    const bool atm_ok = FMT != FMT_F16 && p.wtc != nullptr;  // row-order weights: A can go to TMEM
    const TcTile t = (one_tile && b_rows <= 128) ? TcTile{1, (b_rows + 15) / 16 * 16}
                     : atm_ok                    ? choose_tc_tile_atm(p.n_rows, b_rows, g_n_sm_cache)
                                                 : choose_tc_tile(p.n_rows, b_rows, g_n_sm_cache, EPI != TC_ARGMAX);
    p.bn = t.bn;
    CUtensorMap map, wmap;
    if (!make_act_map(&map, x, rows_alloc, p.k, t.bn)) return cudaErrorInvalidValue;
    if (FMT == FMT_F16) {
        if (!w16 || !make_act_map(&wmap, w16, p.n_rows, p.k, TC_BM)) return cudaErrorInvalidValue;
    } else {
        wmap = map;  // unused
    }
    cudaLaunchConfig_t cfg = {};
    if (ksplit > 1 && (EPI != TC_STORE || ksplit > p.k / TC_BK)) return cudaErrorInvalidValue;
    cfg.gridDim = dim3((b_rows + t.bn - 1) / t.bn, p.n_rows / (TC_BM * t.mh), ksplit);
    cfg.blockDim = dim3(TC_THREADS);
    p.max_stages = max_stages;
    const bool atm = tc_a_in_tmem(FMT, p.wtc != nullptr, t.mh, t.bn);
    cfg.dynamicSmemBytes =
        TcLayout(t.bn, t.mh, FMT, EPI == TC_ARGMAX, max_stages, atm, tc_kb(atm, p.k / TC_BK, ksplit)).alloc;
    cfg.stream = s;
    // programmatic dependent launch: only where the weights are not the previous kernel's output
    // (engine matrices); the kernel waits for the previous kernel before its activation loads
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    p.pdl = pdl ? 1 : 0;
    if (t.mh == 2) {
        if constexpr (EPI != TC_ARGMAX) return cudaLaunchKernelEx(&cfg, tc_gemm_kernel<EPI, FMT, 2>, map, wmap, p);
        return cudaErrorInvalidValue;
    }
    return cudaLaunchKernelEx(&cfg, tc_gemm_kernel<EPI, FMT, 1>, map, wmap, p);
}

constexpr int SPLITK_MAX = 8;      // K slices of the batched GEMMs
static_assert(SPLITK_MAX <= TC_SPLITK_MAX && SPLITK_MAX <= ATT_QKV_PARTS_MAX, "finish kernels unroll over the slices");
// Pipeline depth of the batched 4-bit GEMMs: with the A tiles in tensor memory a stage holds only
// the quantised weights and the activation tile in shared memory (12.6 KB at 64 rows), so two CTAs
// (this GEMM's and the next kernel's, programmatic launch) still fit on an SM at this depth.
constexpr int BATCH_STAGES_4BIT = 6;
constexpr int SPLITK_MAX_ROWS = 128;  // split K only for batches of up to this many rows

// Batched-decode GEMM over few rows: when the weight-row tiles alone cannot fill the GPU, K is
// split over up to 8 CTA slices whose partial products a finish kernel sums in slice order
// (deterministic) before the epilogue.
// norm_w / norm_out (TC_RESID): the RMSNorm of the updated residual rows that follows, written
// as fp16 rows; with split K it runs inside the finish kernel.  parts_out (TC_STORE): the caller
// consumes the partial products itself (e->splitk_part, [parts][m][n]); *parts_out = the K split,
// 1 when the GEMM stored its result in p.out.
// x: the first B row of the caller's row group, rows_alloc: B rows from x to the end of the
// buffer; splitk: the group's split-K scratch ([parts][m][n], at most SPLITK_MAX x m_tok x n).
template <int EPI>
cudaError_t batch_gemm(icua_engine* e, const Matrix& m, const void* x, int rows_alloc, float* splitk, TcGemmParams p,
                       cudaStream_t s, const float* norm_w = nullptr, __half* norm_out = nullptr,
                       int* parts_out = nullptr) {
    // the batched step's activations are fp16 hi / lo row pairs (2 max_pass rows per buffer);
    // its SwiGLU output (the down GEMM's input) and the norms after the residual GEMMs are too
    p.hilo = 1;
    if (EPI == TC_SWIGLU) p.hilo_out = 1;
    const int rows = rows_alloc;
    const TcTile t = 2 * p.m_tok <= 128 ? TcTile{1, (2 * p.m_tok + 15) / 16 * 16}
                                        : choose_tc_tile(p.n_rows, 2 * p.m_tok, e->n_sm, true);
    const int tiles = (p.n_rows / (TC_BM * t.mh)) * ((2 * p.m_tok + t.bn - 1) / t.bn);
    int ks = std::min(SPLITK_MAX, e->n_sm / std::max(tiles, 1));
    ks = std::min(ks, p.k / TC_BK / 4);  // at least four k-blocks per slice
    auto run = [&](auto epi_tag, const TcGemmParams& q, int ksplit) -> cudaError_t {
        constexpr int E = decltype(epi_tag)::value;
        if (m.fmt == FMT_F16)
            return launch_tc_gemm<E, FMT_F16>(x, rows, q, s, reinterpret_cast<const __half*>(m.dev), ksplit, true, 3,
                                              true);
        if (m.fmt == FMT_Q8) return launch_tc_gemm<E, FMT_Q8>(x, rows, q, s, nullptr, ksplit, true, 3, true);
        if (m.fmt == FMT_Q4A)
            return launch_tc_gemm<E, FMT_Q4A>(x, rows, q, s, nullptr, ksplit, true, BATCH_STAGES_4BIT, true);
        return launch_tc_gemm<E, FMT_Q4S>(x, rows, q, s, nullptr, ksplit, true, BATCH_STAGES_4BIT, true);
    };
    if (parts_out) *parts_out = 1;
    cudaError_t err;
    if (ks < 2 || p.m_tok > SPLITK_MAX_ROWS) {
        if ((err = run(std::integral_constant<int, EPI>{}, p, 1)) != cudaSuccess) return err;
        if (EPI == TC_RESID && norm_w)
            return launch(rmsnorm_rows_f16_kernel<true>, p.m_tok, 256, 0, s, true, (const float*)p.out, norm_w,
                          p.m_tok, norm_out);
        return cudaSuccess;
    }
    TcGemmParams q = p;
    q.out = splitk;
    q.ldo = p.n_rows;
    q.out_zstride = (long long)p.m_tok * p.n_rows;
    if ((err = run(std::integral_constant<int, TC_STORE>{}, q, ks)) != cudaSuccess) return err;
    if (EPI == TC_STORE && parts_out) {
        *parts_out = ks;
        return cudaSuccess;
    }
    if (EPI == TC_RESID && norm_w && p.n_rows == H)
        return launch(splitk_resid_norm_kernel, p.m_tok, 256, 0, s, true, (const float*)splitk, ks, p.m_tok, p.out,
                      norm_w, norm_out, 1);
    const long long total = (long long)p.m_tok * p.n_rows;
    const int grid = (int)std::min<long long>((total + 255) / 256, 4LL * e->n_sm);
    if ((err = launch(splitk_finish_kernel<EPI>, grid, 256, 0, s, true, (const float*)splitk, ks, p.m_tok, p.n_rows,
                      p.out, p.out_h, p.hilo_out)) != cudaSuccess)
        return err;
    if (EPI == TC_RESID && norm_w)
        return launch(rmsnorm_rows_f16_kernel<true>, p.m_tok, 256, 0, s, true, (const float*)p.out, norm_w, p.m_tok,
                      norm_out);
    return cudaSuccess;
}

cudaError_t launch_dequant_f16(const Matrix& m, __half* out, int n_sm, cudaStream_t s) {
    const long long n8 = (long long)m.n_rows * (m.k / 8);
    const int grid = (int)std::min<long long>((n8 + 255) / 256, 8LL * n_sm);
    if (m.fmt == FMT_Q8)
        return launch(dequant_q8_f16_kernel, grid, 256, 0, s, false, (const uint8_t*)m.dev, m.n_rows, m.k, out);
    if (m.fmt == FMT_Q4A)
        return launch(dequant_q4a_f16_kernel, grid, 256, 0, s, false, (const uint8_t*)m.dev, m.n_rows, m.k, out);
    return launch(dequant_q4s_f16_kernel, grid, 256, 0, s, false, (const uint8_t*)m.dev, m.n_rows, m.k, out);
}

cudaError_t set_smem_attrs() {
    static bool done = false;
    if (done) return cudaSuccess;
    const int big = 220 * 1024;
    cudaError_t e;
    // Every kernel asks for the largest shared-memory carveout: an SM configured for a kernel
    // with a small carveout cannot take the next kernel's CTAs until it drains, which would defeat
    // programmatic dependent launch (the next kernel's weight prefetch overlapping this one).
#define SETA(K)                                                                                           \
    e = cudaFuncSetAttribute(K, cudaFuncAttributeMaxDynamicSharedMemorySize, big);                       \
    if (e != cudaSuccess) return e;                                                                      \
    e = cudaFuncSetAttribute(K, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared); \
    if (e != cudaSuccess) return e;
    SETA((gemv_kernel<FMT_Q4S, EPI_STORE, 2048, false, IN_F32>));
    SETA((gemv_kernel<FMT_Q4S, EPI_STORE, 2048, false, IN_EMBED>));
    SETA((gemv_kernel<FMT_Q4S, EPI_RESID, 2048, false, IN_ATTN>));
    SETA((gemv_kernel<FMT_Q4S, EPI_SWIGLU, 2048, false, IN_F32>));
    SETA((gemv_kernel<FMT_Q4S, EPI_RESID, 6144, false, IN_F32>));
    SETA((gemv_kernel<FMT_Q8, EPI_LOGITS, 2048, true, IN_F32>));
    SETA((gemv_kernel<FMT_Q4S, EPI_STORE, 2048, false, IN_BF16>));
    SETA((gemv_kernel<FMT_Q4S, EPI_STORE, 6144, false, IN_F32>));
    SETA((gemv_kernel<FMT_Q4S, EPI_STORE, 6144, false, IN_BF16>));
    SETA((gemv_kernel<FMT_Q8, EPI_STORE, 2048, true, IN_F32>));
    SETA((gemv_kernel<FMT_Q8, EPI_STORE, 2048, true, IN_BF16>));
    SETA((gemv_kernel<FMT_Q8, EPI_STORE, 2048, true, IN_EMBED>));
    SETA((gemv_kernel<FMT_Q8, EPI_RESID, 2048, true, IN_ATTN>));
    SETA((gemv_kernel<FMT_Q8, EPI_SWIGLU, 2048, true, IN_F32>));
    SETA((gemv_kernel<FMT_Q8, EPI_RESID, 6144, true, IN_F32>));
    SETA((gemv_kernel<FMT_Q4A, EPI_STORE, 2048, false, IN_EMBED>));
    SETA((gemv_kernel<FMT_Q4A, EPI_STORE, 2048, false, IN_F32>));
    SETA((gemv_kernel<FMT_Q4A, EPI_RESID, 2048, false, IN_ATTN>));
    SETA((gemv_kernel<FMT_Q4A, EPI_SWIGLU, 2048, false, IN_F32>));
    SETA((gemv_kernel<FMT_Q4A, EPI_RESID, 6144, false, IN_F32>));
    SETA((gemv_kernel<FMT_Q4A, EPI_LOGITS, 2048, true, IN_F32>));
    SETA((gemv_kernel<FMT_Q4A, EPI_LOGITS, 2048, false, IN_F32>));
    SETA((attn_decode_kernel<__half>));
    SETA((attn_decode_kernel<__nv_bfloat16>));
    // the two-token kernels of grammar-commit engines
    SETA((gemv_kernel<FMT_Q4S, EPI_STORE, 2048, false, IN_F32, true>));
    SETA((gemv_kernel<FMT_Q4S, EPI_STORE, 2048, false, IN_EMBED, true>));
    SETA((gemv_kernel<FMT_Q4S, EPI_RESID, 2048, false, IN_ATTN, true>));
    SETA((gemv_kernel<FMT_Q4S, EPI_SWIGLU, 2048, false, IN_F32, true>));
    SETA((gemv_kernel<FMT_Q4S, EPI_RESID, 6144, false, IN_F32, true>));
    SETA((gemv_kernel<FMT_Q8, EPI_STORE, 2048, true, IN_F32, true>));
    SETA((gemv_kernel<FMT_Q8, EPI_STORE, 2048, true, IN_EMBED, true>));
    SETA((gemv_kernel<FMT_Q8, EPI_RESID, 2048, true, IN_ATTN, true>));
    SETA((gemv_kernel<FMT_Q8, EPI_SWIGLU, 2048, true, IN_F32, true>));
    SETA((gemv_kernel<FMT_Q8, EPI_RESID, 6144, true, IN_F32, true>));
    SETA((gemv_kernel<FMT_Q4A, EPI_STORE, 2048, false, IN_F32, true>));
    SETA((gemv_kernel<FMT_Q4A, EPI_STORE, 2048, false, IN_EMBED, true>));
    SETA((gemv_kernel<FMT_Q4A, EPI_RESID, 2048, false, IN_ATTN, true>));
    SETA((gemv_kernel<FMT_Q4A, EPI_SWIGLU, 2048, false, IN_F32, true>));
    SETA((gemv_kernel<FMT_Q4A, EPI_RESID, 6144, false, IN_F32, true>));
    SETA((gemv_kernel<FMT_Q8, EPI_LOGITS, 2048, true, IN_F32, true>));
    SETA((gemv_kernel<FMT_Q4A, EPI_LOGITS, 2048, true, IN_F32, true>));
    SETA((gemv_kernel<FMT_Q4A, EPI_LOGITS, 2048, false, IN_F32, true>));
    SETA((attn_decode_kernel<__half, true>));
    SETA((attn_decode_kernel<__nv_bfloat16, true>));
    SETA((attn_decode_kernel<__half, false, true>));
    SETA((attn_decode_kernel<__nv_bfloat16, false, true>));
    SETA(commit_kernel);
    SETA(advance_kernel);
    SETA(decode_mk_kernel<__half>);
    SETA(decode_mk_kernel<__nv_bfloat16>);
    SETA(argmax_parts_kernel);
#undef SETA
    for (const void* k :
         {(const void*)tc_gemm_kernel<TC_STORE, FMT_Q4S, 1>, (const void*)tc_gemm_kernel<TC_RESID, FMT_Q4S, 1>,
          (const void*)tc_gemm_kernel<TC_SWIGLU, FMT_Q4S, 1>, (const void*)tc_gemm_kernel<TC_STORE, FMT_Q4S, 2>,
          (const void*)tc_gemm_kernel<TC_RESID, FMT_Q4S, 2>, (const void*)tc_gemm_kernel<TC_SWIGLU, FMT_Q4S, 2>,
          (const void*)tc_gemm_kernel<TC_ARGMAX, FMT_Q8, 1>, (const void*)tc_gemm_kernel<TC_STORE, FMT_F16, 1>,
          (const void*)tc_gemm_kernel<TC_RESID, FMT_F16, 1>, (const void*)tc_gemm_kernel<TC_SWIGLU, FMT_F16, 1>,
          (const void*)tc_gemm_kernel<TC_STORE, FMT_F16, 2>, (const void*)tc_gemm_kernel<TC_RESID, FMT_F16, 2>,
          (const void*)tc_gemm_kernel<TC_SWIGLU, FMT_F16, 2>, (const void*)tc_gemm_kernel<TC_STORE, FMT_Q8, 1>,
          (const void*)tc_gemm_kernel<TC_RESID, FMT_Q8, 1>, (const void*)tc_gemm_kernel<TC_SWIGLU, FMT_Q8, 1>,
          (const void*)tc_gemm_kernel<TC_STORE, FMT_Q8, 2>, (const void*)tc_gemm_kernel<TC_RESID, FMT_Q8, 2>,
          (const void*)tc_gemm_kernel<TC_SWIGLU, FMT_Q8, 2>, (const void*)tc_gemm_kernel<TC_STORE, FMT_Q4A, 1>,
          (const void*)tc_gemm_kernel<TC_RESID, FMT_Q4A, 1>, (const void*)tc_gemm_kernel<TC_SWIGLU, FMT_Q4A, 1>,
          (const void*)tc_gemm_kernel<TC_STORE, FMT_Q4A, 2>, (const void*)tc_gemm_kernel<TC_RESID, FMT_Q4A, 2>,
          (const void*)tc_gemm_kernel<TC_SWIGLU, FMT_Q4A, 2>, (const void*)tc_gemm_kernel<TC_ARGMAX, FMT_Q4A, 1>,
          (const void*)tc_gemm_kernel<TC_ARGMAX, FMT_F16, 1>, (const void*)tc_gemm_kernel<TC_GELU, FMT_F16, 1>,
          (const void*)tc_gemm_kernel<TC_GELU, FMT_F16, 2>}) {
        if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024)) != cudaSuccess)
            return e;
    }
    if ((e = cudaFuncSetAttribute(vit_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  VitAttnSmem::alloc)) != cudaSuccess)
        return e;
    for (const void* k : {(const void*)prefill_attn_tc_kernel<__half>, (const void*)prefill_attn_tc_kernel<__nv_bfloat16>}) {
        if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, PrefillTcSmem::alloc)) != cudaSuccess)
            return e;
    }
    done = true;
    return cudaSuccess;
}

GemvParams base_params(icua_engine* e, const Matrix& m) {
    GemvParams p{};
    p.w = m.dev;
    p.n_rows = m.n_rows;
    p.k = m.k;
    p.upt = m.k / 64;
    p.n_tiles = m.n_tiles;
    p.n_slots = m.n_slots;
    p.chunk = m.chunk;
    p.embed = e->embed.dev;
    p.embed_tiles = e->embed.n_tiles;
    p.embed_fmt = e->embed.fmt;
    return p;
}

// ---- one decode / prefill step ------------------------------------------------------------------
// L2 prefetch two launches ahead: QKV(l) -> O(l) weights, attention(l) -> GU(l), O(l) -> D(l),
// GU(l) -> QKV(l+1), D(l) -> cache rows of layer l+1 (or the lm_head after the last layer).
L2Plan plan_weights(const Matrix& m) {
    L2Plan pl{};
    pl.ptr[0] = m.dev;
    pl.bytes[0] = icua_packed_bytes(m.fmt, m.n_rows, m.k);
    pl.n = 1;
    return pl;
}

L2Plan plan_kv(icua_engine* e, Session& S, int layer) {
    L2Plan pl{};
    const size_t kv_layer = (size_t)NKV * e->cfg.max_context * HD * 2;
    pl.kv_k = reinterpret_cast<const uint8_t*>(S.kc) + kv_layer * layer;
    pl.kv_v = reinterpret_cast<const uint8_t*>(S.vc) + kv_layer * layer;
    pl.kv_head_stride = (uint64_t)e->cfg.max_context * HD * 2;
    pl.kv_row_bytes = HD * 2;
    return pl;
}

// Layer GEMV launch for the engine's weight format: q4s matrices run the whole-tile path, q8
// matrices (reference FMT 1 files) the streaming path.
template <int EPI, int KMAX, int IN, bool DUAL = false>
cudaError_t launch_layer_gemv(const icua_engine* e, const Matrix& m, const GemvParams& p, cudaStream_t s) {
    if (m.fmt == FMT_Q8) return launch_gemv<FMT_Q8, EPI, KMAX, true, IN, DUAL>(m, p, s);
    if (m.fmt == FMT_Q4A) return launch_gemv<FMT_Q4A, EPI, KMAX, false, IN, DUAL>(m, p, s);
    return launch_gemv<FMT_Q4S, EPI, KMAX, false, IN, DUAL>(m, p, s);
}

// DUAL: the kernels of grammar-commit engines (passes of one or two tokens).
// Every layer of one step as one cooperative launch (decode_mk_kernel).
template <typename KVT>
cudaError_t launch_mk(icua_engine* e, Session& S) {
    MkParams<KVT> p{};
    p.stream = e->mk_stream;
    p.cta_base = e->mk_cta_base;
    p.layers = e->mk_layers;
    p.n_layers = e->cfg.n_layers;
    p.S = e->mk_S;
    p.st = S.st;
    p.prompt = S.prompt;
    p.pooler = e->pooler;
    for (int i = 0; i < 3; ++i) p.deepstack[i] = e->deepstack[i];
    p.rope = S.rope;
    p.kc = reinterpret_cast<KVT*>(S.kc);
    p.vc = reinterpret_cast<KVT*>(S.vc);
    p.max_ctx = e->cfg.max_context;
    p.embed = e->embed.dev;
    p.embed_tiles = e->embed.n_tiles;
    p.embed_fmt = e->embed.fmt;
    unsigned long long* w = e->mk_words;
    p.qkv = w;
    p.att = w + 4096;
    p.xmid = w + 6144;
    p.xout = w + 8192;
    p.hbuf = w + 10240;
    p.parts = e->mk_parts;
    p.fin = e->mk_cnt;
    p.epoch = e->mk_cnt + 1;
    p.abort = e->mk_abort;
    p.x_final = e->x;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(e->n_sm);
    cfg.blockDim = dim3(MK_THREADS);
    cfg.dynamicSmemBytes = MkSmem::total;
    cfg.stream = e->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_mk_kernel<KVT>, p);
}

// One layer's attention with the o-projection folded in (attn_decode_kernel<KVT, false, true>):
// NKV clusters of e->attn_o CTAs, the head pairs' o-proj partial products into e->o_part.
template <typename KVT>
cudaError_t launch_attn_o(icua_engine* e, Session& S, const Layer& ly, int l, const L2Plan& l2) {
    const size_t kv_layer = (size_t)NKV * e->cfg.max_context * HD;
    AttnParams<KVT> a{};
    a.qkv = e->qkv;
    a.q_norm = ly.q_norm;
    a.k_norm = ly.k_norm;
    a.rope = S.rope;
    a.kc = reinterpret_cast<KVT*>(S.kc) + kv_layer * l;
    a.vc = reinterpret_cast<KVT*>(S.vc) + kv_layer * l;
    a.max_ctx = e->cfg.max_context;
    a.n_split = e->attn_o;
    a.cluster = e->attn_o;
    a.st = S.st;
    a.l2 = l2;
    a.wo = ly.o.dev;
    a.o_part = e->o_part;
    return launch_cluster(attn_decode_kernel<KVT, false, true>, NKV * e->attn_o, e->attn_o, 256,
                          AttnSmem<KVT, 1, 16>::total, e->stream, a);
}

template <bool DUAL>
cudaError_t record_layers_t(icua_engine* e, Session& S) {
    cudaError_t err;
    const int L = e->cfg.n_layers;
    if (!DUAL && e->mk)
        return e->cfg.kv_dtype == ICUA_KV_BF16 ? launch_mk<__nv_bfloat16>(e, S) : launch_mk<__half>(e, S);
    for (int l = 0; l < L; ++l) {
        Layer& ly = e->layers[l];
        if (!DUAL && e->attn_o && ly.o.fmt == FMT_Q4S) {
            // QKV -> attention + o-proj -> gate/up -> down; L2 prefetch: QKV(l) the o-proj and gate/up
            // matrices, attention(l) the down matrix, gate/up(l) QKV(l+1), down(l) the next cache rows
            GemvParams p = base_params(e, ly.qkv);
            p.in_mode = (l == 0) ? IN_EMBED : IN_F32;
            p.x = e->x;
            p.norm_w = ly.attn_norm;
            p.prompt = S.prompt;
            p.pooler = e->pooler;
            p.x_resid = e->x;
            p.out = e->qkv;
            p.st = S.st;
            p.l2 = plan_weights(ly.o);
            p.l2.ptr[1] = ly.gu.dev;
            p.l2.bytes[1] = icua_packed_bytes(ly.gu.fmt, ly.gu.n_rows, ly.gu.k);
            p.l2.n = 2;
            err = (l == 0) ? launch_layer_gemv<EPI_STORE, 2048, IN_EMBED>(e, ly.qkv, p, e->stream)
                           : launch_layer_gemv<EPI_STORE, 2048, IN_F32>(e, ly.qkv, p, e->stream);
            if (err != cudaSuccess) return err;
            err = e->cfg.kv_dtype == ICUA_KV_BF16 ? launch_attn_o<__nv_bfloat16>(e, S, ly, l, plan_weights(ly.d))
                                                  : launch_attn_o<__half>(e, S, ly, l, plan_weights(ly.d));
            if (err != cudaSuccess) return err;
            p = base_params(e, ly.gu);
            p.in_mode = IN_F32;
            p.x = e->x;
            p.in_add = e->o_part;
            p.norm_w = ly.mlp_norm;
            p.out = e->h;
            p.st = S.st;
            if (l + 1 < L) p.l2 = plan_weights(e->layers[l + 1].qkv);
            if ((err = launch_layer_gemv<EPI_SWIGLU, 2048, IN_F32>(e, ly.gu, p, e->stream)) != cudaSuccess) return err;
            p = base_params(e, ly.d);
            p.in_mode = IN_F32;
            p.x = e->h;
            p.x_resid = e->x;
            p.resid_add = e->o_part;
            p.deepstack = (l < 3) ? e->deepstack[l] : nullptr;
            p.st = S.st;
            p.l2 = (l + 1 < L) ? plan_kv(e, S, l + 1) : plan_weights(e->embed);
            if ((err = launch_layer_gemv<EPI_RESID, 6144, IN_F32>(e, ly.d, p, e->stream)) != cudaSuccess) return err;
            continue;
        }
        // 1. RMSNorm + QKV projection (layer 0 embeds the input row first)
        GemvParams p = base_params(e, ly.qkv);
        p.in_mode = (l == 0) ? IN_EMBED : IN_F32;
        p.x = e->x;
        p.norm_w = ly.attn_norm;
        p.embed = e->embed.dev;
        p.prompt = S.prompt;
        p.pooler = e->pooler;
        p.x_resid = e->x;
        p.out = e->qkv;
        p.st = S.st;
        p.l2 = plan_weights(ly.o);
        err = (l == 0) ? launch_layer_gemv<EPI_STORE, 2048, IN_EMBED, DUAL>(e, ly.qkv, p, e->stream)
                       : launch_layer_gemv<EPI_STORE, 2048, IN_F32, DUAL>(e, ly.qkv, p, e->stream);
        if (err != cudaSuccess) return err;
        // 2. QK norm + RoPE + KV append + split-K attention (clusters combine the splits)
        const size_t kv_layer = (size_t)NKV * e->cfg.max_context * HD;
        if (e->cfg.kv_dtype == ICUA_KV_BF16) {
            AttnParams<__nv_bfloat16> a{};
            a.qkv = e->qkv;
            a.q_norm = ly.q_norm;
            a.k_norm = ly.k_norm;
            a.rope = S.rope;
            a.kc = reinterpret_cast<__nv_bfloat16*>(S.kc) + kv_layer * l;
            a.vc = reinterpret_cast<__nv_bfloat16*>(S.vc) + kv_layer * l;
            a.max_ctx = e->cfg.max_context;
            a.n_split = e->att_split;
            a.cluster = e->att_cluster;
            a.part = e->att_part;
            a.st = S.st;
            a.l2 = plan_weights(ly.gu);
            err = launch_cluster(attn_decode_kernel<__nv_bfloat16, DUAL>, NKV * e->att_split, e->att_cluster, 256,
                                 AttnSmem<__nv_bfloat16, DUAL ? 2 : 1>::total, e->stream, a);
        } else {
            AttnParams<__half> a{};
            a.qkv = e->qkv;
            a.q_norm = ly.q_norm;
            a.k_norm = ly.k_norm;
            a.rope = S.rope;
            a.kc = reinterpret_cast<__half*>(S.kc) + kv_layer * l;
            a.vc = reinterpret_cast<__half*>(S.vc) + kv_layer * l;
            a.max_ctx = e->cfg.max_context;
            a.n_split = e->att_split;
            a.cluster = e->att_cluster;
            a.part = e->att_part;
            a.st = S.st;
            a.l2 = plan_weights(ly.gu);
            err = launch_cluster(attn_decode_kernel<__half, DUAL>, NKV * e->att_split, e->att_cluster, 256,
                                 AttnSmem<__half, DUAL ? 2 : 1>::total, e->stream, a);
        }
        if (err != cudaSuccess) return err;
        // 3. o-proj + residual
        p = base_params(e, ly.o);
        p.in_mode = IN_ATTN;
        p.att_part = e->att_part;
        p.att_parts = e->att_split / e->att_cluster;
        p.x_resid = e->x;
        p.st = S.st;
        p.l2 = plan_weights(ly.d);
        if ((err = launch_layer_gemv<EPI_RESID, 2048, IN_ATTN, DUAL>(e, ly.o, p, e->stream)) != cudaSuccess) return err;
        // 4. RMSNorm + gate/up + SwiGLU
        p = base_params(e, ly.gu);
        p.in_mode = IN_F32;
        p.x = e->x;
        p.norm_w = ly.mlp_norm;
        p.out = e->h;
        p.st = S.st;
        if (l + 1 < L) p.l2 = plan_weights(e->layers[l + 1].qkv);
        if ((err = launch_layer_gemv<EPI_SWIGLU, 2048, IN_F32, DUAL>(e, ly.gu, p, e->stream)) != cudaSuccess) return err;
        // 5. down + residual (+ DeepStack rows after layers 0..2 while prefilling visual rows)
        p = base_params(e, ly.d);
        p.in_mode = IN_F32;
        p.x = e->h;
        p.x_resid = e->x;
        p.deepstack = (l < 3) ? e->deepstack[l] : nullptr;
        p.st = S.st;
        p.l2 = (l + 1 < L) ? plan_kv(e, S, l + 1) : plan_weights(e->embed);
        if ((err = launch_layer_gemv<EPI_RESID, 6144, IN_F32, DUAL>(e, ly.d, p, e->stream)) != cudaSuccess) return err;
    }
    return cudaSuccess;
}

cudaError_t record_layers(icua_engine* e, Session& S) {
    return e->grammar ? record_layers_t<true>(e, S) : record_layers_t<false>(e, S);
}

cudaError_t record_head(icua_engine* e, Session& S) {
    GemvParams p = base_params(e, e->embed);
    p.in_mode = IN_F32;
    p.x = e->x;
    p.norm_w = e->final_norm;
    p.logits = e->logits;
    p.cta_best_v = e->cta_best_v;
    p.cta_best_i = e->cta_best_i;
    p.step_logits = e->step_logits;
    p.st = S.st;
    // q8 heads always stream; a q4a head streams unless the vocabulary is small (tests).  Grammar
    // engines' heads read the last row of the pass.
    cudaError_t err;
    if (!e->grammar && e->mk)
        err = launch_gemv<FMT_Q8, EPI_LOGITS, 2048, true, IN_F32>(e->embed, p, e->stream, false);
    else if (e->grammar)
        err = e->embed.fmt != FMT_Q4A ? launch_gemv<FMT_Q8, EPI_LOGITS, 2048, true, IN_F32, true>(e->embed, p, e->stream)
              : e->embed.stream       ? launch_gemv<FMT_Q4A, EPI_LOGITS, 2048, true, IN_F32, true>(e->embed, p, e->stream)
                                      : launch_gemv<FMT_Q4A, EPI_LOGITS, 2048, false, IN_F32, true>(e->embed, p, e->stream);
    else
        err = e->embed.fmt != FMT_Q4A ? launch_gemv<FMT_Q8, EPI_LOGITS, 2048, true, IN_F32>(e->embed, p, e->stream)
              : e->embed.stream       ? launch_gemv<FMT_Q4A, EPI_LOGITS, 2048, true, IN_F32>(e->embed, p, e->stream)
                                      : launch_gemv<FMT_Q4A, EPI_LOGITS, 2048, false, IN_F32>(e->embed, p, e->stream);
    if (err != cudaSuccess) return err;
    GrammarRule rule = e->rule;
    if (!e->grammar) rule.n_action = -1;  // the commit never applies the rule
    return launch(commit_kernel, 1, 256, 0, e->stream, true, (const float*)e->cta_best_v, (const int*)e->cta_best_i,
                  e->embed.grid, S.out_tokens, S.st, rule, e->cfg.vocab);
}

icua_status build_graph(icua_engine* eng, Session& S, int kind, cudaGraphExec_t* out) {
    // kind 0: prefill token (layers + advance); 1: one decode step; 2: steps_per_graph steps
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(eng->stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t err = cudaSuccess;
    if (kind == 0) {
        err = record_layers(eng, S);
        if (err == cudaSuccess) err = launch(advance_kernel, 1, 32, 0, eng->stream, !(eng->mk && !eng->grammar), S.st);
    } else {
        const int n = kind == 1 ? 1 : eng->cfg.steps_per_graph;
        for (int i = 0; i < n && err == cudaSuccess; ++i) {
            err = record_layers(eng, S);
            if (err == cudaSuccess) err = record_head(eng, S);
        }
    }
    cudaError_t e2 = cudaStreamEndCapture(eng->stream, &g);
    if (err != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return fail(eng, ICUA_ERR_CUDA, "graph capture: %s", cudaGetErrorString(err));
    }
    if (e2 != cudaSuccess) return fail(eng, ICUA_ERR_CUDA, "end capture: %s", cudaGetErrorString(e2));
    cudaError_t e3 = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e3 != cudaSuccess) return fail(eng, ICUA_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e3));
    return ICUA_OK;
}

void drop_graphs(Session& S) {
    if (S.g_prefill_tok) cudaGraphExecDestroy(S.g_prefill_tok);
    if (S.g_step1) cudaGraphExecDestroy(S.g_step1);
    if (S.g_stepn) cudaGraphExecDestroy(S.g_stepn);
    S.g_prefill_tok = S.g_step1 = S.g_stepn = nullptr;
}

icua_status ensure_graphs(icua_engine* eng, Session& S) {
    icua_status s;
    if (eng->cfg.format == ICUA_FMT_F16) return ICUA_OK;  // f16 engines decode through the batched step
    if (eng->mk && !eng->grammar && !S.g_step1) {
        // the cooperative launch must be capturable; if this driver cannot, decode by the launch chain
        if (build_graph(eng, S, 1, &S.g_step1) != ICUA_OK) {
            cudaGetLastError();
            eng->mk = false;
            S.g_step1 = nullptr;
        }
    }
    if (!S.g_prefill_tok && (s = build_graph(eng, S, 0, &S.g_prefill_tok)) != ICUA_OK) return s;
    if (!S.g_step1 && (s = build_graph(eng, S, 1, &S.g_step1)) != ICUA_OK) return s;
    if (!S.g_stepn && (s = build_graph(eng, S, 2, &S.g_stepn)) != ICUA_OK) return s;
    return ICUA_OK;
}

// ---- M-RoPE table (reference prepareMRoPE, Engine.swift:254-298) ---------------------------------
// Slots >= start get angles for positions laid out as the reference: text slots before the visual
// block use t=h=w=slot, visual slots (visOffset + v) use (visOffset, visOffset + v / llm_w,
// visOffset + v % llm_w), later slots use slot + rope_delta.  Frequency i < 60 takes H when
// i % 3 == 1 and W when i % 3 == 2, T otherwise.  inv_freq follows the fp32 oracle formula.
void fill_rope(icua_engine* e, std::vector<float2>& tab, int start, int vis_abs, int llm_h, int llm_w,
               int rope_delta) {
    const int n_vis = llm_h * llm_w;
    for (int slot = start; slot < e->cfg.max_context; ++slot) {
        int pt, ph, pw;
        if (vis_abs < 0 || slot < vis_abs) {
            pt = ph = pw = slot + (vis_abs < 0 ? rope_delta : 0);
        } else if (slot < vis_abs + n_vis) {
            const int v = slot - vis_abs;
            pt = vis_abs;
            ph = vis_abs + v / llm_w;
            pw = vis_abs + v % llm_w;
        } else {
            pt = ph = pw = slot + rope_delta;
        }
        for (int i = 0; i < 64; ++i) {
            const int pv = (i < 60 && i % 3 == 1) ? ph : (i < 60 && i % 3 == 2) ? pw : pt;
            const float ang = (float)pv * e->inv_freq[i];
            tab[(size_t)slot * 64 + i] = make_float2((float)cos((double)ang), (float)sin((double)ang));
        }
    }
}

icua_status check_ready(icua_engine* eng) {
    if (eng->failed) return fail(eng, ICUA_ERR_STATE, "engine failed earlier: %s", eng->err.c_str());
    if (!eng->uploaded) return fail(eng, ICUA_ERR_STATE, "weights are not complete (icua_engine_ready)");
    return ICUA_OK;
}

Session* get_session(icua_engine* eng, int s) {
    if (s < 0 || s >= (int)eng->sessions.size()) return nullptr;
    return &eng->sessions[s];
}

icua_status sync_and_check(icua_engine* eng, Session& S) {
    CK(cudaStreamSynchronize(eng->stream));
    DevState hs;
    CK(cudaMemcpy(&hs, S.st, sizeof hs, cudaMemcpyDeviceToHost));
    S.pos = hs.pos;
    S.step = hs.step;
    S.done = hs.done;
    if (hs.error) {
        eng->failed = true;
        if (hs.error == ERR_BAD_TOKEN)
            return fail(eng, ICUA_ERR_STATE, "no finite logit at step %d (NaN/inf activations); the session stopped",
                        hs.step);
        return fail(eng, ICUA_ERR_TIMEOUT, "a bounded device wait gave up (flags 0x%x)", hs.error);
    }
    return ICUA_OK;
}

// ---- weights --------------------------------------------------------------------------------
size_t expected_bytes(const icua_engine* e, int id) {
    const int fmt = e->cfg.format;
    const size_t V = (size_t)e->cfg.vocab;
    // embedding: q8 codes + scales, except in reference q4 files (affine q4 like every matrix) and
    // f16 files (fp16 values, no scale tensors)
    if (id == ICUA_TID_EMBED) return fmt == ICUA_FMT_Q4 ? V * H / 2 : fmt == ICUA_FMT_F16 ? V * H * 2 : V * H;
    if (id == ICUA_TID_EMBED_SB) return fmt == ICUA_FMT_Q4 ? V * (H / 64) * 4 : fmt == ICUA_FMT_F16 ? 0 : V * (H / 32) * 2;
    if (id == ICUA_TID_FINAL_NORM) return H * 4;
    const int rel = id - ICUA_TID_LAYER_BASE;
    const int slot = rel % ICUA_TID_PER_LAYER;
    auto mat = [&](int rows, int k) -> size_t {
        if (fmt == ICUA_FMT_F16) return (size_t)rows * k * 2;
        return (fmt == ICUA_FMT_Q4S || fmt == ICUA_FMT_Q4) ? (size_t)rows * k / 2 : (size_t)rows * k;
    };
    auto sb = [&](int rows, int k) -> size_t {
        if (fmt == ICUA_FMT_F16) return 0;
        return fmt == ICUA_FMT_Q4 ? (size_t)rows * (k / 64) * 4 : (size_t)rows * (k / 32) * 2;  // half2 / half
    };
    switch (slot) {
        case ICUA_SLOT_ATTN_NORM:
        case ICUA_SLOT_MLP_NORM: return H * 4;
        case ICUA_SLOT_Q_NORM:
        case ICUA_SLOT_K_NORM: return HD * 4;
        case ICUA_SLOT_WQKV: return mat(QKV_ROWS, H);
        case ICUA_SLOT_WQKV_SB: return sb(QKV_ROWS, H);
        case ICUA_SLOT_WO: return mat(H, H);
        case ICUA_SLOT_WO_SB: return sb(H, H);
        case ICUA_SLOT_WGU: return mat(GU_ROWS, H);
        case ICUA_SLOT_WGU_SB: return sb(GU_ROWS, H);
        case ICUA_SLOT_WD: return mat(H, FF);
        case ICUA_SLOT_WD_SB: return sb(H, FF);
        default: return 0;
    }
}

bool id_used(const icua_engine* e, int id) {
    if (expected_bytes(e, id) == 0) return false;  // f16 files carry no scale tensors
    if (id == ICUA_TID_EMBED || id == ICUA_TID_EMBED_SB || id == ICUA_TID_FINAL_NORM) return true;
    const int rel = id - ICUA_TID_LAYER_BASE;
    if (rel < 0 || rel >= e->cfg.n_layers * ICUA_TID_PER_LAYER) return false;
    return (rel % ICUA_TID_PER_LAYER) <= ICUA_SLOT_WD_SB;
}

icua_status upload_f32(icua_engine* eng, float** dst, const std::vector<uint8_t>& src) {
    icua_status s = dalloc(eng, reinterpret_cast<void**>(dst), src.size());
    if (s != ICUA_OK) return s;
    CK(cudaMemcpy(*dst, src.data(), src.size(), cudaMemcpyHostToDevice));
    return ICUA_OK;
}

// Reference f16 files: the matrix stays row-major fp16 (rows permuted by row_map), the operand of
// the tensor-core GEMMs as it is.
icua_status upload_f16_matrix(icua_engine* eng, Matrix& m, int rows, int k, const std::vector<uint8_t>& codes,
                              const int* row_map) {
    m.fmt = FMT_F16;
    m.n_rows = rows;
    m.k = k;
    m.n_tiles = rows / 16;
    const size_t row_bytes = (size_t)k * 2;
    std::vector<uint8_t> host(codes.size());
    for (int d = 0; d < rows; ++d)
        std::memcpy(host.data() + d * row_bytes, codes.data() + (size_t)(row_map ? row_map[d] : d) * row_bytes, row_bytes);
    icua_status s = dalloc(eng, reinterpret_cast<void**>(&m.dev), host.size());
    if (s != ICUA_OK) return s;
    CK(cudaMemcpy(m.dev, host.data(), host.size(), cudaMemcpyHostToDevice));
    return ICUA_OK;
}

icua_status upload_matrix(icua_engine* eng, Matrix& m, int fmt, int rows, int k, const std::vector<uint8_t>& codes,
                          const std::vector<uint8_t>& sb, const int* row_map) {
    if (fmt == FMT_F16) return upload_f16_matrix(eng, m, rows, k, codes, row_map);
    setup_matrix(m, fmt, rows, k, eng->n_sm);
    const size_t bytes = icua_packed_bytes(fmt, rows, k);
    std::vector<uint8_t> packed(bytes);
    if (fmt == FMT_Q4S)
        icua_host::pack_q4s(rows, k, codes.data(), reinterpret_cast<const uint16_t*>(sb.data()), row_map, packed.data());
    else if (fmt == FMT_Q4A)
        icua_host::pack_q4a(rows, k, codes.data(), reinterpret_cast<const uint16_t*>(sb.data()), row_map, packed.data());
    else
        icua_host::pack_q8(rows, k, reinterpret_cast<const int8_t*>(codes.data()),
                           reinterpret_cast<const uint16_t*>(sb.data()), row_map, packed.data());
    icua_status s = dalloc(eng, reinterpret_cast<void**>(&m.dev), bytes);
    if (s != ICUA_OK) return s;
    CK(cudaMemcpy(m.dev, packed.data(), bytes, cudaMemcpyHostToDevice));
    return ICUA_OK;
}

// The tensor-core order of a quantised matrix (each 128-row block of a k-block contiguous, one
// bulk copy per GEMM stage; rows of 32 bytes for the 4-bit formats) is a second copy of it, read
// only by the batched decode GEMMs.  It is made on the first batched decode, so that batch-1 engines, whose GEMVs read the
// device tile layout, hold each matrix once.
icua_status ensure_tc_order(icua_engine* eng) {
    if (eng->tc_ready) return ICUA_OK;
    std::vector<Matrix*> ms{&eng->embed};
    for (Layer& ly : eng->layers) ms.insert(ms.end(), {&ly.qkv, &ly.o, &ly.gu, &ly.d});
    icua_status s;
    for (Matrix* m : ms) {
        if (m->fmt == FMT_F16 || m->tc || m->n_rows % TC_BM) continue;
        const size_t bytes = icua_packed_bytes(m->fmt, m->n_rows, m->k);
        if ((s = dalloc(eng, reinterpret_cast<void**>(&m->tc), bytes)) != ICUA_OK) return s;
        const long long nv = (long long)bytes / 16;
        const int grid = (int)std::min<long long>((nv + 255) / 256, 4096);
        // row order: each dequantising thread takes 32 consecutive columns of one row
        if (m->fmt == FMT_Q8)
            tc_order_rows_q8_kernel<<<grid, 256, 0, eng->stream>>>(m->dev, m->n_rows / 16, m->k / 64, m->tc);
        else
            tc_order_rows_kernel<<<grid, 256, 0, eng->stream>>>(m->dev, m->fmt, m->n_rows / 16, m->k / 64, m->tc);
        CK(cudaGetLastError());
    }
    CK(cudaStreamSynchronize(eng->stream));
    eng->tc_ready = true;
    return ICUA_OK;
}

// Persistent decode step set-up for q4s engines that ask for it (ICUA_DECODE=mk in the environment
// when the weights are loaded): CTA weight streams (a second copy of the decoder matrices, 0.79 GB
// at 28 layers, ordered by owning CTA), exchange words, counters.  The default decode path is the
// launch chain, which measured a little faster (28.4 vs 29.5 us per layer at 4K context); devices
// with fewer than 128 SMs, or engines where the cooperative grid does not fit, keep the chain too.
icua_status mk_setup(icua_engine* eng) {
    const char* env = getenv("ICUA_DECODE");
    if (!env || strcmp(env, "mk") != 0) return ICUA_OK;
    const int G = eng->n_sm, L = eng->cfg.n_layers;
    int coop = 0, per_sm = 0;
    CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, eng->cfg.device));
    CK(set_smem_attrs());
    cudaError_t oe = eng->cfg.kv_dtype == ICUA_KV_BF16
                         ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_mk_kernel<__nv_bfloat16>,
                                                                         MK_THREADS, MkSmem::total)
                         : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_mk_kernel<__half>, MK_THREADS,
                                                                         MkSmem::total);
    if (oe != cudaSuccess || !coop || per_sm < 1 || G < MK_O_TILES || G / NKV > MK_MAX_S || L > MK_MAX_LAYERS) {
        cudaGetLastError();
        return ICUA_OK;
    }
    std::vector<unsigned long long> base(G);
    unsigned long long total = 0;
    for (int c = 0; c < G; ++c) {
        base[c] = total;
        total += (unsigned long long)L * mk_items_per_layer(c, G) * MK_ITEM;
    }
    icua_status st;
    if ((st = dalloc_t(eng, &eng->mk_stream, total)) != ICUA_OK) return st;
    if ((st = dalloc_t(eng, &eng->mk_cta_base, G)) != ICUA_OK) return st;
    CK(cudaMemcpy(eng->mk_cta_base, base.data(), G * sizeof(unsigned long long), cudaMemcpyHostToDevice));
    std::vector<const uint8_t*> mats(4 * L);
    std::vector<MkLayer> lys(L);
    for (int l = 0; l < L; ++l) {
        const Layer& ly = eng->layers[l];
        mats[4 * l + 0] = ly.qkv.dev;
        mats[4 * l + 1] = ly.o.dev;
        mats[4 * l + 2] = ly.gu.dev;
        mats[4 * l + 3] = ly.d.dev;
        lys[l] = MkLayer{ly.attn_norm, ly.q_norm, ly.k_norm, ly.mlp_norm};
    }
    const uint8_t** mats_dev = nullptr;
    if ((st = dalloc_t(eng, &mats_dev, 4 * L)) != ICUA_OK) return st;
    CK(cudaMemcpy(mats_dev, mats.data(), 4 * L * sizeof(void*), cudaMemcpyHostToDevice));
    if ((st = dalloc_t(eng, &eng->mk_layers, L)) != ICUA_OK) return st;
    CK(cudaMemcpy(eng->mk_layers, lys.data(), L * sizeof(MkLayer), cudaMemcpyHostToDevice));
    mk_pack_kernel<<<G * L, 256>>>(eng->mk_stream, eng->mk_cta_base, mats_dev, L, G);
    CK(cudaGetLastError());
    eng->mk_S = G / NKV;
    constexpr int n_words = 4096 + 2048 + 2048 + 2048 + 6144;
    if ((st = dalloc_t(eng, &eng->mk_words, n_words)) != ICUA_OK) return st;
    if ((st = dalloc_t(eng, &eng->mk_parts, (size_t)NKV * eng->mk_S * ATT_PART)) != ICUA_OK) return st;
    if ((st = dalloc_t(eng, &eng->mk_cnt, 2)) != ICUA_OK) return st;
    if ((st = dalloc_t(eng, &eng->mk_abort, 1)) != ICUA_OK) return st;
    CK(cudaMemset(eng->mk_words, 0, n_words * sizeof(unsigned long long)));
    CK(cudaMemset(eng->mk_cnt, 0, 2 * sizeof(unsigned)));
    CK(cudaMemset(eng->mk_parts, 0, (size_t)NKV * eng->mk_S * ATT_PART * sizeof(unsigned long long)));
    CK(cudaMemset(eng->mk_abort, 0, sizeof(int)));
    const unsigned one = 1;  // epoch 1: no exchange word (tag 0 after the clear) looks current
    CK(cudaMemcpy(eng->mk_cnt + 1, &one, sizeof one, cudaMemcpyHostToDevice));
    CK(cudaDeviceSynchronize());
    eng->mk = true;
    return ICUA_OK;
}

icua_status try_finalize(icua_engine* eng) {
    if (eng->uploaded) return ICUA_OK;
    for (int id = 0; id < ICUA_TENSOR_COUNT; ++id)
        if (id_used(eng, id) && !eng->staged.count(id)) return ICUA_OK;  // not complete yet
    CK(cudaSetDevice(eng->cfg.device));
    icua_status s;
    auto& st = eng->staged;
    // decoder layers in the file's format; the tied embedding is q8, or affine q4 in reference q4 files
    const int cf = eng->cfg.format;
    const int fmt = cf == ICUA_FMT_Q8 ? FMT_Q8 : cf == ICUA_FMT_Q4 ? FMT_Q4A : cf == ICUA_FMT_F16 ? FMT_F16 : FMT_Q4S;
    const int efmt = cf == ICUA_FMT_Q4 ? FMT_Q4A : cf == ICUA_FMT_F16 ? FMT_F16 : FMT_Q8;
    if ((s = upload_matrix(eng, eng->embed, efmt, eng->cfg.vocab, H, st[ICUA_TID_EMBED], st[ICUA_TID_EMBED_SB],
                           nullptr)) != ICUA_OK)
        return s;
    if ((s = upload_f32(eng, &eng->final_norm, st[ICUA_TID_FINAL_NORM])) != ICUA_OK) return s;
    std::vector<int> gu_map(GU_ROWS);
    for (int d = 0; d < GU_ROWS; ++d) {
        const int tile = d / 16, r = d % 16;
        gu_map[d] = r < 8 ? tile * 8 + r : FF + tile * 8 + (r - 8);
    }
    for (int l = 0; l < eng->cfg.n_layers; ++l) {
        Layer& ly = eng->layers[l];
        auto id = [&](int slot) { return ICUA_TID_LAYER_BASE + l * ICUA_TID_PER_LAYER + slot; };
        if ((s = upload_f32(eng, &ly.attn_norm, st[id(ICUA_SLOT_ATTN_NORM)])) != ICUA_OK) return s;
        if ((s = upload_f32(eng, &ly.q_norm, st[id(ICUA_SLOT_Q_NORM)])) != ICUA_OK) return s;
        if ((s = upload_f32(eng, &ly.k_norm, st[id(ICUA_SLOT_K_NORM)])) != ICUA_OK) return s;
        if ((s = upload_f32(eng, &ly.mlp_norm, st[id(ICUA_SLOT_MLP_NORM)])) != ICUA_OK) return s;
        if ((s = upload_matrix(eng, ly.qkv, fmt, QKV_ROWS, H, st[id(ICUA_SLOT_WQKV)], st[id(ICUA_SLOT_WQKV_SB)],
                               nullptr)) != ICUA_OK)
            return s;
        if ((s = upload_matrix(eng, ly.o, fmt, H, H, st[id(ICUA_SLOT_WO)], st[id(ICUA_SLOT_WO_SB)], nullptr)) != ICUA_OK)
            return s;
        if ((s = upload_matrix(eng, ly.gu, fmt, GU_ROWS, H, st[id(ICUA_SLOT_WGU)], st[id(ICUA_SLOT_WGU_SB)],
                               gu_map.data())) != ICUA_OK)
            return s;
        if ((s = upload_matrix(eng, ly.d, fmt, H, FF, st[id(ICUA_SLOT_WD)], st[id(ICUA_SLOT_WD_SB)], nullptr)) != ICUA_OK)
            return s;
    }
    CK(cudaDeviceSynchronize());  // the re-layout kernels ran on the legacy stream
    eng->staged.clear();
    if (fmt == FMT_Q4S && (s = mk_setup(eng)) != ICUA_OK) return s;
    eng->uploaded = true;
    return ICUA_OK;
}

// Prompt rows [0, n_rows) at cache slots S.pos .. through the tensor-core path (reference
// encodePrefill, Engine.swift:476-630): embed, then per layer RMSNorm -> QKV GEMM -> QK norm +
// RoPE + KV append -> causal attention -> o-proj GEMM + residual -> RMSNorm -> gate/up GEMM +
// SwiGLU -> down GEMM + residual (+ DeepStack rows after layers 0..2).  The last layer only
// appends K/V: the prompt's final row, whose logits are needed, runs through the decode step
// afterwards (the reference's last-layer shortcut, Engine.swift:525-528).
// Causal attention of prompt rows [0, n_rows) (cache slots pos0 ..) over slots [0, pos0 + n_rows):
// V^T of the slots (the prompt rows from the projection, earlier slots gathered from the cache),
// then the tensor-core kernel with this layer's TMA maps.
template <typename KVT>
cudaError_t record_prefill_attention(icua_engine* e, const KVT* kc, const KVT* vc, int n_rows, int pos0, int* errp) {
    cudaStream_t st = e->stream;
    cudaError_t err;
    __half* vt = static_cast<__half*>(e->pvt);  // fp16 for both cache types (the P V operand)
    const int vs = e->pvt_stride;
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((n_rows + 31) / 32, NKV * HD / 32);
        cfg.blockDim = dim3(32, 8);
        cfg.stream = st;
        if ((err = cudaLaunchKernelEx(&cfg, prefill_vt_kernel<KVT>, (const float*)e->pqkv, n_rows, pos0, vt, vs)) !=
            cudaSuccess)
            return err;
        if (pos0 > 0) {
            cfg.gridDim = dim3((pos0 + 31) / 32, NKV * HD / 32);
            if ((err = cudaLaunchKernelEx(&cfg, prefill_vt_gather_kernel<KVT>, vc, e->cfg.max_context, pos0, vt, vs)) !=
                cudaSuccess)
                return err;
        }
    }
    auto enc = tensor_map_encoder();
    if (!enc) return cudaErrorNotSupported;
    const CUtensorMapDataType dt =
        std::is_same<KVT, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap qmap, kmap, vtmap;
    const cuuint32_t es[4] = {1, 1, 1, 1};
    const cuuint64_t qd[4] = {64, 2, NQ, (cuuint64_t)n_rows};
    const cuuint64_t qs[3] = {128, 256, (cuuint64_t)NQ * 256};
    const cuuint32_t qb[4] = {64, 1, 1, PT_BQ};
    const cuuint64_t kd[4] = {64, 2, (cuuint64_t)e->cfg.max_context, NKV};
    const cuuint64_t ks[3] = {128, 256, (cuuint64_t)e->cfg.max_context * 256};
    const cuuint32_t kb[4] = {64, 1, PT_BK, 1};
    const cuuint64_t vd[3] = {(cuuint64_t)vs, HD, NKV};
    const cuuint64_t vsd[2] = {(cuuint64_t)vs * 2, (cuuint64_t)vs * HD * 2};
    const cuuint32_t vb[3] = {PT_BK, HD, 1};
    if (enc(&qmap, dt, 4, e->pq, qd, qs, qb, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||

        // the cache rows are stored swizzled already: a plain copy lands them in the 128-byte swizzle
        enc(&kmap, dt, 4, const_cast<KVT*>(kc), kd, ks, kb, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS ||
        enc(&vtmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, vt, vd, vsd, vb, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((n_rows + PT_BQ - 1) / PT_BQ, NQ);
    cfg.blockDim = dim3(PT_THREADS);
    cfg.dynamicSmemBytes = PrefillTcSmem::alloc;
    cfg.stream = st;
    return cudaLaunchKernelEx(&cfg, prefill_attn_tc_kernel<KVT>, qmap, kmap, vtmap, n_rows, pos0, e->pattn, errp);
}

template <typename KVT>
cudaError_t record_prefill_rows(icua_engine* e, Session& S, int n_rows, int vis_off, int n_vis) {
    cudaError_t err;
    cudaStream_t st = e->stream;
    const int L = e->cfg.n_layers, pos0 = S.pos;
    int* errp = &S.st->error;
    if ((err = launch(prefill_embed_kernel, n_rows, 256, 0, st, false, (const int*)S.prompt, n_rows, vis_off, n_vis,
                      (const float*)e->pooler, (const uint8_t*)e->embed.dev, e->embed.n_tiles, e->embed.fmt, e->px)) != cudaSuccess)
        return err;
    const size_t kv_layer = (size_t)NKV * e->cfg.max_context * HD;
    // Launched without programmatic dependent launch: CTAs of a dependent kernel parked at
    // griddepcontrol.wait would hold SMs that the side stream's dequantisation runs on (a run
    // with it measured 3% slower).  The layer matrices in GEMM order (the last layer only projects K/V).  Matrix i is
    // dequantised to fp16 on the side stream while GEMM i-1 runs (after GEMM i-2 has finished), so
    // its tiles are still in L2 when GEMM i reads them; set (layer % 2, kind) holds it.
    std::vector<std::pair<int, int>> seq;  // (layer, kind: 0 QKV, 1 O, 2 gate/up, 3 down)
    for (int l = 0; l < L; ++l)
        for (int kind = 0; kind < (l == L - 1 ? 1 : 4); ++kind) seq.emplace_back(l, kind);
    auto matrix_of = [&](int i) -> const Matrix& {
        const Layer& ly = e->layers[seq[i].first];
        const int kind = seq[i].second;
        return kind == 0 ? ly.qkv : kind == 1 ? ly.o : kind == 2 ? ly.gu : ly.d;
    };
    const bool f16w = e->layers[0].qkv.fmt == FMT_F16;  // reference f16 files: no dequantisation
    auto dequant = [&](int i) -> cudaError_t {
        if (f16w || i >= (int)seq.size()) return cudaSuccess;
        cudaError_t er;
        if (i >= 2 && (er = cudaStreamWaitEvent(e->side, e->ev_done[(i - 2) % 8], 0)) != cudaSuccess) return er;
        if ((er = launch_dequant_f16(matrix_of(i), e->wscr[seq[i].first & 1][seq[i].second], e->n_sm, e->side)) !=
            cudaSuccess)
            return er;
        return cudaEventRecord(e->ev_ready[i % 8], e->side);
    };
    int gi = 0;  // next GEMM of the sequence
    auto gemm_ready = [&]() { return f16w ? cudaSuccess : cudaStreamWaitEvent(st, e->ev_ready[gi % 8], 0); };
    auto gemm_issued = [&]() -> cudaError_t {
        if (f16w) return cudaSuccess;
        cudaError_t er = cudaEventRecord(e->ev_done[gi % 8], st);
        if (er != cudaSuccess) return er;
        ++gi;
        return dequant(gi + 1);
    };
    // the side stream starts behind everything already queued on the main stream
    if (!f16w) {
        if ((err = cudaEventRecord(e->ev_done[7], st)) != cudaSuccess) return err;
        if ((err = cudaStreamWaitEvent(e->side, e->ev_done[7], 0)) != cudaSuccess) return err;
        if ((err = dequant(0)) != cudaSuccess || (err = dequant(1)) != cudaSuccess) return err;
    }
    for (int l = 0; l < L; ++l) {
        Layer& ly = e->layers[l];
        KVT* kc = reinterpret_cast<KVT*>(S.kc) + kv_layer * l;
        KVT* vc = reinterpret_cast<KVT*>(S.vc) + kv_layer * l;
        const __half* w16[4];
        for (int kind = 0; kind < 4; ++kind) w16[kind] = e->wscr[l & 1][kind];
        if (f16w) {
            w16[0] = reinterpret_cast<const __half*>(ly.qkv.dev);
            w16[1] = reinterpret_cast<const __half*>(ly.o.dev);
            w16[2] = reinterpret_cast<const __half*>(ly.gu.dev);
            w16[3] = reinterpret_cast<const __half*>(ly.d.dev);
        }
        if ((err = launch(rmsnorm_rows_f16_kernel<false>, n_rows, 256, 0, st, false, (const float*)e->px,
                          (const float*)ly.attn_norm, n_rows, e->pxn)) != cudaSuccess)
            return err;
        TcGemmParams p = tc_params(ly.qkv, n_rows, errp);
        p.out = e->pqkv;
        p.ldo = QKV_ROWS;
        if ((err = gemm_ready()) != cudaSuccess) return err;
        if ((err = launch_tc_gemm<TC_STORE, FMT_F16>(e->pxn, e->cfg.max_pass, p, st, w16[0])) != cudaSuccess) return err;
        if ((err = gemm_issued()) != cudaSuccess) return err;
        if ((err = launch(qk_rope_kv_kernel<KVT>, n_rows, 256, 0, st, false, (const float*)e->pqkv, n_rows,
                          (const float*)ly.q_norm, (const float*)ly.k_norm, (const float2*)S.rope, pos0, kc, vc,
                          e->cfg.max_context, (KVT*)e->pq)) != cudaSuccess)
            return err;
        if (l == L - 1) break;
        if ((err = record_prefill_attention<KVT>(e, kc, vc, n_rows, pos0, errp)) != cudaSuccess) return err;
        p = tc_params(ly.o, n_rows, errp);
        p.out = e->px;
        p.ldo = H;
        if ((err = gemm_ready()) != cudaSuccess) return err;
        if ((err = launch_tc_gemm<TC_RESID, FMT_F16>(e->pattn, e->cfg.max_pass, p, st, w16[1])) != cudaSuccess) return err;
        if ((err = gemm_issued()) != cudaSuccess) return err;
        if ((err = launch(rmsnorm_rows_f16_kernel<false>, n_rows, 256, 0, st, false, (const float*)e->px,
                          (const float*)ly.mlp_norm, n_rows, e->pxn)) != cudaSuccess)
            return err;
        p = tc_params(ly.gu, n_rows, errp);
        p.out_h = e->ph;
        p.ldh = FF;
        if ((err = gemm_ready()) != cudaSuccess) return err;
        if ((err = launch_tc_gemm<TC_SWIGLU, FMT_F16>(e->pxn, e->cfg.max_pass, p, st, w16[2])) != cudaSuccess) return err;
        if ((err = gemm_issued()) != cudaSuccess) return err;
        p = tc_params(ly.d, n_rows, errp);
        p.out = e->px;
        p.ldo = H;
        if (l < 3 && vis_off >= 0) {
            p.deepstack = e->deepstack[l];
            p.ds_row0 = vis_off;
            p.ds_rows = n_vis;
        }
        if ((err = gemm_ready()) != cudaSuccess) return err;
        if ((err = launch_tc_gemm<TC_RESID, FMT_F16>(e->ph, e->cfg.max_pass, p, st, w16[3])) != cudaSuccess) return err;
        if ((err = gemm_issued()) != cudaSuccess) return err;
    }
    return cudaSuccess;
}

// One batched decode step over rows [r0, r0 + n_rows) (row r -> session eng->batch_rows[r]) on
// stream st: embedding of each session's current token, the layers through the tensor-core GEMMs
// with per-row attention, the tied lm_head GEMM with per-row argmax partials, and the per-session
// commit.  Every row buffer (residual, GEMM inputs as hi / lo row pairs, projections, argmax
// partials, logits) is addressed from the group's first row, so two groups of one step touch
// disjoint memory except for the split-K scratch, which each group brings (splitk) and the error
// flags (atomic OR).
template <typename KVT>
cudaError_t record_batch_rows(icua_engine* e, cudaStream_t st, int r0, int n_rows, float* splitk) {
    cudaError_t err;
    const int L = e->cfg.n_layers;
    const int P2 = 2 * e->cfg.max_pass - 2 * r0;  // hi / lo rows from the group's first one
    const int* rows = e->batch_rows + r0;
    float* px = e->px + (size_t)r0 * H;
    float* pqkv = e->pqkv + (size_t)r0 * QKV_ROWS;
    __half* pxn = e->pxn + (size_t)2 * r0 * H;
    __half* pattn = e->pattn + (size_t)2 * r0 * H;
    __half* ph = e->ph + (size_t)2 * r0 * FF;
    if ((err = launch(batch_embed_kernel, n_rows, 256, 0, st, true, rows, (const DevState*)e->st_all,
                      (const uint8_t*)e->embed.dev, e->embed.n_tiles, e->embed.fmt, px)) != cudaSuccess)
        return err;
    const size_t kv_layer = (size_t)NKV * e->cfg.max_context * HD;
    // the RMSNorm before each projection runs in the finish of the GEMM that updated the residual
    // (o-proj, down), so only layer 0's input norm is a launch of its own
    if ((err = launch(rmsnorm_rows_f16_kernel<true>, n_rows, 256, 0, st, true, (const float*)px,
                      (const float*)e->layers[0].attn_norm, n_rows, pxn)) != cudaSuccess)
        return err;
    for (int l = 0; l < L; ++l) {
        Layer& ly = e->layers[l];
        TcGemmParams p = tc_params(ly.qkv, n_rows, e->gemm_err);
        p.out = pqkv;
        p.ldo = QKV_ROWS;
        int qkv_parts = 1;  // split K: the attention kernel adds the partial products itself
        if ((err = batch_gemm<TC_STORE>(e, ly.qkv, pxn, P2, splitk, p, st, nullptr, nullptr, &qkv_parts)) !=
            cudaSuccess)
            return err;
        {
            AttnParams<KVT> a{};
            a.qkv = qkv_parts > 1 ? splitk : pqkv;
            a.qkv_stride = QKV_ROWS;
            a.qkv_parts = qkv_parts;
            a.qkv_part_stride = (long long)n_rows * QKV_ROWS;
            a.q_norm = ly.q_norm;
            a.k_norm = ly.k_norm;
            a.rope = e->rope_all;
            a.sess_rope_elems = (long long)e->cfg.max_context * 64;
            a.kc = reinterpret_cast<KVT*>(e->kc_all) + kv_layer * l;
            a.vc = reinterpret_cast<KVT*>(e->vc_all) + kv_layer * l;
            a.sess_kv_elems = (long long)e->kv_elems;
            a.max_ctx = e->cfg.max_context;
            // one cluster per (row, kv head): one part, normalised in place.  Cluster size cl splits
            // each row's context over cl CTAs; the choice minimises waves x (streaming time of a
            // CTA + its fixed cost): ceil(rows x 8 x cl / SMs) x (T / cl + O), T = one (row, head)'s
            // cache at the HBM share of an SM (ctx x 512 B / 43 GB/s), O = 5 us of q/k/v staging
            // and combines (measured: at 64 rows and 2K context, cl = 1 beats 2 by 4%, 4 by 22%).
            const double T_us = (double)std::max(e->batch_ctx, 1) * 512.0 / 43.0e3, O_us = 5.0;
            int cl = 1;
            double best = 1e30;
            for (int c = 1; c <= e->att_cluster; c *= 2) {
                const double waves = std::ceil((double)n_rows * NKV * c / e->n_sm);
                const double cost = waves * (T_us / c + O_us);
                if (cost < best - 1e-9) {
                    best = cost;
                    cl = c;
                }
            }
            a.n_split = cl;
            a.cluster = cl;
            a.part = e->att_part;
            a.st = e->st_all;
            a.rows_sess = rows;
            a.out16 = pattn;
            a.out16_hilo = 1;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(NKV * a.n_split, n_rows);
            cfg.blockDim = dim3(256);
            cfg.dynamicSmemBytes = AttnSmem<KVT>::total;
            cfg.stream = st;
            cudaLaunchAttribute attr[2];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = a.cluster;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[1].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 2;
            if ((err = cudaLaunchKernelEx(&cfg, attn_decode_kernel<KVT>, a)) != cudaSuccess) return err;
        }
        p = tc_params(ly.o, n_rows, e->gemm_err);
        p.out = px;
        p.ldo = H;
        if ((err = batch_gemm<TC_RESID>(e, ly.o, pattn, P2, splitk, p, st, ly.mlp_norm, pxn)) != cudaSuccess)
            return err;
        p = tc_params(ly.gu, n_rows, e->gemm_err);
        p.out_h = ph;
        p.ldh = FF;
        if ((err = batch_gemm<TC_SWIGLU>(e, ly.gu, pxn, P2, splitk, p, st)) != cudaSuccess) return err;
        p = tc_params(ly.d, n_rows, e->gemm_err);
        p.out = px;
        p.ldo = H;
        const float* next_norm = l + 1 < L ? e->layers[l + 1].attn_norm : e->final_norm;
        if ((err = batch_gemm<TC_RESID>(e, ly.d, ph, P2, splitk, p, st, next_norm, pxn)) != cudaSuccess) return err;
    }
    const int n_vt = e->cfg.vocab / TC_BM;  // lm_head row tiles: argmax partials [n_vt][n_rows] per group
    TcGemmParams p = tc_params(e->embed, n_rows, e->gemm_err);
    p.best_v = e->batch_best_v + (size_t)n_vt * r0;
    p.best_i = e->batch_best_i + (size_t)n_vt * r0;
    // logits when requested; a one-row step of an f16 engine (its batch-1 decode) keeps them like
    // the GEMV head does
    p.out = e->batch_logits ? e->batch_logits + (size_t)r0 * e->cfg.vocab
                            : (e->embed.fmt == FMT_F16 && n_rows == 1 ? e->logits : nullptr);
    p.ldo = e->cfg.vocab;
    p.hilo = 1;  // the final norm's hi / lo rows
    err = e->embed.fmt == FMT_Q4A ? launch_tc_gemm<TC_ARGMAX, FMT_Q4A>(pxn, P2, p, st, nullptr, 1, true)
        : e->embed.fmt == FMT_F16 ? launch_tc_gemm<TC_ARGMAX, FMT_F16>(pxn, P2, p, st,
                                                                       reinterpret_cast<const __half*>(e->embed.dev), 1,
                                                                       true)
                                  : launch_tc_gemm<TC_ARGMAX, FMT_Q8>(pxn, P2, p, st, nullptr, 1, true);
    if (err != cudaSuccess) return err;
    return launch(batch_commit_kernel, n_rows, 256, 0, st, true, (const float*)p.best_v, (const int*)p.best_i, n_vt,
                  n_rows, rows, e->st_all, e->out_all, e->out_stride, e->cfg.vocab);
}

// Row groups of a batched step.  With ICUA_BATCH_GROUPS=2, two groups (halves of the batch) are
// recorded as two independent chains of the same graph, so that one group's GEMMs (tensor-bound,
// a few dozen CTAs each) can run while the other group's attention streams its caches from HBM;
// each group then reads the layer weights once.  Measured at config 4 (64 sessions, 2K context):
// 4.24 ms per step against 4.28-4.29 ms for one group, inside the run-to-run spread, because the
// attention needs every SM to reach its HBM rate.  One group below 32 rows (the weight reads
// dominate) and above SPLITK_MAX_ROWS (each half must fit its half of the split-K scratch).
int batch_groups(const icua_engine* e, int n_rows) {
    if (e->batch_groups < 2 || n_rows < 32 || n_rows > SPLITK_MAX_ROWS) return 1;
    return 2;
}

template <typename KVT>
cudaError_t record_batch_steps(icua_engine* e, int n_rows, int steps) {
    cudaError_t err = cudaSuccess;
    if (batch_groups(e, n_rows) == 1) {
        for (int i = 0; i < steps && err == cudaSuccess; ++i)
            err = record_batch_rows<KVT>(e, e->stream, 0, n_rows, e->splitk_part);
        return err;
    }
    // group 0 = rows [0, na) on the engine stream, group 1 = rows [na, n_rows) on the side stream,
    // forked from and joined back into the capture; the second half of the split-K scratch
    // (SPLITK_MAX x SPLITK_MAX_ROWS / 2 rows x GU_ROWS) belongs to group 1
    const int na = (n_rows + 1) / 2;
    float* split1 = e->splitk_part + (size_t)SPLITK_MAX * (SPLITK_MAX_ROWS / 2) * GU_ROWS;
    if ((err = cudaEventRecord(e->ev_fork, e->stream)) != cudaSuccess) return err;
    if ((err = cudaStreamWaitEvent(e->side, e->ev_fork, 0)) != cudaSuccess) return err;
    for (int i = 0; i < steps && err == cudaSuccess; ++i) {
        err = record_batch_rows<KVT>(e, e->stream, 0, na, e->splitk_part);
        if (err == cudaSuccess) err = record_batch_rows<KVT>(e, e->side, na, n_rows - na, split1);
    }
    // join on every path, so that ending the capture also ends the side stream's part of it
    const cudaError_t j1 = cudaEventRecord(e->ev_join, e->side);
    const cudaError_t j2 = j1 == cudaSuccess ? cudaStreamWaitEvent(e->stream, e->ev_join, 0) : j1;
    return err != cudaSuccess ? err : j2;
}

void drop_batch_graphs(icua_engine* e) {
    if (e->g_batch1) cudaGraphExecDestroy(e->g_batch1);
    if (e->g_batchn) cudaGraphExecDestroy(e->g_batchn);
    e->g_batch1 = e->g_batchn = nullptr;
    e->batch_key.clear();
}

// The folded o-projection's launch shape (NKV clusters of cl CTAs) is usable when clusters of cl
// are allowed for the kernel and all NKV of them can be resident at once.
template <typename KVT>
bool attn_o_fits_t(int cl) {
    auto k = attn_decode_kernel<KVT, false, true>;
    if ((cl > 8 && cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) ||
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnSmem<KVT, 1, 16>::total) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(NKV * cl);
    lc.blockDim = dim3(256);
    lc.dynamicSmemBytes = AttnSmem<KVT, 1, 16>::total;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = cl;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    int n_clusters = 0;
    const bool ok = cudaOccupancyMaxActiveClusters(&n_clusters, k, &lc) == cudaSuccess && n_clusters >= NKV;
    cudaGetLastError();
    return ok;
}

// Cluster size of the folded o-projection: 16, else 8, else 0 (not usable).
int attn_o_cluster() {
    for (int cl : {16, 8})
        if (attn_o_fits_t<__half>(cl) && attn_o_fits_t<__nv_bfloat16>(cl)) return cl;
    return 0;
}

icua_status build_batch_graph(icua_engine* eng, int n_rows, int steps, cudaGraphExec_t* out) {
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(eng->stream, cudaStreamCaptureModeThreadLocal));
    const cudaError_t err = eng->cfg.kv_dtype == ICUA_KV_BF16 ? record_batch_steps<__nv_bfloat16>(eng, n_rows, steps)
                                                              : record_batch_steps<__half>(eng, n_rows, steps);
    cudaError_t e2 = cudaStreamEndCapture(eng->stream, &g);
    if (err != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return fail(eng, ICUA_ERR_CUDA, "batched graph capture: %s", cudaGetErrorString(err));
    }
    if (e2 != cudaSuccess) return fail(eng, ICUA_ERR_CUDA, "end capture: %s", cudaGetErrorString(e2));
    cudaError_t e3 = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e3 != cudaSuccess) return fail(eng, ICUA_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e3));
    return ICUA_OK;
}

}  // namespace

// =================================================================================================
// C ABI
extern "C" {

const char* icua_global_error(void) { return g_error.c_str(); }
const char* icua_last_error(const icua_engine* eng) { return eng ? eng->err.c_str() : g_error.c_str(); }

void icua_default_config(icua_config* c) {
    if (!c) return;
    c->device = 0;
    c->n_layers = 28;
    c->vocab = 151936;
    c->max_context = 2048;
    c->max_pass = 512;
    c->max_steps = 256;
    c->max_sessions = 1;
    c->format = ICUA_FMT_Q4S;
    c->kv_dtype = ICUA_KV_F16;
    c->steps_per_graph = 8;
    c->prefill_gemm_min = 64;
}

icua_status icua_engine_create(const icua_config* cfg, icua_engine** out) {
    if (!cfg || !out) return fail(nullptr, ICUA_ERR_INVALID, "null argument");
    *out = nullptr;
    if (cfg->format != ICUA_FMT_Q4S && cfg->format != ICUA_FMT_Q8 && cfg->format != ICUA_FMT_Q4 &&
        cfg->format != ICUA_FMT_F16)
        return fail(nullptr, ICUA_ERR_UNSUPPORTED, "weight format %d is not implemented by the kernels", cfg->format);
    if (cfg->n_layers < 1 || cfg->n_layers > 28 || cfg->vocab < 16 || cfg->vocab % 16 || cfg->max_context < 2 ||
        cfg->max_pass < 1 || cfg->max_steps < 1 || cfg->max_sessions < 1 || cfg->steps_per_graph < 1 ||
        (cfg->kv_dtype != ICUA_KV_F16 && cfg->kv_dtype != ICUA_KV_BF16))
        return fail(nullptr, ICUA_ERR_INVALID, "invalid configuration");
    icua_engine* eng = new icua_engine();
    eng->cfg = *cfg;
    cudaError_t e = cudaSetDevice(cfg->device);
    if (e != cudaSuccess) {
        delete eng;
        return fail(nullptr, ICUA_ERR_CUDA, "cudaSetDevice(%d): %s", cfg->device, cudaGetErrorString(e));
    }
    int dev = cfg->device;
    cudaDeviceGetAttribute(&eng->n_sm, cudaDevAttrMultiProcessorCount, dev);
    // 16 splits per kv head (24 and 32 measured 2% slower per step at 4K context); the cluster that
    // combines them is the largest size (8, 4, 2) whose
    // clusters all fit on the GPU at once (a cluster needs its CTAs in one GPC, and GPCs differ
    // in SM count, so large clusters can leave one cluster waiting for a second wave).
    eng->att_split = 16;
    eng->att_cluster = 2;
    if ((e = set_smem_attrs()) == cudaSuccess) {
        for (int cl : {4, 2}) {
            cudaLaunchConfig_t lc = {};
            lc.gridDim = dim3(NKV * eng->att_split);
            lc.blockDim = dim3(256);
            lc.dynamicSmemBytes = AttnSmem<__half>::total;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = cl;
            at[0].val.clusterDim.y = 1;
            at[0].val.clusterDim.z = 1;
            lc.attrs = at;
            lc.numAttrs = 1;
            int n_clusters = 0;
            if (cudaOccupancyMaxActiveClusters(&n_clusters, attn_decode_kernel<__half>, &lc) == cudaSuccess &&
                n_clusters >= NKV * eng->att_split / cl) {
                eng->att_cluster = cl;
                break;
            }
        }
        cudaGetLastError();
    }
    // the o-proj GEMV folds at most ATT_MAX_PARTS parts per kv head
    if (eng->att_split / eng->att_cluster > ATT_MAX_PARTS) eng->att_split = eng->att_cluster * ATT_MAX_PARTS;
    {
        const char* env = getenv("ICUA_ATTN_O");
        if (cfg->format == ICUA_FMT_Q4S && !(env && atoi(env) == 0)) eng->attn_o = attn_o_cluster();
    }
    for (int i = 0; i < 64; ++i) {
        const float a = (float)(2 * i) / 128.0f;
        eng->inv_freq[i] = 1.0f / powf(5000000.0f, a);
    }
    icua_status s = ICUA_OK;
#define TRY(x)                       \
    do {                             \
        if ((s = (x)) != ICUA_OK) {  \
            g_error = eng->err;      \
            icua_engine_destroy(eng); \
            return s;                \
        }                            \
    } while (0)
    if ((e = set_smem_attrs()) != cudaSuccess) {
        fail(eng, ICUA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        s = ICUA_ERR_CUDA;
        g_error = eng->err;
        icua_engine_destroy(eng);
        return s;
    }
    if ((e = cudaStreamCreateWithFlags(&eng->stream, cudaStreamNonBlocking)) != cudaSuccess) {
        delete eng;
        return fail(nullptr, ICUA_ERR_CUDA, "stream: %s", cudaGetErrorString(e));
    }
    for (int i = 0; i < 4; ++i) cudaEventCreate(&eng->ev[i]);
    eng->layers.resize(cfg->n_layers);
    // two rows: a grammar-commit pass may carry two tokens
    TRY(dalloc_t(eng, &eng->x, 2 * H));
    TRY(dalloc_t(eng, &eng->qkv, 2 * QKV_ROWS));
    TRY(dalloc_t(eng, &eng->attn, H));
    TRY(dalloc_t(eng, &eng->h, 2 * FF));
    TRY(dalloc_t(eng, &eng->logits, (size_t)cfg->vocab));
    TRY(dalloc_t(eng, &eng->pooler, (size_t)cfg->max_pass * H));
    for (int i = 0; i < 3; ++i) TRY(dalloc_t(eng, &eng->deepstack[i], (size_t)cfg->max_pass * H));
    TRY(dalloc_t(eng, &eng->att_part, (size_t)2 * NKV * eng->att_split * ATT_PART));
    TRY(dalloc_t(eng, &eng->o_part, (size_t)NKV * H));
    if (cudaMallocHost(reinterpret_cast<void**>(&eng->host_tok), sizeof(int)) != cudaSuccess)
        TRY(fail(eng, ICUA_ERR_CUDA, "cudaMallocHost failed"));
    TRY(dalloc_t(eng, &eng->cta_best_v, (size_t)eng->n_sm));
    TRY(dalloc_t(eng, &eng->cta_best_i, (size_t)eng->n_sm));
    {
        const size_t P = (size_t)cfg->max_pass;
        TRY(dalloc_t(eng, &eng->px, P * H));
        TRY(dalloc_t(eng, &eng->pqkv, P * QKV_ROWS));
        TRY(dalloc(eng, &eng->pq, P * NQ * HD * 2));
        eng->pvt_stride = (cfg->max_context + 63) / 64 * 64 + 64;
        TRY(dalloc(eng, &eng->pvt, (size_t)NKV * HD * eng->pvt_stride * 2));
        cudaMemsetAsync(eng->pvt, 0, (size_t)NKV * HD * eng->pvt_stride * 2, eng->stream);  // slots past a call stay finite
        // 2 P rows: the batched step stores each token's GEMM input as an fp16 hi / lo row pair
        TRY(dalloc_t(eng, &eng->pxn, 2 * P * H));
        TRY(dalloc_t(eng, &eng->pattn, 2 * P * H));
        TRY(dalloc_t(eng, &eng->ph, 2 * P * FF));
        TRY(dalloc_t(eng, &eng->gemm_err, 1));
        TRY(dalloc_t(eng, &eng->splitk_part, (size_t)SPLITK_MAX * SPLITK_MAX_ROWS * GU_ROWS));
        for (int set = 0; set < 2; ++set) {
            TRY(dalloc_t(eng, &eng->wscr[set][0], (size_t)QKV_ROWS * H));
            TRY(dalloc_t(eng, &eng->wscr[set][1], (size_t)H * H));
            TRY(dalloc_t(eng, &eng->wscr[set][2], (size_t)GU_ROWS * H));
            TRY(dalloc_t(eng, &eng->wscr[set][3], (size_t)H * FF));
        }
        for (int i = 0; i < 8; ++i) {
            cudaEventCreateWithFlags(&eng->ev_ready[i], cudaEventDisableTiming);
            cudaEventCreateWithFlags(&eng->ev_done[i], cudaEventDisableTiming);
        }
        cudaStreamCreateWithFlags(&eng->side, cudaStreamNonBlocking);
        cudaEventCreateWithFlags(&eng->ev_fork, cudaEventDisableTiming);
        cudaEventCreateWithFlags(&eng->ev_join, cudaEventDisableTiming);
        if (const char* g = getenv("ICUA_BATCH_GROUPS")) eng->batch_groups = atoi(g) >= 2 ? 2 : 1;
        cudaMemsetAsync(eng->ph, 0, 2 * P * FF * sizeof(__half), eng->stream);
        cudaMemsetAsync(eng->pxn, 0, 2 * P * H * sizeof(__half), eng->stream);
        cudaMemsetAsync(eng->pattn, 0, 2 * P * H * sizeof(__half), eng->stream);
        cudaMemsetAsync(eng->gemm_err, 0, sizeof(int), eng->stream);
        CUtensorMap probe;
        if (!make_act_map(&probe, eng->pxn, (int)P, H, 16))
            TRY(fail(eng, ICUA_ERR_CUDA, "cuTensorMapEncodeTiled is not available"));
    }
    // Sessions live in contiguous per-engine arrays (state, outputs, RoPE tables, caches), so the
    // batched decode reaches session s of any row by one stride.
    eng->sessions.resize(cfg->max_sessions);
    const size_t NS = (size_t)cfg->max_sessions;
    eng->kv_elems = (size_t)cfg->n_layers * NKV * cfg->max_context * HD;
    eng->out_stride = cfg->max_steps + 64;
    TRY(dalloc_t(eng, &eng->st_all, NS));
    TRY(dalloc_t(eng, &eng->out_all, NS * eng->out_stride));
    TRY(dalloc_t(eng, &eng->rope_all, NS * cfg->max_context * 64));
    TRY(dalloc(eng, &eng->kc_all, NS * eng->kv_elems * 2));
    TRY(dalloc(eng, &eng->vc_all, NS * eng->kv_elems * 2));
    TRY(dalloc_t(eng, &eng->batch_rows, (size_t)cfg->max_pass));
    TRY(dalloc_t(eng, &eng->batch_best_v, (size_t)(cfg->vocab / TC_BM) * cfg->max_pass));
    TRY(dalloc_t(eng, &eng->batch_best_i, (size_t)(cfg->vocab / TC_BM) * cfg->max_pass));
    cudaMemsetAsync(eng->st_all, 0, NS * sizeof(DevState), eng->stream);
    // the zero fills are ordered on the engine stream; host-side copies below use the legacy stream
    TRY(cudaStreamSynchronize(eng->stream) == cudaSuccess ? ICUA_OK : fail(eng, ICUA_ERR_CUDA, "zero fill failed"));
    for (size_t i = 0; i < NS; ++i) {
        Session& S = eng->sessions[i];
        S.st = eng->st_all + i;
        TRY(dalloc_t(eng, &S.prompt, (size_t)cfg->max_pass));
        S.out_tokens = eng->out_all + i * eng->out_stride;
        S.rope = eng->rope_all + i * (size_t)cfg->max_context * 64;
        S.kc = static_cast<uint8_t*>(eng->kc_all) + i * eng->kv_elems * 2;
        S.vc = static_cast<uint8_t*>(eng->vc_all) + i * eng->kv_elems * 2;
    }
#undef TRY
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        fail(eng, ICUA_ERR_CUDA, "init: %s", cudaGetErrorString(e));
        g_error = eng->err;
        icua_engine_destroy(eng);
        return ICUA_ERR_CUDA;
    }
    *out = eng;
    for (int i = 0; i < cfg->max_sessions; ++i) icua_reset_session(eng, i);
    return ICUA_OK;
}

void icua_engine_destroy(icua_engine* eng) {
    if (!eng) return;
    cudaSetDevice(eng->cfg.device);
    if (eng->stream) cudaStreamSynchronize(eng->stream);
    for (auto& S : eng->sessions) drop_graphs(S);
    drop_batch_graphs(eng);
    for (void* p : eng->allocations) cudaFree(p);
    for (int i = 0; i < 4; ++i)
        if (eng->ev[i]) cudaEventDestroy(eng->ev[i]);
    for (int i = 0; i < 8; ++i) {
        if (eng->ev_ready[i]) cudaEventDestroy(eng->ev_ready[i]);
        if (eng->ev_done[i]) cudaEventDestroy(eng->ev_done[i]);
    }
    if (eng->host_tok) cudaFreeHost(eng->host_tok);
    if (eng->ev_fork) cudaEventDestroy(eng->ev_fork);
    if (eng->ev_join) cudaEventDestroy(eng->ev_join);
    if (eng->side) {
        cudaStreamSynchronize(eng->side);
        cudaStreamDestroy(eng->side);
    }
    if (eng->stream) cudaStreamDestroy(eng->stream);
    delete eng;
}

// Bytes of vision tensor `id` (reference TensorID 0..314, ModelFile.swift:73-99; storage types of
// Convert.swift:99-152): fp16 matrices [out][in], fp32 vectors and position table.
static size_t vit_tensor_bytes(int id) {
    if (id == 0) return (size_t)VIT_HIDDEN * VIT_PATCH_DIM * 2;
    if (id == 1) return VIT_HIDDEN * 4;
    if (id == 2) return (size_t)VIT_POS_SIDE * VIT_POS_SIDE * VIT_HIDDEN * 4;
    if (id < 3 + VIT_LAYERS * 12) {
        switch ((id - 3) % 12) {
            case 2: return (size_t)VIT_QKV * VIT_HIDDEN * 2;
            case 3: return VIT_QKV * 4;
            case 4: return (size_t)VIT_HIDDEN * VIT_HIDDEN * 2;
            case 8: return (size_t)VIT_FF * VIT_HIDDEN * 2;
            case 9: return VIT_FF * 4;
            case 10: return (size_t)VIT_HIDDEN * VIT_FF * 2;
            default: return VIT_HIDDEN * 4;  // norms, proj / fc2 biases
        }
    }
    const int m = (id - 3 - VIT_LAYERS * 12) / 6, k = (id - 3 - VIT_LAYERS * 12) % 6;
    switch (k) {
        case 0:
        case 1: return (m < 3 ? VIT_MERGED : VIT_HIDDEN) * 4;  // the final merger normalises patches
        case 2: return (size_t)VIT_MERGED * VIT_MERGED * 2;
        case 3: return VIT_MERGED * 4;
        case 4: return (size_t)H * VIT_MERGED * 2;
        default: return H * 4;
    }
}

static icua_status set_vit_tensor(icua_engine* eng, int id, const void* data, uint64_t bytes) {
    const size_t want = vit_tensor_bytes(id);
    if (bytes != want)
        return fail(eng, ICUA_ERR_FORMAT, "vision tensor %d: %llu bytes, expected %zu", id, (unsigned long long)bytes,
                    want);
    CK(cudaSetDevice(eng->cfg.device));
    if (!eng->vit[id]) {
        icua_status s = dalloc(eng, &eng->vit[id], want);
        if (s != ICUA_OK) return s;
        eng->vit_count += 1;
    }
    CK(cudaMemcpy(eng->vit[id], data, want, cudaMemcpyHostToDevice));
    return ICUA_OK;
}

icua_status icua_engine_set_tensor(icua_engine* eng, int32_t id, const void* data, uint64_t bytes) {
    if (!eng || !data) return fail(eng, ICUA_ERR_INVALID, "null argument");
    if (id >= 0 && id < ICUA_VIT_TENSORS) return set_vit_tensor(eng, id, data, bytes);
    if (eng->uploaded) return fail(eng, ICUA_ERR_STATE, "weights already uploaded");
    if (id < 0 || id >= ICUA_TENSOR_COUNT) return fail(eng, ICUA_ERR_INVALID, "tensor id %d out of range", id);
    if (!id_used(eng, id)) return ICUA_OK;  // unused slots (f16 files' scale slots) are ignored
    const size_t want = expected_bytes(eng, id);
    if (bytes != want)
        return fail(eng, ICUA_ERR_FORMAT, "tensor %d: %llu bytes, expected %zu", id, (unsigned long long)bytes, want);
    eng->staged[id] = std::vector<uint8_t>((const uint8_t*)data, (const uint8_t*)data + bytes);
    return try_finalize(eng);
}

icua_status icua_engine_ready(icua_engine* eng) {
    if (!eng) return fail(nullptr, ICUA_ERR_INVALID, "null engine");
    return eng->uploaded ? ICUA_OK : fail(eng, ICUA_ERR_STATE, "weights incomplete");
}

icua_status icua_engine_load_file(icua_engine* eng, const char* path) {
    if (!eng || !path) return fail(eng, ICUA_ERR_INVALID, "null argument");
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(eng, ICUA_ERR_IO, "cannot open %s", path);
    struct stat sb;
    if (fstat(fd, &sb) != 0) {
        close(fd);
        return fail(eng, ICUA_ERR_IO, "cannot stat %s", path);
    }
    const size_t size = (size_t)sb.st_size;
    if (size < 16384 || size % 16384) {
        close(fd);
        return fail(eng, ICUA_ERR_FORMAT, "%s: bad size %zu", path, size);
    }
    void* p = mmap(nullptr, size, PROT_READ, MAP_SHARED, fd, 0);
    close(fd);
    if (p == MAP_FAILED) return fail(eng, ICUA_ERR_IO, "mmap failed for %s", path);
    const uint8_t* base = (const uint8_t*)p;
    uint32_t hdr[4];
    memcpy(hdr, base, 16);
    icua_status s = ICUA_OK;
    if (hdr[0] != 0x31554349u)
        s = fail(eng, ICUA_ERR_FORMAT, "%s: not an instantcua model", path);
    else if (hdr[1] != 1)
        s = fail(eng, ICUA_ERR_FORMAT, "%s: unsupported version", path);
    else if ((int)hdr[2] != eng->cfg.format)
        s = fail(eng, ICUA_ERR_FORMAT, "%s: format %u does not match the engine format %d", path, hdr[2], eng->cfg.format);
    else if (hdr[3] != (uint32_t)ICUA_TENSOR_COUNT)
        s = fail(eng, ICUA_ERR_FORMAT, "%s: tensor table mismatch", path);
    for (int id = 0; s == ICUA_OK && id < ICUA_TENSOR_COUNT; ++id) {
        const bool vit = id < ICUA_VIT_TENSORS;
        if (!vit && !id_used(eng, id)) continue;
        uint64_t off, sz;
        memcpy(&off, base + 16 + 16 * id, 8);
        memcpy(&sz, base + 16 + 16 * id + 8, 8);
        if (vit && sz == 0) continue;  // a file without the vision encoder
        if (off + sz > size) {
            s = fail(eng, ICUA_ERR_FORMAT, "%s: tensor %d outside the file", path, id);
            break;
        }
        s = icua_engine_set_tensor(eng, id, base + off, sz);
    }
    munmap(p, size);
    if (s == ICUA_OK && !eng->uploaded) s = fail(eng, ICUA_ERR_FORMAT, "%s: tensors missing", path);
    return s;
}

icua_status icua_set_eos(icua_engine* eng, int32_t eos0, int32_t eos1, int32_t stop) {
    if (!eng) return fail(nullptr, ICUA_ERR_INVALID, "null engine");
    eng->eos0 = eos0;
    eng->eos1 = eos1;
    eng->stop_on_eos = stop ? 1 : 0;
    return ICUA_OK;
}

static icua_status reset_session_impl(icua_engine* eng, int32_t session, bool keep_prefix);

icua_status icua_reset_session(icua_engine* eng, int32_t session) { return reset_session_impl(eng, session, false); }

icua_status icua_set_prefix_cache(icua_engine* eng, int32_t enable) {
    if (!eng) return fail(nullptr, ICUA_ERR_INVALID, "null engine");
    eng->prefix_cache = enable ? 1 : 0;
    if (!enable)
        for (auto& S : eng->sessions) S.prefix_valid = false;
    return ICUA_OK;
}

icua_status icua_set_grammar_commit(icua_engine* eng, int32_t enable, const icua_grammar* rule) {
    if (!eng) return fail(nullptr, ICUA_ERR_INVALID, "null engine");
    if (enable && eng->cfg.format == ICUA_FMT_F16)
        return fail(eng, ICUA_ERR_INVALID, "grammar commit runs on the batch-1 decode graphs of quantized engines");
    GrammarRule r = eng->rule;
    if (rule) {
        if (rule->n_action < 0 || rule->n_action > 8) return fail(eng, ICUA_ERR_INVALID, "n_action %d", rule->n_action);
        const int V = eng->cfg.vocab;
        auto ok = [V](int t) { return t >= 0 && t < V; };
        for (int i = 0; i < rule->n_action; ++i)
            if (!ok(rule->action[i])) return fail(eng, ICUA_ERR_INVALID, "action id %d", rule->action[i]);
        if (!ok(rule->comma) || !ok(rule->space) || !ok(rule->open) || !ok(rule->close))
            return fail(eng, ICUA_ERR_INVALID, "syntax id outside the vocabulary");
        r.n_action = rule->n_action;
        for (int i = 0; i < 8; ++i) r.action[i] = i < rule->n_action ? rule->action[i] : -1;
        r.comma = rule->comma;
        r.space = rule->space;
        r.open = rule->open;
        r.close = rule->close;
    } else if (enable && (r.space >= eng->cfg.vocab || r.open >= eng->cfg.vocab)) {
        return fail(eng, ICUA_ERR_INVALID, "the reference's syntax ids need a vocabulary of %d", eng->cfg.vocab);
    }
    eng->rule = r;
    eng->grammar = enable != 0;
    // the session graphs hold the one- or two-token kernels and the rule (a kernel parameter)
    CK(cudaSetDevice(eng->cfg.device));
    for (Session& S : eng->sessions) drop_graphs(S);
    return ICUA_OK;
}

static icua_status reset_session_impl(icua_engine* eng, int32_t session, bool keep_prefix) {
    if (!eng) return fail(nullptr, ICUA_ERR_INVALID, "null engine");
    Session* S = get_session(eng, session);
    if (!S) return fail(eng, ICUA_ERR_INVALID, "session %d out of range", session);
    if (!keep_prefix) S->prefix_valid = false;
    CK(cudaSetDevice(eng->cfg.device));
    S->pos = 0;
    S->step = 0;
    S->done = 0;
    S->rope_delta = 0;
    std::vector<float2> tab((size_t)eng->cfg.max_context * 64);
    fill_rope(eng, tab, 0, -1, 0, 0, 0);
    CK(cudaMemcpy(S->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice));
    DevState hs{};
    hs.vis_offset = -1;
    hs.session = session;
    hs.n_tok = 1;
    CK(cudaMemcpy(S->st, &hs, sizeof hs, cudaMemcpyHostToDevice));
    return ICUA_OK;
}

icua_status icua_session_position(icua_engine* eng, int32_t session, int32_t* pos) {
    Session* S = eng ? get_session(eng, session) : nullptr;
    if (!S || !pos) return fail(eng, ICUA_ERR_INVALID, "bad argument");
    *pos = S->pos;
    return ICUA_OK;
}

icua_status icua_inject_kv(icua_engine* eng, int32_t session, const float* k, const float* v, int32_t n_pos) {
    Session* S = eng ? get_session(eng, session) : nullptr;
    if (!S || !k || !v || n_pos < 0) return fail(eng, ICUA_ERR_INVALID, "bad argument");
    if (n_pos >= eng->cfg.max_context) return fail(eng, ICUA_ERR_CAPACITY, "%d positions exceed max_context", n_pos);
    S->prefix_valid = false;
    CK(cudaSetDevice(eng->cfg.device));
    const int L = eng->cfg.n_layers, C = eng->cfg.max_context;
    std::vector<uint16_t> kb((size_t)NKV * n_pos * HD), vb((size_t)NKV * n_pos * HD);
    for (int l = 0; l < L; ++l) {
        for (int p = 0; p < n_pos; ++p)
            for (int h = 0; h < NKV; ++h)
                for (int d = 0; d < HD; ++d) {
                    const size_t src = (((size_t)l * n_pos + p) * NKV + h) * HD + d;
                    const size_t dst = ((size_t)h * n_pos + p) * HD + kv_swz(d, p);  // cache row order
                    if (eng->cfg.kv_dtype == ICUA_KV_F16) {
                        kb[dst] = icua_host::f32_to_f16_bits(k[src]);
                        vb[dst] = icua_host::f32_to_f16_bits(v[src]);
                    } else {
                        auto bf = [](float f) {
                            uint32_t u;
                            memcpy(&u, &f, 4);
                            u += 0x7FFFu + ((u >> 16) & 1u);
                            return (uint16_t)(u >> 16);
                        };
                        kb[dst] = bf(k[src]);
                        vb[dst] = bf(v[src]);
                    }
                }
        for (int h = 0; h < NKV; ++h) {
            const size_t off = (((size_t)l * NKV + h) * C) * HD * 2;
            CK(cudaMemcpy((uint8_t*)S->kc + off, kb.data() + (size_t)h * n_pos * HD, (size_t)n_pos * HD * 2,
                          cudaMemcpyHostToDevice));
            CK(cudaMemcpy((uint8_t*)S->vc + off, vb.data() + (size_t)h * n_pos * HD, (size_t)n_pos * HD * 2,
                          cudaMemcpyHostToDevice));
        }
    }
    S->pos = n_pos;
    CK(cudaMemcpy(&S->st->pos, &n_pos, 4, cudaMemcpyHostToDevice));
    return ICUA_OK;
}

icua_status icua_inject_kv_random(icua_engine* eng, int32_t session, int32_t n_pos, uint64_t seed) {
    Session* S = eng ? get_session(eng, session) : nullptr;
    if (!S || n_pos < 0) return fail(eng, ICUA_ERR_INVALID, "bad argument");
    if (n_pos >= eng->cfg.max_context) return fail(eng, ICUA_ERR_CAPACITY, "%d positions exceed max_context", n_pos);
    S->prefix_valid = false;
    CK(cudaSetDevice(eng->cfg.device));
    if (eng->cfg.kv_dtype == ICUA_KV_F16)
        kv_fill_random_kernel<__half><<<eng->n_sm * 8, 256, 0, eng->stream>>>(
            (__half*)S->kc, (__half*)S->vc, eng->cfg.n_layers, eng->cfg.max_context, n_pos, seed);
    else
        kv_fill_random_kernel<__nv_bfloat16><<<eng->n_sm * 8, 256, 0, eng->stream>>>(
            (__nv_bfloat16*)S->kc, (__nv_bfloat16*)S->vc, eng->cfg.n_layers, eng->cfg.max_context, n_pos, seed);
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(eng->stream));
    S->pos = n_pos;
    CK(cudaMemcpy(&S->st->pos, &n_pos, 4, cudaMemcpyHostToDevice));
    return ICUA_OK;
}

icua_status icua_capture_step_logits(icua_engine* eng, float* host_out, int32_t cap) {
    if (!eng) return fail(nullptr, ICUA_ERR_INVALID, "null engine");
    CK(cudaSetDevice(eng->cfg.device));
    if (host_out == nullptr) {
        eng->step_logits_host = nullptr;
        eng->step_logits_cap = 0;
        return ICUA_OK;
    }
    if (cap < 1 || cap > eng->cfg.max_steps) return fail(eng, ICUA_ERR_CAPACITY, "capacity %d", cap);
    if (!eng->step_logits) {
        icua_status s = dalloc_t(eng, &eng->step_logits, (size_t)(eng->cfg.max_steps + 64) * eng->cfg.vocab);
        if (s != ICUA_OK) return s;
        for (auto& S : eng->sessions) drop_graphs(S);  // graphs bake the capture pointer
    }
    eng->step_logits_host = host_out;
    eng->step_logits_cap = cap;
    return ICUA_OK;
}

// Writes the prompt, visual rows, RoPE table and loop state; returns via *pos0 the start position.
static icua_status prepare_prefill(icua_engine* eng, Session& S, int session, const int32_t* tokens, int n,
                                   const icua_visual* vis, int write_logits, int* vis_off_out, int* n_vis_out) {
    const int C = eng->cfg.max_context;
    if (n < 1 || n > eng->cfg.max_pass) return fail(eng, ICUA_ERR_CAPACITY, "prompt of %d tokens (max_pass %d)", n, eng->cfg.max_pass);
    if (S.pos + n + 1 > C) return fail(eng, ICUA_ERR_CAPACITY, "context %d + %d exceeds max_context %d", S.pos, n, C);
    int vis_off = -1;
    for (int i = 0; i < n; ++i) {
        if (tokens[i] < 0 || (tokens[i] >= eng->cfg.vocab && tokens[i] != IMAGE_PAD_ID))
            return fail(eng, ICUA_ERR_INVALID, "token %d at %d out of range", tokens[i], i);
        if (tokens[i] == IMAGE_PAD_ID && vis_off < 0) vis_off = i;
    }
    if (vis_off >= 0 && (!vis || (!vis->pooler && eng->vis_rows != vis->n_vis)))
        return fail(eng, ICUA_ERR_INVALID, "IMAGE_PAD tokens without visual inputs (host rows, or %d encoder rows)",
                    eng->vis_rows);
    CK(cudaMemcpyAsync(S.prompt, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, eng->stream));
    std::vector<float2> tab((size_t)C * 64);
    CK(cudaMemcpy(tab.data(), S.rope, tab.size() * sizeof(float2), cudaMemcpyDeviceToHost));
    int n_vis = 0;
    if (vis_off >= 0) {
        n_vis = vis->n_vis;
        if (n_vis < 1 || n_vis != vis->llm_h * vis->llm_w || vis_off + n_vis > n)
            return fail(eng, ICUA_ERR_INVALID, "visual block of %d rows (grid %dx%d) does not fit the prompt", n_vis,
                        vis->llm_h, vis->llm_w);
        for (int i = vis_off; i < vis_off + n_vis; ++i)
            if (tokens[i] != IMAGE_PAD_ID) return fail(eng, ICUA_ERR_INVALID, "visual block is not contiguous");
        if (vis->pooler) {  // host rows; else the vision encoder's rows are already in place
            CK(cudaMemcpyAsync(eng->pooler, vis->pooler, (size_t)n_vis * H * 4, cudaMemcpyHostToDevice, eng->stream));
            for (int d = 0; d < 3; ++d) {
                if (vis->deepstack[d])
                    CK(cudaMemcpyAsync(eng->deepstack[d], vis->deepstack[d], (size_t)n_vis * H * 4,
                                       cudaMemcpyHostToDevice, eng->stream));
                else
                    CK(cudaMemsetAsync(eng->deepstack[d], 0, (size_t)n_vis * H * 4, eng->stream));
            }
            eng->vis_rows = -1;  // overwritten
        }
        const int vis_abs = S.pos + vis_off;
        S.rope_delta = std::max(vis->llm_h, vis->llm_w) - n_vis;
        fill_rope(eng, tab, S.pos, vis_abs, vis->llm_h, vis->llm_w, S.rope_delta);
    } else {
        fill_rope(eng, tab, S.pos, -1, 0, 0, S.rope_delta);
    }
    CK(cudaMemcpyAsync(S.rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice, eng->stream));
    DevState hs{};
    hs.pos = S.pos;
    hs.step = 0;
    hs.done = 0;
    hs.max_steps = 1;
    hs.eos0 = eng->eos0;
    hs.eos1 = eng->eos1;
    hs.stop_on_eos = eng->stop_on_eos;
    hs.cur_token = 0;
    hs.prompt_idx = 0;
    hs.prompt_len = n;
    hs.vis_offset = vis_off;
    hs.n_vis = n_vis;
    hs.write_logits = write_logits ? 1 : 0;
    hs.session = session;
    hs.n_tok = 1;
    hs.grammar = eng->grammar ? 1 : 0;
    *vis_off_out = vis_off;
    *n_vis_out = n_vis;
    CK(cudaMemcpyAsync(S.st, &hs, sizeof hs, cudaMemcpyHostToDevice, eng->stream));
    CK(cudaStreamSynchronize(eng->stream));  // host staging buffers go out of scope
    S.step = 0;
    S.done = 0;
    return ICUA_OK;
}

static icua_status decode_batch_impl(icua_engine* eng, const int32_t* sessions, int32_t n_sessions,
                                     const int32_t* in_tokens, int32_t steps, int32_t* out);

icua_status icua_prefill(icua_engine* eng, int32_t session, const int32_t* tokens, int32_t n, const icua_visual* vis,
                         int32_t write_logits, int32_t* first_token) {
    if (!eng || !tokens) return fail(eng, ICUA_ERR_INVALID, "null argument");
    icua_status s;
    if ((s = check_ready(eng)) != ICUA_OK) return s;
    Session* S = get_session(eng, session);
    if (!S) return fail(eng, ICUA_ERR_INVALID, "session %d out of range", session);
    if (S->pos < (int)S->prefix.size()) S->prefix_valid = false;  // this prefill overwrites prefix rows
    CK(cudaSetDevice(eng->cfg.device));
    if ((s = ensure_graphs(eng, *S)) != ICUA_OK) return s;
    int vis_off = -1, n_vis = 0;
    if ((s = prepare_prefill(eng, *S, session, tokens, n, vis, write_logits, &vis_off, &n_vis)) != ICUA_OK) return s;
    CK(cudaEventRecord(eng->ev[0], eng->stream));
    const int n_rows = n - 1;  // rows before the last one, which runs as a decode step
    if (eng->cfg.format == ICUA_FMT_F16) {
        // f16 engines: every row before the last through the tensor-core path, the last one as a
        // one-row batched step (its head gives the first token and keeps the logits)
        if (tokens[n - 1] == IMAGE_PAD_ID)
            return fail(eng, ICUA_ERR_UNSUPPORTED, "f16 engines need a text token at the end of the prompt");
        if (n_rows > 0) {
            const cudaError_t e2 = eng->cfg.kv_dtype == ICUA_KV_BF16
                                       ? record_prefill_rows<__nv_bfloat16>(eng, *S, n_rows, vis_off, n_vis)
                                       : record_prefill_rows<__half>(eng, *S, n_rows, vis_off, n_vis);
            if (e2 != cudaSuccess) return fail(eng, ICUA_ERR_CUDA, "prefill launch: %s", cudaGetErrorString(e2));
        }
        const int pos = S->pos + n_rows;
        CK(cudaMemcpyAsync(&S->st->pos, &pos, 4, cudaMemcpyHostToDevice, eng->stream));
        S->pos = pos;
        int32_t tok1 = 0;
        const float keep_decode_ms = eng->timing.decode_ms;
        if ((s = decode_batch_impl(eng, &session, 1, &tokens[n - 1], 1, &tok1)) != ICUA_OK) return s;
        eng->timing.decode_ms = keep_decode_ms;
        CK(cudaEventRecord(eng->ev[1], eng->stream));
        CK(cudaStreamSynchronize(eng->stream));
        float ms = 0.f;
        cudaEventElapsedTime(&ms, eng->ev[0], eng->ev[1]);
        eng->timing.prefill_ms = ms;
        eng->timing.prefill_tokens = n;
        if (first_token) *first_token = tok1;
        return ICUA_OK;
    }
    if (eng->cfg.prefill_gemm_min > 0 && n_rows >= eng->cfg.prefill_gemm_min) {
        const cudaError_t e2 = eng->cfg.kv_dtype == ICUA_KV_BF16
                                   ? record_prefill_rows<__nv_bfloat16>(eng, *S, n_rows, vis_off, n_vis)
                                   : record_prefill_rows<__half>(eng, *S, n_rows, vis_off, n_vis);
        if (e2 != cudaSuccess) return fail(eng, ICUA_ERR_CUDA, "prefill launch: %s", cudaGetErrorString(e2));
        const int pos = S->pos + n_rows;
        CK(cudaMemcpyAsync(&S->st->pos, &pos, 4, cudaMemcpyHostToDevice, eng->stream));
        CK(cudaMemcpyAsync(&S->st->prompt_idx, &n_rows, 4, cudaMemcpyHostToDevice, eng->stream));
    } else {
        for (int i = 0; i < n_rows; ++i) CK(cudaGraphLaunch(S->g_prefill_tok, eng->stream));
    }
    CK(cudaGraphLaunch(S->g_step1, eng->stream));
    CK(cudaEventRecord(eng->ev[1], eng->stream));
    if ((s = sync_and_check(eng, *S)) != ICUA_OK) return s;
    float ms = 0.f;
    cudaEventElapsedTime(&ms, eng->ev[0], eng->ev[1]);
    eng->timing.prefill_ms = ms;
    eng->timing.prefill_tokens = n;
    int tok = 0;
    CK(cudaMemcpy(&tok, S->out_tokens, 4, cudaMemcpyDeviceToHost));
    if (eng->step_logits_host) CK(cudaMemcpy(eng->step_logits_host, eng->step_logits, (size_t)eng->cfg.vocab * 4, cudaMemcpyDeviceToHost));
    if (first_token) *first_token = tok;
    // the write-logits request applies to the prompt pass only
    const int zero = 0;
    CK(cudaMemcpy(&S->st->write_logits, &zero, 4, cudaMemcpyHostToDevice));
    return ICUA_OK;
}

icua_status icua_decode(icua_engine* eng, int32_t session, int32_t max_new, int32_t* out, int32_t* n_out) {
    if (!eng || !out || !n_out) return fail(eng, ICUA_ERR_INVALID, "null argument");
    if (eng->cfg.format == ICUA_FMT_F16 && max_new > 0) {
        // f16 engines: the batched step with this one session
        std::vector<int32_t> toks(max_new);
        icua_status s2 = decode_batch_impl(eng, &session, 1, nullptr, max_new, toks.data());
        if (s2 != ICUA_OK) return s2;
        int n = 0;
        while (n < max_new && toks[n] >= 0 && !(eng->stop_on_eos && (toks[n] == eng->eos0 || toks[n] == eng->eos1)))
            out[n] = toks[n], ++n;
        *n_out = n;
        return ICUA_OK;
    }
    icua_status s;
    if ((s = check_ready(eng)) != ICUA_OK) return s;
    Session* S = get_session(eng, session);
    if (!S) return fail(eng, ICUA_ERR_INVALID, "session %d out of range", session);
    *n_out = 0;
    if (max_new <= 0) return ICUA_OK;
    CK(cudaSetDevice(eng->cfg.device));
    if ((s = ensure_graphs(eng, *S)) != ICUA_OK) return s;
    if (S->step < 1) return fail(eng, ICUA_ERR_STATE, "decode before prefill");
    if (S->done && S->step >= 1) {
        // a finished prefill (max_steps reached) is resumed; an EOS stop is final
        int last = 0;
        CK(cudaMemcpy(&last, S->out_tokens + S->step - 1, 4, cudaMemcpyDeviceToHost));
        if (eng->stop_on_eos && (last == eng->eos0 || last == eng->eos1)) return ICUA_OK;
    }
    const int base_step = S->step;
    if (base_step + max_new > eng->cfg.max_steps + 1)
        return fail(eng, ICUA_ERR_CAPACITY, "%d steps exceed max_steps %d", base_step + max_new, eng->cfg.max_steps);
    if (S->pos + max_new + eng->cfg.steps_per_graph > eng->cfg.max_context)
        return fail(eng, ICUA_ERR_CAPACITY, "context %d + %d exceeds max_context", S->pos, max_new);
    const int ms_val = base_step + max_new, zero = 0;
    if (eng->grammar) {
        // The commit that ended the previous call (the prefill's first token, or max_steps) did not
        // apply the rule to its token: apply it now, as the reference's single loop would have.
        DevState hs;
        CK(cudaMemcpy(&hs, S->st, sizeof hs, cudaMemcpyDeviceToHost));
        if (hs.n_tok != 2 && hs.cur_token == eng->rule.close) return ICUA_OK;  // ')' ended the output
        hs.grammar = 1;
        hs.max_steps = ms_val;
        hs.done = 0;
        if (hs.n_tok != 2) {
            hs.n_tok = 1;
            const int syn = grammar_syntax(eng->rule, hs.cur_token, hs.step);
            if (syn >= 0) {
                CK(cudaMemcpy(S->out_tokens + hs.step, &syn, 4, cudaMemcpyHostToDevice));
                hs.step += 1;
                hs.n_tok = 2;
                hs.cur_token2 = syn;
                if (hs.step >= ms_val) hs.done = 1;
            }
        }
        // a pass of two tokens follows a commit of two outputs: positions still grow by at most
        // one per output token, so the capacity check above holds
        CK(cudaMemcpy(S->st, &hs, sizeof hs, cudaMemcpyHostToDevice));
    } else {
        CK(cudaMemcpyAsync(&S->st->max_steps, &ms_val, 4, cudaMemcpyHostToDevice, eng->stream));
        CK(cudaMemcpyAsync(&S->st->done, &zero, 4, cudaMemcpyHostToDevice, eng->stream));
    }
    const auto t0 = std::chrono::steady_clock::now();
    CK(cudaEventRecord(eng->ev[2], eng->stream));
    const int spg = eng->cfg.steps_per_graph;
    int launched = 0;
    while (launched + spg <= max_new) {
        CK(cudaGraphLaunch(S->g_stepn, eng->stream));
        launched += spg;
    }
    while (launched < max_new) {
        CK(cudaGraphLaunch(S->g_step1, eng->stream));
        launched += 1;
    }
    CK(cudaEventRecord(eng->ev[3], eng->stream));
    if ((s = sync_and_check(eng, *S)) != ICUA_OK) return s;
    float ms = 0.f;
    cudaEventElapsedTime(&ms, eng->ev[2], eng->ev[3]);
    eng->timing.decode_ms = ms;
    const int got = S->step - base_step;
    std::vector<int32_t> toks(got > 0 ? got : 1);
    if (got > 0) CK(cudaMemcpy(toks.data(), S->out_tokens + base_step, (size_t)got * 4, cudaMemcpyDeviceToHost));
    int n = 0;
    for (int i = 0; i < got; ++i) {
        if (eng->stop_on_eos && (toks[i] == eng->eos0 || toks[i] == eng->eos1)) break;
        out[n++] = toks[i];
    }
    *n_out = n;
    if (eng->step_logits_host && got > 0) {
        const int rows = std::min(got, eng->step_logits_cap);
        CK(cudaMemcpy(eng->step_logits_host, eng->step_logits + (size_t)base_step * eng->cfg.vocab,
                      (size_t)rows * eng->cfg.vocab * 4, cudaMemcpyDeviceToHost));
    }
    eng->timing.generated_tokens = n;
    eng->timing.total_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return ICUA_OK;
}

icua_status icua_decode_step(icua_engine* eng, int32_t session, int32_t in_token, int32_t* out_token) {
    if (!eng || !out_token) return fail(eng, ICUA_ERR_INVALID, "null argument");
    if (eng->cfg.format == ICUA_FMT_F16) return decode_batch_impl(eng, &session, 1, &in_token, 1, out_token);
    icua_status s;
    if ((s = check_ready(eng)) != ICUA_OK) return s;
    Session* S = get_session(eng, session);
    if (!S) return fail(eng, ICUA_ERR_INVALID, "session %d out of range", session);
    if (in_token < 0 || in_token >= eng->cfg.vocab) return fail(eng, ICUA_ERR_INVALID, "token %d out of range", in_token);
    if (S->pos + 1 >= eng->cfg.max_context) return fail(eng, ICUA_ERR_CAPACITY, "context full");
    CK(cudaSetDevice(eng->cfg.device));
    if ((s = ensure_graphs(eng, *S)) != ICUA_OK) return s;
    if (S->step >= eng->cfg.max_steps) S->step = 0;  // wrap the output slot for long host-driven loops
    // the step's loop state (input token, step budget, no prompt rows left) in one small launch,
    // the generated token back through the engine's pinned word
    CK(launch(step_head_kernel, 1, 32, 0, eng->stream, false, S->st, S->step, in_token, eng->grammar ? 1 : 0));
    CK(cudaGraphLaunch(S->g_step1, eng->stream));
    CK(cudaMemcpyAsync(eng->host_tok, S->out_tokens + S->step, 4, cudaMemcpyDeviceToHost, eng->stream));
    CK(cudaStreamSynchronize(eng->stream));
    *out_token = *eng->host_tok;
    S->step += 1;
    S->pos += 1;
    return ICUA_OK;
}

uint64_t icua_device_bytes(const icua_engine* eng) { return eng ? eng->device_bytes : 0; }

int32_t icua_attn_o_cluster(const icua_engine* eng) { return eng ? eng->attn_o : 0; }

int32_t icua_decode_kernels_per_step(const icua_engine* eng) {
    if (!eng) return 0;
    if (eng->mk && !eng->grammar) return 3;  // persistent layers kernel, lm_head GEMV, commit
    if (eng->attn_o && !eng->grammar) return 4 * eng->cfg.n_layers + 2;  // o-proj folded into the attention
    return 5 * eng->cfg.n_layers + 2;
}

icua_status icua_profile_decode(icua_engine* eng, int32_t session, int32_t n_steps, double* layers_ms, double* head_ms) {
    if (!eng || !layers_ms || !head_ms || n_steps < 1) return fail(eng, ICUA_ERR_INVALID, "bad argument");
    if (eng->cfg.format == ICUA_FMT_F16) return fail(eng, ICUA_ERR_UNSUPPORTED, "f16 engines decode through the batched step");
    icua_status s;
    if ((s = check_ready(eng)) != ICUA_OK) return s;
    Session* S = get_session(eng, session);
    if (!S) return fail(eng, ICUA_ERR_INVALID, "session %d out of range", session);
    if (S->step < 1) return fail(eng, ICUA_ERR_STATE, "decode before prefill");
    if (S->step + n_steps > eng->cfg.max_steps + 1 || S->pos + n_steps + 1 > eng->cfg.max_context)
        return fail(eng, ICUA_ERR_CAPACITY, "%d steps exceed the step or context capacity", n_steps);
    CK(cudaSetDevice(eng->cfg.device));
    if ((s = ensure_graphs(eng, *S)) != ICUA_OK) return s;  // the launch path is decided with the graphs
    const int ms_val = S->step + n_steps, zero = 0;
    CK(cudaMemcpyAsync(&S->st->max_steps, &ms_val, 4, cudaMemcpyHostToDevice, eng->stream));
    CK(cudaMemcpyAsync(&S->st->done, &zero, 4, cudaMemcpyHostToDevice, eng->stream));
    std::vector<cudaEvent_t> ev(3 * n_steps);
    for (auto& e : ev) CK(cudaEventCreate(&e));
    cudaError_t err = cudaSuccess;
    for (int i = 0; i < n_steps && err == cudaSuccess; ++i) {
        cudaEventRecord(ev[3 * i], eng->stream);
        err = record_layers(eng, *S);
        cudaEventRecord(ev[3 * i + 1], eng->stream);
        if (err == cudaSuccess) err = record_head(eng, *S);
        cudaEventRecord(ev[3 * i + 2], eng->stream);
    }
    s = err == cudaSuccess ? sync_and_check(eng, *S) : fail(eng, ICUA_ERR_CUDA, "launch: %s", cudaGetErrorString(err));
    double a = 0, b = 0;
    for (int i = 0; i < n_steps && s == ICUA_OK; ++i) {
        float x = 0, y = 0;
        cudaEventElapsedTime(&x, ev[3 * i], ev[3 * i + 1]);
        cudaEventElapsedTime(&y, ev[3 * i + 1], ev[3 * i + 2]);
        a += x;
        b += y;
    }
    for (auto& e : ev) cudaEventDestroy(e);
    *layers_ms = a;
    *head_ms = b;
    return s;
}

icua_status icua_decode_batch(icua_engine* eng, const int32_t* sessions, int32_t n_sessions, const int32_t* in_tokens,
                              int32_t steps, int32_t* out) {
    return decode_batch_impl(eng, sessions, n_sessions, in_tokens, steps, out);
}

static icua_status decode_batch_impl(icua_engine* eng, const int32_t* sessions, int32_t n_sessions,
                                     const int32_t* in_tokens, int32_t steps, int32_t* out) {
    if (!eng || !sessions || !out) return fail(eng, ICUA_ERR_INVALID, "null argument");
    icua_status s;
    if ((s = check_ready(eng)) != ICUA_OK) return s;
    if (n_sessions < 1 || n_sessions > eng->cfg.max_pass)
        return fail(eng, ICUA_ERR_CAPACITY, "%d sessions per batch (1 .. max_pass %d)", n_sessions, eng->cfg.max_pass);
    if (eng->cfg.vocab % TC_BM) return fail(eng, ICUA_ERR_UNSUPPORTED, "batched decode needs vocab %% 128 == 0");
    if (steps <= 0) return ICUA_OK;
    std::vector<int> key(sessions, sessions + n_sessions);
    {
        std::vector<int> sorted = key;
        std::sort(sorted.begin(), sorted.end());
        if (std::adjacent_find(sorted.begin(), sorted.end()) != sorted.end())
            return fail(eng, ICUA_ERR_INVALID, "a session appears twice in the batch");
    }
    for (int i = 0; i < n_sessions; ++i) {
        Session* S = get_session(eng, key[i]);
        if (!S) return fail(eng, ICUA_ERR_INVALID, "session %d out of range", key[i]);
        if (in_tokens && (in_tokens[i] < 0 || in_tokens[i] >= eng->cfg.vocab))
            return fail(eng, ICUA_ERR_INVALID, "token %d out of range", in_tokens[i]);
        if (!in_tokens && S->step < 1) return fail(eng, ICUA_ERR_STATE, "session %d has no token to continue from", key[i]);
        if (S->pos + steps + eng->cfg.steps_per_graph >= eng->cfg.max_context)
            return fail(eng, ICUA_ERR_CAPACITY, "session %d: context %d + %d exceeds max_context", key[i], S->pos, steps);
    }
    CK(cudaSetDevice(eng->cfg.device));
    const int spg = eng->cfg.steps_per_graph;
    if ((s = ensure_tc_order(eng)) != ICUA_OK) return s;
    if (key != eng->batch_key) {
        drop_batch_graphs(eng);
        long long ctx_sum = 0;
        for (int i = 0; i < n_sessions; ++i) ctx_sum += get_session(eng, key[i])->pos;
        eng->batch_ctx = (int)(ctx_sum / n_sessions);
        CK(cudaMemcpy(eng->batch_rows, key.data(), (size_t)n_sessions * 4, cudaMemcpyHostToDevice));
        if (eng->batch_logits_rows > 0 && eng->batch_logits_rows < n_sessions)
            return fail(eng, ICUA_ERR_CAPACITY, "batch logits capture holds %d rows", eng->batch_logits_rows);
        if ((s = build_batch_graph(eng, n_sessions, 1, &eng->g_batch1)) != ICUA_OK) return s;
        if (steps >= spg && (s = build_batch_graph(eng, n_sessions, spg, &eng->g_batchn)) != ICUA_OK) return s;
        eng->batch_key = key;
    } else if (steps >= spg && !eng->g_batchn) {
        if ((s = build_batch_graph(eng, n_sessions, spg, &eng->g_batchn)) != ICUA_OK) return s;
    }
    // per-session step budget: each session runs until it has `steps` more tokens (or stops)
    std::vector<int> base(n_sessions);
    for (int i = 0; i < n_sessions; ++i) {
        Session* S = get_session(eng, key[i]);
        if (S->step + steps > eng->cfg.max_steps) S->step = 0;  // wrap the output slots, as icua_decode_step
        base[i] = S->step;
        struct {
            int step, done, max_steps, eos0, eos1, stop_on_eos;
        } head = {S->step, 0, S->step + steps, eng->eos0, eng->eos1, eng->stop_on_eos};
        CK(cudaMemcpy(&S->st->step, &head, sizeof head, cudaMemcpyHostToDevice));
        if (in_tokens) CK(cudaMemcpyAsync(&S->st->cur_token, &in_tokens[i], 4, cudaMemcpyHostToDevice, eng->stream));
    }
    const int zero = 0;
    CK(cudaMemcpyAsync(eng->gemm_err, &zero, 4, cudaMemcpyHostToDevice, eng->stream));
    const auto t0 = std::chrono::steady_clock::now();
    CK(cudaEventRecord(eng->ev[2], eng->stream));
    int launched = 0;
    while (launched + spg <= steps) {
        CK(cudaGraphLaunch(eng->g_batchn, eng->stream));
        launched += spg;
    }
    while (launched < steps) {
        CK(cudaGraphLaunch(eng->g_batch1, eng->stream));
        launched += 1;
    }
    CK(cudaEventRecord(eng->ev[3], eng->stream));
    CK(cudaStreamSynchronize(eng->stream));
    int gerr = 0;
    CK(cudaMemcpy(&gerr, eng->gemm_err, 4, cudaMemcpyDeviceToHost));
    if (gerr) {
        eng->failed = true;
        return fail(eng, ICUA_ERR_TIMEOUT, "a bounded device wait gave up in the batched step (flags 0x%x)", gerr);
    }
    float ms = 0.f;
    cudaEventElapsedTime(&ms, eng->ev[2], eng->ev[3]);
    int total = 0;
    for (int i = 0; i < n_sessions; ++i) {
        Session* S = get_session(eng, key[i]);
        if ((s = sync_and_check(eng, *S)) != ICUA_OK) return s;
        const int got = S->step - base[i];
        std::vector<int32_t> toks(steps, -1);
        if (got > 0) CK(cudaMemcpy(toks.data(), S->out_tokens + base[i], (size_t)got * 4, cudaMemcpyDeviceToHost));
        bool stopped = false;
        for (int t = 0; t < steps; ++t) {
            if (stopped || t >= got) {
                out[(size_t)i * steps + t] = -1;
                continue;
            }
            out[(size_t)i * steps + t] = toks[t];
            if (eng->stop_on_eos && (toks[t] == eng->eos0 || toks[t] == eng->eos1)) stopped = true;
            else ++total;
        }
    }
    if (eng->batch_logits_host && eng->batch_logits)
        CK(cudaMemcpy(eng->batch_logits_host, eng->batch_logits, (size_t)n_sessions * eng->cfg.vocab * 4,
                      cudaMemcpyDeviceToHost));
    eng->timing.decode_ms = ms;
    eng->timing.generated_tokens = total;
    eng->timing.total_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return ICUA_OK;
}

icua_status icua_capture_batch_logits(icua_engine* eng, float* host_out, int32_t n_rows) {
    if (!eng) return fail(nullptr, ICUA_ERR_INVALID, "null engine");
    CK(cudaSetDevice(eng->cfg.device));
    drop_batch_graphs(eng);  // the graphs bake the logits pointer
    if (!host_out || n_rows <= 0) {
        eng->batch_logits_host = nullptr;
        eng->batch_logits_rows = 0;
        eng->batch_logits = nullptr;  // the allocation stays with the engine
        return ICUA_OK;
    }
    if (n_rows > eng->cfg.max_pass) return fail(eng, ICUA_ERR_CAPACITY, "%d rows (max_pass %d)", n_rows, eng->cfg.max_pass);
    if (n_rows > eng->batch_logits_cap) {  // grow only: re-enabling reuses the buffer
        if (eng->batch_logits_buf) {
            CK(cudaStreamSynchronize(eng->stream));
            auto& A = eng->allocations;
            A.erase(std::remove(A.begin(), A.end(), (void*)eng->batch_logits_buf), A.end());
            cudaFree(eng->batch_logits_buf);
            eng->batch_logits_buf = nullptr;
            eng->batch_logits_cap = 0;
        }
        icua_status s;
        if ((s = dalloc_t(eng, &eng->batch_logits_buf, (size_t)n_rows * eng->cfg.vocab)) != ICUA_OK) return s;
        eng->batch_logits_cap = n_rows;
    }
    eng->batch_logits = eng->batch_logits_buf;
    eng->batch_logits_host = host_out;
    eng->batch_logits_rows = n_rows;
    return ICUA_OK;
}

icua_status icua_generate(icua_engine* eng, int32_t session, const int32_t* tokens, int32_t n, const icua_visual* vis,
                          int32_t max_new, int32_t write_first_logits, int32_t* out, int32_t* n_out) {
    if (!eng || !tokens || !out || !n_out) return fail(eng, ICUA_ERR_INVALID, "null argument");
    const auto t0 = std::chrono::steady_clock::now();
    Session* S = get_session(eng, session);
    if (!S) return fail(eng, ICUA_ERR_INVALID, "session %d out of range", session);
    // System-prompt prefix cache (reference Engine.swift:719-738): when the tokens before the
    // visual block equal those of this session's previous call, their K/V rows are still valid
    // and the prefill starts at the visual block.
    int vis_off = -1;
    for (int i = 0; i < n; ++i)
        if (tokens[i] == IMAGE_PAD_ID) {
            vis_off = i;
            break;
        }
    const bool use_cache = eng->prefix_cache && vis_off > 0 && vis != nullptr;
    const bool hit = use_cache && S->prefix_valid && (int)S->prefix.size() == vis_off &&
                     std::equal(S->prefix.begin(), S->prefix.end(), tokens);
    icua_status s = reset_session_impl(eng, session, hit);
    if (s != ICUA_OK) return s;
    int first = 0;
    if (hit) {
        S->pos = vis_off;  // rows [0, vis_off) of the cache are the prefix's
        if ((s = icua_prefill(eng, session, tokens + vis_off, n - vis_off, vis, write_first_logits, &first)) != ICUA_OK)
            return s;
    } else {
        S->prefix_valid = false;
        if ((s = icua_prefill(eng, session, tokens, n, vis, write_first_logits, &first)) != ICUA_OK) return s;
        if (use_cache) {
            S->prefix.assign(tokens, tokens + vis_off);
            S->prefix_valid = true;
        }
    }
    *n_out = 0;
    if (max_new <= 0) return ICUA_OK;
    if (eng->stop_on_eos && (first == eng->eos0 || first == eng->eos1)) {
        eng->timing.decode_ms = 0;
        eng->timing.generated_tokens = 0;
    } else {
        out[0] = first;
        int m = 0;
        if (max_new > 1) {
            if ((s = icua_decode(eng, session, max_new - 1, out + 1, &m)) != ICUA_OK) return s;
        } else {
            eng->timing.decode_ms = 0;
        }
        *n_out = 1 + m;
        eng->timing.generated_tokens = 1 + m;
    }
    eng->timing.total_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return ICUA_OK;
}

icua_status icua_get_logits(icua_engine* eng, float* host_out) {
    if (!eng || !host_out) return fail(eng, ICUA_ERR_INVALID, "null argument");
    CK(cudaSetDevice(eng->cfg.device));
    CK(cudaMemcpy(host_out, eng->logits, (size_t)eng->cfg.vocab * 4, cudaMemcpyDeviceToHost));
    return ICUA_OK;
}

icua_status icua_get_timing(icua_engine* eng, icua_timing* out) {
    if (!eng || !out) return fail(eng, ICUA_ERR_INVALID, "null argument");
    *out = eng->timing;
    return ICUA_OK;
}

// ---- kernel-level entry points ------------------------------------------------------------------
icua_status icua_gemv(int32_t fmt, int32_t n_rows, int32_t k, const void* packed, const void* x, int32_t x_dtype,
                      float* y, void* stream) {
    icua_engine* eng = nullptr;
    if (!packed || !x || !y) return fail(nullptr, ICUA_ERR_INVALID, "null argument");
    if ((fmt != ICUA_FMT_Q4S && fmt != ICUA_FMT_Q8) || n_rows < 16 || n_rows % 16 || k < 1024 || k % 1024 ||
        k > 6144 || (x_dtype != 0 && x_dtype != 1))
        return fail(nullptr, ICUA_ERR_INVALID, "unsupported gemv shape or type (rows %% 16, k %% 1024, k <= 6144)");
    CK(set_smem_attrs());
    int dev = 0, n_sm = 0;
    CK(cudaGetDevice(&dev));
    CK(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
    Matrix m;
    setup_matrix(m, fmt, n_rows, k, n_sm);
    if (m.stream && fmt == ICUA_FMT_Q4S)
        return fail(nullptr, ICUA_ERR_INVALID, "q4s gemv supports up to %d rows", 16 * SMALL_MAX_TILES * n_sm);
    GemvParams p{};
    p.w = (const uint8_t*)packed;
    p.n_rows = n_rows;
    p.k = k;
    p.upt = k / 64;
    p.n_tiles = m.n_tiles;
    p.n_slots = m.n_slots;
    p.chunk = m.chunk;
    p.in_mode = x_dtype == 0 ? IN_F32 : IN_BF16;
    p.x = x;
    p.out = y;
    p.st = nullptr;
    cudaStream_t s = (cudaStream_t)stream;
    const bool small = k <= 2048;
    cudaError_t err;
    const bool f32 = x_dtype == 0;
    if (fmt == ICUA_FMT_Q4S) {
        if (small)
            err = f32 ? launch_gemv<FMT_Q4S, EPI_STORE, 2048, false, IN_F32>(m, p, s, false)
                      : launch_gemv<FMT_Q4S, EPI_STORE, 2048, false, IN_BF16>(m, p, s, false);
        else
            err = f32 ? launch_gemv<FMT_Q4S, EPI_STORE, 6144, false, IN_F32>(m, p, s, false)
                      : launch_gemv<FMT_Q4S, EPI_STORE, 6144, false, IN_BF16>(m, p, s, false);
    } else {
        if (!small) return fail(nullptr, ICUA_ERR_INVALID, "q8 gemv supports k <= 2048");
        err = f32 ? launch_gemv<FMT_Q8, EPI_STORE, 2048, true, IN_F32>(m, p, s, false)
                  : launch_gemv<FMT_Q8, EPI_STORE, 2048, true, IN_BF16>(m, p, s, false);
    }
    CK(err);
    return ICUA_OK;
}

// Error flags of standalone GEMM calls made without a caller flag (never read back).
static __device__ int g_tc_gemm_err_sink;

icua_status icua_gemm_q4s(int32_t n_rows, int32_t k, int32_t m_tok, const void* packed, const void* x, float* y,
                          int32_t* err_dev, void* stream) {
    icua_engine* eng = nullptr;
    if (!packed || !x || !y) return fail(nullptr, ICUA_ERR_INVALID, "null argument");
    if (n_rows < TC_BM || n_rows % TC_BM || k < 1024 || k % 1024 || k > 6144 || m_tok < 1 || ((uintptr_t)x & 15))
        return fail(nullptr, ICUA_ERR_INVALID, "unsupported gemm shape (rows %% 128, k %% 1024, k <= 6144, m >= 1, x 16-byte aligned)");
    CK(set_smem_attrs());
    int* errp = err_dev;
    if (!errp) CK(cudaGetSymbolAddress(reinterpret_cast<void**>(&errp), g_tc_gemm_err_sink));
    Matrix m;
    m.dev = (uint8_t*)packed;
    m.fmt = FMT_Q4S;
    m.n_rows = n_rows;
    m.k = k;
    m.n_tiles = n_rows / 16;
    TcGemmParams p = tc_params(m, m_tok, errp);
    p.out = y;
    p.ldo = n_rows;
    CK(launch_tc_gemm<TC_STORE>(x, m_tok, p, (cudaStream_t)stream));
    return ICUA_OK;
}

icua_status icua_dequant_q4s_f16(int32_t n_rows, int32_t k, const void* packed, void* out, void* stream) {
    icua_engine* eng = nullptr;
    if (!packed || !out) return fail(nullptr, ICUA_ERR_INVALID, "null argument");
    if (n_rows < 16 || n_rows % 16 || k < 1024 || k % 1024 || ((uintptr_t)out & 15))
        return fail(nullptr, ICUA_ERR_INVALID, "unsupported shape (rows %% 16, k %% 1024, out 16-byte aligned)");
    const long long n8 = (long long)n_rows * (k / 8);
    CK(launch(dequant_q4s_f16_kernel, (int)std::min<long long>((n8 + 255) / 256, 4096), 256, 0, (cudaStream_t)stream,
              false, (const uint8_t*)packed, (int)n_rows, (int)k, (__half*)out));
    return ICUA_OK;
}

icua_status icua_gemm_f16(int32_t n_rows, int32_t k, int32_t m_tok, const void* w16, const void* x, float* y,
                          int32_t* err_dev, void* stream) {
    icua_engine* eng = nullptr;
    if (!w16 || !x || !y) return fail(nullptr, ICUA_ERR_INVALID, "null argument");
    if (n_rows < TC_BM || n_rows % TC_BM || k < 64 || k % 64 || m_tok < 1 || ((uintptr_t)x & 15) || ((uintptr_t)w16 & 15))
        return fail(nullptr, ICUA_ERR_INVALID, "unsupported gemm shape (rows %% 128, k %% 64, m >= 1, 16-byte aligned)");
    CK(set_smem_attrs());
    int* errp = err_dev;
    if (!errp) CK(cudaGetSymbolAddress(reinterpret_cast<void**>(&errp), g_tc_gemm_err_sink));
    Matrix m;
    m.fmt = FMT_F16;
    m.n_rows = n_rows;
    m.k = k;
    m.n_tiles = n_rows / 16;
    TcGemmParams p = tc_params(m, m_tok, errp);
    p.out = y;
    p.ldo = n_rows;
    const cudaError_t err = launch_tc_gemm<TC_STORE, FMT_F16>(x, m_tok, p, (cudaStream_t)stream, (const __half*)w16);
    CK(err);
    return ICUA_OK;
}

// ---- greedy head: final RMSNorm + tied q8 lm_head GEMV + argmax (reference k_lm_head + k_commit) --
static icua_status greedy_head_args(int32_t vocab, const void* packed, const float* x, int32_t* token, int& n_sm,
                                    Matrix& m) {
    icua_engine* eng = nullptr;
    if (!packed || !x || !token) return fail(nullptr, ICUA_ERR_INVALID, "null argument");
    if (vocab < 16 || vocab % 16) return fail(nullptr, ICUA_ERR_INVALID, "vocab %d is not a positive multiple of 16", vocab);
    CK(set_smem_attrs());
    int dev = 0;
    CK(cudaGetDevice(&dev));
    CK(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
    setup_matrix(m, FMT_Q8, vocab, H, n_sm);
    return ICUA_OK;
}

static icua_status greedy_head_launch(const Matrix& m, const void* packed, const float* x, const float* norm_w,
                                      float* logits, int32_t* token, float* best_v, int* best_i, cudaStream_t s) {
    icua_engine* eng = nullptr;
    GemvParams p{};
    p.w = (const uint8_t*)packed;
    p.n_rows = m.n_rows;
    p.k = H;
    p.upt = H / 64;
    p.n_tiles = m.n_tiles;
    p.n_slots = m.n_slots;
    p.chunk = m.chunk;
    p.in_mode = IN_F32;
    p.x = x;
    p.norm_w = norm_w;
    p.logits = logits;
    p.cta_best_v = best_v;
    p.cta_best_i = best_i;
    p.st = nullptr;
    CK((launch_gemv<FMT_Q8, EPI_LOGITS, 2048, true, IN_F32>(m, p, s, false)));
    CK(launch(argmax_parts_kernel, 1, 256, 0, s, true, (const float*)best_v, (const int*)best_i, m.grid, token));
    return ICUA_OK;
}

uint64_t icua_greedy_head_scratch_bytes(int32_t vocab) {
    int dev = 0, n_sm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    const int grid = std::min(n_sm, std::max(vocab, 16) / 16);
    return (uint64_t)grid * 8;
}

icua_status icua_greedy_head(int32_t vocab, const void* packed, const float* x, const float* norm_w, float* logits,
                             int32_t* token, void* scratch, void* stream) {
    if (!scratch) return fail(nullptr, ICUA_ERR_INVALID, "null scratch");
    int n_sm = 0;
    Matrix m;
    icua_status st = greedy_head_args(vocab, packed, x, token, n_sm, m);
    if (st != ICUA_OK) return st;
    float* best_v = (float*)scratch;
    int* best_i = (int*)((uint8_t*)scratch + (size_t)m.grid * 4);
    return greedy_head_launch(m, packed, x, norm_w, logits, token, best_v, best_i, (cudaStream_t)stream);
}

icua_status icua_set_wait_limit(uint32_t polls) {
    icua_engine* eng = nullptr;
    CK(cudaMemcpyToSymbol(c_norm_wait_polls, &polls, sizeof polls));
    CK(cudaDeviceSynchronize());
    return ICUA_OK;
}

// ---- greedy head without allocation ------------------------------------------------------------
// Some callers cannot call cudaMalloc at all: code running under a host allocator or memory
// pool that owns all device memory, a plugin loaded into a process that forbids allocation
// after start-up, or a real-time loop that must not enter the driver's allocator.  For them the
// per-CTA argmax partials live in this fixed file-scope device array instead of caller scratch.
// Every GPU that loads the library keeps these bytes until the process exits.
constexpr int NOALLOC_MAX_PARTS = 1024;  // CTA partials (8 bytes each): grids up to 1024 CTAs
static __device__ __align__(256) uint8_t g_greedy_head_scratch[NOALLOC_MAX_PARTS * 8];
static std::mutex g_noalloc_mu;
static std::map<CUcontext, void*> g_noalloc_addr;  // device address of the array, per CUDA context

static CUcontext current_context() {
    static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    });
    CUcontext c = nullptr;
    if (fn) fn(&c);
    return c;
}

icua_status icua_greedy_head_noalloc(int32_t vocab, const void* packed, const float* x, const float* norm_w,
                                     float* logits, int32_t* token, void* stream) {
    icua_engine* eng = nullptr;
    int n_sm = 0;
    Matrix m;
    icua_status st = greedy_head_args(vocab, packed, x, token, n_sm, m);
    if (st != ICUA_OK) return st;
    if (m.grid > NOALLOC_MAX_PARTS)
        return fail(nullptr, ICUA_ERR_CAPACITY, "greedy head needs %d CTA partials, the fixed scratch holds %d",
                    m.grid, NOALLOC_MAX_PARTS);
    // The array exists once per CUDA context that loaded this library (not once per device), so its
    // address is kept per context.  Outside stream capture it is looked up on every call, which
    // also picks up a context re-created by cudaDeviceReset; during capture the address of an
    // earlier call in the same context is used, so the first call in a context must come before
    // any capture.
    const CUcontext ctx = current_context();
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    CK(cudaStreamIsCapturing((cudaStream_t)stream, &cap));
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (cap == cudaStreamCaptureStatusNone) {
            void* a = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&a, g_greedy_head_scratch);
            if (e != cudaSuccess)
                return fail(nullptr, ICUA_ERR_CUDA, "cudaGetSymbolAddress(greedy head scratch): %s", cudaGetErrorString(e));
            g_noalloc_addr[ctx] = a;
        }
        auto it = g_noalloc_addr.find(ctx);
        if (it == g_noalloc_addr.end())
            return fail(nullptr, ICUA_ERR_STATE,
                        "first icua_greedy_head_noalloc call in this context is under stream capture; call it once before capturing");
        base = it->second;
    }
    // every partial is written by its CTA before it is read: nothing needs clearing between calls
    float* best_v = (float*)base;
    int* best_i = (int*)((uint8_t*)base + (size_t)NOALLOC_MAX_PARTS * 4);
    return greedy_head_launch(m, packed, x, norm_w, logits, token, best_v, best_i, (cudaStream_t)stream);
}

icua_status icua_dequant(int32_t fmt, int32_t n_rows, int32_t k, const void* packed, float* out, void* stream) {
    icua_engine* eng = nullptr;
    if (!packed || !out || icua_packed_bytes(fmt, n_rows, k) == 0) return fail(nullptr, ICUA_ERR_INVALID, "bad argument");
    cudaStream_t s = (cudaStream_t)stream;
    if (fmt == ICUA_FMT_Q4S)
        dequant_kernel<FMT_Q4S><<<1184, 256, 0, s>>>((const uint8_t*)packed, n_rows, k, out);
    else
        dequant_kernel<FMT_Q8><<<1184, 256, 0, s>>>((const uint8_t*)packed, n_rows, k, out);
    CK(cudaGetLastError());
    return ICUA_OK;
}

// ---- vision encoder ------------------------------------------------------------------------

static cudaError_t vit_gemm(icua_engine* e, int epi, const void* x, int rows_alloc, int m, int n_rows, int k,
                            const void* w16, const void* bias, float* out, int ldo, __half* out_h, int ldh,
                            int gelu_erf) {
    TcGemmParams p{};
    p.n_rows = n_rows;
    p.k = k;
    p.n_tiles = n_rows / 16;
    p.upt = k / 64;
    p.m_tok = m;
    p.out = out;
    p.ldo = ldo;
    p.out_h = out_h;
    p.ldh = ldh;
    p.bias = static_cast<const float*>(bias);
    p.gelu_erf = gelu_erf;
    p.err = e->gemm_err;
    const __half* w = static_cast<const __half*>(w16);
    if (epi == TC_STORE) return launch_tc_gemm<TC_STORE, FMT_F16>(x, rows_alloc, p, e->stream, w);
    if (epi == TC_RESID) return launch_tc_gemm<TC_RESID, FMT_F16>(x, rows_alloc, p, e->stream, w);
    return launch_tc_gemm<TC_GELU, FMT_F16>(x, rows_alloc, p, e->stream, w);
}

// Records the encoder for np patches (grid gh x gw) on the engine stream: patchify, position rows,
// patch embedding, 24 blocks (the DeepStack mergers after blocks 5, 11, 17), final merger.
static cudaError_t record_vision(icua_engine* e, int gh, int gw) {
    const int np = gh * gw, nv = np / 4, NP = e->vit_np_max, NV = NP / 4;
    const int npad = (np + 7) / 8 * 8;  // V^T row length: 16-byte row stride for TMA
    cudaStream_t st = e->stream;
    cudaError_t err;
    // per-head 3-D maps of q, k [16][np][64] and V^T [16][64][np (rows of npad)]; rows past np
    // read as zeros
    CUtensorMap qmap, kmap, vtmap;
    {
        auto enc = tensor_map_encoder();
        if (!enc) return cudaErrorNotSupported;
        const cuuint32_t es[3] = {1, 1, 1};
        const cuuint64_t dq[3] = {VIT_HD, (cuuint64_t)np, VIT_HEADS};
        const cuuint64_t sq[2] = {VIT_HD * 2, (cuuint64_t)np * VIT_HD * 2};
        const cuuint32_t bq[3] = {VIT_HD, VT_BQ, 1}, bk[3] = {VIT_HD, VT_BK, 1};
        const cuuint64_t dv[3] = {(cuuint64_t)np, VIT_HD, VIT_HEADS};
        const cuuint64_t sv[2] = {(cuuint64_t)npad * 2, (cuuint64_t)npad * VIT_HD * 2};
        const cuuint32_t bv[3] = {VT_BK, VIT_HD, 1};
        auto make = [&](CUtensorMap* m, void* base, const cuuint64_t* d, const cuuint64_t* str, const cuuint32_t* b) {
            return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, d, str, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                       CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        };
        if (!make(&qmap, e->vq, dq, sq, bq) || !make(&kmap, e->vk, dq, sq, bk) || !make(&vtmap, e->vvt, dv, sv, bv))
            return cudaErrorInvalidValue;
    }
    auto T = [&](int id) { return e->vit[id]; };
    auto F = [&](int id) { return static_cast<const float*>(e->vit[id]); };
#define VK(...)                                        \
    do {                                               \
        if ((err = (__VA_ARGS__)) != cudaSuccess) return err; \
    } while (0)
    VK(launch(vit_patchify_kernel, np, 256, 0, st, false, (const uint8_t*)e->vrgb, gh, gw, e->vpatch));
    VK(launch(vit_pos_init_kernel, np, 256, 0, st, false, F(2), gh, gw, e->vx));
    VK(launch(vit_rope_table_kernel, (np * 32 + 255) / 256, 256, 0, st, false, np, gw, e->vrope));
    VK(vit_gemm(e, TC_RESID, e->vpatch, NP, np, VIT_HIDDEN, VIT_PATCH_DIM, T(0), T(1), e->vx, VIT_HIDDEN, nullptr, 0, 0));
    const int ds_layer[3] = {5, 11, 17};
    for (int l = 0; l < VIT_LAYERS; ++l) {
        const int b = 3 + l * 12;
        VK(launch(vit_layernorm_kernel, np, 256, 0, st, false, (const float*)e->vx, F(b + 0), F(b + 1), VIT_HIDDEN,
                  e->vxn));
        VK(vit_gemm(e, TC_STORE, e->vxn, NP, np, VIT_QKV, VIT_HIDDEN, T(b + 2), T(b + 3), e->vqkv, VIT_QKV, nullptr, 0, 0));
        VK(launch(vit_qkv_rope_kernel, np, 256, 0, st, false, (const float*)e->vqkv, (const float2*)e->vrope, np,
                  e->vq, e->vk));
        {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((np + 31) / 32, VIT_HIDDEN / 32);
            cfg.blockDim = dim3(32, 8);
            cfg.stream = st;
            VK(cudaLaunchKernelEx(&cfg, vit_vt_kernel, (const float*)e->vqkv, np, npad, e->vvt));
        }
        {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((np + VT_BQ - 1) / VT_BQ, VIT_HEADS);
            cfg.blockDim = dim3(VT_THREADS);
            cfg.dynamicSmemBytes = VitAttnSmem::alloc;
            cfg.stream = st;
            VK(cudaLaunchKernelEx(&cfg, vit_attn_tc_kernel, qmap, kmap, vtmap, np, e->vattn, e->gemm_err));
        }
        VK(vit_gemm(e, TC_RESID, e->vattn, NP, np, VIT_HIDDEN, VIT_HIDDEN, T(b + 4), T(b + 5), e->vx, VIT_HIDDEN, nullptr,
                    0, 0));
        VK(launch(vit_layernorm_kernel, np, 256, 0, st, false, (const float*)e->vx, F(b + 6), F(b + 7), VIT_HIDDEN,
                  e->vxn));
        VK(vit_gemm(e, TC_GELU, e->vxn, NP, np, VIT_FF, VIT_HIDDEN, T(b + 8), T(b + 9), nullptr, 0, e->vh, VIT_FF, 0));
        VK(vit_gemm(e, TC_RESID, e->vh, NP, np, VIT_HIDDEN, VIT_FF, T(b + 10), T(b + 11), e->vx, VIT_HIDDEN, nullptr, 0, 0));
        for (int d = 0; d < 3; ++d) {
            if (l != ds_layer[d]) continue;
            // DeepStack merger d: LayerNorm over the 2x2 merged rows [nv][4096] (views of [np][1024])
            const int m = 3 + VIT_LAYERS * 12 + d * 6;
            VK(launch(vit_layernorm_kernel, nv, 256, 0, st, false, (const float*)e->vx, F(m + 0), F(m + 1), VIT_MERGED,
                      e->vxn));
            VK(vit_gemm(e, TC_GELU, e->vxn, NV, nv, VIT_MERGED, VIT_MERGED, T(m + 2), T(m + 3), nullptr, 0, e->vh,
                        VIT_MERGED, 1));
            VK(vit_gemm(e, TC_STORE, e->vh, NV, nv, H, VIT_MERGED, T(m + 4), T(m + 5), e->deepstack[d], H, nullptr, 0, 0));
        }
    }
    // final merger: LayerNorm per patch, then the merged rows [nv][4096]
    const int m = 3 + VIT_LAYERS * 12 + 3 * 6;
    VK(launch(vit_layernorm_kernel, np, 256, 0, st, false, (const float*)e->vx, F(m + 0), F(m + 1), VIT_HIDDEN, e->vxn));
    VK(vit_gemm(e, TC_GELU, e->vxn, NV, nv, VIT_MERGED, VIT_MERGED, T(m + 2), T(m + 3), nullptr, 0, e->vh, VIT_MERGED, 1));
    VK(vit_gemm(e, TC_STORE, e->vh, NV, nv, H, VIT_MERGED, T(m + 4), T(m + 5), e->pooler, H, nullptr, 0, 0));
#undef VK
    return cudaSuccess;
}

icua_status icua_encode_vision(icua_engine* eng, const uint8_t* rgb, int32_t width, int32_t height, float* pooler_out,
                               float* deepstack_out, int32_t* n_vis_out) {
    if (!eng || !rgb) return fail(eng, ICUA_ERR_INVALID, "null argument");
    if (eng->failed) return fail(eng, ICUA_ERR_STATE, "engine failed earlier: %s", eng->err.c_str());
    if (eng->vit_count < ICUA_VIT_TENSORS)
        return fail(eng, ICUA_ERR_STATE, "vision encoder tensors missing (%d of %d)", eng->vit_count, ICUA_VIT_TENSORS);
    if (width < 32 || height < 32 || width % 32 || height % 32)
        return fail(eng, ICUA_ERR_INVALID, "image %dx%d: sides must be positive multiples of 32", width, height);
    const int gh = height / 16, gw = width / 16, np = gh * gw, nv = np / 4;
    if (nv > eng->cfg.max_pass)
        return fail(eng, ICUA_ERR_CAPACITY, "%d visual tokens exceed max_pass %d", nv, eng->cfg.max_pass);
    CK(cudaSetDevice(eng->cfg.device));
    if (!eng->vit_np_max) {
        const size_t NP = (size_t)eng->cfg.max_pass * 4;
        icua_status s;
        if ((s = dalloc_t(eng, &eng->vrgb, NP * VIT_PATCH_DIM)) != ICUA_OK ||
            (s = dalloc_t(eng, &eng->vpatch, NP * VIT_PATCH_DIM)) != ICUA_OK ||
            (s = dalloc_t(eng, &eng->vx, NP * VIT_HIDDEN)) != ICUA_OK ||
            (s = dalloc_t(eng, &eng->vxn, NP * VIT_HIDDEN)) != ICUA_OK ||
            (s = dalloc_t(eng, &eng->vqkv, NP * VIT_QKV)) != ICUA_OK ||
            (s = dalloc_t(eng, &eng->vq, NP * VIT_HIDDEN)) != ICUA_OK ||
            (s = dalloc_t(eng, &eng->vk, NP * VIT_HIDDEN)) != ICUA_OK ||
            (s = dalloc_t(eng, &eng->vattn, NP * VIT_HIDDEN)) != ICUA_OK ||
            (s = dalloc_t(eng, &eng->vh, NP * VIT_FF)) != ICUA_OK ||
            (s = dalloc_t(eng, &eng->vrope, NP * 32)) != ICUA_OK ||
            (s = dalloc_t(eng, &eng->vvt, (NP + 8) * VIT_HIDDEN)) != ICUA_OK)
            return s;
        cudaMemsetAsync(eng->vxn, 0, NP * VIT_HIDDEN * sizeof(__half), eng->stream);  // rows past a call's patches read by TMA
        cudaMemsetAsync(eng->vh, 0, NP * VIT_FF * sizeof(__half), eng->stream);
        cudaMemsetAsync(eng->vattn, 0, NP * VIT_HIDDEN * sizeof(__half), eng->stream);
        cudaMemsetAsync(eng->vpatch, 0, NP * VIT_PATCH_DIM * sizeof(__half), eng->stream);
        eng->vit_np_max = (int)NP;
    }
    CK(cudaMemcpyAsync(eng->vrgb, rgb, (size_t)np * VIT_PATCH_DIM, cudaMemcpyHostToDevice, eng->stream));
    const int zero = 0;
    CK(cudaMemcpyAsync(eng->gemm_err, &zero, 4, cudaMemcpyHostToDevice, eng->stream));
    CK(cudaEventRecord(eng->ev[0], eng->stream));
    const cudaError_t e2 = record_vision(eng, gh, gw);
    if (e2 != cudaSuccess) return fail(eng, ICUA_ERR_CUDA, "vision launch: %s", cudaGetErrorString(e2));
    CK(cudaEventRecord(eng->ev[1], eng->stream));
    CK(cudaStreamSynchronize(eng->stream));
    int gerr = 0;
    CK(cudaMemcpy(&gerr, eng->gemm_err, 4, cudaMemcpyDeviceToHost));
    if (gerr) {
        eng->failed = true;
        return fail(eng, ICUA_ERR_TIMEOUT, "a bounded device wait gave up in the vision encoder (flags 0x%x)", gerr);
    }
    float ms = 0.f;
    cudaEventElapsedTime(&ms, eng->ev[0], eng->ev[1]);
    eng->timing.vision_ms = ms;
    eng->vis_rows = nv;
    if (pooler_out) CK(cudaMemcpy(pooler_out, eng->pooler, (size_t)nv * H * 4, cudaMemcpyDeviceToHost));
    if (deepstack_out)
        for (int d = 0; d < 3; ++d)
            CK(cudaMemcpy(deepstack_out + (size_t)d * nv * H, eng->deepstack[d], (size_t)nv * H * 4,
                          cudaMemcpyDeviceToHost));
    if (n_vis_out) *n_vis_out = nv;
    return ICUA_OK;
}

icua_status icua_generate_rgb(icua_engine* eng, int32_t session, const uint8_t* rgb, int32_t width, int32_t height,
                              const int32_t* tokens, int32_t n, int32_t max_new, int32_t write_first_logits,
                              int32_t* out_tokens, int32_t* n_out) {
    int32_t nv = 0;
    icua_status s = icua_encode_vision(eng, rgb, width, height, nullptr, nullptr, &nv);
    if (s != ICUA_OK) return s;
    const float vision_ms = (float)eng->timing.vision_ms;
    icua_visual v{};
    v.pooler = nullptr;
    v.n_vis = nv;
    v.llm_h = height / 32;
    v.llm_w = width / 32;
    s = icua_generate(eng, session, tokens, n, &v, max_new, write_first_logits, out_tokens, n_out);
    eng->timing.vision_ms = vision_ms;
    return s;
}

}  // extern "C"
