/*
 * icua.h - C ABI of the B200 (sm_100a) engine for the Qwen3VLTextModel token loop.
 *
 * This header is the drop-in boundary: it replaces the Metal-typed surface of the reference's
 * `public final class Engine` (Sources/Engine/Engine.swift) and is the counterpart of the
 * reference's C target `Sources/CShim` (Package.swift:14).  Plain pointers, sizes and status
 * codes only; no CUDA or torch types appear in any signature.
 *
 * Errors: every call returns an icua_status; on failure a message is available from
 * icua_last_error() (per engine) or icua_global_error() (calls without an engine).  This
 * replaces the reference's `throw EngineError(String)` (Sources/Engine/ModelFile.swift:158-161).
 * Threading: one engine per thread; calls on one engine are not reentrant (the reference engine
 * is single-queue and synchronous, Engine.swift:65, 790).
 */
#ifndef ICUA_H
#define ICUA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    ICUA_OK = 0,
    ICUA_ERR_INVALID = 1,     /* bad argument (null pointer, size, id, token out of range) */
    ICUA_ERR_CUDA = 2,        /* a CUDA runtime call failed */
    ICUA_ERR_OOM = 3,         /* device or host allocation failed */
    ICUA_ERR_IO = 4,          /* model file could not be opened, mapped or read */
    ICUA_ERR_FORMAT = 5,      /* model file header or tensor table mismatch */
    ICUA_ERR_STATE = 6,       /* call out of order (weights missing, engine failed) */
    ICUA_ERR_CAPACITY = 7,    /* context, pass, steps or session capacity exceeded */
    ICUA_ERR_UNSUPPORTED = 8, /* weight format not implemented by the kernels */
    ICUA_ERR_TIMEOUT = 9      /* a bounded device-side wait gave up (kernel error flag set) */
} icua_status;

/* Weight formats.  0..2 are the reference WeightFormat raw values (ModelFile.swift:6-9):
 * f16, q8 (symmetric int8, groups of 32, fp16 scale), q4 (affine int4, groups of 64, fp16
 * scale+bias).  3 is the BASELINE format: decoder matrices symmetric int4 in groups of 32 with
 * an fp16 scale (offset-binary nibbles, u = q + 8) and the tied embedding / lm_head in q8. */
enum { ICUA_FMT_F16 = 0, ICUA_FMT_Q8 = 1, ICUA_FMT_Q4 = 2, ICUA_FMT_Q4S = 3 };

/* KV cache element type.  The reference stores fp16 (Shaders.swift:776-783). */
enum { ICUA_KV_F16 = 0, ICUA_KV_BF16 = 1 };

/* Tensor ids: the reference TensorID numbering (ModelFile.swift:62-111). */
enum {
    ICUA_TID_EMBED = 315,
    ICUA_TID_EMBED_SB = 316,
    ICUA_TID_FINAL_NORM = 317,
    ICUA_TID_LAYER_BASE = 318,
    ICUA_TID_PER_LAYER = 14,
    ICUA_SLOT_ATTN_NORM = 0, ICUA_SLOT_WQKV = 1, ICUA_SLOT_WQKV_SB = 2, ICUA_SLOT_Q_NORM = 3,
    ICUA_SLOT_K_NORM = 4, ICUA_SLOT_WO = 5, ICUA_SLOT_WO_SB = 6, ICUA_SLOT_MLP_NORM = 7,
    ICUA_SLOT_WGU = 8, ICUA_SLOT_WGU_SB = 9, ICUA_SLOT_WD = 10, ICUA_SLOT_WD_SB = 11,
    ICUA_TENSOR_COUNT = 710
};

typedef struct icua_engine icua_engine;

/* Engine configuration; mirrors Engine.init(modelPath:maxContext:maxPass:maxSteps:...)
 * (Engine.swift:54-55).  n_layers and vocab are the model's (28, 151936); smaller values are
 * accepted for tests. */
typedef struct {
    int32_t device;         /* CUDA device ordinal */
    int32_t n_layers;       /* decoder layers (28) */
    int32_t vocab;          /* vocabulary rows of the tied embedding (151936) */
    int32_t max_context;    /* KV positions per session (reference default 2048) */
    int32_t max_pass;       /* max prompt tokens per prefill call (reference default 512) */
    int32_t max_steps;      /* max generated tokens per call (reference default 256) */
    int32_t max_sessions;   /* KV caches held (1 for the reference's single session) */
    int32_t format;         /* ICUA_FMT_* */
    int32_t kv_dtype;       /* ICUA_KV_* */
    int32_t steps_per_graph;/* decode steps captured per CUDA graph launch (>=1) */
    int32_t prefill_gemm_min;/* prompts whose rows before the last number at least this many run
                              * through the tensor-core GEMM path; shorter ones through the decode
                              * kernels row by row.  0 = always row by row.  Default 64. */
} icua_config;

/* Mirrors Engine.Timing (Engine.swift:44-51); times are device times from CUDA events. */
typedef struct {
    double vision_ms;       /* always 0: the vision encoder is outside this engine */
    double prefill_ms;
    double decode_ms;
    double total_ms;        /* host wall time of the call */
    int32_t prefill_tokens;
    int32_t generated_tokens;
} icua_timing;

/* Optional visual inputs for a prompt (replace the ViT outputs poolerBuf / deepstackBufs,
 * Engine.swift:20-21).  Host fp32 arrays, row-major [n_vis, 2048]; deepstack[i] may be NULL.
 * pooler == NULL takes the rows that the last icua_encode_vision left on the device. */
typedef struct {
    const float* pooler;
    const float* deepstack[3];
    int32_t n_vis;
    int32_t llm_h, llm_w;   /* merged grid; n_vis == llm_h * llm_w */
} icua_visual;

/* ---- lifecycle -------------------------------------------------------------------------- */
void icua_default_config(icua_config* cfg);
icua_status icua_engine_create(const icua_config* cfg, icua_engine** out);
void icua_engine_destroy(icua_engine* eng);
const char* icua_last_error(const icua_engine* eng);
const char* icua_global_error(void);

/* Loads an .icua model file (ModelFile.swift:113-156 layout: "ICU1", version 1, format,
 * tensor count, (offset,size) table, 256-byte aligned tensors).  Replaces the mmap + MTLBuffer
 * wrap of Engine.init (Engine.swift:62-77). */
icua_status icua_engine_load_file(icua_engine* eng, const char* path);

/* Sets one tensor from host bytes laid out as in the .icua file for that tensor id (row-major
 * codes / packed nibbles, and the SB tensor with the scales).  Matrices are repacked and
 * uploaded once both the codes and the SB tensor of a matrix are present. */
icua_status icua_engine_set_tensor(icua_engine* eng, int32_t tensor_id, const void* data, uint64_t bytes);

/* Returns ICUA_OK when every tensor the kernels need is resident on the device. */
icua_status icua_engine_ready(icua_engine* eng);

/* ---- the token loop (Engine.generateVision without the ViT, Engine.swift:696-827) ---------- */
/* eos tokens (Engine.swift:12) and whether generation stops on them (reference: yes). */
icua_status icua_set_eos(icua_engine* eng, int32_t eos0, int32_t eos1, int32_t stop_on_eos);

/* Prompt pass for `session`: appends tokens[0..n) at the session's current position (0 after a
 * reset), runs all layers and produces the first generated token.  `visual` may be NULL; when
 * given, IMAGE_PAD (151655) rows take pooler rows, DeepStack rows are added after layers 0..2
 * and positions follow the 3D M-RoPE layout (Engine.swift:254-298).  write_logits copies the
 * first-token logits to an internal buffer readable with icua_get_logits. */
icua_status icua_prefill(icua_engine* eng, int32_t session, const int32_t* tokens, int32_t n,
                         const icua_visual* visual, int32_t write_logits, int32_t* first_token);

/* Greedy decode of up to `max_new` tokens after a prefill; out_tokens has room for max_new.
 * Stops early on EOS when enabled.  *n_out receives the count (EOS not included, as
 * Engine.swift:808-816). */
icua_status icua_decode(icua_engine* eng, int32_t session, int32_t max_new, int32_t* out_tokens,
                        int32_t* n_out);

/* One decode step driven from the host: the step input token is copied from host memory and the
 * generated token is copied back (used by callers that interleave their own logic per token).
 * The step's logits are kept for icua_get_logits. */
icua_status icua_decode_step(icua_engine* eng, int32_t session, int32_t in_token, int32_t* out_token);

/* Device memory the engine holds (bytes of its own allocations: weights, KV caches, scratch). The
 * tensor-core tile order copy of the quantised matrices, read only by batched decode, is allocated
 * on the first icua_decode_batch.  0 for NULL. */
uint64_t icua_device_bytes(const icua_engine* eng);

/* CTAs per cluster of the decode attention kernel with the o-projection folded in (q4s engines:
 * one cluster per kv head, 16 when eight clusters of 16 fit on the device at once, else 8), or 0
 * when the engine launches the o-proj GEMV on its own (other formats, grammar-commit passes,
 * ICUA_ATTN_O=0).  No counterpart in the reference (a query of this build's launch shape).  0 for
 * NULL. */
int32_t icua_attn_o_cluster(const icua_engine* eng);

/* Kernels one decode step launches on this engine: 3 for q4s engines on the persistent layers
 * kernel (all layers in one cooperative launch, then the lm_head GEMV and the commit), else
 * 5 x n_layers + 2 (one launch per projection / attention, lm_head, commit).  0 for NULL. */
int32_t icua_decode_kernels_per_step(const icua_engine* eng);

/* Measurement: decodes n_steps greedy steps of `session` (after a prefill, like icua_decode) with
 * every launch issued directly on the engine stream and CUDA events around each step's decoder
 * layers and around its lm_head + commit; *layers_ms / *head_ms receive the summed device times.
 * The tokens are committed as by icua_decode.  Used by the benchmark for per-kernel rooflines. */
icua_status icua_profile_decode(icua_engine* eng, int32_t session, int32_t n_steps, double* layers_ms,
                                double* head_ms);

/* Batched greedy decode (the serving counterpart of icua_decode): every step
 * decodes one token for each of n_sessions sessions together -- tensor-core GEMMs over the session
 * rows, per-session attention over each session's own cache, the tied lm_head with a per-row
 * argmax -- for `steps` steps.  in_tokens: n_sessions input tokens, or NULL to continue each session
 * from its last token (the session must have been prefilled).  out: [n_sessions][steps] tokens; a
 * session that stops (EOS when stop_on_eos, as icua_decode) has -1 after its EOS token.
 * n_sessions <= max_pass; sessions distinct.  The arithmetic is the prefill path's (fp16 operands,
 * fp32 accumulation), so tokens can differ from icua_decode's where two logits nearly tie. */
icua_status icua_decode_batch(icua_engine* eng, const int32_t* sessions, int32_t n_sessions,
                              const int32_t* in_tokens, int32_t steps, int32_t* out);
/* The next icua_decode_batch calls copy the last step's fp32 logits [n_rows][vocab] (rows in the
 * call's session order) to host_out; NULL / 0 turns it off. */
icua_status icua_capture_batch_logits(icua_engine* eng, float* host_out, int32_t n_rows);

/* System-prompt KV prefix cache (reference Engine.usePrefixCache, Engine.swift:40, 719-738; on
 * by default): icua_generate keeps the K/V rows of the tokens before the visual block when they
 * equal the previous call's on that session, and prefills from the visual block on.  Any other
 * write to the session's cache (icua_reset_session, icua_inject_kv*) forgets the prefix. */
icua_status icua_set_prefix_cache(icua_engine* eng, int32_t enable);

/* Grammar-guided 2-token commit (reference k_commit, Shaders.swift:1497-1571; off by default,
 * since it changes greedy output).  After each committed token a deterministic syntax token may
 * follow it without a model step: `open` after an `action` word that is the call's first output,
 * `space` after `comma`; the next decode pass runs both tokens through one read of the weights
 * (the reference's dual-token GEMVs, Shaders.swift:529-595) and predicts the token after the pair.
 * `close` ends the call like EOS.  rule == NULL selects the reference's ids (its tokenizer: '('
 * 7, ')' 8, ',' 11, ' ' 220, eight action words).  Applies to icua_generate / icua_prefill +
 * icua_decode on quantized engines (not to icua_decode_step, whose inputs come from the caller,
 * nor to icua_decode_batch); ICUA_ERR_INVALID on f16 engines or ids outside the vocabulary.
 * Session graphs are rebuilt on the next call. */
typedef struct icua_grammar {
    int32_t n_action;   /* 0..8 */
    int32_t action[8];
    int32_t comma, space, open, close;
} icua_grammar;
icua_status icua_set_grammar_commit(icua_engine* eng, int32_t enable, const icua_grammar* rule);

/* Whole call: reset session (keeping a cached prefix), prefill, decode; returns tokens like
 * generateVision. */
icua_status icua_generate(icua_engine* eng, int32_t session, const int32_t* tokens, int32_t n,
                          const icua_visual* visual, int32_t max_new, int32_t write_first_logits,
                          int32_t* out_tokens, int32_t* n_out);

/* ---- vision encoder (reference encodeVision, Engine.swift:317-473) -------------------------
 * Needs the vision tensors of the model file (ids 0..ICUA_VIT_TENSORS-1: fp16 matrices, fp32
 * biases / norms / position table, Convert.swift:99-152); icua_engine_load_file takes them from
 * the file when present, icua_engine_set_tensor at any time.  rgb is RGB8 [height][width][3] with
 * width and height multiples of 32 (16-pixel patches, 2x2 merge) and at most 4 * max_pass patches.
 * The outputs stay on the device as the next prompt's visual rows (use icua_generate_rgb, or pass
 * an icua_visual whose pooler is NULL and whose n_vis, llm_h, llm_w match); pooler_out [n_vis][2048]
 * and deepstack_out [3][n_vis][2048] receive host copies when not NULL.  *n_vis_out = patches / 4. */
enum { ICUA_VIT_TENSORS = 315 };
icua_status icua_encode_vision(icua_engine* eng, const uint8_t* rgb, int32_t width, int32_t height,
                               float* pooler_out, float* deepstack_out, int32_t* n_vis_out);
/* reference generateVision(rgbBytes:width:height:tokens:maxNewTokens:writeFirstLogits:)
 * (Engine.swift:696-827): vision encoder, then icua_generate with the prompt's IMAGE_PAD block
 * (n_vis = width * height / 1024 tokens) taking the encoder's rows. */
icua_status icua_generate_rgb(icua_engine* eng, int32_t session, const uint8_t* rgb, int32_t width, int32_t height,
                              const int32_t* tokens, int32_t n, int32_t max_new, int32_t write_first_logits,
                              int32_t* out_tokens, int32_t* n_out);

/* Resets a session to position 0 (empty KV). */
icua_status icua_reset_session(icua_engine* eng, int32_t session);

/* Fills a session's KV cache with given values (BASELINE config 2 injection): k and v are host
 * fp32 [n_layers][n_pos][8][128]; they are rounded to the cache type.  Position becomes n_pos. */
icua_status icua_inject_kv(icua_engine* eng, int32_t session, const float* k, const float* v, int32_t n_pos);

/* Same as icua_inject_kv but draws the values on the device from N(0,1) with a counter-based
 * generator (seeded), for long contexts where a host array would be large. */
icua_status icua_inject_kv_random(icua_engine* eng, int32_t session, int32_t n_pos, uint64_t seed);

/* Logits of the last step that was asked to write them (fp32 [vocab]). */
icua_status icua_get_logits(icua_engine* eng, float* host_out);
/* Writes logits at every decode step into a host array [max_new][vocab] on the next
 * icua_decode call (parity runs); pass NULL to switch off. */
icua_status icua_capture_step_logits(icua_engine* eng, float* host_out, int32_t capacity_steps);

icua_status icua_get_timing(icua_engine* eng, icua_timing* out);
icua_status icua_session_position(icua_engine* eng, int32_t session, int32_t* pos);

/* ---- kernel-level entry points (device pointers; used by the microbench and the tests) -------- */
/* Packed device size of an [n_rows, k] matrix in format fmt (ICUA_FMT_Q4S, ICUA_FMT_Q8 or the
 * reference's affine ICUA_FMT_Q4, whose "scales" are the (scale, bias) fp16 pairs per 64 columns). */
uint64_t icua_packed_bytes(int32_t fmt, int32_t n_rows, int32_t k);
/* Repacks reference-layout host codes + scales into the device tile layout (host to host). */
icua_status icua_pack_matrix(int32_t fmt, int32_t n_rows, int32_t k, const void* codes,
                             const uint16_t* scales, void* packed_out);
/* y[n_rows] = W x on the device (the decode GEMV kernel with a plain store epilogue); x is fp32 [k]
 * (x_dtype 0) or bf16 [k] (x_dtype 1); k a multiple of 1024 up to 6144; stream is a cudaStream_t
 * or NULL.  No scratch memory: every CTA owns whole 16-row tiles. */
icua_status icua_gemv(int32_t fmt, int32_t n_rows, int32_t k, const void* packed_dev,
                      const void* x_dev, int32_t x_dtype, float* y_dev, void* stream);
/* y[m_tok, n_rows] (fp32, row-major) = x[m_tok, k] (fp16, row-major, 16-byte aligned) W^T, W a q4s
 * matrix in the device tile layout: the tensor-core dequant-GEMM of prefill (tcgen05.mma with
 * TMEM accumulators, TMA-fed activations; weights dequantised as half(q) * half(scale), the rule
 * of the reference prefill GEMM llm_gemm_tile, Shaders.swift:927-1097) with a plain store
 * epilogue.  n_rows a multiple of 128, k a multiple of 1024 up to 6144, m_tok >= 1.  err_dev:
 * optional device int32 OR-ed with error flags when a bounded wait gives up (NULL: not reported). */
icua_status icua_gemm_q4s(int32_t n_rows, int32_t k, int32_t m_tok, const void* packed_dev, const void* x_dev,
                          float* y_dev, int32_t* err_dev, void* stream);
/* The prefill path's two halves: icua_dequant_q4s_f16 writes the row-major fp16 matrix
 * [n_rows, k] with values half(q) * half(scale) (one rounding of the exact product); icua_gemm_f16
 * is the tensor-core GEMM y[m_tok, n_rows] = x w16^T with both operands brought in by TMA (n_rows
 * a multiple of 128, k of 64; 16-byte aligned pointers).  Same accumulation order as
 * icua_gemm_q4s, so the two routes give identical results. */
icua_status icua_dequant_q4s_f16(int32_t n_rows, int32_t k, const void* packed_dev, void* out_dev, void* stream);
icua_status icua_gemm_f16(int32_t n_rows, int32_t k, int32_t m_tok, const void* w16_dev, const void* x_dev,
                          float* y_dev, int32_t* err_dev, void* stream);
/* Greedy head on the device: token = argmax_v (embed_v . RMSNorm(x) * norm_w), the tied q8 lm_head
 * of the reference (k_lm_head + k_commit, Shaders.swift:1452-1547; lowest index wins ties).
 * packed_embed_dev: q8 [vocab, 2048] in the device layout (icua_pack_matrix); x_dev fp32 [2048];
 * norm_w_dev fp32 [2048] or NULL (no norm); logits_dev fp32 [vocab] or NULL; token_dev int32 [1]
 * receives the argmax, or -1 when no logit is finite (NaN / inf in x or norm_w).
 * scratch_dev: icua_greedy_head_scratch_bytes(vocab) bytes of device memory for the per-CTA argmax
 * partials (no initialisation needed). */
uint64_t icua_greedy_head_scratch_bytes(int32_t vocab);
icua_status icua_greedy_head(int32_t vocab, const void* packed_embed_dev, const float* x_dev,
                             const float* norm_w_dev, float* logits_dev, int32_t* token_dev,
                             void* scratch_dev, void* stream);

/* icua_greedy_head for callers that cannot allocate device memory (a host that owns all device
 * memory through its own pool, a plugin that may not call cudaMalloc after start-up, a real-time
 * loop that must stay out of the allocator).  No reference counterpart: the reference engine
 * allocates its pval/pidx buffers at init (Engine.swift:116-117).  Same arguments and results as
 * icua_greedy_head minus the scratch: the per-CTA partials live in a fixed 8 KiB device array of
 * the library (room for 1024 CTA partials; larger grids are rejected with ICUA_ERR_CAPACITY),
 * which every GPU that loads the library keeps until exit (one copy per CUDA context).  Calls
 * made outside stream capture look up that array's address (cudaGetSymbolAddress) in the current
 * context; a call under capture reuses the address an earlier call in the same context found, so
 * make the first call in a context before any stream capture.  Calls on the same device share
 * the array: serialise calls that could overlap on one device, even on different streams.  Calls
 * on different devices do not interfere. */
icua_status icua_greedy_head_noalloc(int32_t vocab, const void* packed_embed_dev, const float* x_dev,
                                     const float* norm_w_dev, float* logits_dev, int32_t* token_dev,
                                     void* stream);

/* Poll limit of the bounded wait in which a decode GEMV waits for the copy of its RMSNorm weights,
 * on the current device (default 4194304).  No reference counterpart: it exists so that tests can
 * make that wait give up (polls = 0) and check the timeout report -- the kernel flags the step,
 * still waits for its copy with the default bound, the engine call returns ICUA_ERR_TIMEOUT and
 * later calls on that engine ICUA_ERR_STATE.  Set it back before running other work. */
icua_status icua_set_wait_limit(uint32_t polls);

/* Bit-exact dequantization of a packed device matrix to fp32 row-major [n_rows, k]. */
icua_status icua_dequant(int32_t fmt, int32_t n_rows, int32_t k, const void* packed_dev, float* out_dev,
                         void* stream);

/* ---- host quantizers (reference Converter, Convert.swift:208-320) --------------------------- */
/* q8: codes int8 [rows, cols], scales fp16 bits [rows, cols/32] (Convert.swift:215-241). */
icua_status icua_quantize_q8(const float* w, int32_t rows, int32_t cols, int8_t* codes, uint16_t* scales);
/* q4s: packed nibbles [rows, cols/2] (u = q + 8, even index low), scales [rows, cols/32]. */
icua_status icua_quantize_q4s(const float* w, int32_t rows, int32_t cols, uint8_t* packed, uint16_t* scales);

#ifdef __cplusplus
}
#endif
#endif /* ICUA_H */
