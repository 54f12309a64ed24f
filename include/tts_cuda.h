/*
 * tts_cuda.h — C ABI of the B200 (sm_100a) backend for dream-tts's qwen3tts hot path.
 *
 * Each entry point stands in for one operator of the `tts-nn` crate that crates/qwen3tts calls
 * (the reference's plugin surface: candle CustomOps with cpu_fwd/metal_fwd arms), or for the
 * qwen3tts decode step built from them. The citation above each declaration names the
 * reference interface it replaces (paths within the dream-tts project).
 *
 * Conventions
 *  - Plain C types only. Every device pointer is caller-owned, 16-byte aligned, row-major and
 *    contiguous unless stated; `stream` is a cudaStream_t passed as void* (NULL = legacy).
 *  - f16 buffers are IEEE binary16 (`void*`), f32 buffers `float*`.
 *  - Calls are stream-ordered and return without synchronising. A context serialises its
 *    scratch buffers: use one stream per context (the reference's dispatcher is single-stream
 *    too, crates/tts-nn/src/lib.rs:76-88).
 *  - Every function returns a tts_status; on failure tts_last_error() (thread-local) names the
 *    operator and the violated constraint, the way the reference's `bail!`s do. There is no
 *    CPU fallback: a shape the kernels do not take returns TTS_ERR_UNSUPPORTED_SHAPE.
 */
#ifndef TTS_CUDA_H
#define TTS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TTS_CUDA_ABI_VERSION 1

#if defined(__GNUC__)
#define TTS_API __attribute__((visibility("default")))
#else
#define TTS_API
#endif

typedef enum tts_status {
  TTS_OK = 0,
  TTS_ERR_INVALID_ARG = 1,
  TTS_ERR_UNSUPPORTED_SHAPE = 2,
  TTS_ERR_CUDA = 3,
  TTS_ERR_TIMEOUT = 4, /* a bounded device-side wait gave up; results are not valid */
  TTS_ERR_OOM = 5
} tts_status;

typedef struct tts_ctx tts_ctx;
typedef struct tts_stack tts_stack;
typedef struct tts_graph tts_graph;

TTS_API int tts_abi_version(void);
/* Last error message of the calling thread ("" when none). */
TTS_API const char* tts_last_error(void);
/* Per-CTA timeline records of the kernels run on the current device since the last reset
 * (tracing; only in the library built with `build.py --timeline`, which defines TTS_TIMELINE):
 * copies up to `cap` records of 4 x u64 (kind, phase time ns, record time ns, SM id) into
 * `records` and their count into *count; `reset` != 0 clears the log instead. The product
 * library returns TTS_ERR_UNSUPPORTED_SHAPE. No counterpart in the reference (tracing aid). */
TTS_API tts_status tts_timeline_read(unsigned long long* records, int cap, int* count, int reset);

/* One context per device (and per host thread driving it). Allocates the split-K and
 * attention scratch for up to `max_lanes` rows (1..448). Replaces the candle Device the reference opens
 * in crates/qwen3tts/src/engine.rs:529-533. */
TTS_API tts_status tts_ctx_create(int device, int max_lanes, tts_ctx** out);
TTS_API tts_status tts_ctx_destroy(tts_ctx* ctx);
/* Synchronises `stream` and reports what the kernels flagged since the last check (then clears
 * it): TTS_ERR_TIMEOUT if a bounded device-side wait gave up (those results are not valid),
 * else TTS_ERR_INVALID_ARG if device data (positions, spans, block-table pages) was out of
 * range (those rows were skipped or read as zero). */
TTS_API tts_status tts_ctx_check(tts_ctx* ctx, void* stream);

/* ---------------------------------------------------------------- projections
 * Proj::forward for Proj::Half: crates/tts-nn/src/lib.rs:510-533, via skinny::matmul
 * (crates/tts-nn/src/skinny.rs:155-165) and matmul_2d (lib.rs:438-459).
 * y = x[m, k] (f16) . w[n, k]^T (f16, the checkpoint's [out, in] layout), f32 accumulate.
 * m in 1..448, k % 64 == 0, n % 128 == 0. `epilogue`:
 *   TTS_EPI_F32          y f32 [m][ldy]
 *   TTS_EPI_F16          y f16 [m][ldy]
 *   TTS_EPI_RESIDUAL_F32 y f32 [m][ldy] += x.w^T   (qwen3.rs:451 and :463, h += proj)
 *   TTS_EPI_SWIGLU_F16   w is a gate/up pair interleaved by tts_interleave_gate_up;
 *                        y f16 [m][n/2] = silu(gate) * up  (fused.rs:289-386)
 * ldy = 0 means the natural row width. */
typedef enum tts_epilogue {
  TTS_EPI_F32 = 0,
  TTS_EPI_F16 = 1,
  TTS_EPI_RESIDUAL_F32 = 2,
  TTS_EPI_SWIGLU_F16 = 3
} tts_epilogue;
TTS_API tts_status tts_proj_forward(tts_ctx* ctx, const void* x_f16, int m, int k, const void* w_f16,
                            int n, int epilogue, void* y, int ldy, void* stream);

/* Load-time weight layout for the decode GEMM: w [n][k] -> [n/128][k/64][128][64], so each
 * 128 x 64 tile the kernel streams is one contiguous 16 KB block and a tile's k-blocks follow
 * each other (DRAM reads stay sequential). The counterpart of the reference's host-side
 * [out, in] -> [in, out] relayout at load (crates/tts-nn/src/lib.rs:473-489, 1252-1298).
 * n % 128 == 0, k % 64 == 0; `out` must not alias `w`. */
TTS_API tts_status tts_weight_pack(tts_ctx* ctx, const void* w_f16, int n, int k, void* out_f16,
                                   void* stream);
/* tts_proj_forward with a weight packed by tts_weight_pack. */
TTS_API tts_status tts_proj_forward_packed(tts_ctx* ctx, const void* x_f16, int m, int k,
                                           const void* w_packed, int n, int epilogue, void* y,
                                           int ldy, void* stream);
/* The same projection shaped for many token rows (the prompt prefill's Proj::forward at t > 1,
 * crates/tts-nn/src/lib.rs:510-533): any rows >= 1 (not bounded by max_lanes), n % 256 == 0,
 * k % 64 == 0, epilogue TTS_EPI_F32, TTS_EPI_RESIDUAL_F32 or TTS_EPI_SWIGLU_F16. */
TTS_API tts_status tts_proj_forward_rows(tts_ctx* ctx, const void* x_f16, int rows, int k,
                                         const void* w_packed, int n, int epilogue, void* y,
                                         int ldy, void* stream);

/* Gate and up projections [ffn][dim] each -> one [2 ffn][dim] weight whose 128-row tiles hold
 * 64 gate rows then the same 64 up rows, the layout TTS_EPI_SWIGLU_F16 consumes. Load-time
 * step, the counterpart of the q/k/v concatenation in crates/qwen3tts/src/qwen3.rs:70-77. */
TTS_API tts_status tts_interleave_gate_up(tts_ctx* ctx, const void* gate_f16, const void* up_f16,
                                  int ffn, int dim, void* out_f16, void* stream);

/* ---------------------------------------------------------------- norms and elementwise
 * rms_norm: crates/tts-nn/src/lib.rs:1001-1003. y = x / sqrt(mean(x^2) + eps) * w over the
 * last dim, f32 math; either output may be NULL. dim % 4 == 0. */
TTS_API tts_status tts_rms_norm(tts_ctx* ctx, const float* x, const float* w, int rows, int dim,
                        float eps, float* y_f32, void* y_f16, void* stream);

/* fused::swiglu_mul: crates/tts-nn/src/fused.rs:289-386. y = silu(gate) * up. */
TTS_API tts_status tts_swiglu_mul(tts_ctx* ctx, const float* gate, const float* up, long n, void* y,
                          int y_f16, void* stream);

/* fused::snake_beta_nlc: crates/tts-nn/src/fused.rs:526-663. Channels-last [rows][chan],
 * y = x + brecip[c] * sin(alpha[c] * x)^2 in f32; x and y f16 or f32. chan % 8 == 0. */
TTS_API tts_status tts_snake_beta_nlc(tts_ctx* ctx, const void* x, int x_f16, const float* alpha,
                              const float* brecip, long rows, int chan, void* y, int y_f16,
                              void* stream);

/* ---------------------------------------------------------------- attention and KV cache
 * A paged KV cache for one layer: K and V pages f16 [num_blocks][n_kv][block_size][head_dim];
 * block_table [lanes][max_blocks] maps a lane's logical block (position / block_size) to a
 * page. The reference's contiguous per-lane cache [b][n_kv][cap][head_dim]
 * (crates/qwen3tts/src/qwen3.rs:122-212) is the case block_size = cap, block_table[i] = {i}. */
typedef struct tts_kv_cache {
  void* k_pages;
  void* v_pages;
  const int* block_table;
  int max_blocks;
  int block_size;
  int num_blocks;
  int n_kv;
  int head_dim; /* must be 128 */
} tts_kv_cache;

/* qkrope::apply: crates/tts-nn/src/qkrope.rs:26-69 (composed form qwen3.rs:358-394).
 * qkv f32 [lanes][(heads + 2 n_kv) * 128]; norms f32 [2][128] (q weight with 1/sqrt(128)
 * folded in, then k weight); cos/sin f32 [rope_len][64]; positions [lanes] is the position
 * each lane writes. Writes q f32 [lanes][heads][128] and K/V (f16) into the pages. Rows whose
 * position or page is out of range are skipped and reported by tts_ctx_check. */
TTS_API tts_status tts_qk_rope_append(tts_ctx* ctx, const float* qkv, int lanes, int heads,
                                      const float* norms, const float* cos_t,
                                      const float* sin_t, int rope_len, const int* positions,
                                      const tts_kv_cache* kv, float eps, float* q_out,
                                      void* stream);

/* attn::decode_attention: crates/tts-nn/src/attn.rs:22-73. q f32 [lanes][n_kv * gqa][128]
 * with the scale folded in; lane i attends positions [wstart_i, spans[i]) where
 * wstart_i = max(0, spans[i] - window) (window 0 = none). max_span bounds every spans[i].
 * out [lanes][n_kv * gqa * 128], f16 or f32. gqa in {1, 2, 4, 8}; lanes <= max_lanes; block_size
 * a multiple of 8 unless max_blocks == 1 (each lane one contiguous page); pool pointers
 * 16-byte aligned. Pages outside [0, num_blocks) read as zero and are reported. */
TTS_API tts_status tts_decode_attention(tts_ctx* ctx, const float* q, int lanes, int gqa,
                                const tts_kv_cache* kv, const int* spans, int max_span,
                                int window, void* out, int out_f16, void* stream);

/* No counterpart in the reference. The same decode attention (same kernel, same results as
 * tts_decode_attention) for callers that cannot allocate device memory: a real-time audio or
 * streaming thread, where cudaMalloc/cudaFree may synchronise the whole device and take
 * unbounded time, or a host engine that reserves all device memory up front in its own arena
 * and cannot let a library allocate behind its back. It needs no tts_ctx (creating one
 * allocates) and calls no allocator: its scratch is one fixed device array inside the library,
 * 4 MiB of split-KV partials, a status word and 4096 arrival counters, which every GPU that
 * loads the library holds until the process exits. It runs on the current device.
 * Limits: lanes <= 512; gqa in {1, 2, 4, 8}; max_span <= 8192; block_size a multiple of 8 unless
 * max_blocks == 1; lanes * n_kv * ceil(max_span / 128) * gqa * 520 bytes must fit in 4 MiB (e.g.
 * 48 lanes x 8 kv heads x gqa 2 up to max_span 1280) and lanes * n_kv <= 4096. A request beyond
 * a limit returns TTS_ERR_UNSUPPORTED_SHAPE before anything is launched.
 * Set-up: CUDA loads the library's device code lazily, so the first call on a device may load
 * it (creating the array) and looks up the array's device address with that device current;
 * that step can allocate and synchronise. Make one call per device at set-up, outside the
 * real-time thread and before any stream capture. The address stays cached for the process:
 * after a device reset the library must not be used again.
 * All calls share the array and it keeps the last call's contents: the status word and the
 * counters are cleared at the start of every call, and calls that overlap on the GPU (two
 * streams or threads at once) race. Device-side problems (a bounded wait that gave up, a span
 * or a page out of range) do not change the return code, which is decided on the host; they
 * are recorded in the status word, read by tts_decode_attention_static_check. */
TTS_API tts_status tts_decode_attention_static(const float* q, int lanes, int gqa,
                                               const tts_kv_cache* kv, const int* spans,
                                               int max_span, int window, void* out,
                                               int out_f16, void* stream);
/* Synchronises `stream` and reports the status word of the last tts_decode_attention_static call
 * on the current device: TTS_ERR_TIMEOUT if a bounded device-side wait gave up (the output is not
 * valid), TTS_ERR_INVALID_ARG if a span was clamped or a page outside the pool read as zero,
 * else TTS_OK. Allocates nothing. Part of the static entry point above (no reference
 * counterpart). */
TTS_API tts_status tts_decode_attention_static_check(void* stream);

/* ---------------------------------------------------------------- sampling
 * Greedy pick of sample_with_u: crates/qwen3tts/src/talker.rs:154-189. banned[n] (nullable)
 * marks ids forced to -inf; ties go to the highest index (Rust's max_by). */
TTS_API tts_status tts_argmax(tts_ctx* ctx, const float* logits, int rows, int n,
                      const unsigned char* banned, unsigned int* out, void* stream);

/* ---------------------------------------------------------------- codec convolution
 * nlc::causal_conv1d and nlc::snake_conv_residual: crates/tts-nn/src/nlc.rs:40-132 via the
 * NlcConv kernel (crates/tts-nn/src/nlcconv.rs:15-198), extended with pad_left so the centred
 * form (crates/tts-nn/src/lib.rs:736-767) is the same call.
 * y[b, l, co] = bias[co] + sum_t sum_ci s(x)[b, l + t*dil - pad_left, ci] * w[co, t, ci]
 *               (+ res[b, l, co]),   rows outside [0, len) read as zero,
 * s(x) = x + brecip * sin(alpha * x)^2 when alpha is given (SnakeBeta on load), else x.
 * x, res, y f16 channels-last; w f16 [cout][k][cin]; bias/alpha/brecip f32 (nullable).
 * cin % 64 == 0, cout % 32 == 0, (k - 1) * dil <= 128, 0 <= pad_left <= (k - 1) * dil. */
TTS_API tts_status tts_conv1d_nlc(tts_ctx* ctx, const void* x_f16, int b, int len, int cin,
                          const void* w_f16, int cout, int k, int dilation, int pad_left,
                          const float* bias, const float* alpha, const float* brecip,
                          const void* res_f16, void* y_f16, void* stream);

/* Top-k sampling per row (crates/tts-nn/src/topk.rs:98-107): logits f32 [rows][n], draws f32
 * [rows] in [0, 1); out u32 [rows] = the row's pick among its k best (ties by lowest index) at
 * `temperature` (<= 0 means 1), walked with the draw as the reference's host sampler does at
 * top_p = 1. Limits as the reference's: 1 <= k <= min(n, 64), n <= 4096. */
TTS_API tts_status tts_topk_sample(tts_ctx* ctx, const float* logits, int rows, int n,
                                   const float* draws, int k, float temperature,
                                   unsigned int* out, void* stream);

/* ---------------------------------------------------------------- decoder stack
 * The qwen3 decoder stack (crates/qwen3tts/src/qwen3.rs:15-467): geometry, per-layer weights
 * (caller-owned device memory, referenced not copied) and the decode step at t == 1. */
typedef struct tts_stack_geometry {
  int dim, layers, heads, n_kv, head_dim, ffn;
  float eps;
  double rope_base;
  int rope_len;  /* positions the RoPE table covers */
  int codebooks; /* heads after the final norm (0 = none) */
  int vocab;     /* ids per codebook head, multiple of 128 */
} tts_stack_geometry;

typedef struct tts_layer_weights {
  const float* attn_norm; /* [dim] */
  const float* ffn_norm;  /* [dim] */
  /* projection weights are packed by tts_weight_pack */
  const void* wqkv;       /* f16 [(heads + 2 n_kv) * head_dim][dim], q/k/v rows concatenated */
  const float* qk_norms;  /* [2][head_dim]: q_norm * 1/sqrt(head_dim), k_norm (qwen3.rs:82-87) */
  const void* wo;         /* f16 [dim][heads * head_dim] */
  const void* w_gate_up;  /* f16 [2 ffn][dim] from tts_interleave_gate_up */
  const void* w_down;     /* f16 [dim][ffn] */
} tts_layer_weights;

TTS_API tts_status tts_stack_create(tts_ctx* ctx, const tts_stack_geometry* geo, tts_stack** out);
TTS_API tts_status tts_stack_set_layer(tts_stack* s, int layer, const tts_layer_weights* w);
/* final_norm f32 [dim]; heads f16 [codebooks * vocab][dim] packed (NULL = none); embed f16
 * [codebooks][vocab][dim] (NULL = none), the tables whose rows for the picked codes are summed
 * into the next step's input. */
TTS_API tts_status tts_stack_set_head(tts_stack* s, const float* final_norm, const void* heads_f16,
                              const void* embed_f16);
/* The buffer f32 [max_lanes][dim] the step writes the next input into (the sum of the picked
 * codes' embedding rows) and reads when x is NULL. Caller-owned; NULL restores the stack's own
 * buffer. Writing a lane's row restarts that lane from a new state (a lane slot reused by the
 * next segment). */
TTS_API tts_status tts_stack_set_feedback(tts_stack* s, float* x_next);

/* The talker's greedy pick over its codec head (crates/qwen3tts/src/talker.rs:154-189, 940,
 * 971-981), for a stack with one codebook head: ids whose bit is set in `ban` are never picked,
 * nor `eos` while the lane's frames < min_new; then each id's finite logit is divided (if
 * positive) or multiplied (if negative) by `penalty` once for every time the lane has emitted
 * it (`counts`), one f32 operation per occurrence as the reference's loop over its history
 * with repeats does; then the last of equal maxima wins. Each step adds its pick to the lane's
 * `counts` (unless it is eos; saturating at 65535) and adds one to the lane's `frames`. All
 * device memory, caller-owned, 16-byte aligned; a lane slot reused for a new segment is
 * cleared by the caller. NULL restores the plain argmax. */
typedef struct tts_pick_rule {
  const unsigned int* ban;  /* [vocab / 32] bits, or NULL */
  unsigned short* counts;   /* [max_lanes][vocab] times each id was emitted, or NULL (needs
                               penalty == 1) */
  int* frames;              /* [max_lanes], or NULL (needs min_new == 0 or eos < 0) */
  float penalty;            /* repetition penalty, 1 = none */
  int eos;                  /* the end id (-1: none) */
  int min_new;              /* frames before eos may be picked */
} tts_pick_rule;
TTS_API tts_status tts_stack_set_pick(tts_stack* s, const tts_pick_rule* rule);
/* sample_with_u with greedy on (crates/qwen3tts/src/talker.rs:154-189) over rows of logits f32
 * [rows][vocab] (vocab % 32 == 0), under `rule` (tts_pick_rule above; counts and frames are
 * indexed by row): out u32 [rows]. With record != 0 each pick is then added to its row's
 * counts (unless it is eos) and the row's frames advance, as the decode loop's push does
 * (talker.rs:984-996). The same arithmetic as the codec head's pick inside the decode step. */
TTS_API tts_status tts_talker_pick(tts_ctx* ctx, const float* logits, int rows, int vocab,
                                   const tts_pick_rule* rule, int record, unsigned int* out,
                                   void* stream);
TTS_API tts_status tts_stack_destroy(tts_stack* s);

/* Decode-time cache state of one group of lanes, all layers: pages f16
 * [layers][num_blocks][n_kv][block_size][head_dim]. positions[lanes] (device) is each lane's
 * cached length; the step writes there and then advances it by one. max_span bounds
 * positions[i] + 1 for as long as a captured graph is replayed. */
typedef struct tts_decode_state {
  int lanes;
  int* positions;
  const int* block_table;
  int max_blocks;
  int block_size;
  int num_blocks;
  void* k_pages;
  void* v_pages;
  int max_span;
} tts_decode_state;

/* ---------------------------------------------------------------- KV page pool
 * The page allocator of the paged KV cache. The reference keeps one contiguous cache per lane,
 * narrows it when lanes are shed and broadcast-copies a shared prompt prefix into every lane
 * (crates/qwen3tts/src/qwen3.rs:122-212 State/Cache/narrow_to, :261-284 fill_prefix); here a
 * lane owns a row of a block table of fixed-size pages from one pool. Full pages of a shared
 * prefix are shared by reference count, only a partly filled last page is copied. The pool
 * keeps the free list and reference counts on the host; admissions write the lane's table row
 * and position with one stream-ordered launch (no host wait), so they may be interleaved with
 * decode steps on the same stream. Not thread-safe: one pool per host thread, as the
 * reference's dispatcher. */
typedef struct tts_kv_pool tts_kv_pool;
typedef struct tts_kv_pool_desc {
  int layers, n_kv, head_dim; /* the stack's geometry */
  int block_size;             /* positions per page */
  int num_blocks;             /* pages in the pool */
  int max_lanes, max_blocks;  /* block table [max_lanes][max_blocks] */
  /* Device buffers, or NULL for the pool to allocate (and free on destroy):
   * pages f16 [layers][num_blocks][n_kv][block_size][head_dim] (both or neither), the block
   * table int32 [max_lanes][max_blocks], positions int32 [max_lanes]. */
  void* k_pages;
  void* v_pages;
  int* block_table;
  int* positions;
} tts_kv_pool_desc;
TTS_API tts_status tts_kv_pool_create(tts_ctx* ctx, const tts_kv_pool_desc* desc,
                                      tts_kv_pool** out);
TTS_API tts_status tts_kv_pool_destroy(tts_kv_pool* pool);
/* Gives `lane` ceil(capacity / block_size) pages (its previous pages are released first); the
 * lane holds `length` positions already (its position is set to `length`). TTS_ERR_OOM when the
 * pool has too few free pages. */
TTS_API tts_status tts_kv_pool_admit(tts_kv_pool* pool, int lane, int capacity, int length,
                                     void* stream);
/* Admits `lane` with the given free pages, in block-table order (a caller that lays out its own
 * pages, e.g. to scatter a prefilled cache). */
TTS_API tts_status tts_kv_pool_admit_pages(tts_kv_pool* pool, int lane, const int* pages, int n,
                                           int length, void* stream);
/* Admits `lane` holding the first `length` positions of lane `src` (the shared prompt prefix,
 * qwen3.rs:261-284): src's full pages are shared, a partly filled page is copied (every layer,
 * K and V, stream-ordered), fresh pages cover the rest of `capacity`. */
TTS_API tts_status tts_kv_pool_share_prefix(tts_kv_pool* pool, int src, int lane, int length,
                                            int capacity, void* stream);
/* Releases the lane's pages: a page returns to the free list when its last lane lets it go. */
TTS_API tts_status tts_kv_pool_release(tts_kv_pool* pool, int lane);
TTS_API int tts_kv_pool_free_pages(const tts_kv_pool* pool);
/* Lanes holding `page` (0 = free), -1 for a page outside the pool. */
TTS_API int tts_kv_pool_page_refs(const tts_kv_pool* pool, int page);
/* The lane's pages in block-table order: up to `cap` into `pages`, their count into *n. */
TTS_API tts_status tts_kv_pool_lane_pages(const tts_kv_pool* pool, int lane, int* pages,
                                          int cap, int* n);

/* The decode state of the pool's first `lanes` lanes (max_span <= 0: the table's capacity). */
TTS_API tts_status tts_kv_pool_state(const tts_kv_pool* pool, int lanes, int max_span,
                                     tts_decode_state* out);

/* One talker decode step: Stack::forward at t == 1 (qwen3.rs:294-467, the whole layer loop and
 * the final norm), then the codebook heads and a greedy pick per head (talker.rs:956-998), then
 * the sum of the picked codes' embedding rows as the next input (talker.rs:1019-1023, 528-550).
 * x f32 [lanes][dim], or NULL to continue from the previous step's embedding sum. Outputs
 * (nullable): h_out f32 [lanes][dim] normed hidden; logits f32 [lanes][codebooks * vocab];
 * codes u32 [lanes][codebooks]. */
TTS_API tts_status tts_stack_decode_step(tts_stack* s, const tts_decode_state* st, const float* x,
                                 float* h_out, float* logits, unsigned int* codes, void* stream);

/* Stack::forward at t > 1, the prompt's prefill (qwen3.rs:294-467; talker.rs:903-931): lane i
 * appends lens[i] (host array) rows at positions positions[i] .. + lens[i] - 1, causal over the
 * lane's cached and new rows, K/V written into its pages; positions advance by lens[i].
 * x f32 [sum of lens][dim], the lanes' rows one lane after another; h_out (NULL = none) f32
 * [sum of lens][dim] every row's final-normed hidden. st->max_span must cover every lane's new
 * end. Not for stream capture: it uploads the row plan and may grow the stack's prefill scratch
 * (the one allocation a stack makes after creation). */
TTS_API tts_status tts_stack_prefill(tts_stack* s, const tts_decode_state* st, const int* lens,
                                     const float* x, float* h_out, void* stream);

/* The same step captured once into a CUDA graph (stream must not be the legacy stream) and
 * replayed with tts_graph_launch. Pointers are baked in at capture. */
TTS_API tts_status tts_stack_graph_capture(tts_stack* s, const tts_decode_state* st, const float* x,
                                   float* h_out, float* logits, unsigned int* codes,
                                   void* stream, tts_graph** out);
TTS_API tts_status tts_graph_launch(tts_graph* g, void* stream);
TTS_API tts_status tts_graph_destroy(tts_graph* g);

/* ---------------------------------------------------------------- depth predictor
 * The code predictor (crates/qwen3tts/src/talker.rs:255-550): a decoder stack of its own
 * (created with codebooks = 1 and vocab = the residual codebook size, heads left unset), the
 * talker-to-predictor projection with bias, one head per residual codebook, the resized tables
 * (tables[i] projected to the predictor's width, talker.rs:268-273, computed once at load in
 * f32) and the tables at talker width for the embedding sum. */
typedef struct tts_predictor_weights {
  const void* resize;      /* f16 [dim][embed_dim] plain (small_to_mtp_projection.weight) */
  const float* resize_bias; /* f32 [dim] (NULL = none) */
  const void* heads;       /* f16 [steps * vocab][dim] packed by tts_weight_pack */
  const float* resized;    /* f32 [steps][vocab][dim]: tables[i] @ resize^T + bias */
  const void* tables;      /* f16 [steps][vocab][embed_dim] */
  int steps;               /* residual codebooks (15) */
  int embed_dim;           /* talker width (2048), multiple of 64 */
} tts_predictor_weights;

typedef struct tts_predictor tts_predictor;

/* Binds a predictor to `stack` (which it drives; one predictor per stack). Allocates its scratch
 * for up to max_lanes / 2 lanes of the stack's context and the doubled resize weight it uses for
 * an f32-exact projection of f32 inputs. Weights are referenced, not copied. */
TTS_API tts_status tts_predictor_create(tts_stack* stack, const tts_predictor_weights* w,
                                        tts_predictor** out);
TTS_API tts_status tts_predictor_destroy(tts_predictor* p);

/* Samples the depth picks on the device (Predictor::depth_on_device, talker.rs:478-515;
 * tts_topk_sample's rule) instead of the greedy pick: draws f32 [steps][stride] in [0, 1), the
 * frame's lane i at step j taking draws[j * stride + i] (the reference's step-major order over
 * lanes); the caller refills it before each frame. NULL draws restores greedy. Pointers are
 * baked into captured graphs. */
TTS_API tts_status tts_predictor_set_sampling(tts_predictor* p, const float* draws, int stride,
                                              int top_k, float temperature);

/* One frame for st->lanes lanes with greedy picks (Predictor::frame_batch, talker.rs:407-468,
 * and gather_sum, talker.rs:528-550): prefill [hidden, code0_embed] through the projection and
 * the stack (both positions in one pass), then per residual codebook i the head, the pick and,
 * before the next pick, the stack on resized[i][code]. st: the predictor's own KV pages, room for
 * steps + 1 positions per lane (positions are reset by the call; max_span >= steps + 1).
 * hidden, code0_embed f32 [lanes][embed_dim]; codes u32 [lanes][steps]; sum f32
 * [lanes][embed_dim] = code0_embed + the picked codes' table rows (+ the lane's text row, when
 * `text` is given: the talker's next input, talker.rs:1043-1050). sum may be code0_embed. */
typedef struct tts_text_feed {
  const float* rows;  /* f32 [lanes][len][embed_dim]: each lane's trailing text embeddings */
  int len;            /* rows per lane */
  const float* pad;   /* f32 [embed_dim]: the tts_pad embedding, once a lane's rows run out */
  const int* frames;  /* device [lanes]: frames picked so far, this one included; the lane
                       * adds row frames - 1 (the pick rule's counter) */
} tts_text_feed;
TTS_API tts_status tts_predictor_frame(tts_predictor* p, const tts_decode_state* st,
                                       const float* hidden, const float* code0_embed,
                                       const tts_text_feed* text, unsigned int* codes,
                                       float* sum, void* stream);
/* The same frame captured into one CUDA graph (non-legacy stream); pointers baked in. */
TTS_API tts_status tts_predictor_graph_capture(tts_predictor* p, const tts_decode_state* st,
                                               const float* hidden, const float* code0_embed,
                                               const tts_text_feed* text, unsigned int* codes,
                                               float* sum, void* stream, tts_graph** out);

/* One reference-faithful talker frame for st->lanes lanes (talker.rs:953-1057, greedy): the
 * talker stack's decode step from its feedback input with the codec head and its pick rule
 * (code 0, its codec_embed row as the feedback), then the predictor's frame on the step's
 * hidden state and that row, whose sum plus the lane's text row becomes the next feedback
 * input. `talker` needs one codebook head, an embedding table and a caller-owned feedback
 * buffer (tts_stack_set_feedback); hidden f32 [max_lanes][talker dim] scratch; code0 u32
 * [lanes]; codes u32 [lanes][steps] the residual codes. */
TTS_API tts_status tts_talker_frame(tts_stack* talker, const tts_decode_state* talker_st,
                                    tts_predictor* p, const tts_decode_state* pred_st,
                                    const tts_text_feed* text, float* hidden,
                                    unsigned int* code0, unsigned int* codes, void* stream);
TTS_API tts_status tts_talker_frame_capture(tts_stack* talker, const tts_decode_state* talker_st,
                                            tts_predictor* p, const tts_decode_state* pred_st,
                                            const tts_text_feed* text, float* hidden,
                                            unsigned int* code0, unsigned int* codes,
                                            void* stream, tts_graph** out);

/* ---------------------------------------------------------------- codec front
 * The ops the codec decoder's front uses besides projections and convs (crates/qwen3tts/src/
 * codec.rs:161-196, 261-317, 403-424). All f32 unless stated, rows contiguous.
 *
 * Rvq::decode's lookups (codec.rs:285-299): out f32 [T][dim] = sum over q in [q0, q0 + nq) of
 * tables[q - q0][codes[t][q]], codes u32 [T][ncodes], tables f32 [nq][entries][dim]. */
TTS_API tts_status tts_rvq_gather(tts_ctx* ctx, const unsigned int* codes, int T, int ncodes,
                                  int q0, int nq, const float* tables, int entries, int dim,
                                  float* out, void* stream);
/* candle_nn::rotary_emb::rope (half-split) in place on `heads` heads of width hd from column
 * col0 of x [T][ld]; row t at position pos0 + t of cos/sin [positions][hd / 2]. */
TTS_API tts_status tts_rope_rows(tts_ctx* ctx, float* x, int T, int ld, int col0, int heads,
                                 int hd, const float* cos_t, const float* sin_t, int pos0,
                                 void* stream);
/* Causal (optionally windowed) self-attention over one sequence, the prefill branch of
 * Stack::forward with causal_window_mask (qwen3.rs:409-444, lib.rs:1210-1225): qkv f32
 * [T][3 heads hd] (q | k | v, one kv head per q head), row t attends rows [t + 1 - window, t]
 * (window 0: all earlier rows), scores * scale; out [T][heads hd] f16 or f32. hd <= 128. */
TTS_API tts_status tts_window_attention(tts_ctx* ctx, const float* qkv, int T, int heads, int hd,
                                        int window, float scale, void* out, int out_f16,
                                        void* stream);
/* layer_norm (crates/tts-nn/src/lib.rs:1006-1035): y = (x - mean) / sqrt(var + eps) * w + b
 * over the last dim (b may be NULL); y f32 or f16. */
TTS_API tts_status tts_layer_norm(tts_ctx* ctx, const float* x, const float* w, const float* b,
                                  int rows, int dim, float eps, void* y, int y_f16, void* stream);
/* nlc::depthwise (crates/tts-nn/src/nlc.rs:232-256): causal per-channel conv of x [b][L][C]
 * with taps w [C][k] and bias [C] (NULL = none). */
TTS_API tts_status tts_depthwise_conv(tts_ctx* ctx, const float* x, int b, int L, int C,
                                      const float* w, int k, const float* bias, float* y,
                                      void* stream);
/* The epilogue of a projection computed in f32 (Linear's bias, gelu_exact lib.rs:1129, a
 * per-channel scale such as LayerScale or ConvNeXt's gamma, a residual): z = act(y + bias),
 * out = res + scale * z; act 0 none, 1 GELU (erf), 2 SiLU (the text projection's, talker.rs:
 * 607-616). bias, scale, res may be NULL. */
TTS_API tts_status tts_bias_act(tts_ctx* ctx, const float* y, int rows, int n, const float* bias,
                                int act, const float* scale, const float* res, void* out,
                                int out_f16, void* stream);

/* ---------------------------------------------------------------- checkpoint files
 * Memory-mapped safetensors (the reference's Weights over candle's MmapedSafetensors,
 * crates/tts-nn/src/lib.rs:153-373): the header parsed at open, every tensor a view into the
 * mapping (host memory, on-disk dtype). Casts, transposes and folds are the caller's load-time
 * work. Errors name the file and the broken entry; a missing name is "missing tensor <name>". */
typedef struct tts_safetensors tts_safetensors;
typedef enum tts_dtype {
  TTS_DT_F32 = 0, TTS_DT_F16 = 1, TTS_DT_BF16 = 2, TTS_DT_I32 = 3, TTS_DT_I64 = 4,
  TTS_DT_U8 = 5, TTS_DT_F64 = 6, TTS_DT_I8 = 7, TTS_DT_I16 = 8, TTS_DT_BOOL = 9,
  TTS_DT_OTHER = 99
} tts_dtype;
typedef struct tts_tensor_view {
  const char* name;     /* valid while the file is open */
  int dtype;            /* tts_dtype */
  int ndim;
  long long shape[8];
  const void* data;     /* host, read-only */
  size_t nbytes;
} tts_tensor_view;
TTS_API tts_status tts_safetensors_open(const char* path, tts_safetensors** out);
TTS_API int tts_safetensors_count(const tts_safetensors* f);
TTS_API tts_status tts_safetensors_at(const tts_safetensors* f, int i, tts_tensor_view* out);
TTS_API tts_status tts_safetensors_find(const tts_safetensors* f, const char* name,
                                        tts_tensor_view* out);
TTS_API tts_status tts_safetensors_close(tts_safetensors* f);

/* Kernel launches made by the calling thread through this library since the last call
 * (observability: the bench reports it). */
TTS_API long long tts_launch_count(int reset);

#ifdef __cplusplus
}
#endif

#endif /* TTS_CUDA_H */
