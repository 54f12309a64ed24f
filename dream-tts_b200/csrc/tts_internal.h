// Internal C++ interface between the kernel files and the C ABI in runtime.cu.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace tts {

// ------------------------------------------------------------------ errors
void set_error(const std::string& msg);
const char* last_error();

// ------------------------------------------------------------------ device error flags
// Kernels OR these into the context's device flag word; tts_ctx_check reads and clears it.
// Waits that gave up (results of that launch are not valid):
constexpr int kFlagGemmWait = 1 | 2 | 4;
constexpr int kFlagConvWait = 16 | 32 | 64 | 128 | 4096 | 8192;
constexpr int kFlagAttnWait = 2048;
constexpr int kFlagWaitMask = kFlagGemmWait | kFlagConvWait | kFlagAttnWait;
// Device data outside what the launch covers (the rows involved are skipped or read as zero):
constexpr int kFlagRopeRange = 256;   // position outside the RoPE table, block table or pool
constexpr int kFlagSpanRange = 512;   // attention span outside 1..min(max_span, table)
constexpr int kFlagPageRange = 1024;  // attention page outside the pool

// ------------------------------------------------------------------ device properties
int num_sms(int device);

// ------------------------------------------------------------------ decode GEMM
enum Epilogue : int {
  EPI_F32 = 0,       // y[m, n] f32
  EPI_F16 = 1,       // y[m, n] f16
  EPI_RESIDUAL = 2,  // y[m, n] f32 += acc
  EPI_SWIGLU = 3,    // W rows interleaved per 128-row tile: 64 gate then 64 up; y[m, n/2] f16
  EPI_QKROPE = 4,    // QK-norm + RoPE + paged KV append per 128-row head tile
  EPI_ARGMAX = 5,    // greedy pick per (row, codebook); optional f32 logits in y
};

struct QkRopeArgs {
  const float* norms = nullptr;  // [2][128]: q weight (1/sqrt(hd) folded in), k weight
  const float* cos_t = nullptr;  // [positions][64]
  const float* sin_t = nullptr;
  const int* positions = nullptr;    // [lanes] position written this step
  const int* block_table = nullptr;  // [lanes][max_blocks]
  int max_blocks = 0;
  int block_size = 0;
  int num_blocks = 0;        // pages in the pool; out-of-range table entries are skipped
  int rope_len = 0;          // rows of cos_t/sin_t; positions outside are skipped
  int* err = nullptr;        // kFlagRopeRange when a table entry or position is out of range
  __half* k_pool = nullptr;  // this layer's K pages [num_blocks][n_kv][block_size][128]
  __half* v_pool = nullptr;
  float* q_out = nullptr;  // [lanes][heads][128]
  int heads = 0;
  int n_kv = 0;
  float eps = 1e-6f;
  // Optional, per step (launch_qk_rows): each row's operands read once for every layer, which
  // the decode GEMM stages into shared memory ahead of its epilogue. rows_desc [rows] =
  // {position or -1 when outside the RoPE table or the block table, page or -1 when outside
  // the pool, offset in the page, 0}; rows_rope [rows][128] = the RoPE cos row then sin row.
  const int4* rows_desc = nullptr;
  const float* rows_rope = nullptr;
};

// The next projection's packed weights, for an L2 prefetch issued at the end of a kernel's own
// weight or cache stream (when HBM would otherwise idle through that kernel's epilogue and the
// next kernel's start): the first `depth` 128x64 tiles of every (128-row tile, split-K range)
// of the next GEMM, i.e. the blocks its CTAs load first.
struct L2Prefetch {
  const __half* w = nullptr;  // packed [tiles][kb_total][128][64]
  int tiles = 0, kb_total = 0, splits = 1, depth = 0;
};
// The prefetch plan for a packed weight [n][k] read by a GEMM of m lanes, about `budget` bytes.
L2Prefetch gemm_prefetch_plan(const void* w_packed, int m, int k, int n, int device,
                              size_t budget);

// The talker's greedy pick rule (crates/qwen3tts/src/talker.rs:154-189, 940, 971-981), applied
// to the codec head's logits before the argmax: ids with their bit set in `ban` are excluded,
// `eos` too while frames[row] < min_new, and each id's logit is divided (if positive) or
// multiplied (if negative) by `penalty` once per time the row has emitted it (counts). The code
// gather then records the pick (unless it is eos) and counts the row's frame (pick_rule.cuh).
struct PickRule {
  const uint32_t* ban = nullptr;  // [vocab / 32] bits
  uint16_t* counts = nullptr;     // [rows][vocab]: times each id was emitted (saturating)
  int* frames = nullptr;          // [rows]
  float penalty = 1.f;
  int eos = -1, min_new = 0;
  int vocab = 0;                  // ids per row, a multiple of 32 (0: no rule)
};

struct GemmRequest {
  // [n][k] (out-major, K contiguous), or packed: [n/128][k/64][128][64], each 128 x 64 tile
  // one contiguous 16 KB block (tts_weight_pack)
  const __half* w = nullptr;
  bool packed = false;
  const __half* x = nullptr;  // [m][k]
  int m = 0, k = 0, n = 0;
  int epi = EPI_F32;
  void* y = nullptr;
  int ldy = 0;  // elements between rows of y (0 = natural width)
  QkRopeArgs qk;
  unsigned long long* argmax_keys = nullptr;  // [m][codebooks]
  int vocab = 0;
  PickRule pick;  // EPI_ARGMAX with one codebook: the talker's pick rule (empty: plain argmax)
  bool pdl = true;
  int force_splits = 0;  // 0 = automatic
  L2Prefetch next;       // optional: the next GEMM's first weight blocks
  // Deferred RMSNorm. Producer (EPI_RESIDUAL): with norm_w set, the epilogue also writes
  // norm_x16[j] = f16(h[j] * norm_w) (the next projection's x, [m][n]) and, per 128-column
  // tile t, ss_out[t * m + j] = the sum of squares of h[j]'s columns in that tile. Consumer:
  // with ss_in set, every output row j is scaled by 1 / sqrt(sum_t ss_in[t * m + j] / ss_dim +
  // ss_eps) (t < ss_tiles <= 32) before its epilogue, which completes RMSNorm(h) . W^T.
  const float* norm_w = nullptr;
  __half* norm_x16 = nullptr;
  float* ss_out = nullptr;
  const float* ss_in = nullptr;
  int ss_tiles = 0, ss_dim = 0;
  float ss_eps = 0.f;
};

// Prefill-shaped projection (pf_gemm.cu): token rows as the MMA's M, 256 weight rows per tile.
// w packed as for GemmRequest; epi EPI_F32 (y f32), EPI_RESIDUAL (y f32 +=), EPI_SWIGLU (y f16
// [rows][n / 2]).
struct PfGemmRequest {
  const __half* x = nullptr;  // [rows][k]
  const __half* w = nullptr;
  int rows = 0, k = 0, n = 0;
  int epi = EPI_F32;
  void* y = nullptr;
  int ldy = 0;  // 0: n (n / 2 for SwiGLU)
};
bool pf_gemm_supported(int rows, int k, int n, int epi, std::string* why);
cudaError_t launch_pf_gemm(const PfGemmRequest& r, cudaStream_t st, int device, int* err);

// Prompt attention for the layer-major prefill (pf_attn.cu): one CTA per (block of <= 64 new
// positions of a lane, kv head); GQA 2, spans <= 256, block_size % 8 == 0.
struct PfAttnRequest {
  const float* q = nullptr;    // [rows][heads][128]
  const int* blocks = nullptr; // [n_blocks][4]: lane, first row, first new-position offset, rows
  int n_blocks = 0;
  const int* positions = nullptr;  // [lanes] positions held before this prefill
  const int* block_table = nullptr;
  int max_blocks = 0, block_size = 0, num_blocks = 0;
  int heads = 0, n_kv = 0, max_span = 0;
  const __half* k_pool = nullptr;  // this layer's pages
  const __half* v_pool = nullptr;
  __half* out = nullptr;  // [rows][heads][128]
  int* err = nullptr;
};
bool pf_attn_supported(int heads, int n_kv, int block_size, int max_span);
cudaError_t launch_pf_attn(const PfAttnRequest& r, cudaStream_t st);

struct Workspace {
  int* err = nullptr;  // device error flags (bounded waits that gave up, out-of-range rows)
};

constexpr int kMaxGemmRows = 448;
bool gemm_supported(int m, int k, int n, int epi, std::string* why);
cudaError_t launch_gemm(const GemmRequest& r, const Workspace& wsp, cudaStream_t st, int device);



// ------------------------------------------------------------------ decode attention
struct AttnRequest {
  const float* q = nullptr;  // [lanes][n_kv*gqa][128] f32, scale folded in
  const __half* k_pool = nullptr;  // layer view [num_blocks][n_kv][block_size][128]
  const __half* v_pool = nullptr;
  const int* block_table = nullptr;  // [lanes][max_blocks]
  int max_blocks = 0;
  int block_size = 0;
  int num_blocks = 0;
  int* err = nullptr;
  const int* spans = nullptr;  // [lanes]; span of lane i = spans[i] + span_add
  int span_add = 0;
  int max_span = 0;  // upper bound of any span (sizes the grid)
  int window = 0;    // 0 = none; else positions < span - window are masked
  int lanes = 0, n_kv = 0, gqa = 0;
  void* out = nullptr;  // [lanes][n_kv*gqa*128]
  bool out_f16 = true;
  bool pdl = true;
  // The caller guarantees that the spans and the block table are final when the kernel starts
  // (nothing launched earlier in the stream still writes them): the kernel then splits its work
  // and resolves its first pages before waiting for the previous kernel (PDL); every K/V load
  // still waits. The talker's decode step: it starts with a copy (a full stream dependency on
  // the previous step's position advance) and its kernels write neither.
  bool early_meta = false;
  L2Prefetch next;  // optional: the next GEMM's first weight blocks
};
struct AttnWorkspace {
  float* part = nullptr;
  size_t part_bytes = 0;
  unsigned* counters = nullptr;
  int n_counters = 0;
};
// Spans up to kShortSpanMax take the CUDA-core kernel (attn_short.cu): at a few dozen positions
// the tensor-core kernel's fixed cost dominates.
constexpr int kShortSpanMax = 64;
cudaError_t launch_attn_short(const AttnRequest& r, cudaStream_t st);
size_t attn_part_bytes(int lanes, int n_kv, int gqa, int max_span);
cudaError_t launch_attn(const AttnRequest& r, const AttnWorkspace& w, cudaStream_t st);
// The same attention with its scratch in a fixed device array (no allocation anywhere).
cudaError_t launch_attn_static(const AttnRequest& r, cudaStream_t st);
size_t attn_static_part_limit();
int attn_static_counter_limit();
// The error flags the last launch_attn_static on the current device left in its status word
// (synchronises `st` first).
cudaError_t attn_static_status(cudaStream_t st, int* flags);

// ------------------------------------------------------------------ small kernels
// The deferred norm's first stage for rows that no projection produced (the step's input):
// y16[r] = f16(x[r] * w) and ss[r] = the sum of squares of x[r] (one tile: ss_tiles = 1).
cudaError_t launch_norm_defer(const float* x, const float* w, int rows, int dim, __half* y16,
                              float* ss, bool pdl, cudaStream_t st);
cudaError_t launch_rms_norm(const float* x, const float* w, int rows, int dim, float eps,
                            float* y32, __half* y16, unsigned long long* zero_keys, int n_keys,
                            bool pdl, cudaStream_t st);
cudaError_t launch_qk_rope(const float* qkv, const QkRopeArgs& a, int lanes, bool pdl,
                           cudaStream_t st);
cudaError_t launch_swiglu(const float* g, const float* u, void* y, bool y_f16, long n,
                          cudaStream_t st);
cudaError_t launch_snake(const void* x, bool x_f16, const float* alpha, const float* brecip,
                         long rows, int chan, void* y, bool y_f16, cudaStream_t st);
cudaError_t launch_pick(const float* logits, int rows, const PickRule& pick, bool record,
                        uint32_t* out, cudaStream_t st);
// Each row's QK-rope operands for a decode step (QkRopeArgs::rows_desc / rows_rope) from
// the positions, the block table and the RoPE tables; flags out-of-range rows once.
cudaError_t launch_qk_rows(const QkRopeArgs& a, int rows, int4* desc, float* rope, bool pdl,
                           cudaStream_t st);
cudaError_t launch_argmax(const float* logits, int rows, int n, const uint8_t* banned,
                          uint32_t* out, cudaStream_t st);
cudaError_t launch_keys_to_codes(const unsigned long long* keys, int rows, int codebooks,
                                 int vocab, const __half* embed, const float* embed32, int dim,
                                 uint32_t* codes, float* x_next, unsigned long long* keys_reset,
                                 int* positions, const PickRule* pick, bool pdl,
                                 cudaStream_t st);
// The depth predictor's frame ends (predictor.cu): the prefill rows (f32 inputs split into
// f16 hi | lo halves, the projection's bias rows, the paired-lane block table and positions)
// and the codes transpose with the embedding sum at talker width.
cudaError_t launch_predictor_prefill(const float* hidden, const float* code0, int lanes,
                                     int embed_dim, __half* x16, const float* bias, int dim,
                                     float* x0, const int* table, int max_blocks, int* table2,
                                     int* pos2, int* positions, cudaStream_t st);
struct TextFeed {
  const float* rows = nullptr;  // [lanes][len][embed_dim]
  int len = 0;
  const float* pad = nullptr;   // [embed_dim]; null: no text added
  const int* frames = nullptr;  // [lanes]: row frames - 1
};
cudaError_t launch_predictor_finish(const uint32_t* step_codes, int stride, int lanes, int steps,
                                    const __half* tables, int vocab, int embed_dim,
                                    const float* code0, uint32_t* codes, float* sum,
                                    const TextFeed& text, cudaStream_t st);
cudaError_t launch_advance_positions(int* positions, int lanes, bool pdl, cudaStream_t st);
// The codec front's row kernels (codec_front.cu).
cudaError_t launch_rvq_gather(const uint32_t* codes, int ncodes, int q0, int nq,
                              const float* tables, int entries, int dim, float* out, int T,
                              cudaStream_t st);
cudaError_t launch_rope_rows(float* x, int T, int ld, int col0, int heads, int hd,
                             const float* cos_t, const float* sin_t, int pos0, cudaStream_t st);
cudaError_t launch_window_attn(const float* qkv, int T, int ld, int heads, int hd, int window,
                               float scale, void* out, bool out_f16, cudaStream_t st);
cudaError_t launch_layer_norm(const float* x, const float* w, const float* b, int rows, int dim,
                              float eps, void* y, bool y_f16, cudaStream_t st);
cudaError_t launch_depthwise(const float* x, const float* w, const float* bias, int b, int L,
                             int C, int k, float* y, cudaStream_t st);
cudaError_t launch_bias_act(const float* y, int rows, int n, const float* bias, int act,
                            const float* scale, const float* res, void* out, bool out_f16,
                            cudaStream_t st);
// Top-k sampling (topk_sample.cu): rows of logits (row stride ldl), a draw per row (row r
// takes draws[r % draw_rows]), codes[r * code_stride]; optionally the pick's f32 embedding row
// into x_next and the row's position advanced (a decode step's code gather).
constexpr int kTopkMaxN = 4096;
constexpr int kTopkMaxK = 64;
cudaError_t launch_topk_sample(const float* logits, int rows, int n, int ldl, const float* draws,
                               int draw_rows, int k, float temperature, uint32_t* codes,
                               int code_stride, const float* embed32, float* x_next, int dim,
                               int* positions, bool pdl, cudaStream_t st);
cudaError_t launch_cast_f32_f16(const float* x, __half* y, long n, cudaStream_t st);
// Prefill as decode rows (map[r] = (lane, offset)): per-row block-table copies and positions;
// then each lane's position advanced by its row count.
cudaError_t launch_prefill_rows(const int* map, int rows, const int* table, int max_blocks,
                                const int* positions, int* table2, int* pos2, cudaStream_t st);
cudaError_t launch_advance_by(int* positions, const int* lens, int lanes, cudaStream_t st);

// ------------------------------------------------------------------ codec conv
struct ConvRequest {
  const __half* x = nullptr;  // [b][len][cin] channels-last
  const __half* w = nullptr;  // [cout][k][cin] (K-major per output channel)
  const float* bias = nullptr;    // [cout] or null
  const float* alpha = nullptr;   // snake on load: [cin] or null
  const float* brecip = nullptr;  // [cin]
  const __half* res = nullptr;    // [b][len][cout] or null
  __half* y = nullptr;            // [b][len][cout]
  int b = 0, len = 0, cin = 0, cout = 0, k = 0, dil = 1, pad_left = 0;
  bool pdl = false;
};
bool conv_supported(const ConvRequest& r, std::string* why);
cudaError_t launch_conv(const ConvRequest& r, cudaStream_t st, int device, int* err);

// ------------------------------------------------------------------ TMA descriptor encode
bool make_tmap_2d_f16(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                      bool swizzle128);

}  // namespace tts
