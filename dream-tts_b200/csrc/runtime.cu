// C ABI (include/tts_cuda.h) and the native runtime around the kernels: context and scratch
// ownership, argument checks, the decoder stack, the decode step and its CUDA graph.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/tts_cuda.h"
#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

namespace {
thread_local std::string g_err;
thread_local long long g_launches = 0;
}  // namespace

void set_error(const std::string& msg) { g_err = msg; }
const char* last_error() { return g_err.c_str(); }

int num_sms(int device) {
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return 148;
  if (!cache[device]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
      n = 148;
    cache[device] = n;
  }
  return cache[device];
}

}  // namespace tts

using namespace tts;

#ifdef TTS_TIMELINE
namespace tts {
__device__ unsigned long long g_timeline[kTimelineCap * 4];
__device__ unsigned g_timeline_n;
}  // namespace tts
#endif

struct tts_ctx {
  int device = 0;
  int max_lanes = 0;
  Workspace gemm;
  AttnWorkspace attn;
  int* err_host = nullptr;
};

struct tts_stack {
  tts_ctx* ctx = nullptr;
  tts_stack_geometry geo{};
  std::vector<tts_layer_weights> layers;
  const float* final_norm = nullptr;
  const __half* heads = nullptr;
  const __half* embed = nullptr;
  // device buffers owned by the stack
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;
  float* h = nullptr;         // residual stream [max_lanes][dim]
  __half* xn = nullptr;       // normed activations as the next GEMM's x [max_lanes][max(dim, q)]
  float* q = nullptr;         // [max_lanes][heads][head_dim]
  __half* attn = nullptr;     // [max_lanes][heads * head_dim]
  __half* act = nullptr;      // [max_lanes][ffn]
  float* x_next = nullptr;    // [max_lanes][dim] (own buffer)
  float* feedback = nullptr;  // caller's buffer replacing x_next, or null
  // Deferred RMSNorm (on unless TTS_DEFER_NORM=0): the O and down projections' epilogues
  // write the next norm's f16 input h * w and per-tile row sums of squares `ss`
  // [dim / 128][max_lanes]; the QKV and gate/up projections scale their rows by 1 / RMS. The
  // step then runs no norm kernel between layers (one for the input, one final).
  float* ss = nullptr;
  bool defer_norm = true;
  // each lane's QK-rope operands for the step (launch_qk_rows), read by every layer's QKV
  // epilogue from shared memory: int4 [max_lanes] and f32 [max_lanes][128]
  int4* qk_desc = nullptr;
  float* qk_rope = nullptr;
  PickRule pick;              // the codec head's greedy pick rule (vocab == 0: plain argmax)
  // prefill scratch, grown on demand by tts_stack_prefill: per-row (lane, offset) pairs and
  // lane lengths; per-row block-table rows and positions for one chunk of rows
  int* pre_map = nullptr;
  size_t pre_map_ints = 0;
  int* pre_table = nullptr;
  size_t pre_table_ints = 0;
  int* pre_pos = nullptr;
  // layer-major prefill scratch (all of a prompt batch's rows at once), grown on demand
  unsigned char* pf_buf = nullptr;
  size_t pf_bytes = 0;
  int* pf_blocks = nullptr;  // the prompt attention's query blocks [n][4]
  size_t pf_blocks_ints = 0;
  unsigned long long* keys = nullptr;  // [max_lanes][codebooks]
  // bytes of the next projection's weights each kernel prefetches into L2 (0: none). 12 MB
  // measured best for the talker; the depth predictor's stack runs without (its kernels are
  // latency-bound, and the prefetch measured 6% slower per frame at 48 lanes).
  size_t pf_budget = size_t(12) << 20;
};

// The depth predictor: its stack, weights, the doubled resize weight and per-frame scratch
// for up to max_lanes lanes (the prefill runs 2 * max_lanes rows).
constexpr int kPredictorMaxBlocks = 64;
struct tts_predictor {
  tts_stack* s = nullptr;
  tts_predictor_weights w{};
  int max_lanes = 0;
  __half* resize2 = nullptr;     // packed [dim][2 embed_dim]: [W | W]
  __half* x16 = nullptr;         // [2 max_lanes][2 embed_dim]: [hi | lo]
  int* table2 = nullptr;         // [2 max_lanes][kPredictorMaxBlocks]
  int* pos2 = nullptr;           // [2 max_lanes]
  unsigned* step_codes = nullptr;  // [steps][2 max_lanes]
  // top-k sampling of the depth picks (draws [steps][draw_stride]); null draws: greedy
  const float* draws = nullptr;
  int draw_stride = 0, top_k = 0;
  float temperature = 1.f;
  float* logits = nullptr;  // [2 max_lanes][vocab]
};

struct tts_graph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  long long kernels = 0;
};

namespace rt {

tts_status fail(tts_status s, const std::string& msg) {
  set_error(msg);
  return s;
}

tts_status cuda_status(cudaError_t e, const char* op) {
  if (e == cudaSuccess) return TTS_OK;
  if (e == cudaErrorInvalidValue && g_err.size() && g_err.find(op) != std::string::npos)
    return TTS_ERR_UNSUPPORTED_SHAPE;
  set_error(std::string(op) + ": " + cudaGetErrorString(e));
  return e == cudaErrorMemoryAllocation ? TTS_ERR_OOM : TTS_ERR_CUDA;
}

// Every launch goes through here so the launch counter is exact.
tts_status counted(cudaError_t e, const char* op) {
  if (e == cudaSuccess) ++g_launches;
  return cuda_status(e, op);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int ctx_device(const tts_ctx* c) { return c->device; }

cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

template <class T>
cudaError_t dmalloc(T** p, size_t bytes) {
  return cudaMalloc(reinterpret_cast<void**>(p), bytes);
}

__global__ void interleave_gate_up_kernel(const __half* gate, const __half* up, int ffn, int dim,
                                          __half* out) {
  // out row r: tile t = r / 128, within-tile i = r % 128; i < 64 -> gate row t*64+i,
  // else up row t*64 + (i - 64).
  const long total = 2L * ffn * dim / 8;
  for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total;
       e += (long)gridDim.x * blockDim.x) {
    const long el = e * 8;
    const long r = el / dim, c = el % dim;
    const long t = r / 128, i = r % 128;
    const __half* src = i < 64 ? gate + (t * 64 + i) * dim + c : up + (t * 64 + (i - 64)) * dim + c;
    *reinterpret_cast<uint4*>(out + el) = *reinterpret_cast<const uint4*>(src);
  }
}

// w [n][k] -> [n/128][k/64][128][64]: each 128 x 64 tile one contiguous 16 KB block, a tile
// row's k-blocks consecutive, so the GEMM streams its weights sequentially.
__global__ void pack_weight_kernel(const __half* w, int n, int k, __half* out) {
  const long total = long(n) * k / 8;
  const int kb = k / 64;
  for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total;
       e += (long)gridDim.x * blockDim.x) {
    const long el = e * 8;                  // element index in the packed layout
    const long blk = el / (128 * 64);       // (tile, k-block) block
    const int within = int(el % (128 * 64));
    const int r = within / 64, c = within % 64;
    const long t = blk / kb, b = blk % kb;
    const __half* src = w + (t * 128 + r) * long(k) + b * 64 + c;
    *reinterpret_cast<uint4*>(out + el) = *reinterpret_cast<const uint4*>(src);
  }
}

}  // namespace rt
using namespace rt;

extern "C" {

int tts_abi_version(void) { return TTS_CUDA_ABI_VERSION; }

tts_status tts_timeline_read(unsigned long long* records, int cap, int* count, int reset) {
#ifdef TTS_TIMELINE
  if (reset) {
    const unsigned zero = 0;
    return cuda_status(cudaMemcpyToSymbol(tts::g_timeline_n, &zero, sizeof(zero)), "timeline_read");
  }
  if (!records || !count || cap < 0) return fail(TTS_ERR_INVALID_ARG, "timeline_read: NULL argument");
  unsigned n = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&n, tts::g_timeline_n, sizeof(n));
  if (e != cudaSuccess) return cuda_status(e, "timeline_read");
  n = std::min(n, std::min(unsigned(cap), tts::kTimelineCap));
  *count = int(n);
  return cuda_status(
      cudaMemcpyFromSymbol(records, tts::g_timeline, size_t(n) * 4 * sizeof(unsigned long long)),
      "timeline_read");
#else
  (void)records;
  (void)cap;
  (void)count;
  (void)reset;
  return fail(TTS_ERR_UNSUPPORTED_SHAPE, "timeline_read: library built without TTS_TIMELINE");
#endif
}
const char* tts_last_error(void) { return g_err.c_str(); }
long long tts_launch_count(int reset) {
  const long long n = g_launches;
  if (reset) g_launches = 0;
  return n;
}

tts_status tts_ctx_create(int device, int max_lanes, tts_ctx** out) {
  if (!out) return fail(TTS_ERR_INVALID_ARG, "ctx_create: out is NULL");
  if (max_lanes < 1 || max_lanes > kMaxGemmRows)
    return fail(TTS_ERR_INVALID_ARG, "ctx_create: max_lanes must be in 1..448");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
    return fail(TTS_ERR_CUDA, "ctx_create: no such CUDA device");
  DeviceGuard g(device);
  cudaDeviceProp prop{};
  cudaGetDeviceProperties(&prop, device);
  if (prop.major != 10)
    return fail(TTS_ERR_CUDA, "ctx_create: this library is built for sm_100a (B200)");
  auto* c = new tts_ctx();
  c->device = device;
  c->max_lanes = max_lanes;
  const int max_span = 8192, n_kv = 8, gqa = 2;
  c->attn.part_bytes = attn_part_bytes(max_lanes, n_kv, gqa, max_span);
  c->attn.n_counters = max_lanes * 64;
  cudaError_t e = dmalloc(&c->gemm.err, 16);
  if (e == cudaSuccess) e = dmalloc(&c->attn.part, c->attn.part_bytes);
  if (e == cudaSuccess) e = dmalloc(&c->attn.counters, c->attn.n_counters * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(c->attn.counters, 0, c->attn.n_counters * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(c->gemm.err, 0, 16);
  if (e == cudaSuccess) e = cudaMallocHost(reinterpret_cast<void**>(&c->err_host), 16);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    tts_ctx_destroy(c);
    return cuda_status(e, "ctx_create");
  }
  *out = c;
  return TTS_OK;
}

tts_status tts_ctx_destroy(tts_ctx* c) {
  if (!c) return TTS_OK;
  DeviceGuard g(c->device);
  cudaFree(c->gemm.err);
  cudaFree(c->attn.part);
  cudaFree(c->attn.counters);
  if (c->err_host) cudaFreeHost(c->err_host);
  delete c;
  return TTS_OK;
}

tts_status tts_ctx_check(tts_ctx* c, void* stream) {
  if (!c) return fail(TTS_ERR_INVALID_ARG, "ctx_check: ctx is NULL");
  DeviceGuard g(c->device);
  cudaError_t e = cudaMemcpyAsync(c->err_host, c->gemm.err, sizeof(int), cudaMemcpyDeviceToHost,
                                  S(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(S(stream));
  if (e != cudaSuccess) return cuda_status(e, "ctx_check");
  if (c->err_host[0]) {
    const int code = c->err_host[0];
    cudaMemsetAsync(c->gemm.err, 0, sizeof(int), S(stream));
    cudaStreamSynchronize(S(stream));
    if (code & kFlagWaitMask)
      return fail(TTS_ERR_TIMEOUT, "device wait gave up (code " + std::to_string(code) +
                                       "): results of the affected launches are not valid");
    std::string what;
    if (code & kFlagRopeRange) what += " a position outside the RoPE table, block table or pool;";
    if (code & kFlagSpanRange) what += " an attention span outside 1..max_span or the block table;";
    if (code & kFlagPageRange) what += " a block-table page outside the pool;";
    return fail(TTS_ERR_INVALID_ARG, "device data out of range (code " + std::to_string(code) +
                                         "):" + what + " those rows were skipped or read as zero");
  }
  return TTS_OK;
}

tts_status tts_proj_forward(tts_ctx* c, const void* x, int m, int k, const void* w, int n,
                            int epilogue, void* y, int ldy, void* stream) {
  if (!c || !x || !w || !y) return fail(TTS_ERR_INVALID_ARG, "proj: NULL argument");
  if (!aligned16(x) || !aligned16(w) || !aligned16(y))
    return fail(TTS_ERR_INVALID_ARG, "proj: pointers must be 16-byte aligned");
  if (epilogue < TTS_EPI_F32 || epilogue > TTS_EPI_SWIGLU_F16)
    return fail(TTS_ERR_INVALID_ARG, "proj: unknown epilogue");
  std::string why;
  if (!gemm_supported(m, k, n, epilogue, &why))
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "proj: " + why);
  if (m > c->max_lanes)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "proj: m exceeds the context's max_lanes");
  DeviceGuard g(c->device);
  GemmRequest r;
  r.w = static_cast<const __half*>(w);
  r.x = static_cast<const __half*>(x);
  r.m = m;
  r.k = k;
  r.n = n;
  r.epi = epilogue;
  r.y = y;
  r.ldy = ldy;
  r.pdl = false;
  return counted(launch_gemm(r, c->gemm, S(stream), c->device), "proj");
}

tts_status tts_interleave_gate_up(tts_ctx* c, const void* gate, const void* up, int ffn, int dim,
                                  void* out, void* stream) {
  if (!c || !gate || !up || !out) return fail(TTS_ERR_INVALID_ARG, "interleave: NULL argument");
  if (ffn % 64 || dim % 8)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "interleave: ffn % 64 and dim % 8 must be 0");
  DeviceGuard g(c->device);
  interleave_gate_up_kernel<<<1184, 256, 0, S(stream)>>>(static_cast<const __half*>(gate),
                                                        static_cast<const __half*>(up), ffn,
                                                        dim, static_cast<__half*>(out));
  return counted(cudaGetLastError(), "interleave");
}

tts_status tts_weight_pack(tts_ctx* c, const void* w, int n, int k, void* out, void* stream) {
  if (!c || !w || !out) return fail(TTS_ERR_INVALID_ARG, "weight_pack: NULL argument");
  if (n < 128 || n % 128 || k < 64 || k % 64)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "weight_pack: n % 128 and k % 64 must be 0");
  if (!aligned16(w) || !aligned16(out) || w == out)
    return fail(TTS_ERR_INVALID_ARG, "weight_pack: 16-byte aligned, distinct buffers");
  DeviceGuard g(c->device);
  pack_weight_kernel<<<1184, 256, 0, S(stream)>>>(static_cast<const __half*>(w), n, k,
                                                 static_cast<__half*>(out));
  return counted(cudaGetLastError(), "weight_pack");
}

tts_status tts_proj_forward_packed(tts_ctx* c, const void* x, int m, int k, const void* w, int n,
                                   int epilogue, void* y, int ldy, void* stream) {
  if (!c || !x || !w || !y) return fail(TTS_ERR_INVALID_ARG, "proj: NULL argument");
  if (!aligned16(x) || !aligned16(w) || !aligned16(y))
    return fail(TTS_ERR_INVALID_ARG, "proj: pointers must be 16-byte aligned");
  if (epilogue < TTS_EPI_F32 || epilogue > TTS_EPI_SWIGLU_F16)
    return fail(TTS_ERR_INVALID_ARG, "proj: unknown epilogue");
  std::string why;
  if (!gemm_supported(m, k, n, epilogue, &why))
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "proj: " + why);
  if (m > c->max_lanes)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "proj: m exceeds the context's max_lanes");
  DeviceGuard g(c->device);
  GemmRequest r;
  r.w = static_cast<const __half*>(w);
  r.packed = true;
  r.x = static_cast<const __half*>(x);
  r.m = m;
  r.k = k;
  r.n = n;
  r.epi = epilogue;
  r.y = y;
  r.ldy = ldy;
  r.pdl = false;
  return counted(launch_gemm(r, c->gemm, S(stream), c->device), "proj");
}

tts_status tts_proj_forward_rows(tts_ctx* c, const void* x, int rows, int k, const void* w, int n,
                                 int epilogue, void* y, int ldy, void* stream) {
  if (!c || !x || !w || !y) return fail(TTS_ERR_INVALID_ARG, "proj_rows: NULL argument");
  if (!aligned16(x) || !aligned16(w) || !aligned16(y))
    return fail(TTS_ERR_INVALID_ARG, "proj_rows: pointers must be 16-byte aligned");
  std::string why;
  if (!pf_gemm_supported(rows, k, n, epilogue, &why))
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "proj_rows: " + why);
  DeviceGuard g(c->device);
  PfGemmRequest r;
  r.x = static_cast<const __half*>(x);
  r.w = static_cast<const __half*>(w);
  r.rows = rows;
  r.k = k;
  r.n = n;
  r.epi = epilogue;
  r.y = y;
  r.ldy = ldy;
  return counted(launch_pf_gemm(r, S(stream), c->device, c->gemm.err), "proj_rows");
}

tts_status tts_rms_norm(tts_ctx* c, const float* x, const float* w, int rows, int dim, float eps,
                        float* y32, void* y16, void* stream) {
  if (!c || !x || !w || (!y32 && !y16)) return fail(TTS_ERR_INVALID_ARG, "rms_norm: NULL argument");
  DeviceGuard g(c->device);
  return counted(launch_rms_norm(x, w, rows, dim, eps, y32, static_cast<__half*>(y16), nullptr, 0,
                                 false, S(stream)),
                 "rms_norm");
}

tts_status tts_swiglu_mul(tts_ctx* c, const float* gate, const float* up, long n, void* y,
                          int y_f16, void* stream) {
  if (!c || !gate || !up || !y) return fail(TTS_ERR_INVALID_ARG, "swiglu_mul: NULL argument");
  DeviceGuard g(c->device);
  return counted(launch_swiglu(gate, up, y, y_f16 != 0, n, S(stream)), "swiglu_mul");
}

tts_status tts_snake_beta_nlc(tts_ctx* c, const void* x, int x_f16, const float* alpha,
                              const float* brecip, long rows, int chan, void* y, int y_f16,
                              void* stream) {
  if (!c || !x || !alpha || !brecip || !y)
    return fail(TTS_ERR_INVALID_ARG, "snake_beta_nlc: NULL argument");
  DeviceGuard g(c->device);
  return counted(launch_snake(x, x_f16 != 0, alpha, brecip, rows, chan, y, y_f16 != 0, S(stream)),
                 "snake_beta");
}

static bool kv_ok(const tts_kv_cache* kv, std::string* why) {
  if (!kv || !kv->k_pages || !kv->v_pages || !kv->block_table) {
    *why = "kv cache pointers are NULL";
    return false;
  }
  if (kv->head_dim != 128) {
    *why = "head_dim must be 128";
    return false;
  }
  if (kv->block_size < 1 || kv->max_blocks < 1 || kv->n_kv < 1) {
    *why = "empty kv cache geometry";
    return false;
  }
  return true;
}

tts_status tts_qk_rope_append(tts_ctx* c, const float* qkv, int lanes, int heads,
                              const float* norms, const float* cos_t, const float* sin_t,
                              int rope_len, const int* positions, const tts_kv_cache* kv,
                              float eps, float* q_out, void* stream) {
  std::string why;
  if (!c || !qkv || !norms || !cos_t || !sin_t || !positions || !q_out)
    return fail(TTS_ERR_INVALID_ARG, "qk_rope: NULL argument");
  if (!kv_ok(kv, &why)) return fail(TTS_ERR_INVALID_ARG, "qk_rope: " + why);
  if (lanes < 1 || heads < 1) return fail(TTS_ERR_INVALID_ARG, "qk_rope: empty shape");
  DeviceGuard g(c->device);
  QkRopeArgs a;
  a.norms = norms;
  a.cos_t = cos_t;
  a.sin_t = sin_t;
  a.positions = positions;
  a.block_table = kv->block_table;
  a.max_blocks = kv->max_blocks;
  a.block_size = kv->block_size;
  a.num_blocks = kv->num_blocks;
  a.rope_len = rope_len;
  a.err = c->gemm.err;
  a.k_pool = static_cast<__half*>(kv->k_pages);
  a.v_pool = static_cast<__half*>(kv->v_pages);
  a.q_out = q_out;
  a.heads = heads;
  a.n_kv = kv->n_kv;
  a.eps = eps;
  return counted(launch_qk_rope(qkv, a, lanes, false, S(stream)), "qk_rope");
}

tts_status tts_decode_attention(tts_ctx* c, const float* q, int lanes, int gqa,
                                const tts_kv_cache* kv, const int* spans, int max_span,
                                int window, void* out, int out_f16, void* stream) {
  std::string why;
  if (!c || !q || !spans || !out) return fail(TTS_ERR_INVALID_ARG, "decode_attention: NULL argument");
  if (!kv_ok(kv, &why)) return fail(TTS_ERR_INVALID_ARG, "decode_attention: " + why);
  if (gqa != 1 && gqa != 2 && gqa != 4 && gqa != 8)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "decode_attention: gqa must be 1, 2, 4 or 8");
  if (lanes < 1 || lanes > c->max_lanes || max_span < 1 || max_span > 8192)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE,
                "decode_attention: lanes must be in 1..max_lanes and max_span in 1..8192");
  DeviceGuard g(c->device);
  AttnRequest r;
  r.q = q;
  r.k_pool = static_cast<const __half*>(kv->k_pages);
  r.v_pool = static_cast<const __half*>(kv->v_pages);
  r.block_table = kv->block_table;
  r.max_blocks = kv->max_blocks;
  r.block_size = kv->block_size;
  r.num_blocks = kv->num_blocks;
  r.err = c->gemm.err;
  r.spans = spans;
  r.span_add = 0;
  r.max_span = max_span;
  r.window = window;
  r.lanes = lanes;
  r.n_kv = kv->n_kv;
  r.gqa = gqa;
  r.out = out;
  r.out_f16 = out_f16 != 0;
  r.pdl = false;
  return counted(launch_attn(r, c->attn, S(stream)), "decode_attention");
}

tts_status tts_decode_attention_static(const float* q, int lanes, int gqa,
                                       const tts_kv_cache* kv, const int* spans, int max_span,
                                       int window, void* out, int out_f16, void* stream) {
  std::string why;
  if (!q || !spans || !out)
    return fail(TTS_ERR_INVALID_ARG, "decode_attention_static: NULL argument");
  if (!kv_ok(kv, &why)) return fail(TTS_ERR_INVALID_ARG, "decode_attention_static: " + why);
  if (gqa != 1 && gqa != 2 && gqa != 4 && gqa != 8)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "decode_attention_static: gqa must be 1, 2, 4 or 8");
  if (lanes < 1 || max_span < 1 || max_span > 8192)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE,
                "decode_attention_static: lanes must be >= 1 and max_span in 1..8192");
  AttnRequest r;
  r.q = q;
  r.k_pool = static_cast<const __half*>(kv->k_pages);
  r.v_pool = static_cast<const __half*>(kv->v_pages);
  r.block_table = kv->block_table;
  r.max_blocks = kv->max_blocks;
  r.block_size = kv->block_size;
  r.num_blocks = kv->num_blocks;
  r.err = nullptr;
  r.spans = spans;
  r.span_add = 0;
  r.max_span = max_span;
  r.window = window;
  r.lanes = lanes;
  r.n_kv = kv->n_kv;
  r.gqa = gqa;
  r.out = out;
  r.out_f16 = out_f16 != 0;
  r.pdl = false;
  return counted(launch_attn_static(r, S(stream)), "decode_attention_static");
}

tts_status tts_decode_attention_static_check(void* stream) {
  int code = 0;
  const cudaError_t e = attn_static_status(S(stream), &code);
  if (e != cudaSuccess) return cuda_status(e, "decode_attention_static_check");
  if (code & kFlagWaitMask)
    return fail(TTS_ERR_TIMEOUT, "decode_attention_static: device wait gave up (code " +
                                     std::to_string(code) + "): the output is not valid");
  if (code) {
    std::string what;
    if (code & kFlagSpanRange) what += " a span outside 1..max_span or the block table;";
    if (code & kFlagPageRange) what += " a block-table page outside the pool;";
    return fail(TTS_ERR_INVALID_ARG, "decode_attention_static: device data out of range (code " +
                                         std::to_string(code) + "):" + what +
                                         " those positions were clamped or read as zero");
  }
  return TTS_OK;
}

tts_status tts_argmax(tts_ctx* c, const float* logits, int rows, int n,
                      const unsigned char* banned, unsigned int* out, void* stream) {
  if (!c || !logits || !out) return fail(TTS_ERR_INVALID_ARG, "argmax: NULL argument");
  if (rows < 1 || n < 1) return fail(TTS_ERR_INVALID_ARG, "argmax: empty shape");
  DeviceGuard g(c->device);
  return counted(launch_argmax(logits, rows, n, banned, out, S(stream)), "argmax");
}

tts_status tts_conv1d_nlc(tts_ctx* c, const void* x, int b, int len, int cin, const void* w,
                          int cout, int k, int dilation, int pad_left, const float* bias,
                          const float* alpha, const float* brecip, const void* res, void* y,
                          void* stream) {
  if (!c || !x || !w || !y) return fail(TTS_ERR_INVALID_ARG, "conv1d: NULL argument");
  if ((alpha == nullptr) != (brecip == nullptr))
    return fail(TTS_ERR_INVALID_ARG, "conv1d: alpha and brecip come together");
  if (!aligned16(x) || !aligned16(w) || !aligned16(y) || (res && !aligned16(res)))
    return fail(TTS_ERR_INVALID_ARG, "conv1d: pointers must be 16-byte aligned");
  ConvRequest r;
  r.x = static_cast<const __half*>(x);
  r.w = static_cast<const __half*>(w);
  r.bias = bias;
  r.alpha = alpha;
  r.brecip = brecip;
  r.res = static_cast<const __half*>(res);
  r.y = static_cast<__half*>(y);
  r.b = b;
  r.len = len;
  r.cin = cin;
  r.cout = cout;
  r.k = k;
  r.dil = dilation;
  r.pad_left = pad_left;
  std::string why;
  if (!conv_supported(r, &why)) return fail(TTS_ERR_UNSUPPORTED_SHAPE, "conv1d: " + why);
  DeviceGuard g(c->device);
  return counted(launch_conv(r, S(stream), c->device, c->gemm.err), "conv1d");
}

tts_status tts_topk_sample(tts_ctx* c, const float* logits, int rows, int n, const float* draws,
                           int k, float temperature, unsigned int* out, void* stream) {
  if (!c || !logits || !draws || !out) return fail(TTS_ERR_INVALID_ARG, "topk_sample: NULL argument");
  if (rows < 1) return fail(TTS_ERR_INVALID_ARG, "topk_sample: rows must be >= 1");
  if (k < 1 || k > kTopkMaxK || k > n || n > kTopkMaxN)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "topk_sample: k=" + std::to_string(k) + " n=" +
                                               std::to_string(n) + " outside the kernel's limits");
  DeviceGuard g(c->device);
  return counted(launch_topk_sample(logits, rows, n, n, draws, rows, k, temperature, out, 1,
                                    nullptr, nullptr, 0, nullptr, false, S(stream)),
                 "topk_sample");
}

// ---------------------------------------------------------------- codec front

tts_status tts_rvq_gather(tts_ctx* c, const unsigned int* codes, int T, int ncodes, int q0,
                          int nq, const float* tables, int entries, int dim, float* out,
                          void* stream) {
  if (!c || !codes || !tables || !out) return fail(TTS_ERR_INVALID_ARG, "rvq_gather: NULL argument");
  if (T < 1 || nq < 1 || q0 < 0 || q0 + nq > ncodes || entries < 1 || dim < 1)
    return fail(TTS_ERR_INVALID_ARG, "rvq_gather: T, nq >= 1 and q0 + nq <= ncodes");
  DeviceGuard g(c->device);
  return counted(launch_rvq_gather(codes, ncodes, q0, nq, tables, entries, dim, out, T, S(stream)),
                 "rvq_gather");
}

tts_status tts_rope_rows(tts_ctx* c, float* x, int T, int ld, int col0, int heads, int hd,
                         const float* cos_t, const float* sin_t, int pos0, void* stream) {
  if (!c || !x || !cos_t || !sin_t) return fail(TTS_ERR_INVALID_ARG, "rope_rows: NULL argument");
  if (T < 1 || heads < 1 || hd < 2 || hd % 2 || col0 < 0 || col0 + heads * hd > ld || pos0 < 0)
    return fail(TTS_ERR_INVALID_ARG, "rope_rows: even hd, heads fit in the row");
  DeviceGuard g(c->device);
  return counted(launch_rope_rows(x, T, ld, col0, heads, hd, cos_t, sin_t, pos0, S(stream)),
                 "rope_rows");
}

tts_status tts_window_attention(tts_ctx* c, const float* qkv, int T, int heads, int hd,
                                int window, float scale, void* out, int out_f16, void* stream) {
  if (!c || !qkv || !out) return fail(TTS_ERR_INVALID_ARG, "window_attention: NULL argument");
  if (T < 1 || heads < 1 || hd < 1 || hd > 128 || window < 0)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "window_attention: T, heads >= 1, hd in 1..128");
  DeviceGuard g(c->device);
  return counted(launch_window_attn(qkv, T, 3 * heads * hd, heads, hd, window, scale, out,
                                    out_f16 != 0, S(stream)),
                 "window_attention");
}

tts_status tts_layer_norm(tts_ctx* c, const float* x, const float* w, const float* b, int rows,
                          int dim, float eps, void* y, int y_f16, void* stream) {
  if (!c || !x || !w || !y) return fail(TTS_ERR_INVALID_ARG, "layer_norm: NULL argument");
  if (rows < 1 || dim < 1) return fail(TTS_ERR_INVALID_ARG, "layer_norm: empty shape");
  DeviceGuard g(c->device);
  return counted(launch_layer_norm(x, w, b, rows, dim, eps, y, y_f16 != 0, S(stream)),
                 "layer_norm");
}

tts_status tts_depthwise_conv(tts_ctx* c, const float* x, int b, int L, int C, const float* w,
                              int k, const float* bias, float* y, void* stream) {
  if (!c || !x || !w || !y) return fail(TTS_ERR_INVALID_ARG, "depthwise: NULL argument");
  if (b < 1 || L < 1 || C < 1 || k < 1) return fail(TTS_ERR_INVALID_ARG, "depthwise: empty shape");
  DeviceGuard g(c->device);
  return counted(launch_depthwise(x, w, bias, b, L, C, k, y, S(stream)), "depthwise");
}

tts_status tts_bias_act(tts_ctx* c, const float* y, int rows, int n, const float* bias, int act,
                        const float* scale, const float* res, void* out, int out_f16,
                        void* stream) {
  if (!c || !y || !out) return fail(TTS_ERR_INVALID_ARG, "bias_act: NULL argument");
  if (rows < 1 || n < 1 || act < 0 || act > 2)
    return fail(TTS_ERR_INVALID_ARG, "bias_act: empty shape or unknown activation");
  DeviceGuard g(c->device);
  return counted(launch_bias_act(y, rows, n, bias, act, scale, res, out, out_f16 != 0, S(stream)),
                 "bias_act");
}

// ---------------------------------------------------------------- stack

tts_status tts_stack_create(tts_ctx* c, const tts_stack_geometry* geo, tts_stack** out) {
  if (!c || !geo || !out) return fail(TTS_ERR_INVALID_ARG, "stack_create: NULL argument");
  const tts_stack_geometry& gm = *geo;
  if (gm.head_dim != 128 || gm.dim % 128 || gm.ffn % 64 || gm.layers < 1 || gm.heads < 1 ||
      gm.n_kv < 1 || gm.heads % gm.n_kv || (gm.heads / gm.n_kv) > 2 || gm.rope_len < 1)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE,
                "stack_create: need head_dim 128, dim % 128 == 0, ffn % 64 == 0, gqa 1 or 2");
  if (gm.codebooks < 0 || gm.codebooks > 64 || (gm.codebooks && gm.vocab % 128))
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "stack_create: 0..64 codebooks, vocab % 128 == 0");
  DeviceGuard g(c->device);
  auto* s = new tts_stack();
  s->ctx = c;
  s->geo = gm;
  s->layers.resize(gm.layers);
  const int L = c->max_lanes;
  const int qw = gm.heads * gm.head_dim;
  // RoPE table in f64, rounded to f32 (crates/tts-nn/src/lib.rs:1178-1205).
  std::vector<float> cs(size_t(gm.rope_len) * 64), sn(size_t(gm.rope_len) * 64);
  for (int t = 0; t < gm.rope_len; ++t)
    for (int i = 0; i < 64; ++i) {
      const double freq = 1.0 / std::pow(gm.rope_base, 2.0 * double(i) / 128.0);
      const double ph = double(t) * freq;
      cs[size_t(t) * 64 + i] = float(std::cos(ph));
      sn[size_t(t) * 64 + i] = float(std::sin(ph));
    }
  cudaError_t e = dmalloc(&s->rope_cos, cs.size() * 4);
  if (e == cudaSuccess) e = dmalloc(&s->rope_sin, sn.size() * 4);
  if (e == cudaSuccess) e = cudaMemcpy(s->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(s->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = dmalloc(&s->h, size_t(L) * gm.dim * 4);
  if (e == cudaSuccess) e = dmalloc(&s->xn, size_t(L) * std::max(gm.dim, qw) * 2);
  if (e == cudaSuccess) e = dmalloc(&s->q, size_t(L) * qw * 4);
  if (e == cudaSuccess) e = dmalloc(&s->attn, size_t(L) * qw * 2);
  if (e == cudaSuccess) e = dmalloc(&s->act, size_t(L) * gm.ffn * 2);
  if (e == cudaSuccess) e = dmalloc(&s->x_next, size_t(L) * gm.dim * 4);
  if (e == cudaSuccess) e = dmalloc(&s->keys, size_t(L) * std::max(1, gm.codebooks) * 8);
  if (e == cudaSuccess) e = dmalloc(&s->ss, size_t(L) * std::max(1, gm.dim / 128) * 4 + 16);
  if (e == cudaSuccess) e = dmalloc(&s->qk_desc, size_t(L) * sizeof(int4));
  if (e == cudaSuccess) e = dmalloc(&s->qk_rope, size_t(L) * 128 * 4);
  {
    const char* env = getenv("TTS_DEFER_NORM");
    s->defer_norm = !(env && *env == '0') && gm.dim % 128 == 0 && gm.dim / 128 <= 32;
  }
  if (e == cudaSuccess) e = cudaMemset(s->keys, 0, size_t(L) * std::max(1, gm.codebooks) * 8);
  if (e == cudaSuccess) e = cudaMemset(s->x_next, 0, size_t(L) * gm.dim * 4);
  if (e != cudaSuccess) {
    tts_stack_destroy(s);
    return cuda_status(e, "stack_create");
  }
  *out = s;
  return TTS_OK;
}

tts_status tts_stack_set_layer(tts_stack* s, int layer, const tts_layer_weights* w) {
  if (!s || !w) return fail(TTS_ERR_INVALID_ARG, "stack_set_layer: NULL argument");
  if (layer < 0 || layer >= s->geo.layers)
    return fail(TTS_ERR_INVALID_ARG, "stack_set_layer: layer out of range");
  if (!w->attn_norm || !w->ffn_norm || !w->wqkv || !w->qk_norms || !w->wo || !w->w_gate_up ||
      !w->w_down)
    return fail(TTS_ERR_INVALID_ARG, "stack_set_layer: every weight is required");
  s->layers[layer] = *w;
  return TTS_OK;
}

tts_status tts_stack_set_head(tts_stack* s, const float* final_norm, const void* heads,
                              const void* embed) {
  if (!s || !final_norm) return fail(TTS_ERR_INVALID_ARG, "stack_set_head: final_norm is required");
  s->final_norm = final_norm;
  s->heads = static_cast<const __half*>(heads);
  s->embed = static_cast<const __half*>(embed);
  return TTS_OK;
}

// Checks a caller's pick rule for a vocabulary of `vocab` ids and converts it.
static tts_status pick_rule_of(const tts_pick_rule* rule, int vocab, const char* op,
                               PickRule* out) {
  if (vocab < 32 || vocab % 32)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, std::string(op) + ": vocab must be a multiple of 32");
  if (!(rule->penalty > 0.f) || rule->min_new < 0 || rule->eos >= vocab)
    return fail(TTS_ERR_INVALID_ARG, std::string(op) + ": penalty > 0, min_new >= 0, eos < vocab");
  if ((rule->min_new > 0 && rule->eos >= 0 && !rule->frames) ||
      (rule->penalty != 1.f && !rule->counts))
    return fail(TTS_ERR_INVALID_ARG,
                std::string(op) + ": min_new needs frames, a penalty needs the counts");
  if ((rule->ban && !aligned16(rule->ban)) || (rule->counts && !aligned16(rule->counts)))
    return fail(TTS_ERR_INVALID_ARG, std::string(op) + ": ban and counts must be 16-byte aligned");
  PickRule p;
  p.ban = rule->ban;
  p.counts = rule->counts;
  p.frames = rule->frames;
  p.penalty = rule->penalty;
  p.eos = rule->eos;
  p.min_new = rule->min_new;
  p.vocab = vocab;
  *out = p;
  return TTS_OK;
}

tts_status tts_stack_set_pick(tts_stack* s, const tts_pick_rule* rule) {
  if (!s) return fail(TTS_ERR_INVALID_ARG, "stack_set_pick: stack is NULL");
  if (!rule) {
    s->pick = PickRule{};
    return TTS_OK;
  }
  if (s->geo.codebooks != 1)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "stack_set_pick: needs one codebook head");
  PickRule p;
  const tts_status st = pick_rule_of(rule, s->geo.vocab, "stack_set_pick", &p);
  if (st != TTS_OK) return st;
  s->pick = p;
  return TTS_OK;
}

tts_status tts_talker_pick(tts_ctx* c, const float* logits, int rows, int vocab,
                           const tts_pick_rule* rule, int record, unsigned int* out,
                           void* stream) {
  if (!c || !logits || !rule || !out) return fail(TTS_ERR_INVALID_ARG, "talker_pick: NULL argument");
  if (rows < 1) return fail(TTS_ERR_INVALID_ARG, "talker_pick: rows must be >= 1");
  if (!aligned16(logits)) return fail(TTS_ERR_INVALID_ARG, "talker_pick: logits must be 16-byte aligned");
  PickRule p;
  const tts_status st = pick_rule_of(rule, vocab, "talker_pick", &p);
  if (st != TTS_OK) return st;
  DeviceGuard g(c->device);
  return counted(launch_pick(logits, rows, p, record != 0, out, S(stream)), "talker_pick");
}

tts_status tts_stack_set_feedback(tts_stack* s, float* x_next) {
  if (!s) return fail(TTS_ERR_INVALID_ARG, "stack_set_feedback: stack is NULL");
  s->feedback = x_next;
  return TTS_OK;
}

tts_status tts_stack_destroy(tts_stack* s) {
  if (!s) return TTS_OK;
  DeviceGuard g(s->ctx->device);
  cudaFree(s->rope_cos);
  cudaFree(s->rope_sin);
  cudaFree(s->h);
  cudaFree(s->xn);
  cudaFree(s->q);
  cudaFree(s->attn);
  cudaFree(s->act);
  cudaFree(s->x_next);
  cudaFree(s->keys);
  cudaFree(s->ss);
  cudaFree(s->qk_desc);
  cudaFree(s->qk_rope);
  cudaFree(s->pre_map);
  cudaFree(s->pre_table);
  cudaFree(s->pre_pos);
  cudaFree(s->pf_buf);
  cudaFree(s->pf_blocks);
  delete s;
  return TTS_OK;
}

// The heads a step uses in place of the stack's own (the depth predictor's per-step head and
// its f32 resized table as the next input), and where its input and feedback live: with
// `in_h` the input is already in the residual stream buffer (no copy), with `feed_h` the next
// input is written there (the buffer is dead once the final norm has read it).
struct HeadSel {
  const __half* heads = nullptr;
  const float* embed32 = nullptr;
  bool in_h = false;
  bool feed_h = false;
  // top-k sampling in place of the greedy pick: the heads write `logits` [rows][vocab] and
  // row r draws draws[r % draw_rows]
  const float* draws = nullptr;
  int draw_rows = 0, top_k = 0;
  float temperature = 1.f;
  float* logits = nullptr;
};

static tts_status step_impl(tts_stack* s, const tts_decode_state* st, const float* x,
                            float* h_out, float* logits, unsigned int* codes, cudaStream_t cs,
                            const HeadSel* hsel = nullptr) {
  const tts_stack_geometry& gm = s->geo;
  const __half* heads = hsel ? hsel->heads : s->heads;
  const __half* embed16 = hsel ? nullptr : s->embed;
  const float* embed32 = hsel ? hsel->embed32 : nullptr;
  const bool feed = embed16 || embed32;
  tts_ctx* c = s->ctx;
  if (!st || !st->positions || !st->block_table || !st->k_pages || !st->v_pages)
    return fail(TTS_ERR_INVALID_ARG, "decode_step: state pointers are NULL");
  const int B = st->lanes;
  if (B < 1 || B > c->max_lanes)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "decode_step: lanes must be in 1..max_lanes");
  if (st->max_span < 1 || st->max_span > std::min(8192, gm.rope_len))
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "decode_step: max_span must be in 1..min(8192, rope_len)");
  for (int l = 0; l < gm.layers; ++l)
    if (!s->layers[l].wqkv) return fail(TTS_ERR_INVALID_ARG, "decode_step: layer weights not set");
  if (!s->final_norm) return fail(TTS_ERR_INVALID_ARG, "decode_step: final norm not set");
  if ((logits || codes) && !heads)
    return fail(TTS_ERR_INVALID_ARG, "decode_step: logits/codes need codebook heads");

  const int D = gm.dim, qw = gm.heads * gm.head_dim, nqkv = (gm.heads + 2 * gm.n_kv) * 128;
  const size_t layer_pages = size_t(st->num_blocks) * gm.n_kv * st->block_size * 128;
  tts_status rc;
#define TTS_TRY(expr, op)                     \
  do {                                        \
    if ((rc = counted((expr), op)) != TTS_OK) \
      return rc;                              \
  } while (0)

  float* next = hsel && hsel->feed_h ? s->h : (s->feedback ? s->feedback : s->x_next);
  const float* src = x ? x : next;
  // The step begins with a copy into the residual stream (a full stream dependency on
  // everything earlier, the position advance included), and none of its kernels writes the
  // positions or the block table before the final code gather: the attention may split its
  // work and resolve its pages before its dependency wait. TTS_ATTN_EARLY_META=0: off (A/B).
  const bool step_copies_input = !(hsel && hsel->in_h);
  const char* early_env = getenv("TTS_ATTN_EARLY_META");
  const bool early_meta_on = !(early_env && *early_env == '0');
  if (!(hsel && hsel->in_h) &&
      (rc = cuda_status(cudaMemcpyAsync(s->h, src, size_t(B) * D * 4, cudaMemcpyDeviceToDevice, cs),
                        "decode_step")) != TTS_OK)
    return rc;

  // each projection (and the attention) prefetches the head of the next projection's weights
  // into L2 once its own stream is out (separate-kernel path)
  // (TTS_L2_PREFETCH_MB overrides the budget for A/B measurement; 0 turns it off)
  const char* pf_env = getenv("TTS_L2_PREFETCH_MB");
  const size_t pf_budget = pf_env && *pf_env ? size_t(atoi(pf_env)) << 20 : s->pf_budget;
  auto pf = [&](const void* w, int k, int n) {
    return pf_budget ? gemm_prefetch_plan(w, B, k, n, c->device, pf_budget) : L2Prefetch{};
  };
  // each lane's QK-rope operands once per step for every layer's QKV epilogue (the
  // separate-kernel path; TTS_QK_ROWS=0 turns it off for A/B measurement)
  const char* rows_env = getenv("TTS_QK_ROWS");
  const bool rows_on = !(rows_env && *rows_env == '0');
  auto pages = [&](int l, bool v) {
    return (v ? static_cast<__half*>(st->v_pages) : static_cast<__half*>(st->k_pages)) +
           layer_pages * l;
  };
  // the step's projections (qwen3.rs:339-463), as requests for either path
  auto req_qkv = [&](int l) {
    const tts_layer_weights& w = s->layers[l];
    GemmRequest r;
    r.w = static_cast<const __half*>(w.wqkv);
    r.packed = true;
    r.x = s->xn;
    r.m = B;
    r.k = D;
    r.n = nqkv;
    r.epi = EPI_QKROPE;
    r.qk.norms = w.qk_norms;
    r.qk.cos_t = s->rope_cos;
    r.qk.sin_t = s->rope_sin;
    r.qk.positions = st->positions;
    r.qk.block_table = st->block_table;
    r.qk.max_blocks = st->max_blocks;
    r.qk.block_size = st->block_size;
    r.qk.num_blocks = st->num_blocks;
    r.qk.rope_len = gm.rope_len;
    r.qk.err = c->gemm.err;
    r.qk.k_pool = pages(l, false);
    r.qk.v_pool = pages(l, true);
    r.qk.q_out = s->q;
    r.qk.heads = gm.heads;
    r.qk.n_kv = gm.n_kv;
    r.qk.eps = gm.eps;
    if (rows_on) {
      r.qk.rows_desc = s->qk_desc;
      r.qk.rows_rope = s->qk_rope;
    }
    return r;
  };
  auto req_o = [&](int l) {
    GemmRequest o;
    o.w = static_cast<const __half*>(s->layers[l].wo);
    o.packed = true;
    o.x = s->attn;
    o.m = B;
    o.k = qw;
    o.n = D;
    o.epi = EPI_RESIDUAL;
    o.y = s->h;
    return o;
  };
  auto req_gu = [&](int l) {
    GemmRequest gu;
    gu.w = static_cast<const __half*>(s->layers[l].w_gate_up);
    gu.packed = true;
    gu.x = s->xn;
    gu.m = B;
    gu.k = D;
    gu.n = 2 * gm.ffn;
    gu.epi = EPI_SWIGLU;
    gu.y = s->act;
    return gu;
  };
  auto req_dn = [&](int l) {
    GemmRequest dn;
    dn.w = static_cast<const __half*>(s->layers[l].w_down);
    dn.packed = true;
    dn.x = s->act;
    dn.m = B;
    dn.k = gm.ffn;
    dn.n = D;
    dn.epi = EPI_RESIDUAL;
    dn.y = s->h;
    return dn;
  };
  auto req_heads = [&]() {
    GemmRequest hd;
    hd.w = heads;
    hd.packed = true;
    hd.x = s->xn;
    hd.m = B;
    hd.k = D;
    hd.n = gm.codebooks * gm.vocab;
    hd.epi = EPI_ARGMAX;
    hd.y = logits;
    hd.argmax_keys = s->keys;
    hd.vocab = gm.vocab;
    if (!hsel) hd.pick = s->pick;
    if (hsel && hsel->draws) {
      hd.epi = EPI_F32;
      hd.y = hsel->logits;
      hd.argmax_keys = nullptr;
    }
    return hd;
  };
  auto req_attn = [&](int l) {
    AttnRequest ar;
    ar.q = s->q;
    ar.k_pool = pages(l, false);
    ar.v_pool = pages(l, true);
    ar.block_table = st->block_table;
    ar.max_blocks = st->max_blocks;
    ar.block_size = st->block_size;
    ar.num_blocks = st->num_blocks;
    ar.err = c->gemm.err;
    ar.spans = st->positions;
    ar.span_add = 1;
    ar.max_span = st->max_span;
    ar.window = 0;
    ar.lanes = B;
    ar.n_kv = gm.n_kv;
    ar.gqa = gm.heads / gm.n_kv;
    ar.out = s->attn;
    ar.out_f16 = true;
    return ar;
  };
  const int nkeys = heads ? B * gm.codebooks : 0;

  {
    // RMSNorm deferred into the projections: the norm's input is f16(h * w), the projection's
    // rows are divided by the RMS in its epilogue, and the O and down projections produce the
    // next norm's input and sums of squares (every row is complete in their epilogues)
    const bool defer = s->defer_norm;
    const int ss_tiles = D / 128;
    auto consume = [&](GemmRequest& r, int tiles) {
      r.ss_in = s->ss;
      r.ss_tiles = tiles;
      r.ss_dim = D;
      r.ss_eps = gm.eps;
    };
    auto produce = [&](GemmRequest& r, const float* norm_w) {
      r.norm_w = norm_w;
      r.norm_x16 = s->xn;
      r.ss_out = s->ss;
    };
    if (rows_on) TTS_TRY(launch_qk_rows(req_qkv(0).qk, B, s->qk_desc, s->qk_rope, true, cs),
                         "qk_rows");
    if (defer)
      TTS_TRY(launch_norm_defer(s->h, s->layers[0].attn_norm, B, D, s->xn, s->ss, true, cs),
              "rms_norm");
    for (int l = 0; l < gm.layers; ++l) {
      const tts_layer_weights& w = s->layers[l];
      // attention block (qwen3.rs:339-451)
      if (!defer)
        TTS_TRY(launch_rms_norm(s->h, w.attn_norm, B, D, gm.eps, nullptr, s->xn, nullptr, 0, true,
                                cs),
                "rms_norm");
      GemmRequest qkv = req_qkv(l);
      if (defer) consume(qkv, l == 0 ? 1 : ss_tiles);
      TTS_TRY(launch_gemm(qkv, c->gemm, cs, c->device), "proj");
      AttnRequest ar = req_attn(l);
      ar.next = pf(w.wo, qw, D);
      ar.early_meta = step_copies_input && early_meta_on;
      TTS_TRY(launch_attn(ar, c->attn, cs), "decode_attention");
      GemmRequest o = req_o(l);
      o.next = pf(w.w_gate_up, D, 2 * gm.ffn);
      if (defer) produce(o, w.ffn_norm);
      TTS_TRY(launch_gemm(o, c->gemm, cs, c->device), "proj");
      // feed-forward block (qwen3.rs:453-463)
      if (!defer)
        TTS_TRY(launch_rms_norm(s->h, w.ffn_norm, B, D, gm.eps, nullptr, s->xn, nullptr, 0, true,
                                cs),
                "rms_norm");
      GemmRequest gu = req_gu(l);
      gu.next = pf(w.w_down, gm.ffn, D);
      if (defer) consume(gu, ss_tiles);
      TTS_TRY(launch_gemm(gu, c->gemm, cs, c->device), "proj");
      GemmRequest dn = req_dn(l);
      if (l + 1 < gm.layers)
        dn.next = pf(s->layers[l + 1].wqkv, D, nqkv);
      else if (heads)
        dn.next = pf(heads, D, gm.codebooks * gm.vocab);
      if (defer && l + 1 < gm.layers) produce(dn, s->layers[l + 1].attn_norm);
      TTS_TRY(launch_gemm(dn, c->gemm, cs, c->device), "proj");
    }
    // final norm (qwen3.rs:466), heads + greedy pick, next input
    TTS_TRY(launch_rms_norm(s->h, s->final_norm, B, D, gm.eps, h_out, s->xn,
                            heads ? s->keys : nullptr, nkeys, true, cs),
            "rms_norm");
    if (heads) {
      TTS_TRY(launch_gemm(req_heads(), c->gemm, cs, c->device), "proj");
      if (hsel && hsel->draws)
        TTS_TRY(launch_topk_sample(hsel->logits, B, gm.vocab, gm.vocab, hsel->draws,
                                   hsel->draw_rows, hsel->top_k, hsel->temperature, codes, 1,
                                   embed32, feed ? next : nullptr, D, st->positions, true, cs),
                "topk_sample");
      else
        TTS_TRY(launch_keys_to_codes(s->keys, B, gm.codebooks, gm.vocab, embed16, embed32, D,
                                     codes, feed ? next : nullptr, nullptr, st->positions,
                                     hsel ? nullptr : &s->pick, true, cs),
                "keys_to_codes");
    }
  }
  // with heads, the code gather advanced the positions
  if (!heads) TTS_TRY(launch_advance_positions(st->positions, B, true, cs), "advance_positions");
#undef TTS_TRY
  return TTS_OK;
}

extern "C++" {
template <class Fn>
static tts_status capture_graph(cudaStream_t cs, tts_graph** out, Fn&& body) {
  const long long before = g_launches;
  cudaError_t e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return cuda_status(e, "graph_capture");
  tts_status rc = body(cs);
  cudaGraph_t graph = nullptr;
  e = cudaStreamEndCapture(cs, &graph);
  const long long kernels = g_launches - before;
  g_launches = before;  // capture launches nothing
  if (rc != TTS_OK) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) return cuda_status(e, "graph_capture");
  auto* gr = new tts_graph();
  gr->graph = graph;
  gr->kernels = kernels;
  e = cudaGraphInstantiate(&gr->exec, graph, 0);
  if (e != cudaSuccess) {
    tts_graph_destroy(gr);
    return cuda_status(e, "graph_capture");
  }
  *out = gr;
  return TTS_OK;
}
}  // extern "C++"

// Stack::forward at t > 1 (qwen3.rs:294-467 with a multi-position input): every new row of
// every lane runs as a decode row of its own (its lane's pages, its own position), in chunks of
// up to max_lanes rows; the QKV epilogue writes a chunk's K/V before its attention reads them, so
// each row sees the lane's earlier rows, as the causal mask does.
// The prompt prefill layer by layer over every row at once (qwen3.rs:294-467 at t > 1): each
// projection is one prefill-shaped GEMM over all rows (token rows as the MMA's M), the QK-norm,
// RoPE and KV append run per (row, head), the attention per row in runs of at most max_lanes
// rows (each row attends to its lane's positions up to its own, already appended at this layer).
// `s->pre_map` holds the rows' (lane, offset) pairs.
static bool prefill_layer_major_ok(const tts_stack* s) {
  const tts_stack_geometry& gm = s->geo;
  const int D = gm.dim, qw = gm.heads * gm.head_dim, nqkv = (gm.heads + 2 * gm.n_kv) * 128;
  const char* env = getenv("TTS_PREFILL_DECODE");  // 1: the decode-row path, for A/B
  if (env && *env == '1') return false;
  return gm.head_dim == 128 && pf_gemm_supported(1, D, nqkv, EPI_F32, nullptr) &&
         pf_gemm_supported(1, qw, D, EPI_RESIDUAL, nullptr) &&
         pf_gemm_supported(1, D, 2 * gm.ffn, EPI_SWIGLU, nullptr) &&
         pf_gemm_supported(1, gm.ffn, D, EPI_RESIDUAL, nullptr);
}

static tts_status prefill_layer_major(tts_stack* s, const tts_decode_state* st, const int* lens,
                                      long rows, const float* x, float* h_out, cudaStream_t cs) {
  tts_ctx* c = s->ctx;
  const tts_stack_geometry& gm = s->geo;
  const int D = gm.dim, qw = gm.heads * gm.head_dim, nqkv = (gm.heads + 2 * gm.n_kv) * 128;
  const int F = gm.ffn;
  if (!st->k_pages || !st->v_pages)
    return fail(TTS_ERR_INVALID_ARG, "stack_prefill: state pointers are NULL");
  if (st->max_span < 1 || st->max_span > std::min(8192, gm.rope_len))
    return fail(TTS_ERR_UNSUPPORTED_SHAPE,
                "stack_prefill: max_span must be in 1..min(8192, rope_len)");
  for (int l = 0; l < gm.layers; ++l)
    if (!s->layers[l].wqkv) return fail(TTS_ERR_INVALID_ARG, "stack_prefill: layer weights not set");
  if (h_out && !s->final_norm) return fail(TTS_ERR_INVALID_ARG, "stack_prefill: final norm not set");
  auto up = [](size_t b) { return (b + 255) / 256 * 256; };
  const size_t b_h = up(size_t(rows) * D * 4), b_x16 = up(size_t(rows) * std::max(D, qw) * 2);
  const size_t b_qkv = up(size_t(rows) * nqkv * 4), b_q = up(size_t(rows) * qw * 4);
  const size_t b_act = up(size_t(rows) * F * 2), b_tab = up(size_t(rows) * st->max_blocks * 4);
  const size_t b_pos = up(size_t(rows) * 4);
  const size_t need = b_h + b_x16 + b_qkv + b_q + b_act + b_tab + b_pos;
  if (need > s->pf_bytes) {
    cudaFree(s->pf_buf);
    s->pf_buf = nullptr;
    s->pf_bytes = 0;
    cudaError_t e = dmalloc(&s->pf_buf, need);
    if (e != cudaSuccess) return cuda_status(e, "stack_prefill");
    s->pf_bytes = need;
  }
  unsigned char* p = s->pf_buf;
  float* h = reinterpret_cast<float*>(p);
  __half* x16 = reinterpret_cast<__half*>(p += b_h);
  float* qkv = reinterpret_cast<float*>(p += b_x16);
  float* q = reinterpret_cast<float*>(p += b_qkv);
  __half* act = reinterpret_cast<__half*>(p += b_q);
  int* table = reinterpret_cast<int*>(p += b_act);
  int* pos = reinterpret_cast<int*>(p += b_tab);
  const size_t layer_pages = size_t(st->num_blocks) * gm.n_kv * st->block_size * 128;
  tts_status rc;
#define TTS_TRY(expr, op)                     \
  do {                                        \
    if ((rc = counted((expr), op)) != TTS_OK) \
      return rc;                              \
  } while (0)
  TTS_TRY(launch_prefill_rows(s->pre_map, int(rows), st->block_table, st->max_blocks,
                              st->positions, table, pos, cs),
          "stack_prefill");
  if ((rc = cuda_status(cudaMemcpyAsync(h, x, size_t(rows) * D * 4, cudaMemcpyDeviceToDevice, cs),
                        "stack_prefill")) != TTS_OK)
    return rc;
  auto proj = [&](const void* w, const __half* xin, int k, int n, int epi, void* y) {
    PfGemmRequest r;
    r.x = xin;
    r.w = static_cast<const __half*>(w);
    r.rows = int(rows);
    r.k = k;
    r.n = n;
    r.epi = epi;
    r.y = y;
    return launch_pf_gemm(r, cs, c->device, c->gemm.err);
  };
  // the prompt attention (a lane's query rows in blocks of 64 against its keys) where it
  // applies (GQA 2, max_span <= 256: every lane's keys fit its two TMEM chunks); elsewhere, or
  // with TTS_PREFILL_ATTN=0, the decode attention runs per prompt row
  const char* pa_env = getenv("TTS_PREFILL_ATTN");
  const bool use_pfa = !(pa_env && *pa_env == '0') &&
                       pf_attn_supported(gm.heads, gm.n_kv, st->block_size, st->max_span);
  int n_qblocks = 0;
  if (use_pfa) {
    std::vector<int> qb;
    long base = 0;
    for (int b = 0; b < st->lanes; ++b) {
      for (int i0 = 0; i0 < lens[b]; i0 += 64) {
        qb.push_back(b);
        qb.push_back(int(base + i0));
        qb.push_back(i0);
        qb.push_back(std::min(64, lens[b] - i0));
      }
      base += lens[b];
    }
    n_qblocks = int(qb.size() / 4);
    if (qb.size() > s->pf_blocks_ints) {
      cudaFree(s->pf_blocks);
      s->pf_blocks = nullptr;
      s->pf_blocks_ints = 0;
      cudaError_t e = dmalloc(&s->pf_blocks, qb.size() * 4);
      if (e != cudaSuccess) return cuda_status(e, "stack_prefill");
      s->pf_blocks_ints = qb.size();
    }
    // a pageable source: the copy has read it when the call returns
    if ((rc = cuda_status(cudaMemcpyAsync(s->pf_blocks, qb.data(), qb.size() * 4,
                                          cudaMemcpyHostToDevice, cs),
                          "stack_prefill")) != TTS_OK)
      return rc;
  }
  for (int l = 0; l < gm.layers; ++l) {
    const tts_layer_weights& w = s->layers[l];
    __half* kp = static_cast<__half*>(st->k_pages) + layer_pages * l;
    __half* vp = static_cast<__half*>(st->v_pages) + layer_pages * l;
    TTS_TRY(launch_rms_norm(h, w.attn_norm, int(rows), D, gm.eps, nullptr, x16, nullptr, 0, true,
                            cs),
            "rms_norm");
    TTS_TRY(proj(w.wqkv, x16, D, nqkv, EPI_F32, qkv), "proj_rows");
    QkRopeArgs qa;
    qa.norms = w.qk_norms;
    qa.cos_t = s->rope_cos;
    qa.sin_t = s->rope_sin;
    qa.positions = pos;
    qa.block_table = table;
    qa.max_blocks = st->max_blocks;
    qa.block_size = st->block_size;
    qa.num_blocks = st->num_blocks;
    qa.rope_len = gm.rope_len;
    qa.err = c->gemm.err;
    qa.k_pool = kp;
    qa.v_pool = vp;
    qa.q_out = q;
    qa.heads = gm.heads;
    qa.n_kv = gm.n_kv;
    qa.eps = gm.eps;
    TTS_TRY(launch_qk_rope(qkv, qa, int(rows), true, cs), "qk_rope");
    if (use_pfa) {
      PfAttnRequest pa;
      pa.q = q;
      pa.blocks = s->pf_blocks;
      pa.n_blocks = n_qblocks;
      pa.positions = st->positions;
      pa.block_table = st->block_table;
      pa.max_blocks = st->max_blocks;
      pa.block_size = st->block_size;
      pa.num_blocks = st->num_blocks;
      pa.heads = gm.heads;
      pa.n_kv = gm.n_kv;
      pa.max_span = st->max_span;
      pa.k_pool = kp;
      pa.v_pool = vp;
      pa.out = x16;
      pa.err = c->gemm.err;
      TTS_TRY(launch_pf_attn(pa, cs), "prefill_attention");
    }
    for (long r0 = 0; r0 < rows && !use_pfa; r0 += c->max_lanes) {
      const int n = int(std::min<long>(c->max_lanes, rows - r0));
      AttnRequest ar;
      ar.q = q + size_t(r0) * qw;
      ar.k_pool = kp;
      ar.v_pool = vp;
      ar.block_table = table + size_t(r0) * st->max_blocks;
      ar.max_blocks = st->max_blocks;
      ar.block_size = st->block_size;
      ar.num_blocks = st->num_blocks;
      ar.err = c->gemm.err;
      ar.spans = pos + r0;
      ar.span_add = 1;
      ar.max_span = st->max_span;
      ar.window = 0;
      ar.lanes = n;
      ar.n_kv = gm.n_kv;
      ar.gqa = gm.heads / gm.n_kv;
      ar.out = x16 + size_t(r0) * qw;
      ar.out_f16 = true;
      TTS_TRY(launch_attn(ar, c->attn, cs), "decode_attention");
    }
    TTS_TRY(proj(w.wo, x16, qw, D, EPI_RESIDUAL, h), "proj_rows");
    TTS_TRY(launch_rms_norm(h, w.ffn_norm, int(rows), D, gm.eps, nullptr, x16, nullptr, 0, true,
                            cs),
            "rms_norm");
    TTS_TRY(proj(w.w_gate_up, x16, D, 2 * F, EPI_SWIGLU, act), "proj_rows");
    TTS_TRY(proj(w.w_down, act, F, D, EPI_RESIDUAL, h), "proj_rows");
  }
  if (h_out)
    TTS_TRY(launch_rms_norm(h, s->final_norm, int(rows), D, gm.eps, h_out, nullptr, nullptr, 0,
                            true, cs),
            "rms_norm");
#undef TTS_TRY
  return TTS_OK;
}

static tts_status prefill_impl(tts_stack* s, const tts_decode_state* st, const int* lens,
                               const float* x, float* h_out, cudaStream_t cs) {
  tts_ctx* c = s->ctx;
  if (!st || !lens || !x || !st->positions || !st->block_table)
    return fail(TTS_ERR_INVALID_ARG, "stack_prefill: NULL argument");
  const int lanes = st->lanes;
  if (lanes < 1 || st->max_blocks < 1)
    return fail(TTS_ERR_INVALID_ARG, "stack_prefill: lanes and max_blocks must be >= 1");
  std::vector<int> host;
  long rows = 0;
  for (int i = 0; i < lanes; ++i) {
    if (lens[i] < 0) return fail(TTS_ERR_INVALID_ARG, "stack_prefill: negative length");
    rows += lens[i];
  }
  if (rows < 1) return TTS_OK;
  if (rows > (1L << 24)) return fail(TTS_ERR_UNSUPPORTED_SHAPE, "stack_prefill: too many rows");
  host.reserve(size_t(2 * rows + lanes));
  for (int i = 0; i < lanes; ++i)
    for (int t = 0; t < lens[i]; ++t) {
      host.push_back(i);
      host.push_back(t);
    }
  for (int i = 0; i < lanes; ++i) host.push_back(lens[i]);
  const int chunk = c->max_lanes;
  const size_t table_ints = size_t(chunk) * st->max_blocks;
  cudaError_t e = cudaSuccess;
  if (host.size() > s->pre_map_ints) {
    cudaFree(s->pre_map);
    s->pre_map = nullptr;
    s->pre_map_ints = 0;
    e = dmalloc(&s->pre_map, host.size() * 4);
    if (e == cudaSuccess) s->pre_map_ints = host.size();
  }
  if (e == cudaSuccess && table_ints > s->pre_table_ints) {
    cudaFree(s->pre_table);
    cudaFree(s->pre_pos);
    s->pre_table = nullptr;
    s->pre_pos = nullptr;
    s->pre_table_ints = 0;
    e = dmalloc(&s->pre_table, table_ints * 4);
    if (e == cudaSuccess) e = dmalloc(&s->pre_pos, size_t(chunk) * 4);
    if (e == cudaSuccess) s->pre_table_ints = table_ints;
  }
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(s->pre_map, host.data(), host.size() * 4, cudaMemcpyHostToDevice, cs);
  if (e != cudaSuccess) return cuda_status(e, "stack_prefill");
  const int D = s->geo.dim;
  tts_status rc;
  if (prefill_layer_major_ok(s)) {
    if ((rc = prefill_layer_major(s, st, lens, rows, x, h_out, cs)) != TTS_OK) return rc;
    return counted(launch_advance_by(st->positions, s->pre_map + 2 * rows, lanes, cs),
                   "stack_prefill");
  }
  for (long r0 = 0; r0 < rows; r0 += chunk) {
    const int n = int(std::min<long>(chunk, rows - r0));
    if ((rc = counted(launch_prefill_rows(s->pre_map + 2 * r0, n, st->block_table, st->max_blocks,
                                          st->positions, s->pre_table, s->pre_pos, cs),
                      "stack_prefill")) != TTS_OK)
      return rc;
    tts_decode_state rowst = *st;
    rowst.lanes = n;
    rowst.positions = s->pre_pos;
    rowst.block_table = s->pre_table;
    HeadSel none;  // no heads: the prompt's rows pick nothing
    rc = step_impl(s, &rowst, x + size_t(r0) * D, h_out ? h_out + size_t(r0) * D : nullptr,
                   nullptr, nullptr, cs, &none);
    if (rc != TTS_OK) return rc;
  }
  return counted(launch_advance_by(st->positions, s->pre_map + 2 * rows, lanes, cs),
                 "stack_prefill");
}

tts_status tts_stack_prefill(tts_stack* s, const tts_decode_state* st, const int* lens,
                             const float* x, float* h_out, void* stream) {
  if (!s) return fail(TTS_ERR_INVALID_ARG, "stack_prefill: stack is NULL");
  DeviceGuard g(s->ctx->device);
  return prefill_impl(s, st, lens, x, h_out, S(stream));
}

tts_status tts_stack_decode_step(tts_stack* s, const tts_decode_state* st, const float* x,
                                 float* h_out, float* logits, unsigned int* codes, void* stream) {
  if (!s) return fail(TTS_ERR_INVALID_ARG, "decode_step: stack is NULL");
  DeviceGuard g(s->ctx->device);
  return step_impl(s, st, x, h_out, logits, codes, S(stream));
}

tts_status tts_stack_graph_capture(tts_stack* s, const tts_decode_state* st, const float* x,
                                   float* h_out, float* logits, unsigned int* codes, void* stream,
                                   tts_graph** out) {
  if (!s || !out) return fail(TTS_ERR_INVALID_ARG, "graph_capture: NULL argument");
  if (!stream) return fail(TTS_ERR_INVALID_ARG, "graph_capture: needs a non-legacy stream");
  DeviceGuard g(s->ctx->device);
  return capture_graph(S(stream), out, [&](cudaStream_t cs) {
    return step_impl(s, st, x, h_out, logits, codes, cs);
  });
}

tts_status tts_graph_launch(tts_graph* g, void* stream) {
  if (!g) return fail(TTS_ERR_INVALID_ARG, "graph_launch: NULL graph");
  cudaError_t e = cudaGraphLaunch(g->exec, S(stream));
  if (e == cudaSuccess) g_launches += g->kernels;
  return cuda_status(e, "graph_launch");
}

tts_status tts_graph_destroy(tts_graph* g) {
  if (!g) return TTS_OK;
  if (g->exec) cudaGraphExecDestroy(g->exec);
  if (g->graph) cudaGraphDestroy(g->graph);
  delete g;
  return TTS_OK;
}

// ---------------------------------------------------------------- depth predictor

tts_status tts_predictor_create(tts_stack* s, const tts_predictor_weights* w,
                                tts_predictor** out) {
  if (!s || !w || !out) return fail(TTS_ERR_INVALID_ARG, "predictor_create: NULL argument");
  const tts_stack_geometry& gm = s->geo;
  if (!w->resize || !w->heads || !w->resized || !w->tables)
    return fail(TTS_ERR_INVALID_ARG, "predictor_create: resize, heads, resized and tables are required");
  if (gm.codebooks != 1 || gm.vocab < 128)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE,
                "predictor_create: the stack needs codebooks = 1 (one head per depth step)");
  if (w->steps < 1 || w->steps > 64 || w->embed_dim < 64 || w->embed_dim % 64)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "predictor_create: 1..64 steps, embed_dim % 64 == 0");
  if (gm.rope_len < w->steps + 1)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "predictor_create: rope_len must cover steps + 1");
  if (!aligned16(w->resize) || !aligned16(w->heads) || !aligned16(w->resized) ||
      !aligned16(w->tables))
    return fail(TTS_ERR_INVALID_ARG, "predictor_create: weights must be 16-byte aligned");
  tts_ctx* c = s->ctx;
  DeviceGuard g(c->device);
  auto* p = new tts_predictor();
  p->s = s;
  s->pf_budget = 0;
  p->w = *w;
  p->max_lanes = c->max_lanes / 2;
  const int D = gm.dim, E = w->embed_dim, R = 2 * p->max_lanes;
  if (p->max_lanes < 1) {
    delete p;
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "predictor_create: the context needs max_lanes >= 2");
  }
  cudaError_t e = dmalloc(&p->resize2, size_t(D) * 2 * E * 2);
  __half* plain2 = nullptr;
  if (e == cudaSuccess) e = dmalloc(&plain2, size_t(D) * 2 * E * 2);
  // [W | W] along k, then packed for the GEMM
  if (e == cudaSuccess)
    e = cudaMemcpy2D(plain2, size_t(2) * E * 2, w->resize, size_t(E) * 2, size_t(E) * 2, D,
                     cudaMemcpyDeviceToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy2D(plain2 + E, size_t(2) * E * 2, w->resize, size_t(E) * 2, size_t(E) * 2, D,
                     cudaMemcpyDeviceToDevice);
  if (e == cudaSuccess) {
    pack_weight_kernel<<<1184, 256>>>(plain2, D, 2 * E, p->resize2);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaFree(plain2);
  if (e == cudaSuccess) e = dmalloc(&p->x16, size_t(R) * 2 * E * 2);
  if (e == cudaSuccess) e = dmalloc(&p->table2, size_t(R) * kPredictorMaxBlocks * 4);
  if (e == cudaSuccess) e = dmalloc(&p->pos2, size_t(R) * 4);
  if (e == cudaSuccess) e = dmalloc(&p->step_codes, size_t(w->steps) * R * 4);
  if (e == cudaSuccess) e = dmalloc(&p->logits, size_t(R) * gm.vocab * 4);
  if (e == cudaSuccess) e = cudaMemset(p->step_codes, 0, size_t(w->steps) * R * 4);
  if (e != cudaSuccess) {
    tts_predictor_destroy(p);
    return cuda_status(e, "predictor_create");
  }
  *out = p;
  return TTS_OK;
}

tts_status tts_predictor_set_sampling(tts_predictor* p, const float* draws, int stride,
                                      int top_k, float temperature) {
  if (!p) return fail(TTS_ERR_INVALID_ARG, "predictor_set_sampling: predictor is NULL");
  if (!draws) {
    p->draws = nullptr;
    return TTS_OK;
  }
  if (stride < 1 || top_k < 1 || top_k > kTopkMaxK || top_k > p->s->geo.vocab ||
      p->s->geo.vocab > kTopkMaxN)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE,
                "predictor_set_sampling: stride >= 1, 1 <= top_k <= 64, vocab <= 4096");
  p->draws = draws;
  p->draw_stride = stride;
  p->top_k = top_k;
  p->temperature = temperature > 0.f ? temperature : 1.f;
  return TTS_OK;
}

tts_status tts_predictor_destroy(tts_predictor* p) {
  if (!p) return TTS_OK;
  DeviceGuard g(p->s->ctx->device);
  cudaFree(p->resize2);
  cudaFree(p->x16);
  cudaFree(p->table2);
  cudaFree(p->pos2);
  cudaFree(p->step_codes);
  cudaFree(p->logits);
  delete p;
  return TTS_OK;
}

// Predictor::frame_batch with greedy picks (talker.rs:407-468) and gather_sum (:528-550).
static bool text_feed(const tts_text_feed* t, int embed_dim, TextFeed* out) {
  *out = TextFeed{};
  if (!t) return true;
  if (!t->pad || (t->len > 0 && !t->rows) || t->len < 0 || (t->len > 0 && !t->frames))
    return false;
  out->rows = t->rows;
  out->len = t->len;
  out->pad = t->pad;
  out->frames = t->frames;
  (void)embed_dim;
  return true;
}

static tts_status frame_impl(tts_predictor* p, const tts_decode_state* st, const float* hidden,
                             const float* code0, const tts_text_feed* text, unsigned int* codes,
                             float* sum, cudaStream_t cs) {
  tts_stack* s = p->s;
  const tts_stack_geometry& gm = s->geo;
  const tts_predictor_weights& w = p->w;
  if (!st || !st->positions || !st->block_table || !st->k_pages || !st->v_pages)
    return fail(TTS_ERR_INVALID_ARG, "predictor_frame: state pointers are NULL");
  if (!hidden || !code0 || !codes || !sum)
    return fail(TTS_ERR_INVALID_ARG, "predictor_frame: hidden, code0_embed, codes and sum are required");
  const int B = st->lanes;
  if (B < 1 || B > p->max_lanes)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "predictor_frame: lanes must be in 1..max_lanes / 2");
  if (st->max_blocks < 1 || st->max_blocks > kPredictorMaxBlocks ||
      long(st->max_blocks) * st->block_size < w.steps + 1 || st->max_span < w.steps + 1)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE,
                "predictor_frame: pages for steps + 1 positions (max_blocks <= 64), "
                "max_span >= steps + 1");
  if (!aligned16(hidden) || !aligned16(code0) || !aligned16(sum))
    return fail(TTS_ERR_INVALID_ARG, "predictor_frame: hidden, code0_embed, sum 16-byte aligned");
  TextFeed tf;
  if (!text_feed(text, w.embed_dim, &tf))
    return fail(TTS_ERR_INVALID_ARG,
                "predictor_frame: a text feed needs pad, and rows and frames when len > 0");
  const int D = gm.dim, E = w.embed_dim, V = gm.vocab, stride = 2 * p->max_lanes;
  tts_status rc;
#define TTS_TRY(expr, op)                     \
  do {                                        \
    if ((rc = counted((expr), op)) != TTS_OK) \
      return rc;                              \
  } while (0)
  TTS_TRY(launch_predictor_prefill(hidden, code0, B, E, p->x16, w.resize_bias, D, s->h,
                                   st->block_table, st->max_blocks, p->table2, p->pos2,
                                   st->positions, cs),
          "predictor_prefill");
  GemmRequest rz;
  rz.w = p->resize2;
  rz.packed = true;
  rz.x = p->x16;
  rz.m = 2 * B;
  rz.k = 2 * E;
  rz.n = D;
  rz.epi = EPI_RESIDUAL;
  rz.y = s->h;  // the stack's residual stream: the first depth step starts from it
  TTS_TRY(launch_gemm(rz, s->ctx->gemm, cs, s->ctx->device), "proj");
  tts_decode_state pre = *st;
  pre.lanes = 2 * B;
  pre.positions = p->pos2;
  pre.block_table = p->table2;
  pre.max_span = 2;
  for (int i = 0; i < w.steps; ++i) {
    HeadSel hs;
    hs.heads = static_cast<const __half*>(w.heads) + size_t(i) * V * D;
    // the last pick feeds nothing (talker.rs:455: no stack step after the last head)
    hs.embed32 = i + 1 < w.steps ? w.resized + size_t(i) * V * D : nullptr;
    hs.in_h = true;
    hs.feed_h = true;
    if (p->draws) {
      if (B > p->draw_stride)
        return fail(TTS_ERR_UNSUPPORTED_SHAPE, "predictor_frame: more lanes than the draws hold");
      hs.draws = p->draws + size_t(i) * p->draw_stride;
      hs.draw_rows = B;
      hs.top_k = p->top_k;
      hs.temperature = p->temperature;
      hs.logits = p->logits;
    }
    rc = step_impl(s, i == 0 ? &pre : st, nullptr, nullptr, nullptr,
                   p->step_codes + size_t(i) * stride, cs, &hs);
    if (rc != TTS_OK) return rc;
  }
  TTS_TRY(launch_predictor_finish(p->step_codes, stride, B, w.steps,
                                  static_cast<const __half*>(w.tables), V, E, code0, codes, sum,
                                  tf, cs),
          "predictor_finish");
#undef TTS_TRY
  return TTS_OK;
}

tts_status tts_predictor_frame(tts_predictor* p, const tts_decode_state* st, const float* hidden,
                               const float* code0_embed, const tts_text_feed* text,
                               unsigned int* codes, float* sum, void* stream) {
  if (!p) return fail(TTS_ERR_INVALID_ARG, "predictor_frame: predictor is NULL");
  DeviceGuard g(p->s->ctx->device);
  return frame_impl(p, st, hidden, code0_embed, text, codes, sum, S(stream));
}

tts_status tts_predictor_graph_capture(tts_predictor* p, const tts_decode_state* st,
                                       const float* hidden, const float* code0_embed,
                                       const tts_text_feed* text, unsigned int* codes,
                                       float* sum, void* stream, tts_graph** out) {
  if (!p || !out) return fail(TTS_ERR_INVALID_ARG, "graph_capture: NULL argument");
  if (!stream) return fail(TTS_ERR_INVALID_ARG, "graph_capture: needs a non-legacy stream");
  DeviceGuard g(p->s->ctx->device);
  return capture_graph(S(stream), out, [&](cudaStream_t cs) {
    return frame_impl(p, st, hidden, code0_embed, text, codes, sum, cs);
  });
}

// ---------------------------------------------------------------- the talker's frame

// Talker::generate_batch's loop body with greedy picks (talker.rs:953-1057): the talker step
// (head, pick rule, code 0's codec_embed row into the feedback buffer), then the predictor on
// the step's hidden state and that row; the predictor's sum plus the text row replaces the row
// in the feedback buffer, the next step's input.
static tts_status talker_frame_impl(tts_stack* t, const tts_decode_state* tst, tts_predictor* p,
                                    const tts_decode_state* pst, const tts_text_feed* text,
                                    float* hidden, unsigned int* code0, unsigned int* codes,
                                    cudaStream_t cs) {
  if (!t || !tst || !p || !pst || !hidden || !code0 || !codes)
    return fail(TTS_ERR_INVALID_ARG, "talker_frame: NULL argument");
  if (t->geo.codebooks != 1 || !t->heads || !t->embed || !t->feedback)
    return fail(TTS_ERR_INVALID_ARG,
                "talker_frame: the talker needs one codebook head, its embedding table and a "
                "feedback buffer");
  if (t->geo.dim != p->w.embed_dim)
    return fail(TTS_ERR_UNSUPPORTED_SHAPE, "talker_frame: talker dim != predictor embed_dim");
  if (pst->lanes != tst->lanes)
    return fail(TTS_ERR_INVALID_ARG, "talker_frame: talker and predictor lane counts differ");
  tts_status rc = step_impl(t, tst, nullptr, hidden, nullptr, code0, cs);
  if (rc != TTS_OK) return rc;
  return frame_impl(p, pst, hidden, t->feedback, text, codes, t->feedback, cs);
}

tts_status tts_talker_frame(tts_stack* talker, const tts_decode_state* talker_st,
                            tts_predictor* p, const tts_decode_state* pred_st,
                            const tts_text_feed* text, float* hidden, unsigned int* code0,
                            unsigned int* codes, void* stream) {
  if (!talker) return fail(TTS_ERR_INVALID_ARG, "talker_frame: talker is NULL");
  DeviceGuard g(talker->ctx->device);
  return talker_frame_impl(talker, talker_st, p, pred_st, text, hidden, code0, codes, S(stream));
}

tts_status tts_talker_frame_capture(tts_stack* talker, const tts_decode_state* talker_st,
                                    tts_predictor* p, const tts_decode_state* pred_st,
                                    const tts_text_feed* text, float* hidden,
                                    unsigned int* code0, unsigned int* codes, void* stream,
                                    tts_graph** out) {
  if (!talker || !out) return fail(TTS_ERR_INVALID_ARG, "graph_capture: NULL argument");
  if (!stream) return fail(TTS_ERR_INVALID_ARG, "graph_capture: needs a non-legacy stream");
  DeviceGuard g(talker->ctx->device);
  return capture_graph(S(stream), out, [&](cudaStream_t cs) {
    return talker_frame_impl(talker, talker_st, p, pred_st, text, hidden, code0, codes, cs);
  });
}

}  // extern "C"
