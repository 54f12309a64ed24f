// The depth predictor's two frame-boundary kernels (crates/qwen3tts/src/talker.rs:407-550).
// The 15 depth steps in between are decoder-stack steps (runtime.cu) on the same kernels as the
// talker's, at the predictor's width.
#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

namespace {

cudaError_t launch_pdl(void (*kernel)(void*), dim3 grid, dim3 block, cudaStream_t st,
                       void** args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(kernel), args);
}

// The frame's prefill (talker.rs:416-420: cat([hidden, code0_embed]) -> resize -> stack over
// both positions) as one stack step over 2 * lanes rows: row r < lanes is lane r's second
// position (code0_embed), row lanes + r its first (hidden). Both rows of a lane share the lane's
// pages (table2), at positions 1 and 0, so the position-1 row's attention sees both keys.
//
// The projection takes its f32 inputs exactly: each input x becomes f16 hi = rn(x) and f16
// lo = rn(x - hi), laid side by side ([hi | lo], width 2 * embed_dim) against the doubled weight
// [W | W], so W.x = W.hi + W.lo up to f32 accumulation, as the reference's f32 Linear. x0 gets
// the bias rows the residual epilogue accumulates onto.
__global__ void __launch_bounds__(256) predictor_prefill_kernel(
    const float* hidden, const float* code0, int lanes, int embed_dim, __half* x16,
    const float* bias, int dim, float* x0, const int* table, int max_blocks, int* table2,
    int* pos2, int* positions) {
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x;
  const int lane = r < lanes ? r : r - lanes;
  const float* src = (r < lanes ? code0 : hidden) + (size_t)lane * embed_dim;
  __half* hi = x16 + (size_t)r * 2 * embed_dim;
  __half* lo = hi + embed_dim;
  for (int e = threadIdx.x * 2; e < embed_dim; e += blockDim.x * 2) {
    const float2 v = *reinterpret_cast<const float2*>(src + e);
    const __half h0 = __float2half_rn(v.x), h1 = __float2half_rn(v.y);
    const __half l0 = __float2half_rn(v.x - __half2float(h0));
    const __half l1 = __float2half_rn(v.y - __half2float(h1));
    *reinterpret_cast<__half2*>(hi + e) = __halves2half2(h0, h1);
    *reinterpret_cast<__half2*>(lo + e) = __halves2half2(l0, l1);
  }
  for (int d = threadIdx.x; d < dim; d += blockDim.x)
    x0[(size_t)r * dim + d] = bias ? bias[d] : 0.f;
  for (int j = threadIdx.x; j < max_blocks; j += blockDim.x)
    table2[(size_t)r * max_blocks + j] = table[(size_t)lane * max_blocks + j];
  if (threadIdx.x == 0) {
    pos2[r] = r < lanes ? 1 : 0;
    // the lanes' own positions resume after the two prefilled ones
    if (r < lanes) positions[r] = 2;
  }
}

// Frame end (talker.rs:466-467, 528-550): the per-step codes transposed to [lane][step], and
// sum = code0_embed + sum over steps of tables[step][code] at talker width, the table rows summed
// in f32 in step order first, as gather_sum's sum_keepdim, then added to code0_embed.
// With a text feed the lane's text row (its trailing text while rows remain, then the pad
// row) is added last, as the talker adds it to the predictor's sum (talker.rs:1043-1050).
__global__ void __launch_bounds__(256) predictor_finish_kernel(
    const uint32_t* step_codes, int stride, int steps, const __half* tables, int vocab,
    int embed_dim, const float* code0, uint32_t* codes, float* sum, TextFeed text) {
  __shared__ int sc[64];
  pdl_launch_dependents();
  pdl_wait();
  const int lane = blockIdx.x;
  const float* trow = nullptr;
  if (text.pad) {
    const int t = text.frames ? text.frames[lane] - 1 : 0;
    trow = t >= 0 && t < text.len ? text.rows + ((size_t)lane * text.len + t) * embed_dim
                                  : text.pad;
  }
  if (threadIdx.x < steps) {
    const uint32_t c = step_codes[(size_t)threadIdx.x * stride + lane];
    codes[(size_t)lane * steps + threadIdx.x] = c;
    sc[threadIdx.x] = int(c < uint32_t(vocab) ? c : 0);
  }
  __syncthreads();
  for (int e = threadIdx.x * 2; e < embed_dim; e += blockDim.x * 2) {
    float s0 = 0.f, s1 = 0.f;
    for (int q = 0; q < steps; ++q) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(
          tables + (((size_t)q * vocab + sc[q]) * embed_dim + e)));
      s0 += f.x;
      s1 += f.y;
    }
    const float2 c0 = *reinterpret_cast<const float2*>(code0 + (size_t)lane * embed_dim + e);
    float2 r = make_float2(c0.x + s0, c0.y + s1);
    if (trow) {
      const float2 tx = *reinterpret_cast<const float2*>(trow + e);
      r.x += tx.x;
      r.y += tx.y;
    }
    // in place over code0 is allowed: this thread read the element it overwrites
    sum[(size_t)lane * embed_dim + e] = r.x;
    sum[(size_t)lane * embed_dim + e + 1] = r.y;
  }
}

}  // namespace

cudaError_t launch_predictor_prefill(const float* hidden, const float* code0, int lanes,
                                     int embed_dim, __half* x16, const float* bias, int dim,
                                     float* x0, const int* table, int max_blocks, int* table2,
                                     int* pos2, int* positions, cudaStream_t st) {
  if (lanes < 1 || embed_dim % 2 || max_blocks < 1) {
    set_error("predictor_prefill: lanes >= 1, even embed_dim, max_blocks >= 1");
    return cudaErrorInvalidValue;
  }
  void* args[] = {(void*)&hidden, (void*)&code0,  (void*)&lanes,      (void*)&embed_dim,
                  (void*)&x16,    (void*)&bias,   (void*)&dim,        (void*)&x0,
                  (void*)&table,  (void*)&max_blocks, (void*)&table2, (void*)&pos2,
                  (void*)&positions};
  return launch_pdl(reinterpret_cast<void (*)(void*)>(predictor_prefill_kernel),
                    dim3(2 * lanes), dim3(256), st, args);
}

cudaError_t launch_predictor_finish(const uint32_t* step_codes, int stride, int lanes, int steps,
                                    const __half* tables, int vocab, int embed_dim,
                                    const float* code0, uint32_t* codes, float* sum,
                                    const TextFeed& text, cudaStream_t st) {
  if (lanes < 1 || steps < 1 || steps > 64 || embed_dim % 2) {
    set_error("predictor_finish: lanes >= 1, 1..64 steps, even embed_dim");
    return cudaErrorInvalidValue;
  }
  TextFeed tf = text;
  void* args[] = {(void*)&step_codes, (void*)&stride, (void*)&steps, (void*)&tables,
                  (void*)&vocab,      (void*)&embed_dim, (void*)&code0, (void*)&codes,
                  (void*)&sum,        (void*)&tf};
  return launch_pdl(reinterpret_cast<void (*)(void*)>(predictor_finish_kernel), dim3(lanes),
                    dim3(256), st, args);
}

}  // namespace tts
