// Top-k sampling on the device (crates/tts-nn/src/topk.rs:98-107; the host sampler it must
// agree with is sample_with_u at top_p = 1 and no penalty, crates/qwen3tts/src/talker.rs:
// 189-236): per row the k best logits (value descending, index ascending on ties), their
// probabilities exp((v - max) / t) normalised by their sum, then the caller's draw u in [0, 1)
// scaled by the renormalised mass and walked down the k candidates in order.
//
// One CTA per row. The k-th best value is found by a radix select over the rows' order keys
// (four 8-bit passes of a shared-memory histogram), the k winners are gathered (ties at the
// threshold by lowest index, through an ordered prefix over the row), ranked, and one thread
// walks the probabilities in the reference's order. Optionally, as the code gather of a decode
// step, the pick's embedding row becomes the next input and the lane's position advances.
#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

namespace {

constexpr int kThreads = 256;
constexpr int kPer = kTopkMaxN / kThreads;  // row elements per thread (contiguous run)

struct SampleArgs {
  const float* logits;  // [rows][ldl]
  int n, ldl;
  const float* draws;   // [draw_rows], row r takes draws[r % draw_rows]
  int draw_rows;
  int k;
  float temp;
  uint32_t* codes;      // [rows] (stride code_stride)
  int code_stride;
  const float* embed32;  // optional next input: embed32[code] row of dim
  float* x_next;
  int dim;
  int* positions;        // optional: +1 per row
};

__global__ void __launch_bounds__(kThreads) topk_sample_kernel(const SampleArgs a) {
  __shared__ uint32_t keys[kTopkMaxN];
  __shared__ uint32_t hist[256];
  __shared__ uint32_t scan[kThreads];
  __shared__ uint32_t sel_key[kTopkMaxK];
  __shared__ uint32_t sel_idx[kTopkMaxK];
  __shared__ uint32_t ranked_idx[kTopkMaxK];
  __shared__ float ranked_val[kTopkMaxK];
  __shared__ uint32_t s_prefix, s_need, s_count;
  __shared__ int s_pick;
  pdl_launch_dependents();
  pdl_wait();
  const int row = blockIdx.x, t = threadIdx.x;
  const float* x = a.logits + (size_t)row * a.ldl;
  for (int i = t; i < a.n; i += kThreads) keys[i] = float_order_key(x[i]);
  if (t == 0) {
    s_prefix = 0;
    s_need = uint32_t(a.k);
    s_count = 0;
  }
  __syncthreads();
  // ---- radix select of the k-th largest key, most significant byte first
  uint32_t mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    hist[t] = 0;  // 256 threads, 256 bins
    __syncthreads();
    const uint32_t prefix = s_prefix;
    for (int i = t; i < a.n; i += kThreads) {
      const uint32_t kv = keys[i];
      if ((kv & mask) == prefix) atomicAdd(&hist[(kv >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (t == 0) {
      uint32_t need = s_need, cum = 0;
      int b = 255;
      for (; b > 0; --b) {
        if (cum + hist[b] >= need) break;
        cum += hist[b];
      }
      s_need = need - cum;  // still needed from bin b (the bins above are all in)
      s_prefix = prefix | (uint32_t(b) << shift);
    }
    mask |= 255u << shift;
    __syncthreads();
  }
  const uint32_t thr = s_prefix;  // the k-th largest key
  const uint32_t take_eq = s_need;  // how many keys equal to it, lowest indices first
  // ---- gather: keys above the threshold in any order, equal keys in index order
  const int i0 = t * kPer;
  uint32_t eq = 0;
  for (int u = 0; u < kPer; ++u) {
    const int i = i0 + u;
    if (i < a.n && keys[i] == thr) ++eq;
  }
  scan[t] = eq;
  __syncthreads();
  for (int off = 1; off < kThreads; off <<= 1) {  // inclusive scan of the equal counts
    const uint32_t v = t >= off ? scan[t - off] : 0u;
    __syncthreads();
    scan[t] += v;
    __syncthreads();
  }
  uint32_t before = scan[t] - eq;
  for (int u = 0; u < kPer; ++u) {
    const int i = i0 + u;
    if (i >= a.n) break;
    const uint32_t kv = keys[i];
    bool take = kv > thr;
    if (kv == thr) take = before++ < take_eq;
    if (take) {
      const uint32_t slot = atomicAdd(&s_count, 1u);
      if (slot < uint32_t(kTopkMaxK)) {
        sel_key[slot] = kv;
        sel_idx[slot] = uint32_t(i);
      }
    }
  }
  __syncthreads();
  // ---- rank the k winners: value descending, index ascending
  if (t < a.k) {
    const uint32_t kv = sel_key[t], id = sel_idx[t];
    int rank = 0;
    for (int j = 0; j < a.k; ++j) {
      const uint32_t ok = sel_key[j], oi = sel_idx[j];
      rank += (ok > kv || (ok == kv && oi < id)) ? 1 : 0;
    }
    ranked_idx[rank] = id;
    ranked_val[rank] = x[id];
  }
  __syncthreads();
  // ---- probabilities and the walk, in the host sampler's order
  if (t == 0) {
    float p[kTopkMaxK];
    const float mx = ranked_val[0];
    float total = 0.f;
    for (int j = 0; j < a.k; ++j) {
      p[j] = expf(__fdiv_rn(ranked_val[j] - mx, a.temp));
      total += p[j];
    }
    float renorm = 0.f;
    for (int j = 0; j < a.k; ++j) {
      p[j] = __fdiv_rn(p[j], total);
      renorm += p[j];
    }
    float u = a.draws[row % a.draw_rows] * renorm;
    int pick = int(ranked_idx[a.k - 1]);
    for (int j = 0; j < a.k; ++j) {
      u -= p[j];
      if (u <= 0.f) {
        pick = int(ranked_idx[j]);
        break;
      }
    }
    s_pick = pick;
    a.codes[(size_t)row * a.code_stride] = uint32_t(pick);
    if (a.positions) a.positions[row] += 1;
  }
  __syncthreads();
  if (a.embed32 && a.x_next) {
    const float* src = a.embed32 + (size_t)s_pick * a.dim;
    for (int d = t * 2; d < a.dim; d += kThreads * 2)
      *reinterpret_cast<float2*>(a.x_next + (size_t)row * a.dim + d) =
          *reinterpret_cast<const float2*>(src + d);
  }
}

}  // namespace

cudaError_t launch_topk_sample(const float* logits, int rows, int n, int ldl, const float* draws,
                               int draw_rows, int k, float temperature, uint32_t* codes,
                               int code_stride, const float* embed32, float* x_next, int dim,
                               int* positions, bool pdl, cudaStream_t st) {
  if (rows < 1 || n < 1 || n > kTopkMaxN || k < 1 || k > kTopkMaxK || k > n ||
      draw_rows < 1 || (embed32 && dim % 2)) {
    set_error("topk_sample: 1 <= k <= min(n, 64), n <= 4096");
    return cudaErrorInvalidValue;
  }
  SampleArgs a{};
  a.logits = logits;
  a.n = n;
  a.ldl = ldl;
  a.draws = draws;
  a.draw_rows = draw_rows;
  a.k = k;
  a.temp = temperature > 0.f ? temperature : 1.f;
  a.codes = codes;
  a.code_stride = code_stride;
  a.embed32 = embed32;
  a.x_next = x_next;
  a.dim = dim;
  a.positions = positions;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(rows, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, topk_sample_kernel, a);
}

}  // namespace tts
