// The codec decoder's front (crates/qwen3tts/src/codec.rs:161-196, 261-317, 403-424): the
// small row-wise kernels its RVQ dequantiser, pre-transformer and ConvNeXt upsamplers need
// besides the projections and convolutions (gemm_decode.cu, conv_nlc.cu). Each is one coalesced
// pass (or one warp per row) over activations that stay in HBM/L2 between launches.
#include <cstdlib>
#include <mutex>

#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

namespace {

int blocks_for(long n, int per) {
  long g = (n + per - 1) / per;
  if (g > 148L * 32) g = 148L * 32;
  return int(g < 1 ? 1 : g);
}

// Rvq::decode's lookups (codec.rs:285-299): out[t] = sum over codebooks q in [q0, q0 + nq) of
// table[q][codes[t][q]] (f32 rows of `dim`), in codebook order.
__global__ void rvq_gather_kernel(const uint32_t* codes, int ncodes, int q0, int nq,
                                  const float* tables, int entries, int dim, float* out, int T) {
  const int t = blockIdx.x;
  if (t >= T) return;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    float s = 0.f;
    for (int q = 0; q < nq; ++q) {
      uint32_t c = codes[(size_t)t * ncodes + q0 + q];
      if (c >= uint32_t(entries)) c = 0;
      s += tables[((size_t)q * entries + c) * dim + d];
    }
    out[(size_t)t * dim + d] = s;
  }
}

// candle_nn::rotary_emb::rope (half-split rotate_half) in place on `heads` heads of width hd
// starting at column col0 of each row of x [T][ld]; row t rotates by position pos0 + t.
__global__ void rope_rows_kernel(float* x, int T, int ld, int col0, int heads, int hd,
                                 const float* cos_t, const float* sin_t, int pos0) {
  const int half = hd / 2;
  const long total = (long)T * heads * half;
  for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total;
       e += (long)gridDim.x * blockDim.x) {
    const int i = int(e % half);
    const long th = e / half;
    const int h = int(th % heads), t = int(th / heads);
    float* v = x + (size_t)t * ld + col0 + (size_t)h * hd;
    const float c = cos_t[(size_t)(pos0 + t) * half + i], s = sin_t[(size_t)(pos0 + t) * half + i];
    const float a = v[i], b = v[i + half];
    v[i] = a * c - b * s;
    v[i + half] = b * c + a * s;
  }
}

// Causal windowed self-attention over one sequence (the prefill branch of Stack::forward with
// causal_window_mask, qwen3.rs:409-444; lib.rs:1210-1225): row t of head h attends to rows
// [t + 1 - window, t] (all of [0, t] without a window), scores q.k * scale, softmax, sum p v.
// q, k, v are column blocks of qkv [T][ld] (q at 0, k at heads*hd, v at 2*heads*hd; gqa 1).
// One warp per (row, head): keys across the lanes (up to 32 per pass), hd <= 128.
__global__ void window_attn_kernel(const float* qkv, int T, int ld, int heads, int hd,
                                   int window, float scale, void* out, int out_f16) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T * heads) return;
  const int t = warp / heads, h = warp % heads;
  const int lo = window > 0 ? max(0, t + 1 - window) : 0;
  const float* q = qkv + (size_t)t * ld + (size_t)h * hd;
  const int kcol = heads * hd + h * hd, vcol = 2 * heads * hd + h * hd;
  // scores, a key per lane per pass; the running max and sum online over the passes
  float m = -INFINITY, l = 0.f;
  float o[4] = {0.f, 0.f, 0.f, 0.f};  // dims lane, lane + 32, lane + 64, lane + 96
  for (int j0 = lo; j0 <= t; j0 += 32) {
    const int j = j0 + lane;
    float s = -INFINITY;
    if (j <= t) {
      const float* kr = qkv + (size_t)j * ld + kcol;
      float acc = 0.f;
      for (int d = 0; d < hd; ++d) acc += q[d] * kr[d];
      s = acc * scale;
    }
    const float pm = warp_max(s);
    const float mn = fmaxf(m, pm);
    const float corr = m == -INFINITY ? 0.f : expf(m - mn);
    const float p = j <= t ? expf(s - mn) : 0.f;
    l = l * corr + warp_sum(p);
#pragma unroll
    for (int u = 0; u < 4; ++u) o[u] *= corr;
    const int nk = min(32, t + 1 - j0);
    for (int i = 0; i < nk; ++i) {
      const float pi = __shfl_sync(0xffffffffu, p, i);
      const float* vr = qkv + (size_t)(j0 + i) * ld + vcol;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (lane + 32 * u < hd) o[u] += pi * vr[lane + 32 * u];
    }
    m = mn;
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int d = lane + 32 * u;
    if (d >= hd) break;
    const float r = o[u] / l;
    const size_t oi = (size_t)t * heads * hd + (size_t)h * hd + d;
    if (out_f16)
      static_cast<__half*>(out)[oi] = __float2half_rn(r);
    else
      static_cast<float*>(out)[oi] = r;
  }
}

// The same attention for a window > 0, by tiles: one CTA per (block of 32 query rows, head)
// stages the block's q rows and the K and V rows its windows reach ([t0 + 1 - window, t0 + 31])
// in shared memory (K and V rows padded to hd + 1 floats, so the lanes of a warp, one key each,
// read different banks), then a warp per query row runs window_attn_kernel's arithmetic in
// its order (each score a sequential dot product, the softmax online per pass of 32 keys, the
// values summed key by key): the same results, from shared memory instead of every lane
// reading its own key row from global memory.
constexpr int kWinRows = 32;  // query rows per CTA
__global__ void __launch_bounds__(256) window_attn_tiled_kernel(const float* qkv, int T, int ld,
                                                                int heads, int hd, int window,
                                                                float scale, void* out,
                                                                int out_f16) {
  extern __shared__ float wsm[];
  const int h = blockIdx.y;
  const int t0 = blockIdx.x * kWinRows;
  const int t1 = min(T, t0 + kWinRows);  // query rows [t0, t1)
  const int k0 = max(0, t0 + 1 - window);  // key rows [k0, t1)
  const int nk_rows = t1 - k0;
  const int pitch = hd + 1;
  float* qs = wsm;                          // [kWinRows][hd]
  float* ks = qs + kWinRows * hd;           // [nk_rows][pitch]
  float* vs = ks + (kWinRows + window - 1) * pitch;
  const int kcol = heads * hd + h * hd, vcol = 2 * heads * hd + h * hd;
  for (int i = threadIdx.x; i < (t1 - t0) * hd; i += blockDim.x) {
    const int r = i / hd, d = i % hd;
    qs[r * hd + d] = qkv[(size_t)(t0 + r) * ld + (size_t)h * hd + d];
  }
  for (int i = threadIdx.x; i < nk_rows * hd; i += blockDim.x) {
    const int r = i / hd, d = i % hd;
    const float* row = qkv + (size_t)(k0 + r) * ld;
    ks[r * pitch + d] = row[kcol + d];
    vs[r * pitch + d] = row[vcol + d];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = t0 + warp; t < t1; t += blockDim.x >> 5) {
    const int lo = max(0, t + 1 - window);
    const float* q = qs + (t - t0) * hd;
    float m = -INFINITY, l = 0.f;
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j0 = lo; j0 <= t; j0 += 32) {
      const int j = j0 + lane;
      float s = -INFINITY;
      if (j <= t) {
        const float* kr = ks + (j - k0) * pitch;
        float acc = 0.f;
        for (int d = 0; d < hd; ++d) acc += q[d] * kr[d];
        s = acc * scale;
      }
      const float pm = warp_max(s);
      const float mn = fmaxf(m, pm);
      const float corr = m == -INFINITY ? 0.f : expf(m - mn);
      const float p = j <= t ? expf(s - mn) : 0.f;
      l = l * corr + warp_sum(p);
#pragma unroll
      for (int u = 0; u < 4; ++u) o[u] *= corr;
      const int nk = min(32, t + 1 - j0);
      for (int i = 0; i < nk; ++i) {
        const float pi = __shfl_sync(0xffffffffu, p, i);
        const float* vr = vs + (j0 + i - k0) * pitch;
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (lane + 32 * u < hd) o[u] += pi * vr[lane + 32 * u];
      }
      m = mn;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int d = lane + 32 * u;
      if (d >= hd) break;
      const float r = o[u] / l;
      const size_t oi = (size_t)t * heads * hd + (size_t)h * hd + d;
      if (out_f16)
        static_cast<__half*>(out)[oi] = __float2half_rn(r);
      else
        static_cast<float*>(out)[oi] = r;
    }
  }
}

// LayerNorm over the last dim (lib.rs:1006-1035: mean, centred variance, then the affine), one
// CTA per row, f32 math; y f32 or f16.
__global__ void __launch_bounds__(256) layer_norm_kernel(const float* x, const float* w,
                                                         const float* b, int dim, float eps,
                                                         void* y, int y_f16) {
  __shared__ float red[8];
  const int row = blockIdx.x;
  const float* xr = x + (size_t)row * dim;
  auto block_sum = [&](float v) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    if (threadIdx.x < 32) s = warp_sum(s);
    __syncthreads();
    if (threadIdx.x == 0) red[0] = s;
    __syncthreads();
    const float r = red[0];
    __syncthreads();
    return r;
  };
  float s = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) s += xr[i];
  const float mean = block_sum(s) / float(dim);
  float v = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float c = xr[i] - mean;
    v += c * c;
  }
  const float var = block_sum(v) / float(dim);
  const float inv = sqrtf(var + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float o = (xr[i] - mean) / inv * w[i] + (b ? b[i] : 0.f);
    if (y_f16)
      static_cast<__half*>(y)[(size_t)row * dim + i] = __float2half_rn(o);
    else
      static_cast<float*>(y)[(size_t)row * dim + i] = o;
  }
}

// nlc::depthwise (nlc.rs:232-256): causal per-channel conv over [b][L][C] with taps w [C][k]
// summed in tap order, plus bias; f32 in and out.
__global__ void depthwise_kernel(const float* x, const float* w, const float* bias, int b, int L,
                                 int C, int k, float* y) {
  const long total = (long)b * L * C;
  for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total;
       e += (long)gridDim.x * blockDim.x) {
    const int c = int(e % C);
    const long bl = e / C;
    const int l = int(bl % L);
    const long base = (bl - l) * C;  // row 0 of this batch item
    float acc = 0.f;
    for (int tp = 0; tp < k; ++tp) {
      const int src = l + tp - (k - 1);
      const float xv = src >= 0 ? x[base + (size_t)src * C + c] : 0.f;
      const float term = xv * w[(size_t)c * k + tp];
      acc = tp == 0 ? term : acc + term;
    }
    y[e] = bias ? acc + bias[c] : acc;
  }
}

// Row epilogue for projections computed in f32: z = act(y + bias); out = res + scale * z (res
// and scale optional), f32 or f16 out. act 1 is GELU with the exact erf (lib.rs:1129), act 2
// SiLU (the text projection's, talker.rs:607-616).
__global__ void bias_act_kernel(const float* y, int rows, int n, const float* bias, int act,
                                const float* scale, const float* res, void* out, int out_f16) {
  const long total = (long)rows * n;
  for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total;
       e += (long)gridDim.x * blockDim.x) {
    const int c = int(e % n);
    float z = y[e] + (bias ? bias[c] : 0.f);
    if (act == 1) z = 0.5f * z * (1.f + erff(z * 0.70710678118654752f));
    else if (act == 2) z = z / (1.f + expf(-z));  // silu, candle_nn::ops::silu
    if (scale) z = scale[c] * z;
    if (res) z = res[e] + z;
    if (out_f16)
      static_cast<__half*>(out)[e] = __float2half_rn(z);
    else
      static_cast<float*>(out)[e] = z;
  }
}

}  // namespace

cudaError_t launch_rvq_gather(const uint32_t* codes, int ncodes, int q0, int nq,
                              const float* tables, int entries, int dim, float* out, int T,
                              cudaStream_t st) {
  rvq_gather_kernel<<<T, 256, 0, st>>>(codes, ncodes, q0, nq, tables, entries, dim, out, T);
  return cudaGetLastError();
}

cudaError_t launch_rope_rows(float* x, int T, int ld, int col0, int heads, int hd,
                             const float* cos_t, const float* sin_t, int pos0, cudaStream_t st) {
  rope_rows_kernel<<<blocks_for((long)T * heads * hd / 2, 256), 256, 0, st>>>(
      x, T, ld, col0, heads, hd, cos_t, sin_t, pos0);
  return cudaGetLastError();
}

cudaError_t launch_window_attn(const float* qkv, int T, int ld, int heads, int hd, int window,
                               float scale, void* out, bool out_f16, cudaStream_t st) {
  if (hd > 128 || hd < 1) {
    set_error("window_attention: head_dim must be in 1..128");
    return cudaErrorInvalidValue;
  }
  // the tiled form where the window's rows fit in shared memory (TTS_WINDOW_TILED=0: the
  // per-row form, A/B measurement)
  const char* tv = getenv("TTS_WINDOW_TILED");
  const size_t smem = (size_t(kWinRows) * hd + size_t(2) * (kWinRows + window - 1) * (hd + 1)) *
                      sizeof(float);
  if (!(tv && *tv == '0') && window > 0 && smem <= 200 * 1024) {
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    {
      std::lock_guard<std::mutex> lock(mu);
      if (dev >= 0 && dev < 64 && !done[dev]) {
        cudaFuncSetAttribute(window_attn_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             200 * 1024);
        done[dev] = true;
      }
    }
    const dim3 grid((T + kWinRows - 1) / kWinRows, heads);
    window_attn_tiled_kernel<<<grid, 256, smem, st>>>(qkv, T, ld, heads, hd, window, scale, out,
                                                      out_f16 ? 1 : 0);
    return cudaGetLastError();
  }
  const long warps = (long)T * heads;
  window_attn_kernel<<<int((warps + 7) / 8), 256, 0, st>>>(qkv, T, ld, heads, hd, window, scale,
                                                           out, out_f16 ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_layer_norm(const float* x, const float* w, const float* b, int rows, int dim,
                              float eps, void* y, bool y_f16, cudaStream_t st) {
  layer_norm_kernel<<<rows, 256, 0, st>>>(x, w, b, dim, eps, y, y_f16 ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_depthwise(const float* x, const float* w, const float* bias, int b, int L,
                             int C, int k, float* y, cudaStream_t st) {
  depthwise_kernel<<<blocks_for((long)b * L * C, 256), 256, 0, st>>>(x, w, bias, b, L, C, k, y);
  return cudaGetLastError();
}

cudaError_t launch_bias_act(const float* y, int rows, int n, const float* bias, int act,
                            const float* scale, const float* res, void* out, bool out_f16,
                            cudaStream_t st) {
  bias_act_kernel<<<blocks_for((long)rows * n, 256), 256, 0, st>>>(y, rows, n, bias, act, scale,
                                                                  res, out, out_f16 ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace tts
