// Paged decode attention (GQA, head_dim 128, f16 KV pages, f32 math).
//
// The B200 form of tts-nn's `attn::decode_attention` (crates/tts-nn/src/attn.rs:22-73; its
// CPU loops attn.rs:90-126 and 203-238, Metal `decode_attn_f16`): softmax(q . K^T) . V over
// positions [wstart, span) of each lane, with any scale already folded into q. Per-lane spans
// (the reference uses one span for the whole batch) let lanes of different lengths share a
// step, which is what a paged cache is for.
//
// Work unit: one CTA per (chunk of kChunk positions, kv head, lane). Both query heads of a kv
// head are served from one read of each K/V row. Inside a CTA, eight half-warps each take 32
// consecutive positions; each of their 16 lanes owns 8 of the 128 dims (one 16-byte load per
// row). Scores, the running max and the exp-rescaled sums are kept per half-warp, combined
// across half-warps in shared memory, and, when a lane's span needs several chunks, written as
// partials that the last CTA of that (lane, kv head) merges in chunk order (deterministic).
#include <cstdio>
#include <mutex>

#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

namespace {

constexpr int kChunk = 256;  // positions per CTA
constexpr int kHalfWarps = 8;
constexpr int kPerHalf = kChunk / kHalfWarps;  // 32
constexpr int kGroup = 8;                      // rows per inner iteration

struct AttnArgs {
  const float* q;
  const __half* k;
  const __half* v;
  const int* bt;
  int max_blocks, bs, num_blocks;
  int max_span;
  int* err;
  const int* spans;
  int span_add;
  int window;
  int n_kv;
  int max_chunks;
  float* part;  // [lanes][n_kv][max_chunks][GQA][130]: 128 o, m, l
  unsigned* counters;
  void* out;
  int out_f16;
};

__device__ __forceinline__ void load8(const __half* p, float* f) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

template <int GQA>
__global__ void __launch_bounds__(128) attn_decode_kernel(const AttnArgs a) {
  __shared__ float sm_acc[kHalfWarps][GQA][128];
  __shared__ float sm_m[kHalfWarps][GQA];
  __shared__ float sm_l[kHalfWarps][GQA];
  __shared__ int sm_last;

  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  pdl_launch_dependents();
  pdl_wait();

  // Spans and page numbers are device data: clamp to what the grid, the block table and the
  // pool cover, and flag anything outside instead of reading out of bounds.
  int span = a.spans[b] + a.span_add;
  const int lim = min(a.max_blocks * a.bs, a.max_span);
  if (span < 1 || span > lim) {
    if (threadIdx.x == 0 && c == 0 && a.err) atomicOr(a.err, 512);
    span = max(1, min(span, lim));
  }
  const int ws = (a.window > 0 && span > a.window) ? span - a.window : 0;
  const int nch = (span - ws + kChunk - 1) / kChunk;
  if (c >= nch) return;
  const int p0 = ws + c * kChunk;
  const int p1 = min(p0 + kChunk, span);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int hw = warp * 2 + (lane >> 4);
  const int j = lane & 15;
  const int heads = a.n_kv * GQA;

  float qv[GQA][8];
#pragma unroll
  for (int g = 0; g < GQA; ++g) {
    const float4* qp =
        reinterpret_cast<const float4*>(a.q + ((size_t)b * heads + h * GQA + g) * 128 + 8 * j);
    const float4 x0 = qp[0], x1 = qp[1];
    qv[g][0] = x0.x; qv[g][1] = x0.y; qv[g][2] = x0.z; qv[g][3] = x0.w;
    qv[g][4] = x1.x; qv[g][5] = x1.y; qv[g][6] = x1.z; qv[g][7] = x1.w;
  }
  float m[GQA], l[GQA], acc[GQA][8];
#pragma unroll
  for (int g = 0; g < GQA; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int d = 0; d < 8; ++d) acc[g][d] = 0.f;
  }

  const int* bt = a.bt + (size_t)b * a.max_blocks;
  const int q0 = p0 + hw * kPerHalf;
  const int q1 = min(q0 + kPerHalf, p1);
  // The trip count is the same for both half-warps of a warp (their shuffles use the full
  // mask); rows past a half-warp's own range are masked instead.
  for (int it = 0; it < kPerHalf; it += kGroup) {
    const int pg = q0 + it;
    if (__all_sync(0xffffffffu, pg >= q1)) break;
    float kf[kGroup][8], vf[kGroup][8];
#pragma unroll
    for (int u = 0; u < kGroup; ++u) {
      const int p = pg + u;
      const int blk = p < q1 ? bt[p / a.bs] : -1;
      if (blk >= 0 && blk < a.num_blocks) {
        const size_t row = (((size_t)blk * a.n_kv + h) * a.bs + (p % a.bs)) * 128 + 8 * j;
        load8(a.k + row, kf[u]);
        load8(a.v + row, vf[u]);
      } else {
        if (p < q1 && j == 0 && a.err) atomicOr(a.err, 1024);
#pragma unroll
        for (int d = 0; d < 8; ++d) kf[u][d] = vf[u][d] = 0.f;
      }
    }
#pragma unroll
    for (int g = 0; g < GQA; ++g) {
      float s[kGroup];
#pragma unroll
      for (int u = 0; u < kGroup; ++u) {
        float t = 0.f;
#pragma unroll
        for (int d = 0; d < 8; ++d) t += qv[g][d] * kf[u][d];
        t += __shfl_xor_sync(0xffffffffu, t, 8);
        t += __shfl_xor_sync(0xffffffffu, t, 4);
        t += __shfl_xor_sync(0xffffffffu, t, 2);
        t += __shfl_xor_sync(0xffffffffu, t, 1);
        s[u] = (pg + u < q1) ? t : -INFINITY;
      }
      float mx = s[0];
#pragma unroll
      for (int u = 1; u < kGroup; ++u) mx = fmaxf(mx, s[u]);
      const float mn = fmaxf(m[g], mx);
      if (mn != -INFINITY) {
        const float corr = expf(m[g] - mn);
        l[g] *= corr;
#pragma unroll
        for (int d = 0; d < 8; ++d) acc[g][d] *= corr;
#pragma unroll
        for (int u = 0; u < kGroup; ++u) {
          const float p = expf(s[u] - mn);
          l[g] += p;
#pragma unroll
          for (int d = 0; d < 8; ++d) acc[g][d] += p * vf[u][d];
        }
        m[g] = mn;
      }
    }
  }

  // combine the eight half-warps
#pragma unroll
  for (int g = 0; g < GQA; ++g) {
#pragma unroll
    for (int d = 0; d < 8; ++d) sm_acc[hw][g][8 * j + d] = acc[g][d];
    if (j == 0) {
      sm_m[hw][g] = m[g];
      sm_l[hw][g] = l[g];
    }
  }
  __syncthreads();

  constexpr int kDims = 128 * GQA / 128;  // dims per thread: GQA
  const int t = threadIdx.x;
  const int base = (((size_t)b * a.n_kv + h) * a.max_chunks + c) * GQA;
  float o[kDims], M[kDims], L[kDims];
  int gg[kDims], dd[kDims];
#pragma unroll
  for (int e = 0; e < kDims; ++e) {
    const int idx = t + e * 128;  // 0 .. 128*GQA-1
    const int g = idx / 128, d = idx % 128;
    gg[e] = g;
    dd[e] = d;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kHalfWarps; ++w) mm = fmaxf(mm, sm_m[w][g]);
    float ll = 0.f, oo = 0.f;
#pragma unroll
    for (int w = 0; w < kHalfWarps; ++w) {
      if (sm_m[w][g] == -INFINITY) continue;
      const float f = expf(sm_m[w][g] - mm);
      ll += sm_l[w][g] * f;
      oo += sm_acc[w][g][d] * f;
    }
    o[e] = oo;
    M[e] = mm;
    L[e] = ll;
  }

  const size_t out_base = (size_t)b * heads * 128 + (size_t)h * GQA * 128;
  if (nch == 1) {
#pragma unroll
    for (int e = 0; e < kDims; ++e) {
      const float r = o[e] / L[e];
      const size_t oi = out_base + gg[e] * 128 + dd[e];
      if (a.out_f16)
        static_cast<__half*>(a.out)[oi] = __float2half_rn(r);
      else
        static_cast<float*>(a.out)[oi] = r;
    }
    return;
  }

#pragma unroll
  for (int e = 0; e < kDims; ++e) {
    float* pp = a.part + (size_t)(base + gg[e]) * 130;
    pp[dd[e]] = o[e];
    if (dd[e] == 0) {
      pp[128] = M[e];
      pp[129] = L[e];
    }
  }
  __threadfence();
  __syncthreads();
  if (t == 0) {
    const unsigned prev = atomicAdd(&a.counters[b * a.n_kv + h], 1u);
    sm_last = (prev == unsigned(nch - 1));
  }
  __syncthreads();
  if (!sm_last) return;
  __threadfence();
#pragma unroll
  for (int e = 0; e < kDims; ++e) {
    const int g = gg[e], d = dd[e];
    const size_t pb = (((size_t)b * a.n_kv + h) * a.max_chunks) * GQA + g;
    float mm = -INFINITY;
    for (int cc = 0; cc < nch; ++cc) mm = fmaxf(mm, __ldcg(a.part + (pb + (size_t)cc * GQA) * 130 + 128));
    float ll = 0.f, oo = 0.f;
    for (int cc = 0; cc < nch; ++cc) {
      const float* pp = a.part + (pb + (size_t)cc * GQA) * 130;
      const float f = expf(__ldcg(pp + 128) - mm);
      ll += __ldcg(pp + 129) * f;
      oo += __ldcg(pp + d) * f;
    }
    const float r = oo / ll;
    const size_t oi = out_base + g * 128 + d;
    if (a.out_f16)
      static_cast<__half*>(a.out)[oi] = __float2half_rn(r);
    else
      static_cast<float*>(a.out)[oi] = r;
  }
  if (t == 0) a.counters[b * a.n_kv + h] = 0u;
}

}  // namespace

// Scratch for launch_attn_static: the split-KV partials followed by the per-(lane, kv head)
// arrival counters, in one fixed device array so that callers which must not allocate device
// memory can still run the attention. Every GPU that loads the library holds this array until
// the process exits. All calls share it and it keeps the last call's contents, so the counters
// are cleared on every call, and calls that overlap on the GPU (two streams, two threads) race.
constexpr size_t kStaticPartBytes = size_t(4) << 20;  // 4 MiB of partials
constexpr int kStaticCounters = 4096;                  // lanes * n_kv
static __device__ __align__(256) unsigned char g_attn_static_scratch[kStaticPartBytes + kStaticCounters * sizeof(unsigned)];

size_t attn_part_bytes(int lanes, int n_kv, int gqa, int max_span) {
  const int chunks = (max_span + kChunk - 1) / kChunk;
  return size_t(lanes) * n_kv * chunks * gqa * 130 * sizeof(float);
}

cudaError_t launch_attn(const AttnRequest& r, const AttnWorkspace& w, cudaStream_t st) {
  if (r.gqa != 1 && r.gqa != 2) {
    set_error("decode_attention: gqa must be 1 or 2");
    return cudaErrorInvalidValue;
  }
  if (r.lanes < 1 || r.n_kv < 1 || r.max_span < 1 || r.block_size < 1) {
    set_error("decode_attention: empty shape");
    return cudaErrorInvalidValue;
  }
  const int chunks = (r.max_span + kChunk - 1) / kChunk;
  if (attn_part_bytes(r.lanes, r.n_kv, r.gqa, r.max_span) > w.part_bytes ||
      r.lanes * r.n_kv > w.n_counters) {
    set_error("decode_attention: workspace too small");
    return cudaErrorInvalidValue;
  }
  AttnArgs a{};
  a.q = r.q;
  a.k = r.k_pool;
  a.v = r.v_pool;
  a.bt = r.block_table;
  a.max_blocks = r.max_blocks;
  a.bs = r.block_size;
  a.num_blocks = r.num_blocks;
  a.max_span = r.max_span;
  a.err = r.err;
  a.spans = r.spans;
  a.span_add = r.span_add;
  a.window = r.window;
  a.n_kv = r.n_kv;
  a.max_chunks = chunks;
  a.part = w.part;
  a.counters = w.counters;
  a.out = r.out;
  a.out_f16 = r.out_f16 ? 1 : 0;

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(chunks, r.n_kv, r.lanes);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = r.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (r.gqa == 2) return cudaLaunchKernelEx(&cfg, attn_decode_kernel<2>, a);
  return cudaLaunchKernelEx(&cfg, attn_decode_kernel<1>, a);
}

size_t attn_static_part_limit() { return kStaticPartBytes; }
int attn_static_counter_limit() { return kStaticCounters; }

cudaError_t launch_attn_static(const AttnRequest& r, cudaStream_t st) {
  if (attn_part_bytes(r.lanes, r.n_kv, r.gqa, r.max_span) > kStaticPartBytes ||
      r.lanes * r.n_kv > kStaticCounters) {
    set_error("decode_attention_static: lanes x kv heads x chunks of max_span need " +
              std::to_string(attn_part_bytes(r.lanes, r.n_kv, r.gqa, r.max_span)) +
              " bytes of partials (limit " + std::to_string(kStaticPartBytes) +
              ") and lanes x kv heads <= " + std::to_string(kStaticCounters));
    return cudaErrorInvalidValue;
  }
  // The host-side name of the array is not a device address: resolve it once per device, with
  // that device current, and pass the resolved pointer to the kernel.
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) {
    set_error("decode_attention_static: device index out of range");
    return cudaErrorInvalidValue;
  }
  static std::mutex mu;
  static void* scratch[64] = {nullptr};
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!scratch[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_attn_static_scratch);
      if (e != cudaSuccess) {
        set_error(std::string("decode_attention_static: cudaGetSymbolAddress failed: ") +
                  cudaGetErrorString(e));
        return e;
      }
      scratch[dev] = p;
    }
    base = scratch[dev];
  }
  AttnWorkspace w;
  w.part = static_cast<float*>(base);
  w.part_bytes = kStaticPartBytes;
  w.counters = reinterpret_cast<unsigned*>(static_cast<unsigned char*>(base) + kStaticPartBytes);
  w.n_counters = kStaticCounters;
  // The counters must start at zero; a previous call leaves them at zero, but one that was cut
  // short (a bounded wait that gave up elsewhere in the stream) may not, so clear them here.
  e = cudaMemsetAsync(w.counters, 0, size_t(r.lanes) * r.n_kv * sizeof(unsigned), st);
  if (e != cudaSuccess) return e;
  return launch_attn(r, w, st);
}

}  // namespace tts
