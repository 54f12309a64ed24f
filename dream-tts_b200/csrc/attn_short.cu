// a6 for short spans (the depth predictor's <= 17 positions, a talker lane's first steps):
// decode attention on the CUDA cores, one warp per (lane, kv head). At a few dozen positions
// the work is a few KB of K/V per item; the tensor-core kernel's fixed cost (TMEM, barriers,
// tensor maps, the split bookkeeping) would dominate, so these spans take this path.
//
// Arithmetic as crates/tts-nn/src/attn.rs:90-126 (Scores::cpu_fwd) and :203-238
// (Weighted::cpu_fwd) with candle's softmax_last_dim in between: f32 scores q.k (scale folded
// into q), softmax over [wstart, span), o = sum_t p_t v_t; the softmax is taken online over
// groups of positions (max-subtracted exponentials, rescaled per group, one division at the
// end), which equals the reference's up to f32 rounding.
#include "l2_prefetch.cuh"
#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

namespace {

constexpr int kWarps = 4;

struct ShortArgs {
  const float* q;
  const __half* k;
  const __half* v;
  const int* bt;
  int max_blocks, bs, num_blocks;
  int* err;
  const int* spans;
  int span_add, max_span, window;
  int lanes, n_kv;
  void* out;
  int out_f16;
  L2Prefetch pf;
};

TTS_DEV float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

TTS_DEV float4 h4(uint2 u) {
  const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

// positions whose K and V rows are in flight together (fewer with 8 q heads: registers)
template <int G>
constexpr int group_of() { return G >= 8 ? 8 : 16; }

// Each warp: q [G][128] (dims 4 * lane .. + 3 per warp lane), the lane's block-table entries
// (page p in warp lane p % 32, register p / 32), then per group of positions all K and V
// rows loaded at once, scores reduced across the warp, and an online softmax over the groups
// (running max, rescaled sum and output), normalised at the end.
template <int G>
__global__ void __launch_bounds__(kWarps * 32) attn_short_kernel(const ShortArgs a) {
  constexpr int kGroup = group_of<G>();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) issue_l2_prefetch(a.pf, blockIdx.x, gridDim.x);
  const int item = blockIdx.x * kWarps + warp;
  const bool live = item < a.lanes * a.n_kv;
  const int b = live ? item / a.n_kv : 0, h = live ? item % a.n_kv : 0;
  const int lim = min(min(a.max_blocks * a.bs, a.max_span), kShortSpanMax);
  const int npg = min(a.max_blocks, (lim + a.bs - 1) / a.bs);  // <= 64
  pdl_wait();
  if (!live) return;
  // independent loads first: the span, the block-table entries, q
  int span = a.spans[b] + a.span_add;
  int blk0 = lane < npg ? a.bt[(size_t)b * a.max_blocks + lane] : 0;
  int blk1 = lane + 32 < npg ? a.bt[(size_t)b * a.max_blocks + lane + 32] : 0;
  float4 q[G];
#pragma unroll
  for (int j = 0; j < G; ++j)
    q[j] = *reinterpret_cast<const float4*>(a.q + (((size_t)b * a.n_kv + h) * G + j) * 128 +
                                            lane * 4);
  if (span < 1 || span > lim) {
    if (a.err && lane == 0) atomicOr(a.err, kFlagSpanRange);
    span = max(1, min(span, lim));
  }
  const int ws = (a.window > 0 && span > a.window) ? span - a.window : 0;
  bool bad = false;
  float m[G], l[G];
  float4 o[G];
#pragma unroll
  for (int j = 0; j < G; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.f;
    o[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int t0 = ws; t0 < span; t0 += kGroup) {
    uint2 kr[kGroup], vr[kGroup];
#pragma unroll
    for (int u = 0; u < kGroup; ++u) {
      const int t = t0 + u;
      const int pg = t / a.bs;
      const int e0 = __shfl_sync(0xffffffffu, blk0, pg & 31);
      const int e1 = __shfl_sync(0xffffffffu, blk1, pg & 31);
      const int blk = pg < 32 ? e0 : e1;
      kr[u] = make_uint2(0u, 0u);
      vr[u] = make_uint2(0u, 0u);
      if (t < span) {
        if (blk < 0 || blk >= a.num_blocks) {
          bad = true;  // a page outside the pool reads as zeros
        } else {
          const size_t off = (((size_t)blk * a.n_kv + h) * a.bs + t % a.bs) * 128 + lane * 4;
          kr[u] = __ldg(reinterpret_cast<const uint2*>(a.k + off));
          vr[u] = __ldg(reinterpret_cast<const uint2*>(a.v + off));
        }
      }
    }
    float sc[G][kGroup];
    float gm[G];
#pragma unroll
    for (int j = 0; j < G; ++j) gm[j] = -INFINITY;
#pragma unroll
    for (int u = 0; u < kGroup; ++u) {
      const float4 k = h4(kr[u]);
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const float sv = warp_sum(q[j].x * k.x + q[j].y * k.y + q[j].z * k.z + q[j].w * k.w);
        sc[j][u] = t0 + u < span ? sv : -INFINITY;
        gm[j] = fmaxf(gm[j], sc[j][u]);
      }
    }
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const float mn = fmaxf(m[j], gm[j]);
      const float r = expf(m[j] - mn);  // 0 on the first group (m = -inf)
      l[j] *= r;
      o[j].x *= r;
      o[j].y *= r;
      o[j].z *= r;
      o[j].w *= r;
      m[j] = mn;
    }
#pragma unroll
    for (int u = 0; u < kGroup; ++u) {
      const float4 v = h4(vr[u]);
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const float e = expf(sc[j][u] - m[j]);  // 0 past the span
        l[j] += e;
        o[j].x += e * v.x;
        o[j].y += e * v.y;
        o[j].z += e * v.z;
        o[j].w += e * v.w;
      }
    }
  }
  if (bad && a.err) atomicOr(a.err, kFlagPageRange);
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const float inv = 1.f / l[j];
    const float4 r = make_float4(o[j].x * inv, o[j].y * inv, o[j].z * inv, o[j].w * inv);
    const size_t off = (((size_t)b * a.n_kv + h) * G + j) * 128 + lane * 4;
    if (a.out_f16) {
      __half2* y = reinterpret_cast<__half2*>(static_cast<__half*>(a.out) + off);
      y[0] = __floats2half2_rn(r.x, r.y);
      y[1] = __floats2half2_rn(r.z, r.w);
    } else {
      *reinterpret_cast<float4*>(static_cast<float*>(a.out) + off) = r;
    }
  }
}

}  // namespace

cudaError_t launch_attn_short(const AttnRequest& r, cudaStream_t st) {
  if (r.max_span > kShortSpanMax) {
    set_error("decode_attention: short-span path takes max_span <= 64");
    return cudaErrorInvalidValue;
  }
  ShortArgs a{};
  a.q = r.q;
  a.k = r.k_pool;
  a.v = r.v_pool;
  a.bt = r.block_table;
  a.max_blocks = r.max_blocks;
  a.bs = r.block_size;
  a.num_blocks = r.num_blocks;
  a.err = r.err;
  a.spans = r.spans;
  a.span_add = r.span_add;
  a.max_span = r.max_span;
  a.window = r.window;
  a.lanes = r.lanes;
  a.n_kv = r.n_kv;
  a.out = r.out;
  a.out_f16 = r.out_f16 ? 1 : 0;
  a.pf = r.next;
  const int items = r.lanes * r.n_kv;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((items + kWarps - 1) / kWarps, 1, 1);
  cfg.blockDim = dim3(kWarps * 32, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = r.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  switch (r.gqa) {
    case 1: return cudaLaunchKernelEx(&cfg, attn_short_kernel<1>, a);
    case 2: return cudaLaunchKernelEx(&cfg, attn_short_kernel<2>, a);
    case 4: return cudaLaunchKernelEx(&cfg, attn_short_kernel<4>, a);
    default: return cudaLaunchKernelEx(&cfg, attn_short_kernel<8>, a);
  }
}

}  // namespace tts
