// a6 for short spans (the depth predictor's <= 17 positions, a talker lane's first steps):
// decode attention on the CUDA cores, one warp per (lane, q head). At a few dozen positions
// the work is a few KB of K/V per item; the tensor-core kernel's fixed cost (TMEM, barriers,
// tensor maps, the split bookkeeping) would dominate, so these spans take this path.
//
// Arithmetic as crates/tts-nn/src/attn.rs:90-126 (Scores::cpu_fwd) and :203-238
// (Weighted::cpu_fwd) with candle's softmax_last_dim in between: f32 scores q.k (scale folded
// into q), p = exp(s - max) / sum over [wstart, span), o = sum_t p_t v_t in position order.
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
  int lanes, n_kv, gqa;
  void* out;
  int out_f16;
  L2Prefetch pf;
};

TTS_DEV float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

TTS_DEV float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

TTS_DEV float4 h4(uint2 u) {
  const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

// Each warp takes one (lane, q head): enough warps to cover the SMs' latency at a few lanes
// (the kv head's K/V rows are read once per q head of its group, from L2). Positions go across
// the warp, 16 per pass, two warp lanes per position (dims 0..63 and 64..127): a warp lane reads
// its half K row and forms its half score against q in shared memory, one exchange completes
// it; the softmax is two warp reductions; then the warp lanes own 4 dims each and sum p_t v_t
// over the positions in order, p_t broadcast from its lane.
__global__ void __launch_bounds__(kWarps * 32) attn_short_kernel(const ShortArgs a) {
  __shared__ __align__(16) float qs[kWarps][128];
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) issue_l2_prefetch(a.pf, blockIdx.x, gridDim.x);
  const int heads = a.n_kv * a.gqa;
  const int item = blockIdx.x * kWarps + warp;
  const bool live = item < a.lanes * heads;
  const int b = live ? item / heads : 0, qh = live ? item % heads : 0;
  const int h = qh / a.gqa;
  const int lim = min(min(a.max_blocks * a.bs, a.max_span), kShortSpanMax);
  const int npg = min(a.max_blocks, (lim + a.bs - 1) / a.bs);  // <= 64
  pdl_wait();
  if (!live) return;
  // independent loads first: the span, the block-table entries, q
  int span = a.spans[b] + a.span_add;
  const int blk0 = lane < npg ? a.bt[(size_t)b * a.max_blocks + lane] : 0;
  const int blk1 = lane + 32 < npg ? a.bt[(size_t)b * a.max_blocks + lane + 32] : 0;
  *reinterpret_cast<float4*>(&qs[warp][lane * 4]) =
      *reinterpret_cast<const float4*>(a.q + ((size_t)b * heads + qh) * 128 + lane * 4);
  if (span < 1 || span > lim) {
    if (a.err && lane == 0) atomicOr(a.err, kFlagSpanRange);
    span = max(1, min(span, lim));
  }
  const int ws = (a.window > 0 && span > a.window) ? span - a.window : 0;
  const int n = span - ws;  // 1..64 positions
  auto block_of = [&](int t, bool& bad) {
    const int pg = t / a.bs;
    const int e0 = __shfl_sync(0xffffffffu, blk0, pg & 31);
    const int e1 = __shfl_sync(0xffffffffu, blk1, pg & 31);
    const int blk = pg < 32 ? e0 : e1;
    if (blk < 0 || blk >= a.num_blocks) {
      bad = true;  // a page outside the pool reads as zeros
      return -1;
    }
    return blk;
  };
  __syncwarp();
  bool bad = false;
  const int pos = lane & 15, half = lane >> 4;
  // ---- scores: position r * 16 + pos of [ws, span), half the dims per warp lane
  float sc[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    sc[r] = -INFINITY;
    if (r * 16 >= n) continue;  // warp-uniform
    const int i = r * 16 + pos;
    const int t = ws + min(i, n - 1);
    const int blk = block_of(t, bad);
    uint4 kr[8];
    if (blk >= 0 && i < n) {
      const uint4* row = reinterpret_cast<const uint4*>(
          a.k + (((size_t)blk * a.n_kv + h) * a.bs + t % a.bs) * 128 + half * 64);
#pragma unroll
      for (int c = 0; c < 8; ++c) kr[c] = __ldg(row + c);
    } else {
#pragma unroll
      for (int c = 0; c < 8; ++c) kr[c] = make_uint4(0u, 0u, 0u, 0u);
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 qa = *reinterpret_cast<const float4*>(&qs[warp][half * 64 + c * 8]);
      const float4 qb = *reinterpret_cast<const float4*>(&qs[warp][half * 64 + c * 8 + 4]);
      const float4 ka = h4(make_uint2(kr[c].x, kr[c].y));
      const float4 kb = h4(make_uint2(kr[c].z, kr[c].w));
      acc[c & 3] += qa.x * ka.x + qa.y * ka.y + qa.z * ka.z + qa.w * ka.w +
                    qb.x * kb.x + qb.y * kb.y + qb.z * kb.z + qb.w * kb.w;
    }
    const float part = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    const float full = part + __shfl_xor_sync(0xffffffffu, part, 16);
    if (i < n) sc[r] = full;
  }
  // ---- softmax over the positions: max-subtracted exponentials, normalised by their sum
  // (each position's score sits in both of its warp lanes; the lower half counts it)
  const float m = warp_max(fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3])));
  float e[4], part = 0.f;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    e[r] = sc[r] == -INFINITY ? 0.f : expf(sc[r] - m);
    if (half == 0) part += e[r];
  }
  const float l = warp_sum(part);
  float p[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) p[r] = e[r] / l;
  // ---- o = sum_t p_t v_t in position order; this warp lane owns dims 4 * lane .. + 3
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i0 = 0; i0 < n; i0 += 8) {
    uint2 vr[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int t = ws + min(i0 + u, n - 1);
      const int blk = block_of(t, bad);
      vr[u] = blk >= 0 ? __ldg(reinterpret_cast<const uint2*>(
                             a.v + (((size_t)blk * a.n_kv + h) * a.bs + t % a.bs) * 128 +
                             lane * 4))
                       : make_uint2(0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u;
      const float4 v = h4(vr[u]);
      const int r = i >> 4;
      const float pr = r == 0 ? p[0] : r == 1 ? p[1] : r == 2 ? p[2] : p[3];
      const float pi = __shfl_sync(0xffffffffu, pr, i & 15);
      if (i < n) {
        o.x += pi * v.x;
        o.y += pi * v.y;
        o.z += pi * v.z;
        o.w += pi * v.w;
      }
    }
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0 && a.err) atomicOr(a.err, kFlagPageRange);
  const size_t off = ((size_t)b * heads + qh) * 128 + lane * 4;
  if (a.out_f16) {
    __half2* y = reinterpret_cast<__half2*>(static_cast<__half*>(a.out) + off);
    y[0] = __floats2half2_rn(o.x, o.y);
    y[1] = __floats2half2_rn(o.z, o.w);
  } else {
    *reinterpret_cast<float4*>(static_cast<float*>(a.out) + off) = o;
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
  a.gqa = r.gqa;
  a.out = r.out;
  a.out_f16 = r.out_f16 ? 1 : 0;
  a.pf = r.next;
  const int items = r.lanes * r.n_kv * r.gqa;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((items + kWarps - 1) / kWarps, 1, 1);
  cfg.blockDim = dim3(kWarps * 32, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = r.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attn_short_kernel, a);
}

}  // namespace tts
