// Paged decode attention (GQA, head_dim 128, f16 KV pages, f32 math).
//
// The B200 form of tts-nn's `attn::decode_attention` (crates/tts-nn/src/attn.rs:22-73; its
// CPU loops attn.rs:90-126 and 203-238, Metal `decode_attn_f16`): softmax(q . K^T) . V over
// positions [wstart, span) of each lane, with any scale already folded into q. Per-lane spans
// (the reference uses one span for the whole batch) let lanes of different lengths share a
// step, which is what a paged cache is for.
//
// Work unit: one CTA per (chunk of 128 positions, kv head, lane). Both query heads of a kv head
// are served from one read of each K/V row. The CTA first stages its chunk's K and V rows
// (64 KB) into shared memory with bulk async copies completing on one mbarrier, so the whole
// chunk is in flight at once and three CTAs per SM keep ~192 KB of reads outstanding. Then
// eight half-warps each take 16 consecutive positions; each of their 16 lanes owns 8 of the 128
// dims (one 16-byte shared load per row). Scores, the running max and the exp-rescaled sums
// are kept per half-warp, combined across half-warps in shared memory, and, when a lane's span
// needs several chunks, written as partials that the last CTA of that (lane, kv head) merges in
// chunk order (deterministic).
#include <cstdio>
#include <mutex>

#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

namespace {

constexpr int kChunk = 128;  // positions per CTA
constexpr int kHalfWarps = 8;
constexpr int kPerHalf = kChunk / kHalfWarps;  // 16
constexpr int kGroup = 8;                      // rows per inner iteration
constexpr int kMaxPages = kChunk + 1;          // pages one chunk can touch (block_size 1)
constexpr int kMaxChunks = 64;                 // 8192 positions

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

// Dynamic shared memory of one CTA: the chunk's K and V rows (64 KB), the half-warp partials
// and the merge scratch.
struct AttnSmem {
  __half k[kChunk][128];
  __half v[kChunk][128];
  float acc[kHalfWarps][2][128];
  float m[kHalfWarps][2];
  float l[kHalfWarps][2];
  float cm[kMaxChunks][2];
  float cl[kMaxChunks][2];
  int page[kMaxPages];
  uint64_t bar;
  int last;
};

TTS_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <int GQA>
__global__ void __launch_bounds__(128, 3) attn_decode_kernel(const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  AttnSmem& S = *reinterpret_cast<AttnSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                             ~uintptr_t(127));
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
  const int pg0 = p0 / a.bs, npg = (p1 - 1) / a.bs - pg0 + 1;
  const int t = threadIdx.x;

  // ---- stage the chunk's K and V rows into shared memory with bulk copies (one barrier)
  const int* bt = a.bt + (size_t)b * a.max_blocks;
  for (int i = t; i < npg; i += 128) {
    const int blk = bt[pg0 + i];
    S.page[i] = (blk >= 0 && blk < a.num_blocks) ? blk : -1;
  }
  if (t == 0) {
    mbar_init(&S.bar, 1);
    fence_barrier_init();
  }
  __syncthreads();  // barrier initialised, page table visible
  if (t < 32) {
    // warp 0, converged: one elected lane arms the barrier with the chunk's byte count, then
    // each lane issues the copies of its pages
    uint32_t bytes = 0;
    for (int i = t; i < npg; i += 32) {
      const int r0 = max(p0, (pg0 + i) * a.bs), r1 = min(p1, (pg0 + i + 1) * a.bs);
      if (S.page[i] >= 0) bytes += uint32_t(r1 - r0) * 512u;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, o);
    if (elect_one()) mbar_arrive_expect_tx(&S.bar, bytes);
    __syncwarp();
    for (int i = t; i < npg; i += 32) {
      if (S.page[i] < 0) continue;
      const int r0 = max(p0, (pg0 + i) * a.bs), r1 = min(p1, (pg0 + i + 1) * a.bs);
      const size_t src = (((size_t)S.page[i] * a.n_kv + h) * a.bs + (r0 - (pg0 + i) * a.bs)) * 128;
      bulk_g2s(&S.k[r0 - p0][0], a.k + src, uint32_t(r1 - r0) * 256u, &S.bar);
      bulk_g2s(&S.v[r0 - p0][0], a.v + src, uint32_t(r1 - r0) * 256u, &S.bar);
    }
    __syncwarp();
  }
  // rows of pages outside the pool read as zero (and are reported)
  for (int i = 0; i < npg; ++i) {
    if (S.page[i] >= 0) continue;
    const int r0 = max(p0, (pg0 + i) * a.bs), r1 = min(p1, (pg0 + i + 1) * a.bs);
    if (t == 0 && a.err) atomicOr(a.err, 1024);
    for (int e = t; e < (r1 - r0) * 16; e += 128) {
      reinterpret_cast<uint4*>(&S.k[r0 - p0][0])[e] = make_uint4(0, 0, 0, 0);
      reinterpret_cast<uint4*>(&S.v[r0 - p0][0])[e] = make_uint4(0, 0, 0, 0);
    }
  }

  const int lane = t & 31, warp = t >> 5;
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
  __syncthreads();  // zero-filled rows visible
  if (!mbar_wait(&S.bar, 0) && t == 0 && a.err) atomicOr(a.err, 2048);

  const int rows = p1 - p0;
  const int q0 = hw * kPerHalf;
  const int q1 = min(q0 + kPerHalf, rows);
  // The trip count is the same for both half-warps of a warp (their shuffles use the full
  // mask); rows past a half-warp's own range are masked instead.
  for (int it = 0; it < kPerHalf; it += kGroup) {
    const int pg = q0 + it;
    if (__all_sync(0xffffffffu, pg >= q1)) break;
    float kf[kGroup][8], vf[kGroup][8];
#pragma unroll
    for (int u = 0; u < kGroup; ++u) {
      // rows past this half-warp's range hold stale shared memory (possibly NaN patterns):
      // read zeros instead, so a masked row contributes exactly nothing
      const bool valid = pg + u < q1;
      const int p = valid ? pg + u : 0;
      uint4 ku = *reinterpret_cast<const uint4*>(&S.k[p][8 * j]);
      uint4 vu = *reinterpret_cast<const uint4*>(&S.v[p][8 * j]);
      if (!valid) ku = vu = make_uint4(0, 0, 0, 0);
      const __half2* kh = reinterpret_cast<const __half2*>(&ku);
      const __half2* vh = reinterpret_cast<const __half2*>(&vu);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 kk = __half22float2(kh[i]);
        const float2 vv = __half22float2(vh[i]);
        kf[u][2 * i] = kk.x;
        kf[u][2 * i + 1] = kk.y;
        vf[u][2 * i] = vv.x;
        vf[u][2 * i + 1] = vv.y;
      }
    }
#pragma unroll
    for (int g = 0; g < GQA; ++g) {
      float s[kGroup];
#pragma unroll
      for (int u = 0; u < kGroup; ++u) {
        float tt = 0.f;
#pragma unroll
        for (int d = 0; d < 8; ++d) tt += qv[g][d] * kf[u][d];
        tt += __shfl_xor_sync(0xffffffffu, tt, 8);
        tt += __shfl_xor_sync(0xffffffffu, tt, 4);
        tt += __shfl_xor_sync(0xffffffffu, tt, 2);
        tt += __shfl_xor_sync(0xffffffffu, tt, 1);
        s[u] = (pg + u < q1) ? tt : -INFINITY;
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

  // ---- combine the eight half-warps
#pragma unroll
  for (int g = 0; g < GQA; ++g) {
#pragma unroll
    for (int d = 0; d < 8; ++d) S.acc[hw][g][8 * j + d] = acc[g][d];
    if (j == 0) {
      S.m[hw][g] = m[g];
      S.l[hw][g] = l[g];
    }
  }
  __syncthreads();

  constexpr int kDims = GQA;  // (g, d) outputs per thread
  const size_t base = (((size_t)b * a.n_kv + h) * a.max_chunks + c) * GQA;
  float o[kDims], M[kDims], L[kDims];
  int gg[kDims], dd[kDims];
#pragma unroll
  for (int e = 0; e < kDims; ++e) {
    const int idx = t + e * 128;
    const int g = idx / 128, d = idx % 128;
    gg[e] = g;
    dd[e] = d;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kHalfWarps; ++w) mm = fmaxf(mm, S.m[w][g]);
    float ll = 0.f, oo = 0.f;
#pragma unroll
    for (int w = 0; w < kHalfWarps; ++w) {
      if (S.m[w][g] == -INFINITY) continue;
      const float f = expf(S.m[w][g] - mm);
      ll += S.l[w][g] * f;
      oo += S.acc[w][g][d] * f;
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

  // ---- several chunks: write this chunk's partial; the last CTA to arrive merges them in
  // chunk order (deterministic)
#pragma unroll
  for (int e = 0; e < kDims; ++e) {
    float* pp = a.part + (base + gg[e]) * 130;
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
    S.last = (prev == unsigned(nch - 1));
  }
  __syncthreads();
  if (!S.last) return;
  __threadfence();
  const size_t pb = ((size_t)b * a.n_kv + h) * a.max_chunks * GQA;
  for (int i = t; i < nch * GQA; i += 128) {
    const float* pp = a.part + (pb + i) * 130;
    S.cm[i / GQA][i % GQA] = __ldcg(pp + 128);
    S.cl[i / GQA][i % GQA] = __ldcg(pp + 129);
  }
  __syncthreads();
#pragma unroll
  for (int e = 0; e < kDims; ++e) {
    const int g = gg[e], d = dd[e];
    float mm = -INFINITY;
    for (int cc = 0; cc < nch; ++cc) mm = fmaxf(mm, S.cm[cc][g]);
    float ll = 0.f, oo = 0.f;
    for (int c0 = 0; c0 < nch; c0 += 4) {
      float ov[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        ov[u] = (c0 + u < nch) ? __ldcg(a.part + (pb + (size_t)(c0 + u) * GQA + g) * 130 + d) : 0.f;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (c0 + u >= nch) break;
        const float f = expf(S.cm[c0 + u][g] - mm);
        ll += S.cl[c0 + u][g] * f;
        oo += ov[u] * f;
      }
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
  if (chunks > kMaxChunks) {
    set_error("decode_attention: max_span exceeds 8192");
    return cudaErrorInvalidValue;
  }
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
  const size_t smem = sizeof(AttnSmem) + 128;
  {
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !done[dev]) {
      cudaFuncSetAttribute(attn_decode_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      cudaFuncSetAttribute(attn_decode_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      done[dev] = true;
    }
  }
  cfg.gridDim = dim3(chunks, r.n_kv, r.lanes);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.dynamicSmemBytes = smem;
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
