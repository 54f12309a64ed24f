// Paged decode attention on the tensor cores (GQA, head_dim 128, f16 KV pages, f32 results).
//
// The B200 form of tts-nn's `attn::decode_attention` (crates/tts-nn/src/attn.rs:22-73; its
// CPU loops attn.rs:90-126 and 203-238, Metal `decode_attn_f16`): softmax(q . K^T) . V over
// positions [wstart, span) of each lane, with any scale already folded into q. Per-lane spans
// (the reference uses one span for the whole batch) let lanes of different lengths share a
// step, which is what a paged cache is for.
//
// Work: each (lane, kv head) pair's positions are cut into 128-position chunks; all chunks of
// all pairs form one list (lane-major, then kv head, then chunk) that is split into equal
// contiguous ranges, one per CTA, with one persistent CTA per SM. A CTA walks its range with
// three kinds of warps tied together by mbarriers:
//   * warp 4 (loader) stages each chunk's K and V tiles into three-deep rings with TMA
//     (128-byte swizzle, one box per run of a page), reading the block table one chunk ahead;
//   * warp 5 (MMA) issues S = K . Q^T (M = 128 positions, N = 16, K = 128 dims) and
//     O^T = V^T . P^T (M = 128 dims, N = 16, K = 128 positions) on tcgen05, f32 accumulators
//     double-buffered in TMEM, the scores of the next chunk ahead of the values of this one.
//     The N = 16 columns hold each query head twice, as an f16 high part and a scaled f16 low
//     part (q = hi + lo / 2048, likewise p), so the products keep f32-level accuracy;
//   * warps 0-3 (softmax) take one position each for the scores and one output dim each for the
//     values: running max, exp, P written back to shared memory for the MMA warp, and the
//     running sum and output (folded in one chunk late, when that chunk's values are long done).
// A pair wholly inside one CTA writes its output directly. A CTA's first and last segments may
// hold only part of a pair: the softmax warps write a partial (o, max, sum) and hand it to warp
// 6 (epilogue), which counts the pair's arrived chunks and, in the CTA that completes the pair,
// merges the segments in chunk order, so results are deterministic and the softmax warps never
// wait on a global fence or atomic.
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "tts_common.cuh"
#include "tts_internal.h"
#include "l2_prefetch.cuh"

namespace tts {

namespace {

constexpr int kChunk = 128;      // positions per chunk (the MMA's M for S)
constexpr int kStages = 3;       // K and V ring depth
constexpr int kSoftmax = 128;    // warps 0-3: one TMEM lane quarter each
constexpr int kLoaderWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kEpiWarp = 6;
constexpr int kPvWarp = 7;     // issues the O MMAs, beside the score MMAs of kMmaWarp
constexpr int kThreads = 256;
constexpr int kMaxChunks = 64;   // 8192 positions
constexpr int kMaxLanes = 512;
constexpr int kN = 16;           // MMA N: GQA high rows, GQA low rows, zero padding
constexpr float kLo = 2048.f;    // scale of the low f16 parts
constexpr uint32_t kBarSoftmax = 1;  // named barrier: softmax warps
constexpr uint32_t kBarTmem = 2;     // named barrier: softmax + both MMA warps (TMEM release)
constexpr int kTmemBarThreads = kSoftmax + 64;

struct AttnArgs {
  const float* q;
  const int* bt;
  int max_blocks, bs, num_blocks;
  int max_span;
  int box_rows;  // rows per TMA box: divides bs, or 128 when each lane has one page
  int* err;
  const int* spans;
  int span_add;
  int window;
  int lanes, n_kv;
  int max_chunks;
  float* part;  // [lanes][n_kv][max_chunks][GQA][130]: 128 o, m, l
  unsigned* counters;
  void* out;
  int out_f16;
  int early_meta;  // spans, work split and first pages before the dependency wait
  int merge_last;  // the last segment of a split pair merged by the softmax warps when it can
  L2Prefetch pf;   // the next GEMM's first weight blocks
};

// One K or V tile of a chunk: dims 0-63 / 64-127, each 128 rows x 128 B, 128-byte swizzle.
struct __align__(1024) Tile {
  uint8_t d[2][kChunk * 128];
};

struct AttnSmem {
  Tile kt[kStages];
  Tile vt[kStages];
  uint8_t qb[2][2][kN * 128];  // B of S per segment parity: q hi/lo rows, K-major, swizzled
  uint8_t pb[2][2][kN * 128];  // B of O per item parity: p hi/lo rows over the positions
  float red_max[2][4][8];
  float red_sum[2][4][8];
  uint64_t full_k[kStages], full_v[kStages], empty_k[kStages], empty_v[kStages];
  uint64_t s_full[2], s_empty[2], p_full[2], o_full[2], o_empty[2], q_full[2];
  uint64_t seg_done[2];  // partial segment k written (every softmax thread arrives)
  struct {
    int b, h, c_first, len;
  } seg_info[2];
  uint32_t inv_k[kStages];  // boxes of the tile whose page is outside the pool
  uint32_t inv_v[kStages];
  uint32_t tmem;
  int last;
  int merge_here;  // the CTA's last segment is merged by the softmax warps
  unsigned long long tl_p0, tl_plast;  // tracing build: first and last P handed to the O MMA
  unsigned long long tl_q0, tl_q1;     // tracing build: softmax warps past the wait, q staged
  int span[kMaxLanes];
  int cnt[kMaxLanes];         // chunk-list items of each lane (chunks x n_kv)
  int prefix[kMaxLanes + 1];  // chunk-list offset of each lane
};

// Byte offset of element (row r, column e < 64) in a K-major tile of 128-byte rows written
// with the 128-byte swizzle (16-byte chunk index XOR row mod 8).
TTS_DEV uint32_t sw128(int r, int e) {
  return uint32_t(r) * 128u + ((uint32_t((e >> 3) ^ (r & 7))) << 4) + uint32_t(e & 7) * 2u;
}

// Position range of one lane: [ws, span), chunks start at c0 (ws rounded down to 128).
struct LaneRange {
  int span, ws, c0, nch;
};
TTS_DEV LaneRange lane_range(int span, int window) {
  LaneRange r;
  r.span = span;
  r.ws = (window > 0 && span > window) ? span - window : 0;
  r.c0 = (r.ws / kChunk) * kChunk;
  r.nch = (span - r.c0 + kChunk - 1) / kChunk;
  return r;
}

// A place in a CTA's walk over the chunk list: lane, kv head, chunk, and a counter of the
// (lane, kv head) segments started so far.
struct Cursor {
  int b, h, c, seg;
  LaneRange lr;
};
TTS_DEV void cursor_next(Cursor& x, const int* span, const AttnArgs& a) {
  if (++x.c == x.lr.nch) {
    x.c = 0;
    ++x.seg;
    if (++x.h == a.n_kv) {
      x.h = 0;
      if (x.b + 1 < a.lanes) {
        ++x.b;
        x.lr = lane_range(span[x.b], a.window);
      }
    }
  }
}
// Rows [vlo, vhi) of the cursor's chunk hold positions of the lane's range.
TTS_DEV void chunk_rows(const Cursor& x, int& vlo, int& vhi) {
  const int p0 = x.lr.c0 + x.c * kChunk;
  vlo = max(x.lr.ws - p0, 0);
  vhi = min(x.lr.span - p0, kChunk);
}

// Which CTA of `grid` owns item x of a list of `total` split as [total*i/grid, total*(i+1)/grid),
// and where CTA i's range starts. 32-bit arithmetic (the host keeps total x grid below 2^31): a
// 64-bit division is a long software sequence, and the split pairs' merges run these on the
// attention's critical path.
TTS_DEV int owner_of(unsigned x, unsigned total, unsigned grid) {
  return int(((x + 1u) * grid + total - 1u) / total) - 1;
}
TTS_DEV unsigned range_lo(unsigned i, unsigned total, unsigned grid) { return total * i / grid; }

// Zeroes rows of a K or V tile: rows outside [vlo, vhi), and rows of boxes flagged in `inv`
// (pages outside the pool). Thread `tid` of a group of `n` takes every n-th 16-byte piece.
TTS_DEV void zero_rows(Tile& tile, int vlo, int vhi, uint32_t inv, int box, int tid, int n) {
  const int r0 = (vlo / box) * box;
  for (int u = tid; u < kChunk * 16; u += n) {
    const int r = u >> 4;
    const bool bad = r < vlo || r >= vhi || (inv && r >= r0 && ((inv >> ((r - r0) / box)) & 1u));
    if (bad)
      *reinterpret_cast<uint4*>(&tile.d[(u >> 3) & 1][r * 128 + (u & 7) * 16]) =
          make_uint4(0, 0, 0, 0);
  }
}

// One step of merging a pair's parts in chunk order: the running (max, sum, output) takes part
// (cm, cl, ov). Explicit roundings, so the epilogue warp's merge and the softmax warps' merge of
// a CTA's last segment give the same bits whichever of them runs.
TTS_DEV void merge_step(float& mm, float& ll, float& oo, float cm, float cl, float ov) {
  const float mn = fmaxf(mm, cm);
  const float f0 = (mm == -INFINITY) ? 0.f : expf(mm - mn);
  const float f1 = expf(cm - mn);
  ll = __fmaf_rn(ll, f0, __fmul_rn(cl, f1));
  oo = __fmaf_rn(oo, f0, __fmul_rn(ov, f1));
  mm = mn;
}

template <int GQA>
__global__ void __launch_bounds__(kThreads, 1)
    attn_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  [[maybe_unused]] const unsigned long long tl_entry = TTS_TL_NOW();
  extern __shared__ uint8_t smem_raw[];
  AttnSmem& S = *reinterpret_cast<AttnSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  pdl_launch_dependents();

  if (warp == kLoaderWarp && lane == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&S.full_k[s], 1);
      mbar_init(&S.full_v[s], 1);
      mbar_init(&S.empty_k[s], 1);
      mbar_init(&S.empty_v[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.s_full[i], 1);
      mbar_init(&S.o_full[i], 1);
      mbar_init(&S.s_empty[i], 4);  // one arrival per softmax warp
      mbar_init(&S.p_full[i], 4);
      mbar_init(&S.o_empty[i], 4);
      mbar_init(&S.q_full[i], 4);
      mbar_init(&S.seg_done[i], kSoftmax);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&S.tmem, 64);
    tmem_relinquish();
    tc_fence_before();
  }
  // zero the B tiles once: rows past 2 * GQA stay zero for the whole kernel
  for (int i = t; i < int(sizeof(S.qb) + sizeof(S.pb)) / 16; i += kThreads)
    reinterpret_cast<uint4*>(&S.qb[0][0][0])[i] = make_uint4(0, 0, 0, 0);

  // With early_meta the spans and the block table are final already: the work split and the
  // first page lookups go ahead of the dependency wait. Every warp that reads what the previous
  // kernel wrote (q, K/V rows) or writes what earlier kernels read (partials, counters, the
  // output) waits first.
  if (!a.early_meta) pdl_wait();
  [[maybe_unused]] unsigned long long tl_rel = TTS_TL_NOW();
  // ---- spans and the chunk-list offsets of every lane
  for (int b = t; b < a.lanes; b += kThreads) {
    int span = a.spans[b] + a.span_add;
    const int lim = min(a.max_blocks * a.bs, a.max_span);
    if (span < 1 || span > lim) {
      if (a.err && blockIdx.x == 0) atomicOr(a.err, kFlagSpanRange);
      span = max(1, min(span, lim));
    }
    S.span[b] = span;
    S.cnt[b] = lane_range(span, a.window).nch * a.n_kv;
  }
  __syncthreads();
  if (warp == 0) {
    // exclusive scan of the per-lane counts: each lane of warp 0 takes a run of lanes
    const int per = (a.lanes + 31) / 32;
    const int b0 = min(lane * per, a.lanes), b1 = min(b0 + per, a.lanes);
    int sum = 0;
    for (int b = b0; b < b1; ++b) sum += S.cnt[b];
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - sum;
    for (int b = b0; b < b1; ++b) {
      S.prefix[b] = run;
      run += S.cnt[b];
    }
    if (lane == 31) S.prefix[a.lanes] = incl;
  }
  __syncthreads();
  tc_fence_after();

  const int total = S.prefix[a.lanes];
  const int lo = range_lo(blockIdx.x, unsigned(total), gridDim.x);
  const int hi = range_lo(blockIdx.x + 1, unsigned(total), gridDim.x);
  const int n = hi - lo;  // items of this CTA
  const uint32_t tmem = S.tmem;

  // the first item: lane b with prefix[b] <= lo < prefix[b + 1]
  Cursor first{};
  {
    int l = 0, r = a.lanes - 1;
    while (l < r) {
      const int m = (l + r + 1) >> 1;
      if (S.prefix[m] <= lo) l = m; else r = m - 1;
    }
    first.b = n > 0 ? l : 0;
    first.lr = lane_range(S.span[first.b], a.window);
    const int rel = n > 0 ? int(lo - S.prefix[first.b]) : 0;  // 32-bit: a lane's items
    first.h = rel / first.lr.nch;
    first.c = rel % first.lr.nch;
    first.seg = 0;
  }

  if (warp == kLoaderWarp) {
    // ================= loader: K of item k, then V of item k - 1 (the scores run one item
    // ahead of the values). Lane i handles box i of a tile: its block-table read and its two
    // TMA copies (dims 0-63 and 64-127).
    const uint64_t pol = l2_policy_evict_first();
    const int box = a.box_rows;
    const uint32_t box_bytes = uint32_t(box) * 128u;
    struct Boxes {
      int r0, nbox, pos, blk, row;
      bool valid;
      uint32_t vmask, bmask;
    };
    auto lookup = [&](const Cursor& x) {
      Boxes q{};
      int vlo, vhi;
      chunk_rows(x, vlo, vhi);
      q.r0 = (vlo / box) * box;
      q.nbox = (vhi - q.r0 + box - 1) / box;  // 1..16 (box >= 8)
      q.blk = -1;
      if (lane < q.nbox) {
        q.pos = x.lr.c0 + x.c * kChunk + q.r0 + lane * box;
        const int pg = q.pos / a.bs;
        if (pg < a.max_blocks) q.blk = a.bt[(size_t)x.b * a.max_blocks + pg];
      }
      return q;
    };
    auto finish = [&](Boxes& q, int h) {
      q.valid = lane < q.nbox && q.blk >= 0 && q.blk < a.num_blocks;
      q.row = q.valid ? (q.blk * a.n_kv + h) * a.bs + q.pos % a.bs : 0;
      q.vmask = __ballot_sync(0xffffffffu, q.valid);
      q.bmask = (1u << q.nbox) - 1u;
    };
    auto issue = [&](const Boxes& q, const CUtensorMap* tm, Tile& dst, uint64_t* full,
                     uint32_t* inv) {
      if (elect_one()) {
        *inv = q.bmask & ~q.vmask;
        if ((q.bmask & ~q.vmask) && a.err) atomicOr(a.err, kFlagPageRange);
        mbar_arrive_expect_tx(full, uint32_t(__popc(q.vmask)) * box_bytes * 2u);
      }
      __syncwarp();
      if (q.valid) {
        const int r = q.r0 + lane * box;
        tma_load_2d_hint(&dst.d[0][r * 128], tm, full, 0, q.row, pol);
        tma_load_2d_hint(&dst.d[1][r * 128], tm, full, 64, q.row, pol);
      }
      __syncwarp();
    };
    Cursor x = first;
    Boxes next = n > 0 ? lookup(x) : Boxes{}, prev{};
    if (a.early_meta) {
      pdl_wait();  // K/V rows of this step (the newest position) are the previous kernel's
      tl_rel = TTS_TL_NOW();
    }
    bool ok = true;
    int nk = 0, nv = 0;  // tiles issued
    for (int k = 0; k <= n && ok; ++k) {
      Boxes cur{};
      if (k < n) {
        const int s = int(k % kStages);
        if (k >= kStages) ok = mbar_wait(&S.empty_k[s], uint32_t((k / kStages) - 1) & 1);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        cur = next;
        finish(cur, x.h);
        issue(cur, &tmK, S.kt[s], &S.full_k[s], &S.inv_k[s]);
        ++nk;
        cursor_next(x, S.span, a);
        if (k + 1 < n) next = lookup(x);  // read ahead: used next round
      }
      if (k >= 1) {
        const int kv = k - 1;
        const int s = int(kv % kStages);
        if (kv >= kStages) ok = mbar_wait(&S.empty_v[s], uint32_t((kv / kStages) - 1) & 1);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        issue(prev, &tmV, S.vt[s], &S.full_v[s], &S.inv_v[s]);
        ++nv;
      }
      prev = cur;
    }
    // the cache is all requested: start on the output projection's weights
    if (elect_one()) issue_l2_prefetch(a.pf, blockIdx.x, gridDim.x);
    __syncwarp();
    if (!ok && a.err && lane == 0) atomicOr(a.err, kFlagAttnWait);
    // Leave no copy in flight: wait (bounded) for the last tiles issued to land.
    for (int j = max(0, nk - kStages); j < nk; ++j)
      mbar_wait(&S.full_k[j % kStages], uint32_t(j / kStages) & 1);
    for (int j = max(0, nv - kStages); j < nv; ++j)
      mbar_wait(&S.full_v[j % kStages], uint32_t(j / kStages) & 1);
    return;
  }

  const uint32_t idesc_s = idesc_f16_f32(128, kN);
  const uint32_t idesc_o = idesc_f16_f32(128, kN) | (1u << 15);  // A (V^T) MN-major

  // O(i) = V(i)^T . P(i)^T, issued by the O warp when P(i) and V(i) are in place
  auto do_o = [&](int i, bool& ok, int& no) {
    const int s = int(i % kStages);
    ok = mbar_wait(&S.p_full[i & 1], uint32_t(i >> 1) & 1) && ok;
    ok = mbar_wait(&S.full_v[s], uint32_t(i / kStages) & 1) && ok;
    if (i >= 2) ok = mbar_wait(&S.o_empty[i & 1], uint32_t((i >> 1) - 1) & 1) && ok;
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) return;
    if (S.inv_v[s]) {  // rows of pages outside the pool read as zero
      zero_rows(S.vt[s], 0, kChunk, S.inv_v[s], a.box_rows, lane, 32);
      fence_proxy_async();
      __syncwarp();
    }
    tc_fence_after();
    if (elect_one()) {
      const uint32_t vb = smem_u32(&S.vt[s].d[0][0]);
      const uint32_t pb[2] = {smem_u32(&S.pb[i & 1][0][0]), smem_u32(&S.pb[i & 1][1][0])};
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        umma_f16(tmem + 32 + (i & 1) * 16, smem_desc(vb + kk * 2048, kChunk * 128, 1024, 2),
                 desc_k_sw128(pb[kk >> 2] + (kk & 3) * 32), idesc_o, kk > 0);
      umma_commit(&S.o_full[i & 1]);
      umma_commit(&S.empty_v[s]);
    }
    __syncwarp();
    ++no;
  };

  if (warp == kPvWarp) {
    // ================= O warp: O(i) for every item, in order. Its MMAs and the score warp's
    // run side by side (different TMEM columns and operands), so neither chain waits for the
    // other's issue.
    bool ok = true;
    int no = 0;
    for (int i = 0; i < n && ok; ++i) do_o(i, ok, no);
    if (!ok && a.err && lane == 0) atomicOr(a.err, kFlagAttnWait);
    if (!ok && no > 0) mbar_wait(&S.o_full[(no - 1) & 1], uint32_t((no - 1) >> 1) & 1, 100000000ull);
    tc_fence_before();
    bar_and(kBarTmem, kTmemBarThreads, true);
    return;
  }

  if (warp == kMmaWarp) {
    // ================= score warp: S(j) = K(j) . Q^T when K(j) and its segment's q are in place
    bool ok = true;
    int ns = 0;  // MMA groups issued
    [[maybe_unused]] unsigned long long tl_s0 = 0;
    Cursor x = first;
    for (int j = 0; j < n && ok; ++j) {
      const int s = int(j % kStages);
      if (j == 0 || x.c == 0) ok = mbar_wait(&S.q_full[x.seg & 1], uint32_t(x.seg >> 1) & 1) && ok;
      ok = mbar_wait(&S.full_k[s], uint32_t(j / kStages) & 1) && ok;
      if (j >= 2) ok = mbar_wait(&S.s_empty[j & 1], uint32_t((j >> 1) - 1) & 1) && ok;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const uint32_t inv = S.inv_k[s];
      if (inv) {
        // rows of pages outside the pool read as zero
        zero_rows(S.kt[s], 0, kChunk, inv, a.box_rows, lane, 32);
        fence_proxy_async();
        __syncwarp();
      }
      tc_fence_after();
      if (elect_one()) {
        const uint32_t kb[2] = {smem_u32(&S.kt[s].d[0][0]), smem_u32(&S.kt[s].d[1][0])};
        const uint32_t qb[2] = {smem_u32(&S.qb[x.seg & 1][0][0]), smem_u32(&S.qb[x.seg & 1][1][0])};
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16(tmem + (j & 1) * 16, desc_k_sw128(kb[kk >> 2] + (kk & 3) * 32),
                   desc_k_sw128(qb[kk >> 2] + (kk & 3) * 32), idesc_s, kk > 0);
        umma_commit(&S.s_full[j & 1]);
        umma_commit(&S.empty_k[s]);
      }
      __syncwarp();
#ifdef TTS_TIMELINE
      if (j == 0) tl_s0 = TTS_TL_NOW();
#endif
      ++ns;
      cursor_next(x, S.span, a);
    }
    if (!ok && a.err && lane == 0) atomicOr(a.err, kFlagAttnWait);
    // the softmax warps have consumed every result on the normal path; after a timeout, wait
    // (bounded) for what was issued before TMEM is released
    if (!ok && ns > 0)
      mbar_wait(&S.s_full[(ns - 1) & 1], uint32_t((ns - 1) >> 1) & 1, 100000000ull);
    tc_fence_before();
    bar_and(kBarTmem, kTmemBarThreads, true);
    tc_fence_after();
    tmem_dealloc(tmem, 64);
#ifdef TTS_TIMELINE
    // the score warp releases TMEM after every chunk's softmax and output MMA: compute ends
    if (lane == 0) {
      const uint64_t t_end = TTS_TL_NOW();
      timeline_recs<9>({kTlAttn | kTlEntry, kTlAttn | kTlReleased, kTlAttn | kTlCta,
                        kTlAttn | kTlEnd, kTlAttn | kTlAttnFirstS, kTlAttn | kTlAttnFirstP,
                        kTlAttn | kTlAttnLastP, kTlAttn | kTlAttnQWait, kTlAttn | kTlAttnQReady},
                       {tl_entry, tl_rel, uint64_t(blockIdx.x), t_end, tl_s0, S.tl_p0,
                        S.tl_plast, S.tl_q0, S.tl_q1});
    }
#endif
    return;
  }

  if (warp == kEpiWarp) {
    // ================= epilogue warp: arrival counts and merges of split pairs. Only the
    // first and the last segment of a CTA's range can hold part of a pair.
    if (a.early_meta) pdl_wait();
    int expect = 0;
    if (n > 0) {
      Cursor x = first;
      for (int j = 1; j < n; ++j) cursor_next(x, S.span, a);
      const bool first_part = first.c != 0;
      const bool last_part = x.c + 1 != x.lr.nch;
      expect = (x.seg == 0) ? ((first_part || last_part) ? 1 : 0)
                            : int(first_part) + int(last_part);
    }
    const int heads = a.n_kv * GQA;
    for (int k = 0; k < expect; ++k) {
      if (!__all_sync(0xffffffffu, mbar_wait(&S.seg_done[k], 0))) {
        if (a.err && lane == 0) atomicOr(a.err, kFlagAttnWait);
        break;
      }
      if (S.seg_info[k].len == 0) continue;  // merged by the softmax warps (finish_last)
      const int b = S.seg_info[k].b, h = S.seg_info[k].h;
      const int nch = lane_range(S.span[b], a.window).nch;
      unsigned last = 0;
      if (lane == 0) {
        __threadfence();  // release: the softmax warps' partial writes (ordered by the barrier)
        const unsigned len = unsigned(S.seg_info[k].len);
        const unsigned prev = atomicAdd(&a.counters[b * a.n_kv + h], len);
        last = (prev + len == unsigned(nch)) ? 1u : 0u;
        if (last) __threadfence();  // acquire: the other segments' partials
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) continue;
      // merge the pair's segments in chunk order; lane l takes dims 4l .. 4l + 3
      const size_t pbase = ((size_t)b * a.n_kv + h) * a.max_chunks;
      const long long base = S.prefix[b] + (long long)h * nch;
      float mm[GQA], ll[GQA], oo[GQA][4];
#pragma unroll
      for (int g = 0; g < GQA; ++g) {
        mm[g] = -INFINITY;
        ll[g] = 0.f;
#pragma unroll
        for (int u = 0; u < 4; ++u) oo[g][u] = 0.f;
      }
      // the pair's parts in chunk order: chunk 0 and each later CTA's range start in the pair
      const unsigned tot = unsigned(total), gr = gridDim.x;
      const int o0 = owner_of(unsigned(base), tot, gr);
      const int o1 = owner_of(unsigned(base + nch - 1), tot, gr);
      int last_cc = -1;
      for (int ci = o0; ci <= o1; ++ci) {
        const int cc = ci == o0 ? 0 : int(range_lo(unsigned(ci), tot, gr) - unsigned(base));
        if (cc <= last_cc) continue;  // CTAs with empty ranges share a start
        last_cc = cc;
#pragma unroll
        for (int g = 0; g < GQA; ++g) {
          const float* pp = a.part + ((pbase + cc) * GQA + g) * 130;
          const float cm = __ldcg(pp + 128), cl = __ldcg(pp + 129);
          // slots are 130 floats (8-byte aligned): four scalar loads
          const float4 ov = make_float4(__ldcg(pp + lane * 4), __ldcg(pp + lane * 4 + 1),
                                        __ldcg(pp + lane * 4 + 2), __ldcg(pp + lane * 4 + 3));
          const float ov4[4] = {ov.x, ov.y, ov.z, ov.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float m_u = mm[g], l_u = ll[g];
            merge_step(m_u, l_u, oo[g][u], cm, cl, ov4[u]);
            if (u == 3) {
              mm[g] = m_u;
              ll[g] = l_u;
            }
          }
        }
      }
      const size_t out_base = (size_t)b * heads * 128 + (size_t)h * GQA * 128;
#pragma unroll
      for (int g = 0; g < GQA; ++g) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float r = oo[g][u] / ll[g];
          const size_t oi = out_base + g * 128 + lane * 4 + u;
          if (a.out_f16)
            static_cast<__half*>(a.out)[oi] = __float2half_rn(r);
          else
            static_cast<float*>(a.out)[oi] = r;
        }
      }
      if (lane == 0) a.counters[b * a.n_kv + h] = 0u;
    }
#ifdef TTS_TIMELINE
    // the split pairs' merges (this warp's last work; it has none when no pair ends here)
    if (lane == 0) {
      const uint64_t t_end = TTS_TL_NOW();
      timeline_recs<2>({kTlAttn | kTlCta, kTlAttn | kTlMerged}, {uint64_t(blockIdx.x), t_end});
    }
#endif
    return;
  }

  // ================= softmax warps 0-3 (thread t: TMEM lane t = chunk row t = output dim t)
  if (a.early_meta) pdl_wait();  // q is the previous kernel's output
#ifdef TTS_TIMELINE
  if (t == 0) S.tl_q0 = TTS_TL_NOW();
#endif
  const int heads = a.n_kv * GQA;
  const uint32_t lane_base = tmem + (uint32_t(warp * 32) << 16);
  bool ok = true;

  // q of a pair, loaded a segment ahead into registers, written as f16 hi/lo rows of the S
  // operand of its segment's buffer
  float qn[GQA];
  auto load_q = [&](const Cursor& x) {
#pragma unroll
    for (int g = 0; g < GQA; ++g) qn[g] = a.q[((size_t)x.b * heads + x.h * GQA + g) * 128 + t];
  };
  auto store_q = [&](int seg) {
#pragma unroll
    for (int g = 0; g < GQA; ++g) {
      const __half hi16 = __float2half_rn(qn[g]);
      const __half lo16 = __float2half_rn((qn[g] - __half2float(hi16)) * kLo);
      *reinterpret_cast<__half*>(&S.qb[seg & 1][t >> 6][sw128(g, t & 63)]) = hi16;
      *reinterpret_cast<__half*>(&S.qb[seg & 1][t >> 6][sw128(GQA + g, t & 63)]) = lo16;
    }
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.q_full[seg & 1]);
  };
  // the first item of the segment after the one `x` is in (x itself if none follows)
  auto next_segment = [&](Cursor x, int& at) -> Cursor {
    const int left = x.lr.nch - x.c;  // items of x's segment from x on
    at += left;
    x.c = x.lr.nch - 1;
    cursor_next(x, S.span, a);
    return x;
  };

  Cursor cur = first;
  // q of segments 0 and 1 now; registers then hold segment 2's
  int pos1 = 0, pos2 = 0;
  Cursor seg1 = cur, seg2 = cur;
  if (n > 0) {
    load_q(cur);
    store_q(0);
#ifdef TTS_TIMELINE
    if (t == 0) S.tl_q1 = TTS_TL_NOW();
#endif
    seg1 = next_segment(cur, pos1);
    if (pos1 < n) {
      load_q(seg1);
      store_q(1);
      pos2 = pos1;
      seg2 = next_segment(seg1, pos2);
      if (pos2 < n) load_q(seg2);
    }
  }

  // Running state of the current segment (max, sum, output dim t per q head), and the state of
  // a segment that ended at the previous item, set aside until that item is folded in.
  float m_run[GQA], l_run[GQA], acc[GQA];
  float m_fin[GQA], l_fin[GQA], acc_fin[GQA];
  float corr_pend[GQA];  // the pending item's rescale (previous max -> its max)
#pragma unroll
  for (int g = 0; g < GQA; ++g) {
    m_run[g] = -INFINITY;
    l_run[g] = 0.f;
    acc[g] = 0.f;
    m_fin[g] = -INFINITY;
    l_fin[g] = 0.f;
    acc_fin[g] = 0.f;
    corr_pend[g] = 0.f;
  }
  int n_partial = 0;  // partial segments handed to the epilogue warp (at most 2)
  // The item before this one: its sum and values are folded in one item late, after this
  // item's P is out (so its PV has run meanwhile and the chain scores -> P never waits on it);
  // when it ended a segment, that segment is written out then.
  bool pend = false;
  struct {
    int b, h, c_first, c_last, nch;
    bool ends;
  } prev{};
  int c_first = cur.c;

  // folds item i's sum and O into a state (l, acc) at the previous item's scale
  auto fold = [&](int i, float* l, float* o_acc) {
    ok = mbar_wait(&S.o_full[i & 1], uint32_t(i >> 1) & 1) && ok;
    tc_fence_after();
    float ov[16];
    tmem_ld16(lane_base + 32 + (i & 1) * 16, ov);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.o_empty[i & 1]);
#pragma unroll
    for (int g = 0; g < GQA; ++g) {
      l[g] = l[g] * corr_pend[g] + ((S.red_sum[i & 1][0][g] + S.red_sum[i & 1][1][g]) +
                                    (S.red_sum[i & 1][2][g] + S.red_sum[i & 1][3][g]));
      o_acc[g] = o_acc[g] * corr_pend[g] + (ov[g] + ov[GQA + g] * (1.f / kLo));
    }
  };
  // writes a finished segment (max m, sum l, output o_acc): the output of a whole pair, or a
  // partial for the epilogue warp
  auto finish_segment = [&](const float* m, const float* l, const float* o_acc) {
    const size_t out_base = (size_t)prev.b * heads * 128 + (size_t)prev.h * GQA * 128;
    if (prev.c_first == 0 && prev.c_last + 1 == prev.nch) {
#pragma unroll
      for (int g = 0; g < GQA; ++g) {
        const float r = o_acc[g] / l[g];
        const size_t oi = out_base + g * 128 + t;
        if (a.out_f16)
          static_cast<__half*>(a.out)[oi] = __float2half_rn(r);
        else
          static_cast<float*>(a.out)[oi] = r;
      }
    } else if (n_partial < 2) {
      const size_t pbase = ((size_t)prev.b * a.n_kv + prev.h) * a.max_chunks;
#pragma unroll
      for (int g = 0; g < GQA; ++g) {
        float* pp = a.part + ((pbase + prev.c_first) * GQA + g) * 130;
        pp[t] = o_acc[g];
        if (t == 0) {
          pp[128] = m[g];
          pp[129] = l[g];
        }
      }
      if (t == 0) {
        S.seg_info[n_partial].b = prev.b;
        S.seg_info[n_partial].h = prev.h;
        S.seg_info[n_partial].c_first = prev.c_first;
        S.seg_info[n_partial].len = prev.c_last - prev.c_first + 1;
      }
      mbar_arrive(&S.seg_done[n_partial]);
      ++n_partial;
    }
  };
  // The CTA's last segment. When it closes a pair split across CTAs and every other part has
  // arrived already (the next CTA processed its part at the start of its range), it is merged
  // here from registers: one acquire load and one read of the other parts, instead of a partial
  // write, the epilogue warp's arrival count and a merge that reads this part back.
  auto finish_last = [&](const float* m, const float* l, const float* o_acc) {
    const bool whole = prev.c_first == 0 && prev.c_last + 1 == prev.nch;
    if (whole || n_partial >= 2 || !a.merge_last) {
      finish_segment(m, l, o_acc);
      return;
    }
    const unsigned key = unsigned(prev.b * a.n_kv + prev.h);
    const unsigned len = unsigned(prev.c_last - prev.c_first + 1);
    if (t == 0)
      S.merge_here = (ld_acquire_u32(&a.counters[key]) + len == unsigned(prev.nch)) ? 1 : 0;
    bar_and(kBarSoftmax, kSoftmax, true);
    if (!S.merge_here) {
      finish_segment(m, l, o_acc);
      return;
    }
    const size_t pbase = ((size_t)prev.b * a.n_kv + prev.h) * a.max_chunks;
    const long long base = S.prefix[prev.b] + (long long)prev.h * prev.nch;
    const long long total = S.prefix[a.lanes];
    float mm[GQA], ll[GQA], oo[GQA];
#pragma unroll
    for (int g = 0; g < GQA; ++g) {
      mm[g] = -INFINITY;
      ll[g] = 0.f;
      oo[g] = 0.f;
    }
    // the pair's parts in chunk order: chunk 0 and each later CTA's range start in the pair
    const unsigned tot = unsigned(total), gr = gridDim.x;
    const int o0 = owner_of(unsigned(base), tot, gr);
    const int o1 = owner_of(unsigned(base + prev.nch - 1), tot, gr);
    int last_cc = -1;
    for (int ci = o0; ci <= o1; ++ci) {
      const int cc = ci == o0 ? 0 : int(range_lo(unsigned(ci), tot, gr) - unsigned(base));
      if (cc <= last_cc) continue;  // CTAs with empty ranges share a start
      last_cc = cc;
#pragma unroll
      for (int g = 0; g < GQA; ++g) {
        float cm, cl, ov;
        if (cc == prev.c_first) {
          cm = m[g];
          cl = l[g];
          ov = o_acc[g];
        } else {
          const float* pp = a.part + ((pbase + cc) * GQA + g) * 130;
          cm = __ldcg(pp + 128);
          cl = __ldcg(pp + 129);
          ov = __ldcg(pp + t);
        }
        merge_step(mm[g], ll[g], oo[g], cm, cl, ov);
      }
    }
    const size_t out_base = (size_t)prev.b * heads * 128 + (size_t)prev.h * GQA * 128;
#pragma unroll
    for (int g = 0; g < GQA; ++g) {
      const float r = oo[g] / ll[g];
      const size_t oi = out_base + g * 128 + t;
      if (a.out_f16)
        static_cast<__half*>(a.out)[oi] = __float2half_rn(r);
      else
        static_cast<float*>(a.out)[oi] = r;
    }
    if (t == 0) {
      a.counters[key] = 0u;  // every other part has counted in: no one else reads it
      S.seg_info[n_partial].len = 0;  // the epilogue warp has nothing left for this segment
    }
    mbar_arrive(&S.seg_done[n_partial]);
    ++n_partial;
  };

  for (int j = 0; j < n; ++j) {
    const int s = int(j % kStages);
    // first item of a segment after the first: the segment after next gets its q now (its
    // buffer was last read by scores that are complete)
    if (j > 0 && cur.c == 0 && pos2 < n) {
      store_q(cur.seg + 1);
      Cursor nx = seg2;
      int at = pos2;
      seg2 = next_segment(nx, at);
      pos2 = at;
      if (pos2 < n) load_q(seg2);
    }
    // a segment ended at the previous item: set its state aside until that item is folded,
    // and start this segment fresh
    const bool fin = pend && prev.ends;
    if (fin) {
#pragma unroll
      for (int g = 0; g < GQA; ++g) {
        m_fin[g] = m_run[g];
        l_fin[g] = l_run[g];
        acc_fin[g] = acc[g];
        m_run[g] = -INFINITY;
        l_run[g] = 0.f;
        acc[g] = 0.f;
      }
    }
    // ---- scores of item j (thread t = row t)
    int vlo, vhi;
    chunk_rows(cur, vlo, vhi);
    ok = mbar_wait(&S.s_full[j & 1], uint32_t(j >> 1) & 1) && ok;
    tc_fence_after();
    float sv[16];
    tmem_ld16(lane_base + (j & 1) * 16, sv);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.s_empty[j & 1]);
    const bool valid = t >= vlo && t < vhi;
    float sc[GQA];
#pragma unroll
    for (int g = 0; g < GQA; ++g) {
      sc[g] = valid ? sv[g] + sv[GQA + g] * (1.f / kLo) : -INFINITY;
      const float wm = warp_max(sc[g]);
      if (lane == 0) S.red_max[j & 1][warp][g] = wm;
    }
    if (!bar_and(kBarSoftmax, kSoftmax, ok)) {  // also makes item j - 1's sums visible
      ok = false;
      break;
    }
    // ---- softmax of item j; P as f16 hi/lo rows of the O operand
    float corr_new[GQA];
#pragma unroll
    for (int g = 0; g < GQA; ++g) {
      const float cmax = fmaxf(fmaxf(S.red_max[j & 1][0][g], S.red_max[j & 1][1][g]),
                               fmaxf(S.red_max[j & 1][2][g], S.red_max[j & 1][3][g]));
      const float mn = fmaxf(m_run[g], cmax);
      corr_new[g] = (m_run[g] == -INFINITY) ? 0.f : expf(m_run[g] - mn);
      const float p = valid ? expf(sc[g] - mn) : 0.f;
      m_run[g] = mn;
      const __half phi = __float2half_rn(p);
      const __half plo = __float2half_rn((p - __half2float(phi)) * kLo);
      *reinterpret_cast<__half*>(&S.pb[j & 1][t >> 6][sw128(g, t & 63)]) = phi;
      *reinterpret_cast<__half*>(&S.pb[j & 1][t >> 6][sw128(GQA + g, t & 63)]) = plo;
      const float ws = warp_sum(p);
      if (lane == 0) S.red_sum[j & 1][warp][g] = ws;
    }
    // V rows outside [vlo, vhi) must read as zero before the MMA (rows of missing pages are
    // cleared by the MMA warp)
    if (vlo > 0 || vhi < kChunk) {
      ok = mbar_wait(&S.full_v[s], uint32_t(j / kStages) & 1) && ok;
      zero_rows(S.vt[s], vlo, vhi, 0u, a.box_rows, t, kSoftmax);
    }
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.p_full[j & 1]);
#ifdef TTS_TIMELINE
    if (t == 0 && j == 0) S.tl_p0 = TTS_TL_NOW();
    if (t == 0 && j + 1 == n) S.tl_plast = TTS_TL_NOW();
#endif
    // ---- the previous item, now that this item's P is out, and the segment it ended
    if (pend) {
      if (fin) {
        fold(j - 1, l_fin, acc_fin);
        finish_segment(m_fin, l_fin, acc_fin);
      } else {
        fold(j - 1, l_run, acc);
      }
    }
#pragma unroll
    for (int g = 0; g < GQA; ++g) corr_pend[g] = corr_new[g];

    pend = true;
    prev.b = cur.b;
    prev.h = cur.h;
    prev.c_first = c_first;
    prev.c_last = cur.c;
    prev.nch = cur.lr.nch;
    prev.ends = (cur.c + 1 == cur.lr.nch) || (j + 1 == n);
    if (prev.ends) c_first = 0;  // the next item starts a pair
    cursor_next(cur, S.span, a);
  }
  // the last item: its sums need every warp's partial sum, then its segment is written
  if (ok && pend) {
    if (bar_and(kBarSoftmax, kSoftmax, ok)) {
      fold(n - 1, l_run, acc);
      finish_last(m_run, l_run, acc);
    } else {
      ok = false;
    }
  }
  if (!ok && a.err && t == 0) atomicOr(a.err, kFlagAttnWait);
  tc_fence_before();
  bar_and(kBarTmem, kTmemBarThreads, true);
}

}  // namespace

// Scratch for launch_attn_static, one fixed device array so that callers which must not
// allocate device memory can still run the attention: the split-KV partials, then a 256-byte
// status block whose first word collects the kernel's error flags (bounded waits that gave up,
// spans or pages out of range), then the per-(lane, kv head) arrival counters. Every GPU that
// loads the library holds this array until the process exits. All calls share it and it keeps
// the last call's contents, so the status word and the counters are cleared on every call, and
// calls that overlap on the GPU (two streams, two threads) race.
constexpr size_t kStaticPartBytes = size_t(4) << 20;  // 4 MiB of partials
constexpr size_t kStaticStatusBytes = 256;             // the status word, padded
constexpr int kStaticCounters = 4096;                  // lanes * n_kv
static __device__ __align__(256) unsigned char
    g_attn_static_scratch[kStaticPartBytes + kStaticStatusBytes + kStaticCounters * sizeof(unsigned)];

size_t attn_part_bytes(int lanes, int n_kv, int gqa, int max_span) {
  const int chunks = (max_span + kChunk - 1) / kChunk;
  return size_t(lanes) * n_kv * chunks * gqa * 130 * sizeof(float);
}

// Why the kernels cannot take request `r` ("" when they can); the caller prefixes its op name.
std::string attn_shape_error(const AttnRequest& r) {
  if (r.gqa != 1 && r.gqa != 2 && r.gqa != 4 && r.gqa != 8) return "gqa must be 1, 2, 4 or 8";
  if (r.lanes < 1 || r.n_kv < 1 || r.max_span < 1 || r.block_size < 1) return "empty shape";
  if (r.lanes > kMaxLanes) return "at most " + std::to_string(kMaxLanes) + " lanes per call";
  if (r.max_span <= kShortSpanMax) return "";
  if ((r.max_span + kChunk - 1) / kChunk > kMaxChunks)
    return "max_span exceeds " + std::to_string(kMaxChunks * kChunk);
  if (r.max_blocks != 1 && r.block_size % 8)
    return "block_size must be a multiple of 8 (or one page per lane)";
  return "";
}

cudaError_t launch_attn(const AttnRequest& r, const AttnWorkspace& w, cudaStream_t st) {
  const std::string why = attn_shape_error(r);
  if (!why.empty()) {
    set_error("decode_attention: " + why);
    return cudaErrorInvalidValue;
  }
  if (r.max_span <= kShortSpanMax) return launch_attn_short(r, st);
  const int chunks = (r.max_span + kChunk - 1) / kChunk;
  // TMA boxes copy runs of whole rows; a run never crosses a page, so the box height divides
  // the page size (or the lane's single page holds every position).
  int box = 0;
  if (r.max_blocks == 1) {
    box = kChunk;
  } else {
    box = 8;
    while (box < kChunk && r.block_size % (box * 2) == 0) box *= 2;
  }
  if (attn_part_bytes(r.lanes, r.n_kv, r.gqa, r.max_span) > w.part_bytes ||
      r.lanes * r.n_kv > w.n_counters) {
    set_error("decode_attention: workspace too small");
    return cudaErrorInvalidValue;
  }
  const uint64_t rows = uint64_t(r.num_blocks) * r.n_kv * r.block_size;
  CUtensorMap tmK, tmV;
  if (!make_tmap_2d_f16(&tmK, r.k_pool, 128, rows, 256, 64, uint32_t(box), true) ||
      !make_tmap_2d_f16(&tmV, r.v_pool, 128, rows, 256, 64, uint32_t(box), true)) {
    set_error("decode_attention: cuTensorMapEncodeTiled failed (pool pointer must be 16-byte aligned)");
    return cudaErrorInvalidValue;
  }
  AttnArgs a{};
  a.q = r.q;
  a.bt = r.block_table;
  a.max_blocks = r.max_blocks;
  a.bs = r.block_size;
  a.num_blocks = r.num_blocks;
  a.max_span = r.max_span;
  a.box_rows = box;
  a.err = r.err;
  a.spans = r.spans;
  a.span_add = r.span_add;
  a.window = r.window;
  a.lanes = r.lanes;
  a.n_kv = r.n_kv;
  a.max_chunks = chunks;
  a.part = w.part;
  a.counters = w.counters;
  a.out = r.out;
  a.out_f16 = r.out_f16 ? 1 : 0;
  a.early_meta = (r.early_meta && r.pdl) ? 1 : 0;
  {
    // TTS_ATTN_MERGE_LAST=0: every split pair merged by the epilogue warp (A/B)
    const char* e = getenv("TTS_ATTN_MERGE_LAST");
    a.merge_last = (e && *e == '0') ? 0 : 1;
  }
  a.pf = r.next;

  int dev = 0;
  cudaGetDevice(&dev);
  const size_t smem = sizeof(AttnSmem) + 1024;
  {
    static std::mutex mu;
    static bool done[64] = {false};
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !done[dev]) {
      cudaFuncSetAttribute(attn_decode_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      cudaFuncSetAttribute(attn_decode_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      cudaFuncSetAttribute(attn_decode_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      cudaFuncSetAttribute(attn_decode_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      done[dev] = true;
    }
  }
  const long long items = (long long)r.lanes * r.n_kv * chunks;
  const int grid = int(std::min<long long>(num_sms(dev), items));
  if ((items + 1) * grid >= (1ll << 31)) {  // the work split's 32-bit arithmetic
    set_error("decode_attention: lanes x kv heads x chunks too large for one call");
    return cudaErrorInvalidValue;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = r.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  switch (r.gqa) {
    case 1: return cudaLaunchKernelEx(&cfg, attn_decode_kernel<1>, tmK, tmV, a);
    case 2: return cudaLaunchKernelEx(&cfg, attn_decode_kernel<2>, tmK, tmV, a);
    case 4: return cudaLaunchKernelEx(&cfg, attn_decode_kernel<4>, tmK, tmV, a);
    default: return cudaLaunchKernelEx(&cfg, attn_decode_kernel<8>, tmK, tmV, a);
  }
}

size_t attn_static_part_limit() { return kStaticPartBytes; }
int attn_static_counter_limit() { return kStaticCounters; }
cudaError_t attn_static_base(void** base);

cudaError_t launch_attn_static(const AttnRequest& r, cudaStream_t st) {
  // every refusal is decided here, before anything is launched, and named after this op
  std::string why = attn_shape_error(r);
  if (why.empty() && (attn_part_bytes(r.lanes, r.n_kv, r.gqa, r.max_span) > kStaticPartBytes ||
                      r.lanes * r.n_kv > kStaticCounters))
    why = "lanes x kv heads x chunks of max_span need " +
          std::to_string(attn_part_bytes(r.lanes, r.n_kv, r.gqa, r.max_span)) +
          " bytes of partials (limit " + std::to_string(kStaticPartBytes) +
          ") and lanes x kv heads <= " + std::to_string(kStaticCounters);
  if (!why.empty()) {
    set_error("decode_attention_static: " + why);
    return cudaErrorInvalidValue;
  }
  void* base = nullptr;
  cudaError_t e = attn_static_base(&base);
  if (e != cudaSuccess) return e;
  AttnWorkspace w;
  w.part = static_cast<float*>(base);
  w.part_bytes = kStaticPartBytes;
  unsigned char* status = static_cast<unsigned char*>(base) + kStaticPartBytes;
  w.counters = reinterpret_cast<unsigned*>(status + kStaticStatusBytes);
  w.n_counters = kStaticCounters;
  AttnRequest rr = r;
  rr.err = reinterpret_cast<int*>(status);
  // The status word and the counters must start at zero. A previous call leaves the counters at
  // zero, but one that was cut short (a bounded wait that gave up) may not; the status word
  // holds the previous call's flags. One clear covers both (they are adjacent).
  e = cudaMemsetAsync(status, 0, kStaticStatusBytes + size_t(r.lanes) * r.n_kv * sizeof(unsigned),
                      st);
  if (e != cudaSuccess) return e;
  return launch_attn(rr, w, st);
}

// The device address of the fixed array on the current device. The host-side name of a
// __device__ array is not a device address: it is resolved once per device, with that device
// current, and cached (a device reset invalidates the cache; the process must not reuse it).
cudaError_t attn_static_base(void** base) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) {
    set_error("decode_attention_static: device index out of range");
    return cudaErrorInvalidValue;
  }
  static std::mutex mu;
  static void* scratch[64] = {nullptr};
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
  *base = scratch[dev];
  return cudaSuccess;
}

// Reads the status word of the last static call on the current device (after `st` has run it).
cudaError_t attn_static_status(cudaStream_t st, int* flags) {
  void* base = nullptr;
  cudaError_t e = attn_static_base(&base);
  if (e != cudaSuccess) return e;
  int v = 0;
  e = cudaMemcpyAsync(&v, static_cast<unsigned char*>(base) + kStaticPartBytes, sizeof(int),
                      cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return e;
  *flags = v;
  return cudaSuccess;
}

}  // namespace tts
