// Decode-shaped projection GEMM on tcgen05: y[m, n] = x[m, k] . W[n, k]^T, f16 in, f32 acc.
//
// This is the B200 form of tts-nn's `Proj::Half` forward and its `gemm_skinny_f16` kernel
// (crates/tts-nn/src/lib.rs:510-533, crates/tts-nn/src/skinny.rs:155-165): m is the lane
// count (1..384), so the GEMM is a weight stream and HBM-bound below m ~ 260.
//
// Layout: the weight rows are the MMA's M operand (128 rows per tile) and the lanes are its
// N operand, so m = 48 wastes no tensor work. Each CTA owns one 128-row weight tile and a
// contiguous range of 64-deep K blocks (split-K sized so the grid fills the SMs once).
//   warp 0 lane 0  TMA producer: W tile (16 KB, 128B swizzle) + x tile per stage
//   warp 1 lane 0  MMA issuer: 4 x tcgen05.mma (K = 16) per stage into TMEM
//   all 4 warps    epilogue: TMEM -> this CTA's shared memory. The splits of one tile form a
//                  thread-block cluster; after a cluster barrier each CTA reduces a slice of
//                  the lanes by reading every split's partial over DSMEM in rank order
//                  (deterministic, no global scratch) and applies the fused epilogue.
// Weight loads for the first stages are issued before `griddepcontrol.wait`, so under
// programmatic dependent launch they overlap the previous kernel's tail; only the x loads,
// which read the previous kernel's output, wait.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "tts_common.cuh"
#include "tts_internal.h"
#include "gemm_epilogue.cuh"
#include "l2_prefetch.cuh"

namespace tts {

namespace {

constexpr int kTileM = 128;  // weight rows per CTA (= MMA M)
constexpr int kBlockK = 64;  // K per stage: one 128-byte swizzle row of f16
constexpr int kWBytes = kTileM * kBlockK * 2;

struct GemmArgs {
  int m, k, n;
  int kb_total, splits, tiles;
  int groups, ng;  // token groups (<= 2) and MMA N per group (multiple of 16, <= 256)
  int packed;      // W tensor map is the packed [tiles * kb * 128][64] view
  int stages;     // per pipeline
  int pipes;      // independent producer/MMA pipelines per CTA
  int acc_cols;   // TMEM columns per pipeline accumulator
  int tmem_cols;
  int epi;
  int* err;
  void* y;
  int ldy;
  QkRopeArgs qk;
  unsigned long long* keys;
  int vocab;
  int codebooks;
  PickRule pick;  // EPI_ARGMAX: the talker's pick rule (vocab == 0: none)
  L2Prefetch pf;  // the next GEMM's first weight blocks
  // deferred RMSNorm (GemmRequest): producer outputs, consumer row scales
  const float* norm_w;
  __half* norm_x16;
  float* ss_out;
  const float* ss_in;
  int ss_tiles;
  float ss_inv_dim, ss_eps;
  // Epilogue operands staged into shared memory by one bulk copy each, issued right after the
  // dependency wait so that they land during the main loop (their global round trips, slow
  // while the weight stream holds the memory system, otherwise stall the epilogue): the
  // row-scale partial sums [ss_tiles][m] and, for the QKV epilogue, the per-step row
  // operands (QkRopeArgs::rows_desc / rows_rope) and the two norm weights. 0: not staged.
  int ops_ss;     // bytes of row-scale sums (a multiple of 16)
  int ops_rows;   // 1: desc [m] int4 + rope [m][128] f32 + norms [256] f32
  int ops_bytes;  // all staged bytes
  int ops_inv;    // 1: each row's 1 / RMS computed once per CTA from the staged sums
  int dsmem_batch;  // 1: a row's split-K partials all requested before they are summed
};


constexpr int kThreads = 256;  // 8 warps: 0..3 producers, 4..7 MMA issuers + epilogue
// The staged epilogue operands start this far past the stage rings / partial tile (the
// barriers and the TMEM address sit in between).
constexpr uint32_t kOpsOffset = 1024;

// kPipe: the epilogue requests each batch's global operands (row-scale partial sums, residual
// rows, the QKV rows' positions, page numbers and RoPE rows) one batch ahead, so that their
// round trips overlap the previous batch's reduction and stores. Used where a warp reduces
// several batches of rows (hundreds of rows: the prefill); at decode sizes each warp has one or
// two batches and the plain form is used.
// kEpi: an epilogue kind compiled in, or -1 for every kind behind a runtime switch (the form
// launched: one body shared by every projection keeps its code in the instruction caches).
template <bool kPipe, int kEpi>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_decode_kernel(const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmX, const GemmArgs a) {
  const int epi = kEpi >= 0 ? kEpi : a.epi;
  [[maybe_unused]] const unsigned long long tl_entry = TTS_TL_NOW();
  [[maybe_unused]] unsigned long long tl_rel = 0, tl_a = 0, tl_b = 0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int tile = blockIdx.x;
  const int split = blockIdx.y;
  const int kb0 = split * a.kb_total / a.splits;
  const int kb1 = (split + 1) * a.kb_total / a.splits;
  const int nkb = kb1 - kb0;
  const uint32_t x_bytes = uint32_t(a.groups * a.ng * 128);
  const uint32_t stage_bytes = kWBytes + x_bytes;
  const int P = a.pipes, SP = a.stages;  // pipelines and stages per pipeline

  // P stage rings, reused after the main loop for the partial tile [m][128] f32; then barriers
  const uint32_t body =
      max(uint32_t(P * SP) * stage_bytes, uint32_t(a.m) * kTileM * 4u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + body);  // [P][SP]
  uint64_t* empty = full + P * SP;                              // [P][SP]
  uint64_t* done = empty + P * SP;
  uint64_t* ops_bar = done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ops_bar + 1);
  // the staged epilogue operands (GemmArgs::ops_*), past the barriers
  uint8_t* ops = smem + body + kOpsOffset;
  const float* ss_s = reinterpret_cast<const float*>(ops);
  const int4* desc_s = reinterpret_cast<const int4*>(ops + a.ops_ss);
  const float* rope_s = reinterpret_cast<const float*>(ops + a.ops_ss + a.m * 16);
  const float* norms_s = rope_s + a.m * 128;
  // each token row's 1 / RMS of the deferred norm (consumers with staged sums), past the
  // staged operands
  float* inv_s = reinterpret_cast<float*>(ops + a.ops_bytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P * SP; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, P);
    mbar_init(ops_bar, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 4) {
    tmem_alloc(tmem_slot, a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_launch_dependents();

  // Pipeline p streams k-blocks kb0 + p, kb0 + p + P, ... through its own SP stages into its
  // own TMEM accumulator: P independent producer/MMA handshakes keep loads and MMAs
  // overlapped (one pipeline alone serialises load latency and MMA latency per k-block).
  if (warp < 4) {
    const int pp = warp;
    if (pp < P) {
      // ---------------- TMA producer of pipeline pp (converged warp, one elected lane issues)
      const uint64_t pol_w = l2_policy_evict_first();
      const int cnt = nkb > pp ? (nkb - pp + P - 1) / P : 0;  // k-blocks of this pipeline
      const int pre = cnt < SP ? cnt : SP;
      uint8_t* ring = smem + size_t(pp) * SP * stage_bytes;
      uint64_t* fl = full + pp * SP;
      uint64_t* em = empty + pp * SP;
      auto w_x = [&](int kb) { return a.packed ? 0 : kb * kBlockK; };
      auto w_y = [&](int kb) { return a.packed ? (tile * a.kb_total + kb) * kTileM : tile * kTileM; };
      if (elect_one()) {
        for (int i = 0; i < pre; ++i) {
          const int kb = kb0 + pp + i * P;
          mbar_arrive_expect_tx(&fl[i], stage_bytes);
          tma_load_2d_hint(ring + i * stage_bytes, &tmW, &fl[i], w_x(kb), w_y(kb), pol_w);
        }
      }
      __syncwarp();
      pdl_wait();  // x is the previous kernel's output
      if (pp == 0) tl_rel = TTS_TL_NOW();
      if (elect_one()) {
        for (int i = 0; i < pre; ++i) {
          const int kb = kb0 + pp + i * P;
          uint8_t* st = ring + i * stage_bytes + kWBytes;
          for (int g = 0; g < a.groups; ++g)
            tma_load_2d(st + g * a.ng * 128, &tmX, &fl[i], kb * kBlockK, g * a.ng);
        }
        if (pp == 0 && a.ops_bytes) {
          // the epilogue's operands: written by earlier kernels, complete once the wait
          // returned; they arrive while the weights stream
          mbar_arrive_expect_tx(ops_bar, uint32_t(a.ops_bytes));
          if (a.ops_ss) bulk_load(ops, a.ss_in, uint32_t(a.ops_ss), ops_bar);
          if (a.ops_rows) {
            bulk_load(ops + a.ops_ss, a.qk.rows_desc, uint32_t(a.m) * 16u, ops_bar);
            bulk_load(ops + a.ops_ss + a.m * 16, a.qk.rows_rope, uint32_t(a.m) * 512u, ops_bar);
            bulk_load(ops + a.ops_ss + a.m * 16 + a.m * 512, a.qk.norms, 1024u, ops_bar);
          }
        }
      }
      __syncwarp();
      // ring slot and phase of k-block i as running counters (no division by the run-time SP)
      int s = pre % SP;
      uint32_t ph = uint32_t(pre / SP) & 1u;
      for (int i = pre; i < cnt; ++i) {
        if (!mbar_wait_warp(&em[s], ph ^ 1u)) {
          if (lane == 0) atomicOr(a.err, 1);
          break;
        }
        if (elect_one()) {
          const int kb = kb0 + pp + i * P;
          uint8_t* st = ring + s * stage_bytes;
          mbar_arrive_expect_tx(&fl[s], stage_bytes);
          tma_load_2d_hint(st, &tmW, &fl[s], w_x(kb), w_y(kb), pol_w);
          for (int g = 0; g < a.groups; ++g)
            tma_load_2d(st + kWBytes + g * a.ng * 128, &tmX, &fl[s], kb * kBlockK, g * a.ng);
        }
        __syncwarp();
        if (++s == SP) {
          s = 0;
          ph ^= 1u;
        }
      }
      // this pipeline's weights are all requested: start on the next GEMM's
      if (pp == 0 && elect_one())
        issue_l2_prefetch(a.pf, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
      __syncwarp();
    }
  } else {
    const int pp = warp - 4;
    if (pp < P) {
      // ---------------- MMA issuer of pipeline pp (converged warp, one elected lane issues)
      const uint32_t idesc = idesc_f16_f32(kTileM, a.ng);
      const int cnt = nkb > pp ? (nkb - pp + P - 1) / P : 0;
      uint8_t* ring = smem + size_t(pp) * SP * stage_bytes;
      uint64_t* fl = full + pp * SP;
      uint64_t* em = empty + pp * SP;
      const uint32_t acc = tmem + uint32_t(pp * a.acc_cols);
      int s = 0;  // ring slot and phase of k-block i
      uint32_t ph = 0;
      for (int i = 0; i < cnt; ++i) {
        if (!mbar_wait_warp(&fl[s], ph)) {
          if (lane == 0) atomicOr(a.err, 2);
          break;
        }
        tc_fence_after();
        if (elect_one()) {
          const uint32_t wa = smem_u32(ring + s * stage_bytes);
          const uint32_t xa = wa + kWBytes;
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk) {
            const uint64_t ad = desc_k_sw128(wa + kk * 32);
            for (int g = 0; g < a.groups; ++g) {
              const uint64_t bd = desc_k_sw128(xa + g * a.ng * 128 + kk * 32);
              umma_f16(acc + g * a.ng, ad, bd, idesc, (i | kk) != 0);
            }
          }
          umma_commit(&em[s]);
        }
        __syncwarp();
        if (++s == SP) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (elect_one()) umma_commit(done);  // no MMA issued: arrives at once (zero partial)
      __syncwarp();
    }
  }

  // ---------------- epilogue: sum the pipelines' accumulators (pipeline order) into this
  // CTA's partial tile in shared memory. Warps 4..7 own TMEM lane quadrants 0..3.
  const bool ok = mbar_wait(done, 0);
  if (!ok && threadIdx.x == 128) atomicOr(a.err, 4);
  tc_fence_after();
  [[maybe_unused]] const unsigned long long tl_main = TTS_TL_NOW();
  // The producers waited for the previous kernel before loading x, so this returns at once;
  // the residual rows this thread will add are read now, behind the TMEM and cluster steps.
  pdl_wait();
  const int S = a.splits;
  const uint32_t rank = S > 1 ? cluster_rank() : 0u;
  constexpr int nw = kThreads / 32;
  const int stride = nw * S;
  const int j_first = int(rank) + S * warp;
  float4 res_pre[4];
  if (epi == EPI_RESIDUAL) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = j_first + u * stride;
      res_pre[u] = j < a.m ? *reinterpret_cast<const float4*>(static_cast<float*>(a.y) +
                                                              (size_t)j * a.ldy + tile * kTileM +
                                                              4 * lane)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  // staged operands: every thread waits for their bulk copies (long landed by now)
  if (a.ops_bytes && !mbar_wait(ops_bar, 0) && threadIdx.x == 0) atomicOr(a.err, 4);
  // Deferred norm, consumer side: each token row's 1 / RMS once, one thread per row, summing
  // the staged per-tile sums of squares in tile order, while warps 4-7 drain the accumulators
  // (the barrier below publishes them).
  if (a.ops_inv && warp < 4) {
    for (int j = threadIdx.x; j < a.m; j += 128) {
      float t = 0.f;
      for (int q = 0; q < a.ss_tiles; ++q) t += ss_s[q * a.m + j];
      inv_s[j] = 1.f / sqrtf(t * a.ss_inv_dim + a.ss_eps);
    }
  }
  // Every TMA load was consumed by an MMA and every MMA has completed, so the stage buffers
  // are free: the partial tile [m][128] f32 reuses them.
  float* red = reinterpret_cast<float*>(smem);
  if (warp >= 4) {
    const int q = warp - 4;
    const int row = q * 32 + lane;
    const uint32_t lane_addr = tmem + (uint32_t(q * 32) << 16);
    // a pipeline that issued nothing holds no accumulator
    bool has[4];
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) has[pp] = pp < P && nkb > pp;
    for (int c0 = 0; c0 < a.m; c0 += 16) {
      // the same 16 columns of all four accumulators behind one wait (a pipeline beyond P
      // re-reads pipeline 0 and is ignored)
      float v[4][16];
      tmem_ld16x4(lane_addr + c0, lane_addr + uint32_t((P > 1 ? 1 : 0) * a.acc_cols) + c0,
                  lane_addr + uint32_t((P > 2 ? 2 : 0) * a.acc_cols) + c0,
                  lane_addr + uint32_t((P > 3 ? 3 : 0) * a.acc_cols) + c0, v);
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        float sum = has[0] ? v[0][jj] : 0.f;
#pragma unroll
        for (int pp = 1; pp < 4; ++pp)
          if (has[pp]) sum += v[pp][jj];
        const int j = c0 + jj;
        if (j < a.m) red[j * kTileM + row] = sum;
      }
    }
  }
  tc_fence_before();
  if (S > 1)
    cluster_sync();
  else
    __syncthreads();
  [[maybe_unused]] const unsigned long long tl_red = TTS_TL_NOW();
  if (warp == 4) tmem_dealloc(tmem, a.tmem_cols);

  // ---------------- reduce this CTA's rows across the cluster, in rank order. Rows go four at a
  // time: all their loads (and any residual reads) are issued before the first store.
  // deferred norm, producer side: this lane's 4 columns of the next norm's weight
  const float4 nw4 = a.norm_w ? *reinterpret_cast<const float4*>(a.norm_w + tile * kTileM + 4 * lane)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
  // the split-K sum of one batch of rows (S partials over DSMEM in rank order), scaled by the
  // deferred norm's 1/RMS when the row-scale partial sums are given
  auto reduce_batch = [&](const int (&jr)[4], const float (&ssp)[4], float4 (&acc4)[4]) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = jr[u];
      acc4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (j >= a.m) continue;
      const float* src = red + j * kTileM + 4 * lane;
      if (S == 1) {
        acc4[u] = *reinterpret_cast<const float4*>(src);
      } else if (!a.dsmem_batch) {
        acc4[u] = ld_dsmem_f4(src, 0);
        for (int r = 1; r < S; ++r) {
          const float4 p = ld_dsmem_f4(src, r);
          acc4[u].x += p.x;
          acc4[u].y += p.y;
          acc4[u].z += p.z;
          acc4[u].w += p.w;
        }
      } else {
        // every rank's partial requested before the first add (their DSMEM round trips
        // overlap), then summed in rank order
        float4 p[8];
#pragma unroll
        for (int r = 0; r < 8; ++r)
          if (r < S) p[r] = ld_dsmem_f4(src, r);
        acc4[u] = p[0];
#pragma unroll
        for (int r = 1; r < 8; ++r)
          if (r < S) {
            acc4[u].x += p[r].x;
            acc4[u].y += p[r].y;
            acc4[u].z += p[r].z;
            acc4[u].w += p[r].w;
          }
      }
      if (a.ss_in) {
        // j is uniform across the warp: every lane takes this branch together
        const float inv = a.ops_inv ? inv_s[j]
                                    : 1.f / sqrtf(warp_sum(ssp[u]) * a.ss_inv_dim + a.ss_eps);
        acc4[u].x *= inv;
        acc4[u].y *= inv;
        acc4[u].z *= inv;
        acc4[u].w *= inv;
      }
    }
  };
  // y[j] = res[j] + acc[j] for a batch, and the next norm's input and sums of squares
  auto residual_batch = [&](const int (&jr)[4], const float4 (&res)[4], const float4 (&acc4)[4]) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = jr[u];
      if (j >= a.m) continue;
      float4 r = res[u];
      r.x += acc4[u].x;
      r.y += acc4[u].y;
      r.z += acc4[u].z;
      r.w += acc4[u].w;
      *reinterpret_cast<float4*>(static_cast<float*>(a.y) + (size_t)j * a.ldy + tile * kTileM +
                                 4 * lane) = r;
      if (a.norm_w) {
        __half2* d = reinterpret_cast<__half2*>(a.norm_x16 + (size_t)j * a.n + tile * kTileM +
                                                4 * lane);
        d[0] = __floats2half2_rn(r.x * nw4.x, r.y * nw4.y);
        d[1] = __floats2half2_rn(r.z * nw4.z, r.w * nw4.w);
        const float ss = warp_sum(r.x * r.x + r.y * r.y + r.z * r.z + r.w * r.w);
        if (lane == 0) a.ss_out[(size_t)tile * a.m + j] = ss;
      }
    }
  };
  auto batch_rows = [&](int j0, int (&jr)[4]) {
    int n = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      jr[u] = j0 + u * stride;
      if (jr[u] < a.m) n = u + 1;
    }
    return n;
  };
  auto fetch_ss = [&](const int (&jr)[4], float (&d)[4]) {
#pragma unroll
    for (int u = 0; u < 4; ++u)
      d[u] = a.ss_in && !a.ops_inv && jr[u] < a.m && lane < a.ss_tiles
                 ? (a.ops_ss ? ss_s[lane * a.m + jr[u]] : __ldcg(a.ss_in + (size_t)lane * a.m + jr[u]))
                 : 0.f;
  };
  if constexpr (kPipe) {
    // batch b + 1's operands are requested before batch b's reduction (positions) and before
    // its stores (page numbers, RoPE rows, which need the positions)
    int jn[4];
    int nn = batch_rows(j_first, jn);
    float ssn[4];
    float4 resn[4];
    QkRowsPre qkn;
    fetch_ss(jn, ssn);
#pragma unroll
    for (int u = 0; u < 4; ++u) resn[u] = res_pre[u];  // read before the reduction
    if (epi == EPI_QKROPE) {
      qkrope_fetch_pos4(a.qk, jn, nn, qkn);
      qkrope_fetch_rest4(a.qk, tile, jn, nn, lane, qkn);
    }
    for (int j0 = j_first; j0 < a.m; j0 += 4 * stride) {
      int jc[4];
      float ssc[4];
      float4 resc[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        jc[u] = jn[u];
        ssc[u] = ssn[u];
        resc[u] = resn[u];
      }
      const int nc = nn;
      const QkRowsPre qkc = qkn;
      nn = batch_rows(j0 + 4 * stride, jn);
      if (nn) {
        fetch_ss(jn, ssn);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          resn[u] = epi == EPI_RESIDUAL && u < nn
                        ? __ldcg(reinterpret_cast<const float4*>(static_cast<float*>(a.y) +
                                                                 (size_t)jn[u] * a.ldy +
                                                                 tile * kTileM + 4 * lane))
                        : make_float4(0.f, 0.f, 0.f, 0.f);
        if (epi == EPI_QKROPE) qkrope_fetch_pos4(a.qk, jn, nn, qkn);
      }
      float4 acc4[4];
      reduce_batch(jc, ssc, acc4);
      if (nn && epi == EPI_QKROPE) qkrope_fetch_rest4(a.qk, tile, jn, nn, lane, qkn);
      if (epi == EPI_RESIDUAL) {
        residual_batch(jc, resc, acc4);
      } else if (epi == EPI_QKROPE) {
        float v[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          v[u][0] = acc4[u].x;
          v[u][1] = acc4[u].y;
          v[u][2] = acc4[u].z;
          v[u][3] = acc4[u].w;
        }
        qkrope_apply4(a.qk, tile, jc, nc, lane, v, qkc);
      } else {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (jc[u] < a.m) epilogue_row(a, tile, jc[u], lane, acc4[u], epi);
      }
    }
  } else {
    for (int j0 = j_first; j0 < a.m; j0 += 4 * stride) {
      int jc[4];
      batch_rows(j0, jc);
      // lane t < ss_tiles loads tile t's partial sum of squares of each row, ahead of the
      // DSMEM reads (the previous kernel wrote them: L2 reads)
      float ssp[4];
      fetch_ss(jc, ssp);
      float4 acc4[4];
      reduce_batch(jc, ssp, acc4);
#ifdef TTS_TIMELINE
      if (j0 == j_first) tl_a = TTS_TL_NOW();
#endif
      if (epi == EPI_RESIDUAL) {
        float4 res[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = jc[u];
          if (j0 == j_first)
            res[u] = res_pre[u];  // read before the reduction
          else
            res[u] = j < a.m ? *reinterpret_cast<const float4*>(static_cast<float*>(a.y) +
                                                                (size_t)j * a.ldy +
                                                                tile * kTileM + 4 * lane)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        residual_batch(jc, res, acc4);
      } else if (epi == EPI_QKROPE && a.ops_rows) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (jc[u] < a.m) {
            float v[4] = {acc4[u].x, acc4[u].y, acc4[u].z, acc4[u].w};
            qkrope_row_staged(a.qk, tile, jc[u], lane, v, desc_s[jc[u]],
                              rope_s + (size_t)jc[u] * 128, norms_s);
          }
      } else {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (jc[u] < a.m) epilogue_row(a, tile, jc[u], lane, acc4[u], epi);
      }
    }
  }
#ifdef TTS_TIMELINE
  tl_b = TTS_TL_NOW();
#endif
  if (S > 1) cluster_sync();  // no CTA leaves while another may still read its shared memory
#ifdef TTS_TIMELINE
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t_end = TTS_TL_NOW();
    const int k = kTlGemm | (epi << 4);
    timeline_recs<7>({k | kTlEntry, k | kTlReleased, k | kTlMainDone, k | kTlReduced, k | kTlEnd,
                      k | kTlEpiFirst, k | kTlEpiLoop},
                     {tl_entry, tl_rel, tl_main, tl_red, t_end, tl_a, tl_b});
  }
#endif
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct Plan {
  int groups, ng, stages, pipes, acc_cols, splits, tmem_cols;
  size_t smem;
};

int env_int(const char* name, int fallback) {
  const char* v = getenv(name);
  if (!v || !*v) return fallback;
  return atoi(v);
}

// Clusters of `splits` CTAs that can be resident at once for this shared-memory size, cached
// per (device, splits, smem). 0 when the query fails.
int max_active_clusters(int device, int splits, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, size_t>, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_tuple(device, splits, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  cudaFuncSetAttribute(gemm_decode_kernel<false, -1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       227 * 1024);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1, splits, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = splits;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_decode_kernel<false, -1>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache[key] = n;
  return n;
}

// CTAs of the plain decode GEMM that fit on one SM with `smem` bytes of shared memory (its
// registers decide as much as its shared memory), cached per (device, smem).
int ctas_per_sm(int device, size_t smem) {
  static std::mutex mu;
  static std::map<std::pair<int, size_t>, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(device, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  cudaFuncSetAttribute(gemm_decode_kernel<false, -1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       227 * 1024);
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemm_decode_kernel<false, -1>, kThreads,
                                                    smem) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache[key] = n;
  return n;
}

// Tile plan for y[m, n] = x[m, k] W[n, k]^T. The grid is one wave: every CTA (and every
// cluster of split-K CTAs) resident at once, so no tile waits for a second wave.
// TTS_GEMM_STAGES / TTS_GEMM_SPLITS override the choice for A/B measurement.
Plan plan_gemm(int m, int k, int n, int device, int force_splits) {
  Plan p{};
  const int pad = std::max(16, (m + 15) / 16 * 16);
  p.groups = (pad + 255) / 256;
  p.ng = ((pad + p.groups - 1) / p.groups + 15) / 16 * 16;
  const int cols = p.groups * p.ng;
  p.acc_cols = 32;
  while (p.acc_cols < cols) p.acc_cols *= 2;
  // up to 4 pipelines, each with its own TMEM accumulator (512 columns in all)
  p.pipes = std::max(1, std::min(4, 512 / p.acc_cols));
  p.pipes = std::max(1, std::min(4, env_int("TTS_GEMM_PIPES", p.pipes)));
  while (p.pipes > 1 && p.pipes * p.acc_cols > 512) --p.pipes;
  p.tmem_cols = 32;
  while (p.tmem_cols < p.pipes * p.acc_cols) p.tmem_cols *= 2;
  const int stage = kWBytes + cols * 128;
  const int tiles = n / kTileM;
  const int sms = num_sms(device);
  // Many tiles (the heads): two CTAs per SM with one stage per pipeline, where two fit (at
  // decode sizes the kernel's registers allow one CTA per SM: then the tiles run in waves of
  // one CTA per SM, each with deeper rings). Otherwise one CTA per SM with as many stages as
  // 216 KB of rings hold (two per pipeline at decode sizes; three of 72 KB for 448 rows, whose
  // single pipeline otherwise waits on each stage's load).
  const bool two = tiles > sms && ctas_per_sm(device, size_t(100 + 2) * 1024) >= 2;
  const int budget = two ? 100 * 1024 : 216 * 1024;
  p.stages = std::max(1, std::min(4, budget / (stage * p.pipes)));
  p.stages = std::max(1, std::min(8, env_int("TTS_GEMM_STAGES", p.stages)));
  while (p.stages > 1 && size_t(p.stages) * p.pipes * stage > 216 * 1024) --p.stages;
  while (p.pipes > 1 && size_t(p.stages) * p.pipes * stage > 216 * 1024) --p.pipes;
  const size_t red = size_t(m) * kTileM * sizeof(float);
  const size_t rings = size_t(p.stages) * p.pipes * stage;
  p.smem = std::max(rings, red) + 1024 + 512;

  const int kb = k / kBlockK;
  int s = 1;
  for (int c = std::min(8, kb); c >= 2; --c) {
    if (tiles * c > sms) continue;
    if (max_active_clusters(device, c, p.smem) < tiles) continue;
    s = c;
    break;
  }
  const int fs = force_splits > 0 ? force_splits : env_int("TTS_GEMM_SPLITS", 0);
  if (fs > 0) s = std::min(std::min(fs, 8), kb);
  p.splits = s;
  return p;
}

}  // namespace

bool make_tmap_2d_f16(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                      bool swizzle128) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool gemm_supported(int m, int k, int n, int epi, std::string* why) {
  auto no = [&](const char* s) {
    if (why) *why = s;
    return false;
  };
  // the split-K partial tile [m][128] f32 lives in shared memory: 448 rows fit in 227 KB
  if (m < 1 || m > kMaxGemmRows) return no("lanes (m) must be in 1..448");
  if (k < kBlockK || k % kBlockK) return no("k must be a positive multiple of 64");
  if (n < kTileM || n % kTileM) return no("n must be a positive multiple of 128");
  if (epi < EPI_F32 || epi > EPI_ARGMAX) return no("unknown epilogue");
  return true;
}

L2Prefetch gemm_prefetch_plan(const void* w_packed, int m, int k, int n, int device,
                              size_t budget) {
  L2Prefetch pf;
  if (!w_packed || !gemm_supported(m, k, n, EPI_F32, nullptr)) return pf;
  const Plan p = plan_gemm(m, k, n, device, 0);
  pf.w = static_cast<const __half*>(w_packed);
  pf.tiles = n / kTileM;
  pf.kb_total = k / kBlockK;
  pf.splits = p.splits;
  const size_t heads = size_t(pf.tiles) * pf.splits * kWBytes;  // one block per range
  const int per_range = pf.kb_total / pf.splits;
  pf.depth = int(std::max<size_t>(1, budget / heads));
  // no deeper than what the next GEMM's pipelines request at once, nor its range
  pf.depth = std::min(pf.depth, std::min(per_range, p.pipes * p.stages));
  return pf;
}

cudaError_t launch_gemm(const GemmRequest& r, const Workspace& wsp, cudaStream_t st, int device) {
  std::string why;
  if (!gemm_supported(r.m, r.k, r.n, r.epi, &why)) {
    set_error("proj: " + why);
    return cudaErrorInvalidValue;
  }
  const Plan p = plan_gemm(r.m, r.k, r.n, device, r.force_splits);
  const int tiles = r.n / kTileM;
  if (p.smem > 227 * 1024) {
    set_error("proj: shared-memory plan exceeds 227 KB for this lane count");
    return cudaErrorInvalidValue;
  }
  if ((r.norm_w && (r.epi != EPI_RESIDUAL || !r.norm_x16 || !r.ss_out)) ||
      (r.ss_in && (r.ss_tiles < 1 || r.ss_tiles > 32 || r.ss_dim < 1))) {
    set_error("proj: deferred norm needs EPI_RESIDUAL with x16 and ss outputs, 1..32 ss tiles");
    return cudaErrorInvalidValue;
  }
  CUtensorMap tmW, tmX;
  const bool wmap_ok =
      r.packed ? make_tmap_2d_f16(&tmW, r.w, kBlockK, uint64_t(r.n) / kTileM * (r.k / kBlockK) * kTileM,
                                  kBlockK * 2, kBlockK, kTileM, true)
               : make_tmap_2d_f16(&tmW, r.w, r.k, r.n, uint64_t(r.k) * 2, kBlockK, kTileM, true);
  if (!wmap_ok ||
      !make_tmap_2d_f16(&tmX, r.x, r.k, r.m, uint64_t(r.k) * 2, kBlockK, p.ng, true)) {
    set_error("proj: cuTensorMapEncodeTiled failed (pointers must be 16-byte aligned)");
    return cudaErrorInvalidValue;
  }
  GemmArgs a{};
  a.m = r.m;
  a.k = r.k;
  a.n = r.n;
  a.kb_total = r.k / kBlockK;
  a.splits = p.splits;
  a.tiles = tiles;
  a.groups = p.groups;
  a.ng = p.ng;
  a.packed = r.packed ? 1 : 0;
  a.stages = p.stages;
  a.pipes = p.pipes;
  a.acc_cols = p.acc_cols;
  a.tmem_cols = p.tmem_cols;
  a.epi = r.epi;
  a.err = wsp.err;
  a.y = r.y;
  a.ldy = r.ldy > 0 ? r.ldy : (r.epi == EPI_SWIGLU ? r.n / 2 : r.n);
  a.qk = r.qk;
  a.keys = r.argmax_keys;
  a.vocab = r.vocab;
  a.codebooks = r.vocab > 0 ? r.n / r.vocab : 0;
  a.pick = r.pick;
  a.pf = r.next;
  a.norm_w = r.norm_w;
  a.norm_x16 = r.norm_x16;
  a.ss_out = r.ss_out;
  a.ss_in = r.ss_in;
  a.ss_tiles = r.ss_tiles;
  a.ss_inv_dim = r.ss_dim > 0 ? 1.f / float(r.ss_dim) : 0.f;
  a.ss_eps = r.ss_eps;
  // Stage the epilogue's global operands (GemmArgs::ops_*) where the decode epilogue (the
  // plain form) reads them, every source is 16-byte aligned, and the extra shared memory
  // leaves the CTAs per SM unchanged. TTS_GEMM_STAGE_OPS=0 turns it off (A/B).
  size_t smem = p.smem;
  {
    static const int stage_on = env_int("TTS_GEMM_STAGE_OPS", 1);
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    static const int pipe_rows_s = env_int("TTS_GEMM_PIPE_ROWS", 129);
    const bool plain = r.m < pipe_rows_s;
    int ss_b = 0, rows = 0;
    if (stage_on && plain && r.ss_in && al16(r.ss_in))
      ss_b = (r.ss_tiles * r.m * 4 + 15) / 16 * 16;
    if (stage_on && plain && r.epi == EPI_QKROPE && r.qk.rows_desc && r.qk.rows_rope &&
        al16(r.qk.rows_desc) && al16(r.qk.rows_rope) && al16(r.qk.norms))
      rows = 1;
    const int bytes = ss_b + (rows ? r.m * 16 + r.m * 512 + 1024 : 0);
    const int inv_b = ss_b ? (r.m * 4 + 15) / 16 * 16 : 0;  // the rows' 1 / RMS
    const size_t with = p.smem - 512 + kOpsOffset + size_t(bytes) + size_t(inv_b);
    const size_t one_cta = 114 * 1024;  // above this, one CTA per SM either way
    if (bytes > 0 && with <= 227 * 1024 && (p.smem > one_cta || with <= one_cta)) {
      a.ops_ss = ss_b;
      a.ops_rows = rows;
      a.ops_bytes = bytes;
      static const int inv_on = env_int("TTS_GEMM_ROW_INV", 1);
      a.ops_inv = (ss_b && inv_on) ? 1 : 0;
      smem = with;
    }
  }
  static const int dsmem_batch = env_int("TTS_GEMM_DSMEM_BATCH", 1);
  a.dsmem_batch = dsmem_batch;

  {
    // The opt-in shared-memory limit is a per-device function attribute.
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !done[dev]) {
      for (auto fn : {gemm_decode_kernel<false, -1>, gemm_decode_kernel<true, -1>})
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      done[dev] = true;
    }
  }

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(tiles, p.splits, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = r.pdl ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = p.splits;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.splits > 1 ? 2 : 1;
  // the look-ahead epilogue where a warp reduces more than two batches of rows (the prefill's
  // hundreds of rows); TTS_GEMM_PIPE_ROWS overrides the row threshold for A/B measurement
  static const int pipe_rows = env_int("TTS_GEMM_PIPE_ROWS", 129);
  if (r.m >= pipe_rows) return cudaLaunchKernelEx(&cfg, gemm_decode_kernel<true, -1>, tmW, tmX, a);
  // One kernel body for every epilogue kind: the decode step's four projections then run the
  // same instructions, which stay in the instruction caches from one projection to the next
  // (kernels specialised per kind measured 2.18 against 2.06 ms per step).
  return cudaLaunchKernelEx(&cfg, gemm_decode_kernel<false, -1>, tmW, tmX, a);
}

}  // namespace tts
