// The layer chain: a run of decode projections (and the RMS norms between them) as one
// persistent kernel, for lane counts up to 128.
//
// Each GEMM phase is y[m, n] = x[m, k] W[n, k]^T over packed weights (128-row tiles, 64-wide
// k-blocks), with the decode GEMM's fused epilogues (crates/tts-nn/src/skinny.rs:155-165 and
// lib.rs:510-533 for the projection; qwen3.rs:339-463 for the layer order). Its (tile, k-block)
// units are split into equal contiguous ranges, one per CTA (one CTA per SM), so every SM
// streams the same share of the weights whatever the tile count. A tile whose k-range spans
// several CTAs is reduced through global memory: each owner publishes an f32 partial (and
// counts its k-blocks) without waiting; once all have arrived, each owner sums every partial
// in k order for its own slice of the token rows and runs the epilogue on that slice, so the
// reduction is spread over the owners and results are deterministic. A NORM phase normalises the rows of the residual stream into the
// next phase's f16 input (qwen3.rs:339-341, 453-455).
//
// Phases are ordered by device-side counters: a phase's x (or a norm's input) is read only once
// every tile (row) of the phase before it is complete. Weights do not depend on earlier phases,
// so the loader streams the next phase's weights into its ring while the epilogue warps finish
// the current one: the HBM is not left idle between projections the way it is between
// separate kernels. Roles per CTA: warp 0 loads (TMA), warp 1 issues the MMAs (tcgen05, two
// TMEM accumulators so one segment's epilogue overlaps the next segment's MMAs), warps 2-5 run
// the epilogues and norms. Every wait is bounded (2 s) and reports through the error flags.
#include <algorithm>
#include <mutex>

#include "gemm_epilogue.cuh"
#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

namespace {

constexpr int kTileM = 128;
constexpr int kBlockK = 64;
constexpr uint32_t kWBytes = kTileM * kBlockK * 2;
constexpr int kThreads = 192;
constexpr int kLoadWarp = 0, kMmaWarp = 1;
constexpr int kEpiThreads = 128;  // warps 2..5
constexpr uint32_t kBarEpi = 1;
constexpr int kMaxStages = 8;
constexpr int kMaxSegments = 56;  // owners of one tile's k-range (flags[2..57])

struct Phase {
  int kind;  // CHAIN_GEMM or CHAIN_NORM
  // GEMM: geometry and the fields epilogue_row reads
  int n, k, tiles, kb_total, units;
  int epi;
  void* y;
  int ldy;
  QkRopeArgs qk;
  unsigned long long* keys;
  int vocab, codebooks;
  PickRule pick;
  // NORM: y16[r] = src[r] / rms(src[r]) * w, optionally y32 too; zeroes keys[0, n_keys)
  const float* src;
  const float* w;
  __half* dst16;
  float* dst32;
  unsigned long long* zero_keys;
  int n_keys;
};

struct ChainArgs {
  int m, dim;
  float eps;
  int nph;
  int ng;        // MMA N (tokens padded to 16)
  int acc_cols;  // TMEM columns per accumulator
  int stages;
  Phase ph[kMaxChainPhases];
  unsigned long long* done;  // [kMaxChainPhases] rows completed per phase (tiles x m for GEMM)
  unsigned* exit_cnt;
  unsigned* tile_cnt;        // [2][kMaxChainPhases][max_tiles] k-blocks arrived / owners done
  int max_tiles;
  float* part;               // [kMaxChainPhases][grid][2][m][128] f32 partial tiles
  int* err;
};

struct ChainMaps {
  CUtensorMap w[kMaxChainPhases];
  CUtensorMap x[kMaxChainPhases];
};

TTS_DEV unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
TTS_DEV unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Phase p's input is ready: the phase before it has completed every tile (row). Phase 0 reads
// what earlier kernels wrote. With `block` false this only probes; blocking waits are bounded
// (false after ~2 s).
TTS_DEV bool phase_input_ready(const ChainArgs& a, int p, bool block) {
  if (p == 0) {
    if (!block) return false;  // probing does not wait for the previous kernel
    pdl_wait();
    return true;
  }
  const Phase& q = a.ph[p - 1];
  const unsigned long long target =
      (unsigned long long)a.m * (q.kind == CHAIN_NORM ? 1ull : (unsigned long long)q.tiles);
  if (ld_acquire_u64(&a.done[p - 1]) >= target) return true;
  if (!block) return false;
  const uint64_t t0 = global_ns();
  while (ld_acquire_u64(&a.done[p - 1]) < target) {
    __nanosleep(64);
    if (global_ns() - t0 > 2000000000ull) return false;
  }
  return true;
}

TTS_DEV long long range_lo(long long units, int cta, int grid) { return units * cta / grid; }
// Which CTA owns unit x of a phase of `units` split as [units*i/grid, units*(i+1)/grid).
TTS_DEV int unit_owner(long long x, long long units, int grid) {
  return int(((x + 1) * grid + units - 1) / units) - 1;
}

__global__ void __launch_bounds__(kThreads, 1)
    chain_kernel(const __grid_constant__ ChainMaps maps, const ChainArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const int ST = a.stages;
  const uint32_t x_bytes = uint32_t(a.ng) * 128u;
  const uint32_t stage_bytes = kWBytes + x_bytes;
  float* red = reinterpret_cast<float*>(smem + size_t(ST) * stage_bytes);  // [m][128]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + size_t(a.m) * kTileM);
  uint64_t* empty = full + kMaxStages;
  uint64_t* acc_full = empty + kMaxStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] last arrival, [1..] fixup list
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);  // one arrival per epilogue warp
    }
    fence_barrier_init();
    for (int p = 0; p < a.nph; ++p)
      if (a.ph[p].kind == CHAIN_GEMM) {
        tma_prefetch_desc(&maps.w[p]);
        tma_prefetch_desc(&maps.x[p]);
      }
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, uint32_t(2 * a.acc_cols));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == kLoadWarp) {
    // ================= loader: weights run ahead of the phase barriers, x waits for them
    const uint64_t pol_w = l2_policy_evict_first();
    long long g = 0;  // units issued over all phases (ring position)
    bool pdl_done = false;
    for (int p = 0; p < a.nph && ok; ++p) {
      const Phase& ph = a.ph[p];
      if (ph.kind != CHAIN_GEMM) continue;
      const long long lo = range_lo(ph.units, cta, G), hi = range_lo(ph.units, cta + 1, G);
      bool xready = false;
      int npend = 0;
      int pend_s[kMaxStages], pend_kb[kMaxStages];
      auto issue_x = [&](int s, int kb) {
        if (elect_one())
          tma_load_2d(smem + size_t(s) * stage_bytes + kWBytes, &maps.x[p], &full[s], kb * kBlockK, 0);
        __syncwarp();
      };
      auto release = [&](bool block) {
        bool r = (p == 0 && pdl_done) ? true : false;
        if (!r && p == 0 && block) {
          pdl_wait();  // every lane: x of phase 0 is the previous kernel's output
          r = pdl_done = true;
        } else if (!r && p > 0) {
          int v = 0;
          if (lane == 0) v = phase_input_ready(a, p, block) ? 1 : 0;
          r = __shfl_sync(0xffffffffu, v, 0) != 0;
        }
        if (r) {
          fence_proxy_async_global();  // the x rows other CTAs stored are read by TMA
          for (int i = 0; i < npend; ++i) issue_x(pend_s[i], pend_kb[i]);
          npend = 0;
          xready = true;
        }
        return r;
      };
      for (long long u = lo; u < hi; ++u, ++g) {
        const int s = int(g % ST);
        if (g >= ST) {
          const uint32_t par = uint32_t((g / ST) - 1) & 1u;
          if (!xready && npend > 0 && !mbar_try_wait(&empty[s], par)) {
            // the ring is full of stages waiting for x: the phase barrier must pass first
            if (!release(true)) {
              ok = false;
              break;
            }
          }
          if (!mbar_wait_warp(&empty[s], par)) {
            ok = false;
            break;
          }
        }
        const int tile = int(u / ph.kb_total), kb = int(u % ph.kb_total);
        if (elect_one()) {
          mbar_arrive_expect_tx(&full[s], stage_bytes);
          tma_load_2d_hint(smem + size_t(s) * stage_bytes, &maps.w[p], &full[s], 0,
                           (tile * ph.kb_total + kb) * kTileM, pol_w);
        }
        __syncwarp();
        if (xready) {
          issue_x(s, kb);
        } else {
          pend_s[npend] = s;
          pend_kb[npend] = kb;
          ++npend;
          release(false);
        }
      }
      if (ok && npend > 0 && !release(true)) ok = false;
    }
    if (!ok && lane == 0) atomicOr(a.err, kFlagChainWait);
  } else if (warp == kMmaWarp) {
    // ================= MMA issuer: one accumulator per segment, alternating
    const uint32_t idesc = idesc_f16_f32(kTileM, a.ng);
    long long g = 0;
    long long seg = 0;
    for (int p = 0; p < a.nph && ok; ++p) {
      const Phase& ph = a.ph[p];
      if (ph.kind != CHAIN_GEMM) continue;
      const long long lo = range_lo(ph.units, cta, G), hi = range_lo(ph.units, cta + 1, G);
      for (long long u = lo; u < hi; ++u, ++g) {
        const bool first = (u == lo) || (u % ph.kb_total == 0);
        const bool last = (u + 1 == hi) || ((u + 1) % ph.kb_total == 0);
        const int buf = int(seg & 1);
        if (first && seg >= 2 &&
            !mbar_wait_warp(&acc_empty[buf], uint32_t((seg >> 1) - 1) & 1u)) {
          ok = false;
          break;
        }
        const int s = int(g % ST);
        if (!mbar_wait_warp(&full[s], uint32_t(g / ST) & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (elect_one()) {
          const uint32_t wa = smem_u32(smem + size_t(s) * stage_bytes);
          const uint32_t xa = wa + kWBytes;
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk)
            umma_f16(tmem + uint32_t(buf * a.acc_cols), desc_k_sw128(wa + kk * 32),
                     desc_k_sw128(xa + kk * 32), idesc, (!first || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
          if (last) umma_commit(&acc_full[buf]);
        }
        __syncwarp();
        if (last) ++seg;
      }
    }
    if (!ok && lane == 0) atomicOr(a.err, kFlagChainWait);
  } else {
    // ================= epilogue warps 2..5: thread e = tile row e (TMEM lane e)
    const int e = threadIdx.x - 64;
    const int q = warp & 3;  // TMEM lane quadrant of this warp
    const int ew = warp - 2;  // epilogue warp 0..3: token rows ew, ew + 4, ...
    const uint32_t lane_addr = tmem + (uint32_t(q * 32) << 16);
    const int row = q * 32 + lane;
    long long seg = 0;
    pdl_wait();
    for (int p = 0; p < a.nph && ok; ++p) {
      const Phase& ph = a.ph[p];
      if (ph.kind == CHAIN_NORM) {
        // ---- rows cta, cta + G, ... of the residual stream, normalised
        int v = 1;
        if (e == 0) v = phase_input_ready(a, p, true) ? 1 : 0;
        if (!bar_and(kBarEpi, kEpiThreads, v != 0)) {
          ok = false;
          break;
        }
        int nrows = 0;
        float* part_sum = red;  // 4 floats of scratch
        for (int r = cta; r < a.m; r += G, ++nrows) {
          const float* xr = ph.src + (size_t)r * a.dim;
          float ss = 0.f;
          // L2 reads: other CTAs wrote these rows earlier in the kernel
          for (int i = e * 4; i < a.dim; i += kEpiThreads * 4) {
            const float4 x4 = __ldcg(reinterpret_cast<const float4*>(xr + i));
            ss += x4.x * x4.x + x4.y * x4.y + x4.z * x4.z + x4.w * x4.w;
          }
          ss = warp_sum(ss);
          if (lane == 0) part_sum[ew] = ss;
          bar_and(kBarEpi, kEpiThreads, true);
          const float tot = (part_sum[0] + part_sum[1]) + (part_sum[2] + part_sum[3]);
          const float rms = sqrtf(tot / float(a.dim) + a.eps);
          for (int i = e * 4; i < a.dim; i += kEpiThreads * 4) {
            const float4 x4 = __ldcg(reinterpret_cast<const float4*>(xr + i));
            const float4 w4 = *reinterpret_cast<const float4*>(ph.w + i);
            const float4 o = make_float4(x4.x / rms * w4.x, x4.y / rms * w4.y,
                                         x4.z / rms * w4.z, x4.w / rms * w4.w);
            if (ph.dst32) *reinterpret_cast<float4*>(ph.dst32 + (size_t)r * a.dim + i) = o;
            __half2* d = reinterpret_cast<__half2*>(ph.dst16 + (size_t)r * a.dim + i);
            d[0] = __floats2half2_rn(o.x, o.y);
            d[1] = __floats2half2_rn(o.z, o.w);
          }
          bar_and(kBarEpi, kEpiThreads, true);  // part_sum is reused by the next row
        }
        if (ph.zero_keys)
          for (int i = cta * kEpiThreads + e; i < ph.n_keys; i += G * kEpiThreads)
            ph.zero_keys[i] = 0ull;
        fence_proxy_async_global();  // the next phase reads these rows with TMA
        bar_and(kBarEpi, kEpiThreads, true);
        if (e == 0 && nrows > 0) {
          __threadfence();
          atomicAdd(&a.done[p], (unsigned long long)nrows);
        }
        continue;
      }
      // ---- GEMM phase: the segments of this CTA's range, in order
      const long long lo = range_lo(ph.units, cta, G), hi = range_lo(ph.units, cta + 1, G);
      const int kbt = ph.kb_total;
      int npart = 0, part_tile[2] = {0, 0};  // split tiles this CTA reduces a slice of
      for (long long s0 = lo; s0 < hi;) {
        const int tile = int(s0 / kbt);
        const long long t_end = (long long)(tile + 1) * kbt;
        const long long s1 = hi < t_end ? hi : t_end;
        const int len = int(s1 - s0);
        const int buf = int(seg & 1);
        if (!bar_and(kBarEpi, kEpiThreads, mbar_wait(&acc_full[buf], uint32_t(seg >> 1) & 1u))) {
          ok = false;
          break;
        }
        tc_fence_after();
        // accumulator -> red[token][tile row]; 64 columns per wait when the accumulator has them
        const uint32_t acc_addr = lane_addr + uint32_t(buf * a.acc_cols);
        if (a.acc_cols >= 64) {
          for (int c0 = 0; c0 < a.m; c0 += 64) {
            float v[4][16];
            tmem_ld16x4(acc_addr + c0, acc_addr + c0 + 16, acc_addr + c0 + 32, acc_addr + c0 + 48, v);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int jj = 0; jj < 16; ++jj)
                if (c0 + 16 * i + jj < a.m) red[(c0 + 16 * i + jj) * kTileM + row] = v[i][jj];
          }
        } else {
          for (int c0 = 0; c0 < a.m; c0 += 16) {
            float v[16];
            tmem_ld16(acc_addr + c0, v);
#pragma unroll
            for (int jj = 0; jj < 16; ++jj)
              if (c0 + jj < a.m) red[(c0 + jj) * kTileM + row] = v[jj];
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        bar_and(kBarEpi, kEpiThreads, true);
        if (len == kbt) {
          // this CTA holds the whole tile: every row now
          epilogue_rows(ph, tile, ew, 4, a.m, lane, red);
          fence_proxy_async_global();  // the next phase reads these rows with TMA
          bar_and(kBarEpi, kEpiThreads, true);
          if (e == 0) {
            __threadfence();
            atomicAdd(&a.done[p], (unsigned long long)a.m);
          }
        } else {
          // part of the tile: publish it and count the tile's arrived k-blocks; the rows are
          // reduced after this CTA's last segment of the phase, so publishing never waits
          const int end = (tile == int(lo / kbt)) ? 0 : 1;
          float* slot = a.part + ((size_t(p) * G + cta) * 2 + end) * size_t(a.m) * kTileM;
          for (int i = e; i < a.m * kTileM / 4; i += kEpiThreads)
            reinterpret_cast<float4*>(slot)[i] = reinterpret_cast<const float4*>(red)[i];
          bar_and(kBarEpi, kEpiThreads, true);
          if (e == 0) {
            __threadfence();
            atomicAdd(a.tile_cnt + size_t(p) * a.max_tiles + tile, unsigned(len));
          }
          if (npart < 2) part_tile[npart++] = tile;
        }
        bar_and(kBarEpi, kEpiThreads, true);  // red is rewritten by the next segment
        ++seg;
        s0 = s1;
      }
      // ---- the split tiles: once all their k-blocks have arrived, each owner reduces its
      // own slice of the rows, summing the owners' partials in k (CTA) order
      for (int k2 = 0; k2 < npart && ok; ++k2) {
        const int tile = part_tile[k2];
        unsigned* cnt = a.tile_cnt + size_t(p) * a.max_tiles + tile;
        unsigned* fin = a.tile_cnt + size_t(kMaxChainPhases + p) * a.max_tiles + tile;
        int v = 1;
        if (e == 0) {
          const uint64_t t0 = global_ns();
          while (ld_acquire_u32(cnt) < unsigned(kbt)) {
            __nanosleep(32);
            if (global_ns() - t0 > 2000000000ull) {
              v = 0;
              break;
            }
          }
          // owners of the tile in CTA order: flags[1] = count, flags[2 + i] = slot, flags[0] =
          // this CTA's index among them
          const long long t0u = (long long)tile * kbt;
          const int c_first = unit_owner(t0u, ph.units, G);
          const int c_last = unit_owner(t0u + kbt - 1, ph.units, G);
          int nseg = 0;
          for (int c = c_first; c <= c_last && nseg < kMaxSegments; ++c) {
            const long long lo_c = range_lo(ph.units, c, G), hi_c = range_lo(ph.units, c + 1, G);
            if (hi_c <= t0u || lo_c >= t0u + kbt || lo_c == hi_c) continue;
            if (c == cta) flags[0] = nseg;
            const int end_c = (tile == int(lo_c / kbt)) ? 0 : 1;
            flags[2 + nseg++] = (p * G + c) * 2 + end_c;
          }
          flags[1] = nseg;
        }
        if (!bar_and(kBarEpi, kEpiThreads, v != 0)) {
          ok = false;
          break;
        }
        const int nseg = flags[1], me = flags[0];
        const int r0 = me * a.m / nseg, r1 = (me + 1) * a.m / nseg;
        const size_t slot_floats = size_t(a.m) * kTileM;
        for (int i = r0 * (kTileM / 4) + e; i < r1 * (kTileM / 4); i += kEpiThreads) {
          float4 acc4 = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int q2 = 0; q2 < nseg; ++q2) {
            const float4 v4 =
                __ldcg(reinterpret_cast<const float4*>(a.part + size_t(flags[2 + q2]) * slot_floats) + i);
            acc4.x += v4.x;
            acc4.y += v4.y;
            acc4.z += v4.z;
            acc4.w += v4.w;
          }
          reinterpret_cast<float4*>(red)[i] = acc4;
        }
        bar_and(kBarEpi, kEpiThreads, true);
        epilogue_rows(ph, tile, r0 + ew, 4, r1, lane, red);
        fence_proxy_async_global();  // the next phase reads these rows with TMA
        bar_and(kBarEpi, kEpiThreads, true);
        if (e == 0) {
          __threadfence();
          if (r1 > r0) atomicAdd(&a.done[p], (unsigned long long)(r1 - r0));
          // the last owner through resets the tile's counters for the next launch
          if (atomicAdd(fin, 1u) + 1 == unsigned(nseg)) {
            *cnt = 0u;
            *fin = 0u;
            __threadfence();
          }
        }
        bar_and(kBarEpi, kEpiThreads, true);  // flags and red are reused
      }
    }
    if (!ok && e == 0) atomicOr(a.err, kFlagChainWait);
  }

  // ---- all roles done: the last CTA out resets the phase counters for the next launch
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(a.exit_cnt, 1u);
    if (prev + 1 == unsigned(G)) {
      __threadfence();
      for (int p = 0; p < a.nph; ++p) a.done[p] = 0ull;
      *a.exit_cnt = 0u;
      __threadfence();
    }
  }
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, uint32_t(2 * a.acc_cols));
  }
}

}  // namespace

bool chain_supported(int m, std::string* why) {
  if (m < 1 || m > kMaxChainLanes) {
    if (why) *why = "lanes must be in 1..128 for the layer chain";
    return false;
  }
  return true;
}

size_t chain_part_bytes(int m, int grid) {
  return size_t(kMaxChainPhases) * grid * 2 * size_t(m) * kTileM * sizeof(float);
}

cudaError_t launch_chain(const ChainRequest& r, const ChainWorkspace& w, cudaStream_t st,
                         int device) {
  std::string why;
  if (!chain_supported(r.m, &why)) {
    set_error("chain: " + why);
    return cudaErrorInvalidValue;
  }
  if (r.nph < 1 || r.nph > kMaxChainPhases) {
    set_error("chain: 1..6 phases");
    return cudaErrorInvalidValue;
  }
  // One CTA per SM; fewer when a phase is so small that one tile's k-range would be split
  // over more CTAs than the fixup lists.
  int grid = num_sms(device);
  for (int p = 0; p < r.nph; ++p) {
    const GemmRequest& g = r.ph[p].gemm;
    if (r.ph[p].kind != CHAIN_GEMM || g.k < kBlockK || g.n < kTileM) continue;
    const long long kb = g.k / kBlockK, units = (long long)(g.n / kTileM) * kb;
    while (grid > 1 && kb / std::max<long long>(1, units / grid) + 2 > kMaxSegments) --grid;
  }
  if (chain_part_bytes(r.m, grid) > w.part_bytes || !w.done || !w.tile_cnt || !w.exit_cnt) {
    set_error("chain: workspace too small");
    return cudaErrorInvalidValue;
  }
  ChainArgs a{};
  ChainMaps maps;
  memset(&maps, 0, sizeof(maps));
  a.m = r.m;
  a.dim = r.dim;
  a.eps = r.eps;
  a.nph = r.nph;
  a.ng = std::max(16, (r.m + 15) / 16 * 16);
  a.acc_cols = 32;
  while (a.acc_cols < a.ng) a.acc_cols *= 2;
  const size_t red_bytes = size_t(r.m) * kTileM * 4;
  const size_t stage = kWBytes + size_t(a.ng) * 128;
  const size_t budget = 200 * 1024;
  a.stages = int(std::min<size_t>(kMaxStages, (budget - red_bytes) / stage));
  if (a.stages < 2) {
    set_error("chain: shared memory too small for two stages");
    return cudaErrorInvalidValue;
  }
  a.done = w.done;
  a.exit_cnt = w.exit_cnt;
  a.tile_cnt = w.tile_cnt;
  a.max_tiles = w.max_tiles;
  a.part = w.part;
  a.err = w.err;
  for (int p = 0; p < r.nph; ++p) {
    const ChainPhaseRequest& in = r.ph[p];
    Phase& ph = a.ph[p];
    ph.kind = in.kind;
    if (in.kind == CHAIN_GEMM) {
      const GemmRequest& g = in.gemm;
      if (!gemm_supported(g.m, g.k, g.n, g.epi, &why) || g.m != r.m || !g.packed) {
        set_error("chain: phase " + std::to_string(p) + ": " + (why.empty() ? "needs packed weights and the chain's lanes" : why));
        return cudaErrorInvalidValue;
      }
      ph.n = g.n;
      ph.k = g.k;
      ph.tiles = g.n / kTileM;
      ph.kb_total = g.k / kBlockK;
      ph.units = ph.tiles * ph.kb_total;
      if (ph.tiles > w.max_tiles) {
        set_error("chain: too many tiles for the workspace");
        return cudaErrorInvalidValue;
      }
      ph.epi = g.epi;
      ph.y = g.y;
      ph.ldy = g.ldy > 0 ? g.ldy : (g.epi == EPI_SWIGLU ? g.n / 2 : g.n);
      ph.qk = g.qk;
      ph.keys = g.argmax_keys;
      ph.vocab = g.vocab;
      ph.codebooks = g.vocab > 0 ? g.n / g.vocab : 0;
      ph.pick = g.pick;
      if (!make_tmap_2d_f16(&maps.w[p], g.w, kBlockK, uint64_t(ph.tiles) * ph.kb_total * kTileM,
                            kBlockK * 2, kBlockK, kTileM, true) ||
          !make_tmap_2d_f16(&maps.x[p], g.x, g.k, g.m, uint64_t(g.k) * 2, kBlockK, a.ng, true)) {
        set_error("chain: cuTensorMapEncodeTiled failed (pointers must be 16-byte aligned)");
        return cudaErrorInvalidValue;
      }
    } else {
      ph.src = in.norm_src;
      ph.w = in.norm_w;
      ph.dst16 = in.norm_dst16;
      ph.dst32 = in.norm_dst32;
      ph.zero_keys = in.zero_keys;
      ph.n_keys = in.n_keys;
      if (r.dim % 4 || !ph.src || !ph.w || !ph.dst16) {
        set_error("chain: norm phase needs src, weight, f16 output and dim % 4 == 0");
        return cudaErrorInvalidValue;
      }
    }
  }
  const size_t smem = size_t(a.stages) * stage + red_bytes + 512 + 1024;
  {
    static std::mutex mu;
    static bool done[64] = {false};
    std::lock_guard<std::mutex> lock(mu);
    if (device >= 0 && device < 64 && !done[device]) {
      cudaFuncSetAttribute(chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      done[device] = true;
    }
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
  return cudaLaunchKernelEx(&cfg, chain_kernel, maps, a);
}

}  // namespace tts
