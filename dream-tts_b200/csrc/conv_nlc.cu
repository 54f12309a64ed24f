// Channels-last conv1d as an implicit GEMM on tcgen05, with SnakeBeta on load and bias +
// residual in the epilogue.
//
// The B200 form of tts-nn's fused `nlc_conv_f32` (crates/tts-nn/src/nlcconv.rs:15-198 and
// crates/tts-nn/src/nlc.rs:40-132): the tap gather happens inside the GEMM, so no im2col matrix
// exists. GEMM view: M = output positions, N = output channels, K = taps x input channels.
// A CTA computes MS (1 or 2) sub-tiles of 128 positions against the same weight tiles: with
// N <= 256 per CTA the two accumulators fill the 512 TMEM columns and every weight tile read
// from L2 feeds twice the MMAs (the weight stream, not the tensor core, limited the single
// sub-tile form: measured 35% tensor-pipe activity at 1 sub-tile x N = 512).
//
// For each 64-channel block, TMA brings one "halo" of R = 128*MS + (k-1)*dil input rows (as
// one or two boxes of rows per 8-channel slab) into shared memory in the no-swizzle K-major
// core-matrix layout: slab g (8 channels) holds row r at byte r*16, slabs R*16 bytes apart. In
// that layout row r is simply 16*r bytes from the start, so the A operand of sub-tile j and tap
// t is the same halo with the descriptor's start moved by (128*j + t*dil)*16 bytes: all taps
// and both sub-tiles read one load, and SnakeBeta is applied once per halo element (in place)
// rather than once per tap. Rows before 0 or past len are zero-filled by TMA, and snake(0) = 0,
// so padding matches the reference's pad-then-activate order.
//
// CTA pairs: where a tile is 256 output channels, two CTAs of a cluster share it
// (tcgen05 cta_group::2). Each holds its own positions' halo and half of every weight tile (128
// rows), and the even CTA issues M = 256 MMAs that read both CTAs' shared memory and write both
// CTAs' TMEM. Each SM then streams half the weight bytes per MMA and the MMA issuer drives two
// SMs. The odd CTA's halo and epilogue warps report to the even CTA's barriers (remote
// arrivals); its weight loads count on the even CTA's barrier; the MMAs' completions arrive in
// both CTAs (multicast commits). The issue loop precomputes each tap's descriptors (one thread
// issues every MMA, and rebuilding descriptors per MMA made issue, not the tensor pipe, the
// limit).
//
// Persistent: one CTA (pair) per SM (pair of SMs) loops over (position block, batch,
// output-channel slice) tiles.
// Warp roles (384 threads): warp 0 issues the weight tiles (B ring), warp 1 the MMAs (each
// from one elected lane of the converged warp), warps 2..5 run the epilogue of one tile while
// warps 6..11 load the next tile's halos (A ring, one halo per sub-tile) and apply the snake, so
// a tile's loads and snake overlap the previous tile's epilogue. Every wait is bounded; a wait
// that gives up sets an error flag the host reads.
#include <algorithm>
#include <map>
#include <mutex>
#include <utility>

#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

namespace {

constexpr int kRows = 128;      // output positions per sub-tile (the MMA's M)
constexpr int kCB = 64;         // input channels per halo
constexpr int kHaloWarp0 = 6;   // warps 6..11 load and transform the halos
constexpr int kHaloThreads = 192;
// 12 warps: three per SM sub-partition, which caps registers at 168 per thread (as ten would)
constexpr int kThreads = 384;
// TMA epilogue: per epilogue warp, two residual boxes and one output box of 32 rows x 64
// channels (f16, 128-byte swizzle: 4 KB each)
constexpr int kEpiBox = 32 * 64 * 2;
constexpr int kEpiWarpBytes = 3 * kEpiBox;

struct ConvArgs {
  int b, len, cin, cout, k, dil, pad_left;
  int cout_cta;  // output channels per CTA (<= 512)
  int nh, nper;  // MMAs per K step and sub-tile, and N of each
  int ms;        // 128-position sub-tiles per CTA (1 or 2), one accumulator each
  int acc_stride;  // TMEM columns between the sub-tiles' accumulators
  int nbuf;        // accumulator sets (1 or 2): with 2, tile t's epilogue drains one set while
                   // tile t + 1's MMAs fill the other
  int buf_stride;  // TMEM columns between the sets
  int R;         // halo rows covering every sub-tile (multiple of 8)
  int H, nrb;    // rows per halo TMA box and boxes per 8-channel slab (R = H * nrb)
  int as, bs;    // halo and weight ring depths
  int tmem_cols;
  const float* bias;
  int bias_v4;  // bias is 16-byte aligned: read 4 channels per load
  int snake_v4;  // alpha and 1/beta are 16-byte aligned: read 4 channels per load
  int tma_epi;   // residual rows in and output rows out by TMA boxes (else per-thread rows)
  const float* alpha;
  const float* brecip;
  const __half* res;
  __half* y;
  int* err;
};

// SnakeBeta on 8 f16 channels in place. The fast hardware sine is used: its absolute error
// (about 2^-21 near the origin, growing slowly with the argument) stays far below the f16
// rounding of the result, while the accurate sinf's range reduction made the snake, applied to
// every halo element, cost as much as the MMAs it feeds. The channels' alpha and 1/beta are
// in registers (loaded once per 8-channel slab of a halo).
__device__ __forceinline__ void snake8r(uint4& u, const float (&al)[8], const float (&br)[8]) {
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float2 f = __half22float2(h[q]);
    const float s0 = __sinf(al[2 * q] * f.x);
    const float s1 = __sinf(al[2 * q + 1] * f.y);
    f.x = f.x + br[2 * q] * (s0 * s0);
    f.y = f.y + br[2 * q + 1] * (s1 * s1);
    h[q] = __floats2half2_rn(f.x, f.y);
  }
}

// kPair: CTA pairs (2-CTA clusters) share each weight tile; see the file comment.
template <bool kPair>
__global__ void __launch_bounds__(kThreads, 1)
    conv_nlc_kernel(const __grid_constant__ CUtensorMap tmX,
                    const __grid_constant__ CUtensorMap tmW,
                    const __grid_constant__ CUtensorMap tmR,
                    const __grid_constant__ CUtensorMap tmY, const ConvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  constexpr int P = kPair ? 2 : 1;  // CTAs per tile
  const uint32_t rank = kPair ? cluster_rank() : 0u;
  const bool leader = rank == 0;  // the CTA that issues the MMAs
  const int kAStages = a.as, kBStages = a.bs;
  const int ncb = a.cin / kCB;
  const int span = kRows * a.ms * P;  // positions per tile (each CTA kRows * ms of them)
  const int nx = (a.len + span - 1) / span;
  const int nz = a.cout / a.cout_cta;
  const int ntiles = nx * a.b * nz;
  // this CTA's (pair's) tiles: unit, unit + units, ...
  const int unit = blockIdx.x / P, units = gridDim.x / P;
  const int my_tiles = unit < ntiles ? (ntiles - 1 - unit) / units + 1 : 0;
  auto tile_of = [&](int t, int& l0, int& bb, int& co0) {
    const int id = unit + t * units;
    l0 = (id % nx) * span + int(rank) * kRows * a.ms;  // this CTA's first position
    bb = (id / nx) % a.b;
    co0 = (id / (nx * a.b)) * a.cout_cta;
  };
  const uint32_t a_bytes = uint32_t(a.R) * kCB * 2;  // one halo: 8 slabs x R rows x 16 B
  // this CTA's weight rows per step: all cout_cta, or its half of them in a pair
  const uint32_t b_bytes = uint32_t(a.cout_cta / P) * kCB * 2;
  uint8_t* a_base = smem;
  uint8_t* b_base = smem + kAStages * a_bytes;
  // the TMA epilogue's boxes (4 warps), then the barriers
  uint8_t* e_base = b_base + kBStages * b_bytes;
  uint64_t* bars =
      reinterpret_cast<uint64_t*>(e_base + (a.tma_epi ? 4 * kEpiWarpBytes : 0));
  uint64_t* full_a = bars;
  uint64_t* ready_a = bars + kAStages;
  uint64_t* empty_a = bars + 2 * kAStages;
  uint64_t* full_b = bars + 3 * kAStages;
  uint64_t* empty_b = full_b + kBStages;
  uint64_t* tmem_full = empty_b + kBStages;  // [2] MMAs of a tile done (per accumulator set)
  uint64_t* tmem_empty = tmem_full + 2;      // [2] its accumulators read by the epilogue
  uint64_t* res_bar = tmem_empty + 2;        // [4 warps][2] residual boxes landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_bar + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // tracing build: each role's summed wait (or busy) times, recorded at the end
  [[maybe_unused]] const unsigned long long tl_entry = TTS_TL_NOW();
  [[maybe_unused]] unsigned long long tl_w0 = 0, tl_w1 = 0, tl_w2 = 0, tl_t = 0;
  if (threadIdx.x == 0) {
    // in a pair the MMA-side barriers that count both CTAs live in the leader: ready_a
    // (both CTAs' halo threads), full_b (both halves' bytes), tmem_empty (both epilogues)
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&ready_a[s], kHaloThreads * P);
      mbar_init(&empty_a[s], 1);
    }
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(&full_b[s], 1);
      mbar_init(&empty_b[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tmem_full[s], 1);
      mbar_init(&tmem_empty[s], 4 * P);
    }
    for (int s = 0; s < 8; ++s) mbar_init(&res_bar[s], 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
    if (a.tma_epi) {
      tma_prefetch_desc(&tmR);
      tma_prefetch_desc(&tmY);
    }
  }
  if (warp == 1) {
    if constexpr (kPair) {
      tmem_alloc_pair(tmem_slot, a.tmem_cols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, a.tmem_cols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  // a pair's barriers and TMEM exist in both CTAs before either signals the other
  if constexpr (kPair)
    cluster_sync();
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();

  const int steps = ncb * a.k;  // (cb, tap) steps per tile
  if (warp == 0) {
    // ---------------- weight tiles: global step g = (tile, cb, tap)
    const int total = my_tiles * steps;
    // the ring slot and phase of step g, and its (tile, cb, tap), kept as running counters (a
    // division by a run-time divisor is a long instruction sequence)
    int s = 0, tile_i = 0, cb = 0, t = 0;
    uint32_t ph = 0;
    for (int g = 0; g < total; ++g) {
      tl_t = TTS_TL_NOW();
      const bool ok_e = g < kBStages || mbar_wait_warp(&empty_b[s], ph ^ 1u);
      tl_w0 += TTS_TL_NOW() - tl_t;
      if (!ok_e) {
        if (lane == 0) atomicOr(a.err, 16);
        break;
      }
      if (elect_one()) {
        int l0, bb, co0;
        tile_of(tile_i, l0, bb, co0);
        uint8_t* dst = b_base + s * b_bytes;
        if constexpr (kPair) {
          // this CTA's half of the tile's rows; both halves count on the leader's barrier,
          // which expects both
          const uint32_t fb = cluster_addr(&full_b[s], 0);
          if (leader) mbar_arrive_expect_tx(&full_b[s], b_bytes * 2);
          for (int h = 0; h < a.nh; ++h)
            tma_load_2d_pair(dst + h * (a.nper / 2) * 128, &tmW, fb, t * a.cin + cb * kCB,
                             co0 + h * a.nper + int(rank) * (a.nper / 2));
        } else {
          mbar_arrive_expect_tx(&full_b[s], b_bytes);
          for (int h = 0; h < a.nh; ++h)
            tma_load_2d(dst + h * a.nper * 128, &tmW, &full_b[s], t * a.cin + cb * kCB,
                        co0 + h * a.nper);
        }
      }
      __syncwarp();
      if (++t == a.k) {
        t = 0;
        if (++cb == ncb) {
          cb = 0;
          ++tile_i;
        }
      }
      if (++s == kBStages) {
        s = 0;
        ph ^= 1u;
      }
    }
  } else if (warp == 1 && (!kPair || leader)) {
    // ---------------- MMA issuer: the accumulators of one tile at a time (in a pair, M = 256:
    // 128 positions of each CTA, N = a.nper with half of the weight rows in each CTA)
    const uint32_t idesc = idesc_f16_f32(kRows * P, a.nper);
    // the MMAs' completion arrives in both CTAs of a pair
    auto commit = [&](uint64_t* bar) {
      if constexpr (kPair)
        umma_commit_pair(bar, 3);
      else
        umma_commit(bar);
    };
    const uint32_t slab = uint32_t(a.R) * 16;
    bool ok = true;
    // the halo and weight ring slots of the next step and their phases, as running counters
    int sa = 0, sb = 0;
    uint32_t pa = 0, pb = 0;
    for (int tl = 0; tl < my_tiles && ok; ++tl) {
      // accumulator set tl % nbuf, used for the (tl / nbuf)-th time
      const int buf = tl % a.nbuf, use = tl / a.nbuf;
      const uint32_t acc0 = tmem + uint32_t(buf * a.buf_stride);
      tl_t = TTS_TL_NOW();
      const bool ok_t = use == 0 || mbar_wait_warp(&tmem_empty[buf], (use - 1) & 1);
      tl_w0 += TTS_TL_NOW() - tl_t;
      if (!ok_t) {
        if (lane == 0) atomicOr(a.err, 32);
        break;
      }
      tc_fence_after();
      for (int cb = 0; cb < ncb && ok; ++cb) {
        tl_t = TTS_TL_NOW();
        const bool ok_a = mbar_wait_warp(&ready_a[sa], pa);
        tl_w1 += TTS_TL_NOW() - tl_t;
        if (!ok_a) {
          if (lane == 0) atomicOr(a.err, 32);
          ok = false;
          break;
        }
        const uint32_t ha = smem_u32(a_base + sa * a_bytes);
        for (int t = 0; t < a.k; ++t) {
          const int i = cb * a.k + t;
          tl_t = TTS_TL_NOW();
          const bool ok_b = mbar_wait_warp(&full_b[sb], pb);
          tl_w2 += TTS_TL_NOW() - tl_t;
          if (!ok_b) {
            if (lane == 0) atomicOr(a.err, 64);
            ok = false;
            break;
          }
          tc_fence_after();
          if (elect_one()) {
            const uint32_t hb = smem_u32(b_base + sb * b_bytes);
            auto mma = [&](uint32_t d, uint64_t ad, uint64_t bd, uint32_t acc) {
              if constexpr (kPair)
                umma_f16_pair(d, ad, bd, idesc, acc);
              else
                umma_f16(d, ad, bd, idesc, acc);
            };
            // The descriptors of this tap's first MMA; the others differ only in the start
            // address field (bits 0-13, in 16-byte units, no carry below 256 KB): +32 B per
            // 16 channels of the weight rows, +2 slabs per 16 channels of the halo, +128 rows
            // per sub-tile. One thread issues every MMA, so its issue loop is kept this short.
            const uint64_t a_t = desc_k_interleave(ha + t * a.dil * 16, slab);
            const uint64_t b_0 = desc_k_sw128(hb);
            const uint64_t a_kk = 2 * (slab >> 4), a_j = (kRows * 16) >> 4;
            if (a.ms == 2 && a.nh == 1) {
#pragma unroll
              for (int kk = 0; kk < kCB / 16; ++kk) {
                const uint64_t bd = b_0 + uint64_t(kk * 2);
                const uint64_t ad = a_t + uint64_t(kk) * a_kk;
                const uint32_t acc = (i | kk) != 0;
                mma(acc0, ad, bd, acc);
                mma(acc0 + a.acc_stride, ad + a_j, bd, acc);
              }
            } else if (a.ms == 1 && a.nh == 1) {
#pragma unroll
              for (int kk = 0; kk < kCB / 16; ++kk)
                mma(acc0, a_t + uint64_t(kk) * a_kk, b_0 + uint64_t(kk * 2), (i | kk) != 0);
            } else if (a.ms == 1 && a.nh == 2) {
              // two N = nper MMAs per 16 channels on the same halo rows
              const uint64_t b_h = uint64_t(((a.nper / P) * 128) >> 4);
#pragma unroll
              for (int kk = 0; kk < kCB / 16; ++kk) {
                const uint64_t ad = a_t + uint64_t(kk) * a_kk;
                const uint32_t acc = (i | kk) != 0;
                mma(acc0, ad, b_0 + uint64_t(kk * 2), acc);
                mma(acc0 + a.nper, ad, b_0 + b_h + uint64_t(kk * 2), acc);
              }
            } else {
#pragma unroll
              for (int kk = 0; kk < kCB / 16; ++kk) {
                for (int h = 0; h < a.nh; ++h) {
                  const uint64_t bd =
                      b_0 + uint64_t((h * (a.nper / P) * 128) >> 4) + uint64_t(kk * 2);
                  for (int j = 0; j < a.ms; ++j)
                    // sub-tile j starts 128 rows into the shared halo
                    mma(acc0 + j * a.acc_stride + h * a.nper,
                        a_t + uint64_t(kk) * a_kk + uint64_t(j) * a_j, bd, (i | kk) != 0);
                }
              }
            }
            commit(&empty_b[sb]);
          }
          __syncwarp();
          if (++sb == kBStages) {
            sb = 0;
            pb ^= 1u;
          }
        }
        if (ok) {
          if (elect_one()) commit(&empty_a[sa]);
          __syncwarp();
        }
        if (++sa == kAStages) {
          sa = 0;
          pa ^= 1u;
        }
      }
      if (ok) {
        if (elect_one()) commit(&tmem_full[buf]);
        __syncwarp();
      }
    }
  } else if (warp >= 6) {
    // ---------------- halos (global index gc = (tile, cb)): load, snake in place, hand over
    const int tt = threadIdx.x - kHaloWarp0 * 32;  // 0..kHaloThreads-1
    const int total = my_tiles * ncb;
    auto issue = [&](int gi) {  // by all of the first halo warp
      const int s = gi % kAStages;
      if (gi >= kAStages && !mbar_wait_warp(&empty_a[s], ((gi / kAStages) + 1) & 1)) {
        if (lane == 0) atomicOr(a.err, 128);
        return;
      }
      if (elect_one()) {
        int l0, bb, co0;
        tile_of(gi / ncb, l0, bb, co0);
        const int cb = gi % ncb;
        mbar_arrive_expect_tx(&full_a[s], a_bytes);
        // slab g (8 channels) holds rows [0, R) at 16 B each: nrb boxes of H rows per slab
        for (int gq = 0; gq < kCB / 8; ++gq)
          for (int rb = 0; rb < a.nrb; ++rb)
            tma_load_4d(a_base + s * a_bytes + (gq * a.R + rb * a.H) * 16, &tmX, &full_a[s], 0,
                        l0 + rb * a.H - a.pad_left, cb * (kCB / 8) + gq, bb);
      }
      __syncwarp();
    };
    if (warp == kHaloWarp0)
      for (int gi = 0; gi < std::min(total, kAStages - 1); ++gi) issue(gi);
    for (int gi = 0; gi < total; ++gi) {
      const int s = gi % kAStages;
      tl_t = TTS_TL_NOW();
      const bool ok_h = mbar_wait(&full_a[s], (gi / kAStages) & 1);
      tl_w0 += TTS_TL_NOW() - tl_t;
      tl_t = TTS_TL_NOW();
      if (!ok_h) {
        if (tt == 0) atomicOr(a.err, 4096);
      }
      if (a.alpha) {
        uint8_t* halos = a_base + s * a_bytes;
        const int cb = gi % ncb;
        uint4* p = reinterpret_cast<uint4*>(halos);
        // Elements c = slab * R + row, two per thread per pass (kHaloThreads apart: the
        // sine's latency dominates), the slab tracked as the row wraps rather than divided
        // out (R >= 128: a step of kHaloThreads wraps at most twice).
        auto ab = [&](int g, float (&al)[8], float (&br)[8]) {
          const int ch = cb * kCB + g * 8;
          if (a.snake_v4) {
            const float4* a4 = reinterpret_cast<const float4*>(a.alpha + ch);
            const float4* b4 = reinterpret_cast<const float4*>(a.brecip + ch);
            const float4 a0 = __ldg(a4), a1 = __ldg(a4 + 1), b0 = __ldg(b4), b1 = __ldg(b4 + 1);
            al[0] = a0.x, al[1] = a0.y, al[2] = a0.z, al[3] = a0.w;
            al[4] = a1.x, al[5] = a1.y, al[6] = a1.z, al[7] = a1.w;
            br[0] = b0.x, br[1] = b0.y, br[2] = b0.z, br[3] = b0.w;
            br[4] = b1.x, br[5] = b1.y, br[6] = b1.z, br[7] = b1.w;
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              al[e] = __ldg(a.alpha + ch + e);
              br[e] = __ldg(a.brecip + ch + e);
            }
          }
        };
        int g0 = 0, r0 = tt;
        while (r0 >= a.R) r0 -= a.R, ++g0;
        while (g0 < kCB / 8) {
          int g1 = g0, r1 = r0 + kHaloThreads;
          while (r1 >= a.R) r1 -= a.R, ++g1;
          const bool two = g1 < kCB / 8;
          uint4 u0 = p[g0 * a.R + r0];
          uint4 u1 = two ? p[g1 * a.R + r1] : make_uint4(0, 0, 0, 0);
          float al0[8], br0[8], al1[8], br1[8];
          ab(g0, al0, br0);
          ab(two ? g1 : g0, al1, br1);
          snake8r(u0, al0, br0);
          snake8r(u1, al1, br1);
          p[g0 * a.R + r0] = u0;
          if (two) p[g1 * a.R + r1] = u1;
          g0 = g1;
          r0 = r1 + kHaloThreads;
          while (r0 >= a.R) r0 -= a.R, ++g0;
        }
        tl_w1 += TTS_TL_NOW() - tl_t;
        tl_t = TTS_TL_NOW();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tl_w2 += TTS_TL_NOW() - tl_t;
        tl_t = TTS_TL_NOW();
      }
      tl_w1 += TTS_TL_NOW() - tl_t;
      // the halo is ready for the MMAs (in a pair: on the leader's barrier)
      if (kPair && !leader)
        mbar_arrive_cluster(cluster_addr(&ready_a[s], 0));
      else
        mbar_arrive(&ready_a[s]);
      if (warp == kHaloWarp0 && gi + kAStages - 1 < total) issue(gi + kAStages - 1);
    }
  } else if (warp >= 2) {
    // ---------------- epilogue (warps 2..5: TMEM lane quadrant = warp % 4), one tile at a time
    const int quad = warp & 3;
    // 64 columns per TMEM wait; the residual of the next 64 columns is read while this batch
    // is finished, so the row's residual loads overlap instead of adding up
    auto finish16 = [&](float* v, const uint4* rr, int c0, int co0, size_t row, bool live) {
      if (!live) return;
      if (a.bias && a.bias_v4) {
        // four 16-byte loads (the same addresses across the warp: broadcasts)
        const float4* b4 = reinterpret_cast<const float4*>(a.bias + co0 + c0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 b = __ldg(b4 + q);
          v[4 * q] += b.x;
          v[4 * q + 1] += b.y;
          v[4 * q + 2] += b.z;
          v[4 * q + 3] += b.w;
        }
      } else if (a.bias) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] += __ldg(a.bias + co0 + c0 + i);
      }
      if (a.res) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const __half2* h2 = reinterpret_cast<const __half2*>(&rr[hh]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = __half22float2(h2[q]);
            v[hh * 8 + 2 * q] += f.x;
            v[hh * 8 + 2 * q + 1] += f.y;
          }
        }
      }
      uint4 o[2];
      __half2* oh = reinterpret_cast<__half2*>(o);
#pragma unroll
      for (int q = 0; q < 8; ++q) oh[q] = __floats2half2_rn(v[2 * q], v[2 * q + 1]);
      uint4* yp = reinterpret_cast<uint4*>(a.y + row + c0);
      yp[0] = o[0];
      yp[1] = o[1];
    };
    const int c64 = a.cout_cta / 64 * 64;  // columns done 64 at a time
    // TMA epilogue: this warp's boxes and residual barriers; rk counts its 64-column batches
    // (batch k uses residual box k & 1, for the (k >> 1)-th time)
    uint8_t* rbox = e_base + (warp - 2) * kEpiWarpBytes;
    uint8_t* obox = rbox + 2 * kEpiBox;
    uint64_t* rbar = res_bar + 2 * (warp - 2);
    uint32_t rk = 0;
    // byte offset of row r's 16-byte chunk q in a 128-byte-swizzled box
    auto swz = [](int r, int q) { return r * 128 + ((q ^ (r & 7)) << 4); };
    for (int tl = 0; tl < my_tiles; ++tl) {
      const int buf = tl % a.nbuf;
      tl_t = TTS_TL_NOW();
      if (!mbar_wait(&tmem_full[buf], (tl / a.nbuf) & 1) && lane == 0) atomicOr(a.err, 8192);
      tl_w0 += TTS_TL_NOW() - tl_t;
      tl_t = TTS_TL_NOW();
      tc_fence_after();
      int l0, bb, co0;
      tile_of(tl, l0, bb, co0);
      for (int j = 0; j < a.ms; ++j) {
        const int l = l0 + j * kRows + quad * 32 + lane;
        const bool live = l < a.len;
        if (a.tma_epi) {
          // the warp's 32 rows as boxes of 64 channels: residual in by TMA one batch ahead,
          // the finished f16 rows out by TMA (rows past len are neither read nor written)
          const int lw = l0 + j * kRows + quad * 32;
          if (lw >= a.len) continue;  // no row of this warp exists (warp-uniform)
          const uint32_t acc = tmem + (uint32_t(quad * 32) << 16) +
                               uint32_t(buf * a.buf_stride + j * a.acc_stride);
          const int nb = a.cout_cta / 64;
          auto load_res = [&](int b, uint32_t k) {
            if (lane == 0 && a.res) {
              // the box's previous contents were read before the warp's last sync
              fence_proxy_async();
              mbar_arrive_expect_tx(&rbar[k & 1], kEpiBox);
              tma_load_3d(rbox + (k & 1) * kEpiBox, &tmR, &rbar[k & 1], co0 + 64 * b, lw, bb);
            }
          };
          load_res(0, rk);
          for (int b = 0; b < nb; ++b, ++rk) {
            if (b + 1 < nb) load_res(b + 1, rk + 1);
            float v[4][16];
            tmem_ld16x4(acc + 64 * b, acc + 64 * b + 16, acc + 64 * b + 32, acc + 64 * b + 48, v);
            if (a.bias) {
              // the same addresses across the warp: broadcasts
#pragma unroll
              for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int e = 0; e < 16; e += 4) {
                  const float* bp = a.bias + co0 + 64 * b + 16 * i + e;
                  const float4 b4 = a.bias_v4 ? __ldg(reinterpret_cast<const float4*>(bp))
                                              : make_float4(__ldg(bp), __ldg(bp + 1),
                                                            __ldg(bp + 2), __ldg(bp + 3));
                  v[i][e] += b4.x;
                  v[i][e + 1] += b4.y;
                  v[i][e + 2] += b4.z;
                  v[i][e + 3] += b4.w;
                }
            }
            if (a.res) {
              if (!mbar_wait(&rbar[rk & 1], (rk >> 1) & 1) && lane == 0) atomicOr(a.err, 16384);
              const uint8_t* rb = rbox + (rk & 1) * kEpiBox;
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const uint4 u = *reinterpret_cast<const uint4*>(rb + swz(lane, q));
                const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 f = __half22float2(h2[e]);
                  v[q >> 1][(q & 1) * 8 + 2 * e] += f.x;
                  v[q >> 1][(q & 1) * 8 + 2 * e + 1] += f.y;
                }
              }
            }
            // the output box is free once the previous store has read it
            if (lane == 0) bulk_wait_read_all();
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              uint4 o;
              __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
              for (int e = 0; e < 4; ++e)
                oh[e] = __floats2half2_rn(v[q >> 1][(q & 1) * 8 + 2 * e],
                                          v[q >> 1][(q & 1) * 8 + 2 * e + 1]);
              *reinterpret_cast<uint4*>(obox + swz(lane, q)) = o;
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&tmY, obox, co0 + 64 * b, lw, bb);
              bulk_commit_group();
            }
          }
          continue;
        }
        const size_t row = ((size_t)bb * a.len + (live ? l : 0)) * a.cout + co0;
        const uint32_t acc = tmem + (uint32_t(quad * 32) << 16) +
                             uint32_t(buf * a.buf_stride + j * a.acc_stride);
        const uint4* rp = reinterpret_cast<const uint4*>(a.res + row);  // 8 channels per uint4
        const bool rd = a.res && live;
        uint4 rnext[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          rnext[q] = (rd && q * 8 < c64) ? rp[q] : make_uint4(0, 0, 0, 0);
        for (int c0 = 0; c0 < c64; c0 += 64) {
          uint4 rcur[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) rcur[q] = rnext[q];
#pragma unroll
          for (int q = 0; q < 8; ++q)
            rnext[q] = (rd && c0 + 64 + q * 8 < c64) ? rp[(c0 + 64) / 8 + q] : make_uint4(0, 0, 0, 0);
          float v[4][16];
          tmem_ld16x4(acc + c0, acc + c0 + 16, acc + c0 + 32, acc + c0 + 48, v);
#pragma unroll
          for (int i = 0; i < 4; ++i) finish16(v[i], rcur + 2 * i, c0 + 16 * i, co0, row, live);
        }
        for (int c0 = c64; c0 < a.cout_cta; c0 += 16) {
          float v[16];
          tmem_ld16(acc + c0, v);
          uint4 rr[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
          if (rd) {
            rr[0] = rp[c0 / 8];
            rr[1] = rp[c0 / 8 + 1];
          }
          finish16(v, rr, c0, co0, row, live);
        }
      }
      // the accumulators may be overwritten by the next tile's MMAs
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        // in a pair the leader's MMAs wait for both CTAs' epilogues
        if (kPair && !leader)
          mbar_arrive_cluster(cluster_addr(&tmem_empty[buf], 0));
        else
          mbar_arrive(&tmem_empty[buf]);
      }
      tl_w1 += TTS_TL_NOW() - tl_t;
    }
    // every output box written before the CTA ends
    if (lane == 0 && a.tma_epi) bulk_wait_all();
    __syncwarp();
  }
#ifdef TTS_TIMELINE
  if (lane == 0 && (warp <= 2 || warp == kHaloWarp0)) {
    const uint64_t t_end = TTS_TL_NOW();
    const int k = kTlConv | (warp << 4);
    timeline_recs<6>({k | kTlCta, k | kTlEntry, k | 1, k | 2, k | 3, k | kTlEnd},
                     {uint64_t(blockIdx.x), tl_entry, tl_w0, tl_w1, tl_w2, t_end});
  }
#endif
  tc_fence_before();
  // a pair: neither CTA leaves (or frees TMEM) while the other may still signal its barriers
  if constexpr (kPair)
    cluster_sync();
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (kPair)
      tmem_dealloc_pair(tmem, a.tmem_cols);
    else
      tmem_dealloc(tmem, a.tmem_cols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 conv_encode_fn() {
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

}  // namespace

bool conv_supported(const ConvRequest& r, std::string* why) {
  auto no = [&](const char* s) {
    if (why) *why = s;
    return false;
  };
  if (r.b < 1 || r.len < 1) return no("empty input");
  if (r.cin < kCB || r.cin % kCB) return no("cin must be a positive multiple of 64");
  if (r.cout < 32 || r.cout % 32) return no("cout must be a positive multiple of 32");
  if (r.k < 1 || r.dil < 1) return no("k and dilation must be >= 1");
  if ((r.k - 1) * r.dil > 128) return no("(k - 1) * dilation must be <= 128");
  if (r.pad_left < 0 || r.pad_left > (r.k - 1) * r.dil)
    return no("pad_left must be in 0..(k-1)*dilation");
  return true;
}

cudaError_t launch_conv(const ConvRequest& r, cudaStream_t st, int device, int* err) {
  std::string why;
  if (!conv_supported(r, &why)) {
    set_error("conv1d: " + why);
    return cudaErrorInvalidValue;
  }
  auto fn = conv_encode_fn();
  if (!fn) {
    set_error("conv1d: cuTensorMapEncodeTiled unavailable");
    return cudaErrorInvalidValue;
  }
  ConvArgs a{};
  a.b = r.b;
  a.len = r.len;
  a.cin = r.cin;
  a.cout = r.cout;
  a.k = r.k;
  a.dil = r.dil;
  a.pad_left = r.pad_left;
  // Output channels per CTA: all of them up to 256, else 256 when it divides cout, else all
  // up to 512 (two MMAs of N = cout/2), else the largest of 128/64/32 that divides cout. With
  // N <= 256 a CTA takes two 128-position sub-tiles (when the input is that long).
  if (r.cout <= 256)
    a.cout_cta = r.cout;
  else if (r.cout % 256 == 0)
    a.cout_cta = 256;
  else if (r.cout <= 512)
    a.cout_cta = r.cout;
  else {
    a.cout_cta = 32;
    for (int c : {128, 64})
      if (r.cout % c == 0) {
        a.cout_cta = c;
        break;
      }
  }
  a.nh = a.cout_cta > 256 ? 2 : 1;
  a.nper = a.cout_cta / a.nh;
  a.ms = (a.cout_cta <= 256 && r.len > kRows) ? 2 : 1;
  {
    // TTS_CONV_SUBTILES=1 forces one sub-tile per CTA (A/B measurement)
    const char* v = getenv("TTS_CONV_SUBTILES");
    if (v && *v == '1') a.ms = 1;
  }
  // CTA pairs: the two CTAs of a cluster take 128 * ms positions each and half of every weight
  // tile, and the even one issues M = 256 MMAs for both. Where the output channels come in
  // 512s a pair's tile is 128 positions per CTA x 512 channels (two N = 256 MMAs per 16 input
  // channels on the same halo rows, so each input row is loaded and activated once per 512
  // output channels); where a tile is 256 channels, 2 x 128 positions per CTA x 256 channels.
  // TTS_CONV_WIDE=0 turns the 512-channel tile off, TTS_CONV_PAIR=0 keeps one CTA per tile,
  // TTS_CONV_ACC_SETS=2 double-buffers the accumulators with one sub-tile per CTA (A/B
  // measurement; each measured slower on the codec's block).
  a.nbuf = 1;
  bool pair = false;
  {
    const char* vp = getenv("TTS_CONV_PAIR");
    const char* vs = getenv("TTS_CONV_ACC_SETS");
    const bool pair_on = !(vp && *vp == '0');
    const bool two_sets = vs && *vs == '2';
    // pairs for 256-channel tiles and for tiles of two MMAs per 16 input channels (e.g. 384
    // channels as two N = 192 MMAs: 0.1348 -> 0.1224 ms at 4 x 10000 positions); single-MMA
    // tiles below 256 channels stay on one CTA (128 channels: 0.230 vs 0.237 ms in pairs)
    if (pair_on && a.cout_cta == 256 && a.nh == 1) pair = true;
    if (pair_on && a.nh == 2 && a.nper % 32 == 0) pair = true;
    const char* vw = getenv("TTS_CONV_WIDE");
    if (pair_on && !(vw && *vw == '0') && r.cout % 512 == 0 && !two_sets) {
      pair = true;
      a.cout_cta = 512;
      a.nh = 2;
      a.nper = 256;
      a.ms = 1;
    }
    // a pair's tile spans 2 * 128 * ms positions: one sub-tile each for short inputs
    if (pair && a.ms == 2 && r.len <= 2 * kRows) a.ms = 1;
    if (two_sets && a.cout_cta <= 256) {
      a.ms = 1;
      a.nbuf = 2;
    }
  }
  const int P = pair ? 2 : 1;
  a.acc_stride = 32;
  while (a.acc_stride < a.cout_cta) a.acc_stride *= 2;
  a.buf_stride = a.acc_stride * a.ms;
  // a second accumulator set wherever two fit in TMEM's 512 columns (tiles of <= 128 output
  // channels): the next tile's MMAs then run while this tile's epilogue drains the other set
  // (TTS_CONV_ACC_SETS=1 keeps one, A/B measurement)
  {
    const char* vs = getenv("TTS_CONV_ACC_SETS");
    if (a.nbuf == 1 && 2 * a.buf_stride <= 512 && !(vs && *vs == '1')) a.nbuf = 2;
  }
  a.tmem_cols = a.buf_stride * a.nbuf;
  // one halo for all sub-tiles: ms * 128 + (k-1)*dil rows, loaded as nrb boxes of H rows
  // (a box is at most 256 rows; H a multiple of 8 keeps every box 128-byte aligned)
  {
    const int need = kRows * a.ms + (r.k - 1) * r.dil;
    a.nrb = need > 256 ? 2 : 1;
    a.H = ((need + a.nrb - 1) / a.nrb + 7) / 8 * 8;
    a.R = a.H * a.nrb;
  }
  // TMA epilogue where the tile's channels come in 64-channel boxes and the output and residual
  // rows are 16-byte aligned (TTS_CONV_TMA_EPI=0: per-thread rows, A/B measurement)
  {
    const char* v = getenv("TTS_CONV_TMA_EPI");
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    a.tma_epi = !(v && *v == '0') && a.cout_cta % 64 == 0 && r.cout % 8 == 0 && al16(r.y) &&
                        (!r.res || al16(r.res))
                    ? 1
                    : 0;
  }
  // ring depths: the weight tiles are the steady stream (one per tap), halos one per 64 input
  // channels; fill what fits in 224 KB beside the epilogue's boxes: three halos where four or
  // more weight stages still fit, else two; at least two of each
  {
    const size_t halo = size_t(a.R) * kCB * 2, wt = size_t(a.cout_cta / P) * kCB * 2;
    const size_t budget = 224 * 1024 - (a.tma_epi ? 4 * kEpiWarpBytes : 0);
    const size_t bs_max = wt <= 16384 ? 6 : 4;
    const size_t bs_min3 = wt <= 16384 ? 4 : 3;  // weight stages that justify a third halo
    if (budget > 3 * halo && (budget - 3 * halo) / wt >= bs_min3) {
      a.as = 3;
      a.bs = int(std::min<size_t>(bs_max, (budget - 3 * halo) / wt));
    } else {
      a.as = 2;
      a.bs = budget > 2 * halo ? int(std::min<size_t>(bs_max, (budget - 2 * halo) / wt)) : 2;
      if (a.bs < 2) a.bs = 2;
    }
    // TTS_CONV_AS / TTS_CONV_BS override the ring depths (A/B measurement)
    const char* va = getenv("TTS_CONV_AS");
    const char* vb = getenv("TTS_CONV_BS");
    if (va && *va) a.as = std::max(2, std::min(4, atoi(va)));
    if (vb && *vb) a.bs = std::max(2, std::min(6, atoi(vb)));
  }
  a.bias = r.bias;
  a.bias_v4 = (reinterpret_cast<uintptr_t>(r.bias) & 15u) == 0 ? 1 : 0;
  a.snake_v4 = ((reinterpret_cast<uintptr_t>(r.alpha) | reinterpret_cast<uintptr_t>(r.brecip)) &
                15u) == 0
                   ? 1
                   : 0;
  a.alpha = r.alpha;
  a.brecip = r.brecip;
  a.res = r.res;
  a.y = r.y;
  a.err = err;

  // Halo map over x [b][len][cin]: dims (8 channels, len, cin/8 slabs, b). A box
  // {8, H, 1, 1} is H rows of one slab: nrb of them per slab build the [slab][row][8 ch]
  // core-matrix layout the MMA reads.
  CUtensorMap tmX, tmW;
  {
    cuuint64_t dims[4] = {8, cuuint64_t(r.len), cuuint64_t(r.cin / 8), cuuint64_t(r.b)};
    cuuint64_t strides[3] = {cuuint64_t(r.cin) * 2, 16, cuuint64_t(r.len) * r.cin * 2};
    cuuint32_t box[4] = {8, cuuint32_t(a.H), 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    if (fn(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(r.x), dims, strides, box,
           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
           CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      set_error("conv1d: halo tensor map rejected");
      return cudaErrorInvalidValue;
    }
  }
  if (!make_tmap_2d_f16(&tmW, r.w, uint64_t(r.k) * r.cin, uint64_t(r.cout),
                        uint64_t(r.k) * r.cin * 2, kCB, a.nper / P, true)) {
    set_error("conv1d: weight tensor map rejected");
    return cudaErrorInvalidValue;
  }
  // The epilogue's residual and output maps over [b][len][cout] f16: a box is 64 channels x 32
  // rows of one batch entry (rows past len are zero-filled on load and not written on store).
  CUtensorMap tmR{}, tmY{};
  if (a.tma_epi) {
    auto rows_map = [&](CUtensorMap* m, const void* ptr) {
      cuuint64_t dims[3] = {cuuint64_t(r.cout), cuuint64_t(r.len), cuuint64_t(r.b)};
      cuuint64_t strides[2] = {cuuint64_t(r.cout) * 2, cuuint64_t(r.len) * r.cout * 2};
      cuuint32_t box[3] = {64, 32, 1};
      cuuint32_t estr[3] = {1, 1, 1};
      return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims, strides,
                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    if (!rows_map(&tmY, r.y) || (r.res && !rows_map(&tmR, r.res))) {
      set_error("conv1d: epilogue tensor map rejected");
      return cudaErrorInvalidValue;
    }
  }
  const size_t smem = size_t(a.as) * a.R * kCB * 2 +
                      size_t(a.bs) * (a.cout_cta / P) * kCB * 2 +
                      (a.tma_epi ? 4 * kEpiWarpBytes : 0) + 1024 + 512;
  {
    // The opt-in shared-memory limit is a per-device function attribute.
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !done[dev]) {
      for (auto fn_k : {conv_nlc_kernel<false>, conv_nlc_kernel<true>})
        cudaFuncSetAttribute(fn_k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      done[dev] = true;
    }
  }
  if (smem > 227 * 1024) {
    set_error("conv1d: shared memory plan exceeds 227 KB");
    return cudaErrorInvalidValue;
  }
  cudaLaunchConfig_t cfg{};
  // persistent: one CTA (pair) per SM (pair of SMs), or per tile when there are fewer, each
  // looping over tiles
  const int span = kRows * a.ms * P;
  const long long ntiles = (long long)((r.len + span - 1) / span) * r.b * (r.cout / a.cout_cta);
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (ntiles > (1ll << 31) - 1) {
    set_error("conv1d: too many tiles");
    return cudaErrorInvalidValue;
  }
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = r.pdl ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!pair) {
    cfg.gridDim = dim3(unsigned(std::min<long long>(ntiles, std::max(1, sms))), 1, 1);
    return cudaLaunchKernelEx(&cfg, conv_nlc_kernel<false>, tmX, tmW, tmR, tmY, a);
  }
  // as many pairs as can be resident at once (a pair's SMs share a GPC); the occupancy query
  // depends only on the device and the shared memory, so it runs once per pair of them
  cfg.numAttrs = 2;
  int clusters = 0;
  {
    static std::mutex mu;
    static std::map<std::pair<int, size_t>, int> cache;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_pair(device, smem);
    auto it = cache.find(key);
    if (it != cache.end()) {
      clusters = it->second;
    } else {
      cfg.gridDim = dim3(2 * unsigned(std::max(1, sms / 2)), 1, 1);
      if (cudaOccupancyMaxActiveClusters(&clusters, conv_nlc_kernel<true>, &cfg) != cudaSuccess ||
          clusters < 1) {
        cudaGetLastError();
        clusters = std::max(1, sms / 2);
      }
      cache.emplace(key, clusters);
    }
  }
  cfg.gridDim = dim3(2 * unsigned(std::min<long long>(ntiles, clusters)), 1, 1);
  return cudaLaunchKernelEx(&cfg, conv_nlc_kernel<true>, tmX, tmW, tmR, tmY, a);
}

}  // namespace tts
