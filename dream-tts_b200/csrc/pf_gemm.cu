// Prefill-shaped projection GEMM on tcgen05: y[rows, n] = x[rows, k] . W[n, k]^T for thousands
// of token rows (the prompt prefill, crates/qwen3tts/src/qwen3.rs:294-467 at t > 1), f16 in,
// f32 accumulate.
//
// The decode GEMM (gemm_decode.cu) puts the weight rows on the MMA's M and the few lanes on its
// N, splits K over a cluster and reduces the partials row by row: right for 48 lanes, but at
// hundreds of rows its row-serial epilogue dominates. Here the token rows are the MMA's M (128
// per tile) and the weights its N (256 per tile: two packed 128-row weight tiles), every tile
// covers all of K in one CTA, and the accumulator is read straight from TMEM by the thread that
// owns its row: no reduction, no shared-memory transpose.
//
// Persistent: one CTA per SM walks tiles t = blockIdx.x, + gridDim.x, ... (tiles ordered m-fastest
// so that the CTAs running at once share each weight tile through L2). Warp roles (256 threads):
//   warp 0 (one elected lane)  TMA producer: x tile 16 KB + W tiles 32 KB per 64-deep K block
//   warp 1 (one elected lane)  MMA issuer: 4 x tcgen05.mma M128 N256 K16 per K block into one of
//                              two TMEM accumulators (256 columns each)
//   warp 2                     TMEM allocation (512 columns)
//   warps 4..7                 epilogue of the previous tile (TMEM lane quadrant = warp - 4),
//                              overlapping the next tile's main loop
// Every wait is bounded; a wait that gives up sets an error flag that the host reads.
#include <algorithm>
#include <mutex>

#include "gemm_epilogue.cuh"
#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

namespace {

constexpr int kPfM = 128;     // token rows per tile (MMA M)
constexpr int kPfN = 256;     // weight rows per tile (MMA N)
constexpr int kPfK = 64;      // K per stage: one 128-byte swizzle row of f16
constexpr int kPfStages = 4;
constexpr int kPfThreads = 256;
constexpr uint32_t kXBytes = kPfM * kPfK * 2;   // 16 KB
constexpr uint32_t kWBytesPf = kPfN * kPfK * 2;  // 32 KB
constexpr uint32_t kStageBytes = kXBytes + kWBytesPf;

struct PfArgs {
  int rows, k, n, kb, m_tiles, tiles, epi;
  void* y;
  int ldy;
  int* err;
};

__global__ void __launch_bounds__(kPfThreads, 1)
    pf_gemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                   const PfArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPfStages * kStageBytes);
  uint64_t* empty = full + kPfStages;
  uint64_t* tfull = empty + kPfStages;  // [2] accumulator ready
  uint64_t* tempty = tfull + 2;         // [2] accumulator read by the epilogue
  uint64_t* drain = tempty + 2;         // an aborted MMA warp's last commit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  __shared__ int s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int my_tiles = blockIdx.x < a.tiles ? (a.tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(drain, 1);
    s_abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  int issued = 0;  // producer: K blocks whose loads were issued (32-bit: tiles x K blocks)

  if (warp == 0) {
    // ---------------- producer
    const uint64_t pol_w = l2_policy_evict_last();  // every m tile of this n tile reads it
    int g = 0;  // K blocks issued over all tiles
    for (int i = 0; i < my_tiles && ok; ++i) {
      const int t = blockIdx.x + i * gridDim.x;
      const int m0 = (t % a.m_tiles) * kPfM;
      const int nt = t / a.m_tiles;
      for (int kb = 0; kb < a.kb && ok; ++kb, ++g) {
        const int s = int(g % kPfStages);
        if (g >= kPfStages) ok = mbar_wait_warp(&empty[s], uint32_t((g / kPfStages) - 1) & 1);
        if (!ok) break;
        issued = g + 1;
        if (elect_one()) {
          uint8_t* st = smem + size_t(s) * kStageBytes;
          mbar_arrive_expect_tx(&full[s], kStageBytes);
          tma_load_2d(st, &tmX, &full[s], kb * kPfK, m0);
          // packed weights: the 128 x 64 block of (128-row tile T, K block kb) is rows
          // (T * kb_total + kb) * 128 of the [tiles * kb_total * 128][64] view
          tma_load_2d_hint(st + kXBytes, &tmW, &full[s], 0, ((2 * nt) * a.kb + kb) * 128, pol_w);
          tma_load_2d_hint(st + kXBytes + kWBytesPf / 2, &tmW, &full[s], 0,
                           ((2 * nt + 1) * a.kb + kb) * 128, pol_w);
        }
        __syncwarp();
      }
    }
    if (!ok && lane == 0) {
      atomicOr(a.err, 16);
      s_abort = 1;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    const uint32_t idesc = idesc_f16_f32(kPfM, kPfN);
    int g = 0;
    for (int i = 0; i < my_tiles && ok; ++i) {
      const int b = i & 1;
      if (i >= 2) ok = mbar_wait_warp(&tempty[b], uint32_t((i >> 1) - 1) & 1);
      if (!ok) break;
      tc_fence_after();
      const uint32_t acc = tmem + uint32_t(b * kPfN);
      for (int kb = 0; kb < a.kb && ok; ++kb, ++g) {
        const int s = int(g % kPfStages);
        ok = mbar_wait_warp(&full[s], uint32_t(g / kPfStages) & 1);
        if (!ok) break;
        tc_fence_after();
        if (elect_one()) {
          const uint32_t xa = smem_u32(smem + size_t(s) * kStageBytes);
          const uint32_t wa = xa + kXBytes;
#pragma unroll
          for (int kk = 0; kk < kPfK / 16; ++kk)
            umma_f16(acc, desc_k_sw128(xa + kk * 32), desc_k_sw128(wa + kk * 32), idesc,
                     (kb | kk) != 0);
          umma_commit(&empty[s]);
        }
        __syncwarp();
      }
      if (ok) {
        if (elect_one()) umma_commit(&tfull[b]);
        __syncwarp();
      }
    }
    if (!ok && lane == 0) {
      atomicOr(a.err, 32);
      s_abort = 1;
    }
  } else if (warp >= 4) {
    // ---------------- epilogue: thread (warp 4 + q, lane) owns token row m0 + 32 q + lane
    const int q = warp - 4;
    for (int i = 0; i < my_tiles; ++i) {
      const int b = i & 1;
      if (!mbar_wait(&tfull[b], uint32_t(i >> 1) & 1)) {
        atomicOr(a.err, 64);
        s_abort = 1;
        break;
      }
      tc_fence_after();
      const int t = blockIdx.x + i * gridDim.x;
      const int r = (t % a.m_tiles) * kPfM + q * 32 + lane;
      const int nt = t / a.m_tiles;
      const uint32_t base = tmem + (uint32_t(q * 32) << 16) + uint32_t(b * kPfN);
      const bool live = r < a.rows;
      if (a.epi == EPI_SWIGLU) {
        // the two 128-row weight tiles each hold 64 gate rows then the matching 64 up rows;
        // output features (2 nt + h) * 64 + c
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int c0 = 0; c0 < 64; c0 += 32) {
            float v[4][16];
            const uint32_t g0 = base + uint32_t(h * 128 + c0);
            tmem_ld16x4(g0, g0 + 64, g0 + 16, g0 + 80, v);
            if (live) {
              __half* dst = static_cast<__half*>(a.y) + (size_t)r * a.ldy + (2 * nt + h) * 64 + c0;
#pragma unroll
              for (int p = 0; p < 2; ++p) {
                uint4 pk[2];
                __half2* h2 = reinterpret_cast<__half2*>(pk);
#pragma unroll
                for (int e = 0; e < 8; ++e)
                  h2[e] = __floats2half2_rn(silu(v[2 * p][2 * e]) * v[2 * p + 1][2 * e],
                                            silu(v[2 * p][2 * e + 1]) * v[2 * p + 1][2 * e + 1]);
                reinterpret_cast<uint4*>(dst + p * 16)[0] = pk[0];
                reinterpret_cast<uint4*>(dst + p * 16)[1] = pk[1];
              }
            }
          }
        }
      } else {
        // EPI_F32: y = acc; EPI_RESIDUAL: y += acc (f32 rows of ldy)
#pragma unroll
        for (int c0 = 0; c0 < kPfN; c0 += 64) {
          float v[4][16];
          const uint32_t g0 = base + uint32_t(c0);
          tmem_ld16x4(g0, g0 + 16, g0 + 32, g0 + 48, v);
          if (live) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.y) + (size_t)r * a.ldy +
                                                    nt * kPfN + c0);
#pragma unroll
            for (int p = 0; p < 4; ++p) {
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float4 o = make_float4(v[p][4 * e], v[p][4 * e + 1], v[p][4 * e + 2],
                                       v[p][4 * e + 3]);
                if (a.epi == EPI_RESIDUAL) {
                  const float4 old = dst[p * 4 + e];
                  o.x += old.x;
                  o.y += old.y;
                  o.z += old.z;
                  o.w += old.w;
                }
                dst[p * 4 + e] = o;
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[b]);
    }
  }
  // On the normal path every MMA completed before the epilogue read its tile. After a wait gave
  // up, the MMA warp waits (bounded) for the MMAs it issued and the producer for its loads still
  // in flight, so that neither lands after TMEM or shared memory is released.
  tc_fence_before();
  __syncthreads();
  if (s_abort) {
    if (warp == 1) {
      if (elect_one()) umma_commit(drain);
      __syncwarp();
      mbar_wait(drain, 0, 100000000ull);
    } else if (warp == 0 && lane == 0) {
      for (int gg = issued > kPfStages ? issued - kPfStages : 0; gg < issued; ++gg)
        mbar_wait(&full[gg % kPfStages], uint32_t(gg / kPfStages) & 1, 100000000ull);
    }
  }
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

bool pf_gemm_supported(int rows, int k, int n, int epi, std::string* why) {
  auto no = [&](const char* s) {
    if (why) *why = s;
    return false;
  };
  if (rows < 1) return no("rows must be >= 1");
  if (k < kPfK || k % kPfK) return no("k must be a positive multiple of 64");
  if (n < kPfN || n % kPfN) return no("n must be a positive multiple of 256");
  if (epi != EPI_F32 && epi != EPI_RESIDUAL && epi != EPI_SWIGLU)
    return no("epilogue must be f32, residual or swiglu");
  return true;
}

cudaError_t launch_pf_gemm(const PfGemmRequest& r, cudaStream_t st, int device, int* err) {
  std::string why;
  if (!pf_gemm_supported(r.rows, r.k, r.n, r.epi, &why)) {
    set_error("prefill proj: " + why);
    return cudaErrorInvalidValue;
  }
  CUtensorMap tmX, tmW;
  const uint64_t w_rows = uint64_t(r.n) / 128 * (r.k / kPfK) * 128;
  if (!make_tmap_2d_f16(&tmX, r.x, r.k, r.rows, uint64_t(r.k) * 2, kPfK, kPfM, true) ||
      !make_tmap_2d_f16(&tmW, r.w, kPfK, w_rows, kPfK * 2, kPfK, 128, true)) {
    set_error("prefill proj: cuTensorMapEncodeTiled failed (pointers must be 16-byte aligned)");
    return cudaErrorInvalidValue;
  }
  PfArgs a{};
  a.rows = r.rows;
  a.k = r.k;
  a.n = r.n;
  a.kb = r.k / kPfK;
  a.m_tiles = (r.rows + kPfM - 1) / kPfM;
  a.tiles = a.m_tiles * (r.n / kPfN);
  a.epi = r.epi;
  a.y = r.y;
  a.ldy = r.ldy > 0 ? r.ldy : (r.epi == EPI_SWIGLU ? r.n / 2 : r.n);
  a.err = err;
  const size_t smem = size_t(kPfStages) * kStageBytes + 1024 + 256;  // tiles, alignment, barriers
  {
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !done[dev]) {
      cudaFuncSetAttribute(pf_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      done[dev] = true;
    }
  }
  const int grid = std::min(a.tiles, num_sms(device));
  pf_gemm_kernel<<<grid, kPfThreads, smem, st>>>(tmX, tmW, a);
  return cudaGetLastError();
}

}  // namespace tts
