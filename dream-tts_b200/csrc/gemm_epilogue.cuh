// Epilogue of one token row of a 128-row weight tile of the decode GEMM: lane l holds rows
// 4l .. 4l + 3 of the tile for token row j.
#pragma once
#include "pick_rule.cuh"
#include "qkrope_row.cuh"
#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

constexpr int kTileRows = 128;

// x * sigmoid(x) with the fast exponential and division intrinsics: the result is rounded to
// f16, far coarser than their few-ulp error, and the IEEE division's branchy slow path kept the
// rows of the epilogue from overlapping (measured ~3x slower per row).
__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// One token row of one 128-row tile: lane owns rows 4*lane .. 4*lane + 3. `epi` is the
// epilogue kind (a compile-time constant where the caller's kernel is specialised on it).
template <typename A>
__device__ __forceinline__ void epilogue_row(const A& a, int tile, int j, int lane,
                                             float4 acc, int epi) {
  const int f0 = tile * kTileRows + 4 * lane;
  switch (epi) {
    case EPI_F32: {
      float* y = static_cast<float*>(a.y) + (size_t)j * a.ldy + f0;
      *reinterpret_cast<float4*>(y) = acc;
      break;
    }
    case EPI_F16: {
      __half2* y = reinterpret_cast<__half2*>(static_cast<__half*>(a.y) + (size_t)j * a.ldy + f0);
      y[0] = __floats2half2_rn(acc.x, acc.y);
      y[1] = __floats2half2_rn(acc.z, acc.w);
      break;
    }
    case EPI_RESIDUAL: {
      // an L2 read of the residual stream
      float4* y = reinterpret_cast<float4*>(static_cast<float*>(a.y) + (size_t)j * a.ldy + f0);
      float4 r = __ldcg(y);
      r.x += acc.x;
      r.y += acc.y;
      r.z += acc.z;
      r.w += acc.w;
      *y = r;
      break;
    }
    case EPI_SWIGLU: {
      // rows 0..63 of the tile are gate features, 64..127 the matching up features.
      float4 p;
      p.x = __shfl_xor_sync(0xffffffffu, acc.x, 16);
      p.y = __shfl_xor_sync(0xffffffffu, acc.y, 16);
      p.z = __shfl_xor_sync(0xffffffffu, acc.z, 16);
      p.w = __shfl_xor_sync(0xffffffffu, acc.w, 16);
      if (lane < 16) {
        const int f = tile * (kTileRows / 2) + 4 * lane;
        __half2* y = reinterpret_cast<__half2*>(static_cast<__half*>(a.y) + (size_t)j * a.ldy + f);
        y[0] = __floats2half2_rn(silu(acc.x) * p.x, silu(acc.y) * p.y);
        y[1] = __floats2half2_rn(silu(acc.z) * p.z, silu(acc.w) * p.w);
      }
      break;
    }
    case EPI_QKROPE: {
      // 128 rows = one head: q heads, then k heads, then v heads
      float v[4] = {acc.x, acc.y, acc.z, acc.w};
      qkrope_row(a.qk, tile, j, lane, v);
      break;
    }
    case EPI_ARGMAX: {
      if (a.y) {
        float* y = static_cast<float*>(a.y) + (size_t)j * a.ldy + f0;
        *reinterpret_cast<float4*>(y) = acc;
      }
      const int cb = (tile * kTileRows) / a.vocab;
      const int id0 = f0 - cb * a.vocab;
      float v[4] = {acc.x, acc.y, acc.z, acc.w};
      if (a.pick.vocab) pick_rule4(a.pick, j, id0, v);
      unsigned long long best = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        unsigned long long key =
            (static_cast<unsigned long long>(float_order_key(v[i])) << 32) | unsigned(id0 + i);
        best = key > best ? key : best;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      if (lane == 0) atomicMax(a.keys + (size_t)j * a.codebooks + cb, best);
      break;
    }
    default:
      break;
  }
}

}  // namespace tts
