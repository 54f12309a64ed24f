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
//   all 4 warps    epilogue: TMEM -> registers -> split-K partials; the last CTA to arrive
//                  on a tile sums the partials in split order (deterministic) and applies
//                  the fused epilogue.
// Weight loads for the first stages are issued before `griddepcontrol.wait`, so under
// programmatic dependent launch they overlap the previous kernel's tail; only the x loads,
// which read the previous kernel's output, wait.
#include <algorithm>
#include <cstdio>
#include <mutex>

#include "tts_common.cuh"
#include "tts_internal.h"
#include "qkrope_row.cuh"

namespace tts {

namespace {

constexpr int kTileM = 128;  // weight rows per CTA (= MMA M)
constexpr int kBlockK = 64;  // K per stage: one 128-byte swizzle row of f16
constexpr int kWBytes = kTileM * kBlockK * 2;

struct GemmArgs {
  int m, k, n;
  int kb_total, splits, tiles;
  int groups, ng;  // token groups (<= 2) and MMA N per group (multiple of 16, <= 256)
  int stages;
  int tmem_cols;
  int epi;
  float* ws;
  unsigned* counters;
  int* err;
  void* y;
  int ldy;
  QkRopeArgs qk;
  unsigned long long* keys;
  int vocab;
  int codebooks;
};

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

// One token row of one 128-row tile: lane owns rows 4*lane .. 4*lane + 3.
__device__ __forceinline__ void epilogue_row(const GemmArgs& a, int tile, int j, int lane,
                                             float4 acc) {
  const int f0 = tile * kTileM + 4 * lane;
  switch (a.epi) {
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
      float4* y = reinterpret_cast<float4*>(static_cast<float*>(a.y) + (size_t)j * a.ldy + f0);
      float4 r = *y;
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
        const int f = tile * (kTileM / 2) + 4 * lane;
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
      const int cb = (tile * kTileM) / a.vocab;
      const int id0 = f0 - cb * a.vocab;
      float v[4] = {acc.x, acc.y, acc.z, acc.w};
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

__global__ void __launch_bounds__(128, 1)
    gemm_decode_kernel(const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmX, const GemmArgs a) {
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

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.stages * stage_bytes);
  uint64_t* empty = full + a.stages;
  uint64_t* done = empty + a.stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_launch_dependents();

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer
    const uint64_t pol_w = l2_policy_evict_first();
    const int pre = nkb < a.stages ? nkb : a.stages;
    for (int i = 0; i < pre; ++i) {
      uint8_t* st = smem + i * stage_bytes;
      mbar_arrive_expect_tx(&full[i], stage_bytes);
      tma_load_2d_hint(st, &tmW, &full[i], (kb0 + i) * kBlockK, tile * kTileM, pol_w);
    }
    pdl_wait();  // x is the previous kernel's output
    for (int i = 0; i < pre; ++i) {
      uint8_t* st = smem + i * stage_bytes + kWBytes;
      for (int g = 0; g < a.groups; ++g)
        tma_load_2d(st + g * a.ng * 128, &tmX, &full[i], (kb0 + i) * kBlockK, g * a.ng);
    }
    for (int i = pre; i < nkb; ++i) {
      const int s = i % a.stages;
      if (!mbar_wait(&empty[s], ((i / a.stages) + 1) & 1)) {
        atomicOr(a.err, 1);
        break;
      }
      uint8_t* st = smem + s * stage_bytes;
      mbar_arrive_expect_tx(&full[s], stage_bytes);
      tma_load_2d_hint(st, &tmW, &full[s], (kb0 + i) * kBlockK, tile * kTileM, pol_w);
      for (int g = 0; g < a.groups; ++g)
        tma_load_2d(st + kWBytes + g * a.ng * 128, &tmX, &full[s], (kb0 + i) * kBlockK,
                    g * a.ng);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    const uint32_t idesc = idesc_f16_f32(kTileM, a.ng);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % a.stages;
      if (!mbar_wait(&full[s], (i / a.stages) & 1)) {
        atomicOr(a.err, 2);
        break;
      }
      tc_fence_after();
      const uint32_t wa = smem_u32(smem + s * stage_bytes);
      const uint32_t xa = wa + kWBytes;
#pragma unroll
      for (int kk = 0; kk < kBlockK / 16; ++kk) {
        const uint64_t ad = desc_k_sw128(wa + kk * 32);
        for (int g = 0; g < a.groups; ++g) {
          const uint64_t bd = desc_k_sw128(xa + g * a.ng * 128 + kk * 32);
          umma_f16(tmem + g * a.ng, ad, bd, idesc, (i | kk) != 0);
        }
      }
      umma_commit(&empty[s]);
    }
    umma_commit(done);
  }
  __syncwarp();

  // ---------------- epilogue: TMEM -> split-K partials
  const bool ok = mbar_wait(done, 0);
  if (!ok && threadIdx.x == 64) atomicOr(a.err, 4);
  tc_fence_after();
  pdl_wait();
  const int row = warp * 32 + lane;
  float* part = a.ws + ((size_t)split * a.tiles + tile) * a.m * kTileM;
  for (int c0 = 0; c0 < a.m; c0 += 16) {
    float v[16];
    tmem_ld16(tmem + (uint32_t(warp * 32) << 16) + c0, v);
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) {
      const int j = c0 + jj;
      if (j < a.m) part[(size_t)j * kTileM + row] = v[jj];
    }
  }
  tc_fence_before();
  __threadfence();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, a.tmem_cols);
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&a.counters[tile], 1u);
    *last_flag = (prev == unsigned(a.splits - 1));
  }
  __syncthreads();
  if (!*last_flag) return;
  __threadfence();

  // ---------------- last CTA on this tile: reduce in split order, fused epilogue
  for (int j = warp; j < a.m; j += 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < a.splits; ++s) {
      const float4 p = __ldcg(reinterpret_cast<const float4*>(
                                  a.ws + (((size_t)s * a.tiles + tile) * a.m + j) * kTileM) +
                              lane);
      acc.x += p.x;
      acc.y += p.y;
      acc.z += p.z;
      acc.w += p.w;
    }
    epilogue_row(a, tile, j, lane, acc);
  }
  if (threadIdx.x == 0) a.counters[tile] = 0u;
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
  int groups, ng, stages, splits, tmem_cols;
  size_t smem;
};

Plan plan_gemm(int m, int k, int n, int device, int force_splits) {
  Plan p{};
  const int pad = std::max(16, (m + 15) / 16 * 16);
  p.groups = (pad + 255) / 256;
  p.ng = ((pad + p.groups - 1) / p.groups + 15) / 16 * 16;
  const int cols = p.groups * p.ng;
  p.tmem_cols = 32;
  while (p.tmem_cols < cols) p.tmem_cols *= 2;
  const int stage = kWBytes + cols * 128;
  // Two CTAs per SM when stages fit in ~100 KB: one drains its epilogue while the other
  // streams; wide token counts take one CTA per SM with deeper stages.
  const bool two = stage * 4 <= 100 * 1024;
  const int budget = two ? 100 * 1024 : 200 * 1024;
  p.stages = std::max(2, std::min(8, budget / stage));
  p.smem = size_t(p.stages) * stage + 1024 + 256;
  const int tiles = n / kTileM;
  const int kb = k / kBlockK;
  const int slots = num_sms(device) * (two ? 2 : 1);
  int s = std::max(1, slots / tiles);
  s = std::min(s, std::max(1, kb / 2));
  if (force_splits > 0) s = std::min(force_splits, kb);
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
  if (m < 1 || m > 512) return no("lanes (m) must be in 1..512");
  if (k < kBlockK || k % kBlockK) return no("k must be a positive multiple of 64");
  if (n < kTileM || n % kTileM) return no("n must be a positive multiple of 128");
  if (epi < EPI_F32 || epi > EPI_ARGMAX) return no("unknown epilogue");
  return true;
}

cudaError_t launch_gemm(const GemmRequest& r, const Workspace& wsp, cudaStream_t st, int device) {
  std::string why;
  if (!gemm_supported(r.m, r.k, r.n, r.epi, &why)) {
    set_error("proj: " + why);
    return cudaErrorInvalidValue;
  }
  const Plan p = plan_gemm(r.m, r.k, r.n, device, r.force_splits);
  const int tiles = r.n / kTileM;
  const size_t need = size_t(p.splits) * tiles * r.m * kTileM * sizeof(float);
  if (need > wsp.ws_bytes || tiles > wsp.n_counters) {
    set_error("proj: split-K workspace too small for this shape");
    return cudaErrorInvalidValue;
  }
  CUtensorMap tmW, tmX;
  if (!make_tmap_2d_f16(&tmW, r.w, r.k, r.n, uint64_t(r.k) * 2, kBlockK, kTileM, true) ||
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
  a.stages = p.stages;
  a.tmem_cols = p.tmem_cols;
  a.epi = r.epi;
  a.ws = wsp.ws;
  a.counters = wsp.counters;
  a.err = wsp.err;
  a.y = r.y;
  a.ldy = r.ldy > 0 ? r.ldy : (r.epi == EPI_SWIGLU ? r.n / 2 : r.n);
  a.qk = r.qk;
  a.keys = r.argmax_keys;
  a.vocab = r.vocab;
  a.codebooks = r.vocab > 0 ? r.n / r.vocab : 0;

  {
    // The opt-in shared-memory limit is a per-device function attribute.
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !done[dev]) {
      cudaFuncSetAttribute(gemm_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      done[dev] = true;
    }
  }

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(tiles, p.splits, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = r.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_decode_kernel, tmW, tmX, a);
}

}  // namespace tts
