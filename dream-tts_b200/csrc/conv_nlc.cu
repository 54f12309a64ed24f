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
// Persistent: one CTA per SM loops over (position block, batch, output-channel slice) tiles.
// Warp roles (320 threads): warp 0 issues the weight tiles (B ring), warp 1 the MMAs (each
// from one elected lane of the converged warp), warps 2..5 run the epilogue of one tile while
// warps 6..9 load the next tile's halos (A ring, one halo per sub-tile) and apply the snake, so
// a tile's loads and snake overlap the previous tile's epilogue. Every wait is bounded; a wait
// that gives up sets an error flag the host reads.
#include <algorithm>
#include <mutex>

#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

namespace {

constexpr int kRows = 128;      // output positions per sub-tile (the MMA's M)
constexpr int kCB = 64;         // input channels per halo
constexpr int kHaloWarp0 = 6;   // warps 6..9 load and transform the halos
constexpr int kHaloThreads = 128;
constexpr int kThreads = 320;

struct ConvArgs {
  int b, len, cin, cout, k, dil, pad_left;
  int cout_cta;  // output channels per CTA (<= 512)
  int nh, nper;  // MMAs per K step and sub-tile, and N of each
  int ms;        // 128-position sub-tiles per CTA (1 or 2), one accumulator each
  int acc_stride;  // TMEM columns between the sub-tiles' accumulators
  int R;         // halo rows covering every sub-tile (multiple of 8)
  int H, nrb;    // rows per halo TMA box and boxes per 8-channel slab (R = H * nrb)
  int as, bs;    // halo and weight ring depths
  int tmem_cols;
  const float* bias;
  const float* alpha;
  const float* brecip;
  const __half* res;
  __half* y;
  int* err;
};

// SnakeBeta on 8 f16 channels in place. The fast hardware sine is used: its absolute error
// (about 2^-21 near the origin, growing slowly with the argument) stays far below the f16
// rounding of the result, while the accurate sinf's range reduction made the snake, applied to
// every halo element, cost as much as the MMAs it feeds.
__device__ __forceinline__ void snake8(uint4& u, const float* alpha, const float* brecip) {
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float2 f = __half22float2(h[q]);
    const float s0 = __sinf(__ldg(alpha + 2 * q) * f.x);
    const float s1 = __sinf(__ldg(alpha + 2 * q + 1) * f.y);
    f.x = f.x + __ldg(brecip + 2 * q) * (s0 * s0);
    f.y = f.y + __ldg(brecip + 2 * q + 1) * (s1 * s1);
    h[q] = __floats2half2_rn(f.x, f.y);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    conv_nlc_kernel(const __grid_constant__ CUtensorMap tmX,
                    const __grid_constant__ CUtensorMap tmW, const ConvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int kAStages = a.as, kBStages = a.bs;
  const int ncb = a.cin / kCB;
  const int nx = (a.len + kRows * a.ms - 1) / (kRows * a.ms);
  const int nz = a.cout / a.cout_cta;
  const int ntiles = nx * a.b * nz;
  // this CTA's tiles: blockIdx.x, blockIdx.x + gridDim.x, ...
  const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  auto tile_of = [&](int t, int& l0, int& bb, int& co0) {
    const int id = blockIdx.x + t * gridDim.x;
    l0 = (id % nx) * kRows * a.ms;
    bb = (id / nx) % a.b;
    co0 = (id / (nx * a.b)) * a.cout_cta;
  };
  const uint32_t a_bytes = uint32_t(a.R) * kCB * 2;        // one halo: 8 slabs x R rows x 16 B
  const uint32_t b_bytes = uint32_t(a.cout_cta) * kCB * 2;  // cout_cta rows x 128 B
  uint8_t* a_base = smem;
  uint8_t* b_base = smem + kAStages * a_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(b_base + kBStages * b_bytes);
  uint64_t* full_a = bars;
  uint64_t* ready_a = bars + kAStages;
  uint64_t* empty_a = bars + 2 * kAStages;
  uint64_t* full_b = bars + 3 * kAStages;
  uint64_t* empty_b = full_b + kBStages;
  uint64_t* tmem_full = empty_b + kBStages;  // MMAs of a tile done
  uint64_t* tmem_empty = tmem_full + 1;      // its accumulators read by the epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&ready_a[s], kHaloThreads);
      mbar_init(&empty_a[s], 1);
    }
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(&full_b[s], 1);
      mbar_init(&empty_b[s], 1);
    }
    mbar_init(tmem_full, 1);
    mbar_init(tmem_empty, 4);
    fence_barrier_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
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
  pdl_wait();

  const int steps = ncb * a.k;  // (cb, tap) steps per tile
  if (warp == 0) {
    // ---------------- weight tiles: global step g = (tile, cb, tap)
    const int total = my_tiles * steps;
    for (int g = 0; g < total; ++g) {
      const int s = g % kBStages;
      if (g >= kBStages && !mbar_wait_warp(&empty_b[s], ((g / kBStages) + 1) & 1)) {
        if (lane == 0) atomicOr(a.err, 16);
        break;
      }
      if (elect_one()) {
        int l0, bb, co0;
        tile_of(g / steps, l0, bb, co0);
        const int i = g % steps, cb = i / a.k, t = i % a.k;
        uint8_t* dst = b_base + s * b_bytes;
        mbar_arrive_expect_tx(&full_b[s], b_bytes);
        for (int h = 0; h < a.nh; ++h)
          tma_load_2d(dst + h * a.nper * 128, &tmW, &full_b[s], t * a.cin + cb * kCB,
                      co0 + h * a.nper);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: the accumulators of one tile at a time
    const uint32_t idesc = idesc_f16_f32(kRows, a.nper);
    const uint32_t slab = uint32_t(a.R) * 16;
    bool ok = true;
    int gc = 0, g = 0;  // global halo and step counters
    for (int tl = 0; tl < my_tiles && ok; ++tl) {
      if (tl > 0 && !mbar_wait_warp(tmem_empty, (tl - 1) & 1)) {
        if (lane == 0) atomicOr(a.err, 32);
        break;
      }
      tc_fence_after();
      for (int cb = 0; cb < ncb && ok; ++cb, ++gc) {
        const int sa = gc % kAStages;
        if (!mbar_wait_warp(&ready_a[sa], (gc / kAStages) & 1)) {
          if (lane == 0) atomicOr(a.err, 32);
          ok = false;
          break;
        }
        const uint32_t ha = smem_u32(a_base + sa * a_bytes);
        for (int t = 0; t < a.k; ++t, ++g) {
          const int i = cb * a.k + t;
          const int sb = g % kBStages;
          if (!mbar_wait_warp(&full_b[sb], (g / kBStages) & 1)) {
            if (lane == 0) atomicOr(a.err, 64);
            ok = false;
            break;
          }
          tc_fence_after();
          if (elect_one()) {
            const uint32_t hb = smem_u32(b_base + sb * b_bytes);
#pragma unroll
            for (int kk = 0; kk < kCB / 16; ++kk) {
              for (int h = 0; h < a.nh; ++h) {
                const uint64_t bd = desc_k_sw128(hb + h * a.nper * 128 + kk * 32);
                for (int j = 0; j < a.ms; ++j) {
                  // sub-tile j starts 128 rows into the shared halo
                  const uint64_t ad = desc_k_interleave(
                      ha + 2 * kk * slab + (j * kRows + t * a.dil) * 16, slab);
                  umma_f16(tmem + j * a.acc_stride + h * a.nper, ad, bd, idesc, (i | kk) != 0);
                }
              }
            }
            umma_commit(&empty_b[sb]);
          }
          __syncwarp();
        }
        if (ok) {
          if (elect_one()) umma_commit(&empty_a[sa]);
          __syncwarp();
        }
      }
      if (ok) {
        if (elect_one()) umma_commit(tmem_full);
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
      if (!mbar_wait(&full_a[s], (gi / kAStages) & 1)) {
        if (tt == 0) atomicOr(a.err, 4096);
      }
      if (a.alpha) {
        uint8_t* halos = a_base + s * a_bytes;
        const int cb = gi % ncb;
        for (int c = tt; c < 8 * a.R; c += kHaloThreads) {
          const int gq = c / a.R;
          const int ch = cb * kCB + gq * 8;
          uint4* p = reinterpret_cast<uint4*>(halos) + c;
          uint4 u = *p;
          snake8(u, a.alpha + ch, a.brecip + ch);
          *p = u;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
      mbar_arrive(&ready_a[s]);
      if (warp == kHaloWarp0 && gi + kAStages - 1 < total) issue(gi + kAStages - 1);
    }
  } else {
    // ---------------- epilogue (warps 2..5: TMEM lane quadrant = warp % 4), one tile at a time
    const int quad = warp & 3;
    // 64 columns per TMEM wait; the residual of the next 64 columns is read while this batch
    // is finished, so the row's residual loads overlap instead of adding up
    auto finish16 = [&](float* v, const uint4* rr, int c0, int co0, size_t row, bool live) {
      if (!live) return;
      if (a.bias) {
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
    for (int tl = 0; tl < my_tiles; ++tl) {
      if (!mbar_wait(tmem_full, tl & 1) && lane == 0) atomicOr(a.err, 8192);
      tc_fence_after();
      int l0, bb, co0;
      tile_of(tl, l0, bb, co0);
      for (int j = 0; j < a.ms; ++j) {
        const int l = l0 + j * kRows + quad * 32 + lane;
        const bool live = l < a.len;
        const size_t row = ((size_t)bb * a.len + (live ? l : 0)) * a.cout + co0;
        const uint32_t acc = tmem + (uint32_t(quad * 32) << 16) + uint32_t(j * a.acc_stride);
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
      if (lane == 0) mbar_arrive(tmem_empty);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
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
  a.acc_stride = 32;
  while (a.acc_stride < a.cout_cta) a.acc_stride *= 2;
  a.tmem_cols = a.acc_stride * a.ms;
  // one halo for all sub-tiles: ms * 128 + (k-1)*dil rows, loaded as nrb boxes of H rows
  // (a box is at most 256 rows; H a multiple of 8 keeps every box 128-byte aligned)
  {
    const int need = kRows * a.ms + (r.k - 1) * r.dil;
    a.nrb = need > 256 ? 2 : 1;
    a.H = ((need + a.nrb - 1) / a.nrb + 7) / 8 * 8;
    a.R = a.H * a.nrb;
  }
  // ring depths: the weight tiles are the steady stream (one per tap), halos one per 64 input
  // channels; fill what fits in 224 KB, at least two of each
  {
    const size_t halo = size_t(a.R) * kCB * 2, wt = size_t(a.cout_cta) * kCB * 2;
    const size_t budget = 224 * 1024;
    a.as = 2;
    a.bs = int(std::min<size_t>(4, (budget - 2 * halo) / wt));
    if (a.bs < 2) a.bs = 2;
    if (a.bs >= 4 && 3 * halo + 4 * wt <= budget) a.as = 3;
    // TTS_CONV_AS / TTS_CONV_BS override the ring depths (A/B measurement)
    const char* va = getenv("TTS_CONV_AS");
    const char* vb = getenv("TTS_CONV_BS");
    if (va && *va) a.as = std::max(2, std::min(4, atoi(va)));
    if (vb && *vb) a.bs = std::max(2, std::min(6, atoi(vb)));
  }
  a.bias = r.bias;
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
                        uint64_t(r.k) * r.cin * 2, kCB, a.nper, true)) {
    set_error("conv1d: weight tensor map rejected");
    return cudaErrorInvalidValue;
  }
  const size_t smem = size_t(a.as) * a.R * kCB * 2 + size_t(a.bs) * a.cout_cta * kCB * 2 +
                      1024 + 256;
  {
    // The opt-in shared-memory limit is a per-device function attribute.
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !done[dev]) {
      cudaFuncSetAttribute(conv_nlc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      done[dev] = true;
    }
  }
  if (smem > 227 * 1024) {
    set_error("conv1d: shared memory plan exceeds 227 KB");
    return cudaErrorInvalidValue;
  }
  cudaLaunchConfig_t cfg{};
  // persistent: one CTA per SM (or per tile when there are fewer), each looping over tiles
  const long long ntiles = (long long)((r.len + kRows * a.ms - 1) / (kRows * a.ms)) * r.b *
                           (r.cout / a.cout_cta);
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (ntiles > (1ll << 31) - 1) {
    set_error("conv1d: too many tiles");
    return cudaErrorInvalidValue;
  }
  cfg.gridDim = dim3(unsigned(std::min<long long>(ntiles, std::max(1, sms))), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = r.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, conv_nlc_kernel, tmX, tmW, a);
}

}  // namespace tts
