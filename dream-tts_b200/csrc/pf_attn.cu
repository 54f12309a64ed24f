// Prompt attention on tcgen05 for the layer-major prefill (the t > 1 branch of Stack::forward,
// crates/qwen3tts/src/qwen3.rs:409-444: causal softmax(q.k) v per head, GQA 2, the scale folded
// into q's norm weight; K and V already normed/rotated and appended to the pages).
//
// One CTA per (query block of <= 64 new positions of one lane, kv head): its 128 query rows are
// the block's positions for the group's 2 q heads (row m: head 2h + m / 64, position m % 64), so
// the scores S = Q.K^T put one query row per TMEM lane and the softmax needs no cross-thread
// reduction. The lane's keys (its cached prefix and the prompt, up to 256 positions) are at most
// two 128-position chunks: both chunks' scores stay in TMEM, so an exact two-pass softmax (max
// and sum, then p) replaces the running rescale of the output, and O = P0.V0 + P1.V1 accumulates
// in TMEM. K and V come from the pages by TMA (runs of rows within a page, 128-byte swizzle);
// P is written over the K tiles once the scores are out.
//
// 128 threads: thread t owns query row t (TMEM lane t) through the softmax and the output; one
// elected lane of warp 0 issues the copies and the MMAs. Every wait is bounded (error flags).
#include <mutex>

#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

namespace {

constexpr int kPaRows = 128;    // query rows per CTA (MMA M): 64 positions x 2 heads
constexpr int kPaChunk = 128;   // keys per chunk (MMA N of the scores)
constexpr int kPaMaxKeys = 256;  // two chunks
constexpr int kPaThreads = 128;

// one operand tile: 128 rows x 128 f16 as two 64-column halves, 128-byte swizzled rows
struct PaTile {
  uint8_t d[2][kPaChunk * 128];
};
struct PaSmem {
  PaTile q;      // A of S: query rows x dims
  PaTile k[2];   // B of S: keys x dims; then A of O: P as query rows x keys
  PaTile v[2];   // B of O (MN-major): keys x dims
  uint64_t tma_bar, s_bar, o_bar;
  uint32_t tmem;
};

TTS_DEV uint32_t pa_sw128(int r, int e) {  // byte offset of (row r, column e < 64) in a half
  return uint32_t(r) * 128u + ((uint32_t((e >> 3) ^ (r & 7))) << 4) + uint32_t(e & 7) * 2u;
}

struct PaArgs {
  const float* q;       // [rows][heads][128] (normed, rotated, scale folded)
  const int4* blocks;   // [n] (lane, first row, first new position offset, rows in block)
  const int* positions; // [lanes] positions held before this prefill (the prompt starts there)
  const int* bt;        // [lanes][max_blocks]
  int max_blocks, bs, num_blocks, box;
  int heads, n_kv;
  __half* out;          // [rows][heads][128]
  int* err;
};

__global__ void __launch_bounds__(kPaThreads, 1)
    pf_attn_kernel(const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const PaArgs a) {
  extern __shared__ uint8_t smem_raw[];
  PaSmem& S = *reinterpret_cast<PaSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                         ~uintptr_t(1023));
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int4 blk4 = a.blocks[blockIdx.x];
  const int b = blk4.x, row0 = blk4.y, i0 = blk4.z, nq = blk4.w;
  const int h = blockIdx.y;
  const int start = a.positions[b];
  const int kmax = start + i0 + nq;  // keys [0, kmax) are visible to this block
  const int nch = (kmax + kPaChunk - 1) / kPaChunk;
  if (kmax > kPaMaxKeys || nq < 1 || nq > 64) {
    if (t == 0 && a.err) atomicOr(a.err, kFlagSpanRange);
    return;  // uniform across the CTA, before any barrier or allocation
  }

  if (t == 0) {
    mbar_init(&S.tma_bar, 1);
    mbar_init(&S.s_bar, 1);
    mbar_init(&S.o_bar, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 0) {
    tmem_alloc(&S.tmem, 512);
    tmem_relinquish();
  }
  // zero the K and V tiles of the chunks in use (rows past kmax stay zero: no NaN reaches P.V),
  // and write Q as f16 in the swizzled layout: thread t fills query row t
  for (int c = 0; c < nch; ++c)
    for (int u = t; u < 2 * kPaChunk * 128 / 16; u += kPaThreads) {
      reinterpret_cast<uint4*>(&S.k[c].d[0][0])[u] = make_uint4(0, 0, 0, 0);
      reinterpret_cast<uint4*>(&S.v[c].d[0][0])[u] = make_uint4(0, 0, 0, 0);
    }
  {
    const int g = t >> 6, i = t & 63;
    const bool live = i < nq;
    const float* src = a.q + ((size_t)(row0 + i) * a.heads + 2 * h + g) * 128;
#pragma unroll 4
    for (int e8 = 0; e8 < 16; ++e8) {  // 8 dims at a time
      uint4 pk = make_uint4(0, 0, 0, 0);
      if (live) {
        const float4 x0 = __ldcg(reinterpret_cast<const float4*>(src + e8 * 8));
        const float4 x1 = __ldcg(reinterpret_cast<const float4*>(src + e8 * 8 + 4));
        __half2* p2 = reinterpret_cast<__half2*>(&pk);
        p2[0] = __floats2half2_rn(x0.x, x0.y);
        p2[1] = __floats2half2_rn(x0.z, x0.w);
        p2[2] = __floats2half2_rn(x1.x, x1.y);
        p2[3] = __floats2half2_rn(x1.z, x1.w);
      }
      const int e = e8 * 8;
      *reinterpret_cast<uint4*>(&S.q.d[e >> 6][pa_sw128(t, e & 63)]) = pk;
    }
  }
  fence_proxy_async();  // the generic writes above before the copies and MMAs that follow
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem;
  bool ok = true;

  if (warp == 0) {
    // ---- K and V chunks: runs of `box` rows within a page, both 64-dim halves
    if (elect_one()) {
      uint32_t bytes = 0;
      const int nbox = kPaChunk / a.box;
      for (int c = 0; c < nch; ++c)
        for (int j = 0; j < nbox; ++j) {
          const int pos = c * kPaChunk + j * a.box;
          if (pos >= kmax) break;
          const int pg = pos / a.bs;
          const int blk = pg < a.max_blocks ? a.bt[(size_t)b * a.max_blocks + pg] : -1;
          if (blk < 0 || blk >= a.num_blocks) {
            if (a.err) atomicOr(a.err, kFlagPageRange);
            continue;  // rows stay zero
          }
          bytes += uint32_t(a.box) * 128u * 4u;
        }
      mbar_arrive_expect_tx(&S.tma_bar, bytes);
      for (int c = 0; c < nch; ++c)
        for (int j = 0; j < nbox; ++j) {
          const int pos = c * kPaChunk + j * a.box;
          if (pos >= kmax) break;
          const int pg = pos / a.bs;
          const int blk = pg < a.max_blocks ? a.bt[(size_t)b * a.max_blocks + pg] : -1;
          if (blk < 0 || blk >= a.num_blocks) continue;
          const int row = (blk * a.n_kv + h) * a.bs + pos % a.bs;
          const int r = j * a.box;
          tma_load_2d(&S.k[c].d[0][r * 128], &tmK, &S.tma_bar, 0, row);
          tma_load_2d(&S.k[c].d[1][r * 128], &tmK, &S.tma_bar, 64, row);
          tma_load_2d(&S.v[c].d[0][r * 128], &tmV, &S.tma_bar, 0, row);
          tma_load_2d(&S.v[c].d[1][r * 128], &tmV, &S.tma_bar, 64, row);
        }
    }
    __syncwarp();
    ok = mbar_wait_warp(&S.tma_bar, 0);
    if (ok) {
      // the last box may run past the visible keys into rows this prefill has not written (or
      // stale ones): zero those V rows, whose p is 0, so that no NaN enters P.V (their K rows
      // only reach masked scores)
      const int c = nch - 1;
      const int r_lo = kmax - c * kPaChunk;
      const int r_hi = min(kPaChunk, (r_lo + a.box - 1) / a.box * a.box);
      for (int u = lane; u < (r_hi - r_lo) * 16; u += 32) {
        const int r = r_lo + (u >> 4), piece = u & 15;
        *reinterpret_cast<uint4*>(&S.v[c].d[piece >> 3][r * 128 + (piece & 7) * 16]) =
            make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async();
      __syncwarp();
    }
    // ---- S_c = Q . K_c^T into TMEM columns [128 c, 128 c + 128)
    if (ok) {
      tc_fence_after();
      if (elect_one()) {
        const uint32_t idesc = idesc_f16_f32(kPaRows, kPaChunk);
        const uint32_t qb[2] = {smem_u32(&S.q.d[0][0]), smem_u32(&S.q.d[1][0])};
        for (int c = 0; c < nch; ++c) {
          const uint32_t kb[2] = {smem_u32(&S.k[c].d[0][0]), smem_u32(&S.k[c].d[1][0])};
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16(tmem + uint32_t(c * kPaChunk), desc_k_sw128(qb[kk >> 2] + (kk & 3) * 32),
                     desc_k_sw128(kb[kk >> 2] + (kk & 3) * 32), idesc, kk > 0);
        }
        umma_commit(&S.s_bar);
      }
      __syncwarp();
    }
  }
  // ---- softmax of query row t over the visible keys (exact: max and sum, then p)
  ok = __syncthreads_and(ok);
  if (ok) ok = mbar_wait(&S.s_bar, 0);
  ok = __syncthreads_and(ok);
  tc_fence_after();
  const int i = t & 63;
  const int qpos = start + i0 + i;  // this row's position; keys <= qpos are visible
  const bool live = i < nq;
  const uint32_t lane_addr = tmem + (uint32_t(warp * 32) << 16);
  float mx = -INFINITY, l = 0.f;
  if (ok) {
    for (int c = 0; c < nch; ++c)
      for (int c0 = 0; c0 < kPaChunk; c0 += 64) {
        float v[4][16];
        const uint32_t g0 = lane_addr + uint32_t(c * kPaChunk + c0);
        tmem_ld16x4(g0, g0 + 16, g0 + 32, g0 + 48, v);
        float cm = -INFINITY;
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (c * kPaChunk + c0 + p * 16 + e <= qpos) cm = fmaxf(cm, v[p][e]);
        if (cm > mx) {
          l = (mx == -INFINITY) ? 0.f : l * expf(mx - cm);
          mx = cm;
        }
        float sum = 0.f;
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (c * kPaChunk + c0 + p * 16 + e <= qpos) sum += expf(v[p][e] - mx);
        l += sum;
      }
    // p = exp(s - max) / sum as f16, written over the K tiles as the A operand of O (row t,
    // keys as columns); rows past the block and keys past the row's position are 0
    const float inv = (live && l > 0.f) ? 1.f / l : 0.f;
    for (int c = 0; c < nch; ++c)
      for (int c0 = 0; c0 < kPaChunk; c0 += 64) {
        float v[4][16];
        const uint32_t g0 = lane_addr + uint32_t(c * kPaChunk + c0);
        tmem_ld16x4(g0, g0 + 16, g0 + 32, g0 + 48, v);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          uint4 pk[2];
          __half2* p2 = reinterpret_cast<__half2*>(pk);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int k0 = c * kPaChunk + c0 + p * 16 + 2 * e;
            const float p0 = k0 <= qpos ? expf(v[p][2 * e] - mx) * inv : 0.f;
            const float p1 = k0 + 1 <= qpos ? expf(v[p][2 * e + 1] - mx) * inv : 0.f;
            p2[e] = __floats2half2_rn(p0, p1);
          }
          const int col = c0 + p * 16;  // key column within the chunk
          *reinterpret_cast<uint4*>(&S.k[c].d[col >> 6][pa_sw128(t, col & 63)]) = pk[0];
          *reinterpret_cast<uint4*>(&S.k[c].d[col >> 6][pa_sw128(t, (col & 63) + 8)]) = pk[1];
        }
      }
  }
  fence_proxy_async();
  tc_fence_before();
  ok = __syncthreads_and(ok);
  // ---- O = sum_c P_c . V_c into TMEM columns [256, 384) (V as the MN-major B operand)
  if (ok && warp == 0) {
    tc_fence_after();
    if (elect_one()) {
      const uint32_t idesc_o = idesc_f16_f32(kPaRows, 128) | (1u << 16);  // B (V) MN-major
      for (int c = 0; c < nch; ++c) {
        const uint32_t pb[2] = {smem_u32(&S.k[c].d[0][0]), smem_u32(&S.k[c].d[1][0])};
        const uint32_t vb = smem_u32(&S.v[c].d[0][0]);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16(tmem + 256, desc_k_sw128(pb[kk >> 2] + (kk & 3) * 32),
                   smem_desc(vb + kk * 2048, kPaChunk * 128, 1024, 2), idesc_o, (c | kk) != 0);
      }
      umma_commit(&S.o_bar);
    }
    __syncwarp();
  }
  if (ok) ok = mbar_wait(&S.o_bar, 0);
  // one verdict for the whole CTA: the TMEM loads below are warp-collective, and each thread's
  // bounded wait could give up on its own
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (ok) {
    // every lane of a warp issues the TMEM loads (warp-collective, aligned); only rows of the
    // block store
    __half* dst = a.out + ((size_t)(row0 + i) * a.heads + 2 * h + (t >> 6)) * 128;
    for (int c0 = 0; c0 < 128; c0 += 64) {
      float v[4][16];
      const uint32_t g0 = lane_addr + 256u + uint32_t(c0);
      tmem_ld16x4(g0, g0 + 16, g0 + 32, g0 + 48, v);
      if (live) {
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          uint4 pk[2];
          __half2* p2 = reinterpret_cast<__half2*>(pk);
#pragma unroll
          for (int e = 0; e < 8; ++e) p2[e] = __floats2half2_rn(v[p][2 * e], v[p][2 * e + 1]);
          reinterpret_cast<uint4*>(dst + c0 + p * 16)[0] = pk[0];
          reinterpret_cast<uint4*>(dst + c0 + p * 16)[1] = pk[1];
        }
      }
    }
  }
  if (!ok && t == 0 && a.err) atomicOr(a.err, kFlagAttnWait);
  // nothing may still write TMEM or shared memory: on a failed wait, wait (bounded) for the
  // copies and MMAs that were issued
  if (!ok && t == 0) {
    mbar_wait(&S.tma_bar, 0, 100000000ull);
    mbar_wait(&S.s_bar, 0, 100000000ull);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

bool pf_attn_supported(int heads, int n_kv, int block_size, int max_span) {
  return heads == 2 * n_kv && block_size % 8 == 0 && max_span <= kPaMaxKeys && max_span >= 1;
}

cudaError_t launch_pf_attn(const PfAttnRequest& r, cudaStream_t st) {
  if (!pf_attn_supported(r.heads, r.n_kv, r.block_size, r.max_span)) {
    set_error("prefill attention: gqa 2, block_size % 8 == 0 and spans <= 256 only");
    return cudaErrorInvalidValue;
  }
  int box = 8;
  while (box < 128 && r.block_size % (box * 2) == 0) box *= 2;
  const uint64_t rows = uint64_t(r.num_blocks) * r.n_kv * r.block_size;
  CUtensorMap tmK, tmV;
  if (!make_tmap_2d_f16(&tmK, r.k_pool, 128, rows, 256, 64, uint32_t(box), true) ||
      !make_tmap_2d_f16(&tmV, r.v_pool, 128, rows, 256, 64, uint32_t(box), true)) {
    set_error("prefill attention: cuTensorMapEncodeTiled failed (pools must be 16-byte aligned)");
    return cudaErrorInvalidValue;
  }
  PaArgs a{};
  a.q = r.q;
  a.blocks = reinterpret_cast<const int4*>(r.blocks);
  a.positions = r.positions;
  a.bt = r.block_table;
  a.max_blocks = r.max_blocks;
  a.bs = r.block_size;
  a.num_blocks = r.num_blocks;
  a.box = box;
  a.heads = r.heads;
  a.n_kv = r.n_kv;
  a.out = r.out;
  a.err = r.err;
  const size_t smem = sizeof(PaSmem) + 1024;
  {
    // the opt-in shared-memory limit is a per-device function attribute
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !done[dev]) {
      cudaFuncSetAttribute(pf_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      done[dev] = true;
    }
  }
  pf_attn_kernel<<<dim3(r.n_blocks, r.n_kv), kPaThreads, smem, st>>>(tmK, tmV, a);
  return cudaGetLastError();
}

}  // namespace tts
