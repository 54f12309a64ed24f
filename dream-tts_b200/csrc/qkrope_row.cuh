// QK-norm + RoPE + paged KV append for one (lane, head) row of 128 values held by a warp,
// four per thread (thread t owns dims 4t .. 4t+3).
//
// Restates crates/qwen3tts/src/qwen3.rs:358-394 (rms_norm over the head dim, then
// candle_nn::rotary_emb::rope's rotate_half form: dims i and i + 64 rotate together) and
// crates/tts-nn/src/qkrope.rs:26-69 (the fused kernel writes k and v as f16 into the cache at
// the lane's position). Used by the QKV GEMM's epilogue and by the standalone op.
#pragma once
#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

// head < heads: q head -> q_out (f32). heads <= head < heads + n_kv: k head -> K page.
// Otherwise: v head -> V page (no norm, no rotation).
__device__ __forceinline__ void qkrope_row(const QkRopeArgs& q, int head, int j, int lane,
                                           float v[4]) {
  // Positions and page numbers are device data: a row outside the RoPE table, the lane's
  // block table or the pool is skipped and flagged, never written out of bounds.
  // (j, head) is the same for the whole warp, so the early return is warp-uniform.
  const int pos = q.positions[j];
  if (pos < 0 || pos >= q.rope_len || pos >= q.max_blocks * q.block_size) {
    if (lane == 0 && q.err) atomicOr(q.err, kFlagRopeRange);
    return;
  }
  int blk = 0;
  const int off = pos % q.block_size;
  if (head >= q.heads) {
    blk = q.block_table[(size_t)j * q.max_blocks + pos / q.block_size];
    if (blk < 0 || blk >= q.num_blocks) {
      if (lane == 0 && q.err) atomicOr(q.err, kFlagRopeRange);
      return;
    }
  }
  if (head < q.heads + q.n_kv) {
    const float* w = q.norms + (head < q.heads ? 0 : 128) + 4 * lane;
    float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
    ss = warp_sum(ss);
    const float rms = sqrtf(ss / 128.0f + q.eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = v[i] / rms * w[i];
    float pr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) pr[i] = __shfl_xor_sync(0xffffffffu, v[i], 16);
    const int fi = (lane & 15) * 4;
    const float* ct = q.cos_t + (size_t)pos * 64 + fi;
    const float* st = q.sin_t + (size_t)pos * 64 + fi;
    float o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = lane < 16 ? v[i] * ct[i] - pr[i] * st[i] : v[i] * ct[i] + pr[i] * st[i];
    if (head < q.heads) {
      float4* dst =
          reinterpret_cast<float4*>(q.q_out + ((size_t)j * q.heads + head) * 128 + 4 * lane);
      *dst = make_float4(o[0], o[1], o[2], o[3]);
    } else {
      const int h = head - q.heads;
      __half2* dst = reinterpret_cast<__half2*>(
          q.k_pool + (((size_t)blk * q.n_kv + h) * q.block_size + off) * 128 + 4 * lane);
      dst[0] = __floats2half2_rn(o[0], o[1]);
      dst[1] = __floats2half2_rn(o[2], o[3]);
    }
  } else {
    const int h = head - q.heads - q.n_kv;
    __half2* dst = reinterpret_cast<__half2*>(
        q.v_pool + (((size_t)blk * q.n_kv + h) * q.block_size + off) * 128 + 4 * lane);
    dst[0] = __floats2half2_rn(v[0], v[1]);
    dst[1] = __floats2half2_rn(v[2], v[3]);
  }
}

// qkrope_row with the row's operands already in shared memory (the decode GEMM stages the
// per-step QkRopeArgs::rows_desc / rows_rope and the norm weights ahead of its epilogue): the
// same arithmetic in the same order, no global loads. d = {position or -1, page or -1, offset
// in the page}; rows out of range were flagged when the operands were built.
__device__ __forceinline__ void qkrope_row_staged(const QkRopeArgs& q, int head, int j, int lane,
                                                  float v[4], int4 d, const float* rope_row,
                                                  const float* norms) {
  if (d.x < 0) return;                       // position outside the table (warp-uniform)
  if (head >= q.heads && d.y < 0) return;    // page outside the pool: k and v rows skipped
  const int blk = d.y, off = d.z;
  if (head < q.heads + q.n_kv) {
    const float* w = norms + (head < q.heads ? 0 : 128) + 4 * lane;
    float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
    ss = warp_sum(ss);
    const float rms = sqrtf(ss / 128.0f + q.eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = v[i] / rms * w[i];
    float pr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) pr[i] = __shfl_xor_sync(0xffffffffu, v[i], 16);
    const int fi = (lane & 15) * 4;
    const float* ct = rope_row + fi;
    const float* st = rope_row + 64 + fi;
    float o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = lane < 16 ? v[i] * ct[i] - pr[i] * st[i] : v[i] * ct[i] + pr[i] * st[i];
    if (head < q.heads) {
      float4* dst =
          reinterpret_cast<float4*>(q.q_out + ((size_t)j * q.heads + head) * 128 + 4 * lane);
      *dst = make_float4(o[0], o[1], o[2], o[3]);
    } else {
      const int h = head - q.heads;
      __half2* dst = reinterpret_cast<__half2*>(
          q.k_pool + (((size_t)blk * q.n_kv + h) * q.block_size + off) * 128 + 4 * lane);
      dst[0] = __floats2half2_rn(o[0], o[1]);
      dst[1] = __floats2half2_rn(o[2], o[3]);
    }
  } else {
    const int h = head - q.heads - q.n_kv;
    __half2* dst = reinterpret_cast<__half2*>(
        q.v_pool + (((size_t)blk * q.n_kv + h) * q.block_size + off) * 128 + 4 * lane);
    dst[0] = __floats2half2_rn(v[0], v[1]);
    dst[1] = __floats2half2_rn(v[2], v[3]);
  }
}

// The global operands of up to four token rows j[0..n) of one head (positions, page numbers,
// RoPE rows, the head's norm weights), fetched ahead of qkrope_apply4. The fetch has two
// levels (page numbers and RoPE rows depend on the positions), so a caller can issue the
// positions early and the rest later. Positions and block tables are device data written by
// earlier kernels (read through L2); the RoPE tables and norm weights are constant.
struct QkRowsPre {
  int pos[4], blk[4];
  bool ok[4];
  float4 ct[4], st[4], w4;
};

__device__ __forceinline__ void qkrope_fetch_pos4(const QkRopeArgs& q, const int j[4], int n,
                                                  QkRowsPre& p) {
#pragma unroll
  for (int u = 0; u < 4; ++u) p.pos[u] = u < n ? __ldcg(q.positions + j[u]) : -1;
}

__device__ __forceinline__ void qkrope_fetch_rest4(const QkRopeArgs& q, int head, const int j[4],
                                                   int n, int lane, QkRowsPre& p) {
  const bool rot = head < q.heads + q.n_kv;  // q and k heads are normed and rotated
  const int fi = (lane & 15) * 4;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int pos = p.pos[u];
    p.ok[u] = u < n && pos >= 0 && pos < q.rope_len && pos < q.max_blocks * q.block_size;
    p.blk[u] = 0;
    if (p.ok[u] && head >= q.heads)
      p.blk[u] = __ldcg(q.block_table + (size_t)j[u] * q.max_blocks + pos / q.block_size);
    p.ct[u] = p.st[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (p.ok[u] && rot) {
      p.ct[u] = __ldg(reinterpret_cast<const float4*>(q.cos_t + (size_t)pos * 64 + fi));
      p.st[u] = __ldg(reinterpret_cast<const float4*>(q.sin_t + (size_t)pos * 64 + fi));
    }
  }
  p.w4 = rot ? __ldg(reinterpret_cast<const float4*>(q.norms + (head < q.heads ? 0 : 128) + 4 * lane))
             : make_float4(0.f, 0.f, 0.f, 0.f);
}

// qkrope_row on up to four token rows of one head with operands from the fetches above.
__device__ __forceinline__ void qkrope_apply4(const QkRopeArgs& q, int head, const int j[4], int n,
                                              int lane, float v[4][4], const QkRowsPre& p) {
  const bool rot = head < q.heads + q.n_kv;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    if (u >= n) break;  // n is warp-uniform
    if (!p.ok[u] || (head >= q.heads && (p.blk[u] < 0 || p.blk[u] >= q.num_blocks))) {
      if (lane == 0 && q.err) atomicOr(q.err, kFlagRopeRange);
      continue;
    }
    const int off = p.pos[u] % q.block_size;
    float* x = v[u];
    if (rot) {
      float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
      ss = warp_sum(ss);
      const float rms = sqrtf(ss / 128.0f + q.eps);
      x[0] = x[0] / rms * p.w4.x;
      x[1] = x[1] / rms * p.w4.y;
      x[2] = x[2] / rms * p.w4.z;
      x[3] = x[3] / rms * p.w4.w;
      float pr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pr[i] = __shfl_xor_sync(0xffffffffu, x[i], 16);
      const float c4[4] = {p.ct[u].x, p.ct[u].y, p.ct[u].z, p.ct[u].w};
      const float s4[4] = {p.st[u].x, p.st[u].y, p.st[u].z, p.st[u].w};
      float o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        o[i] = lane < 16 ? x[i] * c4[i] - pr[i] * s4[i] : x[i] * c4[i] + pr[i] * s4[i];
      if (head < q.heads) {
        float4* dst =
            reinterpret_cast<float4*>(q.q_out + ((size_t)j[u] * q.heads + head) * 128 + 4 * lane);
        *dst = make_float4(o[0], o[1], o[2], o[3]);
      } else {
        const int h = head - q.heads;
        __half2* dst = reinterpret_cast<__half2*>(
            q.k_pool + (((size_t)p.blk[u] * q.n_kv + h) * q.block_size + off) * 128 + 4 * lane);
        dst[0] = __floats2half2_rn(o[0], o[1]);
        dst[1] = __floats2half2_rn(o[2], o[3]);
      }
    } else {
      const int h = head - q.heads - q.n_kv;
      __half2* dst = reinterpret_cast<__half2*>(
          q.v_pool + (((size_t)p.blk[u] * q.n_kv + h) * q.block_size + off) * 128 + 4 * lane);
      dst[0] = __floats2half2_rn(x[0], x[1]);
      dst[1] = __floats2half2_rn(x[2], x[3]);
    }
  }
}


}  // namespace tts
