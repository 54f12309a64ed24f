// The decode step's small kernels: RMSNorm, standalone QK-norm/RoPE/append, SwiGLU, SnakeBeta,
// greedy argmax, code gather + embedding sum, position advance. Each is one coalesced pass;
// the talker step fuses most of them into the GEMM epilogues and keeps only RMSNorm, the code
// gather and the position advance as launches.
#include "pick_rule.cuh"
#include "qkrope_row.cuh"
#include "tts_common.cuh"
#include "tts_internal.h"

namespace tts {

namespace {

cudaError_t launch_ex(void (*kernel)(void*), dim3 grid, dim3 block, cudaStream_t st, bool pdl,
                      void** args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(kernel), args);
}

// a3: y = x / sqrt(mean(x^2) + eps) * w, one CTA per row (crates/tts-nn/src/lib.rs:1001-1003).
// Optionally zeroes a range of argmax keys so the heads GEMM that follows starts clean.
__global__ void __launch_bounds__(256) rms_norm_kernel(const float* x, const float* w, int dim,
                                                       float eps, float* y32, __half* y16,
                                                       unsigned long long* keys, int n_keys) {
  [[maybe_unused]] const unsigned long long tl_entry = TTS_TL_NOW();
  __shared__ float red[8];
  pdl_launch_dependents();
  pdl_wait();
  [[maybe_unused]] const unsigned long long tl_rel = TTS_TL_NOW();
  const int row = blockIdx.x;
  const float* xr = x + (size_t)row * dim;
  float ss = 0.f;
  for (int i = threadIdx.x * 4; i < dim; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float rms = sqrtf(red[0] / (float)dim + eps);
  for (int i = threadIdx.x * 4; i < dim; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    const float4 g = *reinterpret_cast<const float4*>(w + i);
    const float4 o = make_float4(v.x / rms * g.x, v.y / rms * g.y, v.z / rms * g.z,
                                 v.w / rms * g.w);
    if (y32) *reinterpret_cast<float4*>(y32 + (size_t)row * dim + i) = o;
    if (y16) {
      __half2* d = reinterpret_cast<__half2*>(y16 + (size_t)row * dim + i);
      d[0] = __floats2half2_rn(o.x, o.y);
      d[1] = __floats2half2_rn(o.z, o.w);
    }
  }
  if (keys) {
    for (int i = row * blockDim.x + threadIdx.x; i < n_keys; i += gridDim.x * blockDim.x)
      keys[i] = 0ull;
  }
#ifdef TTS_TIMELINE
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t_end = TTS_TL_NOW();
    timeline_recs<3>({kTlNorm | kTlEntry, kTlNorm | kTlReleased, kTlNorm | kTlEnd},
                     {tl_entry, tl_rel, t_end});
  }
#endif
}

// The deferred norm's first stage (the step input's rows): y16 = f16(x * w) and ss = the row's
// sum of squares; the projection that reads y16 divides its outputs by the row's RMS.
__global__ void __launch_bounds__(256) norm_defer_kernel(const float* x, const float* w, int dim,
                                                         __half* y16, float* ss_out) {
  [[maybe_unused]] const unsigned long long tl_entry = TTS_TL_NOW();
  __shared__ float red[8];
  pdl_launch_dependents();
  pdl_wait();
  [[maybe_unused]] const unsigned long long tl_rel = TTS_TL_NOW();
  const int row = blockIdx.x;
  const float* xr = x + (size_t)row * dim;
  float ss = 0.f;
  for (int i = threadIdx.x * 4; i < dim; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    const float4 g = *reinterpret_cast<const float4*>(w + i);
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    __half2* d = reinterpret_cast<__half2*>(y16 + (size_t)row * dim + i);
    d[0] = __floats2half2_rn(v.x * g.x, v.y * g.y);
    d[1] = __floats2half2_rn(v.z * g.z, v.w * g.w);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) ss_out[row] = t;
  }
#ifdef TTS_TIMELINE
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t_end = TTS_TL_NOW();
    timeline_recs<3>({kTlNorm | 0x10 | kTlEntry, kTlNorm | 0x10 | kTlReleased,
                      kTlNorm | 0x10 | kTlEnd},
                     {tl_entry, tl_rel, t_end});
  }
#endif
}

// a4 standalone: one warp per (lane, head) over qkv [lanes][(heads + 2 n_kv) * 128] f32.
__global__ void __launch_bounds__(128) qk_rope_kernel(const float* qkv, QkRopeArgs a, int lanes) {
  pdl_launch_dependents();
  pdl_wait();
  const int nh = a.heads + 2 * a.n_kv;
  const int wid = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (wid >= lanes * nh) return;
  const int j = wid / nh, head = wid % nh, lane = threadIdx.x & 31;
  const float4 x =
      *reinterpret_cast<const float4*>(qkv + ((size_t)j * nh + head) * 128 + 4 * lane);
  float v[4] = {x.x, x.y, x.z, x.w};
  qkrope_row(a, head, j, lane, v);
}

// a7: silu(g) * u (crates/tts-nn/src/fused.rs:311-318).
__global__ void swiglu_kernel(const float* g, const float* u, void* y, int y_f16, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
       i += (long)gridDim.x * blockDim.x) {
    const float x = g[i];
    const float r = (x / (1.0f + expf(-x))) * u[i];
    if (y_f16)
      static_cast<__half*>(y)[i] = __float2half_rn(r);
    else
      static_cast<float*>(y)[i] = r;
  }
}

// a12: SnakeBeta channels-last, x + brecip[c] * sin(alpha[c] * x)^2, f32 math
// (crates/tts-nn/src/fused.rs:564-600), f16 or f32 in and out, 8 channels per thread.
__global__ void snake_kernel(const void* x, int x_f16, const float* alpha, const float* brecip,
                             long rows, int chan, void* y, int y_f16) {
  const long n8 = rows * (long)chan / 8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8;
       i += (long)gridDim.x * blockDim.x) {
    const long e = i * 8;
    const int c0 = int(e % chan);
    float v[8];
    if (x_f16) {
      const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const __half*>(x) + e);
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 t = __half22float2(h[q]);
        v[2 * q] = t.x;
        v[2 * q + 1] = t.y;
      }
    } else {
      const float4 a0 = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + e);
      const float4 a1 = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + e + 4);
      v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w;
      v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float s = sinf(alpha[c0 + q] * v[q]);
      v[q] = v[q] + brecip[c0 + q] * (s * s);
    }
    if (y_f16) {
      uint4 o;
      __half2* h = reinterpret_cast<__half2*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) h[q] = __floats2half2_rn(v[2 * q], v[2 * q + 1]);
      *reinterpret_cast<uint4*>(static_cast<__half*>(y) + e) = o;
    } else {
      float* d = static_cast<float*>(y) + e;
      *reinterpret_cast<float4*>(d) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(d + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
  }
}

// a18: greedy pick per row, banned ids at -inf, ties to the highest index
// (crates/qwen3tts/src/talker.rs:182-189; Rust's max_by keeps the last maximum).
__global__ void __launch_bounds__(256) argmax_kernel(const float* logits, int n,
                                                     const uint8_t* banned, uint32_t* out) {
  __shared__ unsigned long long red[8];
  const int row = blockIdx.x;
  const float* lr = logits + (size_t)row * n;
  unsigned long long best = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = (banned && banned[i]) ? -INFINITY : lr[i];
    const unsigned long long key =
        (static_cast<unsigned long long>(float_order_key(v)) << 32) | unsigned(i);
    best = key > best ? key : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
    best = red[0] > best ? red[0] : best;
    out[row] = unsigned(best & 0xffffffffu);
  }
}

// The talker's greedy pick over rows of logits (sample_with_u with greedy on,
// crates/qwen3tts/src/talker.rs:154-189): the rule of pick_rule4 on every id, then the last of
// equal maxima. With `record` the pick joins the row's history as the decode loop's push does
// (talker.rs:984-996). One block per row; the rule's state is indexed by the row.
__global__ void __launch_bounds__(256) pick_kernel(const float* logits, int vocab, PickRule pick,
                                                   int record, uint32_t* out) {
  __shared__ unsigned long long red[8];
  const int row = blockIdx.x;
  const float* lr = logits + (size_t)row * vocab;
  unsigned long long best = 0;
  for (int id0 = threadIdx.x * 4; id0 < vocab; id0 += blockDim.x * 4) {
    const float4 x = *reinterpret_cast<const float4*>(lr + id0);
    float v[4] = {x.x, x.y, x.z, x.w};
    pick_rule4(pick, row, id0, v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const unsigned long long key =
          (static_cast<unsigned long long>(float_order_key(v[i])) << 32) | unsigned(id0 + i);
      best = key > best ? key : best;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
    best = red[0] > best ? red[0] : best;
    const unsigned c = unsigned(best & 0xffffffffu);
    out[row] = c;
    if (record) pick_record(pick, row, c);
  }
}

// Per decode step, each row's QK-rope operands, read once here instead of by every layer's
// QKV epilogue: the position (-1 when outside the RoPE table or the row's block table), the page
// holding it (-1 when the table entry is outside the pool), its offset in the page, and the
// RoPE table's cos and sin rows at that position. Out-of-range rows are flagged once; the
// epilogue skips them as qkrope_row does (a q head only needs the position).
__global__ void __launch_bounds__(64) qk_rows_kernel(QkRopeArgs a, int4* desc, float* rope) {
  pdl_launch_dependents();
  pdl_wait();
  const int j = blockIdx.x, t = threadIdx.x;
  const int pos = a.positions[j];
  const bool ok = pos >= 0 && pos < a.rope_len && pos < a.max_blocks * a.block_size;
  int blk = ok ? a.block_table[(size_t)j * a.max_blocks + pos / a.block_size] : -1;
  if (blk < 0 || blk >= a.num_blocks) blk = -1;
  if (t == 0) {
    desc[j] = make_int4(ok ? pos : -1, blk, ok ? pos % a.block_size : 0, 0);
    if ((!ok || blk < 0) && a.err) atomicOr(a.err, kFlagRopeRange);
  }
  rope[(size_t)j * 128 + t] = ok ? a.cos_t[(size_t)pos * 64 + t] : 0.f;
  rope[(size_t)j * 128 + 64 + t] = ok ? a.sin_t[(size_t)pos * 64 + t] : 0.f;
}

// Codes from the heads GEMM's argmax keys, and the next step's input as the sum of each
// codebook's embedding row (the talker's codec_embed lookup + the predictor's gather_sum,
// crates/qwen3tts/src/talker.rs:1019-1023, 528-550). Resets the keys for the next step.
__global__ void __launch_bounds__(256) keys_to_codes_kernel(const unsigned long long* keys,
                                                            int codebooks, int vocab,
                                                            const __half* embed,
                                                            const float* embed32, int dim,
                                                            uint32_t* codes, float* x_next,
                                                            unsigned long long* keys_reset,
                                                            int* positions, PickRule pick) {
  __shared__ int sc[64];
  pdl_launch_dependents();
  pdl_wait();
  const int row = blockIdx.x;
  // the step's last reader of the positions has finished: advance this lane's
  if (positions && threadIdx.x == 0) positions[row] += 1;
  // the pick rule's history (one codebook): the pick joins the row's history unless it is eos
  // (talker.rs:984-996), and the row has one more frame
  if (pick.vocab && threadIdx.x == 0) pick_record(pick, row, unsigned(keys[row] & 0xffffffffu));
  if (threadIdx.x < codebooks) {
    const unsigned c = unsigned(keys[(size_t)row * codebooks + threadIdx.x] & 0xffffffffu);
    sc[threadIdx.x] = int(c < unsigned(vocab) ? c : 0);
    if (codes) codes[(size_t)row * codebooks + threadIdx.x] = c;
  }
  __syncthreads();
  if (embed && x_next) {
    for (int d = threadIdx.x * 2; d < dim; d += blockDim.x * 2) {
      float s0 = 0.f, s1 = 0.f;
      for (int q = 0; q < codebooks; ++q) {
        const __half2 e = *reinterpret_cast<const __half2*>(
            embed + (((size_t)q * vocab + sc[q]) * dim + d));
        const float2 f = __half22float2(e);
        s0 += f.x;
        s1 += f.y;
      }
      x_next[(size_t)row * dim + d] = s0;
      x_next[(size_t)row * dim + d + 1] = s1;
    }
  } else if (embed32 && x_next) {
    // f32 tables (the predictor's resized rows, summed in codebook order)
    for (int d = threadIdx.x * 2; d < dim; d += blockDim.x * 2) {
      float s0 = 0.f, s1 = 0.f;
      for (int q = 0; q < codebooks; ++q) {
        const float2 f = *reinterpret_cast<const float2*>(
            embed32 + (((size_t)q * vocab + sc[q]) * dim + d));
        s0 += f.x;
        s1 += f.y;
      }
      x_next[(size_t)row * dim + d] = s0;
      x_next[(size_t)row * dim + d + 1] = s1;
    }
  }
  __syncthreads();
  if (keys_reset && threadIdx.x < codebooks)
    keys_reset[(size_t)row * codebooks + threadIdx.x] = 0ull;
}

__global__ void advance_positions_kernel(int* positions, int lanes) {
  pdl_launch_dependents();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < lanes) positions[i] += 1;
}

// Prefill rows as decode rows: row r is (lane, offset) map[r]; it gets the lane's block-table
// row and the position the lane's offset-th new row takes.
__global__ void prefill_rows_kernel(const int* map, int rows, const int* table, int max_blocks,
                                    const int* positions, int* table2, int* pos2) {
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x;
  if (r >= rows) return;
  const int lane = map[2 * r], off = map[2 * r + 1];
  for (int j = threadIdx.x; j < max_blocks; j += blockDim.x)
    table2[(size_t)r * max_blocks + j] = table[(size_t)lane * max_blocks + j];
  if (threadIdx.x == 0) pos2[r] = positions[lane] + off;
}

__global__ void advance_by_kernel(int* positions, const int* lens, int lanes) {
  pdl_launch_dependents();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < lanes) positions[i] += lens[i];
}

__global__ void cast_kernel(const float* x, __half* y, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
       i += (long)gridDim.x * blockDim.x)
    y[i] = __float2half_rn(x[i]);
}

int grid_for(long n, int block) {
  long g = (n + block - 1) / block;
  if (g > 148L * 16) g = 148L * 16;
  return int(g < 1 ? 1 : g);
}

}  // namespace

cudaError_t launch_rms_norm(const float* x, const float* w, int rows, int dim, float eps,
                            float* y32, __half* y16, unsigned long long* zero_keys, int n_keys,
                            bool pdl, cudaStream_t st) {
  if (dim % 4 != 0 || rows < 1) {
    set_error("rms_norm: dim must be a multiple of 4 and rows >= 1");
    return cudaErrorInvalidValue;
  }
  void* args[] = {(void*)&x, (void*)&w, (void*)&dim, (void*)&eps, (void*)&y32,
                  (void*)&y16, (void*)&zero_keys, (void*)&n_keys};
  return launch_ex(reinterpret_cast<void (*)(void*)>(rms_norm_kernel), dim3(rows), dim3(256),
                   st, pdl, args);
}

cudaError_t launch_norm_defer(const float* x, const float* w, int rows, int dim, __half* y16,
                              float* ss, bool pdl, cudaStream_t st) {
  if (dim % 4 != 0 || rows < 1) {
    set_error("norm_defer: dim must be a multiple of 4 and rows >= 1");
    return cudaErrorInvalidValue;
  }
  void* args[] = {(void*)&x, (void*)&w, (void*)&dim, (void*)&y16, (void*)&ss};
  return launch_ex(reinterpret_cast<void (*)(void*)>(norm_defer_kernel), dim3(rows), dim3(256),
                   st, pdl, args);
}

cudaError_t launch_qk_rope(const float* qkv, const QkRopeArgs& a, int lanes, bool pdl,
                           cudaStream_t st) {
  const int warps = lanes * (a.heads + 2 * a.n_kv);
  QkRopeArgs aa = a;
  void* args[] = {(void*)&qkv, (void*)&aa, (void*)&lanes};
  return launch_ex(reinterpret_cast<void (*)(void*)>(qk_rope_kernel), dim3((warps + 3) / 4),
                   dim3(128), st, pdl, args);
}

cudaError_t launch_swiglu(const float* g, const float* u, void* y, bool y_f16, long n,
                          cudaStream_t st) {
  swiglu_kernel<<<grid_for(n, 256), 256, 0, st>>>(g, u, y, y_f16 ? 1 : 0, n);
  return cudaGetLastError();
}

cudaError_t launch_snake(const void* x, bool x_f16, const float* alpha, const float* brecip,
                         long rows, int chan, void* y, bool y_f16, cudaStream_t st) {
  if (chan % 8 != 0) {
    set_error("snake_beta: channels must be a multiple of 8");
    return cudaErrorInvalidValue;
  }
  snake_kernel<<<grid_for(rows * chan / 8, 256), 256, 0, st>>>(x, x_f16 ? 1 : 0, alpha, brecip,
                                                               rows, chan, y, y_f16 ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_argmax(const float* logits, int rows, int n, const uint8_t* banned,
                          uint32_t* out, cudaStream_t st) {
  argmax_kernel<<<rows, 256, 0, st>>>(logits, n, banned, out);
  return cudaGetLastError();
}

cudaError_t launch_pick(const float* logits, int rows, const PickRule& pick, bool record,
                        uint32_t* out, cudaStream_t st) {
  if (pick.vocab < 32 || pick.vocab % 32) {
    set_error("talker_pick: vocab must be a positive multiple of 32");
    return cudaErrorInvalidValue;
  }
  pick_kernel<<<rows, 256, 0, st>>>(logits, pick.vocab, pick, record ? 1 : 0, out);
  return cudaGetLastError();
}

cudaError_t launch_qk_rows(const QkRopeArgs& a, int rows, int4* desc, float* rope, bool pdl,
                           cudaStream_t st) {
  QkRopeArgs args = a;
  void* params[] = {(void*)&args, (void*)&desc, (void*)&rope};
  return launch_ex(reinterpret_cast<void (*)(void*)>(qk_rows_kernel), dim3(rows), dim3(64), st,
                   pdl, params);
}

cudaError_t launch_keys_to_codes(const unsigned long long* keys, int rows, int codebooks,
                                 int vocab, const __half* embed, const float* embed32, int dim,
                                 uint32_t* codes, float* x_next, unsigned long long* keys_reset,
                                 int* positions, const PickRule* pick, bool pdl,
                                 cudaStream_t st) {
  PickRule pr = pick ? *pick : PickRule{};
  if (pr.vocab && codebooks != 1) {
    set_error("keys_to_codes: a pick rule takes one codebook");
    return cudaErrorInvalidValue;
  }
  if (codebooks > 64 || codebooks < 1 || ((embed || embed32) && dim % 2)) {
    set_error("keys_to_codes: 1..64 codebooks, even dim");
    return cudaErrorInvalidValue;
  }
  void* args[] = {(void*)&keys, (void*)&codebooks, (void*)&vocab,  (void*)&embed,
                  (void*)&embed32, (void*)&dim,    (void*)&codes, (void*)&x_next,
                  (void*)&keys_reset, (void*)&positions, (void*)&pr};
  return launch_ex(reinterpret_cast<void (*)(void*)>(keys_to_codes_kernel), dim3(rows),
                   dim3(256), st, pdl, args);
}

cudaError_t launch_advance_positions(int* positions, int lanes, bool pdl, cudaStream_t st) {
  void* args[] = {(void*)&positions, (void*)&lanes};
  return launch_ex(reinterpret_cast<void (*)(void*)>(advance_positions_kernel),
                   dim3((lanes + 127) / 128), dim3(128), st, pdl, args);
}

cudaError_t launch_prefill_rows(const int* map, int rows, const int* table, int max_blocks,
                                const int* positions, int* table2, int* pos2, cudaStream_t st) {
  void* args[] = {(void*)&map,       (void*)&rows,      (void*)&table, (void*)&max_blocks,
                  (void*)&positions, (void*)&table2,    (void*)&pos2};
  return launch_ex(reinterpret_cast<void (*)(void*)>(prefill_rows_kernel), dim3(rows), dim3(64),
                   st, true, args);
}

cudaError_t launch_advance_by(int* positions, const int* lens, int lanes, cudaStream_t st) {
  void* args[] = {(void*)&positions, (void*)&lens, (void*)&lanes};
  return launch_ex(reinterpret_cast<void (*)(void*)>(advance_by_kernel),
                   dim3((lanes + 127) / 128), dim3(128), st, true, args);
}

cudaError_t launch_cast_f32_f16(const float* x, __half* y, long n, cudaStream_t st) {
  cast_kernel<<<grid_for(n, 256), 256, 0, st>>>(x, y, n);
  return cudaGetLastError();
}

}  // namespace tts
