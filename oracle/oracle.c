/*
 * CPU oracle for the qwen3tts hot path — TEST INFRASTRUCTURE ONLY.
 *
 * This is a plain-C restatement of the arithmetic that dream-tts's portable CPU build
 * (`--no-default-features`) runs for the talker decode step and the codec's conv stack.
 * It is the checker that the CUDA kernels are compared against, and the timed CPU
 * baseline in bench.py. Nothing in the product library links, loads or calls it; only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg do.
 *
 * PARITY UNPINNED: the reference ships no golden vectors for these ops (its own tests
 * compare its Metal kernels against its CPU loops on random inputs), its Rust crates
 * cannot be built in this image (no cargo, no crates.io), and no checkpoint or fixture
 * tensors exist here. This restatement is instead cross-checked against independent
 * PyTorch-CPU formulas of the same operations (tests/test_oracle.py), and against the
 * structural identities the reference's own tests assert (polyphase transposed conv,
 * lane-window cache writes, channels-last vs channel-major conv).
 *
 * Each function cites the reference file:line it restates. Third-party arithmetic the
 * reference delegates to (candle-core / candle-nn 0.10.2: rms_norm, rotary_emb::rope,
 * softmax_last_dim; gemm 0.18/0.19 for CPU f16 matmul) is restated from its published
 * definition at the cited call site.
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp). All buffers are caller-owned, row-major.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#include <omp.h>
#include <immintrin.h>

typedef _Float16 f16;

static inline float h2f(uint16_t h) { f16 v; memcpy(&v, &h, 2); return (float)v; }
static inline uint16_t f2h(float f) { f16 v = (f16)f; uint16_t h; memcpy(&h, &v, 2); return h; }

int orc_num_threads(void) { return omp_get_max_threads(); }
void orc_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }

/* IEEE binary16 conversions, round-to-nearest-even (half::f16::from_f32 semantics). */
void orc_f32_to_f16(const float* x, uint16_t* y, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) y[i] = f2h(x[i]);
}
void orc_f16_to_f32(const uint16_t* x, float* y, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) y[i] = h2f(x[i]);
}

/*
 * a1. Proj::Half forward: y[m,n] = sum_k f16(x)[m,k] * W[n,k], f32 accumulate.
 *     crates/tts-nn/src/lib.rs:516-529 (x cast to f16 at :517, GEMM, cast to f32 at :528);
 *     Metal arm crates/tts-nn/src/skinny.rs:155-165 (f32 accumulate, f32 out).
 * W is given in the checkpoint's [out, in] layout (the reference transposes it to [in, out]
 * at load, lib.rs:1252-1269; the arithmetic is the same). round_f16 != 0 rounds the result
 * to f16 as the CPU arm's f16 matmul output does before its cast back to f32 (lib.rs:528);
 * 0 keeps f32 as the device arm does. The reduction order is fixed: eight interleaved f32
 * partial sums over k (fused multiply-adds), combined in order; outputs are computed in 4 x 4
 * blocks (dot4x4) without changing any output's arithmetic.
 */
/* Dot products of 4 rows of x with 4 rows of W (f32, k a multiple of 8), each with the
 * arithmetic of the scalar form: lane l of an 8-wide accumulator sums x[kk + l] * w[kk + l]
 * (fused multiply-add) over kk, then the lanes are added in order. 16 independent chains keep
 * the FMA units busy; the result of every (i, j) is the same as one chain at a time. */
static void dot4x4(const float* const xi[4], const float* const wj[4], int k, float out[4][4]) {
    __m256 acc[4][4];
    for (int r = 0; r < 4; r++)
        for (int c = 0; c < 4; c++) acc[r][c] = _mm256_setzero_ps();
    for (int kk = 0; kk < k; kk += 8) {
        __m256 xv[4], wv[4];
        for (int r = 0; r < 4; r++) xv[r] = _mm256_loadu_ps(xi[r] + kk);
        for (int c = 0; c < 4; c++) wv[c] = _mm256_loadu_ps(wj[c] + kk);
        for (int r = 0; r < 4; r++)
            for (int c = 0; c < 4; c++) acc[r][c] = _mm256_fmadd_ps(xv[r], wv[c], acc[r][c]);
    }
    for (int r = 0; r < 4; r++)
        for (int c = 0; c < 4; c++) {
            float l[8];
            _mm256_storeu_ps(l, acc[r][c]);
            float s = 0.f;
            for (int q = 0; q < 8; q++) s += l[q];
            out[r][c] = s;
        }
}

void orc_proj(const uint16_t* x, const uint16_t* w, float* y, int m, int k, int n, int round_f16) {
    float* xf = (float*)malloc(sizeof(float) * (size_t)m * k);
    for (int64_t i = 0; i < (int64_t)m * k; i++) xf[i] = h2f(x[i]);
    const int k8 = k - k % 8;
#pragma omp parallel
    {
        float* wr = (float*)malloc(sizeof(float) * (size_t)k * 4);
#pragma omp for schedule(static)
        for (int j0 = 0; j0 < n; j0 += 4) {
            const int nj = n - j0 < 4 ? n - j0 : 4;
            for (int c = 0; c < nj; c++) {
                const uint16_t* wj = w + (size_t)(j0 + c) * k;
                float* dst = wr + (size_t)c * k;
                int kk = 0;
                for (; kk + 8 <= k; kk += 8)  /* F16C: exact f16 -> f32 conversion, 8 at a time */
                    _mm256_storeu_ps(dst + kk,
                                     _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(wj + kk))));
                for (; kk < k; kk++) dst[kk] = h2f(wj[kk]);
            }
            for (int i0 = 0; i0 < m; i0 += 4) {
                const int ni = m - i0 < 4 ? m - i0 : 4;
                const float* xi[4];
                const float* wj[4];
                for (int r = 0; r < 4; r++) xi[r] = xf + (size_t)(i0 + (r < ni ? r : 0)) * k;
                for (int c = 0; c < 4; c++) wj[c] = wr + (size_t)(c < nj ? c : 0) * k;
                float o[4][4];
                dot4x4(xi, wj, k8, o);
                for (int r = 0; r < ni; r++)
                    for (int c = 0; c < nj; c++) {
                        float s = o[r][c];
                        if (k8 < k) {
                            /* a k that is not a multiple of 8: the scalar form's tail, lane
                               kk & 7, folded in after the full lanes */
                            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                            for (int kk = 0; kk < k8; kk++) acc[kk & 7] += xi[r][kk] * wj[c][kk];
                            for (int kk = k8; kk < k; kk++) acc[kk & 7] += xi[r][kk] * wj[c][kk];
                            s = 0.f;
                            for (int l = 0; l < 8; l++) s += acc[l];
                        }
                        y[(size_t)(i0 + r) * n + j0 + c] = round_f16 ? h2f(f2h(s)) : s;
                    }
            }
        }
        free(wr);
    }
    free(xf);
}

/*
 * a3. rms_norm over the last dim, f32: y = x / sqrt(mean(x^2) + eps) * w.
 *     crates/tts-nn/src/lib.rs:1001-1003 -> candle_nn::ops::rms_norm (CPU: sum of squares in
 *     f32, m = sqrt(sum/dim + eps), y = x / m * w).
 */
void orc_rms_norm(const float* x, const float* w, float* y, int64_t rows, int dim, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        const float* xr = x + r * dim;
        float s = 0.f;
        for (int i = 0; i < dim; i++) s += xr[i] * xr[i];
        float m = sqrtf(s / (float)dim + eps);
        for (int i = 0; i < dim; i++) y[r * dim + i] = xr[i] / m * w[i];
    }
}

/*
 * a17. RoPE table, half-split pairs, computed in f64 and rounded to f32.
 *      crates/tts-nn/src/lib.rs:1178-1205 (freq_i = base^(-2i/hd), phase = t * freq).
 */
void orc_rope_table(int len, int hd, double base, float* cos_out, float* sin_out) {
    int half = hd / 2;
    for (int t = 0; t < len; t++)
        for (int i = 0; i < half; i++) {
            double freq = 1.0 / pow(base, 2.0 * (double)i / (double)hd);
            double ph = (double)t * freq;
            cos_out[t * half + i] = (float)cos(ph);
            sin_out[t * half + i] = (float)sin(ph);
        }
}

/* candle_nn::rotary_emb::rope on one head vector (rotate_half form): pairs (i, i + hd/2). */
static void rope_one(float* v, const float* c, const float* s, int hd) {
    int half = hd / 2;
    for (int i = 0; i < half; i++) {
        float x1 = v[i], x2 = v[i + half];
        v[i] = x1 * c[i] - x2 * s[i];
        v[i + half] = x2 * c[i] + x1 * s[i];
    }
}

static void rms_one(const float* x, const float* w, float* y, int n, float eps) {
    float s = 0.f;
    for (int i = 0; i < n; i++) s += x[i] * x[i];
    float m = sqrtf(s / (float)n + eps);
    for (int i = 0; i < n; i++) y[i] = x[i] / m * w[i];
}

/*
 * a4. QK-norm + RoPE for one decode position per lane (the composed CPU form,
 *     crates/qwen3tts/src/qwen3.rs:358-394; fused form crates/tts-nn/src/qkrope.rs:26-69).
 *     qkv [b, (heads + 2 n_kv) hd] f32; norms [2, hd] (q weight already scaled by 1/sqrt(hd),
 *     qwen3.rs:82-87); cos/sin [positions, hd/2]; pos[b] the position written by each lane.
 *     Out: q [b, heads, hd] f32, k and v [b, n_kv, hd] f32 (the caller casts k and v to f16
 *     into its cache, qwen3.rs:391-392).
 */
void orc_qk_rope(const float* qkv, const float* norms, const float* cos_t, const float* sin_t,
                 const int* pos, int b, int heads, int n_kv, int hd, float eps,
                 float* q, float* k, float* v) {
    int width = (heads + 2 * n_kv) * hd, half = hd / 2;
#pragma omp parallel for schedule(static)
    for (int l = 0; l < b; l++) {
        const float* row = qkv + (size_t)l * width;
        const float* c = cos_t + (size_t)pos[l] * half;
        const float* s = sin_t + (size_t)pos[l] * half;
        for (int h = 0; h < heads; h++) {
            float* out = q + ((size_t)l * heads + h) * hd;
            rms_one(row + h * hd, norms, out, hd, eps);
            rope_one(out, c, s, hd);
        }
        for (int h = 0; h < n_kv; h++) {
            float* out = k + ((size_t)l * n_kv + h) * hd;
            rms_one(row + (heads + h) * hd, norms + hd, out, hd, eps);
            rope_one(out, c, s, hd);
            memcpy(v + ((size_t)l * n_kv + h) * hd, row + (heads + n_kv + h) * hd, sizeof(float) * hd);
        }
    }
}

/*
 * a6. Decode attention over an f16 cache [b, n_kv, cap, hd], q [b, n_kv, gqa, hd] f32
 *     with any scale already folded in. Positions < wstart are masked (-inf) and positions
 *     >= span are absent. crates/tts-nn/src/attn.rs:90-126 (scores), candle
 *     softmax_last_dim (max-subtract, exp, divide by the sum; attn.rs:61), attn.rs:203-238
 *     (weighted sum). Per-lane span/wstart generalise the reference's batch-wide values.
 */
void orc_decode_attention(const float* q, const uint16_t* kc, const uint16_t* vc,
                          const int* span, const int* wstart, int b, int n_kv, int gqa,
                          int hd, int cap, float* out) {
#pragma omp parallel
    {
        float* sc = (float*)malloc(sizeof(float) * (size_t)cap);
        float* kt = (float*)malloc(sizeof(float) * (size_t)hd * 8);  /* 8 positions, d-major */
        float* vr = (float*)malloc(sizeof(float) * (size_t)hd);
#pragma omp for schedule(dynamic) collapse(2)
        for (int l = 0; l < b; l++)
            for (int h = 0; h < n_kv; h++) {
                int sp = span[l], ws = wstart[l];
                const uint16_t* kb = kc + ((size_t)l * n_kv + h) * cap * hd;
                const uint16_t* vb = vc + ((size_t)l * n_kv + h) * cap * hd;
                for (int g = 0; g < gqa; g++) {
                    const float* qv = q + (((size_t)l * n_kv + h) * gqa + g) * hd;
                    float mx = -INFINITY;
                    for (int p = 0; p < ws && p < sp; p++) sc[p] = -INFINITY;
                    int p = ws;
                    /* 8 positions at a time: SIMD lane i sums q[d] * k[p + i][d] over d in order,
                       a product then a sum as in the scalar loop, so every score is unchanged */
                    for (; p + 8 <= sp; p += 8) {
                        for (int i = 0; i < 8; i++) {
                            const uint16_t* kr = kb + (size_t)(p + i) * hd;
                            for (int d = 0; d < hd; d++) kt[(size_t)d * 8 + i] = h2f(kr[d]);
                        }
                        __m256 acc = _mm256_setzero_ps();
                        for (int d = 0; d < hd; d++)
                            acc = _mm256_add_ps(acc, _mm256_mul_ps(_mm256_set1_ps(qv[d]),
                                                  _mm256_loadu_ps(kt + (size_t)d * 8)));
                        _mm256_storeu_ps(sc + p, acc);
                    }
                    for (; p < sp; p++) {
                        float acc = 0.f;
                        for (int d = 0; d < hd; d++) acc += qv[d] * h2f(kb[(size_t)p * hd + d]);
                        sc[p] = acc;
                    }
                    for (p = ws; p < sp; p++)
                        if (sc[p] > mx) mx = sc[p];
                    float sum = 0.f;
                    for (p = 0; p < sp; p++) { sc[p] = expf(sc[p] - mx); sum += sc[p]; }
                    for (p = 0; p < sp; p++) sc[p] /= sum;
                    float* o = out + (((size_t)l * n_kv + h) * gqa + g) * hd;
                    for (int d = 0; d < hd; d++) o[d] = 0.f;
                    for (p = 0; p < sp; p++) {
                        const float wgt = sc[p];
                        const uint16_t* vp = vb + (size_t)p * hd;
                        int d = 0;
                        if (hd % 8 == 0) {
                            const __m256 wv = _mm256_set1_ps(wgt);
                            for (; d < hd; d += 8) {
                                const __m256 v8 = _mm256_cvtph_ps(
                                    _mm_loadu_si128((const __m128i*)(vp + d)));
                                _mm256_storeu_ps(o + d, _mm256_add_ps(_mm256_loadu_ps(o + d),
                                                                      _mm256_mul_ps(wv, v8)));
                            }
                        }
                        for (; d < hd; d++) o[d] += wgt * h2f(vp[d]);
                    }
                }
            }
        free(sc);
        free(kt);
        free(vr);
    }
}

/* a7. silu(g) * u, crates/tts-nn/src/fused.rs:311-318 (x / (1 + exp(-x)) * u). */
void orc_swiglu(const float* g, const float* u, float* y, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        float x = g[i];
        y[i] = (x / (1.0f + expf(-x))) * u[i];
    }
}

/*
 * a12. SnakeBeta, channels-last: y = x + brecip[c] * sin(alpha[c] * x)^2.
 *      crates/tts-nn/src/fused.rs:564-600 (alpha and brecip already folded at load,
 *      crates/qwen3tts/src/codec.rs:61-68). Snake (x + sin^2(ax)/a) is brecip = 1/alpha.
 */
void orc_snake_beta(const float* x, const float* alpha, const float* brecip, float* y,
                    int64_t rows, int chan) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++)
        for (int c = 0; c < chan; c++) {
            float v = x[r * chan + c];
            float s = sinf(alpha[c] * v);
            y[r * chan + c] = v + brecip[c] * (s * s);
        }
}

/*
 * a13/a14. Channels-last conv1d with the tap gather in the loop:
 *   y[b,l,co] = bias[co] + sum_t sum_ci xs[b, l + t*dil - pad_left, ci] * w[t, ci, co] (+ res[b,l,co])
 * where xs = snake(x) when alpha is given (the fused snake-on-load of
 * crates/tts-nn/src/nlc.rs:40-68) and rows outside [0, len) are zero.
 * crates/tts-nn/src/nlcconv.rs:33-73 is the causal case pad_left = (k-1)*dil; the centred
 * case follows crates/tts-nn/src/lib.rs:736-767. w_tap is [k, cin, cout] (nlc.rs:30-33).
 * Any of bias, alpha/brecip, res may be NULL.
 */
void orc_conv1d_nlc(const float* x, const float* w, const float* bias, const float* alpha,
                    const float* brecip, const float* res, float* y, int b, int len, int cin,
                    int cout, int k, int dil, int pad_left) {
#pragma omp parallel
    {
        float* xs = (float*)malloc(sizeof(float) * (size_t)cin);
#pragma omp for schedule(static) collapse(2)
        for (int bb = 0; bb < b; bb++)
            for (int l = 0; l < len; l++) {
                float* row = y + ((size_t)bb * len + l) * cout;
                for (int co = 0; co < cout; co++) row[co] = bias ? bias[co] : 0.f;
                for (int t = 0; t < k; t++) {
                    int s = l + t * dil - pad_left;
                    if (s < 0 || s >= len) continue;
                    const float* xr = x + ((size_t)bb * len + s) * cin;
                    for (int ci = 0; ci < cin; ci++) {
                        float v = xr[ci];
                        if (alpha) { float q = sinf(alpha[ci] * v); v = v + brecip[ci] * (q * q); }
                        xs[ci] = v;
                    }
                    for (int ci = 0; ci < cin; ci++) {
                        float xv = xs[ci];
                        const float* wr = w + ((size_t)t * cin + ci) * cout;
                        for (int co = 0; co < cout; co++) row[co] += xv * wr[co];
                    }
                }
                if (res) {
                    const float* rr = res + ((size_t)bb * len + l) * cout;
                    for (int co = 0; co < cout; co++) row[co] += rr[co];
                }
            }
        free(xs);
    }
}

/*
 * a18. Greedy pick per row: argmax over logits with banned ids at -inf.
 *      crates/qwen3tts/src/talker.rs:154-189. Rust's Iterator::max_by returns the LAST of
 *      equal maxima, so ties go to the highest index. banned may be NULL.
 */
void orc_argmax(const float* logits, const uint8_t* banned, uint32_t* out, int rows, int n) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        const float* lr = logits + (size_t)r * n;
        float best = 0.f; int bi = -1;
        for (int i = 0; i < n; i++) {
            float v = (banned && banned[i]) ? -INFINITY : lr[i];
            if (bi < 0 || v >= best) { best = v; bi = i; }
        }
        out[r] = (uint32_t)(bi < 0 ? 0 : bi);
    }
}
