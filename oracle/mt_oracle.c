/*
 * TEST INFRASTRUCTURE — CPU restatement of the region arithmetic.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this library, as the checker and as the timed CPU baseline; the product
 * (libmt.so) never calls it.
 *
 * The reference (shivamg05/metal-autotune) has no arithmetic of its own for
 * these regions: it dispatches to MLX 0.32.2 (uv.lock:575) and mlx-lm
 * 0.31.3 (uv.lock:611), neither of which is present here. Each function
 * restates the algorithm as the reference itself writes it down in its
 * naive lowering (autotuner/scaffold/lower.py) or, where the reference has
 * no restatement, from the published definition named in the comment.
 * Floating-point parity with MLX is therefore UNPINNED: no golden vector of
 * these ops exists in the reference (its parity tests compare against MLX at
 * run time). Compiled with -ffp-contract=off so every product and sum rounds
 * as written.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>


enum { DT_BF16 = 0, DT_F16 = 1, DT_F32 = 2 };

/* fp32 -> bf16 -> fp32, round to nearest even (NaN stays NaN). */
static float round_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) {
    u |= 0x00400000u;
    u &= 0xFFFF0000u;
  } else {
    u += 0x7FFFu + ((u >> 16) & 1u);
    u &= 0xFFFF0000u;
  }
  memcpy(&f, &u, 4);
  return f;
}

/* fp32 -> fp16 -> fp32, round to nearest even, with subnormals and overflow to inf. */
static float round_f16(float f) {
  if (f != f) return f;
  const float a = fabsf(f);
  if (a >= 65520.0f) return f < 0 ? -INFINITY : INFINITY;
  if (a < 6.103515625e-05f) {           /* subnormal range: quantum 2^-24 */
    const float q = 5.9604644775390625e-08f;
    return nearbyintf(f / q) * q;       /* exact scaling by a power of two */
  }
  int e;
  frexpf(a, &e);                        /* a = m * 2^e, m in [0.5, 1) */
  const float quantum = ldexpf(1.0f, e - 11);
  return nearbyintf(f / quantum) * quantum;
}

static float round_dt(float v, int dt) {
  return dt == DT_BF16 ? round_bf16(v) : dt == DT_F16 ? round_f16(v) : v;
}

float orc_round(float v, int dt) { return round_dt(v, dt); }

/* MLX affine dequantisation in the element type: round(round(s*q) + b)
 * (quantized.h `dequantize`, restated in the LFM2 kernel header `mlx_deq8`,
 * examples/lfm2_5_1_2b_prefill/lfm2_5_1_2b_prefill_artifact/kernels/
 * r1f9367e50750eb01_unroll_hoist.launch.json). */
static float dequant(uint32_t q, float s, float b, int dt) {
  return round_dt(round_dt(s * (float)q, dt) + b, dt);
}

static uint32_t unpack(const uint32_t* row, int64_t k, int bits) {
  const int per = 32 / bits;
  return (row[k / per] >> ((k % per) * bits)) & ((1u << bits) - 1u);
}

/* qmm_t (prefill): y = round(sum_k x[m,k] * w~[n,k]) with the dequantised
 * weights rounded to the element type, fp32 accumulation in k order
 * (autotuner/scaffold/lower.py:1109-1142 matmul over the library's
 * dequantised tile; layout lower.py:468-514). */
void orc_qmm_t(const float* x, const uint32_t* w, const float* s, const float* b, float* y, int64_t M,
               int64_t N, int64_t K, int group, int bits, int dt) {
  const int64_t words = K * bits / 32, G = K / group;
#pragma omp parallel
  {
    float* wrow = (float*)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
      const uint32_t* wr = w + n * words;
      for (int64_t k = 0; k < K; ++k)
        wrow[k] = dequant(unpack(wr, k, bits), s[n * G + k / group], b[n * G + k / group], dt);
      for (int64_t m = 0; m < M; ++m) {
        float acc = 0.0f;
        const float* xr = x + m * K;
        for (int64_t k = 0; k < K; ++k) acc += xr[k] * wrow[k];
        y[m * N + n] = round_dt(acc, dt);
      }
    }
    free(wrow);
  }
}

/* qmv (decode): per group acc += scale*sum(x*q) + bias*sum(x), fp32, k in
 * order (autotuner/scaffold/lower.py:1179-1234). */
void orc_qmv(const float* x, const uint32_t* w, const float* s, const float* b, float* y, int64_t M, int64_t N,
             int64_t K, int group, int bits, int dt) {
  const int64_t words = K * bits / 32, G = K / group;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    const uint32_t* wr = w + n * words;
    for (int64_t m = 0; m < M; ++m) {
      float acc = 0.0f;
      for (int64_t g = 0; g < G; ++g) {
        float dq = 0.0f, dx = 0.0f;
        for (int64_t k = g * group; k < (g + 1) * group; ++k) {
          const float xv = x[m * K + k];
          dq += xv * (float)unpack(wr, k, bits);
          dx += xv;
        }
        acc += s[n * G + g] * dq + b[n * G + g] * dx;
      }
      y[m * N + n] = round_dt(acc, dt);
    }
  }
}

/* mx.fast.rms_norm: y = round(x * rsqrt(mean(x^2)+eps) * w)
 * (autotuner/scaffold/lower.py:1318-1355). */
void orc_rms_norm(const float* x, const float* w, float eps, float* y, int64_t rows, int64_t D, int dt) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    float ss = 0.0f;
    for (int64_t j = 0; j < D; ++j) ss += x[r * D + j] * x[r * D + j];
    const float scale = 1.0f / sqrtf(ss / (float)D + eps);
    for (int64_t j = 0; j < D; ++j) y[r * D + j] = round_dt(x[r * D + j] * scale * w[j], dt);
  }
}

/* mx.fast.layer_norm: two-pass mean / centred variance, then the optional
 * affine (autotuner/scaffold/lower.py:1357-1410). */
void orc_layer_norm(const float* x, const float* w, const float* b, float eps, float* y, int64_t rows,
                    int64_t D, int dt) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    float sx = 0.0f;
    for (int64_t j = 0; j < D; ++j) sx += x[r * D + j];
    const float mean = sx / (float)D;
    float sv = 0.0f;
    for (int64_t j = 0; j < D; ++j) {
      const float c = x[r * D + j] - mean;
      sv += c * c;
    }
    const float scale = 1.0f / sqrtf(sv / (float)D + eps);
    for (int64_t j = 0; j < D; ++j) {
      float v = (x[r * D + j] - mean) * scale;
      if (w) v = v * w[j];
      if (b) v = v + b[j];
      y[r * D + j] = round_dt(v, dt);
    }
  }
}

/* inverse frequencies base^(-2j/dims), computed in double then rounded to fp32 */
static void rope_freqs(float* f, int dims, double base) {
  for (int j = 0; j < dims / 2; ++j) f[j] = (float)pow(base, -2.0 * j / dims);
}

/* mx.fast.rope over rows of [R, L, D]: position (l + offset) * scale,
 * theta_j = position * base^(-2j/dims); non-traditional rotates (j, j+dims/2),
 * traditional (2j, 2j+1); the tail past dims is copied
 * (autotuner/scaffold/lower.py:1236-1294). */
void orc_rope(const float* x, float* y, int64_t R, int64_t L, int64_t D, int dims, int traditional, float base,
              float scale, int64_t offset, int dt) {
  float f[256];
  rope_freqs(f, dims, base);
  const int half = dims / 2;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < R * L; ++r) {
    const int64_t l = r % L;
    const float* xr = x + r * D;
    float* yr = y + r * D;
    const float pos = (float)(l + offset) * scale;
    for (int j = 0; j < half; ++j) {
      const float th = pos * f[j];
      const float c = cosf(th), s = sinf(th);
      const int d0 = traditional ? 2 * j : j, d1 = traditional ? 2 * j + 1 : j + half;
      const float a = xr[d0], bb = xr[d1];
      yr[d0] = round_dt(a * c - bb * s, dt);
      yr[d1] = round_dt(a * s + bb * c, dt);
    }
    for (int64_t d = dims; d < D; ++d) yr[d] = xr[d];
  }
}

/* Qwen3 attention prologue (mlx-lm qwen3 Attention: q_norm/k_norm RMSNorm
 * over head_dim, rope at cache.offset, cache.update_and_fetch): q [T, Hq*D],
 * k/v [T, Hkv*D] -> q_out [Hq, T, D], caches [Hkv, cap, D] at offset. */
void orc_qk_norm_rope_cache(const float* q, const float* k, const float* v, const float* qw, const float* kw,
                            float eps, float* q_out, float* k_cache, float* v_cache, int64_t T, int64_t Hq,
                            int64_t Hkv, int64_t D, int64_t cap, int64_t offset, float base, int dt) {
  float f[256];
  rope_freqs(f, (int)D, base);
  const int64_t half = D / 2;
  for (int64_t t = 0; t < T; ++t) {
    for (int64_t hh = 0; hh < Hq + Hkv; ++hh) {
      const int is_q = hh < Hq;
      const int64_t h = is_q ? hh : hh - Hq;
      const float* src = is_q ? q + t * Hq * D + h * D : k + t * Hkv * D + h * D;
      const float* nw = is_q ? qw : kw;
      float n[256];
      float ss = 0.0f;
      for (int64_t d = 0; d < D; ++d) ss += src[d] * src[d];
      const float scale = 1.0f / sqrtf(ss / (float)D + eps);
      for (int64_t d = 0; d < D; ++d) n[d] = round_dt(src[d] * scale * nw[d], dt);
      const float pos = (float)(t + offset);
      float* dst = is_q ? q_out + (h * T + t) * D : k_cache + (h * cap + offset + t) * D;
      for (int64_t j = 0; j < half; ++j) {
        const float th = pos * f[j];
        const float c = cosf(th), s = sinf(th);
        dst[j] = round_dt(n[j] * c - n[j + half] * s, dt);
        dst[j + half] = round_dt(n[j] * s + n[j + half] * c, dt);
      }
      if (!is_q)
        for (int64_t d = 0; d < D; ++d) v_cache[(h * cap + offset + t) * D + d] = v[t * Hkv * D + h * D + d];
    }
  }
}

/* mlx_lm swiglu = silu(gate) * up, silu(x) = x * sigmoid(x), sigmoid =
 * 1/(1+exp(-x)) (autotuner/scaffold/lower.py:80); each op rounded. */
void orc_swiglu(const float* g, const float* u, float* y, int64_t n, int dt) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float sg = round_dt(1.0f / (1.0f + expf(-g[i])), dt);
    const float a = round_dt(g[i] * sg, dt);
    y[i] = round_dt(a * u[i], dt);
  }
}

/* Scaled dot-product attention from its definition, softmax(q k^T * scale +
 * mask) v, GQA head map h -> h / (Hq/Hkv); causal: key j visible to query i
 * iff j <= q_offset + i. Dense layouts q [B,Hq,Lq,D], k/v [B,Hkv,Lk,D],
 * o [B,Hq,Lq,D]; fp32 throughout, output rounded. */
void orc_sdpa(const float* q, const float* k, const float* v, float* o, int64_t B, int64_t Hq, int64_t Hkv,
              int64_t Lq, int64_t Lk, int64_t D, float scale, int causal, int64_t q_offset, int dt) {
  const int64_t rep = Hq / Hkv;
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t b = 0; b < B; ++b)
    for (int64_t h = 0; h < Hq; ++h) {
      const int64_t kh = h / rep;
      float* sc = (float*)malloc(sizeof(float) * (size_t)(Lk > 0 ? Lk : 1));
      for (int64_t i = 0; i < Lq; ++i) {
        const float* qi = q + ((b * Hq + h) * Lq + i) * D;
        float mx = -INFINITY;
        for (int64_t j = 0; j < Lk; ++j) {
          const int ok = !causal || j <= q_offset + i;
          float s = -INFINITY;
          if (ok) {
            const float* kj = k + ((b * Hkv + kh) * Lk + j) * D;
            float d = 0.0f;
            for (int64_t e = 0; e < D; ++e) d += qi[e] * kj[e];
            s = d * scale;
          }
          sc[j] = s;
          if (s > mx) mx = s;
        }
        float sum = 0.0f;
        for (int64_t j = 0; j < Lk; ++j) {
          sc[j] = (sc[j] == -INFINITY) ? 0.0f : expf(sc[j] - mx);
          sum += sc[j];
        }
        float* oi = o + ((b * Hq + h) * Lq + i) * D;
        for (int64_t e = 0; e < D; ++e) {
          float acc = 0.0f;
          for (int64_t j = 0; j < Lk; ++j) acc += sc[j] * v[((b * Hkv + kh) * Lk + j) * D + e];
          oi[e] = round_dt(sum > 0.0f ? acc / sum : 0.0f, dt);
        }
      }
      free(sc);
    }
}

/* mlx.nn.QuantizedEmbedding: out[t] = dequantize(w[tok]) with MLX rounding. */
void orc_quantized_embedding(const int32_t* tok, const uint32_t* w, const float* s, const float* b, float* out,
                             int64_t T, int64_t vocab, int64_t D, int group, int bits, int dt) {
  const int64_t words = D * bits / 32, G = D / group;
  for (int64_t t = 0; t < T; ++t) {
    const int64_t id = tok[t];
    for (int64_t d = 0; d < D; ++d) {
      if (id < 0 || id >= vocab) {
        out[t * D + d] = 0.0f;
        continue;
      }
      out[t * D + d] = dequant(unpack(w + id * words, d, bits), s[id * G + d / group], b[id * G + d / group], dt);
    }
  }
}

/* generate_step's greedy pick (autotuner_runtime/inference.py:140-147):
 * lse = log(sum exp(x - max)) + max in fp32; logprobs = round(x - round(lse));
 * token = first argmax of logprobs. */
void orc_logits_pick(const float* x, int64_t n, int dt, int32_t* token, float* logprob, float* lse_out) {
  float mx = -INFINITY;
  for (int64_t i = 0; i < n; ++i)
    if (x[i] > mx) mx = x[i];
  double sum = 0.0;
  for (int64_t i = 0; i < n; ++i) sum += (double)expf(x[i] - mx);
  const float lse = logf((float)sum) + mx;
  const float lr = round_dt(lse, dt);
  float best = -INFINITY;
  int64_t bi = -1;
  for (int64_t i = 0; i < n; ++i) {
    const float lp = round_dt(x[i] - lr, dt);
    if (bi < 0 || lp > best) {
      best = lp;
      bi = i;
    }
  }
  *token = (int32_t)bi;
  *logprob = best;
  *lse_out = lse;
}

/* mlx.nn.gelu (exact form): x * (1 + erf(x / sqrt(2))) / 2, each operation
 * rounded to fp32 as written, erf from the C library (glibc erff). This is
 * the oracle's own erf: the CUDA kernels call the device library's erff, so
 * the two sides are independent implementations and agree only within their
 * error bounds (glibc erff <= 1 ulp; CUDA erff <= 2 ulp). MLX's own CPU erf
 * is not available here, so bit-exactness against MLX cannot be checked. */
static float gelu_f32(float x) {
  const float u = 1.0f + erff(x / 1.41421356237309505f);
  return x * u / 2.0f;
}

/* Dense linear + bias (+ GELU) with a sequential-k fused multiply-add
 * accumulation (the reference's matmul restatement,
 * autotuner/scaffold/lower.py:1109-1142), bias added once, then GELU. */
void orc_linear(const float* x, const float* w, const float* bias, float* y, int64_t M, int64_t N, int64_t K,
                int act) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      float acc = 0.0f;
      for (int64_t k = 0; k < K; ++k) acc = fmaf(x[m * K + k], w[n * K + k], acc);
      if (bias) acc = acc + bias[n];
      if (act == 1) acc = gelu_f32(acc);
      y[m * N + n] = acc;
    }
}

float orc_erf(float x) { return erff(x); }
float orc_gelu(float x) { return gelu_f32(x); }

static float softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

/* Mamba-1 selective scan (Gu & Dao 2023, mlx-lm 0.31.3 mamba ssm_step):
 * dt = softplus(dt_raw + dt_bias); h = exp(dt*A) h + (dt*B) x;
 * y = sum_s C h + D x; y *= silu(z). fp32 state, t in order. */
void orc_mamba_scan(const float* x, const float* dtr, const float* dt_bias, const float* A, const float* Bm,
                    const float* Cm, const float* Dv, const float* z, float* y, float* h_state, int64_t L,
                    int64_t d_inner, int64_t d_state, int dt) {
#pragma omp parallel for schedule(static)
  for (int64_t c = 0; c < d_inner; ++c) {
    float h[64];
    for (int64_t s = 0; s < d_state; ++s) h[s] = h_state ? h_state[c * d_state + s] : 0.0f;
    for (int64_t t = 0; t < L; ++t) {
      const float xv = x[t * d_inner + c];
      const float d = softplus(dtr[t * d_inner + c] + (dt_bias ? dt_bias[c] : 0.0f));
      float acc = 0.0f;
      for (int64_t s = 0; s < d_state; ++s) {
        const float dA = expf(d * A[c * d_state + s]);
        h[s] = dA * h[s] + (d * Bm[t * d_state + s]) * xv;
        acc += Cm[t * d_state + s] * h[s];
      }
      const float yv = acc + (Dv ? Dv[c] : 0.0f) * xv;
      const float zv = z[t * d_inner + c];
      const float sg = 1.0f / (1.0f + expf(-zv));
      y[t * d_inner + c] = round_dt(yv * (zv * sg), dt);
    }
    if (h_state)
      for (int64_t s = 0; s < d_state; ++s) h_state[c * d_state + s] = h[s];
  }
}

/* Depthwise causal conv1d over [L, C] (kernel [C, W], left context from
 * `state` [C, W-1] or zeros), bias, then SiLU with each op rounded. */
void orc_causal_conv1d(const float* x, const float* wt, const float* bias, const float* state, float* y, int64_t L,
                       int64_t C, int W, int silu, int dt) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t l = 0; l < L; ++l)
    for (int64_t c = 0; c < C; ++c) {
      float acc = 0.0f;
      for (int j = 0; j < W; ++j) {
        const int64_t src = l - (W - 1) + j;
        const float xv = src >= 0 ? x[src * C + c] : (state ? state[c * (W - 1) + (W - 1 + src)] : 0.0f);
        acc = fmaf(wt[c * W + j], xv, acc);
      }
      if (bias) acc = acc + bias[c];
      float v = round_dt(acc, dt);
      if (silu) {
        const float sg = round_dt(1.0f / (1.0f + expf(-v)), dt);
        v = v * sg;
      }
      y[l * C + c] = round_dt(v, dt);
    }
}

/* mx.conv1d over channels-last x [N, L, Cin] with w [Cout, K, Cin]
 * (stride, zero padding `pad` on both sides), as mlx.nn.Conv1d with its bias
 * and the encoder's GELU after it (mlx-whisper conv1/conv2): the conv sum in
 * fp32 over (tap, channel) in order, each of conv / +bias / gelu rounded to
 * the element type as the separate MLX ops materialise them. act: 0 none,
 * 1 GELU (erf form, evaluated in fp32 on the rounded input). */
void orc_conv1d(const float* x, const float* w, const float* bias, float* y, int64_t N, int64_t L, int64_t Cin,
                int64_t Cout, int K, int stride, int pad, int act, int dt) {
  const int64_t Lout = (L + 2 * pad - K) / stride + 1;
#pragma omp parallel for collapse(3) schedule(static)
  for (int64_t n = 0; n < N; ++n)
    for (int64_t t = 0; t < Lout; ++t)
      for (int64_t co = 0; co < Cout; ++co) {
        float acc = 0.0f;
        for (int k = 0; k < K; ++k) {
          const int64_t src = t * stride + k - pad;
          if (src < 0 || src >= L) continue;
          const float* xr = x + (n * L + src) * Cin;
          const float* wr = w + (co * K + k) * Cin;
          for (int64_t ci = 0; ci < Cin; ++ci) acc = fmaf(xr[ci], wr[ci], acc);
        }
        float v = round_dt(acc, dt);
        if (bias) v = round_dt(v + bias[co], dt);
        if (act == 1) v = round_dt(gelu_f32(v), dt);
        y[(n * Lout + t) * Cout + co] = v;
      }
}

/* nn.Linear in a 16-bit dtype (mx.addmm(bias, x, w.T) then nn.gelu):
 * y = round(sum_k x w + bias), GELU in fp32 on that rounded value, rounded. */
void orc_linear_lp(const float* x, const float* w, const float* bias, float* y, int64_t M, int64_t N, int64_t K,
                   int act, int dt) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      float acc = 0.0f;
      for (int64_t k = 0; k < K; ++k) acc = fmaf(x[m * K + k], w[n * K + k], acc);
      float v = round_dt(bias ? acc + bias[n] : acc, dt);
      if (act == 1) v = round_dt(gelu_f32(v), dt);
      y[m * N + n] = v;
    }
}
