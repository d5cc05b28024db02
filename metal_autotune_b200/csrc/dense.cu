// fp32 dense linear (+bias, +GELU) for the GELU-MLP region (tiny MLP).
//
// Fixed order: each output accumulates k = 0..K-1 in order with one fused
// multiply-add per term (bit-identical to a sequential CPU restatement), adds
// the bias once, then applies GELU with the device library's erff. The tiny
// MLP is launch-bound (33.5 MFLOP), so this favours exactness over tensor
// cores (TF32 would change every product). linear_f32_burst_kernel serves K
// up to 1152 (a multiple of 4) with its whole K span staged at once;
// linear_f32_kernel, 32 x 32 tiles staged 32 values of K at a time, serves
// the rest. The accumulation order is the same in both.
#include "mt_common.cuh"

namespace mt {

__global__ void __launch_bounds__(256) linear_f32_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                         const float* __restrict__ bias, float* __restrict__ y,
                                                         int M, int N, int K, int act) {
  __shared__ float xs[32][33];
  __shared__ float wsm[32][33];
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  const int m0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; k0 < K; k0 += 32) {
    for (int i = ty; i < 32; i += 8) {
      const int m = m0 + i, n = n0 + i, k = k0 + tx;
      xs[i][tx] = (m < M && k < K) ? x[static_cast<int64_t>(m) * K + k] : 0.f;
      wsm[i][tx] = (n < N && k < K) ? w[static_cast<int64_t>(n) * K + k] : 0.f;
    }
    __syncthreads();
    const int kmax = K - k0 < 32 ? K - k0 : 32;
    for (int kk = 0; kk < kmax; ++kk) {
      const float wv = wsm[tx][kk];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = fmaf(xs[ty + 8 * i][kk], wv, acc[i]);
    }
    __syncthreads();
  }
  const int n = n0 + tx;
  if (n < N) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = m0 + ty + 8 * i;
      if (m >= M) continue;
      float v = acc[i];
      if (bias) v = __fadd_rn(v, bias[n]);
      if (act == 1) v = gelu_erf_f32(v);
      y[static_cast<int64_t>(m) * N + n] = v;
    }
  }
}

// Same outputs, same order of operations, for K up to kLfMaxK (a multiple of
// 4, 16-byte aligned rows): a CTA's 32 x-rows and 16 w-rows, all of K, are
// brought into shared memory in batches of 16 independent 16-byte loads per
// thread (all of a batch in flight at once: a few memory latencies instead
// of one per 32-wide chunk), then each thread runs its two outputs'
// sequential k = 0..K-1 fused multiply-add chains out of shared memory,
// reading 4 values of k per 16-byte load. 32 x 16 tiles give the tiny MLP's
// second linear (N = 256) 16 CTAs instead of 8. Rows are padded to K + 4
// floats: 16-byte aligned, and the 8 w-rows a quarter-warp reads start 4
// banks apart, so its 16-byte reads do not collide.
constexpr int kLfBM = 32, kLfBN = 16, kLfMaxK = 1152, kLfBatch = 16;

__global__ void __launch_bounds__(256) linear_f32_burst_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                               const float* __restrict__ bias, float* __restrict__ y,
                                                               int M, int N, int K, int act) {
  extern __shared__ __align__(16) float lf_smem[];
  const int P = K + 4;
  float* xs = lf_smem;               // [kLfBM][P]
  float* wsm = lf_smem + kLfBM * P;  // [kLfBN][P]
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  const int m0 = blockIdx.y * kLfBM, n0 = blockIdx.x * kLfBN;
  const int v4 = K / 4;  // 16-byte vectors per row
  const int total = (kLfBM + kLfBN) * v4;
  for (int base = threadIdx.x; base < total; base += blockDim.x * kLfBatch) {
    float4 v[kLfBatch];
#pragma unroll
    for (int u = 0; u < kLfBatch; ++u) {
      const int idx = base + u * blockDim.x;
      v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (idx < total) {
        const int row = idx / v4, c = idx - row * v4;
        if (row < kLfBM) {
          const int m = m0 + row;
          if (m < M) v[u] = *reinterpret_cast<const float4*>(x + static_cast<int64_t>(m) * K + 4 * c);
        } else {
          const int n = n0 + row - kLfBM;
          if (n < N) v[u] = *reinterpret_cast<const float4*>(w + static_cast<int64_t>(n) * K + 4 * c);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kLfBatch; ++u) {
      const int idx = base + u * blockDim.x;
      if (idx < total) {
        const int row = idx / v4, c = idx - row * v4;
        float* dst = row < kLfBM ? xs + row * P + 4 * c : wsm + (row - kLfBM) * P + 4 * c;
        *reinterpret_cast<float4*>(dst) = v[u];
      }
    }
  }
  __syncthreads();
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int nl = tx & 15;                        // output column in the tile
  const int ml0 = (tx >> 4) * 16 + ty;           // output rows ml0 and ml0 + 8
  const float4* wr = reinterpret_cast<const float4*>(wsm + nl * P);
  const float4* xr0 = reinterpret_cast<const float4*>(xs + ml0 * P);
  const float4* xr1 = reinterpret_cast<const float4*>(xs + (ml0 + 8) * P);
  float a0 = 0.f, a1 = 0.f;
#pragma unroll 4
  for (int k4 = 0; k4 < v4; ++k4) {
    const float4 wv = wr[k4], p = xr0[k4], q = xr1[k4];
    a0 = fmaf(p.x, wv.x, a0);
    a1 = fmaf(q.x, wv.x, a1);
    a0 = fmaf(p.y, wv.y, a0);
    a1 = fmaf(q.y, wv.y, a1);
    a0 = fmaf(p.z, wv.z, a0);
    a1 = fmaf(q.z, wv.z, a1);
    a0 = fmaf(p.w, wv.w, a0);
    a1 = fmaf(q.w, wv.w, a1);
  }
  const int n = n0 + nl;
  if (n >= N) return;
  const float accs[2] = {a0, a1};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int m = m0 + ml0 + 8 * i;
    if (m >= M) continue;
    float v = accs[i];
    if (bias) v = __fadd_rn(v, bias[n]);
    if (act == 1) v = gelu_erf_f32(v);
    y[static_cast<int64_t>(m) * N + n] = v;
  }
}

}  // namespace mt

using namespace mt;

namespace mt {
int conv1d_run(const void* x, const void* w, const void* bias, void* y, int64_t N, int64_t L, int64_t Cin,
               int64_t Cout, int K, int stride, int padding, int act, int dtype, int bias_fused, cudaStream_t stream);
int gemm_tc_run(const void* x, const void* w, const void* bias, const void* residual, void* y, int64_t B,
                int64_t L, int64_t Cin, int64_t Cout, int taps, int stride, int padding, int act, int dtype,
                int bias_fused, int64_t ldy, cudaStream_t stream);
}

extern "C" int mt_linear(const void* x, const void* w, const void* bias, void* y, int64_t M, int64_t N, int64_t K,
                         int act, int dtype, mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(x && w && y, "mt_linear: null pointer");
  if (dtype == MT_BF16 || dtype == MT_F16) {
    // tensor-core path (the Whisper MLP sizes): x [M, K] @ w[N, K]^T as a
    // one-tap conv over M positions, bias added before the single rounding
    // (mx.addmm), GELU rounded after it
    MT_CHECK_ARG(act == 0 || act == 1, "mt_linear: act must be 0 (identity) or 1 (gelu)");
    MT_CHECK_ARG(M >= 0 && N > 0 && K > 0, "mt_linear: bad shape");
    if (M == 0) return MT_OK;
    return conv1d_run(x, w, bias, y, 1, M, K, N, 1, 1, 0, act, dtype, 1, (cudaStream_t)stream);
  }
  MT_CHECK_ARG(dtype == MT_F32, "mt_linear: dtype %d is not built (fp32, bf16, f16)", dtype);
  MT_CHECK_ARG(act == 0 || act == 1, "mt_linear: act must be 0 (identity) or 1 (gelu)");
  MT_CHECK_ARG(M >= 0 && N > 0 && K > 0 && M < (1 << 30) && N < (1 << 30) && K < (1 << 30),
               "mt_linear: bad shape");
  if (M == 0) return MT_OK;
  if (K % 4 == 0 && K <= kLfMaxK && aligned(x, 16) && aligned(w, 16) && (M + kLfBM - 1) / kLfBM < 65535) {
    const size_t smem = static_cast<size_t>(kLfBM + kLfBN) * (K + 4) * sizeof(float);
    if (int e = ensure_smem(linear_f32_burst_kernel, static_cast<int>(smem))) return e;
    const dim3 grid(static_cast<unsigned>((N + kLfBN - 1) / kLfBN), static_cast<unsigned>((M + kLfBM - 1) / kLfBM));
    return launch(linear_f32_burst_kernel, grid, dim3(256), smem, (cudaStream_t)stream, (const float*)x,
                  (const float*)w, (const float*)bias, (float*)y, (int)M, (int)N, (int)K, act);
  }
  const dim3 grid(static_cast<unsigned>((N + 31) / 32), static_cast<unsigned>((M + 31) / 32));
  return launch(linear_f32_kernel, grid, dim3(256), 0, (cudaStream_t)stream, (const float*)x, (const float*)w,
                (const float*)bias, (float*)y, (int)M, (int)N, (int)K, act);
}

// nn.Linear (+ bias) then + residual, in 16 bits: y = round(round(x w^T + b) + r)
// (mlx's `x + linear(...)` of a residual block), on the tcgen05 GEMM.
extern "C" int mt_linear_residual(const void* x, const void* w, const void* bias, const void* residual, void* y,
                                  int64_t M, int64_t N, int64_t K, int dtype, mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(x && w && y && residual, "mt_linear_residual: null pointer");
  MT_CHECK_ARG(M >= 0 && N > 0 && K > 0 && M < (int64_t(1) << 31) && N < (1 << 24) && K < (1 << 24),
               "mt_linear_residual: bad shape M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  if (dtype != MT_BF16 && dtype != MT_F16) {
    set_error("mt_linear_residual: dtype %d is not built (bf16 or f16)", dtype);
    return MT_ERR_UNSUPPORTED;
  }
  if (M == 0) return MT_OK;
  const int rc = gemm_tc_run(x, w, bias, residual, y, 1, M, K, N, 1, 1, 0, 0, dtype, 1, N, (cudaStream_t)stream);
  if (rc == MT_ERR_UNSUPPORTED)
    set_error("mt_linear_residual: K=%lld must be a multiple of 8 and x, w 16-byte aligned", (long long)K);
  return rc;
}
