// Elementwise and gather regions: SwiGLU, the residual / positional add, the
// dense and the quantized embedding gathers and the greedy pick from the
// last row of logits.
#include <cooperative_groups.h>

#include "mt_common.cuh"
#include "qmm_common.cuh"

namespace mt {

template <int DT>
__global__ void __launch_bounds__(256) swiglu_kernel(const void* __restrict__ gp, const void* __restrict__ up,
                                                     void* __restrict__ yp, int64_t n) {
  using T = typename Elem<DT>::T;
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  const T* g = static_cast<const T*>(gp);
  const T* u = static_cast<const T*>(up);
  T* y = static_cast<T*>(yp);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte vector
  if (((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(u) | reinterpret_cast<uintptr_t>(y)) & 15) == 0) {
    // 16-byte vectors, the same per-element arithmetic; the tail past the
    // last whole vector element by element
    const int64_t nv = n / V;
    for (int64_t v = tid; v < nv; v += stride) {
      const uint4 gv = *reinterpret_cast<const uint4*>(g + v * V);
      const uint4 uv = *reinterpret_cast<const uint4*>(u + v * V);
      uint4 yv;
      const T* ge = reinterpret_cast<const T*>(&gv);
      const T* ue = reinterpret_cast<const T*>(&uv);
      T* ye = reinterpret_cast<T*>(&yv);
#pragma unroll
      for (int e = 0; e < V; ++e) ye[e] = Elem<DT>::from_f(swiglu_rounded<DT>(Elem<DT>::to_f(ge[e]), Elem<DT>::to_f(ue[e])));
      *reinterpret_cast<uint4*>(y + v * V) = yv;
    }
    for (int64_t i = nv * V + tid; i < n; i += stride)
      y[i] = Elem<DT>::from_f(swiglu_rounded<DT>(Elem<DT>::to_f(g[i]), Elem<DT>::to_f(u[i])));
    return;
  }
  for (int64_t i = tid; i < n; i += stride)
    y[i] = Elem<DT>::from_f(swiglu_rounded<DT>(Elem<DT>::to_f(g[i]), Elem<DT>::to_f(u[i])));
}

// y[i] = round(x[i] + r[i mod period]): a residual or positional add with the
// second operand repeated every `period` elements (period = n: plain add).
template <int DT>
__global__ void __launch_bounds__(256) add_kernel(const void* __restrict__ xp, const void* __restrict__ rp,
                                                  void* __restrict__ yp, int64_t n, int64_t period) {
  using T = typename Elem<DT>::T;
  griddep_wait();
  griddep_launch();
  const T* x = static_cast<const T*>(xp);
  const T* r = static_cast<const T*>(rp);
  T* y = static_cast<T*>(yp);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  constexpr int V = 16 / sizeof(T);
  const bool vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(r) | reinterpret_cast<uintptr_t>(y)) &
                    15) == 0 && period % V == 0;
  if (vec) {
    const int64_t nv = n / V;
    for (int64_t v = tid; v < nv; v += stride) {
      const uint4 xv = *reinterpret_cast<const uint4*>(x + v * V);
      const uint4 rv = *reinterpret_cast<const uint4*>(r + (v * V) % period);
      uint4 yv;
      const T* xe = reinterpret_cast<const T*>(&xv);
      const T* re = reinterpret_cast<const T*>(&rv);
      T* ye = reinterpret_cast<T*>(&yv);
#pragma unroll
      for (int e = 0; e < V; ++e) ye[e] = Elem<DT>::from_f(Elem<DT>::to_f(xe[e]) + Elem<DT>::to_f(re[e]));
      *reinterpret_cast<uint4*>(y + v * V) = yv;
    }
    for (int64_t i = nv * V + tid; i < n; i += stride)
      y[i] = Elem<DT>::from_f(Elem<DT>::to_f(x[i]) + Elem<DT>::to_f(r[i % period]));
    return;
  }
  for (int64_t i = tid; i < n; i += stride)
    y[i] = Elem<DT>::from_f(Elem<DT>::to_f(x[i]) + Elem<DT>::to_f(r[i % period]));
}

// out[t, :] = table[tok[t], :] (a dense embedding gather, 16-byte copies);
// an id outside [0, vocab) writes zeros and records the device status.
__global__ void __launch_bounds__(128) embed_kernel(const int32_t* __restrict__ tokens, const uint8_t* __restrict__ table,
                                                    uint8_t* __restrict__ out, int64_t vocab, int64_t row_bytes) {
  griddep_wait();
  griddep_launch();
  const int t = blockIdx.x;
  const int tok = tokens[t];
  uint8_t* dst = out + static_cast<int64_t>(t) * row_bytes;
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) report_status(0x501);
    for (int64_t i = threadIdx.x; i < row_bytes; i += blockDim.x) dst[i] = 0;
    return;
  }
  const uint8_t* src = table + static_cast<int64_t>(tok) * row_bytes;
  if (row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    for (int64_t i = threadIdx.x; i < row_bytes / 16; i += blockDim.x)
      reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  } else {
    for (int64_t i = threadIdx.x; i < row_bytes; i += blockDim.x) dst[i] = src[i];
  }
}

// out[t, k] = round(round(s*q) + b) for token tok[t]; one CTA per token.
template <int DT>
__global__ void __launch_bounds__(256) qembed_kernel(const int32_t* __restrict__ tokens, const uint32_t* __restrict__ w,
                                                     const void* __restrict__ sp, const void* __restrict__ bp,
                                                     void* __restrict__ outp, int64_t vocab, int D, int group,
                                                     int bits) {
  using T = typename Elem<DT>::T;
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  const int t = blockIdx.x;
  const int tok = tokens[t];
  T* out = static_cast<T*>(outp) + static_cast<int64_t>(t) * D;
  if (tok < 0 || tok >= vocab) {
    for (int k = threadIdx.x; k < D; k += blockDim.x) out[k] = Elem<DT>::from_f(0.f);
    if (threadIdx.x == 0) report_status(0x601);
    return;
  }
  const int per = 32 / bits;
  const int G = D / group;
  const uint32_t* wr = w + static_cast<int64_t>(tok) * (D / per);
  const T* sr = static_cast<const T*>(sp) + static_cast<int64_t>(tok) * G;
  const T* br = static_cast<const T*>(bp) + static_cast<int64_t>(tok) * G;
  const uint32_t mask = (1u << bits) - 1u;
  for (int k = threadIdx.x; k < D; k += blockDim.x) {
    const uint32_t q = (wr[k / per] >> ((k % per) * bits)) & mask;
    const float s = Elem<DT>::to_f(sr[k / group]);
    const float b = Elem<DT>::to_f(br[k / group]);
    const float sq = round_to<DT>(__fmul_rn(s, static_cast<float>(q)));
    out[k] = Elem<DT>::from_f(__fadd_rn(sq, b));
  }
}

// Single CTA of 1024 threads: pass 1 logsumexp (per-thread online max/sum,
// fixed-order tree), pass 2 argmax of round(x - round(lse)) with the lowest
// index on ties, as mlx-lm's `logits - logsumexp(logits)` then argmax.
// Greedy pick over one row of logits (autotuner_runtime/inference.py:140-147,
// mlx-lm generate_step): lse = log(sum exp(x - max)) + max in fp32,
// logprobs = round(x - round(lse)), token = first argmax of the logprobs.
// One cluster of 8 CTAs x 1024 threads, CTA r owning the contiguous chunk
// [r*n/8, (r+1)*n/8): three passes over the chunk (max, sum of exp, argmax of
// the rounded log-probabilities), the CTAs' partial results exchanged through
// distributed shared memory and combined in rank order, so every CTA forms
// the same max and lse and the result does not depend on timing.
constexpr int kLpCtas = 8;
constexpr int kLpThreads = 1024;

template <int DT>
__global__ void __cluster_dims__(kLpCtas, 1, 1) __launch_bounds__(kLpThreads)
    logits_pick_kernel(const void* __restrict__ lp, int64_t n, int32_t* __restrict__ token,
                       float* __restrict__ logprob, float* __restrict__ lse_out) {
  namespace cg = cooperative_groups;
  using T = typename Elem<DT>::T;
  __shared__ float sm_f[32];
  __shared__ int64_t sm_i[32];
  __shared__ float pub_m, pub_s, pub_best;  // this CTA's partials, read by the cluster
  __shared__ int64_t pub_bi;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t lo = n * rank / kLpCtas, hi = n * (rank + 1) / kLpCtas;
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  const T* x = static_cast<const T*>(lp);

  // pass 1: max
  float m = -INFINITY;
  for (int64_t i = lo + tid; i < hi; i += kLpThreads) m = fmaxf(m, Elem<DT>::to_f(x[i]));
  m = warp_max(m);
  if (lane == 0) sm_f[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = warp_max(sm_f[lane]);
    if (lane == 0) pub_m = m;
  }
  cluster.sync();
  float gmax = -INFINITY;
  for (int r = 0; r < kLpCtas; ++r) gmax = fmaxf(gmax, *cluster.map_shared_rank(&pub_m, r));

  // pass 2: sum of exp(x - max)
  float s = 0.f;
  if (gmax != -INFINITY)
    for (int64_t i = lo + tid; i < hi; i += kLpThreads) s += expf(Elem<DT>::to_f(x[i]) - gmax);
  s = warp_sum(s);
  __syncthreads();
  if (lane == 0) sm_f[warp] = s;
  __syncthreads();
  if (warp == 0) {
    s = warp_sum(sm_f[lane]);
    if (lane == 0) pub_s = s;
  }
  cluster.sync();
  float gsum = 0.f;
  for (int r = 0; r < kLpCtas; ++r) gsum += *cluster.map_shared_rank(&pub_s, r);
  const float lse = logf(gsum) + gmax;
  const float lse_r = round_to<DT>(lse);

  // pass 3: first argmax of the rounded log-probabilities
  float best = -INFINITY;
  int64_t bi = -1;
  for (int64_t i = lo + tid; i < hi; i += kLpThreads) {
    const float v = round_to<DT>(__fsub_rn(Elem<DT>::to_f(x[i]), lse_r));
    if (bi < 0 || v > best) {
      best = v;
      bi = i;
    }
  }
  auto better = [](float b2, int64_t i2, float b, int64_t i) {
    return i2 >= 0 && (i < 0 || b2 > b || (b2 == b && i2 < i));
  };
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float b2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(b2, i2, best, bi)) {
      best = b2;
      bi = i2;
    }
  }
  if (lane == 0) {
    sm_f[warp] = best;
    sm_i[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    best = sm_f[lane];
    bi = sm_i[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float b2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(b2, i2, best, bi)) {
        best = b2;
        bi = i2;
      }
    }
    if (lane == 0) {
      pub_best = best;
      pub_bi = bi;
    }
  }
  cluster.sync();
  if (rank == 0 && tid == 0) {
    float b = -INFINITY;
    int64_t ib = -1;
    for (int r = 0; r < kLpCtas; ++r) {
      const float b2 = *cluster.map_shared_rank(&pub_best, r);
      const int64_t i2 = *cluster.map_shared_rank(&pub_bi, r);
      if (better(b2, i2, b, ib)) {
        b = b2;
        ib = i2;
      }
    }
    *token = static_cast<int32_t>(ib);
    *logprob = b;
    if (lse_out) *lse_out = lse;
  }
  cluster.sync();  // the other CTAs' shared memory stays alive until rank 0 has read it
}

}  // namespace mt

using namespace mt;

extern "C" {

int mt_swiglu(const void* gate, const void* up, void* y, int64_t n, int dtype, mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(gate && up && y, "mt_swiglu: null pointer");
  MT_CHECK_ARG(n >= 0, "mt_swiglu: negative size");
  if (n == 0) return MT_OK;
  int sms = 148;
  int rc = device_sm_count(&sms);
  if (rc) return rc;
  const int64_t want = (n + 255) / 256;
  const dim3 grid(static_cast<unsigned>(want < sms * 16 ? want : sms * 16));  // grid-stride loops
  switch (dtype) {
    case MT_BF16: return launch(swiglu_kernel<MT_BF16>, grid, dim3(256), 0, (cudaStream_t)stream, gate, up, y, n);
    case MT_F16: return launch(swiglu_kernel<MT_F16>, grid, dim3(256), 0, (cudaStream_t)stream, gate, up, y, n);
    case MT_F32: return launch(swiglu_kernel<MT_F32>, grid, dim3(256), 0, (cudaStream_t)stream, gate, up, y, n);
    default: set_error("mt_swiglu: unsupported dtype %d", dtype); return MT_ERR_UNSUPPORTED;
  }
}

int mt_add(const void* x, const void* r, void* y, int64_t n, int64_t period, int dtype, mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(x && r && y, "mt_add: null pointer");
  MT_CHECK_ARG(n >= 0 && period > 0 && (n == 0 || n % period == 0), "mt_add: n=%lld must be a multiple of period=%lld",
               (long long)n, (long long)period);
  if (n == 0) return MT_OK;
  int sms = 148;
  int rc = device_sm_count(&sms);
  if (rc) return rc;
  const int64_t want = (n + 255) / 256;
  const dim3 grid(static_cast<unsigned>(want < sms * 16 ? want : sms * 16));
  switch (dtype) {
    case MT_BF16: return launch(add_kernel<MT_BF16>, grid, dim3(256), 0, (cudaStream_t)stream, x, r, y, n, period);
    case MT_F16: return launch(add_kernel<MT_F16>, grid, dim3(256), 0, (cudaStream_t)stream, x, r, y, n, period);
    case MT_F32: return launch(add_kernel<MT_F32>, grid, dim3(256), 0, (cudaStream_t)stream, x, r, y, n, period);
    default: set_error("mt_add: unsupported dtype %d", dtype); return MT_ERR_UNSUPPORTED;
  }
}

int mt_embedding(const int32_t* tokens, const void* table, void* out, int64_t T, int64_t vocab, int64_t D, int dtype,
                 mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(tokens && table && out, "mt_embedding: null pointer");
  MT_CHECK_ARG(T >= 0 && T < (1 << 30) && vocab > 0 && D > 0, "mt_embedding: bad shape");
  int esz = 0;
  switch (dtype) {
    case MT_BF16:
    case MT_F16: esz = 2; break;
    case MT_F32: esz = 4; break;
    default: set_error("mt_embedding: unsupported dtype %d", dtype); return MT_ERR_UNSUPPORTED;
  }
  if (T == 0) return MT_OK;
  return launch(embed_kernel, dim3(static_cast<unsigned>(T)), dim3(128), 0, (cudaStream_t)stream, tokens,
                static_cast<const uint8_t*>(table), static_cast<uint8_t*>(out), vocab, D * esz);
}

int mt_quantized_embedding(const int32_t* tokens, const uint32_t* w, const void* scales, const void* biases,
                           void* out, int64_t T, int64_t vocab, int64_t D, int group_size, int bits, int dtype,
                           mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(tokens && w && scales && biases && out, "mt_quantized_embedding: null pointer");
  MT_CHECK_ARG(bits == 4 || bits == 8, "mt_quantized_embedding: bits=%d", bits);
  MT_CHECK_ARG(group_size == 32 || group_size == 64 || group_size == 128, "mt_quantized_embedding: group %d",
               group_size);
  MT_CHECK_ARG(D > 0 && D % group_size == 0 && D < (1 << 24) && vocab > 0 && T >= 0 && T < (1 << 30),
               "mt_quantized_embedding: bad shape");
  if (T == 0) return MT_OK;
  const dim3 grid(static_cast<unsigned>(T));
  if (dtype == MT_BF16)
    return launch(qembed_kernel<MT_BF16>, grid, dim3(256), 0, (cudaStream_t)stream, tokens, w, scales, biases, out,
                  vocab, (int)D, group_size, bits);
  if (dtype == MT_F16)
    return launch(qembed_kernel<MT_F16>, grid, dim3(256), 0, (cudaStream_t)stream, tokens, w, scales, biases, out,
                  vocab, (int)D, group_size, bits);
  set_error("mt_quantized_embedding: dtype must be bf16 or f16");
  return MT_ERR_UNSUPPORTED;
}

int mt_logits_pick(const void* logits, int64_t n, int dtype, int32_t* token, float* logprob, float* lse,
                   mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(logits && token && logprob, "mt_logits_pick: null pointer");
  MT_CHECK_ARG(n > 0, "mt_logits_pick: empty row");
  switch (dtype) {
    case MT_BF16:
      return launch(logits_pick_kernel<MT_BF16>, dim3(kLpCtas), dim3(kLpThreads), 0, (cudaStream_t)stream, logits, n, token,
                    logprob, lse);
    case MT_F16:
      return launch(logits_pick_kernel<MT_F16>, dim3(kLpCtas), dim3(kLpThreads), 0, (cudaStream_t)stream, logits, n, token,
                    logprob, lse);
    case MT_F32:
      return launch(logits_pick_kernel<MT_F32>, dim3(kLpCtas), dim3(kLpThreads), 0, (cudaStream_t)stream, logits, n, token,
                    logprob, lse);
    default: set_error("mt_logits_pick: unsupported dtype %d", dtype); return MT_ERR_UNSUPPORTED;
  }
}

}  // extern "C"
