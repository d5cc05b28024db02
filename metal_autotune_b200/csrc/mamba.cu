// Mamba-1 selective scan and depthwise causal conv1d.
//
// Scan: lanes (channel, state) — d_state lanes per channel, 32/d_state
// channels per warp — hold h in fp32 registers and walk the L steps in
// order; y_t = sum_s C[t,s] h[s] is a shuffle reduction inside the channel's
// lane group. The recurrence is sequential in t, so one channel's latency
// is L dependent steps; channels are independent (2048 per Mamba-370m
// layer) and fill the GPU. Steps run in chunks of 8: the chunk's inputs load
// while the previous chunk computes; inside a chunk the step-independent
// arithmetic (softplus and gate once per channel, spread over the group's
// lanes; exp(dt A), dt B x) runs for all 8 steps side by side, then the
// recurrence in h, then 8 interleaved reductions over the states.
#include "mt_common.cuh"

namespace mt {

__device__ __forceinline__ float softplus_f32(float x) { return x > 20.f ? x : log1pf(expf(x)); }

template <int DT, int NS>
__global__ void __launch_bounds__(256) mamba_scan_kernel(const void* __restrict__ xp, const void* __restrict__ dtp,
                                                         const float* __restrict__ dt_bias, const float* __restrict__ A,
                                                         const void* __restrict__ Bp, const void* __restrict__ Cp,
                                                         const float* __restrict__ Dv, const void* __restrict__ zp,
                                                         void* __restrict__ yp, float* __restrict__ hstate, int L,
                                                         int d_inner) {
  using T = typename Elem<DT>::T;
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  constexpr int CPW = 32 / NS;  // channels per warp
  const int lane = threadIdx.x & 31;
  const int s = lane % NS;
  const int c = (blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5)) * CPW + lane / NS;
  const bool active = c < d_inner;
  const int cc = active ? c : 0;
  const T* x = static_cast<const T*>(xp);
  const T* dtr = static_cast<const T*>(dtp);
  const T* Bm = static_cast<const T*>(Bp);
  const T* Cm = static_cast<const T*>(Cp);
  const T* z = static_cast<const T*>(zp);
  T* y = static_cast<T*>(yp);
  const float a = A[static_cast<int64_t>(cc) * NS + s];
  const float bias = dt_bias ? dt_bias[cc] : 0.f;
  const float dd = Dv ? Dv[cc] : 0.f;
  float h = (hstate && active) ? hstate[static_cast<int64_t>(cc) * NS + s] : 0.f;
  // the inputs of the next kCh steps load while the current kCh steps run
  // (one step's arithmetic is far shorter than a memory round trip)
  constexpr int kCh = 8;
  float cx[kCh], cdt[kCh], cz[kCh], cb[kCh], ccv[kCh];
  auto fetch = [&](int t0, float (&fx)[kCh], float (&fdt)[kCh], float (&fz)[kCh], float (&fb)[kCh],
                   float (&fc)[kCh]) {
#pragma unroll
    for (int j = 0; j < kCh; ++j) {
      const int64_t r = t0 + j;
      if (r < L) {
        fx[j] = Elem<DT>::to_f(x[r * d_inner + cc]);
        fdt[j] = Elem<DT>::to_f(dtr[r * d_inner + cc]);
        fz[j] = Elem<DT>::to_f(z[r * d_inner + cc]);
        fb[j] = Elem<DT>::to_f(Bm[r * NS + s]);
        fc[j] = Elem<DT>::to_f(Cm[r * NS + s]);
      } else {
        fx[j] = fdt[j] = fz[j] = fb[j] = fc[j] = 0.f;
      }
    }
  };
  fetch(0, cx, cdt, cz, cb, ccv);
  for (int t0 = 0; t0 < L; t0 += kCh) {
    float px[kCh], pdt[kCh], pz[kCh], pb[kCh], pc[kCh];
    fetch(t0 + kCh, px, pdt, pz, pb, pc);
    // the step-independent arithmetic of the chunk first (kCh steps side by
    // side), then the short recurrence in h, then kCh interleaved reductions
    // over the states; each step's operations and roundings are the same as
    // in one step at a time
    // lane s of a channel's group evaluates the per-channel softplus (and
    // below the output gate) of step s mod kCh only; the group shares them
    // by shuffles
    const int jm = s % kCh;
    const int gbase = lane - s;  // first lane of the channel's group
    float dtm = cdt[0], xm = cx[0], zm = cz[0];
#pragma unroll
    for (int j = 1; j < kCh; ++j)
      if (j == jm) {
        dtm = cdt[j];
        xm = cx[j];
        zm = cz[j];
      }
    dtm = softplus_f32(__fadd_rn(dtm, bias));
    float dA[kCh], u[kCh], part[kCh];
#pragma unroll
    for (int j = 0; j < kCh; ++j) {
      const float dt = __shfl_sync(0xffffffffu, dtm, gbase + j);
      dA[j] = expf(__fmul_rn(dt, a));
      u[j] = __fmul_rn(__fmul_rn(dt, cb[j]), cx[j]);
    }
#pragma unroll
    for (int j = 0; j < kCh; ++j) {
      if (t0 + j < L) h = __fadd_rn(__fmul_rn(dA[j], h), u[j]);
      part[j] = __fmul_rn(ccv[j], h);
    }
#pragma unroll
    for (int o = NS / 2; o > 0; o >>= 1)
#pragma unroll
      for (int j = 0; j < kCh; ++j) part[j] += __shfl_xor_sync(0xffffffffu, part[j], o);
    // lane s < kCh of the group finishes and stores step s of the chunk
    float pm = part[0];
#pragma unroll
    for (int j = 1; j < kCh; ++j)
      if (j == jm) pm = part[j];
    const int t = t0 + jm;
    if (s < kCh && active && t < L) {
      const float yv = __fadd_rn(pm, __fmul_rn(dd, xm));
      const float sg = 1.0f / (1.0f + expf(-zm));
      y[static_cast<int64_t>(t) * d_inner + c] = Elem<DT>::from_f(__fmul_rn(yv, __fmul_rn(zm, sg)));
    }
#pragma unroll
    for (int j = 0; j < kCh; ++j) {
      cx[j] = px[j];
      cdt[j] = pdt[j];
      cz[j] = pz[j];
      cb[j] = pb[j];
      ccv[j] = pc[j];
    }
  }
  if (hstate && active) hstate[static_cast<int64_t>(c) * NS + s] = h;
}

// Chunked scan for long prompts. The sequential kernel above runs one lane
// per (channel, state): 32768 lanes for a Mamba-370m layer, about 7 warps per
// SM, so every step waits on its predecessor's latency. Here the L steps
// are cut into KC chunks and warp k of a CTA runs chunk k of the CTA's
// channels, KC times the parallelism:
//   pass 1  each chunk's recurrence from h = 0: its end state e_k and the
//           product P_k of its decays exp(dt A) (the same a_t and u_t as pass 3);
//   fold    chunk k's carry-in h_k = P_{k-1} h_{k-1} + e_{k-1} (h_0 the state
//           carried into the call), from shared memory;
//   pass 3  the recurrence again from h_k, emitting y_t = (C_t h_t + D x_t) z_t sigma(z_t).
// Every step's a_t, u_t and h update are the sequential kernel's operations
// (no contraction); only the chunk carry-ins are reassociated. Steps run in
// blocks of NS: lane s of a channel's group computes the softplus of step s
// of the block and loads its x and z, shared by shuffles; the NS per-step
// state reductions of a block are interleaved, and lane s finishes step s.
template <int DT, int NS, int KC>
__global__ void __launch_bounds__(KC * 32) mamba_scan_chunked_kernel(
    const void* __restrict__ xp, const void* __restrict__ dtp, const float* __restrict__ dt_bias,
    const float* __restrict__ A, const void* __restrict__ Bp, const void* __restrict__ Cp,
    const float* __restrict__ Dv, const void* __restrict__ zp, void* __restrict__ yp, float* __restrict__ hstate,
    int L, int d_inner, int CL) {
  using T = typename Elem<DT>::T;
  constexpr int CPW = 32 / NS;  // channels per warp (and per CTA)
  __shared__ float s_end[KC][CPW][NS];
  __shared__ float s_prod[KC][CPW][NS];
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  const int lane = threadIdx.x & 31;
  const int k = threadIdx.x >> 5;  // chunk
  const int s = lane % NS;
  const int g = lane / NS;         // channel within the CTA
  const int gbase = lane - s;
  const int c = blockIdx.x * CPW + g;
  const bool active = c < d_inner;
  const int cc = active ? c : 0;
  const T* x = static_cast<const T*>(xp);
  const T* dtr = static_cast<const T*>(dtp);
  const T* Bm = static_cast<const T*>(Bp);
  const T* Cm = static_cast<const T*>(Cp);
  const T* z = static_cast<const T*>(zp);
  T* y = static_cast<T*>(yp);
  const float a = A[static_cast<int64_t>(cc) * NS + s];
  const float bias = dt_bias ? dt_bias[cc] : 0.f;
  const float dd = Dv ? Dv[cc] : 0.f;
  const int t_lo = k * CL;
  const int t_hi = min(L, t_lo + CL);

  // one block of NS steps from t0: this lane's step t0 + s supplies dt, x (and z)
  auto step_inputs = [&](int t0, float& dtm, float& xm, float& zm, bool want_z) {
    const int t = t0 + s;
    dtm = xm = zm = 0.f;
    if (t < t_hi) {
      dtm = softplus_f32(__fadd_rn(Elem<DT>::to_f(dtr[static_cast<int64_t>(t) * d_inner + cc]), bias));
      xm = Elem<DT>::to_f(x[static_cast<int64_t>(t) * d_inner + cc]);
      if (want_z) zm = Elem<DT>::to_f(z[static_cast<int64_t>(t) * d_inner + cc]);
    }
  };

  // ---- pass 1: the chunk from h = 0
  float h = 0.f, prod = 1.f;
  for (int t0 = t_lo; t0 < t_hi; t0 += NS) {
    float dtm, xm, zm;
    step_inputs(t0, dtm, xm, zm, false);
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      const float dt = __shfl_sync(0xffffffffu, dtm, gbase + j);
      const float xv = __shfl_sync(0xffffffffu, xm, gbase + j);
      if (t0 + j < t_hi) {
        const float bv = Elem<DT>::to_f(Bm[static_cast<int64_t>(t0 + j) * NS + s]);
        const float dA = expf(__fmul_rn(dt, a));
        const float u = __fmul_rn(__fmul_rn(dt, bv), xv);
        h = __fadd_rn(__fmul_rn(dA, h), u);
        prod = __fmul_rn(prod, dA);
      }
    }
  }
  s_end[k][g][s] = h;
  s_prod[k][g][s] = prod;
  // the carried-in state is read before the barrier: after it the last chunk may overwrite it
  h = (hstate && active) ? hstate[static_cast<int64_t>(cc) * NS + s] : 0.f;
  __syncthreads();

  // ---- carry-in of chunk k
  for (int j = 0; j < k; ++j) h = __fadd_rn(__fmul_rn(s_prod[j][g][s], h), s_end[j][g][s]);

  // ---- pass 3: the chunk from its carry-in, emitting y
  for (int t0 = t_lo; t0 < t_hi; t0 += NS) {
    float dtm, xm, zm;
    step_inputs(t0, dtm, xm, zm, true);
    float part[NS];
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      const float dt = __shfl_sync(0xffffffffu, dtm, gbase + j);
      const float xv = __shfl_sync(0xffffffffu, xm, gbase + j);
      part[j] = 0.f;
      if (t0 + j < t_hi) {
        const float bv = Elem<DT>::to_f(Bm[static_cast<int64_t>(t0 + j) * NS + s]);
        const float cv = Elem<DT>::to_f(Cm[static_cast<int64_t>(t0 + j) * NS + s]);
        const float dA = expf(__fmul_rn(dt, a));
        const float u = __fmul_rn(__fmul_rn(dt, bv), xv);
        h = __fadd_rn(__fmul_rn(dA, h), u);
        part[j] = __fmul_rn(cv, h);
      }
    }
#pragma unroll
    for (int o = NS / 2; o > 0; o >>= 1)
#pragma unroll
      for (int j = 0; j < NS; ++j) part[j] += __shfl_xor_sync(0xffffffffu, part[j], o);
    float pm = part[0];
#pragma unroll
    for (int j = 1; j < NS; ++j)
      if (j == s) pm = part[j];
    const int t = t0 + s;
    if (active && t < t_hi) {
      const float yv = __fadd_rn(pm, __fmul_rn(dd, xm));
      const float sg = 1.0f / (1.0f + expf(-zm));
      y[static_cast<int64_t>(t) * d_inner + c] = Elem<DT>::from_f(__fmul_rn(yv, __fmul_rn(zm, sg)));
    }
  }
  // the state after the last step: the last chunk's final h (chunks past L end where they start)
  if (hstate && active && t_lo < L && t_hi == L) hstate[static_cast<int64_t>(c) * NS + s] = h;
}

// prompts of at least this many steps take the chunked scan, in kScanChunks chunks
constexpr int kScanChunkedMinL = 128;
constexpr int kScanChunks = 8;

template <int DT>
__global__ void __launch_bounds__(256) causal_conv1d_kernel(const void* __restrict__ xp, const void* __restrict__ wp,
                                                            const void* __restrict__ bp, const void* __restrict__ sp,
                                                            void* __restrict__ yp, int L, int C, int W, int silu) {
  using T = typename Elem<DT>::T;
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(L) * C) return;
  const int l = static_cast<int>(i / C), c = static_cast<int>(i % C);
  const T* x = static_cast<const T*>(xp);
  const T* w = static_cast<const T*>(wp) + static_cast<int64_t>(c) * W;
  const T* st = sp ? static_cast<const T*>(sp) + static_cast<int64_t>(c) * (W - 1) : nullptr;
  float acc = 0.f;
  for (int j = 0; j < W; ++j) {
    const int src = l - (W - 1) + j;
    float xv;
    if (src >= 0) xv = Elem<DT>::to_f(x[static_cast<int64_t>(src) * C + c]);
    else xv = st ? Elem<DT>::to_f(st[W - 1 + src]) : 0.f;
    acc = fmaf(Elem<DT>::to_f(w[j]), xv, acc);
  }
  if (bp) acc = __fadd_rn(acc, Elem<DT>::to_f(static_cast<const T*>(bp)[c]));
  float v = round_to<DT>(acc);
  if (silu) {
    const float sg = round_to<DT>(1.0f / (1.0f + expf(-v)));
    v = __fmul_rn(v, sg);
  }
  static_cast<T*>(yp)[i] = Elem<DT>::from_f(v);
}

// New state = the last W-1 entries of [old state, x]; one thread per channel
// shifts its own row in registers, so reading and rewriting the same buffer
// cannot race.
template <int DT>
__global__ void conv_state_kernel(const void* __restrict__ xp, void* sp, int L, int C, int W) {
  using T = typename Elem<DT>::T;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  T* st = static_cast<T*>(sp) + static_cast<int64_t>(c) * (W - 1);
  T old[15];
  for (int j = 0; j < W - 1; ++j) old[j] = st[j];
  for (int j = 0; j < W - 1; ++j) {
    const int src = L - (W - 1) + j;  // index into x; negative reaches back into the old state
    st[j] = src >= 0 ? static_cast<const T*>(xp)[static_cast<int64_t>(src) * C + c] : old[W - 1 + src];
  }
}

}  // namespace mt

using namespace mt;

extern "C" {

int mt_mamba_scan(const void* x, const void* dt_raw, const float* dt_bias, const float* A, const void* Bm,
                  const void* Cm, const float* Dv, const void* z, void* y, float* h_state, int64_t L,
                  int64_t d_inner, int64_t d_state, int dtype, mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(x && dt_raw && A && Bm && Cm && z && y, "mt_mamba_scan: null pointer");
  MT_CHECK_ARG(d_state == 16 || d_state == 8 || d_state == 32, "mt_mamba_scan: d_state %lld (8, 16 or 32)",
               (long long)d_state);
  MT_CHECK_ARG(L >= 0 && d_inner > 0 && L < (1 << 30) && d_inner < (1 << 24), "mt_mamba_scan: bad shape");
  MT_CHECK_ARG(dtype == MT_BF16 || dtype == MT_F16 || dtype == MT_F32, "mt_mamba_scan: bad dtype");
  if (L == 0) return MT_OK;
  const int cpw = 32 / static_cast<int>(d_state);
  cudaStream_t s = (cudaStream_t)stream;
  if (L >= kScanChunkedMinL) {
    // chunked in time: kScanChunks warps per CTA (one per chunk), the CTA's cpw channels
    constexpr int KC = kScanChunks;
    const int CL = static_cast<int>((((L + KC - 1) / KC) + d_state - 1) / d_state * d_state);
    const dim3 cgrid(static_cast<unsigned>((d_inner + cpw - 1) / cpw));
#define MT_CSCAN(DTV, NSV)                                                                                        \
  return launch(mamba_scan_chunked_kernel<DTV, NSV, KC>, cgrid, dim3(KC * 32), 0, s, x, dt_raw, dt_bias, A, Bm, \
                Cm, Dv, z, y, h_state, (int)L, (int)d_inner, CL)
#define MT_CSCAN_NS(DTV)                  \
  if (d_state == 8) MT_CSCAN(DTV, 8);    \
  if (d_state == 16) MT_CSCAN(DTV, 16);  \
  MT_CSCAN(DTV, 32)
    if (dtype == MT_BF16) { MT_CSCAN_NS(MT_BF16); }
    if (dtype == MT_F16) { MT_CSCAN_NS(MT_F16); }
    MT_CSCAN_NS(MT_F32);
#undef MT_CSCAN_NS
#undef MT_CSCAN
  }
  const int64_t warps = (d_inner + cpw - 1) / cpw;
  const dim3 grid(static_cast<unsigned>((warps + 7) / 8));
#define MT_SCAN(DTV, NSV)                                                                                   \
  return launch(mamba_scan_kernel<DTV, NSV>, grid, dim3(256), 0, s, x, dt_raw, dt_bias, A, Bm, Cm, Dv, z, y, \
                h_state, (int)L, (int)d_inner)
#define MT_SCAN_NS(DTV)        \
  if (d_state == 8) MT_SCAN(DTV, 8); \
  if (d_state == 16) MT_SCAN(DTV, 16); \
  MT_SCAN(DTV, 32)
  if (dtype == MT_BF16) { MT_SCAN_NS(MT_BF16); }
  if (dtype == MT_F16) { MT_SCAN_NS(MT_F16); }
  MT_SCAN_NS(MT_F32);
#undef MT_SCAN_NS
#undef MT_SCAN
}

int mt_causal_conv1d(const void* x, const void* weight, const void* bias, void* conv_state, void* y, int64_t L,
                     int64_t C, int width, int silu, int dtype, mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(x && weight && y, "mt_causal_conv1d: null pointer");
  MT_CHECK_ARG(width >= 1 && width <= 16 && L >= 0 && C > 0 && L * C < (int64_t(1) << 40),
               "mt_causal_conv1d: bad shape");
  MT_CHECK_ARG(x != y, "mt_causal_conv1d: y must not alias x");
  if (L == 0) return MT_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const dim3 grid(static_cast<unsigned>((L * C + 255) / 256));
  int rc;
  switch (dtype) {
    case MT_BF16:
      rc = launch(causal_conv1d_kernel<MT_BF16>, grid, dim3(256), 0, s, x, weight, bias, conv_state, y, (int)L,
                  (int)C, width, silu);
      break;
    case MT_F16:
      rc = launch(causal_conv1d_kernel<MT_F16>, grid, dim3(256), 0, s, x, weight, bias, conv_state, y, (int)L,
                  (int)C, width, silu);
      break;
    case MT_F32:
      rc = launch(causal_conv1d_kernel<MT_F32>, grid, dim3(256), 0, s, x, weight, bias, conv_state, y, (int)L,
                  (int)C, width, silu);
      break;
    default: set_error("mt_causal_conv1d: bad dtype"); return MT_ERR_UNSUPPORTED;
  }
  if (rc != MT_OK || !conv_state || width == 1) return rc;
  // Stream order puts the state update after every read of the old state.
  const dim3 g2(static_cast<unsigned>((C + 255) / 256));
  switch (dtype) {
    case MT_BF16: conv_state_kernel<MT_BF16><<<g2, 256, 0, s>>>(x, conv_state, (int)L, (int)C, width); break;
    case MT_F16: conv_state_kernel<MT_F16><<<g2, 256, 0, s>>>(x, conv_state, (int)L, (int)C, width); break;
    default: conv_state_kernel<MT_F32><<<g2, 256, 0, s>>>(x, conv_state, (int)L, (int)C, width); break;
  }
  MT_CUDA(cudaGetLastError());
  count_launch();
  return MT_OK;
}

}  // extern "C"
