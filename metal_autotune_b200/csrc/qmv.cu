// Affine-quantized matrix-vector product for decode (M <= 8 rows of x).
//
// HBM-bound: every packed weight byte is read once. One half-warp owns one
// output row; lane j streams the row's 16-byte chunks j, j+16, ... (32 4-bit
// or 16 8-bit values each, always inside one quantisation group), keeping up
// to four 16-byte loads in flight. x is staged once per CTA in shared memory
// as fp32, XOR-swizzled per chunk so that the 16 lanes of a half-warp, which
// read 16 different chunks, hit different banks.
//
// Arithmetic per group (autotuner/scaffold/lower.py:1179-1234, the MLX qmv
// form): acc += scale * sum(x*q) + bias * sum(x), fp32. For 4-bit the
// nibbles are widened through the bf16 bit pattern 0x4300|q = 128 + q, so a
// pair of nibbles costs one byte-permute and one logic op; the chunk sum
// sum(x*(128+q)) is corrected by 128 * sum(x) (chunk sums precomputed once).
#include "mt_common.cuh"
#include "qmm_common.cuh"

namespace mt {

template <int BITS> struct QmvChunk {
  static constexpr int kValues = BITS == 4 ? 32 : 16;  // values per 16-byte chunk
};

struct QmvSet {
  const uint32_t* w;
  const void* s;
  const void* b;
  void* y;
  int N;
};

struct QmvParams {
  const void* x;
  const void* residual;
  QmvSet set[3];
  int row_start[4];  // prefix sums of N over the sets (multi mode)
  int M, K, group;
  int ldx, ldy;      // row strides of x and of y / residual, elements
};

// swizzled float4 slot of (chunk c, slot f) for 4-bit (8 float4 per chunk)
// or 8-bit (4 float4 per chunk)
template <int BITS>
__device__ __forceinline__ int xs_index(int c, int f) {
  constexpr int F = QmvChunk<BITS>::kValues / 4;
  return c * F + (f ^ (c & (F - 1)));
}

template <int DT, int BITS, int MR>
__device__ __forceinline__ void qmv_row(const uint32_t* __restrict__ wrow,
                                        const typename Elem<DT>::T* __restrict__ srow,
                                        const typename Elem<DT>::T* __restrict__ brow, int nchunk,
                                        int group, const float4* __restrict__ xs,
                                        const float* __restrict__ xsum, int K, int j,
                                        float (&acc)[MR]) {
  constexpr int V = QmvChunk<BITS>::kValues;
  const int xs_stride = K / 4;  // float4 per x row
#pragma unroll
  for (int m = 0; m < MR; ++m) acc[m] = 0.f;
  for (int c0 = j; c0 < nchunk; c0 += 64) {
    uint4 wv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c = c0 + 16 * u;
      if (c < nchunk) wv[u] = ld_stream_v4(wrow + c * 4);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c = c0 + 16 * u;
      if (c >= nchunk) break;
      const int g = (c * V) / group;
      const float s = Elem<DT>::to_f(srow[g]);
      const float b = Elem<DT>::to_f(brow[g]);
      const uint32_t words[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        const float4* xr = xs + m * xs_stride;
        float a = 0.f;
        if constexpr (BITS == 4) {
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const uint32_t lo = words[wi], hi = words[wi] >> 4;
            const float4 xa = xr[xs_index<BITS>(c, 2 * wi)];
            const float4 xb = xr[xs_index<BITS>(c, 2 * wi + 1)];
            const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              const uint32_t v = nibble_pair_bf16(lo, hi, p);  // bf16x2 (128+q[2p], 128+q[2p+1])
              a = fmaf(xv[2 * p], __uint_as_float(v << 16), a);
              a = fmaf(xv[2 * p + 1], __uint_as_float(v & 0xFFFF0000u), a);
            }
          }
          const float xsm = xsum[m * nchunk + c];
          acc[m] += s * a + (b - 128.f * s) * xsm;
        } else {
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const float4 xa = xr[xs_index<BITS>(c, wi)];
            const float xv[4] = {xa.x, xa.y, xa.z, xa.w};
#pragma unroll
            for (int p = 0; p < 4; ++p)
              a = fmaf(xv[p], static_cast<float>((words[wi] >> (8 * p)) & 0xFFu), a);
          }
          acc[m] += s * a + b * xsum[m * nchunk + c];
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    float v = acc[m];
    v += __shfl_xor_sync(0xffffffffu, v, 8);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    acc[m] = v;
  }
}

// MODE: 0 plain (up to 3 sets, concatenated rows), 1 residual (set 0),
// 2 SwiGLU (set 0 gate, set 1 up).
template <int DT, int BITS, int MR, int MODE>
__global__ void __launch_bounds__(256) qmv_kernel(const QmvParams p) {
  using T = typename Elem<DT>::T;
  extern __shared__ float4 smem4[];
  constexpr int V = QmvChunk<BITS>::kValues;
  const int K = p.K;
  const int nchunk = K / V;
  float4* xs = smem4;                                  // [MR][K/4]
  float* xsum = reinterpret_cast<float*>(xs + MR * (K / 4));  // [MR][nchunk]

  griddep_wait();

  griddep_launch();  // dependents may launch now; their own wait covers this grid
  const T* x = static_cast<const T*>(p.x);
  for (int i = threadIdx.x; i < MR * (K / 4); i += blockDim.x) {
    const int m = i / (K / 4), q = i % (K / 4);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (m < p.M) {
      const T* src = x + static_cast<int64_t>(m) * p.ldx + 4 * q;
      v = make_float4(Elem<DT>::to_f(src[0]), Elem<DT>::to_f(src[1]), Elem<DT>::to_f(src[2]),
                      Elem<DT>::to_f(src[3]));
    }
    const int c = (4 * q) / V, f = ((4 * q) % V) / 4;
    xs[m * (K / 4) + xs_index<BITS>(c, f)] = v;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < MR * nchunk; i += blockDim.x) {
    const int m = i / nchunk, c = i % nchunk;
    float s = 0.f;
    for (int f = 0; f < V / 4; ++f) {
      const float4 v = xs[m * (K / 4) + xs_index<BITS>(c, f)];
      s += v.x + v.y + v.z + v.w;
    }
    xsum[i] = s;
  }
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const int j = lane & 15;
  const int row = blockIdx.x * 16 + (threadIdx.x >> 4);
  const int G = K / p.group;
  const int words_per_row = K * BITS / 32;

  if constexpr (MODE == 2) {
    if (row >= p.set[0].N) return;
    float ag[MR], au[MR];
    qmv_row<DT, BITS, MR>(p.set[0].w + static_cast<int64_t>(row) * words_per_row,
                          static_cast<const T*>(p.set[0].s) + static_cast<int64_t>(row) * G,
                          static_cast<const T*>(p.set[0].b) + static_cast<int64_t>(row) * G, nchunk,
                          p.group, xs, xsum, K, j, ag);
    qmv_row<DT, BITS, MR>(p.set[1].w + static_cast<int64_t>(row) * words_per_row,
                          static_cast<const T*>(p.set[1].s) + static_cast<int64_t>(row) * G,
                          static_cast<const T*>(p.set[1].b) + static_cast<int64_t>(row) * G, nchunk,
                          p.group, xs, xsum, K, j, au);
    if (j == 0) {
      T* y = static_cast<T*>(p.set[0].y);
#pragma unroll
      for (int m = 0; m < MR; ++m)
        if (m < p.M)
          y[static_cast<int64_t>(m) * p.ldy + row] =
              Elem<DT>::from_f(swiglu_rounded<DT>(round_to<DT>(ag[m]), round_to<DT>(au[m])));
    }
  } else {
    if (row >= p.row_start[3]) return;
    int si = 0;
    if (row >= p.row_start[1]) si = 1;
    if (row >= p.row_start[2]) si = 2;
    const QmvSet& st = p.set[si];
    const int r = row - p.row_start[si];
    float acc[MR];
    qmv_row<DT, BITS, MR>(st.w + static_cast<int64_t>(r) * words_per_row,
                          static_cast<const T*>(st.s) + static_cast<int64_t>(r) * G,
                          static_cast<const T*>(st.b) + static_cast<int64_t>(r) * G, nchunk,
                          p.group, xs, xsum, K, j, acc);
    if (j == 0) {
      T* y = static_cast<T*>(st.y);
      const int ldy = (MODE == 0) ? st.N : p.ldy;
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        if (m >= p.M) break;
        float v = round_to<DT>(acc[m]);
        if constexpr (MODE == 1)
          v = v + Elem<DT>::to_f(static_cast<const T*>(p.residual)[static_cast<int64_t>(m) * ldy + r]);
        y[static_cast<int64_t>(m) * ldy + r] = Elem<DT>::from_f(v);
      }
    }
  }
}

template <int DT, int BITS, int MODE>
static int qmv_dispatch_mr(QmvParams& p, int total_rows, cudaStream_t stream) {
  const int K = p.K;
  constexpr int V = QmvChunk<BITS>::kValues;
  auto smem_for = [&](int mr) { return static_cast<size_t>(mr) * (K * 4 + (K / V) * 4); };
  const dim3 grid((total_rows + 15) / 16);
  int mr = p.M <= 1 ? 1 : p.M <= 2 ? 2 : p.M <= 4 ? 4 : 8;
  while (mr > 1 && smem_for(mr) > 200 * 1024) mr >>= 1;
  if (smem_for(mr) > 200 * 1024) {
    set_error("qmv: K=%d too large for one staged row of x", K);
    return MT_ERR_UNSUPPORTED;
  }
  // Rows of x beyond the staged MR are handled by further launches.
  const int M = p.M;
  const void* x0 = p.x;
  const void* r0 = p.residual;
  void* y0[3] = {p.set[0].y, p.set[1].y, p.set[2].y};
  for (int m0 = 0; m0 < M; m0 += mr) {
    using T = typename Elem<DT>::T;
    p.M = (M - m0 < mr) ? (M - m0) : mr;
    p.x = static_cast<const T*>(x0) + static_cast<int64_t>(m0) * p.ldx;
    if (r0) p.residual = static_cast<const T*>(r0) + static_cast<int64_t>(m0) * p.ldy;
    for (int s = 0; s < 3; ++s)
      if (y0[s]) {
        const int ld = (MODE == 0) ? p.set[s].N : p.ldy;
        p.set[s].y = static_cast<T*>(y0[s]) + static_cast<int64_t>(m0) * ld;
      }
    int rc;
    const size_t smem = smem_for(mr);
    switch (mr) {
      case 1: {
        auto k = qmv_kernel<DT, BITS, 1, MODE>;
        if (int e = ensure_smem(k, smem)) return e;
        rc = launch(k, grid, dim3(256), smem, stream, p);
        break;
      }
      case 2: {
        auto k = qmv_kernel<DT, BITS, 2, MODE>;
        if (int e = ensure_smem(k, smem)) return e;
        rc = launch(k, grid, dim3(256), smem, stream, p);
        break;
      }
      case 4: {
        auto k = qmv_kernel<DT, BITS, 4, MODE>;
        if (int e = ensure_smem(k, smem)) return e;
        rc = launch(k, grid, dim3(256), smem, stream, p);
        break;
      }
      default: {
        auto k = qmv_kernel<DT, BITS, 8, MODE>;
        if (int e = ensure_smem(k, smem)) return e;
        rc = launch(k, grid, dim3(256), smem, stream, p);
        break;
      }
    }
    if (rc != MT_OK) return rc;
  }
  return MT_OK;
}

template <int MODE>
static int qmv_dispatch(QmvParams& p, int bits, int dtype, int total_rows, cudaStream_t stream) {
  if (dtype == MT_BF16)
    return bits == 4 ? qmv_dispatch_mr<MT_BF16, 4, MODE>(p, total_rows, stream)
                     : qmv_dispatch_mr<MT_BF16, 8, MODE>(p, total_rows, stream);
  return bits == 4 ? qmv_dispatch_mr<MT_F16, 4, MODE>(p, total_rows, stream)
                   : qmv_dispatch_mr<MT_F16, 8, MODE>(p, total_rows, stream);
}

int qmv_run(const QmmRequest& r, cudaStream_t stream) {
  // 4-bit decode shapes whose rows fit the streamed kernel's shared memory
  if (qmv_stream_eligible(r)) return qmv_stream_run(r, stream);
  QmvParams p = {};
  p.x = r.x;
  p.residual = r.residual;
  p.M = static_cast<int>(r.M);
  p.K = static_cast<int>(r.K);
  p.group = r.group;
  p.ldx = static_cast<int>(r.K);
  int total = 0;
  p.row_start[0] = 0;
  for (int s = 0; s < 3; ++s) {
    p.set[s] = {r.set[s].w, r.set[s].s, r.set[s].b, r.set[s].y, static_cast<int>(r.set[s].N)};
    if (r.kind != QMM_SWIGLU) total += static_cast<int>(r.set[s].N);
    p.row_start[s + 1] = total;
  }
  p.ldy = static_cast<int>(r.set[0].N);
  if (r.kind == QMM_SWIGLU) return qmv_dispatch<2>(p, r.bits, r.dtype, (int)r.set[0].N, stream);
  if (r.kind == QMM_RESIDUAL) return qmv_dispatch<1>(p, r.bits, r.dtype, total, stream);
  return qmv_dispatch<0>(p, r.bits, r.dtype, total, stream);
}

}  // namespace mt
