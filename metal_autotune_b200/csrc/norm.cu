// Row normalisations and rotary embedding (HBM-bound elementwise/row work).
//
// rms_norm / add_rms_norm / layer_norm: one warp per row, 16-byte vector
// loads when the row allows, fp32 accumulation, the row re-read from L1/L2
// for the second pass. rope: one thread per rotated pair. The Qwen3
// attention prologue (q/k RMSNorm -> RoPE -> head-major q, KV-cache append)
// is one warp per (token, head): 128 values = 4 per lane, the rotation
// partner d+64 sits in lane l+16.
//
// Products that the oracle computes without contraction use __fmul_rn /
// __fadd_rn so the GPU and the CPU restatement round identically.
#include "mt_common.cuh"
#include "rope_common.cuh"

namespace mt {

template <int DT>
__device__ __forceinline__ void load8(const typename Elem<DT>::T* p, float* v) {
  if constexpr (DT == MT_F32) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const typename Elem<DT>::T* e = reinterpret_cast<const typename Elem<DT>::T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = Elem<DT>::to_f(e[i]);
  }
}
template <int DT>
__device__ __forceinline__ void store8(typename Elem<DT>::T* p, const float* v) {
  if constexpr (DT == MT_F32) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint4 u;
    typename Elem<DT>::T* e = reinterpret_cast<typename Elem<DT>::T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = Elem<DT>::from_f(v[i]);
    *reinterpret_cast<uint4*>(p) = u;
  }
}

// y = x * rsqrt(mean(x^2) + eps) * w   (HAS_RES: x = round(x + res) first, written to h)
template <int DT, bool HAS_RES, bool VEC>
__global__ void __launch_bounds__(256) rms_norm_kernel(const void* __restrict__ xp, const void* __restrict__ rp,
                                                       const void* __restrict__ wp, float eps,
                                                       void* __restrict__ hp, void* __restrict__ yp,
                                                       int64_t rows, int dim) {
  using T = typename Elem<DT>::T;
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* x = static_cast<const T*>(xp) + row * dim;
  const T* res = HAS_RES ? static_cast<const T*>(rp) + row * dim : nullptr;
  T* h = HAS_RES ? static_cast<T*>(hp) + row * dim : nullptr;
  const T* w = static_cast<const T*>(wp);
  T* y = static_cast<T*>(yp) + row * dim;
  float ss = 0.f;
  if (VEC) {
    for (int i = lane * 8; i < dim; i += 256) {
      float v[8];
      load8<DT>(x + i, v);
      if (HAS_RES) {
        float r[8];
        load8<DT>(res + i, r);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = round_to<DT>(__fadd_rn(v[e], r[e]));
        store8<DT>(h + i, v);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
    }
  } else {
    for (int i = lane; i < dim; i += 32) {
      float v = Elem<DT>::to_f(x[i]);
      if (HAS_RES) {
        v = round_to<DT>(__fadd_rn(v, Elem<DT>::to_f(res[i])));
        h[i] = Elem<DT>::from_f(v);
      }
      ss = fmaf(v, v, ss);
    }
  }
  ss = warp_sum(ss);
  const float scale = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(dim)), eps));
  if (HAS_RES) __syncwarp();
  const T* src = HAS_RES ? h : x;
  if (VEC) {
    for (int i = lane * 8; i < dim; i += 256) {
      float v[8], g[8];
      load8<DT>(src + i, v);
      load8<DT>(w + i, g);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(__fmul_rn(v[e], scale), g[e]);
      store8<DT>(y + i, v);
    }
  } else {
    for (int i = lane; i < dim; i += 32)
      y[i] = Elem<DT>::from_f(__fmul_rn(__fmul_rn(Elem<DT>::to_f(src[i]), scale), Elem<DT>::to_f(w[i])));
  }
}

// rms_norm with the row held in registers: dim = 256 * NC, lane l owns the
// 8-value chunks l, l+32, ...; all loads of the row (x, residual) are issued
// before the first use, so the row costs one memory round trip. Same
// arithmetic in the same order as rms_norm_kernel (bit-identical results).
template <int DT, bool HAS_RES, int NC>
__global__ void __launch_bounds__(128) rms_norm_reg_kernel(const void* __restrict__ xp, const void* __restrict__ rp,
                                                           const void* __restrict__ wp, float eps,
                                                           void* __restrict__ hp, void* __restrict__ yp,
                                                           int64_t rows) {
  using T = typename Elem<DT>::T;
  constexpr int dim = 256 * NC;
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* x = static_cast<const T*>(xp) + row * dim;
  const T* w = static_cast<const T*>(wp);
  float v[NC][8];
#pragma unroll
  for (int c = 0; c < NC; ++c) load8<DT>(x + lane * 8 + c * 256, v[c]);
  if (HAS_RES) {
    const T* res = static_cast<const T*>(rp) + row * dim;
    T* h = static_cast<T*>(hp) + row * dim;
    float r[NC][8];
#pragma unroll
    for (int c = 0; c < NC; ++c) load8<DT>(res + lane * 8 + c * 256, r[c]);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[c][e] = round_to<DT>(__fadd_rn(v[c][e], r[c][e]));
      store8<DT>(h + lane * 8 + c * 256, v[c]);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(v[c][e], v[c][e], ss);
  ss = warp_sum(ss);
  const float scale = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(dim)), eps));
  T* y = static_cast<T*>(yp) + row * dim;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    float g[8], o[8];
    load8<DT>(w + lane * 8 + c * 256, g);  // the weight row is shared by every row: an L1/L2 hit
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __fmul_rn(__fmul_rn(v[c][e], scale), g[e]);
    store8<DT>(y + lane * 8 + c * 256, o);
  }
}

// Launches rms_norm_reg_kernel when dim is a multiple of 256 with a register
// specialisation; returns 1 when it does not apply.
template <int DT, bool HAS_RES>
static int rms_norm_reg_launch(const void* x, const void* res, const void* w, float eps, void* h, void* y,
                               int64_t rows, int64_t dim, cudaStream_t stream) {
  // up to 1024 rows: a warp per CTA, so the rows spread over more SMs (each
  // row is one memory round trip); more rows: 4 warps per CTA
  const int wpb = rows <= 1024 ? 1 : 4;
  const dim3 grid(static_cast<unsigned>((rows + wpb - 1) / wpb)), block(32 * wpb);
  switch (dim) {
    case 1024: return launch(rms_norm_reg_kernel<DT, HAS_RES, 4>, grid, block, 0, stream, x, res, w, eps, h, y, rows);
    case 2048: return launch(rms_norm_reg_kernel<DT, HAS_RES, 8>, grid, block, 0, stream, x, res, w, eps, h, y, rows);
    case 2560: return launch(rms_norm_reg_kernel<DT, HAS_RES, 10>, grid, block, 0, stream, x, res, w, eps, h, y, rows);
    case 3072: return launch(rms_norm_reg_kernel<DT, HAS_RES, 12>, grid, block, 0, stream, x, res, w, eps, h, y, rows);
    case 4096: return launch(rms_norm_reg_kernel<DT, HAS_RES, 16>, grid, block, 0, stream, x, res, w, eps, h, y, rows);
    default: return 1;
  }
}

// layer norm with the row held in registers (dim = 256 * NC, bf16/f16): lane
// l owns the 8-value chunks l, l+32, ...; one read of the row, then the same
// two passes (mean, centred variance) and affine as layer_norm_kernel, with
// each lane's partial sums taken over its chunks.
template <int DT, int NC>
__global__ void __launch_bounds__(128) layer_norm_reg_kernel(const void* __restrict__ xp, const void* __restrict__ wp,
                                                             const void* __restrict__ bp, float eps,
                                                             void* __restrict__ yp, int64_t rows) {
  using T = typename Elem<DT>::T;
  constexpr int dim = 256 * NC;
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* x = static_cast<const T*>(xp) + row * dim;
  float v[NC][8];
#pragma unroll
  for (int c = 0; c < NC; ++c) load8<DT>(x + lane * 8 + c * 256, v[c]);
  float sx = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int e = 0; e < 8; ++e) sx += v[c][e];
  sx = warp_sum(sx);
  const float mean = __fdiv_rn(sx, static_cast<float>(dim));
  float sv = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float d = __fsub_rn(v[c][e], mean);
      sv = fmaf(d, d, sv);
    }
  sv = warp_sum(sv);
  const float scale = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(sv, static_cast<float>(dim)), eps));
  T* y = static_cast<T*>(yp) + row * dim;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    float g[8], bb[8], o[8];
    if (wp) load8<DT>(static_cast<const T*>(wp) + lane * 8 + c * 256, g);
    if (bp) load8<DT>(static_cast<const T*>(bp) + lane * 8 + c * 256, bb);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float u = __fmul_rn(__fsub_rn(v[c][e], mean), scale);
      if (wp) u = __fmul_rn(u, g[e]);
      if (bp) u = __fadd_rn(u, bb[e]);
      o[e] = u;
    }
    store8<DT>(y + lane * 8 + c * 256, o);
  }
}

// two-pass layer norm: mean, centred variance, optional affine
template <int DT>
__global__ void __launch_bounds__(256) layer_norm_kernel(const void* __restrict__ xp, const void* __restrict__ wp,
                                                         const void* __restrict__ bp, float eps,
                                                         void* __restrict__ yp, int64_t rows, int dim) {
  using T = typename Elem<DT>::T;
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* x = static_cast<const T*>(xp) + row * dim;
  const T* w = static_cast<const T*>(wp);
  const T* b = static_cast<const T*>(bp);
  T* y = static_cast<T*>(yp) + row * dim;
  float sx = 0.f;
  for (int i = lane; i < dim; i += 32) sx += Elem<DT>::to_f(x[i]);
  sx = warp_sum(sx);
  const float mean = __fdiv_rn(sx, static_cast<float>(dim));
  float sv = 0.f;
  for (int i = lane; i < dim; i += 32) {
    const float c = __fsub_rn(Elem<DT>::to_f(x[i]), mean);
    sv = fmaf(c, c, sv);
  }
  sv = warp_sum(sv);
  const float scale = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(sv, static_cast<float>(dim)), eps));
  for (int i = lane; i < dim; i += 32) {
    float v = __fmul_rn(__fsub_rn(Elem<DT>::to_f(x[i]), mean), scale);
    if (w) v = __fmul_rn(v, Elem<DT>::to_f(w[i]));
    if (b) v = __fadd_rn(v, Elem<DT>::to_f(b[i]));
    y[i] = Elem<DT>::from_f(v);
  }
}

// x, y: [B*H, L, D]. One CTA per position l and group of kRopeRows of the
// B*H rows at that position: the CTA computes the angles of its position once
// (dims/2 of them, shared memory), then its threads take (row, pair j) items
// plus the tail copies past `dims`. The angle expression is the per-element
// one, so the result does not depend on the grouping.
constexpr int kRopeRows = 32;
// Element strides of x and y over (batch, head, position); D is contiguous.
struct RopeStrides {
  int64_t H, xb, xh, xl, yb, yh, yl;
};
template <int DT, bool STRIDED>
__global__ void __launch_bounds__(256) rope_kernel(const void* __restrict__ xp, void* __restrict__ yp,
                                                   int64_t BH, int L, int D, int dims, int traditional,
                                                   float scale, int64_t offset, const RopeFreqs f, int vec,
                                                   const RopeStrides st) {
  using T = typename Elem<DT>::T;
  __shared__ float2 cs[128];
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  const int l = blockIdx.x;
  const int half = dims / 2;
  const float pos = __fmul_rn(static_cast<float>(static_cast<int64_t>(l) + offset), scale);
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    float sn, cn;
    sincosf(__fmul_rn(pos, f.inv_freq[j]), &sn, &cn);
    cs[j] = make_float2(sn, cn);
  }
  __syncthreads();
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * kRopeRows;
  const int64_t nr = (BH - r0) < kRopeRows ? (BH - r0) : kRopeRows;
  const int hdiv = static_cast<int>(st.H);  // B*H < 2^21 (grid.y limit), so rows fit 32 bits
  if (vec) {
    // 4 pairs per item (8-byte accesses), then the tail copies
    const int hv = half / 4, per_row = hv + (D - dims);
    for (int64_t i = threadIdx.x; i < nr * per_row; i += blockDim.x) {
      const int q = static_cast<int>(i % per_row);
      const T* x;
      T* y;
      if constexpr (STRIDED) {
        const int bh = static_cast<int>(r0 + i / per_row), bb = bh / hdiv, hh = bh - bb * hdiv;
        x = static_cast<const T*>(xp) + bb * st.xb + hh * st.xh + l * st.xl;
        y = static_cast<T*>(yp) + bb * st.yb + hh * st.yh + l * st.yl;
      } else {
        const int64_t row = (r0 + i / per_row) * L + l;
        x = static_cast<const T*>(xp) + row * D;
        y = static_cast<T*>(yp) + row * D;
      }
      if (q >= hv) {
        const int d = dims + (q - hv);
        y[d] = x[d];
        continue;
      }
      const int j0 = 4 * q;
      T a[4], b[4];
      if (traditional) {  // pairs (2j, 2j+1): 8 consecutive values
        const uint2 lo = *reinterpret_cast<const uint2*>(x + 2 * j0), hi = *reinterpret_cast<const uint2*>(x + 2 * j0 + 4);
        const T* e0 = reinterpret_cast<const T*>(&lo);
        const T* e1 = reinterpret_cast<const T*>(&hi);
        a[0] = e0[0]; b[0] = e0[1]; a[1] = e0[2]; b[1] = e0[3];
        a[2] = e1[0]; b[2] = e1[1]; a[3] = e1[2]; b[3] = e1[3];
      } else {  // pairs (j, j + half)
        const uint2 va = *reinterpret_cast<const uint2*>(x + j0), vb = *reinterpret_cast<const uint2*>(x + j0 + half);
        const T* ea = reinterpret_cast<const T*>(&va);
        const T* eb = reinterpret_cast<const T*>(&vb);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          a[e] = ea[e];
          b[e] = eb[e];
        }
      }
      T oa[4], ob[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float o0, o1;
        rope_pair(Elem<DT>::to_f(a[e]), Elem<DT>::to_f(b[e]), cs[j0 + e].y, cs[j0 + e].x, o0, o1);
        oa[e] = Elem<DT>::from_f(o0);
        ob[e] = Elem<DT>::from_f(o1);
      }
      if (traditional) {
        uint2 lo, hi;
        T* e0 = reinterpret_cast<T*>(&lo);
        T* e1 = reinterpret_cast<T*>(&hi);
        e0[0] = oa[0]; e0[1] = ob[0]; e0[2] = oa[1]; e0[3] = ob[1];
        e1[0] = oa[2]; e1[1] = ob[2]; e1[2] = oa[3]; e1[3] = ob[3];
        *reinterpret_cast<uint2*>(y + 2 * j0) = lo;
        *reinterpret_cast<uint2*>(y + 2 * j0 + 4) = hi;
      } else {
        *reinterpret_cast<uint2*>(y + j0) = *reinterpret_cast<const uint2*>(oa);
        *reinterpret_cast<uint2*>(y + j0 + half) = *reinterpret_cast<const uint2*>(ob);
      }
    }
    return;
  }
  const int per_row = half + (D - dims);
  for (int64_t i = threadIdx.x; i < nr * per_row; i += blockDim.x) {
    const int j = static_cast<int>(i % per_row);
    const T* x;
    T* y;
    if constexpr (STRIDED) {
      const int bh = static_cast<int>(r0 + i / per_row), bb = bh / hdiv, hh = bh - bb * hdiv;
      x = static_cast<const T*>(xp) + bb * st.xb + hh * st.xh + l * st.xl;
      y = static_cast<T*>(yp) + bb * st.yb + hh * st.yh + l * st.yl;
    } else {
      const int64_t row = (r0 + i / per_row) * L + l;
      x = static_cast<const T*>(xp) + row * D;
      y = static_cast<T*>(yp) + row * D;
    }
    if (j >= half) {  // tail beyond `dims` copies through
      const int d = dims + (j - half);
      y[d] = x[d];
      continue;
    }
    const int d0 = traditional ? 2 * j : j;
    const int d1 = traditional ? 2 * j + 1 : j + half;
    float o0, o1;
    rope_pair(Elem<DT>::to_f(x[d0]), Elem<DT>::to_f(x[d1]), cs[j].y, cs[j].x, o0, o1);
    y[d0] = Elem<DT>::from_f(o0);
    y[d1] = Elem<DT>::from_f(o1);
  }
}

// Qwen3 attention prologue, D = 128: warp per (token, head) over Hq + Hkv heads.
template <int DT>
__global__ void __launch_bounds__(256) qk_norm_rope_cache_kernel(
    const void* __restrict__ qp, const void* __restrict__ kp, const void* __restrict__ vp, int64_t q_stride,
    int64_t kv_stride, const void* __restrict__ qwp, const void* __restrict__ kwp, float eps,
    void* __restrict__ qo, void* __restrict__ kc, void* __restrict__ vc, int T_, int Hq, int Hkv,
    int64_t cap, int64_t offset, const __grid_constant__ RopeFreqs f) {
  using T = typename Elem<DT>::T;
  // (sin, cos) of the CTA's token positions: its 8 rows span at most
  // kRopeTok tokens, and each angle is computed once instead of once per head
  constexpr int kRopeTok = 9;
  __shared__ float2 sc_tab[kRopeTok][64];
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  const int heads = Hq + Hkv;
  const int64_t rows = static_cast<int64_t>(T_) * heads;
  const int64_t w0 = static_cast<int64_t>(blockIdx.x) * 8;
  const int t0 = static_cast<int>(w0 / heads);
  const int ntok = static_cast<int>(((w0 + 7 < rows ? w0 + 7 : rows - 1) / heads)) - t0 + 1;
  for (int i = threadIdx.x; i < ntok * 64; i += blockDim.x) {
    float s, c;
    rope_angle(static_cast<int64_t>(t0 + i / 64) + offset, f, i % 64, s, c);
    sc_tab[i / 64][i % 64] = make_float2(s, c);
  }
  __syncthreads();
  const int64_t wid = w0 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (wid >= rows) return;
  const int t = static_cast<int>(wid / heads);
  const int hh = static_cast<int>(wid % heads);
  const bool is_q = hh < Hq;
  const int h = is_q ? hh : hh - Hq;
  const T* src = is_q ? static_cast<const T*>(qp) + t * q_stride + h * 128
                      : static_cast<const T*>(kp) + t * kv_stride + h * 128;
  const T* nw = static_cast<const T*>(is_q ? qwp : kwp);
  // a k head's v row is loaded together with the k row (one memory round trip)
  uint2 vrow = make_uint2(0, 0);
  if (!is_q) vrow = *reinterpret_cast<const uint2*>(static_cast<const T*>(vp) + t * kv_stride + h * 128 + 4 * lane);
  const float2* tab = sc_tab[t - t0];
  const uint2 out = qk_norm_rope_vals<DT>(*reinterpret_cast<const uint2*>(src + 4 * lane),
                                          *reinterpret_cast<const uint2*>(nw + 4 * lane), eps,
                                          [&](int j, float& s, float& c) {
                                            s = tab[j].x;
                                            c = tab[j].y;
                                          },
                                          lane);
  if (is_q) {
    *reinterpret_cast<uint2*>(static_cast<T*>(qo) + (static_cast<int64_t>(h) * T_ + t) * 128 + 4 * lane) = out;
  } else {
    const int64_t crow = static_cast<int64_t>(h) * cap + offset + t;
    *reinterpret_cast<uint2*>(static_cast<T*>(kc) + crow * 128 + 4 * lane) = out;
    *reinterpret_cast<uint2*>(static_cast<T*>(vc) + crow * 128 + 4 * lane) = vrow;
  }
}

}  // namespace mt

using namespace mt;

#define MT_DT_SWITCH(dtype, KERNEL_CALL)                                        \
  switch (dtype) {                                                             \
    case MT_BF16: { constexpr int DT = MT_BF16; KERNEL_CALL; } break;          \
    case MT_F16: { constexpr int DT = MT_F16; KERNEL_CALL; } break;            \
    case MT_F32: { constexpr int DT = MT_F32; KERNEL_CALL; } break;            \
    default: set_error("unsupported dtype %d", dtype); return MT_ERR_UNSUPPORTED; \
  }


extern "C" {

int mt_rms_norm(const void* x, const void* w, float eps, void* y, int64_t rows, int64_t dim, int dtype,
                mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(x && w && y, "mt_rms_norm: null pointer");
  MT_CHECK_ARG(rows >= 0 && dim > 0 && dim <= (1 << 24), "mt_rms_norm: rows=%lld dim=%lld", (long long)rows,
               (long long)dim);
  if (rows == 0) return MT_OK;
  const bool vec = dim % 8 == 0 && aligned(x, 16) && aligned(y, 16) && aligned(w, 16);
  const dim3 grid(static_cast<unsigned>((rows + 7) / 8));
  int rc = MT_OK;
  if (vec && (dtype == MT_BF16 || dtype == MT_F16)) {
    rc = dtype == MT_BF16 ? rms_norm_reg_launch<MT_BF16, false>(x, nullptr, w, eps, nullptr, y, rows, dim,
                                                                   (cudaStream_t)stream)
                          : rms_norm_reg_launch<MT_F16, false>(x, nullptr, w, eps, nullptr, y, rows, dim,
                                                               (cudaStream_t)stream);
    if (rc != 1) return rc;
    rc = MT_OK;
  }
  MT_DT_SWITCH(dtype, rc = vec ? launch(rms_norm_kernel<DT, false, true>, grid, dim3(256), 0, (cudaStream_t)stream, x,
                                        nullptr, w, eps, nullptr, y, rows, (int)dim)
                               : launch(rms_norm_kernel<DT, false, false>, grid, dim3(256), 0,
                                        (cudaStream_t)stream, x, nullptr, w, eps, nullptr, y, rows, (int)dim));
  return rc;
}

int mt_add_rms_norm(const void* x, const void* residual, const void* w, float eps, void* h, void* y, int64_t rows,
                    int64_t dim, int dtype, mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(x && residual && w && h && y, "mt_add_rms_norm: null pointer");
  MT_CHECK_ARG(rows >= 0 && dim > 0 && dim <= (1 << 24), "mt_add_rms_norm: rows=%lld dim=%lld",
               (long long)rows, (long long)dim);
  if (rows == 0) return MT_OK;
  const bool vec = dim % 8 == 0 && aligned(x, 16) && aligned(y, 16) && aligned(w, 16) && aligned(h, 16) &&
                   aligned(residual, 16);
  const dim3 grid(static_cast<unsigned>((rows + 7) / 8));
  int rc = MT_OK;
  if (vec && (dtype == MT_BF16 || dtype == MT_F16)) {
    rc = dtype == MT_BF16 ? rms_norm_reg_launch<MT_BF16, true>(x, residual, w, eps, h, y, rows, dim,
                                                                  (cudaStream_t)stream)
                          : rms_norm_reg_launch<MT_F16, true>(x, residual, w, eps, h, y, rows, dim,
                                                              (cudaStream_t)stream);
    if (rc != 1) return rc;
    rc = MT_OK;
  }
  MT_DT_SWITCH(dtype, rc = vec ? launch(rms_norm_kernel<DT, true, true>, grid, dim3(256), 0, (cudaStream_t)stream, x,
                                        residual, w, eps, h, y, rows, (int)dim)
                               : launch(rms_norm_kernel<DT, true, false>, grid, dim3(256), 0,
                                        (cudaStream_t)stream, x, residual, w, eps, h, y, rows, (int)dim));
  return rc;
}

int mt_layer_norm(const void* x, const void* w, const void* b, float eps, void* y, int64_t rows, int64_t dim,
                  int dtype, mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(x && y, "mt_layer_norm: null pointer");
  MT_CHECK_ARG(rows >= 0 && dim > 0 && dim <= (1 << 24), "mt_layer_norm: rows=%lld dim=%lld", (long long)rows,
               (long long)dim);
  if (rows == 0) return MT_OK;
  const bool vec = (dtype == MT_BF16 || dtype == MT_F16) && dim % 256 == 0 && dim <= 4096 && aligned(x, 16) &&
                   aligned(y, 16) && (!w || aligned(w, 16)) && (!b || aligned(b, 16));
  if (vec) {
    const dim3 g4(static_cast<unsigned>((rows + 3) / 4)), blk(128);
    const cudaStream_t s = (cudaStream_t)stream;
#define MT_LN_REG(DTV)                                                                                         \
  switch (dim / 256) {                                                                                         \
    case 1: return launch(layer_norm_reg_kernel<DTV, 1>, g4, blk, 0, s, x, w, b, eps, y, rows);                \
    case 2: return launch(layer_norm_reg_kernel<DTV, 2>, g4, blk, 0, s, x, w, b, eps, y, rows);                \
    case 3: return launch(layer_norm_reg_kernel<DTV, 3>, g4, blk, 0, s, x, w, b, eps, y, rows);                \
    case 4: return launch(layer_norm_reg_kernel<DTV, 4>, g4, blk, 0, s, x, w, b, eps, y, rows);                \
    case 5: return launch(layer_norm_reg_kernel<DTV, 5>, g4, blk, 0, s, x, w, b, eps, y, rows);                \
    case 6: return launch(layer_norm_reg_kernel<DTV, 6>, g4, blk, 0, s, x, w, b, eps, y, rows);                \
    case 8: return launch(layer_norm_reg_kernel<DTV, 8>, g4, blk, 0, s, x, w, b, eps, y, rows);                \
    case 10: return launch(layer_norm_reg_kernel<DTV, 10>, g4, blk, 0, s, x, w, b, eps, y, rows);              \
    case 12: return launch(layer_norm_reg_kernel<DTV, 12>, g4, blk, 0, s, x, w, b, eps, y, rows);              \
    case 16: return launch(layer_norm_reg_kernel<DTV, 16>, g4, blk, 0, s, x, w, b, eps, y, rows);              \
    default: break;                                                                                            \
  }
    if (dtype == MT_BF16) { MT_LN_REG(MT_BF16) } else { MT_LN_REG(MT_F16) }
#undef MT_LN_REG
  }
  const dim3 grid(static_cast<unsigned>((rows + 7) / 8));
  int rc = MT_OK;
  MT_DT_SWITCH(dtype, rc = launch(layer_norm_kernel<DT>, grid, dim3(256), 0, (cudaStream_t)stream, x, w, b, eps, y,
                                  rows, (int)dim));
  return rc;
}

static int rope_run(const void* x, void* y, int64_t B, int64_t H, int64_t L, int64_t D, int dims, int traditional,
                    float base, float scale, int64_t offset, const RopeStrides& st, bool strided, int dtype,
                    mt_stream_t stream, const char* who) {
  clear_error();
  MT_CHECK_ARG(x && y, "%s: null pointer", who);
  MT_CHECK_ARG(B >= 0 && H >= 0 && L >= 0 && D > 0, "%s: bad shape", who);
  MT_CHECK_ARG(dims >= 2 && dims % 2 == 0 && dims <= D && dims <= 256, "%s: dims=%d vs D=%lld", who, dims,
               (long long)D);
  MT_CHECK_ARG(base > 0.f, "%s: base must be positive", who);
  const int64_t rows = B * H * L;
  if (rows == 0) return MT_OK;
  MT_CHECK_ARG(L < (int64_t(1) << 31) && (B * H + kRopeRows - 1) / kRopeRows < 65536,
               "%s: L=%lld or B*H=%lld too large for the grid", who, (long long)L, (long long)(B * H));
  const RopeFreqs f = make_freqs(dims, base);
  const dim3 grid(static_cast<unsigned>(L), static_cast<unsigned>((B * H + kRopeRows - 1) / kRopeRows));
  int rc = MT_OK;
  // 4 pairs per thread when every row and both halves start on 8 bytes
  const bool rows8 = st.xb % 4 == 0 && st.xh % 4 == 0 && st.xl % 4 == 0 && st.yb % 4 == 0 && st.yh % 4 == 0 &&
                     st.yl % 4 == 0;
  const int vec = dtype != MT_F32 && (dims / 2) % 4 == 0 && D % 4 == 0 && rows8 && aligned(x, 8) && aligned(y, 8);
  if (strided) {
    MT_DT_SWITCH(dtype, rc = launch((rope_kernel<DT, true>), grid, dim3(256), 0, (cudaStream_t)stream, x, y, B * H,
                                    (int)L, (int)D, dims, traditional, scale, offset, f, vec, st));
  } else {
    MT_DT_SWITCH(dtype, rc = launch((rope_kernel<DT, false>), grid, dim3(256), 0, (cudaStream_t)stream, x, y, B * H,
                                    (int)L, (int)D, dims, traditional, scale, offset, f, vec, st));
  }
  return rc;
}

int mt_rope(const void* x, void* y, int64_t B, int64_t H, int64_t L, int64_t D, int dims, int traditional,
            float base, float scale, int64_t offset, int dtype, mt_stream_t stream) {
  const RopeStrides st = {H > 0 ? H : 1, H * L * D, L * D, D, H * L * D, L * D, D};
  return rope_run(x, y, B, H, L, D, dims, traditional, base, scale, offset, st, false, dtype, stream, "mt_rope");
}

int mt_rope_strided(const void* x, void* y, int64_t B, int64_t H, int64_t L, int64_t D, int dims, int traditional,
                    float base, float scale, int64_t offset, int64_t x_sb, int64_t x_sh, int64_t x_sl, int64_t y_sb,
                    int64_t y_sh, int64_t y_sl, int dtype, mt_stream_t stream) {
  const RopeStrides st = {H > 0 ? H : 1, x_sb, x_sh, x_sl, y_sb, y_sh, y_sl};
  return rope_run(x, y, B, H, L, D, dims, traditional, base, scale, offset, st, true, dtype, stream,
                  "mt_rope_strided");
}

int mt_qk_norm_rope_cache(const void* q, const void* k, const void* v, int64_t q_stride, int64_t kv_stride,
                          const void* q_norm_w, const void* k_norm_w, float eps, void* q_out, void* k_cache,
                          void* v_cache, int64_t T, int64_t Hq, int64_t Hkv, int64_t D, int64_t cache_cap,
                          int64_t offset, float rope_base, int dtype, mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(q && k && v && q_norm_w && k_norm_w && q_out && k_cache && v_cache,
               "mt_qk_norm_rope_cache: null pointer");
  MT_CHECK_ARG(D == 128, "mt_qk_norm_rope_cache: head_dim %lld, only 128 is built", (long long)D);
  MT_CHECK_ARG(dtype == MT_BF16 || dtype == MT_F16, "mt_qk_norm_rope_cache: dtype must be bf16 or f16");
  MT_CHECK_ARG(T >= 0 && Hq > 0 && Hkv > 0 && offset >= 0 && offset + T <= cache_cap,
               "mt_qk_norm_rope_cache: offset %lld + T %lld exceeds cache capacity %lld", (long long)offset,
               (long long)T, (long long)cache_cap);
  MT_CHECK_ARG(q_stride % 4 == 0 && kv_stride % 4 == 0 && aligned(q, 8) && aligned(k, 8) && aligned(v, 8),
               "mt_qk_norm_rope_cache: rows must be 8-byte aligned");
  if (T == 0) return MT_OK;
  const RopeFreqs f = make_freqs(128, rope_base);
  const int64_t warps = T * (Hq + Hkv);
  const dim3 grid(static_cast<unsigned>((warps + 7) / 8));
  int rc = MT_OK;
  if (dtype == MT_BF16)
    rc = launch(qk_norm_rope_cache_kernel<MT_BF16>, grid, dim3(256), 0, (cudaStream_t)stream, q, k, v, q_stride,
                kv_stride, q_norm_w, k_norm_w, eps, q_out, k_cache, v_cache, (int)T, (int)Hq, (int)Hkv, cache_cap,
                offset, f);
  else
    rc = launch(qk_norm_rope_cache_kernel<MT_F16>, grid, dim3(256), 0, (cudaStream_t)stream, q, k, v, q_stride,
                kv_stride, q_norm_w, k_norm_w, eps, q_out, k_cache, v_cache, (int)T, (int)Hq, (int)Hkv, cache_cap,
                offset, f);
  return rc;
}

}  // extern "C"
