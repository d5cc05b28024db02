// RoPE frequencies and the Qwen3 per-head q/k prologue (RMSNorm over the
// head's 128 values, then RoPE at the token's position), shared by the
// standalone prologue kernel and the fused decode attention so that both
// produce bit-identical rotated rows.
#pragma once
#include <cmath>

#include "mt_common.cuh"

namespace mt {

struct RopeFreqs {
  float inv_freq[128];  // base^(-2j/dims), j < dims/2, computed on the host in double
};

inline RopeFreqs make_freqs(int dims, double base) {
  RopeFreqs f;
  for (int j = 0; j < 128; ++j)
    f.inv_freq[j] = j < dims / 2 ? static_cast<float>(pow(base, -2.0 * j / dims)) : 0.f;
  return f;
}

__device__ __forceinline__ void rope_pair(float a, float b, float c, float s, float& oa, float& ob) {
  // first = a*c - b*s, second = b*c + a*s  (autotuner/scaffold/lower.py:1279)
  oa = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
  ob = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
}

// sin and cos of the RoPE angle pos * inv_freq[j]: every caller derives them
// from this one expression, so a table of them and a direct call agree bitwise
__device__ __forceinline__ void rope_angle(int64_t pos, const RopeFreqs& f, int j, float& s, float& c) {
  sincosf(__fmul_rn(static_cast<float>(pos), f.inv_freq[j]), &s, &c);
}

// One head row of 128 values, one warp: lane l holds values 4l..4l+3 (`u`,
// and the norm weights in `uw`, as loaded). rms_norm(row, nw, eps) rounded to
// the element type (mx.fast.rms_norm), then rope (non-traditional: pairs
// (d, d+64)) with the angles angle(j, s, c), j < 64, rounded. Returns the
// lane's 4 output values packed (8 bytes).
template <int DT, class Angle>
__device__ __forceinline__ uint2 qk_norm_rope_vals(const uint2 u, const uint2 uw, float eps, const Angle& angle,
                                                   int lane) {
  using T = typename Elem<DT>::T;
  float v[4], g[4];
  {
    const T* e = reinterpret_cast<const T*>(&u);
    const T* ew = reinterpret_cast<const T*>(&uw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = Elem<DT>::to_f(e[i]);
      g[i] = Elem<DT>::to_f(ew[i]);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = fmaf(v[i], v[i], ss);
  ss = warp_sum(ss);
  const float scale = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, 128.f), eps));
  float n[4], p[4], o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) n[i] = round_to<DT>(__fmul_rn(__fmul_rn(v[i], scale), g[i]));
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = __shfl_xor_sync(0xffffffffu, n[i], 16);
  const bool first = lane < 16;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int j = (4 * lane + i) & 63;
    float s, c;
    angle(j, s, c);
    float o0, o1;
    if (first) {
      rope_pair(n[i], p[i], c, s, o0, o1);
      o[i] = o0;
    } else {
      rope_pair(p[i], n[i], c, s, o0, o1);
      o[i] = o1;
    }
  }
  uint2 out;
  T* eo = reinterpret_cast<T*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) eo[i] = Elem<DT>::from_f(o[i]);
  return out;
}

// qk_norm_rope_vals at position `pos`, the angles computed in place
template <int DT>
__device__ __forceinline__ uint2 qk_norm_rope_vals(const uint2 u, const uint2 uw, float eps, int64_t pos,
                                                   const RopeFreqs& f, int lane) {
  return qk_norm_rope_vals<DT>(u, uw, eps, [&](int j, float& s, float& c) { rope_angle(pos, f, j, s, c); }, lane);
}

}  // namespace mt
