// Shared pieces of the affine-quantized matmul kernels.
#pragma once
#include "mt_common.cuh"

namespace mt {

enum QmmKind { QMM_PLAIN = 0, QMM_RESIDUAL = 1, QMM_SWIGLU = 2 };

struct QmmSetReq {
  const uint32_t* w;
  const void* s;
  const void* b;
  void* y;
  int64_t N;
  int64_t ldy;  // elements between output rows (and residual rows); 0 means N
};

// One quantized-matmul launch request as the entry points describe it.
struct QmmRequest {
  const void* x;
  const void* residual;  // QMM_RESIDUAL: [M, N] added after rounding
  QmmSetReq set[3];      // plain: up to 3 projections; SwiGLU: gate, up
  int64_t M, K;
  int group, bits, dtype;
  QmmKind kind;
  void* ws;
  size_t ws_bytes;
  const void* norm_w;  // non-NULL: x is first RMS-normalised with this weight (decode only)
  float norm_eps;
};

int qmv_run(const QmmRequest& r, cudaStream_t stream);
bool qmv_stream_eligible(const QmmRequest& r);
int qmv_stream_run(const QmmRequest& r, cudaStream_t stream);
int qmm_tc_run(const QmmRequest& r, cudaStream_t stream);
size_t qmm_tc_workspace(int64_t M, int64_t n_total, int64_t K, int bits, int kind);

// Streaming 16-byte load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ld_stream_v4(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Nibbles 2p and 2p+1 of a packed word as the bf16x2 bit patterns 0x4300|q,
// i.e. the values 128+q (exact in bf16). `lo` is the word, `hi` the word >> 4.
__device__ __forceinline__ uint32_t nibble_pair_bf16(uint32_t lo, uint32_t hi, int p) {
  const uint32_t sel = static_cast<uint32_t>(p | (p << 4) | ((4 + p) << 8) | ((4 + p) << 12));
  return (__byte_perm(lo, hi, sel) & 0x000F000Fu) | 0x43004300u;
}
// Same for fp16 with 0x6400|q = 1024+q.
__device__ __forceinline__ uint32_t nibble_pair_f16(uint32_t lo, uint32_t hi, int p) {
  const uint32_t sel = static_cast<uint32_t>(p | (p << 4) | ((4 + p) << 8) | ((4 + p) << 12));
  return (__byte_perm(lo, hi, sel) & 0x000F000Fu) | 0x64006400u;
}
// Bytes 2p and 2p+1 of a word as fp16x2 1024+q (8-bit values fit the fp16 mantissa).
__device__ __forceinline__ uint32_t byte_pair_f16(uint32_t w, int p) {
  const uint32_t sel = static_cast<uint32_t>((2 * p) | (4 << 4) | ((2 * p + 1) << 8) | (4 << 12));
  return __byte_perm(w, 0x64u, sel);  // byte 4 of {0x64, w} = 0x64: (0x64 << 8) | b
}

__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) {
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ __nv_bfloat162 bits_bf2(uint32_t v) {
  return *reinterpret_cast<__nv_bfloat162*>(&v);
}
__device__ __forceinline__ uint32_t h2_bits(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __half2 bits_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }

// MLX affine dequantisation of one 16-byte chunk into packed element pairs,
// w = round(round(scale * q) + bias) in the element type (MLX's
// quantized.h `dequantize`, restated in the LFM2 kernel header `mlx_deq8`:
// examples/lfm2_5_1_2b_prefill/lfm2_5_1_2b_prefill_artifact/kernels/
// r1f9367e50750eb01_unroll_hoist.launch.json). 4-bit: 32 values -> 16
// pairs; 8-bit: 16 values -> 8 pairs.
//
// bf16, 4-bit: (128+q)*s - 128*s in one fused op is exactly s*q before its
// single rounding, so round(s*q) costs one HFMA2; -128*s is exact for every
// finite bf16 scale below 2^120. fp16: (1024+q) - 1024 is exact, then one
// rounded multiply (__hmul2_rn: a plain __hmul2 followed by the bias add may
// be contracted into one fused multiply-add, which skips the rounding of s*q
// and moves the result by up to a few ulps). bf16, 8-bit: q and s*q are
// exact in fp32, then rounded once to bf16.
template <int DT, int BITS>
__device__ __forceinline__ void dequant_chunk(const uint4 wv, float s, float b, uint32_t* out);

template <>
__device__ __forceinline__ void dequant_chunk<MT_BF16, 4>(const uint4 wv, float s, float b,
                                                          uint32_t* out) {
  const __nv_bfloat162 s2 = __float2bfloat162_rn(s);
  const __nv_bfloat162 m2 = __float2bfloat162_rn(-128.f * __bfloat162float(__float2bfloat16_rn(s)));
  const __nv_bfloat162 b2 = __float2bfloat162_rn(b);
  const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int wi = 0; wi < 4; ++wi) {
    const uint32_t lo = words[wi], hi = words[wi] >> 4;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const __nv_bfloat162 v = bits_bf2(nibble_pair_bf16(lo, hi, p));
      out[wi * 4 + p] = bf2_bits(__hadd2(__hfma2(v, s2, m2), b2));
    }
  }
}

template <>
__device__ __forceinline__ void dequant_chunk<MT_F16, 4>(const uint4 wv, float s, float b,
                                                         uint32_t* out) {
  const __half2 s2 = __float2half2_rn(s);
  const __half2 b2 = __float2half2_rn(b);
  const __half2 k1024 = __float2half2_rn(1024.f);
  const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int wi = 0; wi < 4; ++wi) {
    const uint32_t lo = words[wi], hi = words[wi] >> 4;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const __half2 q = __hsub2(bits_h2(nibble_pair_f16(lo, hi, p)), k1024);
      out[wi * 4 + p] = h2_bits(__hadd2(__hmul2_rn(q, s2), b2));
    }
  }
}

template <>
__device__ __forceinline__ void dequant_chunk<MT_BF16, 8>(const uint4 wv, float s, float b,
                                                          uint32_t* out) {
  const float sr = __bfloat162float(__float2bfloat16_rn(s));
  const __nv_bfloat162 b2 = __float2bfloat162_rn(b);
  const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int wi = 0; wi < 4; ++wi) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const float q0 = static_cast<float>((words[wi] >> (16 * p)) & 0xFFu);
      const float q1 = static_cast<float>((words[wi] >> (16 * p + 8)) & 0xFFu);
      const __nv_bfloat162 t = __floats2bfloat162_rn(sr * q0, sr * q1);
      out[wi * 2 + p] = bf2_bits(__hadd2(t, b2));
    }
  }
}

template <>
__device__ __forceinline__ void dequant_chunk<MT_F16, 8>(const uint4 wv, float s, float b,
                                                         uint32_t* out) {
  const __half2 s2 = __float2half2_rn(s);
  const __half2 b2 = __float2half2_rn(b);
  const __half2 k1024 = __float2half2_rn(1024.f);
  const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int wi = 0; wi < 4; ++wi) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const __half2 q = __hsub2(bits_h2(byte_pair_f16(words[wi], p)), k1024);
      out[wi * 2 + p] = h2_bits(__hadd2(__hmul2_rn(q, s2), b2));
    }
  }
}

// silu(g) * u with each op rounded to the element type, sigmoid written as
// 1 / (1 + exp(-x)) (autotuner/scaffold/lower.py:80). Inputs are already
// rounded values; the caller rounds the result.
template <int DT>
__device__ __forceinline__ float swiglu_rounded(float g, float u) {
  const float sg = round_to<DT>(1.0f / (1.0f + expf(-g)));
  const float a = round_to<DT>(g * sg);
  return a * u;
}

// swiglu_rounded for two values, the sigmoid from the hardware exponential
// and reciprocal approximations (a few fp32 ulps; the bf16 / f16 roundings that
// follow hide the difference except near rounding boundaries, where the result
// moves by one ulp of the element type) and each rounding done for both values
// with one packed conversion. g and u are the raw fp32 accumulators.
template <int DT>
__device__ __forceinline__ typename Elem<DT>::T2 swiglu2_fast(float g0, float g1, float u0, float u1) {
  const float2 g = round2_to<DT>(g0, g1);
  const float2 u = round2_to<DT>(u0, u1);
  const float2 sg = round2_to<DT>(__fdividef(1.0f, 1.0f + __expf(-g.x)), __fdividef(1.0f, 1.0f + __expf(-g.y)));
  const float2 a = round2_to<DT>(g.x * sg.x, g.y * sg.y);
  return Elem<DT>::pack2(a.x * u.x, a.y * u.y);
}

}  // namespace mt
