// C entry points of the affine-quantized matmul family: argument checks and
// the choice between the vector kernel (M <= 8, decode) and the tcgen05
// matrix kernel (prefill).
#include "mt_common.cuh"
#include <cstdlib>

#include "qmm_common.cuh"

namespace mt {

constexpr int64_t kQmvMaxRows = 8;

static int check_common(const QmmRequest& r, const char* who) {
  MT_CHECK_ARG(r.x, "%s: x is NULL", who);
  MT_CHECK_ARG(r.bits == 4 || r.bits == 8, "%s: bits=%d (4 or 8)", who, r.bits);
  MT_CHECK_ARG(r.group == 32 || r.group == 64 || r.group == 128, "%s: group_size=%d (32, 64 or 128)", who,
               r.group);
  if (r.dtype != MT_BF16 && r.dtype != MT_F16) {
    set_error("%s: dtype %d is not built (bf16 or f16)", who, r.dtype);
    return MT_ERR_UNSUPPORTED;
  }
  MT_CHECK_ARG(r.M >= 0 && r.M < (int64_t(1) << 31), "%s: M=%lld", who, (long long)r.M);
  MT_CHECK_ARG(r.K > 0 && r.K % r.group == 0 && r.K < (int64_t(1) << 24),
               "%s: K=%lld must be a positive multiple of group_size %d", who, (long long)r.K, r.group);
  MT_CHECK_ARG(r.K % 64 == 0, "%s: K=%lld must be a multiple of 64", who, (long long)r.K);
  int nsets = 0;
  for (int s = 0; s < 3; ++s) {
    const QmmSetReq& q = r.set[s];
    if (q.N == 0) continue;
    MT_CHECK_ARG(q.N > 0 && q.N < (int64_t(1) << 31), "%s: N=%lld", who, (long long)q.N);
    MT_CHECK_ARG(q.w && q.s && q.b, "%s: weight set %d has a NULL pointer", who, s);
    MT_CHECK_ARG(q.y || (r.kind == QMM_SWIGLU && s == 1), "%s: output %d is NULL", who, s);
    MT_CHECK_ARG(aligned(q.w, 16), "%s: packed weights must be 16-byte aligned", who);
    ++nsets;
  }
  MT_CHECK_ARG(nsets > 0, "%s: no output", who);
  MT_CHECK_ARG(aligned(r.x, 16), "%s: x must be 16-byte aligned", who);
  if (r.kind == QMM_RESIDUAL) MT_CHECK_ARG(r.residual, "%s: residual is NULL", who);
  return MT_OK;
}

// Operand bytes a tensor-core launch keeps live: its block of x rows and its
// block of weight rows are each held under this, so both stay in the 126 MB
// L2 while the launch's tiles stream them. One launch over a large M x N
// spreads its CTAs' contiguous tile ranges over every token tile and every
// weight tile at once and misses L2 on both (Llama-3-8B gate/up at M = 16384:
// 20.9 GB read from DRAM per launch for 0.26 GB of operands). The 60 MB
// default measured best of 16/24/40/60/96 MB and unblocked on B200 (gate/up
// 5% faster than one launch, down unchanged; 16-24 MB blocks cost down 13-30%
// in launches). The environment variable MT_QMM_L2_BLOCK_BYTES overrides it
// (tests use a small value to reach the blocked path at small sizes).
static int64_t l2_block_bytes() {
  const char* e = getenv("MT_QMM_L2_BLOCK_BYTES");
  const long long v = e ? atoll(e) : 0;
  return v > 0 ? static_cast<int64_t>(v) : (int64_t(60) << 20);
}

// The tensor-core path over blocks of at most mc token rows x nc weight rows,
// weight blocks outermost so each stays in L2 while the token blocks pass.
// Only one projection or the SwiGLU pair is split by weight rows (the q/k/v
// triple only by token rows); outputs and residual keep the full row pitch.
static int run_tc_blocked(const QmmRequest& r, cudaStream_t stream) {
  const int64_t esz = 2;
  const int64_t budget = l2_block_bytes();
  const bool dual = r.kind == QMM_SWIGLU;
  int nsets = 0;
  for (int s = 0; s < 3; ++s) nsets += r.set[s].N > 0 ? 1 : 0;
  const bool split_n = dual || nsets == 1;
  int64_t mc = budget / (r.K * esz) / 128 * 128;
  if (mc < 128) mc = 128;
  const int64_t sets_n = dual ? 2 : 1;
  const int64_t row_bytes = sets_n * (r.K * r.bits / 8 + (r.K / r.group) * 2 * esz);
  // Sets with N = 0 are skipped: a q/k/v call may fill only set 1 or 2, and
  // the split then follows the first set that has rows (check_common has
  // seen at least one).
  int si = 0;
  while (si < 2 && r.set[si].N == 0) ++si;
  const int64_t N0 = r.set[si].N;
  int64_t nc = N0;
  if (split_n) {
    nc = budget / row_bytes / 128 * 128;
    if (nc < 128) nc = 128;
    if (nc > N0) nc = N0;
  }
  if (r.M <= mc && nc == N0) return qmm_tc_run(r, stream);
  // equal blocks (multiples of 128) rather than full ones and a small remainder
  const int64_t nbm = (r.M + mc - 1) / mc, nbn = (N0 + nc - 1) / nc;
  mc = ((r.M + nbm - 1) / nbm + 127) / 128 * 128;
  nc = ((N0 + nbn - 1) / nbn + 127) / 128 * 128;
  const int64_t words = r.K * r.bits / 32, G = r.K / r.group;
  for (int64_t n0 = 0; n0 < N0; n0 += nc) {
    for (int64_t m0 = 0; m0 < r.M; m0 += mc) {
      QmmRequest c = r;
      c.M = r.M - m0 < mc ? r.M - m0 : mc;
      c.x = static_cast<const char*>(r.x) + m0 * r.K * esz;
      int64_t ldy0 = 0;
      for (int s = 0; s < 3; ++s) {
        const QmmSetReq& q = r.set[s];
        if (q.N == 0) continue;
        QmmSetReq& o = c.set[s];
        const int64_t ldy = q.ldy > 0 ? q.ldy : q.N;
        if (s == si) ldy0 = ldy;
        o.ldy = ldy;
        const int64_t col = split_n ? n0 : 0;
        if (split_n) {
          o.N = N0 - n0 < nc ? N0 - n0 : nc;
          o.w = q.w + n0 * words;
          o.s = static_cast<const char*>(q.s) + n0 * G * esz;
          o.b = static_cast<const char*>(q.b) + n0 * G * esz;
        }
        if (q.y) o.y = static_cast<char*>(q.y) + (m0 * ldy + col) * esz;
      }
      if (r.residual) c.residual = static_cast<const char*>(r.residual) + (m0 * ldy0 + (split_n ? n0 : 0)) * esz;
      const int rc = qmm_tc_run(c, stream);
      if (rc != MT_OK) return rc;
    }
  }
  return MT_OK;
}

// ---------------------------------------------------------------- many rows
// From kGemmMinRows rows of x up, the weights are dequantised once into the
// workspace (MLX rounding, the same dequant_chunk as the fused kernels) and
// the product runs on the tcgen05 bf16/f16 GEMM of the dense path. The fused
// kernel dequantises every weight tile once per 128-token tile, so at large M
// its dequantiser warps bound it near a third of the tensor peak; one
// HBM-bound dequantisation pass (read N*K*bits/8, write N*K*2 bytes) plus a
// GEMM near 80% of the peak (SwiGLU applied in its epilogue) is the faster
// form there (Llama-3-8B prefill,
// M = 16384, 8-bit: gate 1.49 vs 3.68 ms, down 1.44 vs 3.92 ms). The products
// are the same dequantised weights times x, accumulated in fp32 in another
// order. MT_QMM_GEMM_MIN_ROWS overrides the threshold (tests use it to compare
// both forms).
constexpr int64_t kGemmMinRows = 1024;

static int64_t gemm_min_rows() {
  const char* e = getenv("MT_QMM_GEMM_MIN_ROWS");
  const long long v = e ? atoll(e) : 0;
  return v > 0 ? static_cast<int64_t>(v) : kGemmMinRows;
}

int gemm_tc_run(const void* x, const void* w, const void* bias, const void* residual, void* y, int64_t B,
                int64_t L, int64_t Cin, int64_t Cout, int taps, int stride, int padding, int act, int dtype,
                int bias_fused, int64_t ldy, cudaStream_t stream);

// One thread per 16-byte chunk of packed weights (32 values at 4 bits, 16 at
// 8): out[row, k] = round(round(s * q) + b), rows of K values. Weight row n
// goes to row n, or with inter >= 0 (the SwiGLU pair) to row
// 256 * (n / 128) + inter + n % 128: gate (inter 0) and up (inter 128) rows
// of the same 128 outputs side by side, as the GEMM's SwiGLU epilogue reads
// them.
template <int DT, int BITS>
__global__ void __launch_bounds__(256) dequant_rows_kernel(const uint8_t* __restrict__ w,
                                                           const uint16_t* __restrict__ s,
                                                           const uint16_t* __restrict__ b,
                                                           uint4* __restrict__ out, int64_t N, int K, int G,
                                                           int gshift, int inter) {
  constexpr int kVals = 128 / BITS;  // values per chunk
  // the previous kernel on the stream may still read `out` (the GEMM of the
  // set before, which shares this buffer)
  griddep_wait();
  griddep_launch();
  const int64_t per_row = K / kVals;
  const int64_t total = N * per_row;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = i / per_row;
    const int c = static_cast<int>(i - n * per_row);
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + n * (K * BITS / 8)) + c);
    const int g = (c * kVals) >> gshift;
    const uint16_t sb = __ldg(s + n * G + g), bb = __ldg(b + n * G + g);
    float sf, bf;
    if constexpr (DT == MT_BF16) {
      sf = __uint_as_float(static_cast<uint32_t>(sb) << 16);
      bf = __uint_as_float(static_cast<uint32_t>(bb) << 16);
    } else {
      sf = __half2float(__ushort_as_half(sb));
      bf = __half2float(__ushort_as_half(bb));
    }
    uint32_t o[kVals / 2];
    dequant_chunk<DT, BITS>(wv, sf, bf, o);
    const int64_t orow = inter < 0 ? n : (n >> 7) * 256 + inter + (n & 127);
    uint4* dst = out + (orow * K + static_cast<int64_t>(c) * kVals) / 8;
#pragma unroll
    for (int v = 0; v < kVals / 8; ++v) dst[v] = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
  }
}

static int dequant_rows(const QmmSetReq& q, int64_t K, int group, int bits, int dtype, void* out, int inter,
                        cudaStream_t stream) {
  int sms = 148;
  if (int rc = device_sm_count(&sms)) return rc;
  const int64_t chunks = q.N * (K * bits / 128);
  const int64_t want = (chunks + 255) / 256;
  const dim3 grid(static_cast<unsigned>(want < sms * 16 ? want : sms * 16));
  const int G = static_cast<int>(K / group), gshift = group == 32 ? 5 : group == 64 ? 6 : 7;
  const auto* w = reinterpret_cast<const uint8_t*>(q.w);
  const auto* s = static_cast<const uint16_t*>(q.s);
  const auto* b = static_cast<const uint16_t*>(q.b);
  auto* o = static_cast<uint4*>(out);
  const int k = static_cast<int>(K);
  if (dtype == MT_BF16)
    return bits == 4 ? launch(dequant_rows_kernel<MT_BF16, 4>, grid, dim3(256), 0, stream, w, s, b, o, q.N, k, G, gshift, inter)
                     : launch(dequant_rows_kernel<MT_BF16, 8>, grid, dim3(256), 0, stream, w, s, b, o, q.N, k, G, gshift, inter);
  return bits == 4 ? launch(dequant_rows_kernel<MT_F16, 4>, grid, dim3(256), 0, stream, w, s, b, o, q.N, k, G, gshift, inter)
                   : launch(dequant_rows_kernel<MT_F16, 8>, grid, dim3(256), 0, stream, w, s, b, o, q.N, k, G, gshift, inter);
}

// The path's buffers sit past the fused kernel's workspace area, whose
// counters the fused kernel expects to find zeroed.
static size_t gemm_ws_offset(int64_t M, int64_t n_total, int64_t K, int bits, int kind) {
  return (qmm_tc_workspace(M, n_total, K, bits, kind) + 4095) / 4096 * 4096;
}
static size_t gemm_ws_bytes(int64_t M, int64_t n_total, int64_t K, int kind) {
  (void)M;
  // one set's dequantised weights (n_total bounds every set); for SwiGLU the
  // gate and up rows interleaved in blocks of 128 (n_total = 2N)
  const int64_t rows = kind == 1 ? 256 * ((n_total / 2 + 127) / 128) : n_total;
  return static_cast<size_t>(rows) * K * 2;
}

// MT_ERR_UNSUPPORTED (nothing written) when the request does not fit this
// path: the caller then runs the fused kernel.
static int run_dequant_gemm(const QmmRequest& r, cudaStream_t stream) {
  const bool dual = r.kind == QMM_SWIGLU;
  int64_t n_total = 0;
  for (int s = 0; s < 3; ++s) n_total += r.set[s].N;
  const int kind = dual ? 1 : 0;
  const size_t off = gemm_ws_offset(r.M, n_total, r.K, r.bits, kind);
  if (!r.ws || r.ws_bytes < off + gemm_ws_bytes(r.M, n_total, r.K, kind)) return MT_ERR_UNSUPPORTED;
  char* wbuf = static_cast<char*>(r.ws) + off;
  if (dual) {
    // gate and up rows interleaved in 128-row blocks, one GEMM whose epilogue
    // applies SwiGLU to each (gate, up) column pair
    const int64_t N = r.set[0].N;
    const int64_t ldy = r.set[0].ldy > 0 ? r.set[0].ldy : N;
    for (int s = 0; s < 2; ++s)
      if (int rc = dequant_rows(r.set[s], r.K, r.group, r.bits, r.dtype, wbuf, 128 * s, stream)) return rc;
    return gemm_tc_run(r.x, wbuf, nullptr, nullptr, r.set[0].y, 1, r.M, r.K, N, 1, 1, 0, 2, r.dtype, 1, ldy, stream);
  }
  for (int s = 0; s < 3; ++s) {
    const QmmSetReq& q = r.set[s];
    if (q.N == 0) continue;
    const int64_t ldy = q.ldy > 0 ? q.ldy : q.N;
    if (int rc = dequant_rows(q, r.K, r.group, r.bits, r.dtype, wbuf, -1, stream)) return rc;
    const void* res = r.kind == QMM_RESIDUAL ? r.residual : nullptr;
    if (int rc = gemm_tc_run(r.x, wbuf, nullptr, res, q.y, 1, r.M, r.K, q.N, 1, 1, 0, 0, r.dtype, 1, ldy, stream))
      return rc;
  }
  return MT_OK;
}

static int run(const QmmRequest& r, cudaStream_t stream, const char* who) {
  clear_error();
  const int rc = check_common(r, who);
  if (rc != MT_OK) return rc;
  if (r.M == 0) return MT_OK;
  if (r.M <= kQmvMaxRows) return qmv_run(r, stream);
  if (r.M >= gemm_min_rows()) {
    const int g = run_dequant_gemm(r, stream);
    if (g != MT_ERR_UNSUPPORTED) return g;
    clear_error();
  }
  return run_tc_blocked(r, stream);
}

}  // namespace mt

using namespace mt;

extern "C" {

int mt_quantized_matmul(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y,
                        int64_t M, int64_t N, int64_t K, int group_size, int bits, int dtype, void* workspace,
                        size_t workspace_bytes, mt_stream_t stream) {
  QmmRequest r = {};
  r.x = x;
  r.set[0] = {w, scales, biases, y, N};
  r.M = M;
  r.K = K;
  r.group = group_size;
  r.bits = bits;
  r.dtype = dtype;
  r.kind = QMM_PLAIN;
  r.ws = workspace;
  r.ws_bytes = workspace_bytes;
  MT_CHECK_ARG(N > 0, "mt_quantized_matmul: N=%lld", (long long)N);
  return run(r, (cudaStream_t)stream, "mt_quantized_matmul");
}

int mt_quantized_matmul_residual(const void* x, const uint32_t* w, const void* scales, const void* biases,
                                 const void* residual, void* y, int64_t M, int64_t N, int64_t K, int group_size,
                                 int bits, int dtype, void* workspace, size_t workspace_bytes, mt_stream_t stream) {
  QmmRequest r = {};
  r.x = x;
  r.residual = residual;
  r.set[0] = {w, scales, biases, y, N};
  r.M = M;
  r.K = K;
  r.group = group_size;
  r.bits = bits;
  r.dtype = dtype;
  r.kind = QMM_RESIDUAL;
  r.ws = workspace;
  r.ws_bytes = workspace_bytes;
  MT_CHECK_ARG(N > 0, "mt_quantized_matmul_residual: N=%lld", (long long)N);
  return run(r, (cudaStream_t)stream, "mt_quantized_matmul_residual");
}

int mt_quantized_matmul_residual_rms_norm(const void* x, const uint32_t* w, const void* scales, const void* biases,
                                          const void* residual, const void* norm_w, float eps, void* h, void* y,
                                          int64_t M, int64_t N, int64_t K, int group_size, int bits, int dtype,
                                          void* workspace, size_t workspace_bytes, mt_stream_t stream) {
  MT_CHECK_ARG(norm_w && h && y, "mt_quantized_matmul_residual_rms_norm: null output or norm weight");
  int rc = mt_quantized_matmul_residual(x, w, scales, biases, residual, h, M, N, K, group_size, bits, dtype,
                                        workspace, workspace_bytes, stream);
  if (rc != MT_OK) return rc;
  return mt_rms_norm(h, norm_w, eps, y, M, N, dtype, stream);
}

int mt_quantized_matmul_swiglu(const void* x, const uint32_t* wg, const void* sg, const void* bg, const uint32_t* wu,
                               const void* su, const void* bu, void* y, int64_t M, int64_t N, int64_t K,
                               int group_size, int bits, int dtype, void* workspace, size_t workspace_bytes,
                               mt_stream_t stream) {
  QmmRequest r = {};
  r.x = x;
  r.set[0] = {wg, sg, bg, y, N};
  r.set[1] = {wu, su, bu, nullptr, N};
  r.M = M;
  r.K = K;
  r.group = group_size;
  r.bits = bits;
  r.dtype = dtype;
  r.kind = QMM_SWIGLU;
  r.ws = workspace;
  r.ws_bytes = workspace_bytes;
  MT_CHECK_ARG(N > 0, "mt_quantized_matmul_swiglu: N=%lld", (long long)N);
  return run(r, (cudaStream_t)stream, "mt_quantized_matmul_swiglu");
}

int mt_quantized_matmul_multi(const void* x, const uint32_t* w0, const void* s0, const void* b0, void* y0, int64_t N0,
                              const uint32_t* w1, const void* s1, const void* b1, void* y1, int64_t N1,
                              const uint32_t* w2, const void* s2, const void* b2, void* y2, int64_t N2, int64_t M,
                              int64_t K, int group_size, int bits, int dtype, void* workspace,
                              size_t workspace_bytes, mt_stream_t stream) {
  QmmRequest r = {};
  r.x = x;
  r.set[0] = {w0, s0, b0, y0, N0};
  r.set[1] = {w1, s1, b1, y1, N1};
  r.set[2] = {w2, s2, b2, y2, N2};
  r.M = M;
  r.K = K;
  r.group = group_size;
  r.bits = bits;
  r.dtype = dtype;
  r.kind = QMM_PLAIN;
  r.ws = workspace;
  r.ws_bytes = workspace_bytes;
  MT_CHECK_ARG(N0 >= 0 && N1 >= 0 && N2 >= 0, "mt_quantized_matmul_multi: negative N");
  return run(r, (cudaStream_t)stream, "mt_quantized_matmul_multi");
}

// RMSNorm fused into the decode matmul's staging of x (M <= 4): every CTA of
// the streamed kernel normalises the rows it stages, so no normalised copy of
// x is written.
static int run_normed(QmmRequest& r, const void* norm_w, float eps, cudaStream_t stream, const char* who) {
  clear_error();
  MT_CHECK_ARG(norm_w, "%s: norm weight is NULL", who);
  MT_CHECK_ARG(aligned(norm_w, 16), "%s: norm weight must be 16-byte aligned", who);
  MT_CHECK_ARG(eps >= 0.f, "%s: eps=%g", who, static_cast<double>(eps));
  r.norm_w = norm_w;
  r.norm_eps = eps;
  const int rc = check_common(r, who);
  if (rc != MT_OK) return rc;
  if (r.M == 0) return MT_OK;
  if (!qmv_stream_eligible(r)) {
    set_error("%s: needs the streamed decode kernel (M <= 4, 4-bit, bf16/f16, K <= 16384; M=%lld bits=%d)", who,
              (long long)r.M, r.bits);
    return MT_ERR_UNSUPPORTED;
  }
  return qmv_stream_run(r, stream);
}

int mt_rms_norm_quantized_matmul_multi(const void* x, const void* norm_w, float eps, const uint32_t* w0,
                                       const void* s0, const void* b0, void* y0, int64_t N0, const uint32_t* w1,
                                       const void* s1, const void* b1, void* y1, int64_t N1, const uint32_t* w2,
                                       const void* s2, const void* b2, void* y2, int64_t N2, int64_t M, int64_t K,
                                       int group_size, int bits, int dtype, mt_stream_t stream) {
  QmmRequest r = {};
  r.x = x;
  r.set[0] = {w0, s0, b0, y0, N0};
  r.set[1] = {w1, s1, b1, y1, N1};
  r.set[2] = {w2, s2, b2, y2, N2};
  r.M = M;
  r.K = K;
  r.group = group_size;
  r.bits = bits;
  r.dtype = dtype;
  r.kind = QMM_PLAIN;
  MT_CHECK_ARG(N0 >= 0 && N1 >= 0 && N2 >= 0, "mt_rms_norm_quantized_matmul_multi: negative N");
  return run_normed(r, norm_w, eps, (cudaStream_t)stream, "mt_rms_norm_quantized_matmul_multi");
}

int mt_rms_norm_quantized_matmul_swiglu(const void* x, const void* norm_w, float eps, const uint32_t* wg,
                                        const void* sg, const void* bg, const uint32_t* wu, const void* su,
                                        const void* bu, void* y, int64_t M, int64_t N, int64_t K, int group_size,
                                        int bits, int dtype, mt_stream_t stream) {
  QmmRequest r = {};
  r.x = x;
  r.set[0] = {wg, sg, bg, y, N};
  r.set[1] = {wu, su, bu, nullptr, N};
  r.M = M;
  r.K = K;
  r.group = group_size;
  r.bits = bits;
  r.dtype = dtype;
  r.kind = QMM_SWIGLU;
  MT_CHECK_ARG(N > 0, "mt_rms_norm_quantized_matmul_swiglu: N=%lld", (long long)N);
  return run_normed(r, norm_w, eps, (cudaStream_t)stream, "mt_rms_norm_quantized_matmul_swiglu");
}

size_t mt_qmm_workspace_bytes(int64_t M, int64_t n_total, int64_t K, int bits, int kind) {
  if (M <= kQmvMaxRows) return 0;
  if (M >= gemm_min_rows() && kind <= 1)
    return gemm_ws_offset(M, n_total, K, bits, kind) + gemm_ws_bytes(M, n_total, K, kind);
  return qmm_tc_workspace(M, n_total, K, bits, kind);
}

}  // extern "C"
