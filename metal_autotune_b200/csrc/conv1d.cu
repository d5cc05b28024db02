// mx.conv1d for the Whisper encoder's conv stem (mlx-whisper conv1: 128 ->
// 1280, k3 s1 p1; conv2: 1280 -> 1280, k3 s2 p1; each followed by its bias and
// GELU), as one implicit GEMM with the bias and GELU in the epilogue.
//
// Channels-last x [N, L, Cin], w [Cout, K, Cin] (mlx layouts), y [N, Lout, Cout].
// GEMM view: rows m = (n, t) over N*Lout output positions, columns = Cout, and
// the reduction runs over (tap k, input channel ci): row m's slice for tap k is
// x[n, t*stride + k - pad, :], contiguous in ci (zero outside [0, L)), and
// column co's slice is w[co, k, :], contiguous too. A CTA computes a 128 x 128
// output tile over 32-wide reduction chunks (each inside one tap, so Cin must
// be a multiple of 32): both operand tiles are copied with cp.async into a
// 4-stage ring of XOR-swizzled shared memory and multiplied with mma.sync
// m16n8k16 (bf16/f16 in, fp32 accumulate; 8 warps of 64 x 32). The epilogue
// rounds as the separate MLX ops would: conv, + bias, GELU, each to the
// element type (GELU evaluated in fp32 on the rounded input, device erff), and
// stages the tile in shared memory for 16-byte coalesced stores.
#include "mma_sync.cuh"
#include "mt_common.cuh"

namespace mt {

constexpr int kCvBM = 128, kCvBN = 128, kCvBK = 32;
constexpr int kCvThreads = 256;
constexpr int kCvTileBytes = kCvBM * kCvBK * 2;  // one operand tile: 128 rows x 64 bytes
constexpr int kCvStages = 4;                        // cp.async ring depth
constexpr int kCvSmem = kCvStages * 2 * kCvTileBytes;
static_assert(kCvBM * (kCvBN + 8) * 2 <= kCvSmem, "the staged output tile reuses the ring");

struct Conv1dParams {
  const void* x;
  const void* w;
  const void* bias;
  void* y;
  int64_t M;  // N * Lout
  int L, Lout, Cin, Cout, K, stride, pad;
  int bias_fused;  // 1: round(sum + bias) once (mx.addmm, nn.Linear); 0: round(round(sum) + bias) (conv, then + bias)
};

// byte offset of 16-byte chunk c (0..3) of row r in a tile of 64-byte rows:
// the XOR spreads the 8 rows an ldmatrix reads over all 32 banks
__device__ __forceinline__ int cv_swz(int r, int c) { return r * 64 + ((c ^ ((r >> 1) & 3)) << 4); }

template <int DT, int ACT>
__global__ void __launch_bounds__(kCvThreads, 2) conv1d_kernel(const Conv1dParams p) {
  using T = typename Elem<DT>::T;
  extern __shared__ __align__(128) uint8_t cv_smem[];
  auto sa = [&](int s) { return cv_smem + s * 2 * kCvTileBytes; };
  auto sb = [&](int s) { return cv_smem + s * 2 * kCvTileBytes + kCvTileBytes; };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wm = warp >> 2, wn = warp & 3;  // warp tile: rows wm*64.., columns wn*32..
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kCvBM;
  const int n0 = blockIdx.x * kCvBN;
  const T* x = static_cast<const T*>(p.x);
  const T* w = static_cast<const T*>(p.w);

  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid

  // per-thread copy slots: 2 chunks of A and 2 of B per reduction step
  // (512 16-byte chunks each), fixed rows for the whole K loop
  int a_r[2], a_c[2];
  int64_t a_base[2];  // element offset of (n, t*stride - pad, 0), or -1 past the last row
  int a_t0[2];        // t*stride - pad of the row
  for (int i = 0; i < 2; ++i) {
    const int idx = tid + i * kCvThreads;
    a_r[i] = idx >> 2;
    a_c[i] = idx & 3;
    const int64_t m = m0 + a_r[i];
    if (m < p.M) {
      const int64_t n = m / p.Lout;
      const int t = static_cast<int>(m - n * p.Lout);
      a_t0[i] = t * p.stride - p.pad;
      a_base[i] = n * p.L;
    } else {
      a_t0[i] = 0;
      a_base[i] = -1;
    }
  }
  const int nk = p.K * p.Cin / kCvBK;
  auto load = [&](int kc, int buf) {
    const int e0 = kc * kCvBK;
    const int tap = e0 / p.Cin, ci0 = e0 - tap * p.Cin;
    for (int i = 0; i < 2; ++i) {
      const int src = a_t0[i] + tap;
      const bool ok = a_base[i] >= 0 && src >= 0 && src < p.L;
      const T* g = ok ? x + (a_base[i] + src) * p.Cin + ci0 + a_c[i] * 8 : x;
      cp_async16(sa(buf) + cv_swz(a_r[i], a_c[i]), g, ok);
      const int co = n0 + a_r[i];
      const bool okb = co < p.Cout;
      const T* gb = okb ? w + (static_cast<int64_t>(co) * p.K + tap) * p.Cin + ci0 + a_c[i] * 8 : w;
      cp_async16(sb(buf) + cv_swz(a_r[i], a_c[i]), gb, okb);
    }
  };

  float acc[4][4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.f;

  // ring of kCvStages chunks: chunk kc lives in stage kc % kCvStages; the
  // copies of the next kCvStages - 1 chunks are in flight while one is used
#pragma unroll
  for (int s = 0; s < kCvStages - 1; ++s) {
    if (s < nk) load(s, s);
    cp_async_commit();
  }
  for (int kc = 0; kc < nk; ++kc) {
    const int buf = kc % kCvStages;
    cp_async_wait<kCvStages - 2>();
    __syncthreads();  // chunk kc landed for every thread; stage (kc - 1) % kCvStages is free
    if (kc + kCvStages - 1 < nk) load(kc + kCvStages - 1, (kc + kCvStages - 1) % kCvStages);
    cp_async_commit();
    const uint32_t abase = smem_addr(sa(buf)), bbase = smem_addr(sb(buf));
#pragma unroll
    for (int ks = 0; ks < kCvBK / 16; ++ks) {
      uint32_t af[4][4];
#pragma unroll
      for (int mi = 0; mi < 4; ++mi) {
        const int r = wm * 64 + mi * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = ks * 2 + (lane >> 4);
        ldsm_x4(abase + cv_swz(r, c), af[mi][0], af[mi][1], af[mi][2], af[mi][3]);
      }
#pragma unroll
      for (int nj = 0; nj < 4; nj += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = wn * 32 + nj * 8 + (lane & 7) + (lane >> 4) * 8;
        const int c = ks * 2 + ((lane >> 3) & 1);
        ldsm_x4(bbase + cv_swz(r, c), b0, b1, b2, b3);
#pragma unroll
        for (int mi = 0; mi < 4; ++mi) {
          mma16816<DT>(acc[mi][nj], af[mi], b0, b1);
          mma16816<DT>(acc[mi][nj + 1], af[mi], b2, b3);
        }
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // every warp is done with the ring: it now stages the output tile

  // epilogue: conv -> round, + bias -> round, GELU -> round, into a shared
  // 128 x 128 tile (rows padded by 16 bytes), then 16-byte coalesced stores
  constexpr int kPitch = kCvBN + 8;  // elements per staged row
  T* tile = reinterpret_cast<T*>(cv_smem);
  const T* bias = static_cast<const T*>(p.bias);
  const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int rl = wm * 64 + mi * 16 + g + h * 8;
#pragma unroll
      for (int nj = 0; nj < 4; ++nj) {
        const int cl = wn * 32 + nj * 8 + 2 * t4;
        const int co = n0 + cl;
        float v[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float b = (bias && co + e < p.Cout) ? Elem<DT>::to_f(bias[co + e]) : 0.f;
          float u = p.bias_fused ? round_to<DT>(acc[mi][nj][h * 2 + e] + b)
                                 : round_to<DT>(round_to<DT>(acc[mi][nj][h * 2 + e]) + b);
          if (ACT == 1) u = round_to<DT>(gelu_erf_f32(u));
          v[e] = u;
        }
        *reinterpret_cast<typename Elem<DT>::T2*>(tile + rl * kPitch + cl) = Elem<DT>::pack2(v[0], v[1]);
      }
    }
  __syncthreads();
  T* y = static_cast<T*>(p.y);
  const bool vec = (p.Cout & 7) == 0 && (reinterpret_cast<uintptr_t>(p.y) & 15) == 0;
  for (int i = tid; i < kCvBM * (kCvBN / 8); i += kCvThreads) {
    const int rl = i / (kCvBN / 8), c8 = (i % (kCvBN / 8)) * 8;
    const int64_t m = m0 + rl;
    const int co = n0 + c8;
    if (m >= p.M || co >= p.Cout) continue;
    const T* src = tile + rl * kPitch + c8;
    T* dst = y + m * p.Cout + co;
    if (vec && co + 8 <= p.Cout) {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
    } else {
      for (int e = 0; e < 8 && co + e < p.Cout; ++e) dst[e] = src[e];
    }
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

extern "C" int mt_conv1d(const void* x, const void* w, const void* bias, void* y, int64_t N, int64_t L, int64_t Cin,
                         int64_t Cout, int K, int stride, int padding, int act, int dtype, mt_stream_t stream) {
  clear_error();
  return conv1d_run(x, w, bias, y, N, L, Cin, Cout, K, stride, padding, act, dtype, 0, (cudaStream_t)stream);
}

// The implicit GEMM for mt_conv1d and the 16-bit mt_linear (one tap, bias
// fused before the rounding as mx.addmm does).
int mt::conv1d_run(const void* x, const void* w, const void* bias, void* y, int64_t N, int64_t L, int64_t Cin,
                   int64_t Cout, int K, int stride, int padding, int act, int dtype, int bias_fused,
                   cudaStream_t stream) {
  MT_CHECK_ARG(x && w && y, "mt_conv1d: null pointer");
  MT_CHECK_ARG(N >= 0 && L >= 1 && Cin >= 1 && Cout >= 1 && K >= 1 && stride >= 1 && padding >= 0,
               "mt_conv1d: N=%lld L=%lld Cin=%lld Cout=%lld K=%d stride=%d padding=%d", (long long)N, (long long)L,
               (long long)Cin, (long long)Cout, K, stride, padding);
  MT_CHECK_ARG(act == 0 || act == 1, "mt_conv1d: act=%d (0 none, 1 GELU)", act);
  MT_CHECK_ARG(L + 2 * static_cast<int64_t>(padding) >= K, "mt_conv1d: input of %lld + 2*%d is shorter than the kernel %d",
               (long long)L, padding, K);
  MT_CHECK_ARG(L < (1 << 30) && Cout < (1 << 30) && static_cast<int64_t>(K) * Cin < (1 << 30), "mt_conv1d: too large");
  if (dtype != MT_BF16 && dtype != MT_F16) {
    set_error("mt_conv1d: dtype %d is not built (bf16 or f16)", dtype);
    return MT_ERR_UNSUPPORTED;
  }
  MT_CHECK_ARG(aligned(x, 16) && aligned(w, 16) && aligned(y, 4), "mt_conv1d: x and w must be 16-byte aligned");
  const int64_t Lout = (L + 2 * padding - K) / stride + 1;
  if (N == 0) return MT_OK;
  // the tcgen05 kernel takes every shape of the targets (Cin a multiple of
  // 64, or of 8 for one tap; stride 1 or 2 with L a multiple of it; up to 4
  // taps); the mma.sync kernel below serves the rest
  const int tc = gemm_tc_run(x, w, bias, nullptr, y, N, L, Cin, Cout, K, stride, padding, act, dtype, bias_fused,
                             Cout, stream);
  if (tc != MT_ERR_UNSUPPORTED) return tc;
  clear_error();
  if (Cin % kCvBK != 0) {
    set_error("mt_conv1d: Cin=%lld must be a multiple of %d", (long long)Cin, kCvBK);
    return MT_ERR_UNSUPPORTED;
  }
  Conv1dParams p = {x, w, bias, y, N * Lout, (int)L, (int)Lout, (int)Cin, (int)Cout, K, stride, padding, bias_fused};
  MT_CHECK_ARG(p.M / kCvBM < 65535, "mt_conv1d: %lld output rows exceed the grid", (long long)p.M);
  const dim3 grid(static_cast<unsigned>((Cout + kCvBN - 1) / kCvBN), static_cast<unsigned>((p.M + kCvBM - 1) / kCvBM));
  const cudaStream_t s = stream;
  auto run = [&](auto kern) -> int {
    if (int e = ensure_smem(kern, kCvSmem)) return e;
    return launch(kern, grid, dim3(kCvThreads), kCvSmem, s, p);
  };
  if (dtype == MT_BF16) return act ? run(conv1d_kernel<MT_BF16, 1>) : run(conv1d_kernel<MT_BF16, 0>);
  return act ? run(conv1d_kernel<MT_F16, 1>) : run(conv1d_kernel<MT_F16, 0>);
}
