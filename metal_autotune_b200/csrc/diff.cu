// Output-diff reduction for the verification ladder: one read of candidate a
// and reference b produces every statistic the reference's comparison
// policy needs (autotuner_runtime/numeric.py:50-107, exact.py:5-10,
// autotuner/ladder/numeric.py:22-35, autotuner/artifact/validate.py:64-103).
//
// The per-element excess is computed in fp32 exactly as the policy states it
// (allowed = max(atol + rtol*|b|, wobble); excess = |a-b| - allowed, with the
// overflow-safe scaled form where that is NaN), so max/argmax/count match a
// CPU restatement bit for bit. Block partials go to the workspace and the
// last block to finish (atomic counter) folds them with all its threads in a
// fixed order (thread t: blocks t, t+256, ...; then a fixed warp and block
// merge), so the fp64 cosine sums do not depend on scheduling either. The
// block count depends only on n. Inputs are read as 16-byte vectors when both
// are 16-byte aligned, the next vectors in flight while one is visited.
#include <type_traits>

#include "mt_common.cuh"

namespace mt {

struct DiffPartial {
  float max_excess;
  float max_abs;
  float amax_a, amax_b;
  int64_t excess_index;
  int64_t over, viol, first_viol, mism, first_mism, nan_ex;
  double dab, daa, dbb;
};

__device__ __forceinline__ void merge(DiffPartial& x, const DiffPartial& y) {
  if (y.excess_index >= 0 &&
      (x.excess_index < 0 || y.max_excess > x.max_excess ||
       (y.max_excess == x.max_excess && y.excess_index < x.excess_index))) {
    x.max_excess = y.max_excess;
    x.excess_index = y.excess_index;
  }
  x.max_abs = fmaxf(x.max_abs, y.max_abs);
  x.amax_a = fmaxf(x.amax_a, y.amax_a);
  x.amax_b = fmaxf(x.amax_b, y.amax_b);
  x.over += y.over;
  x.viol += y.viol;
  x.mism += y.mism;
  x.nan_ex += y.nan_ex;
  if (y.first_viol >= 0 && (x.first_viol < 0 || y.first_viol < x.first_viol)) x.first_viol = y.first_viol;
  if (y.first_mism >= 0 && (x.first_mism < 0 || y.first_mism < x.first_mism)) x.first_mism = y.first_mism;
  x.dab += y.dab;
  x.daa += y.daa;
  x.dbb += y.dbb;
}

__device__ __forceinline__ void init(DiffPartial& x) {
  x.max_excess = 0.f;
  x.max_abs = 0.f;
  x.amax_a = 0.f;
  x.amax_b = 0.f;
  x.excess_index = -1;
  x.over = x.viol = x.mism = x.nan_ex = 0;
  x.first_viol = x.first_mism = -1;
  x.dab = x.daa = x.dbb = 0.0;
}

template <typename T> __device__ __forceinline__ float fval(T v);
template <> __device__ __forceinline__ float fval<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float fval<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float fval<float>(float v) { return v; }

template <typename T> struct Bits;
template <> struct Bits<__nv_bfloat16> { using U = uint16_t; };
template <> struct Bits<__half> { using U = uint16_t; };
template <> struct Bits<float> { using U = uint32_t; };

// float element: full policy
template <typename T>
__device__ __forceinline__ void visit_float(const T av, const T bv, int64_t i, float rtol, float atol, float wobble,
                                            DiffPartial& p) {
  using U = typename Bits<T>::U;
  if (*reinterpret_cast<const U*>(&av) != *reinterpret_cast<const U*>(&bv)) {
    ++p.mism;
    if (p.first_mism < 0) p.first_mism = i;
  }
  const float c = fval<T>(av), r = fval<T>(bv);
  const bool cf = isfinite(c), rf = isfinite(r);
  const bool ok = (rf && cf) || (isnan(r) && isnan(c)) || (isinf(r) && c == r);
  if (!ok) {
    ++p.viol;
    if (p.first_viol < 0) p.first_viol = i;
  }
  float excess = 0.f;
  if (rf && ok) {
    const float allowed = fmaxf(__fadd_rn(atol, __fmul_rn(rtol, fabsf(r))), wobble);
    const float ad = fabsf(__fsub_rn(c, r));
    excess = __fsub_rn(ad, allowed);
    if (isnan(excess)) {
      const float scale = fmaxf(fmaxf(fabsf(c), fabsf(r)), 1.0f);
      const float cs = __fdiv_rn(c, scale), rs = __fdiv_rn(r, scale);
      const float se = __fsub_rn(fabsf(__fsub_rn(cs, rs)),
                                 __fadd_rn(__fdiv_rn(atol, scale), __fmul_rn(rtol, fabsf(rs))));
      excess = __fmul_rn(se, scale);
    }
    p.max_abs = fmaxf(p.max_abs, ad);
  }
  if (isnan(excess)) {
    ++p.nan_ex;
  } else {
    if (excess > 0.f) ++p.over;
    if (p.excess_index < 0 || excess > p.max_excess) {
      p.max_excess = excess;
      p.excess_index = i;
    }
  }
  const float a0 = cf ? c : 0.f, b0 = rf ? r : 0.f;
  p.amax_a = fmaxf(p.amax_a, fabsf(a0));
  p.amax_b = fmaxf(p.amax_b, fabsf(b0));
  p.dab += static_cast<double>(a0) * static_cast<double>(b0);
  p.daa += static_cast<double>(a0) * static_cast<double>(a0);
  p.dbb += static_cast<double>(b0) * static_cast<double>(b0);
}

// Eight 16-bit elements (one 16-byte vector of each input) at indices
// i0 .. i0+7. When no element of either vector is Inf or NaN (the exponent
// test runs on packed pairs) the policy reduces to its finite branch:
// excess = |a - b| - max(atol + rtol |b|, wobble) per element, and the
// vector's bit mismatches are counted on packed pairs. The maximum excess
// keeps the first index of its value (elements visited in order, a strict
// comparison), as the element-by-element visit does. The cosine sums take
// the vector's three fp32 sums of exact products and add them in fp64 (fp64
// products when a magnitude in the vector is above 2^62 or below 2^-60). A
// vector holding a non-finite value takes the full per-element policy; an
// element whose excess is NaN (|b| and |a - b| both overflowing) gets the
// policy's scaled form, as in the full visit.
template <typename T>
__device__ __forceinline__ void visit_vec16(const uint4 va, const uint4 vb, int64_t i0, float rtol, float atol,
                                            float wobble, DiffPartial& p) {
  // a half's exponent field is all ones (Inf or NaN) exactly when adding its
  // lowest exponent bit carries into the half's sign position; the masked
  // fields cannot carry across halves
  constexpr bool kBf = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kExp = kBf ? 0x7F807F80u : 0x7C007C00u;
  constexpr uint32_t kLsb = kBf ? 0x00800080u : 0x04000400u;
  const uint32_t wa[4] = {va.x, va.y, va.z, va.w};
  const uint32_t wb[4] = {vb.x, vb.y, vb.z, vb.w};
  uint32_t special = 0, diff = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    special |= ((wa[k] & kExp) + kLsb) | ((wb[k] & kExp) + kLsb);
    diff |= wa[k] ^ wb[k];
  }
  special &= 0x80008000u;
  const T* ea = reinterpret_cast<const T*>(wa);
  const T* eb = reinterpret_cast<const T*>(wb);
  if (special) {
#pragma unroll
    for (int e = 0; e < 8; ++e) visit_float<T>(ea[e], eb[e], i0 + e, rtol, atol, wobble, p);
    return;
  }
  if (diff) {
#pragma unroll
    for (int k = 0; k < 4; ++k) p.mism += __popc(__vcmpne2(wa[k], wb[k])) >> 4;
    if (p.first_mism < 0) {
      for (int e = 0; e < 8; ++e) {
        const uint32_t x = (wa[e >> 1] ^ wb[e >> 1]) >> ((e & 1) * 16);
        if (x & 0xFFFFu) {
          p.first_mism = i0 + e;
          break;
        }
      }
    }
  }
  float best = 0.f;
  int best_e = -1;
  float sab = 0.f, saa = 0.f, sbb = 0.f, vmax = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float c = fval<T>(ea[e]), r = fval<T>(eb[e]);
    vmax = fmaxf(vmax, fmaxf(fabsf(c), fabsf(r)));
    const float allowed = fmaxf(__fadd_rn(atol, __fmul_rn(rtol, fabsf(r))), wobble);
    const float ad = fabsf(__fsub_rn(c, r));
    float excess = __fsub_rn(ad, allowed);
    if (excess != excess) {
      // |b| and |a - b| overflowed together: the policy's scaled form
      const float scale = fmaxf(fmaxf(fabsf(c), fabsf(r)), 1.0f);
      const float cs = __fdiv_rn(c, scale), rs = __fdiv_rn(r, scale);
      const float se = __fsub_rn(fabsf(__fsub_rn(cs, rs)),
                                 __fadd_rn(__fdiv_rn(atol, scale), __fmul_rn(rtol, fabsf(rs))));
      excess = __fmul_rn(se, scale);
    }
    p.max_abs = fmaxf(p.max_abs, ad);
    if (excess != excess) {
      ++p.nan_ex;
    } else {
      if (excess > 0.f) ++p.over;
      if (best_e < 0 || excess > best) {
        best = excess;
        best_e = e;
      }
    }
    p.amax_a = fmaxf(p.amax_a, fabsf(c));
    p.amax_b = fmaxf(p.amax_b, fabsf(r));
    sab = fmaf(c, r, sab);
    saa = fmaf(c, c, saa);
    sbb = fmaf(r, r, sbb);
  }
  if (best_e >= 0 && (p.excess_index < 0 || best > p.max_excess)) {
    p.max_excess = best;
    p.excess_index = i0 + best_e;
  }
  if (vmax <= 0x1p62f && vmax >= 0x1p-60f) {
    // products and 8-term sums stay well inside fp32's range
    p.dab += static_cast<double>(sab);
    p.daa += static_cast<double>(saa);
    p.dbb += static_cast<double>(sbb);
  } else if (vmax != 0.f) {
    // magnitudes whose fp32 products could overflow or vanish: fp64 products
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const double c = fval<T>(ea[e]), r = fval<T>(eb[e]);
      p.dab += c * r;
      p.daa += c * c;
      p.dbb += r * r;
    }
  }
}

template <typename U>
__device__ __forceinline__ void visit_bits(const U av, const U bv, int64_t i, DiffPartial& p) {
  if (av != bv) {
    ++p.mism;
    if (p.first_mism < 0) p.first_mism = i;
  }
}

constexpr int kDiffThreads = 256;

static inline int diff_blocks(int64_t n) {
  const int64_t b = (n + 8191) / 8192;
  return static_cast<int>(b < 1 ? 1 : (b > 1184 ? 1184 : b));  // at most 8 blocks per SM of 148
}

template <typename T, bool FLOAT>
__global__ void __launch_bounds__(kDiffThreads, 3) diff_kernel(const T* __restrict__ a, const T* __restrict__ b, int64_t n,
                                                            float rtol, float atol, float wobble,
                                                            DiffPartial* __restrict__ parts, uint32_t* counter,
                                                            mt_diff_stats* __restrict__ out) {
  __shared__ DiffPartial sp[kDiffThreads / 32];
  __shared__ int am_last;
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  DiffPartial p;
  init(p);
  // contiguous slice per block (a multiple of one 16-byte vector), strided by
  // thread inside it: every index is visited once and each thread's indices
  // increase (first-index tracking)
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte vector
  int64_t per = (n + gridDim.x - 1) / gridDim.x;
  per = (per + V - 1) / V * V;
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * per;
  const int64_t hi = lo + per < n ? lo + per : n;
  const bool vec = FLOAT && ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) == 0;
  if (vec) {
    // one 16-byte vector of each input per step, the next step's vectors
    // loaded before this one is visited (two steps of loads in flight)
    const int64_t step = static_cast<int64_t>(kDiffThreads) * V;
    int64_t i = lo + static_cast<int64_t>(threadIdx.x) * V;
    uint4 va = make_uint4(0, 0, 0, 0), vb = make_uint4(0, 0, 0, 0);
    if (i + V <= hi) {
      va = *reinterpret_cast<const uint4*>(a + i);
      vb = *reinterpret_cast<const uint4*>(b + i);
    }
    while (i < hi) {
      const int64_t nx = i + step;
      uint4 na = make_uint4(0, 0, 0, 0), nb = make_uint4(0, 0, 0, 0);
      if (nx + V <= hi) {
        na = *reinterpret_cast<const uint4*>(a + nx);
        nb = *reinterpret_cast<const uint4*>(b + nx);
      }
      if (i + V <= hi) {
        if constexpr (FLOAT && sizeof(T) == 2) {
          visit_vec16<T>(va, vb, i, rtol, atol, wobble, p);
        } else {
          const T* ea = reinterpret_cast<const T*>(&va);
          const T* eb = reinterpret_cast<const T*>(&vb);
#pragma unroll
          for (int e = 0; e < V; ++e) {
            if constexpr (FLOAT) visit_float<T>(ea[e], eb[e], i + e, rtol, atol, wobble, p);
          }
        }
      } else {
        for (int64_t j = i; j < hi; ++j) {
          if constexpr (FLOAT) visit_float<T>(a[j], b[j], j, rtol, atol, wobble, p);
        }
      }
      va = na;
      vb = nb;
      i = nx;
    }
  } else {
    for (int64_t i = lo + threadIdx.x; i < hi; i += kDiffThreads) {
      if constexpr (FLOAT) visit_float<T>(a[i], b[i], i, rtol, atol, wobble, p);
      else visit_bits<T>(a[i], b[i], i, p);
    }
  }
  // warp then block merge, fixed order; the block's result is valid in thread 0
  auto block_merge = [&](DiffPartial v) {
    for (int o = 1; o < 32; o <<= 1) {
      DiffPartial q;
      q.max_excess = __shfl_down_sync(0xffffffffu, v.max_excess, o);
      q.max_abs = __shfl_down_sync(0xffffffffu, v.max_abs, o);
      q.amax_a = __shfl_down_sync(0xffffffffu, v.amax_a, o);
      q.amax_b = __shfl_down_sync(0xffffffffu, v.amax_b, o);
      q.excess_index = __shfl_down_sync(0xffffffffu, v.excess_index, o);
      q.over = __shfl_down_sync(0xffffffffu, v.over, o);
      q.viol = __shfl_down_sync(0xffffffffu, v.viol, o);
      q.first_viol = __shfl_down_sync(0xffffffffu, v.first_viol, o);
      q.mism = __shfl_down_sync(0xffffffffu, v.mism, o);
      q.first_mism = __shfl_down_sync(0xffffffffu, v.first_mism, o);
      q.nan_ex = __shfl_down_sync(0xffffffffu, v.nan_ex, o);
      q.dab = __shfl_down_sync(0xffffffffu, v.dab, o);
      q.daa = __shfl_down_sync(0xffffffffu, v.daa, o);
      q.dbb = __shfl_down_sync(0xffffffffu, v.dbb, o);
      if ((threadIdx.x & 31) + o < 32) merge(v, q);
    }
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) sp[warp] = v;
    __syncthreads();
    DiffPartial acc = sp[0];
    if (threadIdx.x == 0)
      for (int w = 1; w < kDiffThreads / 32; ++w) merge(acc, sp[w]);
    __syncthreads();  // sp is reused by a second merge
    return acc;
  };
  const DiffPartial mine = block_merge(p);
  if (threadIdx.x == 0) {
    parts[blockIdx.x] = mine;
    __threadfence();
    const uint32_t prev = atomicAdd(counter, 1u);
    am_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (am_last) {
    // the last block folds every block's partial: thread t takes blocks t,
    // t + 256, ... in order, then the same fixed-order merge (partials read
    // from L2: they were written by other SMs)
    __threadfence();
    DiffPartial v;
    init(v);
    for (unsigned blk = threadIdx.x; blk < gridDim.x; blk += kDiffThreads) {
      const DiffPartial* src = parts + blk;
      DiffPartial q;
      q.max_excess = __ldcg(&src->max_excess);
      q.max_abs = __ldcg(&src->max_abs);
      q.amax_a = __ldcg(&src->amax_a);
      q.amax_b = __ldcg(&src->amax_b);
      q.excess_index = __ldcg(reinterpret_cast<const long long*>(&src->excess_index));
      q.over = __ldcg(reinterpret_cast<const long long*>(&src->over));
      q.viol = __ldcg(reinterpret_cast<const long long*>(&src->viol));
      q.first_viol = __ldcg(reinterpret_cast<const long long*>(&src->first_viol));
      q.mism = __ldcg(reinterpret_cast<const long long*>(&src->mism));
      q.first_mism = __ldcg(reinterpret_cast<const long long*>(&src->first_mism));
      q.nan_ex = __ldcg(reinterpret_cast<const long long*>(&src->nan_ex));
      q.dab = __ldcg(&src->dab);
      q.daa = __ldcg(&src->daa);
      q.dbb = __ldcg(&src->dbb);
      merge(v, q);
    }
    const DiffPartial acc = block_merge(v);
    if (threadIdx.x != 0) return;
    out->max_excess = acc.max_excess;
    out->max_abs = acc.max_abs;
    out->dot_ab = acc.dab;
    out->dot_aa = acc.daa;
    out->dot_bb = acc.dbb;
    out->amax_a = acc.amax_a;
    out->amax_b = acc.amax_b;
    out->excess_index = acc.excess_index;
    out->over_count = acc.over;
    out->nonfinite_violations = acc.viol;
    out->first_violation = acc.first_viol;
    out->bit_mismatches = acc.mism;
    out->first_mismatch = acc.first_mism;
    out->nan_excess = acc.nan_ex;
    *counter = 0;  // ready for the next call
  }
}

// counter in the workspace's control region, block partials after it
size_t diff_workspace(int64_t n) { return kWsCtlBytes + static_cast<size_t>(diff_blocks(n)) * sizeof(DiffPartial); }

// Scratch of mt_diff_reduce_noalloc: the completion counter (first 256 bytes)
// and one partial per block. Every GPU that loads the library holds this
// array until the process exits; every call of the entry point on a device
// shares it.
constexpr int kNoAllocBlocks = 128;
constexpr int64_t kNoAllocMaxN = static_cast<int64_t>(kNoAllocBlocks) * 8192;  // MT_DIFF_NOALLOC_MAX_ELEMS
static __device__ __align__(256) uint8_t g_diff_noalloc_scratch[256 + kNoAllocBlocks * sizeof(DiffPartial)];

// Device address of the scratch array in the current context. Host code may
// not pass the array's name to a kernel (it is only a host-side stand-in), so
// the address is looked up on every call, with the calling device current.
// No cache: the lookup is cheap, shares no state between host threads and
// stays right after a cudaDeviceReset or a primary-context reset gives the
// array a new address.
static int noalloc_scratch(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_diff_noalloc_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_diff_noalloc_scratch)");
  *out = p;
  return MT_OK;
}

}  // namespace mt

using namespace mt;

extern "C" {

size_t mt_diff_workspace_bytes(int64_t n) { return diff_workspace(n); }

int mt_diff_reduce(const void* a, const void* b, int64_t n, int dtype, float rtol, float atol, float wobble,
                   mt_diff_stats* stats, void* workspace, size_t workspace_bytes, mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(stats, "mt_diff_reduce: stats is NULL");
  MT_CHECK_ARG(n >= 0, "mt_diff_reduce: negative size");
  MT_CHECK_ARG(n == 0 || (a && b), "mt_diff_reduce: null input");
  if (!workspace || workspace_bytes < diff_workspace(n) || !aligned(workspace, 256)) {
    set_error("mt_diff_reduce: workspace of %zu bytes (256-aligned, zero-filled) required, got %zu",
              diff_workspace(n), workspace_bytes);
    return MT_ERR_WORKSPACE;
  }
  uint32_t* counter = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + kWsDiffCounter);
  DiffPartial* parts = reinterpret_cast<DiffPartial*>(static_cast<uint8_t*>(workspace) + kWsCtlBytes);
  const dim3 grid(diff_blocks(n)), block(kDiffThreads);
  cudaStream_t s = (cudaStream_t)stream;
  switch (dtype) {
    case MT_BF16:
      return launch(diff_kernel<__nv_bfloat16, true>, grid, block, 0, s, (const __nv_bfloat16*)a,
                    (const __nv_bfloat16*)b, n, rtol, atol, wobble, parts, counter, stats);
    case MT_F16:
      return launch(diff_kernel<__half, true>, grid, block, 0, s, (const __half*)a, (const __half*)b, n, rtol, atol,
                    wobble, parts, counter, stats);
    case MT_F32:
      return launch(diff_kernel<float, true>, grid, block, 0, s, (const float*)a, (const float*)b, n, rtol, atol,
                    wobble, parts, counter, stats);
    case MT_I32:
    case MT_U32:
      return launch(diff_kernel<uint32_t, false>, grid, block, 0, s, (const uint32_t*)a, (const uint32_t*)b, n, rtol,
                    atol, wobble, parts, counter, stats);
    case MT_I64:
    case MT_U64:
      return launch(diff_kernel<unsigned long long, false>, grid, block, 0, s, (const unsigned long long*)a,
                    (const unsigned long long*)b, n, rtol, atol, wobble, parts, counter, stats);
    case MT_I16:
    case MT_U16:
      return launch(diff_kernel<uint16_t, false>, grid, block, 0, s, (const uint16_t*)a, (const uint16_t*)b, n, rtol,
                    atol, wobble, parts, counter, stats);
    case MT_U8:
    case MT_I8:
    case MT_BOOL:
      return launch(diff_kernel<uint8_t, false>, grid, block, 0, s, (const uint8_t*)a, (const uint8_t*)b, n, rtol,
                    atol, wobble, parts, counter, stats);
    default: set_error("mt_diff_reduce: unsupported dtype %d", dtype); return MT_ERR_UNSUPPORTED;
  }
}

// Same statistics as mt_diff_reduce, with its scratch in the library's own
// static device array instead of a caller workspace. For callers that must
// not allocate device memory. Same kernel and the same block partition as
// mt_diff_reduce, so both return identical statistics for the same input.
int mt_diff_reduce_noalloc(const void* a, const void* b, int64_t n, int dtype, float rtol, float atol, float wobble,
                           mt_diff_stats* stats, mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(stats, "mt_diff_reduce_noalloc: stats is NULL");
  MT_CHECK_ARG(n >= 0, "mt_diff_reduce_noalloc: negative size");
  MT_CHECK_ARG(n == 0 || (a && b), "mt_diff_reduce_noalloc: null input");
  MT_CHECK_ARG(n <= kNoAllocMaxN,
               "mt_diff_reduce_noalloc: n=%lld exceeds the static scratch maximum of %lld elements "
               "(%d block partials); use mt_diff_reduce with a workspace",
               (long long)n, (long long)kNoAllocMaxN, kNoAllocBlocks);
  if (diff_blocks(n) > kNoAllocBlocks) {
    set_error("mt_diff_reduce_noalloc: %d blocks exceed the static scratch", diff_blocks(n));
    return MT_ERR_INVALID_ARGUMENT;
  }
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc != MT_OK) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  // The array keeps the previous call's contents; the counter must start at zero.
  MT_CUDA(cudaMemsetAsync(scratch, 0, sizeof(uint32_t), s));
  uint32_t* counter = static_cast<uint32_t*>(scratch);
  DiffPartial* parts = reinterpret_cast<DiffPartial*>(static_cast<uint8_t*>(scratch) + 256);
  const dim3 grid(diff_blocks(n)), block(kDiffThreads);
  switch (dtype) {
    case MT_BF16:
      return launch(diff_kernel<__nv_bfloat16, true>, grid, block, 0, s, (const __nv_bfloat16*)a,
                    (const __nv_bfloat16*)b, n, rtol, atol, wobble, parts, counter, stats);
    case MT_F16:
      return launch(diff_kernel<__half, true>, grid, block, 0, s, (const __half*)a, (const __half*)b, n, rtol, atol,
                    wobble, parts, counter, stats);
    case MT_F32:
      return launch(diff_kernel<float, true>, grid, block, 0, s, (const float*)a, (const float*)b, n, rtol, atol,
                    wobble, parts, counter, stats);
    case MT_I32:
    case MT_U32:
      return launch(diff_kernel<uint32_t, false>, grid, block, 0, s, (const uint32_t*)a, (const uint32_t*)b, n, rtol,
                    atol, wobble, parts, counter, stats);
    case MT_I64:
    case MT_U64:
      return launch(diff_kernel<unsigned long long, false>, grid, block, 0, s, (const unsigned long long*)a,
                    (const unsigned long long*)b, n, rtol, atol, wobble, parts, counter, stats);
    case MT_I16:
    case MT_U16:
      return launch(diff_kernel<uint16_t, false>, grid, block, 0, s, (const uint16_t*)a, (const uint16_t*)b, n, rtol,
                    atol, wobble, parts, counter, stats);
    case MT_U8:
    case MT_I8:
    case MT_BOOL:
      return launch(diff_kernel<uint8_t, false>, grid, block, 0, s, (const uint8_t*)a, (const uint8_t*)b, n, rtol,
                    atol, wobble, parts, counter, stats);
    default: set_error("mt_diff_reduce_noalloc: unsupported dtype %d", dtype); return MT_ERR_UNSUPPORTED;
  }
}

}  // extern "C"
