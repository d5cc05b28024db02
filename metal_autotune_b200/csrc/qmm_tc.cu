// Affine-quantized matmul for prefill on the 5th-generation tensor cores.
//
// y[M, N] = x[M, K] · dequant(w)[N, K]^T. One CTA owns a tile of 128 weight
// rows (the MMA's M) and TN tokens (the MMA's N), and walks K in stages of
// 128. Roles:
//   warp 0      TMA producer: the packed weight tile (128 rows x 64 B for
//               4-bit, swizzled) and the x tile (TN rows x 128 bf16, 128-byte
//               swizzle) of each stage, into a ring of SS shared-memory slots.
//   warp 1      TMEM owner and MMA issuer: tcgen05.mma.kind::f16 with the
//               dequantised weights as the A operand read from tensor memory
//               and x as the B operand read from shared memory; fp32
//               accumulators in tensor memory.
//   warps 4-11  dequantisers: thread (warp%4, lane) owns weight row
//               32*(warp%4)+lane, turns its packed words into bf16 pairs
//               (MLX rounding, see dequant_chunk) and stores them straight
//               into tensor memory with tcgen05.st — dequantised weights never
//               touch shared memory. After the K loop the same warps run the
//               epilogue (tcgen05.ld of the accumulators, rounding, residual
//               or SwiGLU, store).
// Small-M shapes give few tiles, so K may be split over blockIdx.z; each
// split writes an fp32 partial to the workspace and the last split of a tile
// to arrive (atomic counter) sums the partials in split order — the result
// does not depend on arrival order — applies the epilogue and re-zeroes the
// counter.
//
// Every mbarrier wait is bounded (mbar_wait); on expiry the CTA records the
// site in the device status word, stops issuing work, waits (bounded) for
// its in-flight copies and MMAs and frees its tensor memory.
#include <algorithm>

#include "mt_common.cuh"
#include "mt_tma.h"
#include "qmm_common.cuh"

namespace mt {

constexpr int kBM = 128;      // weight rows per tile (MMA M)
constexpr int kBK = 128;      // K per stage
constexpr int kThreads = 384; // 12 warps
constexpr int kMaxSS = 8;
constexpr int kTmemCols = 512;
constexpr int kAccCols = 256; // accumulators occupy columns [0, 256)

struct QmmTcParams {
  CUtensorMap tmx;     // x [M, K]
  CUtensorMap tmw[3];  // packed weights of each set [N_s, K*bits/32]
  const void* s[3];
  const void* b[3];
  void* y[3];
  const void* residual;
  uint32_t* counters;
  float* partials;
  int N[3];
  int tile_start[4];   // prefix sums of feature tiles per set
  int M, K, G, group;
  int TN, TNp, SS, splits, nk, kind;
};

template <int BITS>
struct WLayout {
  static constexpr int kRowBytes = kBK * BITS / 8;  // packed bytes per row per stage
  static constexpr int kChunks = kRowBytes / 16;    // 16-byte chunks per row
  static constexpr int kValuesPerChunk = 128 / BITS;
  // physical 16-byte chunk of logical chunk c in row r under the TMA swizzle
  static __device__ __forceinline__ int phys(int r, int c) {
    return BITS == 4 ? (c ^ ((r >> 1) & 3)) : (c ^ (r & 7));
  }
};

template <int DT, int BITS, int DUAL>
__global__ void __launch_bounds__(kThreads, 1) qmm_tc_kernel(const __grid_constant__ QmmTcParams p) {
  using T = typename Elem<DT>::T;
  using WL = WLayout<BITS>;
  constexpr int NACC = DUAL ? 2 : 1;
  constexpr int TS = DUAL ? 2 : 4;  // tensor-memory A stages
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int TN = p.TN, SS = p.SS;
  const int x_stage_bytes = TN * 256;                 // 2 boxes of TN rows x 128 B
  const int w_set_bytes = kBM * WL::kRowBytes;
  const int w_stage_bytes = NACC * w_set_bytes;
  uint8_t* xs = smem;
  uint8_t* ws_ = smem + SS * x_stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ws_ + SS * w_stage_bytes);
  uint64_t* w_full = bars;
  uint64_t* x_full = bars + kMaxSS;
  uint64_t* s_empty = bars + 2 * kMaxSS;
  uint64_t* a_full = bars + 3 * kMaxSS;
  uint64_t* a_empty = a_full + 4;
  uint64_t* acc_full = a_empty + 4;
  uint64_t* drain = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- tile coordinates
  const int ft = blockIdx.x;
  int set = 0;
  if (!DUAL) {
    if (ft >= p.tile_start[1]) set = 1;
    if (ft >= p.tile_start[2]) set = 2;
  }
  const int n0 = (ft - p.tile_start[set]) * kBM;
  const int tok0 = blockIdx.y * TN;
  const int split = blockIdx.z;
  const int k_begin = static_cast<int>((static_cast<int64_t>(split) * p.nk) / p.splits);
  const int k_end = static_cast<int>((static_cast<int64_t>(split + 1) * p.nk) / p.splits);
  const int nkl = k_end - k_begin;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kMaxSS; ++i) {
      mbar_init(&w_full[i], 1);
      mbar_init(&x_full[i], 1);
      mbar_init(&s_empty[i], 1 + 8);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&a_full[i], 8);
      mbar_init(&a_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tmx);
    for (int a = 0; a < NACC; ++a) prefetch_tmap(&p.tmw[DUAL ? a : set]);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Dependents only start their own set-up before griddep_wait(); letting
  // them launch now overlaps their launch latency with this kernel.
  griddep_launch();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const int kw_per_stage = kBK * BITS / 32;  // words of K per stage
      const int pre = nkl < SS ? nkl : SS;
      auto issue_w = [&](int i) {
        const int s = i % SS;
        const int kstage = k_begin + i;
        mbar_arrive_expect_tx(&w_full[s], w_stage_bytes);
        for (int a = 0; a < NACC; ++a)
          tma_load_2d(ws_ + s * w_stage_bytes + a * w_set_bytes, &p.tmw[DUAL ? a : set], &w_full[s],
                      kstage * kw_per_stage, n0);
      };
      auto issue_x = [&](int i) {
        const int s = i % SS;
        const int kstage = k_begin + i;
        mbar_arrive_expect_tx(&x_full[s], x_stage_bytes);
        for (int j = 0; j < 2; ++j)
          tma_load_2d(xs + s * x_stage_bytes + j * TN * 128, &p.tmx, &x_full[s],
                      kstage * kBK + 64 * j, tok0);
      };
      // Weights do not depend on the previous kernel: start them before the
      // grid dependency resolves.
      int issued_w = 0, issued_x = 0;
      for (int i = 0; i < pre; ++i, ++issued_w) issue_w(i);
      griddep_wait();
      for (int i = 0; i < pre; ++i, ++issued_x) issue_x(i);
      for (int i = pre; i < nkl; ++i) {
        const int s = i % SS;
        if (!mbar_wait(&s_empty[s], ((i / SS) & 1) ^ 1, abort_flag, 0x101)) break;
        issue_w(i);
        ++issued_w;
        issue_x(i);
        ++issued_x;
      }
      if (*abort_flag) {
        // let every copy this thread issued land before shared memory is released
        for (int i = (issued_w > SS ? issued_w - SS : 0); i < issued_w; ++i)
          mbar_wait_drain(&w_full[i % SS], (i / SS) & 1, 200000000ull);
        for (int i = (issued_x > SS ? issued_x - SS : 0); i < issued_x; ++i)
          mbar_wait_drain(&x_full[i % SS], (i / SS) & 1, 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kBM, TN, DT == MT_BF16);
      bool issued = false;
      for (int i = 0; i < nkl; ++i) {
        const int s = i % SS, t = i % TS;
        if (!mbar_wait(&x_full[s], (i / SS) & 1, abort_flag, 0x201)) break;
        if (!mbar_wait(&a_full[t], (i / TS) & 1, abort_flag, 0x202)) break;
        tc_fence_after();
        const uint32_t xbase = smem_addr(xs + s * x_stage_bytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t bdesc = smem_desc_k_sw128(xbase + (kk >> 2) * TN * 128 + (kk & 3) * 32);
#pragma unroll
          for (int a = 0; a < NACC; ++a) {
            const uint32_t a_tmem = tmem + kAccCols + (t * NACC + a) * 64 + kk * 8;
            const uint32_t d_tmem = tmem + a * TN;
            tc_mma_ts(d_tmem, a_tmem, bdesc, idesc, (i > 0 || kk > 0) ? 1u : 0u);
          }
        }
        issued = true;
        tc_commit(&s_empty[s]);
        tc_commit(&a_empty[t]);
      }
      if (issued) tc_commit(acc_full);
      if (*abort_flag && issued) {
        // MMAs still read tensor and shared memory: wait for them before teardown
        tc_commit(drain);
        mbar_wait_drain(drain, 0, 200000000ull);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ dequantisers
    const int q = warp & 3;
    const int wg = (warp - 4) >> 2;
    const int r = q * 32 + lane;                 // weight row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    // single: WG wg converts chunks [wg*C/2, (wg+1)*C/2) of set `set`
    // dual:   WG wg converts all chunks of set wg (0 gate, 1 up)
    constexpr int kMyChunks = DUAL ? WL::kChunks : WL::kChunks / 2;
    const int aset = DUAL ? wg : 0;
    const int wset = DUAL ? wg : set;
    const int c0 = DUAL ? 0 : wg * kMyChunks;
    const int n = n0 + r;
    const bool row_ok = n < p.N[wset];
    const T* srow = static_cast<const T*>(p.s[wset]) + static_cast<int64_t>(row_ok ? n : 0) * p.G;
    const T* brow = static_cast<const T*>(p.b[wset]) + static_cast<int64_t>(row_ok ? n : 0) * p.G;
    bool ok = true;
    for (int i = 0; i < nkl && ok; ++i) {
      const int s = i % SS, t = i % TS;
      const int kst = (k_begin + i) * kBK;
      float sc[kMyChunks], bi[kMyChunks];
#pragma unroll
      for (int c = 0; c < kMyChunks; ++c) {
        const int g = (kst + (c0 + c) * WL::kValuesPerChunk) / p.group;
        const bool gok = row_ok && g < p.G;
        sc[c] = gok ? Elem<DT>::to_f(srow[g]) : 0.f;
        bi[c] = gok ? Elem<DT>::to_f(brow[g]) : 0.f;
      }
      if (!mbar_wait(&w_full[s], (i / SS) & 1, abort_flag, 0x301)) { ok = false; break; }
      uint4 wv[kMyChunks];
      const uint8_t* wrow = ws_ + s * w_stage_bytes + aset * w_set_bytes + r * WL::kRowBytes;
#pragma unroll
      for (int c = 0; c < kMyChunks; ++c)
        wv[c] = *reinterpret_cast<const uint4*>(wrow + WL::phys(r, c0 + c) * 16);
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[s]);
      if (!mbar_wait(&a_empty[t], ((i / TS) & 1) ^ 1, abort_flag, 0x302)) { ok = false; break; }
      constexpr int kPairsPerChunk = WL::kValuesPerChunk / 2;
      constexpr int kCols = kMyChunks * kPairsPerChunk;  // 32 (single) or 64 (dual)
      const uint32_t col0 = kAccCols + (t * NACC + aset) * 64 + (DUAL ? 0 : wg * 32);
#pragma unroll
      for (int h = 0; h < kCols / 32; ++h) {
        uint32_t out[32];
        constexpr int kChunksPer32 = 32 / kPairsPerChunk;
#pragma unroll
        for (int c = 0; c < kChunksPer32; ++c)
          dequant_chunk<DT, BITS>(wv[h * kChunksPer32 + c], sc[h * kChunksPer32 + c],
                                  bi[h * kChunksPer32 + c], out + c * kPairsPerChunk);
        tmem_st32(tmem + lane_base + col0 + h * 32, out);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[t]);
    }

    // ------------------------------------------------------------ epilogue
    // Every dequantiser thread reaches this barrier (all waits above are
    // bounded); the decision to run the epilogue is then uniform, so the
    // named barriers inside it cannot be left waiting.
    const bool accd = ok && nkl > 0 && mbar_wait(acc_full, 0, abort_flag, 0x401);
    if (!accd) *last_flag = 2;
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const bool run_epilogue = (*last_flag != 2);
    asm volatile("bar.sync 1, 256;" ::: "memory");
    if (run_epilogue) {
      tc_fence_after();
      griddep_wait();
      const int nchunks = (TN + 31) / 32;
      const int tile_id = ft * gridDim.y + blockIdx.y;
      bool finish = true;
      if (p.splits > 1) {
        // write this split's partial, [acc][row][TNp] per (tile, split)
        for (int ci = wg; ci < nchunks; ci += 2) {
#pragma unroll
          for (int a = 0; a < NACC; ++a) {
            uint32_t v[32];
            tmem_ld32(tmem + lane_base + a * TN + ci * 32, v);
            tmem_wait_ld();
            float* dst = p.partials +
                         ((static_cast<int64_t>(tile_id) * p.splits + split) * NACC + a) * kBM * p.TNp +
                         static_cast<int64_t>(r) * p.TNp + ci * 32;
#pragma unroll
            for (int e = 0; e < 32; e += 4)
              __stcg(reinterpret_cast<float4*>(dst + e),
                     make_float4(__uint_as_float(v[e]), __uint_as_float(v[e + 1]),
                                 __uint_as_float(v[e + 2]), __uint_as_float(v[e + 3])));
          }
        }
        __threadfence();
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (threadIdx.x == 128) {
          const uint32_t prev = atomicAdd(&p.counters[tile_id], 1u);
          const int last = (prev == static_cast<uint32_t>(p.splits - 1));
          if (last) p.counters[tile_id] = 0;  // ready for the next call
          *last_flag = last;
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
        finish = *last_flag != 0;
        if (finish) __threadfence();
      }
      if (finish) {
        T* y = static_cast<T*>(p.y[DUAL ? 0 : set]);
        const int N = p.N[DUAL ? 0 : set];
        const T* res = static_cast<const T*>(p.residual);
        for (int ci = wg; ci < nchunks; ci += 2) {
          float acc[NACC][32];
#pragma unroll
          for (int a = 0; a < NACC; ++a) {
            uint32_t v[32];
            tmem_ld32(tmem + lane_base + a * TN + ci * 32, v);
            tmem_wait_ld();
            if (p.splits > 1) {
#pragma unroll
              for (int e = 0; e < 32; ++e) acc[a][e] = 0.f;
              for (int sp = 0; sp < p.splits; ++sp) {
                if (sp == split) {
#pragma unroll
                  for (int e = 0; e < 32; ++e) acc[a][e] += __uint_as_float(v[e]);
                } else {
                  const float* src = p.partials +
                                     ((static_cast<int64_t>(tile_id) * p.splits + sp) * NACC + a) * kBM * p.TNp +
                                     static_cast<int64_t>(r) * p.TNp + ci * 32;
#pragma unroll
                  for (int e = 0; e < 32; e += 4) {
                    const float4 f = __ldcg(reinterpret_cast<const float4*>(src + e));
                    acc[a][e] += f.x;
                    acc[a][e + 1] += f.y;
                    acc[a][e + 2] += f.z;
                    acc[a][e + 3] += f.w;
                  }
                }
              }
            } else {
#pragma unroll
              for (int e = 0; e < 32; ++e) acc[a][e] = __uint_as_float(v[e]);
            }
          }
          if (n < N) {
            const int tcount = (TN - ci * 32) < 32 ? (TN - ci * 32) : 32;
#pragma unroll 4
            for (int e = 0; e < tcount; ++e) {
              const int tok = tok0 + ci * 32 + e;
              if (tok >= p.M) break;
              const int64_t off = static_cast<int64_t>(tok) * N + n;
              float v;
              if (DUAL) {
                v = swiglu_rounded<DT>(round_to<DT>(acc[0][e]), round_to<DT>(acc[NACC - 1][e]));
              } else {
                v = round_to<DT>(acc[0][e]);
                if (p.kind == QMM_RESIDUAL) v += Elem<DT>::to_f(res[off]);
              }
              y[off] = Elem<DT>::from_f(v);
            }
          }
        }
      }
    }
  }

  // ---- teardown: every thread arrives here, including after an abort
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------- host

static size_t smem_bytes_for(int TN, int SS, int bits, int dual) {
  const int nacc = dual ? 2 : 1;
  const size_t stage = static_cast<size_t>(TN) * 256 + static_cast<size_t>(nacc) * kBM * (kBK * bits / 8);
  return 1024 + SS * stage + 512;
}

static int pick_ss(int TN, int bits, int dual) {
  int ss = kMaxSS;
  while (ss > 2 && smem_bytes_for(TN, ss, bits, dual) > 220 * 1024) --ss;
  return ss;
}

static int tile_tn(int64_t M, int dual) {
  const int64_t cap = dual ? 128 : 256;
  int64_t tn = M < cap ? M : cap;
  tn = (tn + 15) / 16 * 16;
  return static_cast<int>(tn);
}

static size_t ws_need(int64_t tiles, int splits, int nacc, int TNp) {
  if (splits <= 1) return 0;
  const size_t counters = (static_cast<size_t>(tiles) * 4 + 255) / 256 * 256;
  return counters + static_cast<size_t>(tiles) * splits * nacc * kBM * TNp * 4;
}

static int choose_splits(int64_t tiles, int nk, int sms, size_t ws_bytes, int nacc, int TNp) {
  if (tiles >= sms) return 1;
  int best = 1;
  double best_cost = 1e30;
  const int max_s = std::min(nk, 16);
  for (int s = 1; s <= max_s; ++s) {
    if (ws_need(tiles, s, nacc, TNp) > ws_bytes) break;
    const int64_t waves = (tiles * s + sms - 1) / sms;
    const double per = static_cast<double>((nk + s - 1) / s);
    // the split reduction costs roughly a stage per extra partial
    const double cost = waves * per + (s > 1 ? 0.5 + 0.1 * s : 0.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

size_t qmm_tc_workspace(int64_t M, int64_t n_total, int64_t K, int bits, int kind) {
  (void)bits;
  const int dual = kind == 1;
  const int TN = tile_tn(M, dual);
  const int TNp = (TN + 31) / 32 * 32;
  const int64_t ttiles = (M + TN - 1) / TN;
  const int64_t ft = dual ? (n_total / 2 + kBM - 1) / kBM : (n_total + kBM - 1) / kBM + 2;
  const int nk = static_cast<int>((K + kBK - 1) / kBK);
  return ws_need(ft * ttiles, std::min(nk, 16), dual ? 2 : 1, TNp);
}

template <int DT, int BITS, int DUAL>
static int launch_tc(QmmTcParams& p, dim3 grid, size_t smem, cudaStream_t stream) {
  auto k = qmm_tc_kernel<DT, BITS, DUAL>;
  static bool configured[64] = {false};
  int dev = 0;
  MT_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    MT_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  return launch(k, grid, dim3(kThreads), smem, stream, p);
}

int qmm_tc_run(const QmmRequest& r, cudaStream_t stream) {
  const int dual = r.kind == QMM_SWIGLU ? 1 : 0;
  const int esz = 2;
  MT_CHECK_ARG(r.K % 64 == 0, "qmm: K=%lld must be a multiple of 64", (long long)r.K);
  MT_CHECK_ARG(aligned(r.x, 16), "qmm: x must be 16-byte aligned");
  int sms = 148;
  int rc = device_sm_count(&sms);
  if (rc != MT_OK) return rc;

  QmmTcParams p;
  memset(&p, 0, sizeof(p));
  p.M = static_cast<int>(r.M);
  p.K = static_cast<int>(r.K);
  p.group = r.group;
  p.G = static_cast<int>(r.K / r.group);
  p.kind = r.kind;
  p.residual = r.residual;
  p.TN = tile_tn(r.M, dual);
  p.TNp = (p.TN + 31) / 32 * 32;
  p.SS = pick_ss(p.TN, r.bits, dual);
  p.nk = static_cast<int>((r.K + kBK - 1) / kBK);

  const CUtensorMapDataType xdt =
      r.dtype == MT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  rc = make_tmap_2d(&p.tmx, r.x, xdt, esz, r.K, r.M, r.K * esz, 64, p.TN,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != MT_OK) return rc;
  const int words = static_cast<int>(r.K * r.bits / 32);
  const int nsets = dual ? 2 : 3;
  int tiles = 0;
  p.tile_start[0] = 0;
  for (int s = 0; s < 3; ++s) {
    const QmmSetReq& q = r.set[s];
    p.N[s] = static_cast<int>(q.N);
    if (s < nsets && q.N > 0) {
      MT_CHECK_ARG(aligned(q.w, 16), "qmm: packed weights must be 16-byte aligned");
      rc = make_tmap_2d(&p.tmw[s], q.w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, words, q.N,
                        static_cast<uint64_t>(words) * 4, kBK * r.bits / 32, kBM,
                        r.bits == 4 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc != MT_OK) return rc;
      p.s[s] = q.s;
      p.b[s] = q.b;
      p.y[s] = q.y;
      if (!dual) tiles += static_cast<int>((q.N + kBM - 1) / kBM);
    }
    p.tile_start[s + 1] = tiles;
  }
  if (dual) {
    tiles = static_cast<int>((r.set[0].N + kBM - 1) / kBM);
    p.N[1] = p.N[0];
  }
  const int ttiles = static_cast<int>((r.M + p.TN - 1) / p.TN);
  const int64_t tiles_total = static_cast<int64_t>(tiles) * ttiles;
  MT_CHECK_ARG(ttiles <= 65535, "qmm: M=%lld too large", (long long)r.M);
  p.splits = choose_splits(tiles_total, p.nk, sms, r.ws ? r.ws_bytes : 0, dual ? 2 : 1, p.TNp);
  if (p.splits > 1) {
    const size_t counters = (static_cast<size_t>(tiles_total) * 4 + 255) / 256 * 256;
    p.counters = static_cast<uint32_t*>(r.ws);
    p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(r.ws) + counters);
    MT_CHECK_ARG(aligned(r.ws, 256), "qmm: workspace must be 256-byte aligned");
  }
  const size_t smem = smem_bytes_for(p.TN, p.SS, r.bits, dual);
  const dim3 grid(tiles, ttiles, p.splits);
  const bool bf = r.dtype == MT_BF16;
  if (dual) {
    if (bf) return r.bits == 4 ? launch_tc<MT_BF16, 4, 1>(p, grid, smem, stream)
                               : launch_tc<MT_BF16, 8, 1>(p, grid, smem, stream);
    return r.bits == 4 ? launch_tc<MT_F16, 4, 1>(p, grid, smem, stream)
                       : launch_tc<MT_F16, 8, 1>(p, grid, smem, stream);
  }
  if (bf) return r.bits == 4 ? launch_tc<MT_BF16, 4, 0>(p, grid, smem, stream)
                             : launch_tc<MT_BF16, 8, 0>(p, grid, smem, stream);
  return r.bits == 4 ? launch_tc<MT_F16, 4, 0>(p, grid, smem, stream)
                     : launch_tc<MT_F16, 8, 0>(p, grid, smem, stream);
}

}  // namespace mt
