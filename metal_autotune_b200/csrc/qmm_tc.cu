// Affine-quantized matmul for prefill on the 5th-generation tensor cores.
//
// y[M, N] = x[M, K] · dequant(w)[N, K]^T, as a persistent stream-K kernel.
//
// Work: a tile is 128 weight rows (the MMA's M) x TN <= 128 tokens (the MMA's
// N); a unit is one tile's K-stage of 128. The grid has one CTA per SM; CTA c
// owns the contiguous unit range [c*U/P, (c+1)*U/P), so every SM gets the
// same number of K-stages whatever the tile count, and a CTA's pipeline runs
// across tile boundaries without draining.
//
// Roles (512 threads):
//   warps 0,2,3 TMA producers, one per stream: warp 0 the x tile (TN rows x
//               2 x 64 bf16, 128-byte swizzle, one 3-D copy), warp 2 (and 3
//               for the second weight set of SwiGLU) the packed weight tile
//               (128 rows x 64 B for 4-bit, 64-byte swizzle), into a ring of SS
//               shared-memory slots. The first SS weight tiles are issued
//               before the grid dependency resolves (weights never depend on
//               the previous kernel).
//   warp 1      TMEM owner and MMA issuer: tcgen05.mma.kind::f16 with the
//               dequantised weights as the A operand read from tensor memory
//               and x as the B operand from shared memory; fp32 accumulators
//               in tensor memory, two accumulator slots when they fit, so the
//               epilogue of one tile overlaps the next tile's MMAs.
//   warps 4-11  dequantisers: thread (warp%4, lane) owns weight row
//               32*(warp%4)+lane and converts its packed words into element
//               pairs with MLX rounding (dequant_chunk), stored straight into
//               tensor memory with tcgen05.st; scales/biases for the next unit
//               are loaded while the current one is converted.
//   warps 12-15 epilogue: tcgen05.ld of the accumulators. A tile finished by
//               one CTA is rounded (and SwiGLU-combined), staged in shared
//               memory and written with coalesced 16-byte stores (+ residual).
//               A tile shared by several CTAs: each participant writes its
//               fp32 partial to the workspace and raises a flag; after its
//               own range every participant waits for the tile's flags and
//               reduces one slice of the tile's rows, summing the partials in
//               K order — the result does not depend on timing — then the last
//               participant to finish clears the tile's flags.
//
// Every wait (mbarriers, partial flags) is bounded (2 s); on expiry the CTA
// records the site in the device status word, stops, drains its in-flight
// copies and MMAs (bounded) and frees its tensor memory.
#include "mt_common.cuh"
#include "mt_tma.h"
#include "qmm_common.cuh"

namespace mt {

constexpr int kBM = 128;       // weight rows per tile (MMA M)
constexpr int kBK = 128;       // K per unit
constexpr int kThreads = 512;  // 16 warps
constexpr int kMaxSS = 6;
constexpr int kTmemCols = 512;
constexpr int kAccCols = 256;  // accumulator slots live in columns [0, 256)
constexpr int kEpiWarp0 = 12;
constexpr int kEpiBar = 2;     // named barrier of the epilogue warpgroup
constexpr int kAllBar = 1;     // named barrier of all 512 threads
constexpr int kSmemLimit = 232448;
constexpr int kMaxP = 256;     // CTAs the workspace query provisions for

struct QmmTcParams {
  CUtensorMap tmx;     // x [M, K]
  CUtensorMap tmw[3];  // packed weights of each set [N_s, K*bits/32]
  const void* s[3];
  const void* b[3];
  void* y[3];
  const void* residual;
  uint32_t* flags;     // [P][2]: partial of slot published
  uint32_t* done;      // [tiles]: participants finished with a shared tile
  float* partials;     // [P][2][NACC][16 groups][TNp][8 rows]
  long long units;
  uint64_t p_magic;      // ceil(2^64 / P), 0 when P == 1
  uint64_t units_magic;  // ceil(2^64 / units), 0 when units == 1
  int N[3];
  int tile_start[4];   // prefix sums of feature tiles per set
  int M, K, G, group;
  int TN, TNp, SS, nk, kind, n_tt, tiles, P, acc_slots, vec, sb_vec, gshift;
};

template <int BITS>
struct WLayout {
  static constexpr int kRowBytes = kBK * BITS / 8;  // packed bytes per row per unit
  static constexpr int kChunks = kRowBytes / 16;    // 16-byte chunks per row
  static constexpr int kValuesPerChunk = 128 / BITS;
  // physical 16-byte chunk of logical chunk c in row r under the TMA swizzle
  static __device__ __forceinline__ int phys(int r, int c) {
    return BITS == 4 ? (c ^ ((r >> 1) & 3)) : (c ^ (r & 7));
  }
};

// floor(n / d) as a multiply-high by the host-computed magic ceil(2^64 / d)
// (0 for d = 1); exact while n * d < 2^64, which the host checks.
__device__ __forceinline__ long long div_magic(uint64_t n, uint64_t magic) {
  return static_cast<long long>(magic ? __umul64hi(n, magic) : n);
}

// first unit of CTA c: floor(c * units / P)
__device__ __forceinline__ long long unit_begin(const QmmTcParams& p, long long c) {
  return div_magic(static_cast<uint64_t>(c) * static_cast<uint64_t>(p.units), p.p_magic);
}

// CTA whose unit range contains unit x
__device__ __forceinline__ int owner_of(const QmmTcParams& p, long long x) {
  int c = static_cast<int>(div_magic(static_cast<uint64_t>(x) * static_cast<uint64_t>(p.P), p.units_magic));
  while (c + 1 < p.P && unit_begin(p, c + 1) <= x) ++c;
  while (c > 0 && unit_begin(p, c) > x) --c;
  return c;
}

struct TileInfo {
  int set, n0, tok0;
};

__device__ __forceinline__ TileInfo tile_info(const QmmTcParams& p, int tile, bool dual) {
  TileInfo ti;
  const int ft = p.n_tt == 1 ? tile : tile / p.n_tt;
  ti.tok0 = (tile - ft * p.n_tt) * p.TN;
  int set = 0;
  if (!dual) {
    if (ft >= p.tile_start[1]) set = 1;
    if (ft >= p.tile_start[2]) set = 2;
  }
  ti.set = set;
  ti.n0 = (ft - p.tile_start[set]) * kBM;
  return ti;
}

// Finished values of two outputs from their fp32 accumulators (gate and up
// for SwiGLU): the element-type result, residual not included.
template <int DT, int NACC>
__device__ __forceinline__ typename Elem<DT>::T2 finish2(float a0, float a1, float b0, float b1) {
  if constexpr (NACC == 2) return swiglu2_fast<DT>(a0, a1, b0, b1);
  else return Elem<DT>::pack2(a0, a1);
}

// Bytes of the output staging area: TN x 128 finished 16-bit values.
__host__ __device__ constexpr int stage_bytes_for(int TN) { return TN * kBM * 2; }

template <int DT, int BITS, int DUAL>
__global__ void __launch_bounds__(kThreads, 1) qmm_tc_kernel(const __grid_constant__ QmmTcParams p) {
  using T = typename Elem<DT>::T;
  using WL = WLayout<BITS>;
  constexpr int NACC = DUAL ? 2 : 1;
  constexpr int TS = DUAL ? 2 : 4;  // tensor-memory A stages
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int TN = p.TN, SS = p.SS, nk = p.nk;
  const int x_stage_bytes = TN * 256;                 // 2 boxes of TN rows x 128 B
  const int w_set_bytes = kBM * WL::kRowBytes;
  const int w_stage_bytes = NACC * w_set_bytes;
  uint8_t* xs = smem;
  uint8_t* ws_ = smem + SS * x_stage_bytes;
  // output staging: [TN][128] finished values
  T* stage_out = reinterpret_cast<T*>(ws_ + SS * w_stage_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(stage_out) + stage_bytes_for(TN));
  uint64_t* w_full = bars;                // [2][kMaxSS]: weight set 0 / 1 landed
  uint64_t* x_full = bars + 2 * kMaxSS;
  uint64_t* s_empty = bars + 3 * kMaxSS;
  uint64_t* a_full = bars + 4 * kMaxSS;
  uint64_t* a_empty = a_full + 4;
  uint64_t* acc_full = a_empty + 4;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* red_bar = drain + 1;  // partial slices landed (reduction)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* shared_tile_slot = abort_flag + 1;  // [2]: tiles this CTA shares (first / last segment)
  volatile int* last_seg = shared_tile_slot + 2;  // [5]: tile, shared, pslot, slot, parity of the last segment

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const long long u0 = unit_begin(p, c);
  const long long u1 = unit_begin(p, c + 1);
  const int nunits = static_cast<int>(u1 - u0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kMaxSS; ++i) {
      mbar_init(&w_full[i], 1);
      mbar_init(&w_full[kMaxSS + i], 1);
      mbar_init(&x_full[i], 1);
      mbar_init(&s_empty[i], 1 + 8);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&a_full[i], 8);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(drain, 1);
    mbar_init(red_bar, 1);
    *abort_flag = 0;
    shared_tile_slot[0] = -1;
    shared_tile_slot[1] = -1;
    last_seg[0] = -1;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tmx);
    for (int a = 0; a < (DUAL ? 2 : 3); ++a)
      if (p.N[a] > 0) prefetch_tmap(&p.tmw[a]);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Dependents only run set-up before their own griddep_wait(); letting them
  // launch now hides their launch latency behind this kernel.
  griddep_launch();

  // ---- accumulator segments: a segment is the part of one tile a CTA's
  // range covers. seg_load reads the accumulator slot (rows of subpartition q,
  // 32-token chunks from chunk0 in steps of cstep) and either writes the fp32
  // partial to the workspace (a tile shared with other CTAs) or the finished
  // values to the staging area; seg_publish then raises the partial's flag or
  // writes the staged tile with coalesced stores (+ residual). Both are run by
  // a group of gsize threads (gt = index in the group) with named barrier bar.
  const T* res = static_cast<const T*>(p.residual);
  auto seg_load = [&](int tile, bool shared, int pslot, int slot, int q, int ln, int chunk0, int cstep) {
    const int r = q * 32 + ln;
    const uint32_t acc_base = tmem + (static_cast<uint32_t>(q * 32) << 16) + slot * NACC * TN;
    (void)tile;
    for (int c0 = chunk0; c0 < TN; c0 += cstep) {
      const int w = (TN - c0) < 32 ? (TN - c0) : 32;
      uint32_t v[NACC][32];
#pragma unroll
      for (int a = 0; a < NACC; ++a) {
        if (w == 32) tmem_ld32(acc_base + a * TN + c0, v[a]);
        else tmem_ld16(acc_base + a * TN + c0, v[a]);
      }
      tmem_wait_ld();
      if (shared) {
        // fp32 partial, layout [8-row group][token][8 rows], so that a row
        // range of all tokens is contiguous; for each token a warp's store
        // covers four full 32-byte sectors
#pragma unroll
        for (int a = 0; a < NACC; ++a) {
          float* dst = p.partials + ((static_cast<long long>(c) * 2 + pslot) * NACC + a) * p.TNp * kBM +
                       (r >> 3) * (p.TNp * 8) + c0 * 8 + (r & 7);
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (e < w) __stcg(dst + e * 8, __uint_as_float(v[a][e]));
        }
      } else {
        // the residual is added at the coalesced store
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          if (e < w) {
            const typename Elem<DT>::T2 o =
                finish2<DT, NACC>(__uint_as_float(v[0][e]), __uint_as_float(v[0][e + 1]),
                                  __uint_as_float(v[NACC - 1][e]), __uint_as_float(v[NACC - 1][e + 1]));
            stage_out[(c0 + e) * kBM + r] = o.x;
            stage_out[(c0 + e + 1) * kBM + r] = o.y;
          }
        }
      }
    }
  };
  auto seg_publish = [&](int tile, bool shared, int pslot, int gt, int gsize, int bar) {
    named_barrier(bar, gsize);
    if (shared) {
      if (gt == 0) {
        __threadfence();
        st_release_gpu(&p.flags[c * 2 + pslot], 1u);
        shared_tile_slot[pslot] = tile;
      }
      return;
    }
    const TileInfo ti = tile_info(p, tile, DUAL);
    T* y = static_cast<T*>(p.y[DUAL ? 0 : ti.set]);
    const int N = p.N[DUAL ? 0 : ti.set];
    for (int idx = gt; idx < TN * 16; idx += gsize) {
      const int tok = idx >> 4, cc = idx & 15;
      const int token = ti.tok0 + tok, n = ti.n0 + cc * 8;
      if (token >= p.M || n >= N) continue;
      const T* src = stage_out + tok * kBM + cc * 8;
      const long long off = static_cast<long long>(token) * N + n;
      if (p.vec && n + 8 <= N) {
        uint4 val = *reinterpret_cast<const uint4*>(src);
        if (!DUAL && p.kind == QMM_RESIDUAL) {
          const uint4 rv = *reinterpret_cast<const uint4*>(res + off);
          T* ve = reinterpret_cast<T*>(&val);
          const T* re = reinterpret_cast<const T*>(&rv);
#pragma unroll
          for (int e = 0; e < 8; ++e) ve[e] = Elem<DT>::from_f(Elem<DT>::to_f(ve[e]) + Elem<DT>::to_f(re[e]));
        }
        *reinterpret_cast<uint4*>(y + off) = val;
      } else {
        for (int e = 0; e < 8 && n + e < N; ++e) {
          float vv = Elem<DT>::to_f(src[e]);
          if (!DUAL && p.kind == QMM_RESIDUAL) vv = vv + Elem<DT>::to_f(res[off + e]);
          y[off + e] = Elem<DT>::from_f(vv);
        }
      }
    }
    named_barrier(bar, gsize);
  };

  if (warp == 0 || warp == 2 || (DUAL && warp == 3)) {
    // ------------------------------------------------------------ producers
    // One warp per stream (x; weight set 0; weight set 1 when dual): copies
    // issued by different warps are in flight together, while one thread's
    // successive copies largely serialise.
    if (lane == 0) {
      const bool is_x = warp == 0;
      const int a = warp == 3 ? 1 : 0;
      const int kw_per_stage = kBK * BITS / 32;  // words of K per unit
      const int pre = nunits < SS ? nunits : SS;
      const int tile0 = static_cast<int>(u0) / nk;
      int it_tile = tile0, it_k = static_cast<int>(u0 - static_cast<long long>(tile0) * nk);
      uint64_t* full = is_x ? x_full : w_full + a * kMaxSS;
      const int bytes = is_x ? x_stage_bytes : w_set_bytes;
      auto issue = [&](int i) {
        const TileInfo ti = tile_info(p, it_tile, DUAL);
        const int s = i % SS;
        mbar_arrive_expect_tx(&full[s], bytes);
        if (is_x)
          tma_load_3d(xs + s * x_stage_bytes, &p.tmx, &full[s], 0, ti.tok0, it_k * 2);
        else
          tma_load_2d(ws_ + s * w_stage_bytes + a * w_set_bytes, &p.tmw[DUAL ? a : ti.set], &full[s],
                      it_k * kw_per_stage, ti.n0);
        if (++it_k == nk) {
          it_k = 0;
          ++it_tile;
        }
      };
      int issued = 0;
      // weights never depend on the previous kernel: their first stages are
      // issued before the grid dependency resolves
      if (is_x) griddep_wait();
      for (int i = 0; i < pre; ++i, ++issued) issue(i);
      for (int i = pre; i < nunits; ++i) {
        const int s = i % SS;
        if (!mbar_wait(&s_empty[s], ((i / SS) & 1) ^ 1, abort_flag, is_x ? 0x101 : 0x102)) break;
        issue(i);
        ++issued;
      }
      if (*abort_flag) {
        for (int i = (issued > SS ? issued - SS : 0); i < issued; ++i)
          mbar_wait_drain(&full[i % SS], (i / SS) & 1, 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop (its waits and bookkeeping stay warp-uniform)
    // and one elected lane issues; descriptors are formed once, and each MMA
    // only adds a precomputed offset, so the issue rate is the tensor core's.
    const uint32_t idesc = idesc_f16(kBM, TN, DT == MT_BF16);
    const uint64_t xdesc0 = smem_desc_k_sw128(smem_addr(xs));
    uint32_t koff[kBK / 16];  // descriptor address offset of each 16-wide K step
#pragma unroll
    for (int kk = 0; kk < kBK / 16; ++kk) koff[kk] = static_cast<uint32_t>(((kk >> 2) * TN * 128 + (kk & 3) * 32) >> 4);
    const uint32_t xstep = static_cast<uint32_t>(x_stage_bytes >> 4);
    bool issued = false;
    int use[2] = {0, 0};
    int slot = 0;
    int s = 0, sph = 0, t = 0, tph = 0;
    bool ok = true;
    long long u = u0;
    while (u < u1 && ok) {
      const int klo = static_cast<int>(u) % nk;
      const int len = static_cast<int>(((nk - klo) < (u1 - u)) ? (nk - klo) : (u1 - u));
      if (!mbar_wait_warp(&acc_empty[slot], (use[slot] & 1) ^ 1, abort_flag, 0x203)) break;
      tc_fence_after();
      const uint32_t d_base = tmem + slot * NACC * TN;
      for (int j = 0; j < len; ++j) {
        if (!mbar_wait_warp(&x_full[s], sph, abort_flag, 0x201) ||
            !mbar_wait_warp(&a_full[t], tph, abort_flag, 0x202)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t sdesc = xdesc0 + s * xstep;
        const uint32_t abase = tmem + kAccCols + t * NACC * 64;
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
#pragma unroll
            for (int a = 0; a < NACC; ++a)
              tc_mma_ts(d_base + a * TN, abase + a * 64 + kk * 8, sdesc + koff[kk], idesc,
                        (j > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&s_empty[s]);
          tc_commit(&a_empty[t]);
        }
        __syncwarp();
        issued = true;
        if (++s == SS) {
          s = 0;
          sph ^= 1;
        }
        if (++t == TS) {
          t = 0;
          tph ^= 1;
        }
      }
      if (!ok) break;
      if (elect_one()) tc_commit(&acc_full[slot]);
      __syncwarp();
      ++use[slot];
      slot = (slot + 1) % p.acc_slots;
      u += len;
    }
    if (__any_sync(0xffffffffu, *abort_flag != 0) && issued) {
      if (elect_one()) {
        tc_commit(drain);
        mbar_wait_drain(drain, 0, 200000000ull);
      }
      __syncwarp();
    }
  } else if (warp >= 4 && warp < kEpiWarp0) {
    // ------------------------------------------------------------ dequantisers
    const int q = warp & 3;
    const int wg = (warp - 4) >> 2;
    const int r = q * 32 + lane;  // weight row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    // single: WG wg converts chunks [wg*C/2, (wg+1)*C/2); dual: all chunks of set wg
    constexpr int kMyChunks = DUAL ? WL::kChunks : WL::kChunks / 2;
    const int aset = DUAL ? wg : 0;
    const int c0 = DUAL ? 0 : wg * kMyChunks;
    constexpr int kPairsPerChunk = WL::kValuesPerChunk / 2;
    constexpr int kCols = kMyChunks * kPairsPerChunk;  // 32 (single) or 64 (dual)
    // Scales and biases: each thread holds an aligned block of 8 consecutive
    // groups of its row (one 16-byte load each, raw element bits), which
    // covers group/16 units (4 at group 64). Rows are G*2 bytes apart, so
    // per-unit scalar loads would touch one sector per lane per load; block
    // loads cut that 8x. When a block comes into use, the next one is loaded.
    // Unit bookkeeping is incremental: no integer division in the loop.
    const int gshift = p.gshift;            // log2(group)
    const int upb = p.group >> 4;           // units per 8-group block
    uint4 sc_cur = make_uint4(0, 0, 0, 0), bi_cur = sc_cur, sc_nxt = sc_cur, bi_nxt = sc_cur;
    auto load_block = [&](int tile, int k, uint4& s_out, uint4& b_out) {
      const TileInfo ti = tile_info(p, tile, DUAL);
      const int wset = DUAL ? wg : ti.set;
      const int n = ti.n0 + r;
      const bool row_ok = n < p.N[wset];
      const int gb = ((k * kBK) >> gshift) & ~7;
      const T* srow = static_cast<const T*>(p.s[wset]) + static_cast<long long>(row_ok ? n : 0) * p.G;
      const T* brow = static_cast<const T*>(p.b[wset]) + static_cast<long long>(row_ok ? n : 0) * p.G;
      if (row_ok && p.sb_vec && gb + 8 <= p.G) {
        s_out = __ldg(reinterpret_cast<const uint4*>(srow + gb));
        b_out = __ldg(reinterpret_cast<const uint4*>(brow + gb));
      } else {
        uint16_t sv[8], bv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const bool ok = row_ok && gb + e < p.G;
          sv[e] = ok ? reinterpret_cast<const uint16_t*>(srow)[gb + e] : 0;
          bv[e] = ok ? reinterpret_cast<const uint16_t*>(brow)[gb + e] : 0;
        }
        s_out = make_uint4(sv[0] | (uint32_t(sv[1]) << 16), sv[2] | (uint32_t(sv[3]) << 16),
                           sv[4] | (uint32_t(sv[5]) << 16), sv[6] | (uint32_t(sv[7]) << 16));
        b_out = make_uint4(bv[0] | (uint32_t(bv[1]) << 16), bv[2] | (uint32_t(bv[3]) << 16),
                           bv[4] | (uint32_t(bv[5]) << 16), bv[6] | (uint32_t(bv[7]) << 16));
      }
    };
    // element e (0..7) of a block, widened to float
    auto pick = [](const uint4& v, int e) -> float {
      const uint32_t w = (e < 4) ? ((e < 2) ? v.x : v.y) : ((e < 6) ? v.z : v.w);
      const uint32_t bits = (e & 1) ? (w >> 16) : (w & 0xFFFFu);
      if constexpr (DT == MT_BF16) return __uint_as_float(bits << 16);
      else return __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
    };
    // units from (tile, k) to the start of the next block (or of the next tile)
    auto to_next_block = [&](int k) {
      const int a = upb - (k & (upb - 1)), b = nk - k;
      return a < b ? a : b;
    };
    int tile = static_cast<int>(u0) / nk, k = static_cast<int>(u0) - tile * nk;
    int next_start = nunits;  // unit index where the prefetched block takes over
    if (nunits > 0) {
      load_block(tile, k, sc_cur, bi_cur);
      const int d = to_next_block(k);
      if (d < nunits) {
        next_start = d;
        const bool wrap = (k + d == nk);
        load_block(wrap ? tile + 1 : tile, wrap ? 0 : k + d, sc_nxt, bi_nxt);
      }
    }
    // The tensor-memory stores of unit i complete (wait + fence + a_full
    // arrive) after unit i+1's weights are read from shared memory, so their
    // latency overlaps that read; if unit i+1's weights have not landed yet,
    // unit i is completed first rather than held back behind the copy.
    int s = 0, sph = 0, t = 0, tph = 0;
    int pend_t = -1;  // A stage whose stores are issued but not yet published
    auto publish = [&]() {
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[pend_t]);
      pend_t = -1;
    };
    for (int i = 0; i < nunits; ++i) {
      if (i == next_start) {
        sc_cur = sc_nxt;
        bi_cur = bi_nxt;
        const int d = to_next_block(k);
        if (i + d < nunits) {
          next_start = i + d;
          const bool wrap = (k + d == nk);
          load_block(wrap ? tile + 1 : tile, wrap ? 0 : k + d, sc_nxt, bi_nxt);
        }
      }
      uint64_t* wf = &w_full[aset * kMaxSS + s];
      if (pend_t >= 0 && !__all_sync(0xffffffffu, mbar_test(wf, sph))) publish();
      if (!mbar_wait_warp(wf, sph, abort_flag, 0x301)) break;
      uint4 wv[kMyChunks];
      const uint8_t* wrow = ws_ + s * w_stage_bytes + aset * w_set_bytes + r * WL::kRowBytes;
#pragma unroll
      for (int cc = 0; cc < kMyChunks; ++cc)
        wv[cc] = *reinterpret_cast<const uint4*>(wrow + WL::phys(r, c0 + cc) * 16);
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[s]);
      if (pend_t >= 0) publish();
      const int kst = k * kBK;
      const int gb = (kst >> gshift) & ~7;
      if (!mbar_wait_warp(&a_empty[t], tph ^ 1, abort_flag, 0x302)) break;
      const uint32_t col0 = kAccCols + (t * NACC + aset) * 64 + (DUAL ? 0 : wg * 32);
#pragma unroll
      for (int h = 0; h < kCols / 32; ++h) {
        uint32_t out[32];
        constexpr int kChunksPer32 = 32 / kPairsPerChunk;
#pragma unroll
        for (int cc = 0; cc < kChunksPer32; ++cc) {
          const int ch = h * kChunksPer32 + cc;
          const int e = ((kst + (c0 + ch) * WL::kValuesPerChunk) >> gshift) - gb;
          dequant_chunk<DT, BITS>(wv[ch], pick(sc_cur, e), pick(bi_cur, e), out + cc * kPairsPerChunk);
        }
        tmem_st32(tmem + lane_base + col0 + h * 32, out);
      }
      pend_t = t;
      if (++k == nk) {
        k = 0;
        ++tile;
      }
      if (++s == SS) {
        s = 0;
        sph ^= 1;
      }
      if (++t == TS) {
        t = 0;
        tph ^= 1;
      }
    }
    if (pend_t >= 0) publish();
  } else if (warp >= kEpiWarp0) {
    // ------------------------------------------------------------ epilogue
    // Every segment but the CTA's last: the last one is finished by all 16
    // warps once the main loop is over.
    const int q = warp & 3;
    const int et = threadIdx.x - kEpiWarp0 * 32;  // 0..127
    griddep_wait();
    int use[2] = {0, 0};
    int slot = 0;
    long long u = u0;
    while (u < u1) {
      const int tile = static_cast<int>(u) / nk;
      const int klo = static_cast<int>(u) % nk;
      const int len = static_cast<int>(((nk - klo) < (u1 - u)) ? (nk - klo) : (u1 - u));
      const bool shared = !(klo == 0 && len == nk);
      const int pslot = (u == u0) ? 0 : 1;
      if (u + len == u1) {
        if (et == 0) {
          last_seg[0] = tile;
          last_seg[1] = shared ? 1 : 0;
          last_seg[2] = pslot;
          last_seg[3] = slot;
          last_seg[4] = use[slot] & 1;
        }
        break;
      }
      const bool got = mbar_wait(&acc_full[slot], use[slot] & 1, abort_flag, 0x401);
      if (named_barrier_or(kEpiBar, 128, !got || *abort_flag)) break;
      tc_fence_after();
      seg_load(tile, shared, pslot, slot, q, lane, 0, 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[slot]);
      ++use[slot];
      slot = (slot + 1) % p.acc_slots;
      seg_publish(tile, shared, pslot, et, 128, kEpiBar);
      u += len;
    }
  }

  // ---- the CTA's last segment, by all 16 warps: warp w reads subpartition
  // w % 4 and 32-token chunk w / 4 of the accumulator
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (last_seg[0] >= 0) {
    const int slot = last_seg[3];
    const bool got = mbar_wait(&acc_full[slot], static_cast<uint32_t>(last_seg[4]), abort_flag, 0x403);
    if (!named_barrier_or(kAllBar, kThreads, !got || *abort_flag)) {
      tc_fence_after();
      seg_load(last_seg[0], last_seg[1] != 0, last_seg[2], slot, warp & 3, lane, (warp >> 2) * 32, 128);
      seg_publish(last_seg[0], last_seg[1] != 0, last_seg[2], threadIdx.x, kThreads, kAllBar);
    }
  }

  // ---- tensor memory is no longer read: free it before the reductions, so a
  // dependent kernel's CTA waiting on this SM can allocate
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }

  // ---- reductions of the tiles this CTA shares with its neighbours, by all
  // threads. Participant j of a tile's S participants reduces row groups
  // [16j/S, 16(j+1)/S) of 8 rows. The participants' slices of those groups
  // (contiguous in the partial layout) are brought into the idle pipeline
  // buffers with bulk copies (one per participant and accumulator; chunks of
  // participants when they do not all fit), summed in participant (= K) order
  // from shared memory, finished into a padded staging tile and written with
  // coalesced stores.
  const int area = SS * (x_stage_bytes + w_stage_bytes);
  constexpr int kStgPitch = kBM + 8;  // staging row in elements: 272 B, 2-way conflicts at most
  T* stg = reinterpret_cast<T*>(smem + area - TN * kStgPitch * static_cast<int>(sizeof(T)));
  const int slice_bytes = TN * 32;    // one 8-row group of one partial, all tokens
  const int max_slices = (area - TN * kStgPitch * static_cast<int>(sizeof(T))) / slice_bytes;
  uint32_t red_phase = 0;
  for (int ps = 0; ps < 2; ++ps) {
    const int tile = shared_tile_slot[ps];
    if (tile < 0) continue;
    if (ps == 1 && tile == shared_tile_slot[0]) continue;
    const long long t_lo = static_cast<long long>(tile) * nk;
    const int ca = owner_of(p, t_lo);
    const int cb = owner_of(p, t_lo + nk - 1);
    const int S = cb - ca + 1;
    const int j = c - ca;
    // wait for every participant's partial: thread jj polls participant ca+jj
    for (int jj = threadIdx.x; jj < S; jj += kThreads) {
      const int cp = ca + jj;
      const int sl = (unit_begin(p, cp) >= t_lo) ? 0 : 1;
      const uint32_t* f = &p.flags[cp * 2 + sl];
      if (ld_acquire_gpu(f) == 1u) continue;
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_gpu(f) != 1u) {
        if (*abort_flag) break;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          *abort_flag = 1;
          report_status(0x402);
          break;
        }
      }
    }
    // the pollers' acquire loads and the barrier order every thread's reads
    // of the partials after the writers' releases
    if (__syncthreads_or(*abort_flag)) break;
    const int g_lo = (j * 16) / S, g_hi = ((j + 1) * 16) / S;
    const int ng = g_hi - g_lo;
    const int per_part = NACC * ng;  // slices per participant
    const int pc_max = ng > 0 ? max_slices / per_part : S;
    const int nit = ng * TN * 2;     // items: (group, token, 4-row half)
    constexpr int kMaxIt = 4;        // ng <= 8, TN <= 128: at most 4 items per thread
    float acc[kMaxIt][NACC][4];
#pragma unroll
    for (int jj = 0; jj < kMaxIt; ++jj)
#pragma unroll
      for (int a = 0; a < NACC; ++a) acc[jj][a][0] = acc[jj][a][1] = acc[jj][a][2] = acc[jj][a][3] = 0.f;
    bool ok = true;
    for (int pc0 = 0; ng > 0 && pc0 < S; pc0 += pc_max) {
      const int npc = (S - pc0) < pc_max ? (S - pc0) : pc_max;
      if (threadIdx.x == 0)
        mbar_arrive_expect_tx(red_bar, static_cast<uint32_t>(npc * per_part * slice_bytes));
      __syncthreads();  // expect_tx registered; the previous chunk's reads are done
      if (lane == 0) {
        // copies spread over the 16 warps so that they are in flight together
        for (int i = warp; i < npc * NACC; i += kThreads / 32) {
          if (i == warp) {
            fence_proxy_async_global();
            fence_proxy_async_shared();
          }
          const int pi = i / NACC, a = i - pi * NACC;
          const int cp = ca + pc0 + pi;
          const int sl = (unit_begin(p, cp) >= t_lo) ? 0 : 1;
          const float* src = p.partials + ((static_cast<long long>(cp) * 2 + sl) * NACC + a) * p.TNp * kBM +
                             g_lo * (p.TNp * 8);
          bulk_load(smem + (pi * per_part + a * ng) * slice_bytes, src, ng * slice_bytes, red_bar);
        }
      }
      const bool got = mbar_wait(red_bar, red_phase & 1, abort_flag, 0x404);
      ++red_phase;
      if (__syncthreads_or(!got || *abort_flag)) {
        if (threadIdx.x == 0) mbar_wait_drain(red_bar, (red_phase - 1) & 1, 200000000ull);
        ok = false;
        break;
      }
#pragma unroll
      for (int jj = 0; jj < kMaxIt; ++jj) {
        const int it = threadIdx.x + jj * kThreads;
        if (it >= nit) break;
        const int h = it & 1, tg = it >> 1;
        const int gg = tg / TN, tok = tg - gg * TN;
        const uint8_t* base = smem + (gg * TN + tok) * 32 + h * 16;
        for (int pi = 0; pi < npc; ++pi) {
#pragma unroll
          for (int a = 0; a < NACC; ++a) {
            const float4 v = *reinterpret_cast<const float4*>(base + (pi * per_part + a * ng) * slice_bytes);
            acc[jj][a][0] += v.x;
            acc[jj][a][1] += v.y;
            acc[jj][a][2] += v.z;
            acc[jj][a][3] += v.w;
          }
        }
      }
    }
    if (!ok) break;
    // finish into the staging tile (the residual is added at the store)
#pragma unroll
    for (int jj = 0; jj < kMaxIt; ++jj) {
      const int it = threadIdx.x + jj * kThreads;
      if (it >= nit) break;
      const int h = it & 1, tg = it >> 1;
      const int gg = tg / TN, tok = tg - gg * TN;
      typename Elem<DT>::T2 o[2];
#pragma unroll
      for (int e = 0; e < 4; e += 2)
        o[e / 2] = finish2<DT, NACC>(acc[jj][0][e], acc[jj][0][e + 1], acc[jj][NACC - 1][e], acc[jj][NACC - 1][e + 1]);
      *reinterpret_cast<uint2*>(stg + tok * kStgPitch + (g_lo + gg) * 8 + h * 4) =
          *reinterpret_cast<const uint2*>(o);
    }
    __syncthreads();
    {
      const TileInfo ti = tile_info(p, tile, DUAL);
      T* y = static_cast<T*>(p.y[DUAL ? 0 : ti.set]);
      const int N = p.N[DUAL ? 0 : ti.set];
      for (int idx = threadIdx.x; idx < TN * ng; idx += kThreads) {
        const int tok = idx / ng, k8 = idx - tok * ng;
        const int token = ti.tok0 + tok, n = ti.n0 + (g_lo + k8) * 8;
        if (token >= p.M || n >= N) continue;
        const T* src = stg + tok * kStgPitch + (g_lo + k8) * 8;
        const long long off = static_cast<long long>(token) * N + n;
        if (p.vec && n + 8 <= N) {
          uint4 val = *reinterpret_cast<const uint4*>(src);
          if (!DUAL && p.kind == QMM_RESIDUAL) {
            const uint4 rv = *reinterpret_cast<const uint4*>(res + off);
            T* ve = reinterpret_cast<T*>(&val);
            const T* re = reinterpret_cast<const T*>(&rv);
#pragma unroll
            for (int e = 0; e < 8; ++e) ve[e] = Elem<DT>::from_f(Elem<DT>::to_f(ve[e]) + Elem<DT>::to_f(re[e]));
          }
          *reinterpret_cast<uint4*>(y + off) = val;
        } else {
          for (int e = 0; e < 8 && n + e < N; ++e) {
            float vv = Elem<DT>::to_f(src[e]);
            if (!DUAL && p.kind == QMM_RESIDUAL) vv = vv + Elem<DT>::to_f(res[off + e]);
            y[off + e] = Elem<DT>::from_f(vv);
          }
        }
      }
    }
    __syncthreads();  // staging and slices are reused by the next tile
    if (threadIdx.x == 0) {
      const uint32_t prev = atomicAdd(&p.done[tile], 1u);
      if (prev == static_cast<uint32_t>(S - 1)) {
        // every participant has read every partial of this tile: clear for the next call
        for (int cp = ca; cp <= cb; ++cp) {
          const int sl = (unit_begin(p, cp) >= t_lo) ? 0 : 1;
          p.flags[cp * 2 + sl] = 0u;
        }
        p.done[tile] = 0u;
      }
    }
  }
}

// ------------------------------------------------------------------- host

static size_t smem_bytes_for(int TN, int SS, int bits, int dual) {
  const int nacc = dual ? 2 : 1;
  const size_t stage = static_cast<size_t>(TN) * 256 + static_cast<size_t>(nacc) * kBM * (kBK * bits / 8);
  return 1024 + SS * stage + stage_bytes_for(TN) + 512;
}

static int pick_ss(int TN, int bits, int dual) {
  int ss = kMaxSS;
  while (ss > 2 && smem_bytes_for(TN, ss, bits, dual) > static_cast<size_t>(kSmemLimit)) --ss;
  return ss;
}

static int tile_tn(int64_t M) {
  int64_t tn = M < 128 ? M : 128;
  tn = (tn + 15) / 16 * 16;
  return static_cast<int>(tn);
}

struct WsLayout {
  size_t flags, done, partials, total;
};

static WsLayout ws_layout(int P, int64_t tiles, int nacc, int TNp) {
  (void)tiles;
  WsLayout l;
  l.flags = kWsQmmFlags;
  l.done = kWsQmmDone;
  l.partials = kWsCtlBytes;
  l.total = l.partials + static_cast<size_t>(P) * 2 * nacc * TNp * kBM * 4;
  return l;
}

size_t qmm_tc_workspace(int64_t M, int64_t n_total, int64_t K, int bits, int kind) {
  (void)bits;
  (void)K;
  const int dual = kind == 1;
  const int TN = tile_tn(M);
  const int64_t n_tt = (M + TN - 1) / TN;
  const int64_t ft = dual ? (n_total / 2 + kBM - 1) / kBM : (n_total + kBM - 1) / kBM + 3;
  return ws_layout(kMaxP, ft * n_tt, dual ? 2 : 1, TN).total;
}

template <int DT, int BITS, int DUAL>
static int launch_tc(QmmTcParams& p, size_t smem, cudaStream_t stream) {
  auto k = qmm_tc_kernel<DT, BITS, DUAL>;
  if (int e = ensure_smem(k, kSmemLimit)) return e;
  return launch(k, dim3(p.P), dim3(kThreads), smem, stream, p);
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
  p.gshift = r.group == 32 ? 5 : r.group == 64 ? 6 : 7;
  p.G = static_cast<int>(r.K / r.group);
  p.kind = r.kind;
  p.residual = r.residual;
  p.TN = tile_tn(r.M);
  p.TNp = p.TN;
  p.SS = pick_ss(p.TN, r.bits, dual);
  p.nk = static_cast<int>((r.K + kBK - 1) / kBK);
  p.acc_slots = dual ? 1 : 2;
  p.n_tt = static_cast<int>((r.M + p.TN - 1) / p.TN);

  const CUtensorMapDataType xdt =
      r.dtype == MT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  {
    // x as (64 values, M rows, K/64 blocks): one copy brings both 64-wide K
    // halves of a unit, each as TN swizzled rows of 128 B
    const uint64_t dims[3] = {64, static_cast<uint64_t>(r.M), static_cast<uint64_t>(r.K / 64)};
    const uint64_t strides[2] = {static_cast<uint64_t>(r.K) * esz, 64 * esz};
    const uint32_t box[3] = {64, static_cast<uint32_t>(p.TN), 2};
    rc = make_tmap(&p.tmx, r.x, xdt, esz, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (rc != MT_OK) return rc;
  const int words = static_cast<int>(r.K * r.bits / 32);
  const int nsets = dual ? 2 : 3;
  int ftiles = 0;
  bool vec = (r.residual == nullptr || aligned(r.residual, 16));
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
      if (!dual) ftiles += static_cast<int>((q.N + kBM - 1) / kBM);
      if (q.y && (!aligned(q.y, 16) || q.N % 8 != 0)) vec = false;
    }
    p.tile_start[s + 1] = ftiles;
  }
  if (dual) {
    ftiles = static_cast<int>((r.set[0].N + kBM - 1) / kBM);
    p.N[1] = p.N[0];
  }
  p.vec = vec ? 1 : 0;
  {
    bool sbv = (p.G % 8) == 0;
    for (int s2 = 0; s2 < nsets; ++s2)
      if (r.set[s2].N > 0 && (!aligned(r.set[s2].s, 16) || !aligned(r.set[s2].b, 16))) sbv = false;
    p.sb_vec = sbv ? 1 : 0;
  }
  p.tiles = ftiles * p.n_tt;
  p.units = static_cast<long long>(p.tiles) * p.nk;
  p.P = static_cast<int>(p.units < sms ? p.units : sms);
  if (p.P > kMaxP) p.P = kMaxP;
  if (p.units >= (1ll << 28)) {
    set_error("qmm: %lld K-stage units exceed the 2^28 the unit arithmetic supports", p.units);
    return MT_ERR_UNSUPPORTED;
  }
  p.p_magic = p.P > 1 ? ~0ull / static_cast<uint64_t>(p.P) + 1 : 0;
  p.units_magic = p.units > 1 ? ~0ull / static_cast<uint64_t>(p.units) + 1 : 0;
  if (static_cast<size_t>(p.tiles) > kWsQmmMaxTiles) {
    set_error("qmm: %d tiles exceed the workspace's %zu tile counters (M=%lld too large for one call)", p.tiles,
              kWsQmmMaxTiles, (long long)r.M);
    return MT_ERR_UNSUPPORTED;
  }
  const WsLayout wl = ws_layout(p.P, p.tiles, dual ? 2 : 1, p.TNp);
  if (!r.ws || r.ws_bytes < wl.total || !aligned(r.ws, 256)) {
    set_error("qmm: workspace of %zu bytes (256-aligned, zero-filled) required, got %zu", wl.total,
              r.ws ? r.ws_bytes : (size_t)0);
    return MT_ERR_WORKSPACE;
  }
  uint8_t* ws = static_cast<uint8_t*>(r.ws);
  p.flags = reinterpret_cast<uint32_t*>(ws + wl.flags);
  p.done = reinterpret_cast<uint32_t*>(ws + wl.done);
  p.partials = reinterpret_cast<float*>(ws + wl.partials);
  {
    // the reduction's largest chunk (one participant's slices: 8 groups per
    // accumulator) and the padded staging tile must fit the pipeline buffers
    const size_t area = static_cast<size_t>(p.SS) *
                        (static_cast<size_t>(p.TN) * 256 + (dual ? 2 : 1) * kBM * (kBK * r.bits / 8));
    const size_t need = static_cast<size_t>(dual ? 2 : 1) * 8 * p.TN * 32 + static_cast<size_t>(p.TN) * (kBM + 8) * 2;
    if (area < need) {
      set_error("qmm: pipeline buffers (%zu B) smaller than the reduction needs (%zu B)", area, need);
      return MT_ERR_UNSUPPORTED;
    }
  }

  const size_t smem = smem_bytes_for(p.TN, p.SS, r.bits, dual);
  const bool bf = r.dtype == MT_BF16;
  if (dual) {
    if (bf) return r.bits == 4 ? launch_tc<MT_BF16, 4, 1>(p, smem, stream) : launch_tc<MT_BF16, 8, 1>(p, smem, stream);
    return r.bits == 4 ? launch_tc<MT_F16, 4, 1>(p, smem, stream) : launch_tc<MT_F16, 8, 1>(p, smem, stream);
  }
  if (bf) return r.bits == 4 ? launch_tc<MT_BF16, 4, 0>(p, smem, stream) : launch_tc<MT_BF16, 8, 0>(p, smem, stream);
  return r.bits == 4 ? launch_tc<MT_F16, 4, 0>(p, smem, stream) : launch_tc<MT_F16, 8, 0>(p, smem, stream);
}

}  // namespace mt
