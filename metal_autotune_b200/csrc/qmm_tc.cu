// Affine-quantized matmul for prefill on the 5th-generation tensor cores.
//
// y[M, N] = x[M, K] · dequant(w)[N, K]^T, as a persistent cluster stream-K
// kernel.
//
// Work: a tile is 128 weight rows (the MMA's M) x TN <= 128 tokens (the MMA's
// N); a unit is one tile's K-stage of 128. The grid is C clusters of S CTAs
// (one CTA per SM). Cluster j owns the contiguous unit range
// [j*U/C, (j+1)*U/C); the range falls into segments, one per tile it touches,
// and every segment is split by K among the cluster's S CTAs, so the CTAs of a
// cluster always work on the same tile and finish it together.
//
// Reduction of a tile split across CTAs. The cluster holding a tile's first
// K-stage owns it. The other clusters touching the tile hold its later
// K-stages at the START of their ranges, so their fp32 partials (written to
// the workspace, then a flag raised) are ready long before the owner needs
// them. The owner's own partials are the LAST segment of its range: each of
// its CTAs parks its accumulator in its own shared memory, and after a cluster
// barrier CTA r reads row slice r of every CTA's accumulator through
// distributed shared memory, sums it with the workspace partials in K order
// (deterministic), finishes it (rounding, SwiGLU, residual) and stores it.
// With S == 1 a tile wholly inside one CTA's range is finished by that CTA
// directly.
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
//               epilogue of one segment overlaps the next segment's MMAs.
//   warps 4-11  dequantisers: thread (warp%4, lane) owns weight row
//               32*(warp%4)+lane and converts its packed words into element
//               pairs with MLX rounding (dequant_chunk), stored straight into
//               tensor memory with tcgen05.st; scales/biases for the next block
//               of groups are loaded while the current one is converted.
//   warps 12-15 epilogue of every segment but the CTA's last: a tile finished
//               here is rounded (and SwiGLU-combined), staged in shared memory
//               and written with coalesced 16-byte stores (+ residual); a
//               partial is written to the workspace and its flag raised. The
//               last segment is handled by all 16 warps after the main loop.
//
// Every wait on an mbarrier or a partial flag is bounded (2 s); on expiry the
// CTA records the site in the device status word, stops, drains its in-flight
// copies and MMAs (bounded) and frees its tensor memory. Cluster barriers are
// executed by every CTA of a cluster unconditionally (an abort only skips the
// work between them), so no CTA can be left waiting at one.
#include <cooperative_groups.h>

#include <algorithm>
#include <vector>

#include "mt_common.cuh"
#include "mt_tma.h"
#include "qmm_common.cuh"

namespace cg = cooperative_groups;

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
constexpr int kSlots = 2;      // workspace partial slots per CTA
constexpr int kMaxSegK = 3;    // segments per cluster range when S > 1
constexpr int kMaxContrib = 16;  // partials summed into one tile
constexpr int kMaxPass = 3;      // owned tiles reduced per cluster
constexpr int kMaxS = 8;
constexpr int kStgPitch = kBM + 8;  // reduction staging row in elements: 272 B

struct QmmTcParams {
  CUtensorMap tmx;     // x [M, K]
  CUtensorMap tmw[3];  // packed weights of each set [N_s, K*bits/32]
  const void* s[3];
  const void* b[3];
  void* y[3];
  const void* residual;
  uint32_t* flags;     // [P][kSlots]: partial of slot published
  uint32_t* done;      // [tiles]: owner CTAs finished reading a tile's partials
  float* partials;     // [P][kSlots][NACC][16 groups][TN][8 rows]
  long long units;
  uint64_t c_magic;    // ceil(2^64 / C), 0 when C == 1
  int N[3];
  int ldy[3];          // output (and residual) row pitch of each set, in elements
  int tile_start[4];   // prefix sums of feature tiles per set
  int M, K, G, group;
  int TN, SS, nk, kind, n_tt, tiles, S, C, acc_slots, vec, sb_vec, gshift;
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
__host__ __device__ __forceinline__ long long div_magic(uint64_t n, uint64_t magic) {
#ifdef __CUDA_ARCH__
  return static_cast<long long>(magic ? __umul64hi(n, magic) : n);
#else
  return static_cast<long long>(magic ? static_cast<uint64_t>((static_cast<unsigned __int128>(n) * magic) >> 64) : n);
#endif
}

// first unit of cluster j: floor(j * units / C)
__host__ __device__ __forceinline__ long long cluster_begin(const QmmTcParams& p, long long j) {
  return div_magic(static_cast<uint64_t>(j) * static_cast<uint64_t>(p.units), p.c_magic);
}

// Segment idx of the unit range [U0, U1) (t0 = U0 / nk): its tile and the
// K-stages [ka, kb) of that tile the range covers.
struct Seg {
  int tile, ka, kb;
};
__host__ __device__ __forceinline__ Seg seg_of(int nk, long long U0, long long U1, int t0, int idx) {
  Seg s;
  s.tile = t0 + idx;
  const long long base = static_cast<long long>(s.tile) * nk;
  s.ka = idx == 0 ? static_cast<int>(U0 - base) : 0;
  const long long e = U1 - base;
  s.kb = e < nk ? static_cast<int>(e) : nk;
  return s;
}
// rank r's share [lo, hi) of the K-stages [ka, kb): sub_k(ka, kb, S, r) .. sub_k(.., r + 1)
__host__ __device__ __forceinline__ int sub_k(int ka, int kb, int S, int r) { return ka + (r * (kb - ka)) / S; }
// first 8-row group of rank r's reduction slice
__host__ __device__ __forceinline__ int slice_lo(int S, int r) { return (16 * r) / S; }

// A segment is finished by its CTA when it is a whole tile and not split.
__host__ __device__ __forceinline__ bool seg_complete(int S, int nk, const Seg& s) {
  return S == 1 && s.ka == 0 && s.kb == nk;
}
// Workspace slot of a partial segment that is not reduced in the cluster.
__host__ __device__ __forceinline__ int seg_slot(int idx) { return idx == 0 ? 0 : 1; }

// Where a CTA's work lies: cluster j, rank r, the cluster's unit range and
// segment count, the last segment with units for this rank, and whether the
// cluster's last segment is owned and reduced in the cluster (`xchg`, the
// same in every CTA of the cluster).
struct Ctx {
  long long U0, U1;
  int j, rank, t0, nseg, last_run, nunits;
  bool xchg;
};

__device__ __forceinline__ Ctx make_ctx(const QmmTcParams& p) {
  Ctx c;
  c.j = static_cast<int>(blockIdx.x) / p.S;
  c.rank = static_cast<int>(blockIdx.x) - c.j * p.S;
  c.U0 = cluster_begin(p, c.j);
  c.U1 = cluster_begin(p, c.j + 1);
  c.t0 = static_cast<int>(c.U0 / p.nk);
  c.nseg = c.U1 > c.U0 ? static_cast<int>((c.U1 - 1) / p.nk) - c.t0 + 1 : 0;
  c.last_run = -1;
  c.nunits = 0;
  for (int i = 0; i < c.nseg; ++i) {
    const Seg s = seg_of(p.nk, c.U0, c.U1, c.t0, i);
    const int n = sub_k(s.ka, s.kb, p.S, c.rank + 1) - sub_k(s.ka, s.kb, p.S, c.rank);
    if (n > 0) {
      c.last_run = i;
      c.nunits += n;
    }
  }
  c.xchg = false;
  if (c.nseg > 0) {
    const Seg s = seg_of(p.nk, c.U0, c.U1, c.t0, c.nseg - 1);
    c.xchg = s.ka == 0 && !seg_complete(p.S, p.nk, s);
  }
  return c;
}

// Walks this rank's units in order (segment by segment).
struct UnitIt {
  int seg, tile, k, hi;
};
__device__ __forceinline__ void unit_seek(const QmmTcParams& p, const Ctx& c, UnitIt& it, int from) {
  for (int i = from; i < c.nseg; ++i) {
    const Seg s = seg_of(p.nk, c.U0, c.U1, c.t0, i);
    const int lo = sub_k(s.ka, s.kb, p.S, c.rank), hi = sub_k(s.ka, s.kb, p.S, c.rank + 1);
    if (hi > lo) {
      it.seg = i;
      it.tile = s.tile;
      it.k = lo;
      it.hi = hi;
      return;
    }
  }
  it.seg = c.nseg;
  it.tile = -1;
  it.k = 0;
  it.hi = 0;
}
__device__ __forceinline__ void unit_next(const QmmTcParams& p, const Ctx& c, UnitIt& it) {
  if (++it.k == it.hi) unit_seek(p, c, it, it.seg + 1);
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

// One partial summed into an owned tile's slice: element (acc a, 8-row group
// g, token, row) at base + a*astride + g*gstride + token*8 + row.
struct Contrib {
  const float* base;
  uint32_t* flag;  // workspace partial: its flag; null for (distributed) shared memory
  int astride, gstride;
};

// Parked accumulator in shared memory: [acc][16 groups][TN tokens][8 rows],
// groups padded by 8 floats so that the 4 groups a warp's 32 rows span fall
// into distinct banks.
__host__ __device__ __forceinline__ int park_gstride(int TN) { return TN * 8 + 8; }

__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <int DT, int BITS, int DUAL>
__global__ void __launch_bounds__(kThreads, 1) qmm_tc_kernel(const __grid_constant__ QmmTcParams p) {
  using T = typename Elem<DT>::T;
  using WL = WLayout<BITS>;
  constexpr int NACC = DUAL ? 2 : 1;
  constexpr int TS = DUAL ? 2 : 4;  // tensor-memory A stages
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int TN = p.TN, SS = p.SS, nk = p.nk, S = p.S;
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
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_acc = abort_flag + 1;  // [2]: accumulator slot and phase of the last run
  volatile int* n_contrib = last_acc + 2;  // [kMaxPass]
  volatile int* pass_seg = n_contrib + kMaxPass;  // [kMaxPass]: segment of each owned tile, -1 past the last
  Contrib* contrib = reinterpret_cast<Contrib*>(
      smem_raw + ((reinterpret_cast<uintptr_t>(pass_seg + kMaxPass) - reinterpret_cast<uintptr_t>(smem_raw) + 15) &
                  ~uintptr_t(15)));  // [kMaxPass][kMaxContrib]
  // After the main loop the pipeline buffers hold the parked accumulator (at
  // their start) and the reduction's staging tile (at their end).
  const int area = SS * (x_stage_bytes + w_stage_bytes);
  float* park = reinterpret_cast<float*>(smem);
  const int pgs = park_gstride(TN);
  T* stg = reinterpret_cast<T*>(smem + area - TN * kStgPitch * static_cast<int>(sizeof(T)));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const Ctx cx = make_ctx(p);
  const int nunits = cx.nunits;

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
    *abort_flag = 0;
    last_acc[0] = 0;
    last_acc[1] = 0;
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

  // ---- segment epilogue: seg_load reads the accumulator slot (rows of
  // subpartition q, 32-token chunks from chunk0 in steps of cstep) and writes
  // either the fp32 partial to workspace slot pslot (pslot >= 0) or the
  // finished values to the staging area (pslot < 0); seg_publish then raises
  // the partial's flag or writes the staged tile with coalesced stores
  // (+ residual). Both run on a group of gsize threads (gt = index in the
  // group) with named barrier bar.
  const T* res = static_cast<const T*>(p.residual);
  auto seg_load = [&](int pslot, int slot, int q, int ln, int chunk0, int cstep) {
    const int r = q * 32 + ln;
    const uint32_t acc_base = tmem + (static_cast<uint32_t>(q * 32) << 16) + slot * NACC * TN;
    for (int c0 = chunk0; c0 < TN; c0 += cstep) {
      const int w = (TN - c0) < 32 ? (TN - c0) : 32;
      uint32_t v[NACC][32];
#pragma unroll
      for (int a = 0; a < NACC; ++a) {
        if (w == 32) tmem_ld32(acc_base + a * TN + c0, v[a]);
        else tmem_ld16(acc_base + a * TN + c0, v[a]);
      }
      tmem_wait_ld();
      if (pslot >= 0) {
        // fp32 partial, layout [8-row group][token][8 rows], so that a row
        // range of all tokens is contiguous; for each token a warp's store
        // covers four full 32-byte sectors
#pragma unroll
        for (int a = 0; a < NACC; ++a) {
          float* dst = p.partials + ((static_cast<long long>(cta) * kSlots + pslot) * NACC + a) * 16 * TN * 8 +
                       (r >> 3) * (TN * 8) + c0 * 8 + (r & 7);
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
  // coalesced store of rows [n_lo, n_hi) of a tile from a staging tile whose
  // rows are `pitch` elements apart (+ residual)
  auto store_rows = [&](int tile, const T* src_tile, int pitch, int n_lo, int n_hi, int gt, int gsize) {
    const TileInfo ti = tile_info(p, tile, DUAL);
    T* y = static_cast<T*>(p.y[DUAL ? 0 : ti.set]);
    const int N = p.N[DUAL ? 0 : ti.set];
    const int ldy = p.ldy[DUAL ? 0 : ti.set];
    const int n8 = (n_hi - n_lo) >> 3;
    for (int idx = gt; idx < TN * n8; idx += gsize) {
      const int tok = idx / n8, cc = idx - tok * n8;
      const int token = ti.tok0 + tok, nr = n_lo + cc * 8, n = ti.n0 + nr;
      if (token >= p.M || n >= N) continue;
      const T* src = src_tile + tok * pitch + nr;
      const long long off = static_cast<long long>(token) * ldy + n;
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
  };
  auto seg_publish = [&](int tile, int pslot, int gt, int gsize, int bar) {
    named_barrier(bar, gsize);
    if (pslot >= 0) {
      if (gt == 0) {
        __threadfence();
        st_release_gpu(&p.flags[cta * kSlots + pslot], 1u);
      }
      return;
    }
    store_rows(tile, stage_out, kBM, 0, kBM, gt, gsize);
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
      UnitIt it;
      unit_seek(p, cx, it, 0);
      uint64_t* full = is_x ? x_full : w_full + a * kMaxSS;
      const uint64_t wpol = l2_evict_first();  // weights are read once
      const int bytes = is_x ? x_stage_bytes : w_set_bytes;
      int s = 0, sph = 0;
      auto issue = [&]() {
        const TileInfo ti = tile_info(p, it.tile, DUAL);
        mbar_arrive_expect_tx(&full[s], bytes);
        if (is_x)
          tma_load_3d(xs + s * x_stage_bytes, &p.tmx, &full[s], 0, ti.tok0, it.k * 2);
        else
          tma_load_2d_hint(ws_ + s * w_stage_bytes + a * w_set_bytes, &p.tmw[DUAL ? a : ti.set], &full[s],
                           it.k * kw_per_stage, ti.n0, wpol);
        unit_next(p, cx, it);
        if (++s == SS) {
          s = 0;
          sph ^= 1;
        }
      };
      int issued = 0;
      // weights never depend on the previous kernel: their first stages are
      // issued before the grid dependency resolves
      if (is_x) griddep_wait();
      for (int i = 0; i < pre; ++i, ++issued) issue();
      for (int i = pre; i < nunits; ++i) {
        if (!mbar_wait(&s_empty[s], sph ^ 1, abort_flag, is_x ? 0x101 : 0x102)) break;
        issue();
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
    for (int sg = 0; sg < cx.nseg && ok; ++sg) {
      const Seg seg = seg_of(nk, cx.U0, cx.U1, cx.t0, sg);
      const int lo = sub_k(seg.ka, seg.kb, S, cx.rank), hi = sub_k(seg.ka, seg.kb, S, cx.rank + 1);
      if (hi <= lo) continue;
      if (!mbar_wait_warp(&acc_empty[slot], (use[slot] & 1) ^ 1, abort_flag, 0x203)) break;
      tc_fence_after();
      const uint32_t d_base = tmem + slot * NACC * TN;
      for (int j = 0; j < hi - lo; ++j) {
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
    const int gshift = p.gshift;  // log2(group)
    uint4 sc_cur = make_uint4(0, 0, 0, 0), bi_cur = sc_cur, sc_nxt = sc_cur, bi_nxt = sc_cur;
    auto load_block = [&](int tile, int gb, uint4& s_out, uint4& b_out) {
      const TileInfo ti = tile_info(p, tile, DUAL);
      const int wset = DUAL ? wg : ti.set;
      const int n = ti.n0 + r;
      const bool row_ok = n < p.N[wset];
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
    // first 8-group block of unit k, and the first unit past that block
    auto block_of = [&](int k) { return ((k * kBK) >> gshift) & ~7; };
    auto block_end = [&](int gb) { return ((gb + 8) << gshift) / kBK; };
    UnitIt it;
    unit_seek(p, cx, it, 0);
    int cur_tile = -1, cur_gb = 0, nxt_tile = -1, nxt_gb = 0;
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
      const int tile = it.tile, k = it.k;
      const int gb = block_of(k);
      if (tile != cur_tile || gb != cur_gb) {
        if (tile == nxt_tile && gb == nxt_gb) {
          sc_cur = sc_nxt;
          bi_cur = bi_nxt;
        } else {
          load_block(tile, gb, sc_cur, bi_cur);
        }
        cur_tile = tile;
        cur_gb = gb;
        // prefetch the block that follows in this rank's unit order
        const int ke = block_end(gb);
        if (ke < it.hi) {
          nxt_tile = tile;
          nxt_gb = block_of(ke);
        } else {
          UnitIt nx;
          unit_seek(p, cx, nx, it.seg + 1);
          nxt_tile = nx.tile;
          nxt_gb = nx.tile >= 0 ? block_of(nx.k) : 0;
        }
        if (nxt_tile >= 0) load_block(nxt_tile, nxt_gb, sc_nxt, bi_nxt);
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
      unit_next(p, cx, it);
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
    // Every run (non-empty segment share) but the CTA's last: the last one is
    // handled by all 16 warps once the main loop is over.
    const int q = warp & 3;
    const int et = threadIdx.x - kEpiWarp0 * 32;  // 0..127
    if (et == 0) {
      // The partials of every tile this cluster owns, in K order: this
      // cluster's ranks (parked accumulators for the last segment, workspace
      // slots for earlier ones), then the following clusters' first segments.
      // Only parameters are read, so this runs before the grid dependency.
      cg::cluster_group cluster = cg::this_cluster();
      int npass = 0;
      for (int pass = 0; pass < cx.nseg && npass < kMaxPass; ++pass) {
        const int sg = cx.xchg ? (pass == 0 ? cx.nseg - 1 : pass - 1) : pass;
        const Seg seg = seg_of(nk, cx.U0, cx.U1, cx.t0, sg);
        if (seg.ka != 0 || seg_complete(S, nk, seg)) continue;
        const bool parked = cx.xchg && sg == cx.nseg - 1;
        Contrib* list = contrib + npass * kMaxContrib;
        int n = 0;
        for (int rr = 0; rr < S; ++rr) {
          if (sub_k(seg.ka, seg.kb, S, rr + 1) <= sub_k(seg.ka, seg.kb, S, rr)) continue;
          Contrib c;
          if (parked) {
            c.base = S > 1 ? cluster.map_shared_rank(park, rr) : park;
            c.flag = nullptr;
            c.astride = 16 * pgs;
            c.gstride = pgs;
          } else {
            const int src = cx.j * S + rr;
            c.base = p.partials + (static_cast<long long>(src) * kSlots + seg_slot(sg)) * NACC * 16 * TN * 8;
            c.flag = &p.flags[src * kSlots + seg_slot(sg)];
            c.astride = 16 * TN * 8;
            c.gstride = TN * 8;
          }
          if (n < kMaxContrib) list[n] = c;
          ++n;
        }
        const long long tile_end = static_cast<long long>(seg.tile + 1) * nk;
        for (int jj = cx.j + 1; jj < p.C; ++jj) {
          const long long V0 = cluster_begin(p, jj);
          if (V0 >= tile_end) break;
          const long long V1 = cluster_begin(p, jj + 1);
          const int ka = static_cast<int>(V0 - static_cast<long long>(seg.tile) * nk);
          const int kb = V1 < tile_end ? static_cast<int>(V1 - static_cast<long long>(seg.tile) * nk) : nk;
          for (int rr = 0; rr < S; ++rr) {
            if (sub_k(ka, kb, S, rr + 1) <= sub_k(ka, kb, S, rr)) continue;
            const int src = jj * S + rr;
            Contrib c;
            c.base = p.partials + (static_cast<long long>(src) * kSlots + 0) * NACC * 16 * TN * 8;
            c.flag = &p.flags[src * kSlots + 0];
            c.astride = 16 * TN * 8;
            c.gstride = TN * 8;
            if (n < kMaxContrib) list[n] = c;
            ++n;
          }
        }
        if (n > kMaxContrib) {
          *abort_flag = 1;
          report_status(0x406);
        }
        n_contrib[npass] = n < kMaxContrib ? n : static_cast<int>(kMaxContrib);
        pass_seg[npass] = sg;
        ++npass;
      }
      for (int i = npass; i < kMaxPass; ++i) pass_seg[i] = -1;
    }
    griddep_wait();
    int use[2] = {0, 0};
    int slot = 0;
    for (int sg = 0; sg < cx.nseg; ++sg) {
      const Seg seg = seg_of(nk, cx.U0, cx.U1, cx.t0, sg);
      if (sub_k(seg.ka, seg.kb, S, cx.rank + 1) <= sub_k(seg.ka, seg.kb, S, cx.rank)) continue;
      if (sg == cx.last_run) {
        if (et == 0) {
          last_acc[0] = slot;
          last_acc[1] = use[slot] & 1;
        }
        break;
      }
      const int pslot = seg_complete(S, nk, seg) ? -1 : seg_slot(sg);
      const bool got = mbar_wait(&acc_full[slot], use[slot] & 1, abort_flag, 0x401);
      if (named_barrier_or(kEpiBar, 128, !got || *abort_flag)) break;
      tc_fence_after();
      seg_load(pslot, slot, q, lane, 0, 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[slot]);
      ++use[slot];
      slot = (slot + 1) % p.acc_slots;
      seg_publish(seg.tile, pslot, et, 128, kEpiBar);
    }
  }

  // ---- the CTA's last run, by all 16 warps: warp w reads subpartition w % 4
  // and 32-token chunk w / 4 of the accumulator
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  const bool last_xchg = cx.xchg && cx.last_run == cx.nseg - 1;
  if (cx.last_run >= 0 && !last_xchg) {
    const Seg seg = seg_of(nk, cx.U0, cx.U1, cx.t0, cx.last_run);
    const int pslot = seg_complete(S, nk, seg) ? -1 : seg_slot(cx.last_run);
    const int slot = last_acc[0];
    const bool got = mbar_wait(&acc_full[slot], static_cast<uint32_t>(last_acc[1]), abort_flag, 0x403);
    if (!named_barrier_or(kAllBar, kThreads, !got || *abort_flag)) {
      tc_fence_after();
      seg_load(pslot, slot, warp & 3, lane, (warp >> 2) * 32, 128);
      seg_publish(seg.tile, pslot, threadIdx.x, kThreads, kAllBar);
    }
  }
  // ---- the cluster's owned last segment: every CTA parks its accumulator in
  // its own shared memory, then a cluster barrier makes every CTA's parked
  // accumulator readable by the others
  if (cx.xchg) {
    if (last_xchg) {
      const int slot = last_acc[0];
      const bool got = mbar_wait(&acc_full[slot], static_cast<uint32_t>(last_acc[1]), abort_flag, 0x405);
      if (!named_barrier_or(kAllBar, kThreads, !got || *abort_flag)) {
        tc_fence_after();
        const int q = warp & 3, c0 = (warp >> 2) * 32;
        if (c0 < TN) {
          const int r = q * 32 + lane;
          float* dst = park + (r >> 3) * pgs + c0 * 8 + (r & 7);
          const int w = (TN - c0) < 32 ? (TN - c0) : 32;
          const uint32_t acc_base = tmem + (static_cast<uint32_t>(q * 32) << 16) + slot * NACC * TN;
          uint32_t v[NACC][32];
#pragma unroll
          for (int a = 0; a < NACC; ++a) {
            if (w == 32) tmem_ld32(acc_base + a * TN + c0, v[a]);
            else tmem_ld16(acc_base + a * TN + c0, v[a]);
          }
          tmem_wait_ld();
#pragma unroll
          for (int a = 0; a < NACC; ++a)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (e < w) dst[a * 16 * pgs + e * 8] = __uint_as_float(v[a][e]);
        }
      }
    }
    if (S > 1) {
      cluster_arrive_release();
      cluster_wait_acquire();
    } else {
      __syncthreads();
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

  // ---- reductions of the tiles this cluster owns: CTA r sums row slice
  // [16r/S, 16(r+1)/S) of every partial in K order (its own cluster's, then
  // the following clusters'), finishes it into the staging tile and stores it
  const int g_lo = slice_lo(S, cx.rank), g_hi = slice_lo(S, cx.rank + 1), ng = g_hi - g_lo;
  bool arrived = !(cx.xchg && S > 1);  // still owes the cluster its "done reading" arrival
  for (int pass = 0; pass < kMaxPass; ++pass) {
    const int sg = pass_seg[pass];
    if (sg < 0) break;
    const Seg seg = seg_of(nk, cx.U0, cx.U1, cx.t0, sg);
    const Contrib* list = contrib + pass * kMaxContrib;
    const int nc = n_contrib[pass];
    // wait for the workspace partials: thread c polls contribution c
    for (int c = threadIdx.x; c < nc; c += kThreads) {
      const uint32_t* f = list[c].flag;
      if (f == nullptr || ld_acquire_gpu(f) == 1u) continue;
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
    const int nit = ng * TN * 2;  // items: (group, token, 4-row half)
    for (int it = threadIdx.x; it < nit; it += kThreads) {
      const int h = it & 1, tg = it >> 1;
      const int gg = tg / TN, tok = tg - gg * TN;
      const int g = g_lo + gg;
      float acc[NACC][4];
#pragma unroll
      for (int a = 0; a < NACC; ++a) acc[a][0] = acc[a][1] = acc[a][2] = acc[a][3] = 0.f;
      // contributions in groups of 4: the group's loads (distributed shared
      // memory or L2) are all in flight before the first add, in K order
      for (int c0 = 0; c0 < nc; c0 += 4) {
        float4 v[4][NACC];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (c0 + u < nc) {
            const Contrib cb = list[c0 + u];
            const float* src = cb.base + g * cb.gstride + tok * 8 + h * 4;
#pragma unroll
            for (int a = 0; a < NACC; ++a)
              v[u][a] = cb.flag ? __ldcg(reinterpret_cast<const float4*>(src + a * cb.astride))
                                : *reinterpret_cast<const float4*>(src + a * cb.astride);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (c0 + u < nc) {
#pragma unroll
            for (int a = 0; a < NACC; ++a) {
              acc[a][0] += v[u][a].x;
              acc[a][1] += v[u][a].y;
              acc[a][2] += v[u][a].z;
              acc[a][3] += v[u][a].w;
            }
          }
        }
      }
      typename Elem<DT>::T2 o[2];
#pragma unroll
      for (int e = 0; e < 4; e += 2)
        o[e / 2] = finish2<DT, NACC>(acc[0][e], acc[0][e + 1], acc[NACC - 1][e], acc[NACC - 1][e + 1]);
      *reinterpret_cast<uint2*>(stg + tok * kStgPitch + g * 8 + h * 4) = *reinterpret_cast<const uint2*>(o);
    }
    __syncthreads();
    if (!arrived) {
      // every parked accumulator this CTA reads has been read
      cluster_arrive_relaxed();
      arrived = true;
    }
    store_rows(seg.tile, stg, kStgPitch, g_lo * 8, g_hi * 8, threadIdx.x, kThreads);
    __syncthreads();  // staging is reused by the next tile
    if (threadIdx.x == 0) {
      bool any = false;
      for (int c = 0; c < nc; ++c) any = any || list[c].flag != nullptr;
      if (any) {
        const uint32_t prev = atomicAdd(&p.done[seg.tile], 1u);
        if (prev == static_cast<uint32_t>(S - 1)) {
          // every owner CTA has read every partial of this tile: clear for the next call
          for (int c = 0; c < nc; ++c)
            if (list[c].flag) *list[c].flag = 0u;
          p.done[seg.tile] = 0u;
        }
      }
    }
  }
  // no CTA of the cluster leaves while another may still read its parked accumulator
  if (cx.xchg && S > 1) {
    if (!arrived) cluster_arrive_relaxed();
    cluster_wait_acquire();
  }
}

// ------------------------------------------------------------------- host

static size_t smem_bytes_for(int TN, int SS, int bits, int dual) {
  const int nacc = dual ? 2 : 1;
  const size_t stage = static_cast<size_t>(TN) * 256 + static_cast<size_t>(nacc) * kBM * (kBK * bits / 8);
  const size_t b = 1024 + SS * stage + stage_bytes_for(TN) + 2048;
  // at least half an SM's shared memory: one CTA per SM, so a CTA never waits
  // for tensor memory held by another CTA of the grid on the same SM
  return b < 120 * 1024 ? 120 * 1024 : b;
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

static WsLayout ws_layout(int P, int nacc, int TN) {
  WsLayout l;
  l.flags = kWsQmmFlags;
  l.done = kWsQmmDone;
  l.partials = kWsCtlBytes;
  l.total = l.partials + static_cast<size_t>(P) * kSlots * nacc * 16 * TN * 8 * 4;
  return l;
}

size_t qmm_tc_workspace(int64_t M, int64_t n_total, int64_t K, int bits, int kind) {
  (void)bits;
  (void)K;
  (void)n_total;
  const int dual = kind == 1;
  return ws_layout(kMaxP, dual ? 2 : 1, tile_tn(M)).total;
}

// Partition of U = tiles * nk units over C clusters of S CTAs, with what the
// kernel needs to hold: the largest units per CTA, the segments per cluster,
// the partials summed into one tile, and whether some cluster lies wholly
// inside a tile (its partial is then written only at the end of its range,
// and the owner waits for it).
struct PlanStats {
  int max_units, max_seg, max_contrib;
  int max_pass;    // owned tiles reduced by one cluster
  int max_global;  // workspace partials summed into one tile
  bool late;       // some tile waits for a partial written at the end of a range
  bool mid;        // some CTA writes a workspace partial before its last run
};

static PlanStats plan_stats(const QmmTcParams& p) {
  PlanStats st = {0, 0, 0, 0, 0, false, false};
  std::vector<int> contrib(static_cast<size_t>(p.tiles), 0), global(static_cast<size_t>(p.tiles), 0);
  for (int j = 0; j < p.C; ++j) {
    const long long U0 = cluster_begin(p, j), U1 = cluster_begin(p, j + 1);
    if (U1 <= U0) continue;
    const int t0 = static_cast<int>(U0 / p.nk);
    const int nseg = static_cast<int>((U1 - 1) / p.nk) - t0 + 1;
    if (nseg > st.max_seg) st.max_seg = nseg;
    if (nseg == 1 && U0 % p.nk != 0) st.late = true;
    const Seg last = seg_of(p.nk, U0, U1, t0, nseg - 1);
    const bool xchg = last.ka == 0 && !seg_complete(p.S, p.nk, last);
    int passes = 0;
    for (int i = 0; i < nseg; ++i) {
      const Seg s = seg_of(p.nk, U0, U1, t0, i);
      if (s.ka == 0 && !seg_complete(p.S, p.nk, s)) ++passes;
      if (i < nseg - 1 && !seg_complete(p.S, p.nk, s)) st.mid = true;
    }
    if (passes > st.max_pass) st.max_pass = passes;
    for (int r = 0; r < p.S; ++r) {
      int u = 0;
      for (int i = 0; i < nseg; ++i) {
        const Seg s = seg_of(p.nk, U0, U1, t0, i);
        const int n = sub_k(s.ka, s.kb, p.S, r + 1) - sub_k(s.ka, s.kb, p.S, r);
        u += n;
        if (n > 0 && !seg_complete(p.S, p.nk, s)) {
          ++contrib[static_cast<size_t>(s.tile)];
          if (!(xchg && i == nseg - 1)) ++global[static_cast<size_t>(s.tile)];
        }
      }
      if (u > st.max_units) st.max_units = u;
    }
  }
  for (size_t t = 0; t < contrib.size(); ++t) {
    if (contrib[t] > st.max_contrib) st.max_contrib = contrib[t];
    if (global[t] > st.max_global) st.max_global = global[t];
  }
  return st;
}

// Host mirror of the kernel's partition bookkeeping (the same seg_of /
// sub_k / seg_complete / seg_slot / cluster_begin the kernel runs): which CTA
// computes which K-stages, where each partial goes, and which cluster reduces
// which tile from which partials, checked for exact coverage.
static int partition_check(long long tiles, int nk, int S, int C, long long* max_units) {
  if (tiles < 1 || nk < 1 || S < 1 || S > kMaxS || C < 1 || static_cast<long long>(C) * S > kMaxP ||
      (S > 1 && S > nk)) {
    set_error("qmm partition: bad shape tiles=%lld nk=%d S=%d C=%d", tiles, nk, S, C);
    return MT_ERR_INVALID_ARGUMENT;
  }
  QmmTcParams p;
  memset(&p, 0, sizeof(p));
  p.nk = nk;
  p.S = S;
  p.C = C;
  p.units = tiles * nk;
  p.c_magic = C > 1 ? ~0ull / static_cast<uint64_t>(C) + 1 : 0;
  const int P = C * S;
  std::vector<std::vector<int>> cover(static_cast<size_t>(tiles));  // K-stages computed, per tile
  std::vector<int> written(static_cast<size_t>(P) * kSlots, -1);    // tile of each (CTA, slot) partial
  std::vector<int> read(static_cast<size_t>(P) * kSlots, 0);
  std::vector<int> owners(static_cast<size_t>(tiles), 0);
  long long mu = 0;
  auto fail = [&](const char* what, long long a, long long b) {
    set_error("qmm partition (tiles=%lld nk=%d S=%d C=%d): %s (%lld, %lld)", tiles, nk, S, C, what, a, b);
    return MT_ERR_INVALID_ARGUMENT;
  };
  // what every CTA computes and where its partials go
  for (int j = 0; j < C; ++j) {
    const long long U0 = cluster_begin(p, j), U1 = cluster_begin(p, j + 1);
    if (U1 <= U0) continue;
    const int t0 = static_cast<int>(U0 / nk);
    const int nseg = static_cast<int>((U1 - 1) / nk) - t0 + 1;
    if (S > 1 && nseg > kMaxSegK) return fail("segments per cluster", j, nseg);
    const Seg last = seg_of(nk, U0, U1, t0, nseg - 1);
    const bool xchg = last.ka == 0 && !seg_complete(S, nk, last);
    for (int r = 0; r < S; ++r) {
      long long u = 0;
      for (int i = 0; i < nseg; ++i) {
        const Seg s = seg_of(nk, U0, U1, t0, i);
        const int lo = sub_k(s.ka, s.kb, S, r), hi = sub_k(s.ka, s.kb, S, r + 1);
        if (hi <= lo) continue;
        u += hi - lo;
        for (int k = lo; k < hi; ++k) cover[static_cast<size_t>(s.tile)].push_back(k);
        if (seg_complete(S, nk, s) || (xchg && i == nseg - 1)) continue;
        const size_t slot = static_cast<size_t>(j * S + r) * kSlots + seg_slot(i);
        if (written[slot] >= 0) return fail("partial slot written twice", j * S + r, seg_slot(i));
        written[slot] = s.tile;
      }
      if (u > mu) mu = u;
    }
  }
  // what every owner reduces, in the order the kernel sums it
  for (int j = 0; j < C; ++j) {
    const long long U0 = cluster_begin(p, j), U1 = cluster_begin(p, j + 1);
    if (U1 <= U0) continue;
    const int t0 = static_cast<int>(U0 / nk);
    const int nseg = static_cast<int>((U1 - 1) / nk) - t0 + 1;
    const Seg last = seg_of(nk, U0, U1, t0, nseg - 1);
    const bool xchg = last.ka == 0 && !seg_complete(S, nk, last);
    for (int i = 0; i < nseg; ++i) {
      const Seg s = seg_of(nk, U0, U1, t0, i);
      if (seg_complete(S, nk, s)) {
        ++owners[static_cast<size_t>(s.tile)];
        continue;
      }
      if (s.ka != 0) continue;
      ++owners[static_cast<size_t>(s.tile)];
      int kpos = 0;  // the sum runs in K order
      for (int r = 0; r < S; ++r) {
        const int lo = sub_k(s.ka, s.kb, S, r), hi = sub_k(s.ka, s.kb, S, r + 1);
        if (hi <= lo) continue;
        if (lo != kpos) return fail("owner's own partials out of K order", s.tile, lo);
        kpos = hi;
        if (xchg && i == nseg - 1) continue;
        const size_t slot = static_cast<size_t>(j * S + r) * kSlots + seg_slot(i);
        if (written[slot] != s.tile) return fail("owner reads a slot holding another tile", s.tile, written[slot]);
        ++read[slot];
      }
      const long long tile_end = static_cast<long long>(s.tile + 1) * nk;
      for (int jj = j + 1; jj < C; ++jj) {
        const long long V0 = cluster_begin(p, jj);
        if (V0 >= tile_end) break;
        const long long V1 = cluster_begin(p, jj + 1);
        const int ka = static_cast<int>(V0 - static_cast<long long>(s.tile) * nk);
        const int kb = V1 < tile_end ? static_cast<int>(V1 - static_cast<long long>(s.tile) * nk) : nk;
        for (int r = 0; r < S; ++r) {
          const int lo = sub_k(ka, kb, S, r), hi = sub_k(ka, kb, S, r + 1);
          if (hi <= lo) continue;
          if (lo != kpos) return fail("following partials out of K order", s.tile, lo);
          kpos = hi;
          const size_t slot = static_cast<size_t>(jj * S + r) * kSlots;
          if (written[slot] != s.tile) return fail("owner reads a following slot holding another tile", s.tile,
                                                   written[slot]);
          ++read[slot];
        }
      }
      if (kpos != nk) return fail("owner's sum does not reach the tile's last K-stage", s.tile, kpos);
    }
  }
  for (long long t = 0; t < tiles; ++t) {
    std::vector<int>& c = cover[static_cast<size_t>(t)];
    std::sort(c.begin(), c.end());
    if (static_cast<int>(c.size()) != nk) return fail("K-stages computed for a tile", t, static_cast<long long>(c.size()));
    for (int k = 0; k < nk; ++k)
      if (c[static_cast<size_t>(k)] != k) return fail("K-stage computed twice or never", t, k);
    if (owners[static_cast<size_t>(t)] != 1) return fail("owners of a tile", t, owners[static_cast<size_t>(t)]);
  }
  for (size_t i = 0; i < written.size(); ++i)
    if (written[i] >= 0 && read[i] != 1) return fail("partial read by its owner", static_cast<long long>(i), read[i]);
  if (max_units) *max_units = mu;
  return MT_OK;
}

template <int DT, int BITS, int DUAL>
static int launch_tc(QmmTcParams& p, size_t smem, int sms, cudaStream_t stream) {
  auto k = qmm_tc_kernel<DT, BITS, DUAL>;
  if (int e = ensure_smem(k, kSmemLimit)) return e;
  // resident clusters of each size for this shared-memory footprint
  // (queried once per kernel, size and footprint)
  static int occ[kMaxS + 1] = {};
  static size_t occ_smem[kMaxS + 1] = {};
  // Plan: the (S, C) with the least estimated time, from the largest units
  // per CTA (t_u each) and a tail that is short when every late partial is
  // reduced inside its cluster. Estimates in microseconds from measurements
  // of this kernel on B200.
  const double t_u = DUAL ? 1.2 : 0.8;
  // the parked accumulator and the reduction staging tile must fit the
  // pipeline buffers
  const size_t area = static_cast<size_t>(p.SS) *
                      (static_cast<size_t>(p.TN) * 256 + (DUAL ? 2 : 1) * kBM * (kBK * BITS / 8));
  const bool fits = static_cast<size_t>(DUAL ? 2 : 1) * 16 * park_gstride(p.TN) * 4 +
                        static_cast<size_t>(p.TN) * kStgPitch * 2 <= area;
  if (!fits) {
    set_error("qmm: pipeline buffers (%zu B) too small for the reduction", area);
    return MT_ERR_UNSUPPORTED;
  }
  double best = 1e30;
  int bS = 1, bC = static_cast<int>(p.units < sms ? p.units : sms);
  const int cand_s[] = {1, 2, 3, 4, 6, 8};
  for (int S : cand_s) {
    if (S > 1 && S > p.nk) continue;
    int maxc = sms;
    if (S > 1) {
      if (occ_smem[S] != smem) {
        int n = 0;
        if (int e = max_active_clusters(k, kThreads, smem, S, &n)) return e;
        occ[S] = n;
        occ_smem[S] = smem;
      }
      maxc = occ[S];
    }
    if (maxc < 1) continue;
    int cands[2] = {maxc, p.tiles};
    for (int ci = 0; ci < 2; ++ci) {
      long long C = cands[ci];
      if (C > maxc) continue;
      if (S == 1) C = p.units < sms ? p.units : sms;
      if (C < 1 || C * S > kMaxP) continue;
      QmmTcParams q = p;
      q.S = S;
      q.C = static_cast<int>(C);
      q.c_magic = C > 1 ? ~0ull / static_cast<uint64_t>(C) + 1 : 0;
      const PlanStats st = plan_stats(q);
      if (S > 1 && st.max_seg > kMaxSegK) continue;
      if (st.max_contrib > kMaxContrib) continue;
      // The tail: parking, exchange and reduction, which grows with the
      // ranks read per row slice; every reduced tile beyond the first costs
      // another pass over its partials, every workspace partial L2 traffic,
      // and a dual kernel's accumulator drained mid-run stalls its MMAs.
      // Fitted to this kernel's measured times on B200 (Qwen3-4B shapes).
      // A cluster range lying inside one tile writes its partial only at its
      // end, and that tile's owner waits for it.
      const double tail = (S == 1 ? 6.0 : S == 2 ? 7.0 : S == 3 ? 6.5 : S == 4 ? 7.5 : S == 6 ? 10.5 : 12.0) +
                          (st.late ? 5.0 : 0.0);
      const double cost = t_u * st.max_units + tail + 3.0 * (st.max_pass > 1 ? st.max_pass - 1 : 0) +
                          0.4 * st.max_global + (DUAL && st.mid ? 2.0 : 0.0);
      if (cost < best) {
        best = cost;
        bS = S;
        bC = static_cast<int>(C);
      }
    }
  }
  if (best >= 1e29) {
    set_error("qmm: no cluster plan for %lld units (%d tiles x %d)", p.units, p.tiles, p.nk);
    return MT_ERR_UNSUPPORTED;
  }
  p.S = bS;
  p.C = bC;
  p.c_magic = bC > 1 ? ~0ull / static_cast<uint64_t>(bC) + 1 : 0;
  return launch_cluster(k, dim3(static_cast<unsigned>(bS * bC)), dim3(kThreads), smem, bS, stream, p);
}

int qmm_tc_run(const QmmRequest& r, cudaStream_t stream) {
  const int dual = r.kind == QMM_SWIGLU ? 1 : 0;
  const int esz = 2;
  MT_CHECK_ARG(r.K % 64 == 0, "qmm: K=%lld must be a multiple of 64", (long long)r.K);
  MT_CHECK_ARG(aligned(r.x, 16), "qmm: x must be 16-byte aligned");
  int sms = 148;
  int rc = device_sm_count(&sms);
  if (rc != MT_OK) return rc;
  if (sms > kMaxP) sms = kMaxP;

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
    p.ldy[s] = static_cast<int>(q.ldy > 0 ? q.ldy : q.N);
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
      if (q.y && (!aligned(q.y, 16) || q.N % 8 != 0 || p.ldy[s] % 8 != 0)) vec = false;
    }
    p.tile_start[s + 1] = ftiles;
  }
  if (dual) {
    ftiles = static_cast<int>((r.set[0].N + kBM - 1) / kBM);
    p.N[1] = p.N[0];
    p.ldy[1] = p.ldy[0];
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
  if (p.units >= (1ll << 28)) {
    set_error("qmm: %lld K-stage units exceed the 2^28 the unit arithmetic supports", p.units);
    return MT_ERR_UNSUPPORTED;
  }
  if (static_cast<size_t>(p.tiles) > kWsQmmMaxTiles) {
    set_error("qmm: %d tiles exceed the workspace's %zu tile counters (M=%lld too large for one call)", p.tiles,
              kWsQmmMaxTiles, (long long)r.M);
    return MT_ERR_UNSUPPORTED;
  }
  const WsLayout wl = ws_layout(kMaxP, dual ? 2 : 1, p.TN);
  if (!r.ws || r.ws_bytes < wl.total || !aligned(r.ws, 256)) {
    set_error("qmm: workspace of %zu bytes (256-aligned, zero-filled) required, got %zu", wl.total,
              r.ws ? r.ws_bytes : (size_t)0);
    return MT_ERR_WORKSPACE;
  }
  uint8_t* ws = static_cast<uint8_t*>(r.ws);
  p.flags = reinterpret_cast<uint32_t*>(ws + wl.flags);
  p.done = reinterpret_cast<uint32_t*>(ws + wl.done);
  p.partials = reinterpret_cast<float*>(ws + wl.partials);

  const size_t smem = smem_bytes_for(p.TN, p.SS, r.bits, dual);
  const bool bf = r.dtype == MT_BF16;
  if (dual) {
    if (bf) return r.bits == 4 ? launch_tc<MT_BF16, 4, 1>(p, smem, sms, stream) : launch_tc<MT_BF16, 8, 1>(p, smem, sms, stream);
    return r.bits == 4 ? launch_tc<MT_F16, 4, 1>(p, smem, sms, stream) : launch_tc<MT_F16, 8, 1>(p, smem, sms, stream);
  }
  if (bf) return r.bits == 4 ? launch_tc<MT_BF16, 4, 0>(p, smem, sms, stream) : launch_tc<MT_BF16, 8, 0>(p, smem, sms, stream);
  return r.bits == 4 ? launch_tc<MT_F16, 4, 0>(p, smem, sms, stream) : launch_tc<MT_F16, 8, 0>(p, smem, sms, stream);
}

}  // namespace mt

extern "C" int mt_qmm_partition_check(int64_t tiles, int nk, int cluster_size, int clusters, int64_t* max_units_out) {
  mt::clear_error();
  long long mu = 0;
  const int rc = mt::partition_check(tiles, nk, cluster_size, clusters, &mu);
  if (rc == MT_OK && max_units_out) *max_units_out = mu;
  return rc;
}
