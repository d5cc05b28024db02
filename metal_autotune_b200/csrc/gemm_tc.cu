// Dense 16-bit GEMM and implicit-GEMM conv1d on the 5th-generation tensor
// cores (tcgen05 + TMA + tensor memory), for the GELU-MLP linears and the
// conv stem (mx.addmm / nn.Linear, mx.conv1d + bias + GELU).
//
//   y[(b, t), n] = epilogue( sum over taps j, channels c of
//                            x[b, t*stride + j - pad, c] * w[n, j, c] )
//
// A linear is the one-tap case (b = 0, t = row, stride 1, pad 0). x is
// channels-last [B, L, Cin], w is [Cout, taps, Cin] (mlx layouts), y is
// [B, Lout, Cout] with row pitch ldy.
//
// Tiles: 128 output rows (t) x BN output columns (n), BN = 128 or 256, one
// persistent CTA per SM walking the tiles in groups of 8 row tiles per
// column sweep (the row tiles of a group share the weight tiles in L2). The
// reduction runs in K-blocks of 64 channels of one tap, each one TMA copy
// of the x tile and one of the weight tile into a 4-stage shared-memory ring
// (128-byte swizzle). The x copy addresses the input through a 3-D tensor
// map (channels*v, L/v, B) with v = stride: output row t of tap j reads view
// row t + floor((j - pad)/v) at channel offset ((j - pad) mod v)*Cin, so a
// stride-2 conv needs no gather and the zero padding at both ends is the
// copy's out-of-range fill (a negative row coordinate reads zeros).
//
// Roles (320 threads): warp 0 issues the TMA copies; warp 1 owns the tensor
// memory (two BN-column fp32 accumulators) and one elected lane issues
// tcgen05.mma.kind::f16 (M = 128, N = BN, K = 16; both operands from shared
// memory); warps 2-9 are the epilogue: each reads 32 accumulator rows of
// every other 32-column chunk from tensor memory (tcgen05.ld), rounds as the
// MLX ops would, and stores, while the MMAs of the next tile run into the
// other accumulator. GELU here uses the branch-free erf of gelu_as_f32.
//
// Epilogue rounding (element type T = bf16 or f16):
//   conv   (bias_fused = 0): round(acc), + bias -> round, GELU -> round
//   linear (bias_fused = 1): round(acc + bias) (mx.addmm: one rounding),
//                            GELU -> round
//   residual (optional):     + residual -> round
//
// Every mbarrier wait is bounded (2 s); on expiry the CTA records a site code
// in the device status word, stops issuing, drains its in-flight copies and
// MMAs (bounded) and frees its tensor memory.
#include "mt_common.cuh"
#include "mt_tma.h"
#include "qmm_common.cuh"

namespace mt {

constexpr int kGtBM = 128;
constexpr int kGtBK = 64;
constexpr int kGtStages = 4;
constexpr int kGtThreads = 320;
constexpr int kGtEpiWarps = 8;  // two per tensor-memory lane quadrant
constexpr int kGtGroup = 8;  // row tiles per column sweep
constexpr int kGtMaxTaps = 4;

struct GemmTcParams {
  CUtensorMap tma_x;  // (Cin*v, L/v, B), box (64, 128, 1)
  CUtensorMap tma_w;  // (taps*Cin, Cout), box (64, BN)
  const void* bias;
  const void* residual;
  void* y;
  long long ldy;       // y / residual row pitch in elements
  int B, Lout, Cin, Cout, taps, kb_per_tap;
  int dr[kGtMaxTaps];  // view-row offset of each tap
  int dc[kGtMaxTaps];  // channel offset of each tap
  int mt_per_b, num_mt, num_nt, tiles;
  int bias_fused, vec;
  int Nout;  // SwiGLU form: output columns (the weight rows are gate/up blocks of 128)
};

template <int BN>
struct GtSmem {
  static constexpr int kA = kGtBM * kGtBK * 2;  // 16 KB
  static constexpr int kB = BN * kGtBK * 2;     // 16 / 32 KB
  static constexpr int kStage = kA + kB;
  static constexpr int kBars = 1024;            // barriers and flags after the ring
  static constexpr int kTotal = kGtStages * kStage + kBars + 1024;  // + alignment slack
};

struct GtTile {
  int b, t0, n0;
};

__device__ __forceinline__ GtTile gt_tile(const GemmTcParams& p, int id) {
  const int span = kGtGroup * p.num_nt;
  const int group = id / span;
  const int first = group * kGtGroup;
  const int gsz = min(kGtGroup, p.num_mt - first);
  const int in = id - group * span;
  const int m = first + in % gsz;
  GtTile t;
  t.n0 = in / gsz;  // column tile index
  t.b = m / p.mt_per_b;
  t.t0 = (m - t.b * p.mt_per_b) * kGtBM;
  return t;
}

// The epilogue of one accumulator: the calling warp's 32 tensor-memory lanes
// (tacc: lane quadrant and accumulator column already added), every other
// 32-column chunk from `half`; output row pitch offset yrow, first output
// column col0. Rounds as the MLX ops would and stores (16-byte pieces when a
// chunk is whole).
template <int DT, int BN, int ACT>
__device__ __forceinline__ void gt_store_tile(const GemmTcParams& p, uint32_t tacc, int half, bool live,
                                              long long yrow, int col0) {
  using T = typename Elem<DT>::T;
  const T* bias = static_cast<const T*>(p.bias);
  const T* res = static_cast<const T*>(p.residual);
  T* y = static_cast<T*>(p.y);
  // SwiGLU form (ACT 2, BN 256): columns [0, 128) of a tile are gate rows,
  // [128, 256) the up rows of the same 128 outputs
  constexpr int kChunks = ACT == 2 ? 4 : BN / 32;
  const int ncol = ACT == 2 ? p.Nout : p.Cout;
#pragma unroll 1
  for (int ch = half; ch < kChunks; ch += 2) {
    uint32_t r[32];
    __syncwarp();  // tcgen05.ld is .sync.aligned: the whole warp, converged
    tmem_ld32(tacc + ch * 32, r);
    uint32_t r2[ACT == 2 ? 32 : 1];
    if constexpr (ACT == 2) tmem_ld32(tacc + 128 + ch * 32, r2);
    tmem_wait_ld();
    const int n0 = col0 + ch * 32;
    if (!live || n0 >= ncol) continue;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
    if constexpr (ACT == 2) {
      // silu(gate) * up on the rounded products, each op rounded
#pragma unroll
      for (int i = 0; i < 32; ++i)
        v[i] = round_to<DT>(swiglu_rounded<DT>(round_to<DT>(v[i]), round_to<DT>(__uint_as_float(r2[i]))));
    }
    // bias, in 16-byte pieces when the chunk is whole
    float bv[32];
    if (bias) {
      if (p.vec && n0 + 32 <= ncol) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 u = *reinterpret_cast<const uint4*>(bias + n0 + 8 * q);
          const typename Elem<DT>::T2* h = reinterpret_cast<const typename Elem<DT>::T2*>(&u);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = Elem<DT>::unpack2(h[e]);
            bv[8 * q + 2 * e] = f.x;
            bv[8 * q + 2 * e + 1] = f.y;
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) bv[i] = n0 + i < ncol ? Elem<DT>::to_f(bias[n0 + i]) : 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float u;
      if (p.bias_fused)
        u = round_to<DT>(bias ? v[i] + bv[i] : v[i]);
      else
        u = bias ? round_to<DT>(round_to<DT>(v[i]) + bv[i]) : round_to<DT>(v[i]);
      if (ACT == 1) u = round_to<DT>(gelu_as_f32(u));
      if (ACT == 2) u = v[i];
      v[i] = u;
    }
    if (res) {
      if (p.vec && n0 + 32 <= ncol) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 u = *reinterpret_cast<const uint4*>(res + yrow + n0 + 8 * q);
          const typename Elem<DT>::T2* h = reinterpret_cast<const typename Elem<DT>::T2*>(&u);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = Elem<DT>::unpack2(h[e]);
            v[8 * q + 2 * e] = round_to<DT>(v[8 * q + 2 * e] + f.x);
            v[8 * q + 2 * e + 1] = round_to<DT>(v[8 * q + 2 * e + 1] + f.y);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (n0 + i < ncol) v[i] = round_to<DT>(v[i] + Elem<DT>::to_f(res[yrow + n0 + i]));
      }
    }
    if (p.vec && n0 + 32 <= ncol) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 u;
        typename Elem<DT>::T2* h = reinterpret_cast<typename Elem<DT>::T2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) h[e] = Elem<DT>::pack2(v[8 * q + 2 * e], v[8 * q + 2 * e + 1]);
        *reinterpret_cast<uint4*>(y + yrow + n0 + 8 * q) = u;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (n0 + i < ncol) y[yrow + n0 + i] = Elem<DT>::from_f(v[i]);
    }
  }
}

template <int DT, int BN, int ACT>
__global__ void __launch_bounds__(kGtThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmTcParams p) {
  using T = typename Elem<DT>::T;
  using S = GtSmem<BN>;
  extern __shared__ uint8_t gt_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gt_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kGtStages * S::kStage);
  uint64_t* full = bars;                       // [stages]
  uint64_t* empty = bars + kGtStages;          // [stages]
  uint64_t* acc_full = bars + 2 * kGtStages;   // [2]
  uint64_t* acc_empty = acc_full + 2;          // [2]
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kGtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kGtEpiWarps);  // one arrive per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tma_x);
    prefetch_tmap(&p.tma_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  griddep_launch();

  const int kblocks = p.taps * p.kb_per_tap;
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    int s = 0, ph = 0;
    long long issued = 0;
    bool ok = true;
    for (int id = blockIdx.x; id < p.tiles && ok; id += gridDim.x) {
      const GtTile tl = gt_tile(p, id);
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait_warp(&empty[s], ph ^ 1, abort_flag, 0x601)) {
          ok = false;
          break;
        }
        if (elect_one()) {
          const int j = kb / p.kb_per_tap;
          const int c = (kb - j * p.kb_per_tap) * kGtBK;
          uint8_t* a = ring + s * S::kStage;
          mbar_arrive_expect_tx(&full[s], S::kStage);
          tma_load_3d(a, &p.tma_x, &full[s], c + p.dc[j], tl.t0 + p.dr[j], tl.b);
          tma_load_2d(a + S::kA, &p.tma_w, &full[s], j * p.Cin + c, tl.n0 * BN);
        }
        __syncwarp();
        ++issued;
        if (++s == kGtStages) {
          s = 0;
          ph ^= 1;
        }
      }
    }
    if (!ok) {  // let the copies already issued land before the CTA exits
      const long long first = issued > kGtStages ? issued - kGtStages : 0;
      for (long long i = first; i < issued; ++i)
        mbar_wait_drain(&full[i % kGtStages], static_cast<uint32_t>((i / kGtStages) & 1), 200000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = idesc_f16(kGtBM, BN, DT == MT_BF16);
    const uint64_t ring_desc = smem_desc_k_sw128(smem_addr(ring));
    const uint32_t stage_step = S::kStage >> 4, b_off = S::kA >> 4;
    int s = 0, ph = 0, buf = 0;
    int use[2] = {0, 0};
    bool ok = true, issued = false;
    for (int id = blockIdx.x; id < p.tiles && ok; id += gridDim.x) {
      if (!mbar_wait_warp(&acc_empty[buf], (use[buf] & 1) ^ 1, abort_flag, 0x602)) break;
      tc_fence_after();
      const uint32_t d = tmem + buf * BN;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait_warp(&full[s], ph, abort_flag, 0x603)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = ring_desc + s * stage_step;
        const uint64_t bd = ad + b_off;
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < kGtBK / 16; ++kk)
            tc_mma_ss(d, ad + 2 * kk, bd + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&empty[s]);
        }
        __syncwarp();
        issued = true;
        if (++s == kGtStages) {
          s = 0;
          ph ^= 1;
        }
      }
      if (!ok) break;
      if (elect_one()) tc_commit(&acc_full[buf]);
      __syncwarp();
      ++use[buf];
      buf ^= 1;
    }
    if (__any_sync(0xffffffffu, *abort_flag != 0) && issued) {
      if (elect_one()) {
        tc_commit(drain);
        mbar_wait_drain(drain, 0, 200000000ull);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // warps 2-9: warp w reads tensor-memory lanes [32*(w%4), +32) (the lane
    // quadrant its warp index allows) and every other 32-column chunk, the
    // pair of warps of a quadrant splitting the columns between them
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quad * 32 + lane;
    int buf = 0;
    int use[2] = {0, 0};
    for (int id = blockIdx.x; id < p.tiles; id += gridDim.x) {
      const GtTile tl = gt_tile(p, id);
      if (!mbar_wait_warp(&acc_full[buf], use[buf] & 1, abort_flag, 0x604)) break;
      tc_fence_after();
      const int t = tl.t0 + row;
      const bool live = t < p.Lout;
      const long long yrow = (static_cast<long long>(tl.b) * p.Lout + t) * p.ldy;
      gt_store_tile<DT, BN, ACT>(p, tmem + (static_cast<uint32_t>(quad * 32) << 16) + buf * BN, half, live, yrow,
                                 ACT == 2 ? tl.n0 * 128 : tl.n0 * BN);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      ++use[buf];
      buf ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 2 * BN);
}

// ------------------------------------------------------------ CTA pairs
// The same product on pairs of SMs (tcgen05 cta_group::2). A cluster of two
// CTAs computes a 256 x 256 output tile with M = 256 MMAs issued by its even
// CTA. Per K-block each CTA stages its own 128 rows of x and its own 128
// weight rows (half of the tile's columns; the pair's tensor cores share the
// two halves): 32 KB per SM, where the single-SM 128 x 256 tile stages 48 KB
// for the same MMA work, so a 6-stage ring fits in place of 4. Each CTA's
// tensor memory holds its 128 output rows x 256 columns, which its own
// epilogue warps store exactly as above.
//
// Barriers. The copies of both CTAs complete on the even CTA's full[s] (its
// producer expects both CTAs' bytes). The even CTA's MMA issuer commits each
// stage to empty[s] of both CTAs and each accumulator to acc_full[buf] of
// both. The epilogue warps of both CTAs arrive on the even CTA's
// acc_empty[buf]. A wait that gives up also raises the peer's abort flag.
constexpr int kGpStages = 6;
constexpr int kGpRows = 256;  // output rows of a pair tile
constexpr int kGpGroup = 4;   // pair row tiles per column sweep (1024 rows, as above)

struct GpSmem {
  static constexpr int kA = 128 * kGtBK * 2;  // 16 KB: this CTA's rows of x
  static constexpr int kB = 128 * kGtBK * 2;  // 16 KB: this CTA's weight rows
  static constexpr int kStage = kA + kB;
  static constexpr int kBars = 1024;
  static constexpr int kTotal = kGpStages * kStage + kBars + 1024;  // + alignment slack
};

namespace {
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of the same shared-memory offset in CTA `cta`.
__device__ __forceinline__ uint32_t map_to_cta(uint32_t saddr, uint32_t cta) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(cta));
  return d;
}
__device__ __forceinline__ void pair_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Arrive on the mbarrier at shared::cluster address `bar` once the pair's
// earlier MMAs issued by this thread have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// TMA tile copies into this CTA's shared memory completing on the mbarrier at
// shared::cluster address `bar`, which may be the peer CTA's.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
      "l"(map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int x, int y,
                                                 int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_addr(dst)),
      "l"(map), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void raise_peer_abort(volatile int* flag, uint32_t peer) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(map_to_cta(smem_addr(const_cast<int*>(flag)), peer)),
               "r"(1)
               : "memory");
}
}  // namespace

__device__ __forceinline__ GtTile gp_tile(const GemmTcParams& p, int id) {
  const int span = kGpGroup * p.num_nt;
  const int group = id / span;
  const int first = group * kGpGroup;
  const int gsz = min(kGpGroup, p.num_mt - first);
  const int in = id - group * span;
  const int m = first + in % gsz;
  GtTile t;
  t.n0 = in / gsz;
  t.b = m / p.mt_per_b;
  t.t0 = (m - t.b * p.mt_per_b) * kGpRows;
  return t;
}

// p.mt_per_b / p.num_mt count 256-row pair tiles; the weight map's box is 128 rows.
template <int DT, int ACT>
__global__ void __launch_bounds__(kGtThreads, 1) gemm_tc_pair_kernel(const __grid_constant__ GemmTcParams p) {
  using S = GpSmem;
  constexpr int BN = 256;
  extern __shared__ uint8_t gp_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gp_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kGpStages * S::kStage);
  uint64_t* full = bars;                      // [stages], used in the even CTA
  uint64_t* empty = bars + kGpStages;         // [stages]
  uint64_t* acc_full = bars + 2 * kGpStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;         // [2], used in the even CTA
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0 issues the MMAs
  const uint32_t peer = rank ^ 1u;
  const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kGpStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * kGtEpiWarps);  // one arrive per epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tma_x);
    prefetch_tmap(&p.tma_w);
  }
  if (warp == 1) {  // the same warp of both CTAs allocates the pair's columns
    tmem_alloc_pair(tmem_slot, 2 * BN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  pair_barrier();  // both CTAs' barriers exist before either signals the other
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  griddep_launch();

  const int kblocks = p.taps * p.kb_per_tap;
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    int s = 0, ph = 0;
    long long issued = 0;
    bool ok = true;
    for (int id = pair; id < p.tiles && ok; id += npairs) {
      const GtTile tl = gp_tile(p, id);
      const int trow = tl.t0 + 128 * static_cast<int>(rank);
      const int wrow = tl.n0 * BN + 128 * static_cast<int>(rank);
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait_warp(&empty[s], ph ^ 1, abort_flag, 0x611)) {
          ok = false;
          break;
        }
        if (elect_one()) {
          const int j = kb / p.kb_per_tap;
          const int c = (kb - j * p.kb_per_tap) * kGtBK;
          uint8_t* a = ring + s * S::kStage;
          const uint32_t fb = map_to_cta(smem_addr(&full[s]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * S::kStage);
          tma_load_3d_pair(a, &p.tma_x, fb, c + p.dc[j], trow + p.dr[j], tl.b);
          tma_load_2d_pair(a + S::kA, &p.tma_w, fb, j * p.Cin + c, wrow);
        }
        __syncwarp();
        ++issued;
        if (++s == kGpStages) {
          s = 0;
          ph ^= 1;
        }
      }
    }
    if (!ok) {
      if (lane == 0) raise_peer_abort(abort_flag, peer);
      // the even CTA sees its stages land on its own barriers; the odd CTA's
      // copies are covered by the wait before the final pair barrier
      if (rank == 0) {
        const long long first = issued > kGpStages ? issued - kGpStages : 0;
        for (long long i = first; i < issued; ++i)
          mbar_wait_drain(&full[i % kGpStages], static_cast<uint32_t>((i / kGpStages) & 1), 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (rank == 0) {
      const uint32_t idesc = idesc_f16(kGpRows, BN, DT == MT_BF16);
      const uint64_t ring_desc = smem_desc_k_sw128(smem_addr(ring));
      const uint32_t stage_step = S::kStage >> 4, b_off = S::kA >> 4;
      int s = 0, ph = 0, buf = 0;
      int use[2] = {0, 0};
      bool ok = true, issued = false;
      for (int id = pair; id < p.tiles && ok; id += npairs) {
        if (!mbar_wait_warp(&acc_empty[buf], (use[buf] & 1) ^ 1, abort_flag, 0x612)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_warp(&full[s], ph, abort_flag, 0x613)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = ring_desc + s * stage_step;
          const uint64_t bd = ad + b_off;
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < kGtBK / 16; ++kk)
              tc_mma_pair(d, ad + 2 * kk, bd + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            tc_commit_pair(map_to_cta(smem_addr(&empty[s]), 0));
            tc_commit_pair(map_to_cta(smem_addr(&empty[s]), 1));
          }
          __syncwarp();
          issued = true;
          if (++s == kGpStages) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        if (elect_one()) {
          tc_commit_pair(map_to_cta(smem_addr(&acc_full[buf]), 0));
          tc_commit_pair(map_to_cta(smem_addr(&acc_full[buf]), 1));
        }
        __syncwarp();
        ++use[buf];
        buf ^= 1;
      }
      if (!ok && lane == 0) raise_peer_abort(abort_flag, peer);
      if (__any_sync(0xffffffffu, *abort_flag != 0) && issued) {
        if (elect_one()) {
          tc_commit_pair(map_to_cta(smem_addr(drain), 0));
          mbar_wait_drain(drain, 0, 200000000ull);
        }
        __syncwarp();
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // as in gemm_tc_kernel, on this CTA's 128 rows of the pair tile
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quad * 32 + lane;
    int buf = 0;
    int use[2] = {0, 0};
    for (int id = pair; id < p.tiles; id += npairs) {
      const GtTile tl = gp_tile(p, id);
      if (!mbar_wait_warp(&acc_full[buf], use[buf] & 1, abort_flag, 0x614)) {
        if (lane == 0) raise_peer_abort(abort_flag, peer);
        break;
      }
      tc_fence_after();
      const int t = tl.t0 + 128 * static_cast<int>(rank) + row;
      const bool live = t < p.Lout;
      const long long yrow = (static_cast<long long>(tl.b) * p.Lout + t) * p.ldy;
      gt_store_tile<DT, BN, ACT>(p, tmem + (static_cast<uint32_t>(quad * 32) << 16) + buf * BN, half, live, yrow,
                                 ACT == 2 ? tl.n0 * 128 : tl.n0 * BN);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(map_to_cta(smem_addr(&acc_empty[buf]), 0));
      ++use[buf];
      buf ^= 1;
    }
  }
  __syncthreads();
  if (*abort_flag) {  // give copies still in flight (the odd CTA's among them) time to land
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  tc_fence_before();
  __syncthreads();
  pair_barrier();  // no CTA frees its tensor memory or exits while its peer still works
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, 2 * BN);
}

// Tensor-core eligibility and launch. Returns MT_ERR_UNSUPPORTED when the
// shape is outside what this kernel takes (the caller then uses the
// mma.sync implicit GEMM).
int gemm_tc_run(const void* x, const void* w, const void* bias, const void* residual, void* y, int64_t B,
                int64_t L, int64_t Cin, int64_t Cout, int taps, int stride, int padding, int act, int dtype,
                int bias_fused, int64_t ldy, cudaStream_t stream) {
  if (dtype != MT_BF16 && dtype != MT_F16) return MT_ERR_UNSUPPORTED;
  if (taps < 1 || taps > kGtMaxTaps || (stride != 1 && stride != 2)) return MT_ERR_UNSUPPORTED;
  if (taps > 1 ? Cin % kGtBK != 0 : Cin % 8 != 0) return MT_ERR_UNSUPPORTED;
  if (L % stride != 0 || !aligned(x, 16) || !aligned(w, 16)) return MT_ERR_UNSUPPORTED;
  const int64_t Lout = (L + 2 * padding - taps) / stride + 1;
  if (Lout < 1 || B < 1) return MT_ERR_UNSUPPORTED;
  if (B * Lout >= (int64_t(1) << 31) || Cout >= (1 << 24) || taps * Cin >= (1 << 24)) return MT_ERR_UNSUPPORTED;
  // act 2 (SwiGLU): Cout is the output width N; w holds 256 * ceil(N/128)
  // rows, gate and up rows of each 128 outputs in consecutive blocks of 128
  const int64_t Nout = Cout;
  if (act == 2) {
    if (bias || residual || taps != 1) return MT_ERR_UNSUPPORTED;
    Cout = 256 * ((Nout + 127) / 128);
  }

  GemmTcParams p;
  memset(&p, 0, sizeof(p));
  const int BN = act == 2 || Cout > 128 ? 256 : 128;
  const CUtensorMapDataType dt = dtype == MT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(Cin * stride), static_cast<uint64_t>(L / stride),
                              static_cast<uint64_t>(B)};
    const uint64_t strides[2] = {static_cast<uint64_t>(Cin * stride * 2), static_cast<uint64_t>(L * Cin * 2)};
    const uint32_t box[3] = {kGtBK, kGtBM, 1};
    const int rc = make_tmap(&p.tma_x, x, dt, 2, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != MT_OK) return rc;
  }
  // CTA pairs for 256-column tiles once there are enough 256 x 256 tiles to
  // give every pair of SMs one (MT_GEMM_PAIR=0 / 1 forces the choice)
  int sms = 148;
  if (int e = device_sm_count(&sms)) return e;
  const int64_t pair_tiles = B * ((Lout + kGpRows - 1) / kGpRows) * ((Cout + 255) / 256);
  const char* pe = getenv("MT_GEMM_PAIR");
  const int pair_mode = pe ? atoi(pe) : -1;
  const bool pair = BN == 256 && (pair_mode > 0 || (pair_mode < 0 && pair_tiles >= sms / 2));
  {
    const int rc = make_tmap_2d(&p.tma_w, w, dt, 2, static_cast<uint64_t>(taps * Cin), static_cast<uint64_t>(Cout),
                                static_cast<uint64_t>(taps * Cin * 2), kGtBK, pair ? 128 : BN,
                                CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != MT_OK) return rc;
  }
  for (int j = 0; j < taps; ++j) {
    const int o = j - padding;
    const int q = o >= 0 ? o / stride : -((-o + stride - 1) / stride);  // floor division
    p.dr[j] = q;
    p.dc[j] = (o - q * stride) * static_cast<int>(Cin);
  }
  p.bias = bias;
  p.residual = residual;
  p.y = y;
  p.ldy = ldy;
  p.B = static_cast<int>(B);
  p.Lout = static_cast<int>(Lout);
  p.Cin = static_cast<int>(Cin);
  p.Cout = static_cast<int>(Cout);
  p.taps = taps;
  p.kb_per_tap = static_cast<int>((Cin + kGtBK - 1) / kGtBK);
  p.mt_per_b = static_cast<int>((Lout + (pair ? kGpRows : kGtBM) - 1) / (pair ? kGpRows : kGtBM));
  p.num_mt = p.mt_per_b * p.B;
  p.num_nt = static_cast<int>((Cout + BN - 1) / BN);
  const int64_t tiles = static_cast<int64_t>(p.num_mt) * p.num_nt;
  if (tiles >= (int64_t(1) << 31)) return MT_ERR_UNSUPPORTED;
  p.tiles = static_cast<int>(tiles);
  p.bias_fused = bias_fused;
  p.Nout = static_cast<int>(Nout);
  p.vec = (ldy % 8 == 0) && aligned(y, 16) && (!bias || aligned(bias, 16)) && (!residual || aligned(residual, 16));
  const bool bf = dtype == MT_BF16;
  if (pair) {
    auto run_pair = [&](auto kern) -> int {
      if (int e = ensure_smem(kern, GpSmem::kTotal)) return e;
      int clusters = sms / 2;
      if (int e = max_active_clusters(kern, kGtThreads, GpSmem::kTotal, 2, &clusters)) return e;
      if (clusters < 1) return MT_ERR_UNSUPPORTED;
      if (clusters > p.tiles) clusters = p.tiles;
      return launch_cluster(kern, dim3(2 * static_cast<unsigned>(clusters)), dim3(kGtThreads), GpSmem::kTotal, 2,
                            stream, p);
    };
    if (act == 2) return bf ? run_pair(gemm_tc_pair_kernel<MT_BF16, 2>) : run_pair(gemm_tc_pair_kernel<MT_F16, 2>);
    if (act == 1) return bf ? run_pair(gemm_tc_pair_kernel<MT_BF16, 1>) : run_pair(gemm_tc_pair_kernel<MT_F16, 1>);
    return bf ? run_pair(gemm_tc_pair_kernel<MT_BF16, 0>) : run_pair(gemm_tc_pair_kernel<MT_F16, 0>);
  }
  const unsigned grid = static_cast<unsigned>(p.tiles < sms ? p.tiles : sms);
  auto run = [&](auto kern, size_t smem) -> int {
    if (int e = ensure_smem(kern, smem)) return e;
    return launch(kern, dim3(grid), dim3(kGtThreads), smem, stream, p);
  };
  if (BN == 128) {
    const size_t sm = GtSmem<128>::kTotal;
    if (bf) return act ? run(gemm_tc_kernel<MT_BF16, 128, 1>, sm) : run(gemm_tc_kernel<MT_BF16, 128, 0>, sm);
    return act ? run(gemm_tc_kernel<MT_F16, 128, 1>, sm) : run(gemm_tc_kernel<MT_F16, 128, 0>, sm);
  }
  const size_t sm = GtSmem<256>::kTotal;
  if (act == 2) return bf ? run(gemm_tc_kernel<MT_BF16, 256, 2>, sm) : run(gemm_tc_kernel<MT_F16, 256, 2>, sm);
  if (bf) return act ? run(gemm_tc_kernel<MT_BF16, 256, 1>, sm) : run(gemm_tc_kernel<MT_BF16, 256, 0>, sm);
  return act ? run(gemm_tc_kernel<MT_F16, 256, 1>, sm) : run(gemm_tc_kernel<MT_F16, 256, 0>, sm);
}

}  // namespace mt
