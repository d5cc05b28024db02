// Prefill scaled-dot-product attention on the 5th-generation tensor cores
// (flash attention forward: tcgen05.mma with tensor-memory accumulators,
// TMA-staged Q/K/V, online softmax).
//
// Work item = 128 query rows of one (batch, head); KV blocks of 128 keys. A
// persistent grid (one CTA per SM) walks the items heaviest first, so the
// next item's Q copy and first S = Q K^T overlap this item's O store.
//   S_j = Q K_j^T        tcgen05.mma, A = Q and B = K_j from shared memory
//                        (K-major, 128-byte swizzle), fp32 S in tensor memory
//                        (two buffers, so S_{j+1} is computed while the
//                        softmax of block j runs)
//   P_j = exp2(S_j * scale * log2 e - m)   by the softmax warps, one query row
//                        per thread (the row's 128 scores are that thread's
//                        tensor-memory lane: no cross-thread reduction),
//                        rounded to the input type and stored back into
//                        tensor memory (tcgen05.st)
//   O  += P_j V_j        tcgen05.mma with A = P_j from tensor memory and
//                        B = V_j from shared memory read MN-major (V's rows
//                        are keys = the reduction dim, D contiguous), O fp32
//                        in tensor memory
// The running maximum m of a row is raised only when a block's maximum
// exceeds it by more than 8 (log2 units); the exponentials then stay below
// 2^8, and O and the row sum l are rescaled by exp2(m_old - m_new) only then
// (after the previous P V has completed). The result is O / l, rounded.
//
// Q, K, V, O are addressed through element strides (D contiguous) with
// 5-D TMA tensor maps (64, L, D/64, H, B): one copy brings a 128-row tile as
// D/64 swizzled 128-byte-row slabs. Keys past Lk and rows past Lq are the
// copies' zero fill; such keys are masked, such rows not stored. Causal
// blocks past the diagonal are never loaded.
//
// Roles (192 threads): warp 0 issues the TMA copies (Q once, then K and V
// per block into 2-stage rings of their own, K one block ahead of V: a K
// stage is free again once its S = Q K^T has completed, a V stage only after
// its P V), warp 1 owns the tensor memory and issues the MMAs
// from one elected lane, warps 2-5 run the softmax, the O rescaling and the
// final normalisation and store. Every mbarrier wait is bounded (2 s); on
// expiry the CTA records a site code in the device status word, drains its
// in-flight copies and MMAs (bounded) and frees its tensor memory.
#include "mt_common.cuh"
#include "mt_tma.h"

namespace mt {

constexpr int kAtBQ = 128;
constexpr int kAtBK = 128;
constexpr int kAtThreads = 192;
constexpr int kAtStages = 2;
// tensor-memory columns: S[2] at 0 / 128, P[2] (bf16 pairs) at 256 / 320, O at 384
constexpr uint32_t kAtColS = 0, kAtColP = 256, kAtColO = 384;
constexpr float kAtRescale = 8.0f;  // log2 growth of the row maximum that forces a rescale

struct AttnTcParams {
  CUtensorMap tq, tk, tv;  // (64, L, D/64, H, B), box (64, 128, D/64, 1, 1)
  void* o;
  int64_t os_b, os_h, os_l;
  int Hq, Hkv, Lq, Lk;
  int64_t q_offset;
  float scale_log2;
  int causal, vec;
  int B, nq, tiles;  // batch, query blocks per (batch, head), work items = nq * Hq * B
};

template <int D>
struct AtSmem {
  static constexpr int kTile = 128 * D * 2;            // one 128-row tile, D/64 slabs of 16 KB
  static constexpr int kQ = kTile;
  static constexpr int kBars = 1024;
  static constexpr int kUsed = kQ + 2 * kAtStages * kTile + kBars + 1024;  // Q, K ring, V ring
  // at least 120 KB so one CTA holds an SM (its tensor memory is all 512 columns)
  static constexpr int kTotal = kUsed > 120 * 1024 ? kUsed : 120 * 1024;
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Work item `id` of the persistent grid: query block, head, batch and the
// number of key blocks it sees. Items run heaviest first: the last query
// block of every (head, batch) before the one before it, and so on.
struct AtTile {
  int q0, h, b, kvh, nb;
};
__device__ __forceinline__ AtTile at_tile(const AttnTcParams& p, int id) {
  const int hb = p.Hq * p.B;
  const int qi = id / hb;
  const int r = id - qi * hb;
  AtTile t;
  t.q0 = (p.nq - 1 - qi) * kAtBQ;
  t.h = r % p.Hq;
  t.b = r / p.Hq;
  t.kvh = t.h / (p.Hq / p.Hkv);
  int64_t kv_end = p.Lk;  // keys this block can see: [0, kv_end)
  if (p.causal) {
    const int64_t lim = p.q_offset + t.q0 + kAtBQ;
    if (lim < kv_end) kv_end = lim < 0 ? 0 : lim;
  }
  t.nb = static_cast<int>((kv_end + kAtBK - 1) / kAtBK);
  return t;
}

template <int DT, int D>
__global__ void __launch_bounds__(kAtThreads, 1) attn_tc_kernel(const __grid_constant__ AttnTcParams p) {
  using T = typename Elem<DT>::T;
  using S = AtSmem<D>;
  extern __shared__ uint8_t at_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(at_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;
  uint8_t* kring = smem + S::kQ;
  uint8_t* vring = kring + kAtStages * S::kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(vring + kAtStages * S::kTile);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;               // Q read by the tile's last S
  uint64_t* o_free = bars + 2;                // O read out by the softmax warps
  uint64_t* k_full = bars + 3;                // [stages]
  uint64_t* k_empty = k_full + kAtStages;     // [stages]
  uint64_t* v_full = k_empty + kAtStages;     // [stages]
  uint64_t* v_empty = v_full + kAtStages;     // [stages]
  uint64_t* s_full = v_empty + kAtStages;     // [2]
  uint64_t* s_free = s_full + 2;              // [2]
  uint64_t* p_full = s_free + 2;              // [2]
  uint64_t* pv_done = p_full + 2;             // [2]
  uint64_t* drain = pv_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(o_free, 4);
    for (int s = 0; s < kAtStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tq);
    prefetch_tmap(&p.tk);
    prefetch_tmap(&p.tv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  griddep_launch();

  // Counters shared by all roles, over the work items with at least one key
  // block: qt counts items, g counts key blocks (ring stage g % kAtStages,
  // S / P buffer g & 1).
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    int qt = 0, kc = 0, vc = 0;
    bool ok = true;
    // one K or V block copy into the next stage of its ring
    auto copy = [&](bool is_v, const AtTile& t, int j) -> bool {
      int& c = is_v ? vc : kc;
      const int st = c % kAtStages;
      uint64_t* empty = is_v ? v_empty : k_empty;
      uint64_t* full = is_v ? v_full : k_full;
      if (!mbar_wait_warp(&empty[st], ((c / kAtStages) & 1) ^ 1, abort_flag, is_v ? 0x70a : 0x701)) return false;
      if (elect_one()) {
        mbar_arrive_expect_tx(&full[st], S::kTile);
        tma_load_5d((is_v ? vring : kring) + st * S::kTile, is_v ? &p.tv : &p.tk, &full[st], 0, j * kAtBK, 0, t.kvh,
                    t.b);
      }
      __syncwarp();
      ++c;
      return true;
    };
    for (int id = blockIdx.x; id < p.tiles && ok; id += gridDim.x) {
      const AtTile t = at_tile(p, id);
      if (t.nb == 0) continue;
      if (!mbar_wait_warp(q_empty, (qt & 1) ^ 1, abort_flag, 0x70c)) {
        ok = false;
        break;
      }
      if (elect_one()) {
        mbar_arrive_expect_tx(q_full, S::kQ);
        tma_load_5d(sq, &p.tq, q_full, 0, t.q0, 0, t.h, t.b);
      }
      __syncwarp();
      ++qt;
      ok = copy(false, t, 0);
      for (int j = 0; j < t.nb && ok; ++j) {
        if (j + 1 < t.nb && !copy(false, t, j + 1)) {
          ok = false;
          break;
        }
        ok = copy(true, t, j);
      }
    }
    if (!ok) {
      if (qt > 0) mbar_wait_drain(q_full, static_cast<uint32_t>((qt - 1) & 1), 200000000ull);
      for (int i = (kc > kAtStages ? kc - kAtStages : 0); i < kc; ++i)
        mbar_wait_drain(&k_full[i % kAtStages], static_cast<uint32_t>((i / kAtStages) & 1), 200000000ull);
      for (int i = (vc > kAtStages ? vc - kAtStages : 0); i < vc; ++i)
        mbar_wait_drain(&v_full[i % kAtStages], static_cast<uint32_t>((i / kAtStages) & 1), 200000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t id_s = idesc_f16(kAtBQ, kAtBK, DT == MT_BF16);
    const uint32_t id_pv = idesc_f16(kAtBQ, D, DT == MT_BF16) | (1u << 16);  // B (V) MN-major
    const uint64_t qdesc = smem_desc_k_sw128(smem_addr(sq));
    // V read MN-major: 8-key groups 1024 B apart (SBO), 64-column slabs 16 KB apart (LBO)
    auto vdesc_of = [](uint32_t saddr) -> uint64_t {
      uint64_t d = 0;
      d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);
      d |= static_cast<uint64_t>((128 * 128) >> 4) << 16;  // LBO
      d |= static_cast<uint64_t>(1024 >> 4) << 32;         // SBO
      d |= static_cast<uint64_t>(1) << 46;
      d |= static_cast<uint64_t>(2) << 61;
      return d;
    };
    bool ok = true, issued_any = false;
    int qt = 0, gs = 0, gp = 0;  // items, S blocks and P V blocks issued
    // S = Q K^T of the next key block; after the item's last one, Q is free
    auto issue_s = [&](bool last) -> bool {
      const int st = gs % kAtStages, sb = gs & 1;
      if (!mbar_wait_warp(&k_full[st], (gs / kAtStages) & 1, abort_flag, 0x703)) return false;
      if (!mbar_wait_warp(&s_free[sb], ((gs >> 1) & 1) ^ 1, abort_flag, 0x704)) return false;
      tc_fence_after();
      const uint64_t kdesc = smem_desc_k_sw128(smem_addr(kring + st * S::kTile));
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = static_cast<uint32_t>(((kk >> 2) * 128 * 128 + (kk & 3) * 32) >> 4);
          tc_mma_ss(tmem + kAtColS + sb * kAtBK, qdesc + off, kdesc + off, id_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[sb]);
        tc_commit(&k_empty[st]);
        if (last) tc_commit(q_empty);
      }
      __syncwarp();
      issued_any = true;
      ++gs;
      return true;
    };
    for (int id = blockIdx.x; id < p.tiles && ok; id += gridDim.x) {
      const AtTile t = at_tile(p, id);
      if (t.nb == 0) continue;
      if (!mbar_wait_warp(q_full, qt & 1, abort_flag, 0x702)) {
        ok = false;
        break;
      }
      ok = issue_s(t.nb == 1);
      for (int j = 0; j < t.nb && ok; ++j) {
        if (j + 1 < t.nb && !issue_s(j + 2 == t.nb)) {
          ok = false;
          break;
        }
        const int st = gp % kAtStages, pb = gp & 1;
        // the item's first P V overwrites O: the previous item's O must have been read out
        if ((j == 0 && !mbar_wait_warp(o_free, (qt & 1) ^ 1, abort_flag, 0x70d)) ||
            !mbar_wait_warp(&v_full[st], (gp / kAtStages) & 1, abort_flag, 0x70b) ||
            !mbar_wait_warp(&p_full[pb], (gp >> 1) & 1, abort_flag, 0x705)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t vaddr = smem_addr(vring + st * S::kTile);
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < kAtBK / 16; ++kk)
            tc_mma_ts(tmem + kAtColO, tmem + kAtColP + pb * 64 + kk * 8, vdesc_of(vaddr + kk * 2048), id_pv,
                      (j > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&v_empty[st]);
          tc_commit(&pv_done[pb]);
        }
        __syncwarp();
        ++gp;
      }
      ++qt;
    }
    if (__any_sync(0xffffffffu, *abort_flag != 0) && issued_any) {
      if (elect_one()) {
        tc_commit(drain);
        mbar_wait_drain(drain, 0, 200000000ull);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ softmax / correction / store
    const int quad = warp & 3;                 // tensor-memory lanes [32*quad, +32)
    const int row = quad * 32 + lane;          // query row within the block
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    bool ok = true;
    int g = 0;  // key blocks consumed
    for (int id = blockIdx.x; id < p.tiles && ok; id += gridDim.x) {
      const AtTile t = at_tile(p, id);
      T* o = static_cast<T*>(p.o) + t.b * p.os_b + t.h * p.os_h + static_cast<int64_t>(t.q0 + row) * p.os_l;
      const bool live = t.q0 + row < p.Lq;
      if (t.nb == 0) {
        // no visible key (only possible with a negative q_offset): zeros, as the oracle writes
        if (live)
          for (int i = 0; i < D; ++i) o[i] = Elem<DT>::from_f(0.f);
        continue;
      }
      const int64_t qpos = p.q_offset + t.q0 + row;  // absolute position (causal limit)
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < t.nb; ++j, ++g) {
        const int sb = g & 1;
        if (!mbar_wait_warp(&s_full[sb], (g >> 1) & 1, abort_flag, 0x706)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // the row's 128 scores: four loads in flight, one wait
        float sv[kAtBK];
        uint32_t r[kAtBK / 32][32];
#pragma unroll
        for (int c = 0; c < kAtBK / 32; ++c) tmem_ld32(tmem + lane_off + kAtColS + sb * kAtBK + c * 32, r[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < kAtBK / 32; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(r[c][i]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[sb]);
        const int k0 = j * kAtBK;
        const bool edge = k0 + kAtBK > p.Lk || (p.causal && k0 + kAtBK - 1 > p.q_offset + t.q0);
        if (edge) {
#pragma unroll
          for (int i = 0; i < kAtBK; ++i) {
            const int64_t key = k0 + i;
            const bool vis = key < p.Lk && (!p.causal || key <= qpos);
            if (!vis) sv[i] = -INFINITY;
          }
        }
        // the block's maximum of the raw scores in 8 independent chains (one
        // warp per scheduler: a single chain of 128 would expose each step's
        // latency); scale > 0, so it scales to the maximum of the scaled scores
        float mxk[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mxk[u] = sv[u];
#pragma unroll
        for (int i = 8; i < kAtBK; ++i) mxk[i & 7] = fmaxf(mxk[i & 7], sv[i]);
        const float mx = fmaxf(fmaxf(fmaxf(mxk[0], mxk[1]), fmaxf(mxk[2], mxk[3])),
                               fmaxf(fmaxf(mxk[4], mxk[5]), fmaxf(mxk[6], mxk[7]))) * p.scale_log2;
        const float m_new = fmaxf(m_run, mx);
        const bool need = j > 0 && m_new > m_run + kAtRescale;
        if (j == 0) {
          m_run = m_new;
        } else if (__any_sync(0xffffffffu, need)) {
          // the previous P V must have landed in O before O is rescaled
          if (!mbar_wait_warp(&pv_done[(g - 1) & 1], ((g - 1) >> 1) & 1, abort_flag, 0x707)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float alpha = need ? exp2f(m_run - m_new) : 1.0f;
          if (need) {
            m_run = m_new;
            l_run *= alpha;
          }
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t ro[32];
            tmem_ld32(tmem + lane_off + kAtColO + c * 32, ro);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) ro[i] = __float_as_uint(__uint_as_float(ro[i]) * alpha);
            tmem_st32(tmem + lane_off + kAtColO + c * 32, ro);
          }
          tmem_wait_st();
        }
        // P buffer g % 2 was last read by the P V of key block g - 2
        if (g >= 2 && !mbar_wait_warp(&pv_done[sb], ((g - 2) >> 1) & 1, abort_flag, 0x708)) {
          ok = false;
          break;
        }
        // p = 2^(s * scale - m), the scale folded into one FMA; the row sum in
        // 8 independent chains. A row that sees no key yet (m = -inf, only
        // with a negative q_offset) gets p = 0 and, at the end, zeros.
        const float m_use = m_run == -INFINITY ? 0.f : m_run;
        float rsk[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) rsk[u] = 0.f;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float e0 = ex2_approx(fmaf(sv[c * 64 + 2 * i], p.scale_log2, -m_use));
            const float e1 = ex2_approx(fmaf(sv[c * 64 + 2 * i + 1], p.scale_log2, -m_use));
            rsk[(2 * i) & 7] += e0;
            rsk[(2 * i + 1) & 7] += e1;
            typename Elem<DT>::T2 t2 = Elem<DT>::pack2(e0, e1);
            pk[i] = *reinterpret_cast<uint32_t*>(&t2);
          }
          tmem_st32(tmem + lane_off + kAtColP + sb * 64 + c * 32, pk);
        }
        l_run += ((rsk[0] + rsk[1]) + (rsk[2] + rsk[3])) + ((rsk[4] + rsk[5]) + (rsk[6] + rsk[7]));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[sb]);
      }
      if (!ok || !mbar_wait_warp(&pv_done[(g - 1) & 1], ((g - 1) >> 1) & 1, abort_flag, 0x709)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t ro[32];
        tmem_ld32(tmem + lane_off + kAtColO + c * 32, ro);
        tmem_wait_ld();
        if (live) {
          if (p.vec) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 u;
              typename Elem<DT>::T2* hh = reinterpret_cast<typename Elem<DT>::T2*>(&u);
#pragma unroll
              for (int e = 0; e < 4; ++e)
                hh[e] = Elem<DT>::pack2(__uint_as_float(ro[8 * q + 2 * e]) * inv,
                                        __uint_as_float(ro[8 * q + 2 * e + 1]) * inv);
              *reinterpret_cast<uint4*>(o + c * 32 + 8 * q) = u;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[c * 32 + i] = Elem<DT>::from_f(__uint_as_float(ro[i]) * inv);
          }
        }
        __syncwarp();
      }
      // O is read out: the next item's first P V may overwrite it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

static int make_qkv_map(CUtensorMap* m, const void* base, int dtype, int64_t L, int64_t H, int64_t B, int D,
                        int64_t s_b, int64_t s_h, int64_t s_l) {
  const CUtensorMapDataType dt = dtype == MT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t dims[5] = {64, static_cast<uint64_t>(L), static_cast<uint64_t>(D / 64), static_cast<uint64_t>(H),
                            static_cast<uint64_t>(B)};
  const uint64_t strides[4] = {static_cast<uint64_t>(s_l) * 2, 128, static_cast<uint64_t>(s_h) * 2,
                               static_cast<uint64_t>(s_b) * 2};
  const uint32_t box[5] = {64, 128, static_cast<uint32_t>(D / 64), 1, 1};
  return make_tmap(m, base, dt, 2, 5, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// The tcgen05 path of mt_sdpa; MT_ERR_UNSUPPORTED when the layout does not
// suit TMA (the caller then runs the mma.sync kernel).
int attn_tc_run(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t Hq, int64_t Hkv, int64_t Lq,
                int64_t Lk, int64_t D, float scale, int causal, int64_t q_offset, int64_t qs_b, int64_t qs_h,
                int64_t qs_l, int64_t ks_b, int64_t ks_h, int64_t ks_l, int64_t vs_b, int64_t vs_h, int64_t vs_l,
                int64_t os_b, int64_t os_h, int64_t os_l, int dtype, cudaStream_t stream) {
  if ((D != 64 && D != 128) || (dtype != MT_BF16 && dtype != MT_F16)) return MT_ERR_UNSUPPORTED;
  if (!(scale > 0.f)) return MT_ERR_UNSUPPORTED;  // the kernel folds a positive scale into its exponent
  const int64_t st[9] = {qs_b, qs_h, qs_l, ks_b, ks_h, ks_l, vs_b, vs_h, vs_l};
  for (int64_t s : st)
    if (s <= 0 || s % 8 != 0) return MT_ERR_UNSUPPORTED;
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16)) return MT_ERR_UNSUPPORTED;
  if (Lq > (int64_t(1) << 30) || Lk > (int64_t(1) << 30) || Hq > 65535 || B > 65535) return MT_ERR_UNSUPPORTED;
  AttnTcParams p;
  memset(&p, 0, sizeof(p));
  int rc = make_qkv_map(&p.tq, q, dtype, Lq, Hq, B, static_cast<int>(D), qs_b, qs_h, qs_l);
  if (rc == MT_OK) rc = make_qkv_map(&p.tk, k, dtype, Lk, Hkv, B, static_cast<int>(D), ks_b, ks_h, ks_l);
  if (rc == MT_OK) rc = make_qkv_map(&p.tv, v, dtype, Lk, Hkv, B, static_cast<int>(D), vs_b, vs_h, vs_l);
  if (rc != MT_OK) return rc;
  p.o = o;
  p.os_b = os_b;
  p.os_h = os_h;
  p.os_l = os_l;
  p.Hq = static_cast<int>(Hq);
  p.Hkv = static_cast<int>(Hkv);
  p.Lq = static_cast<int>(Lq);
  p.Lk = static_cast<int>(Lk);
  p.q_offset = q_offset;
  p.scale_log2 = scale * 1.44269504088896341f;
  p.causal = causal;
  p.vec = aligned(o, 16) && os_l % 8 == 0 && os_h % 8 == 0 && os_b % 8 == 0;
  p.B = static_cast<int>(B);
  p.nq = static_cast<int>((Lq + kAtBQ - 1) / kAtBQ);
  const int64_t tiles = static_cast<int64_t>(p.nq) * Hq * B;
  if (tiles >= (int64_t(1) << 31)) return MT_ERR_UNSUPPORTED;
  p.tiles = static_cast<int>(tiles);
  int sms = 148;
  if (int e = device_sm_count(&sms)) return e;
  // persistent: one CTA per SM (each holds all 512 tensor-memory columns)
  const dim3 grid(static_cast<unsigned>(p.tiles < sms ? p.tiles : sms));
  auto run = [&](auto kern, size_t smem) -> int {
    if (int e = ensure_smem(kern, smem)) return e;
    return launch(kern, grid, dim3(kAtThreads), smem, stream, p);
  };
  if (dtype == MT_BF16)
    return D == 128 ? run(attn_tc_kernel<MT_BF16, 128>, AtSmem<128>::kTotal)
                    : run(attn_tc_kernel<MT_BF16, 64>, AtSmem<64>::kTotal);
  return D == 128 ? run(attn_tc_kernel<MT_F16, 128>, AtSmem<128>::kTotal)
                  : run(attn_tc_kernel<MT_F16, 64>, AtSmem<64>::kTotal);
}

}  // namespace mt
