// Affine-quantized matrix-vector product for decode (M <= 4 rows of x, 4-bit
// weights), streamed through shared memory.
//
// HBM-bound: every packed weight byte is read once, so the kernel is built to
// keep the memory system busy from its first cycle. One CTA per SM owns the
// contiguous row range [c*R/P, (c+1)*R/P) of the output; the packed rows of
// that range are one contiguous byte stream (rows of the same set are
// adjacent in the MLX layout), which a producer warp copies into a ring of
// 16-64 KB shared-memory stages with bulk copies. The CTA's scales and biases
// are copied once up front; when they do not fit (row ranges of an lm_head),
// each stage receives those of the rows it touches instead. Weights and
// scales never depend
// on the previous kernel, so the producer starts before the grid dependency
// resolves: with programmatic dependent launch the first stages are in flight
// while the predecessor is still finishing. The 16 consumer warps stage x in
// shared memory (after the dependency; with a fused RMSNorm, normalised
// there), then split into row walkers (a warp, or a half-warp for rows of at
// most 128 units): walker w owns stream rows w, w + walkers, ... and walks
// the stages in order, its lanes over the row's 16-byte units.
//
// Arithmetic per 32-value unit (autotuner/scaffold/lower.py:1179-1234, the
// MLX qmv form): acc += scale * sum(x*q) + bias * sum(x), fp32. One logic op
// turns nibbles i and i+4 of a packed word into the element-type pair
// (C+q_i, C+q_{i+4}) (C = 128 for bf16, 1024 for fp16, both exact), and the
// mixed-precision FMA (16-bit inputs, fp32 accumulator) multiplies it with x
// staged as the matching pairs (x_i, x_{i+4}). Products are exact, the unit
// sum is corrected by C * sum(x) with the unit sums of x precomputed once.
// ncu (decode gate_up): 5.6 thread instructions per weight in all, ALU pipe
// 54% and issue 62% active, DRAM 18%: issue-bound, not HBM-bound.
#include "mt_common.cuh"
#include "qmm_common.cuh"

namespace mt {

constexpr int kQsConsumerWarps = 16;
constexpr int kQsThreads = (kQsConsumerWarps + 1) * 32;  // + one producer warp
// Ring stage sizes tried largest first: fewer, larger stages mean fewer
// full/empty hand-offs per row walker (measured on B200, M = 1, K = 2560:
// gate_up 13.3 / 12.1 / 11.5 us with 16 / 32 / 48-64 KB stages; 8 KB: 16.4).
constexpr int kQsStageSizes[4] = {65536, 49152, 32768, 16384};
constexpr int kQsMaxStages = 8;
constexpr int kQsMaxMR = 4;
constexpr int kQsConsumerBar = 1;  // named barrier of the 512 consumer threads
constexpr int kQsSmemLimit = 227 * 1024;

struct QsSet {
  const uint8_t* w;
  const uint8_t* s;
  const uint8_t* b;
  void* y;
  int N;
};

struct QsParams {
  const void* x;
  const void* residual;
  QsSet set[3];
  int row_start[4];  // plain mode: prefix sums of N over the sets
  int M, K, G, gshift;
  int ldx, ldy;
  int rows;          // rows of the output space (plain: all sets; residual / SwiGLU: set 0)
  int P;             // CTAs
  int NST;           // stages in the ring
  int max_rows;      // stream rows of one CTA, upper bound (SwiGLU row sums)
  int spr;           // rows a stage can touch: stage bytes / row bytes + 2
  int stage_sc;      // 1: scales and biases travel with each stage; 0: copied once up front
  int stage_bytes;   // bytes of the weight stream per ring stage (a multiple of 16 KB)
  const void* norm_w;  // non-NULL: stage rms_norm(x, norm_w, eps) instead of x
  float eps;
};

// Byte offsets of the shared-memory regions (host and device agree on them).
// A stage slot: stage_bytes of the weight stream, then (stage_sc) the scales and
// biases ([spr][G] each) of the rows those bytes belong to; without stage_sc
// the CTA's scales and biases ([max_rows][G] each) follow the ring. With a
// fused RMSNorm the norm weight row (K values) and the M row scales follow.
struct QsLayout {
  int slot, sc, sbs, sbb, xs, xsum, gsum, gw, rs, bars, total;
};

__host__ __device__ inline QsLayout qs_layout(int K, int G, int max_rows, int spr, int MR, int NST, int stage_sc,
                                              bool norm, int stage_bytes) {
  QsLayout l;
  l.sc = stage_bytes;  // G*2 is a multiple of 16
  l.slot = stage_sc ? (stage_bytes + 2 * spr * G * 2 + 127) & ~127 : stage_bytes;
  l.sbs = NST * l.slot;
  l.sbb = l.sbs + (stage_sc ? 0 : max_rows * G * 2);
  l.xs = l.sbb + (stage_sc ? 0 : max_rows * G * 2);
  l.xsum = l.xs + MR * K * 2;
  l.gsum = l.xsum + MR * (K / 32) * 4;
  l.gw = (l.gsum + max_rows * MR * 4 + 15) & ~15;
  l.rs = l.gw + (norm ? K * 2 : 0);
  l.bars = l.rs + (norm ? 16 : 0);
  l.total = l.bars + (2 * kQsMaxStages + 2) * 8;
  return l;
}

// x_{8q..8q+7} as loaded (pairs (0,1) (2,3) (4,5) (6,7)) regrouped to the
// pairs (i, i+4), i = 0..3
__device__ __forceinline__ uint4 qs_regroup(uint4 raw) {
  return make_uint4(__byte_perm(raw.x, raw.z, 0x5410), __byte_perm(raw.x, raw.z, 0x7632),
                    __byte_perm(raw.y, raw.w, 0x5410), __byte_perm(raw.y, raw.w, 0x7632));
}

// 16-byte slot of (unit c, word wi) of one staged x row, holding the pairs
// (x_{8wi+i}, x_{8wi+i+4}), i = 0..3: the 32 lanes of a warp read 32
// consecutive units, and the XOR spreads each group of 8 over all banks
__device__ __forceinline__ int qs_xs_index(int c, int wi) { return c * 4 + (wi ^ ((c >> 1) & 3)); }

// Element-type bits of C+q with C = 128 (bf16) or 1024 (fp16): the offset
// that makes the nibble the low mantissa bits.
template <int DT> struct QsNib;
template <> struct QsNib<MT_BF16> {
  static constexpr uint32_t kPair = 0x43004300u;
  static constexpr float kC = 128.f;
};
template <> struct QsNib<MT_F16> {
  static constexpr uint32_t kPair = 0x64006400u;
  static constexpr float kC = 1024.f;
};

// a0 += lo(x) * lo(w), a1 += hi(x) * hi(w): 16-bit inputs, fp32 accumulators
template <int DT>
__device__ __forceinline__ void qs_fma_pair(uint32_t x, uint32_t w, float& a0, float& a1) {
  if constexpr (DT == MT_BF16)
    asm("{ .reg .b16 xl, xh, wl, wh;\n mov.b32 {xl, xh}, %2;\n mov.b32 {wl, wh}, %3;\n"
        " fma.rn.f32.bf16 %0, xl, wl, %0;\n fma.rn.f32.bf16 %1, xh, wh, %1; }"
        : "+f"(a0), "+f"(a1) : "r"(x), "r"(w));
  else
    asm("{ .reg .b16 xl, xh, wl, wh;\n mov.b32 {xl, xh}, %2;\n mov.b32 {wl, wh}, %3;\n"
        " fma.rn.f32.f16 %0, xl, wl, %0;\n fma.rn.f32.f16 %1, xh, wh, %1; }"
        : "+f"(a0), "+f"(a1) : "r"(x), "r"(w));
}

// LPR: lanes per row. 32: a warp walks one row; 16: each half-warp walks its
// own row (rows of 16..128 units, where 32 lanes would leave part of the last
// pass idle, e.g. 80 units at K = 2560).
template <int DT, int MR, int MODE, int LPR>
__global__ void __launch_bounds__(kQsThreads, 1) qmv_stream_kernel(const __grid_constant__ QsParams p) {
  using T = typename Elem<DT>::T;
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = p.K, G = p.G, NST = p.NST;
  const int rowB = K / 2;   // packed bytes per row
  const int rowU = K / 32;  // 16-byte units per row
  const bool norm = p.norm_w != nullptr;
  const QsLayout L = qs_layout(K, G, p.max_rows, p.spr, MR, NST, p.stage_sc, norm, p.stage_bytes);
  const int stage_bytes = p.stage_bytes, stage_units = p.stage_bytes / 16;
  uint8_t* ring = smem;
  T* sbS = reinterpret_cast<T*>(smem + L.sbs);
  T* sbB = reinterpret_cast<T*>(smem + L.sbb);
  uint4* xs = reinterpret_cast<uint4*>(smem + L.xs);  // [MR][K/8] pairs of x
  float* xsum = reinterpret_cast<float*>(smem + L.xsum);
  float* gsum = reinterpret_cast<float*>(smem + L.gsum);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + kQsMaxStages;
  uint64_t* sb_bar = empty + kQsMaxStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sb_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const int ra = static_cast<int>(static_cast<long long>(c) * p.rows / p.P);
  const int rb = static_cast<int>(static_cast<long long>(c + 1) * p.rows / p.P);
  const int nr = rb - ra;

  // the CTA's stream: up to three segments (set, first row in the set, rows)
  int seg_set[3] = {0, 0, 0}, seg_row[3] = {0, 0, 0}, seg_n[3] = {0, 0, 0};
  int nseg = 0;
  if (MODE == 0) {
    for (int s = 0; s < 3; ++s) {
      const int lo = ra > p.row_start[s] ? ra : p.row_start[s];
      const int hi = rb < p.row_start[s + 1] ? rb : p.row_start[s + 1];
      if (lo < hi) {
        seg_set[nseg] = s;
        seg_row[nseg] = lo - p.row_start[s];
        seg_n[nseg] = hi - lo;
        ++nseg;
      }
    }
  } else {
    seg_set[0] = 0;
    seg_row[0] = ra;
    seg_n[0] = nr;
    nseg = 1;
    if (MODE == 2) {
      seg_set[1] = 1;
      seg_row[1] = ra;
      seg_n[1] = nr;
      nseg = 2;
    }
  }
  const int srows = seg_n[0] + seg_n[1] + seg_n[2];
  const int total_units = srows * rowU;
  const int nstage = (total_units + stage_units - 1) / stage_units;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kQsMaxStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kQsConsumerWarps);
    }
    mbar_init(sb_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kQsConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = l2_evict_first();  // weights, scales and biases are read once
      if (!p.stage_sc) {
        // scales and biases of the CTA's rows, once
        mbar_arrive_expect_tx(sb_bar, static_cast<uint32_t>(srows * G * 2 * 2));
        int lr = 0;
        for (int sg = 0; sg < nseg; ++sg) {
          const QsSet& st = p.set[seg_set[sg]];
          const size_t off = static_cast<size_t>(seg_row[sg]) * G * 2;
          bulk_load_hint(sbS + lr * G, st.s + off, seg_n[sg] * G * 2, sb_bar, pol);
          bulk_load_hint(sbB + lr * G, st.b + off, seg_n[sg] * G * 2, sb_bar, pol);
          lr += seg_n[sg];
        }
      }
      const long long total = static_cast<long long>(srows) * rowB;
      int issued = 0;
      for (int k = 0; k < nstage; ++k) {
        const int slot = k % NST;
        if (k >= NST && !mbar_wait(&empty[slot], ((k / NST) - 1) & 1, abort_flag, 0x501)) break;
        long long off = static_cast<long long>(k) * stage_bytes;
        const long long end = (off + stage_bytes < total) ? off + stage_bytes : total;
        // stream rows [r_first, r_last] touched by this stage: their scales and biases
        const int r_first = p.stage_sc ? static_cast<int>(off) / rowB : 0;
        const int r_last = p.stage_sc ? static_cast<int>(end - 1) / rowB : -1;
        const int nrk = r_last - r_first + 1;
        mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(end - off + 2 * nrk * G * 2));
        uint8_t* dst = ring + slot * L.slot;
        if (p.stage_sc) {
          int base = 0;
          for (int sg = 0; sg < nseg; ++sg) {
            const int lo = r_first > base ? r_first : base;
            const int hi = (r_last + 1) < (base + seg_n[sg]) ? (r_last + 1) : (base + seg_n[sg]);
            if (lo < hi) {
              const QsSet& st = p.set[seg_set[sg]];
              const size_t so = static_cast<size_t>(seg_row[sg] + lo - base) * G * 2;
              bulk_load_hint(dst + L.sc + (lo - r_first) * G * 2, st.s + so, (hi - lo) * G * 2, &full[slot], pol);
              bulk_load_hint(dst + L.sc + (p.spr + lo - r_first) * G * 2, st.b + so, (hi - lo) * G * 2, &full[slot],
                             pol);
            }
            base += seg_n[sg];
          }
        }
        long long seg0 = 0;  // stream offset of segment sg
        for (int sg = 0; sg < nseg && off < end; ++sg) {
          const long long seg_bytes = static_cast<long long>(seg_n[sg]) * rowB;
          if (off < seg0 + seg_bytes) {
            const long long n = ((seg0 + seg_bytes) < end ? (seg0 + seg_bytes) : end) - off;
            const uint8_t* src = p.set[seg_set[sg]].w + static_cast<long long>(seg_row[sg]) * rowB + (off - seg0);
            bulk_load_hint(dst + (off - static_cast<long long>(k) * stage_bytes), src, static_cast<uint32_t>(n),
                           &full[slot], pol);
            off += n;
          }
          seg0 += seg_bytes;
        }
        ++issued;
      }
      if (*abort_flag) {
        if (!p.stage_sc) mbar_wait_drain(sb_bar, 0, 200000000ull);
        for (int k = (issued > NST ? issued - NST : 0); k < issued; ++k)
          mbar_wait_drain(&full[k % NST], (k / NST) & 1, 200000000ull);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int ct = threadIdx.x;  // 0..511
  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid
  const T* x = static_cast<const T*>(p.x);
  uint4* gw = reinterpret_cast<uint4*>(smem + L.gw);  // norm weight words, regrouped like x
  float* rscale = reinterpret_cast<float*>(smem + L.rs);
  // x as element-type pairs (x_{8wi+i}, x_{8wi+i+4}), one 16-byte slot per
  // (unit, word), and the fp32 sum of every unit
  for (int i = ct; i < MR * (K / 8); i += kQsConsumerWarps * 32) {
    const int m = i / (K / 8), q = i - m * (K / 8);  // q = word index over K
    uint4 v = make_uint4(0, 0, 0, 0);
    if (m < p.M) {
      const uint4 raw = *reinterpret_cast<const uint4*>(x + static_cast<long long>(m) * p.ldx + 8 * q);
      // raw holds x_{8q..8q+7} as pairs (0,1) (2,3) (4,5) (6,7); regroup to (i, i+4)
      v = qs_regroup(raw);
    }
    if (norm && m == 0) gw[q] = qs_regroup(*reinterpret_cast<const uint4*>(static_cast<const T*>(p.norm_w) + 8 * q));
    xs[m * (K / 8) + qs_xs_index(q >> 2, q & 3)] = v;
  }
  named_barrier(kQsConsumerBar, kQsConsumerWarps * 32);
  if (norm) {
    // RMSNorm row scales: warp m sums the squares of row m in the order of the
    // RMSNorm kernels (lane l: words l, l+32, ..., values 8q..8q+7 in turn),
    // so the normalised x is bit-identical to theirs
    if (warp < p.M) {
      const uint4* xr = xs + warp * (K / 8);
      float ss = 0.f;
      for (int q = lane; q < K / 8; q += 32) {
        const uint4 v = xr[qs_xs_index(q >> 2, q & 3)];
        const uint32_t pr[4] = {v.x, v.y, v.z, v.w};
        float f[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 t = Elem<DT>::unpack2(*reinterpret_cast<const typename Elem<DT>::T2*>(&pr[e]));
          f[e] = t.x;
          f[e + 4] = t.y;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
      }
      ss = warp_sum(ss);
      if (lane == 0) rscale[warp] = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), p.eps));
    }
    named_barrier(kQsConsumerBar, kQsConsumerWarps * 32);
  }
  for (int i = ct; i < MR * rowU; i += kQsConsumerWarps * 32) {
    const int m = i / rowU, u = i - m * rowU;
    const bool nrm = norm && m < p.M;
    const float sc = nrm ? rscale[m] : 0.f;
    float s = 0.f;
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
      uint4* slotp = xs + m * (K / 8) + qs_xs_index(u, wi);
      uint4 v = *slotp;
      uint32_t pr[4] = {v.x, v.y, v.z, v.w};
      const uint4 gv = nrm ? gw[4 * u + wi] : make_uint4(0, 0, 0, 0);
      const uint32_t gp[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = Elem<DT>::unpack2(*reinterpret_cast<const typename Elem<DT>::T2*>(&pr[e]));
        if (nrm) {
          // y = (x * scale) * w rounded to the element type, as the RMSNorm kernels
          const float2 g = Elem<DT>::unpack2(*reinterpret_cast<const typename Elem<DT>::T2*>(&gp[e]));
          const typename Elem<DT>::T2 y =
              Elem<DT>::pack2(__fmul_rn(__fmul_rn(f.x, sc), g.x), __fmul_rn(__fmul_rn(f.y, sc), g.y));
          pr[e] = *reinterpret_cast<const uint32_t*>(&y);
          f = Elem<DT>::unpack2(y);
        }
        s += f.x + f.y;
      }
      if (nrm) *slotp = make_uint4(pr[0], pr[1], pr[2], pr[3]);
    }
    xsum[i] = s;
  }
  named_barrier(kQsConsumerBar, kQsConsumerWarps * 32);
  bool ok = p.stage_sc ? true : mbar_wait_warp(sb_bar, 0, abort_flag, 0x502);

  constexpr int kWorkers = kQsConsumerWarps * (32 / LPR);  // row walkers
  const int sub = lane % LPR;                               // lane within the row walker
  const unsigned wmask = LPR == 32 ? 0xffffffffu : (0xffffu << (lane & 16));
  int lr = warp * (32 / LPR) + lane / LPR;  // stream row of this walker
  float acc[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) acc[m] = 0.f;
  for (int k = 0; ok && k < nstage; ++k) {
    const int slot = k % NST;
    if (!mbar_wait_warp(&full[slot], (k / NST) & 1, abort_flag, 0x503)) break;
    const int u_lo = k * stage_units;
    const int u_hi = (u_lo + stage_units < total_units) ? u_lo + stage_units : total_units;
    const uint8_t* stage = ring + slot * L.slot;
    const int r_first = p.stage_sc ? (k * stage_bytes) / rowB : 0;  // stream offsets fit 32 bits
    // scale rows: the stage's own ([spr][G] from stream row r_first) or the CTA's
    const T* stS = p.stage_sc ? reinterpret_cast<const T*>(stage + L.sc) : sbS;
    const T* stB = p.stage_sc ? stS + p.spr * G : sbB;
    const int sc_row0 = p.stage_sc ? r_first : 0;
    while (lr < srows && lr * rowU < u_hi) {
      const int r_lo = lr * rowU, r_hi = r_lo + rowU;
      const int a = r_lo > u_lo ? r_lo : u_lo;
      const int bnd = r_hi < u_hi ? r_hi : u_hi;
      const T* srow = stS + (lr - sc_row0) * G;
      const T* brow = stB + (lr - sc_row0) * G;
      for (int u = a + sub; u < bnd; u += LPR) {
        const uint4 wv = *reinterpret_cast<const uint4*>(stage + (u - u_lo) * 16);
        const int kc = u - r_lo;  // unit within the row: values [32 kc, 32 kc + 32)
        const int g = (kc * 32) >> p.gshift;
        const float s = Elem<DT>::to_f(srow[g]);
        const float bb = Elem<DT>::to_f(brow[g]);
        const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t wp[4][4];  // (C+q_i, C+q_{i+4}) of word wi, i = 0..3
#pragma unroll
        for (int wi = 0; wi < 4; ++wi)
#pragma unroll
          for (int e = 0; e < 4; ++e) wp[wi][e] = ((words[wi] >> (4 * e)) & 0x000F000Fu) | QsNib<DT>::kPair;
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          const uint4* xr = xs + m * (K / 8);
          float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            const uint4 xp = xr[qs_xs_index(kc, wi)];
            qs_fma_pair<DT>(xp.x, wp[wi][0], a0, a1);
            qs_fma_pair<DT>(xp.y, wp[wi][1], a2, a3);
            qs_fma_pair<DT>(xp.z, wp[wi][2], a0, a1);
            qs_fma_pair<DT>(xp.w, wp[wi][3], a2, a3);
          }
          acc[m] += s * ((a0 + a1) + (a2 + a3)) + (bb - QsNib<DT>::kC * s) * xsum[m * rowU + kc];
        }
      }
      if (r_hi > u_hi) break;  // the row continues in the next stage
      // row complete: reduce over the walker's lanes and write
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        float v = acc[m];
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(wmask, v, o);
        acc[m] = v;
      }
      if (sub == 0) {
        if (MODE == 2) {
#pragma unroll
          for (int m = 0; m < MR; ++m) gsum[lr * MR + m] = acc[m];
        } else {
          int sg = 0, base = 0;
          while (sg + 1 < nseg && lr >= base + seg_n[sg]) base += seg_n[sg++];
          const QsSet& st = p.set[seg_set[sg]];
          const int r = seg_row[sg] + (lr - base);
          const int ld = (MODE == 0) ? st.N : p.ldy;
          T* y = static_cast<T*>(st.y);
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            if (m >= p.M) break;
            float v = round_to<DT>(acc[m]);
            if (MODE == 1) v = v + Elem<DT>::to_f(static_cast<const T*>(p.residual)[static_cast<long long>(m) * ld + r]);
            y[static_cast<long long>(m) * ld + r] = Elem<DT>::from_f(v);
          }
        }
      }
#pragma unroll
      for (int m = 0; m < MR; ++m) acc[m] = 0.f;
      lr += kWorkers;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  if (MODE == 2) {
    // SwiGLU of the gate and up sums (rows lr and lr + nr of the stream)
    if (named_barrier_or(kQsConsumerBar, kQsConsumerWarps * 32, *abort_flag != 0)) return;
    T* y = static_cast<T*>(p.set[0].y);
    for (int i = ct; i < nr * p.M; i += kQsConsumerWarps * 32) {
      const int rl = i / p.M, m = i - rl * p.M;
      const float gs = gsum[rl * MR + m], us = gsum[(rl + nr) * MR + m];
      y[static_cast<long long>(m) * p.ldy + ra + rl] =
          Elem<DT>::from_f(swiglu_rounded<DT>(round_to<DT>(gs), round_to<DT>(us)));
    }
  }
}

// ------------------------------------------------------------------- host

static int qs_max_rows(int rows, int P, int mode) {
  return ((rows + P - 1) / P) * (mode == 2 ? 2 : 1);
}

struct QsGeometry {
  int mode, rows, P, max_rows, spr, MR, NST, stage_sc, stage_bytes;
};

// Grid, stage size and ring depth of a request: the largest stage size whose
// ring of at least 3 stages (4 at 16 KB) fits next to the CTA's scales,
// biases and staged x, scales copied once when they fit, else per stage;
// NST = 0 when nothing fits (then the register-streaming qmv kernel serves
// the request).
static QsGeometry qs_geometry(const QmmRequest& r, int sms) {
  QsGeometry g = {};
  g.mode = r.kind == QMM_SWIGLU ? 2 : r.kind == QMM_RESIDUAL ? 1 : 0;
  g.rows = g.mode == 0 ? static_cast<int>(r.set[0].N + r.set[1].N + r.set[2].N) : static_cast<int>(r.set[0].N);
  if (g.rows <= 0) return g;
  g.P = g.rows < sms ? g.rows : sms;
  g.max_rows = qs_max_rows(g.rows, g.P, g.mode);
  g.MR = r.M <= 1 ? 1 : r.M <= 2 ? 2 : 4;
  const int K = static_cast<int>(r.K), G = static_cast<int>(r.K / r.group);
  const bool norm = r.norm_w != nullptr;
  for (int sb : kQsStageSizes) {
    g.stage_bytes = sb;
    g.spr = sb / static_cast<int>(r.K / 2) + 2;
    const int min_st = sb > 16384 ? 3 : 4;
    for (g.stage_sc = 0; g.stage_sc < 2; ++g.stage_sc) {
      auto fits = [&](int nst) {
        return qs_layout(K, G, g.max_rows, g.spr, g.MR, nst, g.stage_sc, norm, sb).total + 128 <= kQsSmemLimit;
      };
      for (g.NST = kQsMaxStages; g.NST >= min_st; --g.NST)
        if (fits(g.NST)) return g;
    }
  }
  g.NST = 0;
  return g;
}

bool qmv_stream_eligible(const QmmRequest& r) {
  if (r.bits != 4 || r.M < 1 || r.M > kQsMaxMR) return false;
  if (r.dtype != MT_BF16 && r.dtype != MT_F16) return false;
  if (r.group != 32 && r.group != 64 && r.group != 128) return false;
  if (r.K % 32 != 0 || r.K > 16384 || !aligned(r.x, 16)) return false;
  if (r.norm_w && !aligned(r.norm_w, 16)) return false;
  const int G = static_cast<int>(r.K / r.group);
  if ((G * 2) % 16 != 0) return false;  // scale rows must be 16-byte multiples for the bulk copies
  const int nsets = r.kind == QMM_SWIGLU ? 2 : 3;
  for (int s = 0; s < nsets; ++s) {
    if (r.set[s].N <= 0) continue;
    if (!aligned(r.set[s].w, 16) || !aligned(r.set[s].s, 16) || !aligned(r.set[s].b, 16)) return false;
  }
  int sms = 148;
  if (device_sm_count(&sms) != MT_OK) return false;
  const QsGeometry g = qs_geometry(r, sms);
  return g.rows > 0 && g.NST > 0;
}

template <int DT, int MR, int MODE>
static int qs_launch(QsParams& p, cudaStream_t stream) {
  const QsLayout L = qs_layout(p.K, p.G, p.max_rows, p.spr, MR, p.NST, p.stage_sc, p.norm_w != nullptr, p.stage_bytes);
  // half-warp rows up to 128 units (K <= 4096); longer rows keep whole warps,
  // since 32 walkers over long rows would span more stages than the ring holds
  // (measured at K = 2560: gate_up 14.8 -> 13.2 us; K = 9728: 8.6 -> 10.2 us)
  auto k = (p.K / 32 <= 128) ? qmv_stream_kernel<DT, MR, MODE, 16> : qmv_stream_kernel<DT, MR, MODE, 32>;
  if (int e = ensure_smem(k, kQsSmemLimit)) return e;
  return launch(k, dim3(p.P), dim3(kQsThreads), static_cast<size_t>(L.total) + 128, stream, p);
}

template <int DT, int MODE>
static int qs_dispatch_mr(QsParams& p, cudaStream_t stream) {
  if (p.M <= 1) return qs_launch<DT, 1, MODE>(p, stream);
  if (p.M <= 2) return qs_launch<DT, 2, MODE>(p, stream);
  return qs_launch<DT, 4, MODE>(p, stream);
}

int qmv_stream_run(const QmmRequest& r, cudaStream_t stream) {
  int sms = 148;
  if (int rc = device_sm_count(&sms)) return rc;
  QsParams p = {};
  p.x = r.x;
  p.residual = r.residual;
  p.norm_w = r.norm_w;
  p.eps = r.norm_eps;
  p.M = static_cast<int>(r.M);
  p.K = static_cast<int>(r.K);
  p.G = static_cast<int>(r.K / r.group);
  p.gshift = r.group == 32 ? 5 : r.group == 64 ? 6 : 7;
  p.ldx = static_cast<int>(r.K);
  const int mode = r.kind == QMM_SWIGLU ? 2 : r.kind == QMM_RESIDUAL ? 1 : 0;
  int total = 0;
  p.row_start[0] = 0;
  for (int s = 0; s < 3; ++s) {
    p.set[s] = {static_cast<const uint8_t*>(static_cast<const void*>(r.set[s].w)),
                static_cast<const uint8_t*>(r.set[s].s), static_cast<const uint8_t*>(r.set[s].b), r.set[s].y,
                static_cast<int>(r.set[s].N)};
    if (mode == 0) total += static_cast<int>(r.set[s].N);
    p.row_start[s + 1] = total;
  }
  p.ldy = static_cast<int>(r.set[0].N);
  const QsGeometry g = qs_geometry(r, sms);
  if (g.rows <= 0) return MT_OK;
  if (g.NST == 0) {
    set_error("qmv: K=%d with %d rows per CTA does not fit shared memory", p.K, g.max_rows);
    return MT_ERR_UNSUPPORTED;
  }
  p.rows = g.rows;
  p.P = g.P;
  p.max_rows = g.max_rows;
  p.spr = g.spr;
  p.stage_sc = g.stage_sc;
  p.stage_bytes = g.stage_bytes;
  p.NST = g.NST;
  if (r.dtype == MT_BF16) {
    if (mode == 2) return qs_dispatch_mr<MT_BF16, 2>(p, stream);
    if (mode == 1) return qs_dispatch_mr<MT_BF16, 1>(p, stream);
    return qs_dispatch_mr<MT_BF16, 0>(p, stream);
  }
  if (mode == 2) return qs_dispatch_mr<MT_F16, 2>(p, stream);
  if (mode == 1) return qs_dispatch_mr<MT_F16, 1>(p, stream);
  return qs_dispatch_mr<MT_F16, 0>(p, stream);
}

}  // namespace mt
