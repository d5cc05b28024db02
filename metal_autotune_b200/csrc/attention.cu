// Causal GQA scaled-dot-product attention, flash-style (online softmax).
//
// One CTA = 4 warps = 64 query rows of one (batch, head); each warp owns 16
// rows. K/V blocks of 64 keys are double-buffered in shared memory with
// cp.async (XOR-swizzled 16-byte chunks so ldmatrix is conflict-free).
// S = Q K^T and O += P V run on mma.sync m16n8k16 (bf16/fp16 in, fp32
// accumulate); softmax statistics stay in fp32 registers, P is rounded to
// the input type for the P V product. Causal blocks past the diagonal are
// never loaded. At the Qwen3 prefill size (L = 128, 32 heads) the whole op
// is a few microseconds and latency-bound.
#include "mt_common.cuh"
#include "mma_sync.cuh"
#include "rope_common.cuh"

namespace mt {

struct SdpaParams {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  int64_t qs_b, qs_h, qs_l, ks_b, ks_h, ks_l, vs_b, vs_h, vs_l, os_b, os_h, os_l;
  int Hq, Hkv, Lq, Lk;
  int64_t q_offset;
  float scale_log2;  // scale * log2(e)
  int causal;
};

// byte offset of 16-byte chunk c of row r in a tile whose rows are D*2 bytes
template <int D>
__device__ __forceinline__ int swz(int r, int c) {
  return r * (D * 2) + ((c ^ (r & 7)) << 4);
}

template <int DT, int D>
__global__ void __launch_bounds__(128) sdpa_kernel(const SdpaParams p) {
  using T = typename Elem<DT>::T;
  constexpr int BQ = 64, BKV = 64;
  constexpr int CH = D / 8;  // 16-byte chunks per row
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* sq = sm;
  uint8_t* sk = sm + BQ * D * 2;           // 2 buffers
  uint8_t* sv = sk + 2 * BKV * D * 2;      // 2 buffers

  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.Hq / p.Hkv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q0 = qb * BQ;
  const T* qg = static_cast<const T*>(p.q) + b * p.qs_b + h * p.qs_h;
  const T* kg = static_cast<const T*>(p.k) + b * p.ks_b + kvh * p.ks_h;
  const T* vg = static_cast<const T*>(p.v) + b * p.vs_b + kvh * p.vs_h;

  griddep_wait();

  griddep_launch();  // dependents may launch now; their own wait covers this grid
  // keys this block can see: causal limit of its last query row
  int kend = p.Lk;
  if (p.causal) {
    const int64_t lim = p.q_offset + q0 + BQ;  // exclusive
    if (lim < kend) kend = static_cast<int>(lim < 0 ? 0 : lim);
  }
  const int nkb = (kend + BKV - 1) / BKV;

  for (int i = tid; i < BQ * CH; i += 128) {
    const int r = i / CH, c = i % CH;
    const bool ok = q0 + r < p.Lq;
    cp_async16(sq + swz<D>(r, c), qg + static_cast<int64_t>(ok ? q0 + r : 0) * p.qs_l + c * 8, ok);
  }
  auto load_kv = [&](int kb, int buf) {
    for (int i = tid; i < BKV * CH; i += 128) {
      const int r = i / CH, c = i % CH;
      const int key = kb * BKV + r;
      const bool ok = key < p.Lk;
      const int kk = ok ? key : 0;
      cp_async16(sk + buf * BKV * D * 2 + swz<D>(r, c), kg + static_cast<int64_t>(kk) * p.ks_l + c * 8, ok);
      cp_async16(sv + buf * BKV * D * 2 + swz<D>(r, c), vg + static_cast<int64_t>(kk) * p.vs_l + c * 8, ok);
    }
  };
  if (nkb > 0) load_kv(0, 0);
  cp_async_commit();

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const int g = lane >> 2, t4 = lane & 3;
  const int row0 = q0 + warp * 16 + g;  // rows row0 and row0 + 8

  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) load_kv(kb + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    const uint32_t qbase = smem_addr(sq);
    const uint32_t kbase = smem_addr(sk + buf * BKV * D * 2);
    const uint32_t vbase = smem_addr(sv + buf * BKV * D * 2);
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4];
      {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kk * 2 + (lane >> 4);
        ldsm_x4(qbase + swz<D>(r, c), a[0], a[1], a[2], a[3]);
      }
#pragma unroll
      for (int nt = 0; nt < 8; nt += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = nt * 8 + (lane & 7) + (lane >> 4) * 8;
        const int c = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4(kbase + swz<D>(r, c), b0, b1, b2, b3);
        mma16816<DT>(s[nt], a, b0, b1);
        mma16816<DT>(s[nt + 1], a, b2, b3);
      }
    }
    // scale, mask, online softmax
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kb * BKV + nt * 8 + 2 * t4 + (e & 1);
        const int qi = row0 + (e >> 1) * 8;
        float v = s[nt][e] * p.scale_log2;
        const bool ok = key < p.Lk && (!p.causal || key <= p.q_offset + qi);
        v = ok ? v : -INFINITY;
        s[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float corr[2], base[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float mnew = fmaxf(m_r[r], mx[r]);
      base[r] = mnew == -INFINITY ? 0.f : mnew;
      corr[r] = exp2f(m_r[r] - base[r]);
      m_r[r] = mnew;
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pa[4][4];  // P as A fragments, 4 chunks of 16 keys
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = exp2f(s[nt][0] - base[0]);
      const float p1 = exp2f(s[nt][1] - base[0]);
      const float p2 = exp2f(s[nt][2] - base[1]);
      const float p3 = exp2f(s[nt][3] - base[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      const int ch = nt >> 1, hi = nt & 1;
      pa[ch][hi * 2 + 0] = pack2<DT>(p0, p1);
      pa[ch][hi * 2 + 1] = pack2<DT>(p2, p3);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_r[r] = l_r[r] * corr[r] + rs[r];
    }
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      o[dt][0] *= corr[0];
      o[dt][1] *= corr[0];
      o[dt][2] *= corr[1];
      o[dt][3] *= corr[1];
    }
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      // A fragment order: (row g, k lo), (row g+8, k lo), (row g, k hi), (row g+8, k hi)
      const uint32_t a[4] = {pa[ch][0], pa[ch][1], pa[ch][2], pa[ch][3]};
#pragma unroll
      for (int dt = 0; dt < D / 8; dt += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = ch * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = dt + (lane >> 4);
        ldsm_x4_t(vbase + swz<D>(r, c), b0, b1, b2, b3);
        mma16816<DT>(o[dt], a, b0, b1);
        mma16816<DT>(o[dt + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }
  T* og = static_cast<T*>(p.o) + b * p.os_b + h * p.os_h;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = row0 + r * 8;
    if (qi >= p.Lq) continue;
    const float inv = l_r[r] > 0.f ? 1.f / l_r[r] : 0.f;
    T* dst = og + static_cast<int64_t>(qi) * p.os_l;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      const int d = dt * 8 + 2 * t4;
      const uint32_t packed = pack2<DT>(o[dt][2 * r] * inv, o[dt][2 * r + 1] * inv);
      *reinterpret_cast<uint32_t*>(dst + d) = packed;
    }
  }
}

// ------------------------------------------------------------ decode
// Qwen3 decode attention with its prologue fused in (T <= 4 new tokens,
// G*T <= 16 query rows):
// one CTA per kv head h. The CTA q/k-norms and ropes the G = Hq/Hkv query
// heads of its group for the T tokens (rows r = g*T + t of one 16-row MMA
// tile, G*T <= 16) and the T new k rows, appends k'/v to the caches at
// offset..offset+T-1 (the only writer of head h's rows), then its 8 warps
// split the keys [0, offset+T) in blocks of 32 (warp w: blocks w, w+8, ...),
// each with its own online softmax over its blocks, and the CTA merges the 8
// (max, sum, O) partials through shared memory. The q/k rows come from the
// same routine as mt_qk_norm_rope_cache (bit-identical caches); the softmax
// is the flash form of sdpa_kernel with the keys split across warps.
constexpr int kDaWarps = 8, kDaKeys = 32, kDaD = 128;
constexpr int kDaRowBytes = kDaD * 2;
constexpr int kDaQBytes = 16 * kDaRowBytes;                      // the 16-row q tile
constexpr int kDaWarpKV = 2 * kDaKeys * kDaRowBytes;             // one warp's K and V block
constexpr int kDaSmem = kDaQBytes + kDaWarps * kDaWarpKV;        // 132 KB
static_assert(kDaWarps * 16 * kDaD * 4 + kDaWarps * 16 * 2 * 4 <= kDaWarps * kDaWarpKV,
              "the merge area reuses the K/V blocks");

struct DecodeAttnParams {
  const void* q;  // [T, Hq*128] raw projections, rows q_stride apart
  const void* k;  // [T, Hkv*128], rows kv_stride apart
  const void* v;
  int64_t q_stride, kv_stride;
  const void* q_norm_w;
  const void* k_norm_w;
  float eps;
  void* o;  // [T, Hq*128]
  void* k_cache;  // [Hkv, cap, 128]
  void* v_cache;
  int T, Hq, Hkv;
  int64_t cap, offset;
  float scale_log2;
};

// ITEMS: prologue rows per warp (R + T rows over 8 warps: 1 when R + T <= 8,
// the Qwen3 decode case, which keeps one inlined copy of the norm + RoPE code)
template <int DT, int ITEMS>
__global__ void __launch_bounds__(kDaWarps * 32, 1)
    decode_attn_kernel(const __grid_constant__ DecodeAttnParams p, const __grid_constant__ RopeFreqs f) {
  using T = typename Elem<DT>::T;
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* sq = sm;
  uint8_t* skv = sm + kDaQBytes;
  const int hk = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = p.Hq / p.Hkv, Tn = p.T, R = G * Tn;

  griddep_wait();
  griddep_launch();  // dependents may launch now; their own wait covers this grid

  const int L = static_cast<int>(p.offset) + Tn;  // keys
  const int nkb = (L + kDaKeys - 1) / kDaKeys;
  const int old = static_cast<int>(p.offset);       // keys already in the caches
  const T* kg = static_cast<const T*>(p.k_cache) + static_cast<int64_t>(hk) * p.cap * kDaD;
  const T* vg = static_cast<const T*>(p.v_cache) + static_cast<int64_t>(hk) * p.cap * kDaD;
  uint8_t* wk = skv + warp * kDaWarpKV;
  uint8_t* wv = wk + kDaKeys * kDaRowBytes;
  const uint32_t qbase = smem_addr(sq), kbase = smem_addr(wk), vbase = smem_addr(wv);
  // key block kb of K and V into this warp's buffers (16-byte chunks,
  // swizzled rows); keys >= L are zero-filled; with `skip_new` the keys
  // offset..L-1 are left to the prologue, which writes them directly
  auto load_block = [&](int kb, bool skip_new) {
    for (int i = lane; i < kDaKeys * (kDaD / 8); i += 32) {
      const int r = i >> 4, c = i & 15;
      const int key = kb * kDaKeys + r;
      if (skip_new && key >= old && key < L) continue;
      const bool ok = key < L;
      const int kk = ok ? key : 0;
      cp_async16(wk + swz<kDaD>(r, c), kg + static_cast<int64_t>(kk) * kDaD + c * 8, ok);
      cp_async16(wv + swz<kDaD>(r, c), vg + static_cast<int64_t>(kk) * kDaD + c * 8, ok);
    }
    cp_async_commit();
  };
  // the first pass of blocks (one per warp) is fetched while the prologue runs
  if (warp < nkb) load_block(warp, true);

  // prologue: items i = warp, warp + 8, ... over the R q rows, then the T
  // new k rows; every item's loads are issued before any is computed
  constexpr int kItems = ITEMS;  // R + T <= ITEMS * kDaWarps
  uint2 xr[kItems], wr[kItems], vr[kItems];
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const int i = warp + j * kDaWarps;
    xr[j] = wr[j] = vr[j] = make_uint2(0, 0);
    if (i < R) {
      const int g = i / Tn, t = i - g * Tn;
      xr[j] = *reinterpret_cast<const uint2*>(static_cast<const T*>(p.q) + t * p.q_stride +
                                              static_cast<int64_t>(hk * G + g) * kDaD + 4 * lane);
      wr[j] = *reinterpret_cast<const uint2*>(static_cast<const T*>(p.q_norm_w) + 4 * lane);
    } else if (i < R + Tn) {
      const int t = i - R;
      const int64_t off = t * p.kv_stride + static_cast<int64_t>(hk) * kDaD + 4 * lane;
      xr[j] = *reinterpret_cast<const uint2*>(static_cast<const T*>(p.k) + off);
      vr[j] = *reinterpret_cast<const uint2*>(static_cast<const T*>(p.v) + off);
      wr[j] = *reinterpret_cast<const uint2*>(static_cast<const T*>(p.k_norm_w) + 4 * lane);
    }
  }
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const int i = warp + j * kDaWarps;
    if (i < R) {
      const int g = i / Tn, t = i - g * Tn;
      const uint2 out = qk_norm_rope_vals<DT>(xr[j], wr[j], p.eps, p.offset + t, f, lane);
      *reinterpret_cast<uint2*>(sq + swz<kDaD>(i, lane >> 1) + (lane & 1) * 8) = out;
    } else if (i < R + Tn) {
      const int t = i - R;
      const uint2 kr = qk_norm_rope_vals<DT>(xr[j], wr[j], p.eps, p.offset + t, f, lane);
      const int key = old + t;
      const int64_t crow = static_cast<int64_t>(hk) * p.cap + key;
      *reinterpret_cast<uint2*>(static_cast<T*>(p.k_cache) + crow * kDaD + 4 * lane) = kr;
      *reinterpret_cast<uint2*>(static_cast<T*>(p.v_cache) + crow * kDaD + 4 * lane) = vr[j];
      const int kb = key / kDaKeys;
      if (kb < kDaWarps) {
        // the block is in the first pass: straight into its warp's buffers
        uint8_t* bk = skv + kb * kDaWarpKV;
        const int r = key - kb * kDaKeys;
        *reinterpret_cast<uint2*>(bk + swz<kDaD>(r, lane >> 1) + (lane & 1) * 8) = kr;
        *reinterpret_cast<uint2*>(bk + kDaKeys * kDaRowBytes + swz<kDaD>(r, lane >> 1) + (lane & 1) * 8) = vr[j];
      }
    }
  }
  for (int i = R + warp; i < 16; i += kDaWarps)  // q-tile rows past the group's rows
    *reinterpret_cast<uint2*>(sq + swz<kDaD>(i, lane >> 1) + (lane & 1) * 8) = make_uint2(0, 0);
  // later passes read new keys back from the caches
  if (nkb > kDaWarps) __threadfence();
  __syncthreads();

  float o[kDaD / 8][4];
#pragma unroll
  for (int i = 0; i < kDaD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const int g8 = lane >> 2, t4 = lane & 3;
  // the last key each of this thread's two rows may see (-1: not a row)
  int lim[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int r = g8 + e * 8;
    lim[e] = r < R ? static_cast<int>(p.offset) + (r % Tn) : -1;
  }

  for (int kb = warp; kb < nkb; kb += kDaWarps) {
    if (kb >= kDaWarps) load_block(kb, false);
    cp_async_wait<0>();
    __syncwarp();

    float s[kDaKeys / 8][4];
#pragma unroll
    for (int i = 0; i < kDaKeys / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kDaD / 16; ++kk) {
      uint32_t a[4];
      {
        const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kk * 2 + (lane >> 4);
        ldsm_x4(qbase + swz<kDaD>(r, c), a[0], a[1], a[2], a[3]);
      }
#pragma unroll
      for (int nt = 0; nt < kDaKeys / 8; nt += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = nt * 8 + (lane & 7) + (lane >> 4) * 8;
        const int c = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4(kbase + swz<kDaD>(r, c), b0, b1, b2, b3);
        mma16816<DT>(s[nt], a, b0, b1);
        mma16816<DT>(s[nt + 1], a, b2, b3);
      }
    }
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < kDaKeys / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kb * kDaKeys + nt * 8 + 2 * t4 + (e & 1);
        float v = s[nt][e] * p.scale_log2;
        v = key <= lim[e >> 1] ? v : -INFINITY;
        s[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float corr[2], base[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float mnew = fmaxf(m_r[r], mx[r]);
      base[r] = mnew == -INFINITY ? 0.f : mnew;
      corr[r] = exp2f(m_r[r] - base[r]);
      m_r[r] = mnew;
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pa[kDaKeys / 16][4];  // P as A fragments, chunks of 16 keys
#pragma unroll
    for (int nt = 0; nt < kDaKeys / 8; ++nt) {
      const float p0 = exp2f(s[nt][0] - base[0]);
      const float p1 = exp2f(s[nt][1] - base[0]);
      const float p2 = exp2f(s[nt][2] - base[1]);
      const float p3 = exp2f(s[nt][3] - base[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      const int ch = nt >> 1, hi = nt & 1;
      pa[ch][hi * 2 + 0] = pack2<DT>(p0, p1);
      pa[ch][hi * 2 + 1] = pack2<DT>(p2, p3);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_r[r] = l_r[r] * corr[r] + rs[r];
    }
#pragma unroll
    for (int dt = 0; dt < kDaD / 8; ++dt) {
      o[dt][0] *= corr[0];
      o[dt][1] *= corr[0];
      o[dt][2] *= corr[1];
      o[dt][3] *= corr[1];
    }
#pragma unroll
    for (int ch = 0; ch < kDaKeys / 16; ++ch) {
      const uint32_t a[4] = {pa[ch][0], pa[ch][1], pa[ch][2], pa[ch][3]};
#pragma unroll
      for (int dt = 0; dt < kDaD / 8; dt += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = ch * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = dt + (lane >> 4);
        ldsm_x4_t(vbase + swz<kDaD>(r, c), b0, b1, b2, b3);
        mma16816<DT>(o[dt], a, b0, b1);
        mma16816<DT>(o[dt + 1], a, b2, b3);
      }
    }
    __syncwarp();  // the block is consumed before the next one overwrites it
  }

  // merge the warps' partials: O [warp][16][128] and (max, sum) [warp][16]
  __syncthreads();
  float* mo = reinterpret_cast<float*>(skv);
  float* mml = mo + kDaWarps * 16 * kDaD;
#pragma unroll
  for (int dt = 0; dt < kDaD / 8; ++dt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = g8 + (e >> 1) * 8, d = dt * 8 + 2 * t4 + (e & 1);
      mo[(warp * 16 + r) * kDaD + d] = o[dt][e];
    }
  if (t4 == 0) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      mml[(warp * 16 + g8 + e * 8) * 2 + 0] = m_r[e];
      mml[(warp * 16 + g8 + e * 8) * 2 + 1] = l_r[e];
    }
  }
  __syncthreads();
  // thread: row tid / 16, values 8 (tid % 16) .. + 7
  const int r = tid >> 4, d0 = (tid & 15) * 8;
  if (r < R) {
    float mstar = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDaWarps; ++w) mstar = fmaxf(mstar, mml[(w * 16 + r) * 2]);
    float wsc[kDaWarps], lsum = 0.f;
#pragma unroll
    for (int w = 0; w < kDaWarps; ++w) {
      const float mw = mml[(w * 16 + r) * 2];
      wsc[w] = mw == -INFINITY ? 0.f : exp2f(mw - mstar);
      lsum += mml[(w * 16 + r) * 2 + 1] * wsc[w];
    }
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
    for (int w = 0; w < kDaWarps; ++w) {
      const float4* src = reinterpret_cast<const float4*>(mo + (w * 16 + r) * kDaD + d0);
      const float4 x0 = src[0], x1 = src[1];
      acc[0] += x0.x * wsc[w];
      acc[1] += x0.y * wsc[w];
      acc[2] += x0.z * wsc[w];
      acc[3] += x0.w * wsc[w];
      acc[4] += x1.x * wsc[w];
      acc[5] += x1.y * wsc[w];
      acc[6] += x1.z * wsc[w];
      acc[7] += x1.w * wsc[w];
    }
    const int g = r / Tn, t = r - g * Tn;
    uint4 out;
    out.x = pack2<DT>(acc[0] * inv, acc[1] * inv);
    out.y = pack2<DT>(acc[2] * inv, acc[3] * inv);
    out.z = pack2<DT>(acc[4] * inv, acc[5] * inv);
    out.w = pack2<DT>(acc[6] * inv, acc[7] * inv);
    T* og = static_cast<T*>(p.o) + static_cast<int64_t>(t) * p.Hq * kDaD + static_cast<int64_t>(hk * G + g) * kDaD;
    *reinterpret_cast<uint4*>(og + d0) = out;
  }
}

}  // namespace mt

using namespace mt;

extern "C" int mt_qk_norm_rope_sdpa_decode(const void* q, const void* k, const void* v, int64_t q_stride,
                                           int64_t kv_stride, const void* q_norm_w, const void* k_norm_w,
                                           float eps, void* o, void* k_cache, void* v_cache, int64_t T, int64_t Hq,
                                           int64_t Hkv, int64_t D, int64_t cache_cap, int64_t offset,
                                           float rope_base, float scale, int dtype, mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(q && k && v && q_norm_w && k_norm_w && o && k_cache && v_cache,
               "mt_qk_norm_rope_sdpa_decode: null pointer");
  MT_CHECK_ARG(D == 128, "mt_qk_norm_rope_sdpa_decode: head_dim %lld, only 128 is built", (long long)D);
  MT_CHECK_ARG(dtype == MT_BF16 || dtype == MT_F16, "mt_qk_norm_rope_sdpa_decode: dtype must be bf16 or f16");
  MT_CHECK_ARG(Hq > 0 && Hkv > 0 && Hq % Hkv == 0 && Hkv < 65536,
               "mt_qk_norm_rope_sdpa_decode: Hq=%lld must be a multiple of Hkv=%lld", (long long)Hq, (long long)Hkv);
  MT_CHECK_ARG(T >= 0 && T <= 4 && (Hq / Hkv) * T <= 16,
               "mt_qk_norm_rope_sdpa_decode: T = %lld tokens, (Hq/Hkv) * T = %lld query rows per kv head; "
               "decode takes at most 4 tokens and 16 rows",
               (long long)T, (long long)((Hq / Hkv) * T));
  MT_CHECK_ARG(offset >= 0 && offset + T <= cache_cap && cache_cap < (int64_t(1) << 30),
               "mt_qk_norm_rope_sdpa_decode: offset %lld + T %lld exceeds cache capacity %lld", (long long)offset,
               (long long)T, (long long)cache_cap);
  MT_CHECK_ARG(q_stride % 4 == 0 && kv_stride % 4 == 0 && aligned(q, 8) && aligned(k, 8) && aligned(v, 8) &&
                   aligned(k_cache, 16) && aligned(v_cache, 16) && aligned(o, 16),
               "mt_qk_norm_rope_sdpa_decode: q/k/v rows must be 8-byte aligned, caches and output 16-byte aligned");
  if (T == 0) return MT_OK;
  DecodeAttnParams p = {q, k, v, q_stride, kv_stride, q_norm_w, k_norm_w, eps, o, k_cache, v_cache,
                        (int)T, (int)Hq, (int)Hkv, cache_cap, offset, scale * 1.4426950408889634f};
  const RopeFreqs f = make_freqs(128, rope_base);
  auto run = [&](auto kern) -> int {
    if (int e = ensure_smem(kern, kDaSmem)) return e;
    return launch(kern, dim3(static_cast<unsigned>(Hkv)), dim3(kDaWarps * 32), kDaSmem, (cudaStream_t)stream, p, f);
  };
  const bool one = (Hq / Hkv) * T + T <= kDaWarps;
  if (dtype == MT_BF16) return one ? run(decode_attn_kernel<MT_BF16, 1>) : run(decode_attn_kernel<MT_BF16, 3>);
  return one ? run(decode_attn_kernel<MT_F16, 1>) : run(decode_attn_kernel<MT_F16, 3>);
}

namespace mt {
int attn_tc_run(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t Hq, int64_t Hkv, int64_t Lq,
                int64_t Lk, int64_t D, float scale, int causal, int64_t q_offset, int64_t qs_b, int64_t qs_h,
                int64_t qs_l, int64_t ks_b, int64_t ks_h, int64_t ks_l, int64_t vs_b, int64_t vs_h, int64_t vs_l,
                int64_t os_b, int64_t os_h, int64_t os_l, int dtype, cudaStream_t stream);
}

extern "C" int mt_sdpa(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t Hq, int64_t Hkv,
                       int64_t Lq, int64_t Lk, int64_t D, float scale, int causal, int64_t q_offset, int64_t qs_b,
                       int64_t qs_h, int64_t qs_l, int64_t ks_b, int64_t ks_h, int64_t ks_l, int64_t vs_b,
                       int64_t vs_h, int64_t vs_l, int64_t os_b, int64_t os_h, int64_t os_l, int dtype,
                       mt_stream_t stream) {
  clear_error();
  MT_CHECK_ARG(q && k && v && o, "mt_sdpa: null pointer");
  MT_CHECK_ARG(D == 64 || D == 128, "mt_sdpa: head_dim %lld, only 64 and 128 are built", (long long)D);
  MT_CHECK_ARG(dtype == MT_BF16 || dtype == MT_F16, "mt_sdpa: dtype must be bf16 or f16");
  MT_CHECK_ARG(B >= 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0, "mt_sdpa: Hq=%lld must be a multiple of Hkv=%lld",
               (long long)Hq, (long long)Hkv);
  MT_CHECK_ARG(Lq >= 0 && Lk >= 0 && Lq < (1 << 30) && Lk < (1 << 30), "mt_sdpa: bad lengths");
  MT_CHECK_ARG(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(o, 4) && qs_l % 8 == 0 &&
                   ks_l % 8 == 0 && vs_l % 8 == 0 && qs_h % 8 == 0 && ks_h % 8 == 0 && vs_h % 8 == 0 &&
                   qs_b % 8 == 0 && ks_b % 8 == 0 && vs_b % 8 == 0 && os_l % 2 == 0,
               "mt_sdpa: q/k/v rows must be 16-byte aligned");
  if (B == 0 || Lq == 0) return MT_OK;
  // tensor-core flash attention (tcgen05, TMA) for sequences of several key
  // blocks in any layout TMA can address (measured on B200: Llama-3-8B
  // prefill [8, 32/8, 2048, 128] causal 1040 -> 512 us, mlx-whisper encoder
  // [8, 20, 1500, 64] 406 -> 254 us); short ones (the Qwen3 prefill, 128 x 128
  // per head: 5.4 us here against 7.0 us there, the tensor-memory set-up of a
  // one-block CTA not amortised) and other layouts stay on the mma.sync kernel
  const int tc = (Lq < 64 || Lk < 384) ? MT_ERR_UNSUPPORTED : attn_tc_run(q, k, v, o, B, Hq, Hkv, Lq, Lk, D, scale, causal, q_offset, qs_b, qs_h, qs_l, ks_b, ks_h,
                             ks_l, vs_b, vs_h, vs_l, os_b, os_h, os_l, dtype, (cudaStream_t)stream);
  if (tc != MT_ERR_UNSUPPORTED) return tc;
  clear_error();
  SdpaParams p = {q, k, v, o, qs_b, qs_h, qs_l, ks_b, ks_h, ks_l, vs_b, vs_h, vs_l, os_b, os_h, os_l,
                  (int)Hq, (int)Hkv, (int)Lq, (int)Lk, q_offset, scale * 1.4426950408889634f, causal};
  const dim3 grid(static_cast<unsigned>((Lq + 63) / 64), static_cast<unsigned>(Hq), static_cast<unsigned>(B));
  const size_t smem = static_cast<size_t>(64 * D * 2) * 5;
  auto run = [&](auto kern) -> int {
    if (int e = ensure_smem(kern, smem)) return e;
    return launch(kern, grid, dim3(128), smem, (cudaStream_t)stream, p);
  };
  if (dtype == MT_BF16) return D == 128 ? run(sdpa_kernel<MT_BF16, 128>) : run(sdpa_kernel<MT_BF16, 64>);
  return D == 128 ? run(sdpa_kernel<MT_F16, 128>) : run(sdpa_kernel<MT_F16, 64>);
}
