/*
 * mt.h — C ABI of libmt.so, the B200 (sm_100a) region kernels.
 *
 * Every entry point is `extern "C"`, takes plain device pointers and integer
 * sizes, launches on the caller's `cudaStream_t` (always the last argument)
 * and returns an int: MT_OK (0) or a negative MT_ERR_* code, with a message
 * in mt_last_error_string() (thread-local). The caller owns every buffer. No
 * entry point allocates device memory: kernels that need scratch space take
 * a caller-provided workspace and report its size through a *_workspace
 * query. All tensors are dense row-major unless a stride argument says
 * otherwise. Launches are asynchronous; argument errors are reported before
 * anything is enqueued.
 *
 * Workspaces: the first 64 KiB of a workspace are control words (flags and
 * counters at fixed offsets) that every kernel leaves zero when it completes;
 * data regions start at 64 KiB. One zero-filled workspace can therefore be
 * shared by all calls issued in order on one stream.
 *
 * Each declaration names the reference interface it replaces (file:line in
 * shivamg05/metal-autotune). The reference dispatches these regions through
 * autotuner_runtime/kernels.py:247-268 (`call` / `try_call` / `try_sized`)
 * into MLX ops or `mx.fast.metal_kernel`; the arithmetic itself is MLX 0.32.2
 * (quantized_matmul, fast.rms_norm, fast.rope, fast.scaled_dot_product_attention,
 * fast.layer_norm) and mlx-lm 0.31.3 (swiglu, Qwen3/Llama/Mamba model code).
 */
#ifndef MT_H_
#define MT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* mt_stream_t; /* binary-compatible with cudaStream_t */

/* Element types (the `dtype` argument). */
enum {
  MT_BF16 = 0,
  MT_F16 = 1,
  MT_F32 = 2,
  MT_I32 = 3,
  MT_U32 = 4,
  MT_I64 = 5,
  MT_U8 = 6,
  MT_BOOL = 7,
  MT_I8 = 8,
  MT_I16 = 9,
  MT_U16 = 10,
  MT_U64 = 11
};

/* Return codes. */
enum {
  MT_OK = 0,
  MT_ERR_INVALID_ARGUMENT = -1, /* shapes, dtypes, pointers or alignment rejected */
  MT_ERR_UNSUPPORTED = -2,      /* valid request this build does not cover      */
  MT_ERR_WORKSPACE = -3,        /* workspace missing or too small               */
  MT_ERR_CUDA = -4,             /* a CUDA runtime/driver call failed            */
  MT_ERR_DEVICE_TIMEOUT = -5    /* a kernel's bounded wait expired (device flag) */
};

/* Library version, (major << 16) | (minor << 8) | patch. */
int mt_version(void);

/* Message for the last error on this host thread ("" when none). */
const char* mt_last_error_string(void);

/*
 * Device-side status word of the current device: 0 when every kernel's
 * bounded waits completed, else the first MT_ERR_DEVICE_TIMEOUT site code.
 * Synchronises the device. `clear` != 0 resets it to 0.
 */
int mt_device_status(int* status_out, int clear);

/* Number of streaming multiprocessors of the current device (host query). */
int mt_sm_count(int* sm_count_out);

/*
 * Kernels this library has launched in the process so far: a host-side count
 * of successful launches (one entry point may launch several kernels; a
 * launch recorded into a CUDA graph counts once, when it is captured).
 * Library plumbing, no reference counterpart.
 */
uint64_t mt_kernel_launches(void);

/* ------------------------------------------------------------------------ */
/* a-1 / a-2: MLX-affine quantized matmul, y = x · dequant(w)^T              */
/* ------------------------------------------------------------------------ */
/*
 * Replaces mx.quantized_matmul(x, w, scales, biases, transpose=True,
 * group_size, bits, mode="affine") as the reference restates it in
 * autotuner/scaffold/lower.py:468-514 (layout) and :1179-1234 (math); the
 * stitched library kernels it must agree with are autotuner/scaffold/stitch.py:176
 * (qmv, decode) and :246 (qmm_t, prefill).
 *
 *   x       [M, K]      dtype (bf16 / f16), rows of the flattened leading dims
 *   w       [N, K*bits/32] uint32, value j of a word at bits [j*bits, (j+1)*bits)
 *   scales  [N, K/group_size] dtype
 *   biases  [N, K/group_size] dtype
 *   y       [M, N]      dtype
 *
 * Dequantisation follows MLX: w = round(round(scale*q) + bias) in the
 * element type; products accumulate in fp32. group_size = 64, 128 or 32;
 * bits = 4 or 8; K a multiple of group_size and of 128 / bits * 8.
 * M <= 8 runs the vector kernel (qmv); larger M the tcgen05/TMEM kernel,
 * which may split K and then needs `workspace` (see mt_qmm_workspace_bytes;
 * the workspace must be zero-filled once before first use, and every call
 * that completes leaves the counters at its start zeroed). From 1024 rows of
 * x (environment variable MT_QMM_GEMM_MIN_ROWS overrides it), given the
 * workspace mt_qmm_workspace_bytes asks for, the weights are dequantised into
 * the workspace past those counters and multiplied on the tcgen05 GEMM of
 * mt_linear: same dequantised values, fp32 sums in another order.
 * A product whose x rows or weight rows exceed an L2-sized block (60 MB of
 * operand bytes; environment variable MT_QMM_L2_BLOCK_BYTES overrides it) is
 * issued as several launches on `stream`, one per block, reusing the same
 * workspace in turn.
 */
int mt_quantized_matmul(const void* x, const uint32_t* w, const void* scales,
                        const void* biases, void* y, int64_t M, int64_t N,
                        int64_t K, int group_size, int bits, int dtype,
                        void* workspace, size_t workspace_bytes,
                        mt_stream_t stream);

/*
 * Host-only check of the prefill kernel's work partition (no GPU needed): C
 * thread-block clusters of S CTAs over `tiles` x `nk` K-stages, each cluster's
 * unit range split by tile segment and each segment by K among its CTAs.
 * Verifies that every K-stage of every tile is computed exactly once, that
 * every tile split across CTAs has exactly one owner reducing it from
 * partials that are all produced, each workspace partial slot written at most
 * once per CTA and read by its owner, and the K order of the owner's sum.
 * Writes the largest number of K-stages of one CTA to *max_units_out.
 * Returns MT_OK, or MT_ERR_INVALID_ARGUMENT naming the broken rule.
 */
int mt_qmm_partition_check(int64_t tiles, int nk, int cluster_size, int clusters, int64_t* max_units_out);

/*
 * Fused region: y = residual + quantized_matmul(x, w, ...), each step rounded
 * to dtype as the unfused ops would (the `v22 = v0 + v21` cut of the
 * reference's generated wrapper,
 * examples/lfm2_5_1_2b_prefill/lfm2_5_1_2b_prefill_artifact/patch/wrappers.py:68-77).
 * residual and y are [M, N]; y may alias residual.
 */
int mt_quantized_matmul_residual(const void* x, const uint32_t* w,
                                 const void* scales, const void* biases,
                                 const void* residual, void* y, int64_t M,
                                 int64_t N, int64_t K, int group_size, int bits,
                                 int dtype, void* workspace,
                                 size_t workspace_bytes, mt_stream_t stream);

/*
 * Fused region with two outputs: h = residual + qmm(x), y = rms_norm(h, norm_w, eps)
 * (the r95aa6c37bb25ef99 cut: wrappers.py:68-77, kernels/r95aa6c37bb25ef99_prefill_bk64.launch.json).
 */
int mt_quantized_matmul_residual_rms_norm(
    const void* x, const uint32_t* w, const void* scales, const void* biases,
    const void* residual, const void* norm_w, float eps, void* h, void* y,
    int64_t M, int64_t N, int64_t K, int group_size, int bits, int dtype,
    void* workspace, size_t workspace_bytes, mt_stream_t stream);

/*
 * Fused gate/up projections + SwiGLU: y = silu(qmm(x, wg)) * qmm(x, wu)
 * (the gate/up pair kernels/r1f9367e50750eb01_unroll_hoist.launch.json followed by
 * mlx_lm.models.activations.swiglu, wrappers.py:93-96). Both weights [N, ...].
 */
int mt_quantized_matmul_swiglu(const void* x, const uint32_t* wg,
                               const void* sg, const void* bg,
                               const uint32_t* wu, const void* su,
                               const void* bu, void* y, int64_t M, int64_t N,
                               int64_t K, int group_size, int bits, int dtype,
                               void* workspace, size_t workspace_bytes,
                               mt_stream_t stream);

/*
 * Up to three projections of the same x in one launch (q/k/v): set i is
 * (w_i, scales_i, biases_i, y_i, N_i); a set with N_i == 0 is skipped.
 * Equivalent to three mt_quantized_matmul calls.
 */
int mt_quantized_matmul_multi(const void* x, const uint32_t* w0,
                              const void* s0, const void* b0, void* y0,
                              int64_t N0, const uint32_t* w1, const void* s1,
                              const void* b1, void* y1, int64_t N1,
                              const uint32_t* w2, const void* s2,
                              const void* b2, void* y2, int64_t N2, int64_t M,
                              int64_t K, int group_size, int bits, int dtype,
                              void* workspace, size_t workspace_bytes,
                              mt_stream_t stream);

/*
 * Decode regions with the RMSNorm before them fused in (M <= 4):
 * y_i = quantized_matmul(rms_norm(x, norm_w, eps), w_i, ...) for up to three
 * sets, and y = silu(qmm(xn, wg)) * qmm(xn, wu) with xn = rms_norm(x, ...).
 * Same results as mt_rms_norm followed by mt_quantized_matmul_multi /
 * mt_quantized_matmul_swiglu (the normalised rows are never written). They
 * replace the rms_norm -> qkv and rms_norm -> gate/up region pairs of the
 * reference's decoder-layer wrapper
 * (examples/lfm2_5_1_2b_prefill/lfm2_5_1_2b_prefill_artifact/patch/wrappers.py:38-106)
 * at decode, where the reference's cuts keep them apart. No workspace.
 * MT_ERR_UNSUPPORTED when the shape needs more than the streamed decode
 * kernel (M > 4, bits != 4, K > 16384, norm_w not 16-byte aligned).
 */
int mt_rms_norm_quantized_matmul_multi(
    const void* x, const void* norm_w, float eps, const uint32_t* w0,
    const void* s0, const void* b0, void* y0, int64_t N0, const uint32_t* w1,
    const void* s1, const void* b1, void* y1, int64_t N1, const uint32_t* w2,
    const void* s2, const void* b2, void* y2, int64_t N2, int64_t M, int64_t K,
    int group_size, int bits, int dtype, mt_stream_t stream);

int mt_rms_norm_quantized_matmul_swiglu(
    const void* x, const void* norm_w, float eps, const uint32_t* wg,
    const void* sg, const void* bg, const uint32_t* wu, const void* su,
    const void* bu, void* y, int64_t M, int64_t N, int64_t K, int group_size,
    int bits, int dtype, mt_stream_t stream);

/*
 * Bytes of workspace the quantized-matmul entry points need for this shape.
 * `n_total` is the summed N over all sets (2N for the SwiGLU pair);
 * `kind` is 0 (plain/residual/multi) or 1 (SwiGLU pair). From M = 1024 rows
 * up it includes room for one set's dequantised weights (n_total*K elements;
 * for the SwiGLU pair 256*ceil(N/128)*K: gate and up rows interleaved in
 * blocks of 128, one GEMM with SwiGLU in its epilogue): those shapes
 * dequantise the weights once and multiply on the tcgen05 GEMM. Given less
 * than this, they run the fused kernel instead.
 */
size_t mt_qmm_workspace_bytes(int64_t M, int64_t n_total, int64_t K, int bits,
                              int kind);

/* ------------------------------------------------------------------------ */
/* a-3: RMSNorm and fused residual add + RMSNorm                             */
/* ------------------------------------------------------------------------ */
/* mx.fast.rms_norm(x, w, eps): y = x * rsqrt(mean(x^2) + eps) * w, fp32
 * accumulation (autotuner/scaffold/lower.py:434-446, :1318-1355). */
int mt_rms_norm(const void* x, const void* w, float eps, void* y, int64_t rows,
                int64_t dim, int dtype, mt_stream_t stream);

/* h = x + residual (rounded to dtype), y = rms_norm(h, w, eps); two outputs
 * (metalbench/published/2026-09-19-m4/fused_add_rms_norm). */
int mt_add_rms_norm(const void* x, const void* residual, const void* w,
                    float eps, void* h, void* y, int64_t rows, int64_t dim,
                    int dtype, mt_stream_t stream);

/* ------------------------------------------------------------------------ */
/* a-4: RoPE with offset                                                     */
/* ------------------------------------------------------------------------ */
/* mx.fast.rope(x, dims, traditional, base, scale, offset) over x [B, H, L, D]
 * (autotuner/scaffold/lower.py:515-560, :1236-1294): position = (l + offset)
 * * scale, theta_j = position * base^(-2j/dims), leading `dims` rotated, the
 * tail copied. y may alias x. */
int mt_rope(const void* x, void* y, int64_t B, int64_t H, int64_t L,
            int64_t D, int dims, int traditional, float base, float scale,
            int64_t offset, int dtype, mt_stream_t stream);

/* mt_rope over strided x and y: element (b, h, l, d) of x sits at
 * x_sb*b + x_sh*h + x_sl*l + d (in elements), of y likewise. MLX applies rope
 * to the transposed view of the q/k projections (mlx-lm llama: reshape
 * [B, L, H, D] then transpose to [B, H, L, D] before rope); one call reads the
 * token-major projection output and writes the head-major rotated tensor.
 * y must not overlap x unless both have the same strides. */
int mt_rope_strided(const void* x, void* y, int64_t B, int64_t H, int64_t L,
                    int64_t D, int dims, int traditional, float base,
                    float scale, int64_t offset, int64_t x_sb, int64_t x_sh,
                    int64_t x_sl, int64_t y_sb, int64_t y_sh, int64_t y_sl,
                    int dtype, mt_stream_t stream);

/*
 * Qwen3 attention prologue as one region: per token t and head h,
 * q' = rope(rms_norm(q[t,h,:], q_norm_w), offset+t), k' likewise with
 * k_norm_w, v copied; q' written head-major to q_out [Hq, T, D], k'/v'
 * appended to the caches k_cache/v_cache [Hkv, cache_cap, D] at rows
 * offset..offset+T-1. Each step rounds to dtype as the separate MLX ops do
 * (rms_norm, transpose, rope, cache.update_and_fetch). q/k/v rows are
 * `q_stride`/`kv_stride` elements apart.
 */
int mt_qk_norm_rope_cache(const void* q, const void* k, const void* v,
                          int64_t q_stride, int64_t kv_stride,
                          const void* q_norm_w, const void* k_norm_w, float eps,
                          void* q_out, void* k_cache, void* v_cache, int64_t T,
                          int64_t Hq, int64_t Hkv, int64_t D, int64_t cache_cap,
                          int64_t offset, float rope_base, int dtype,
                          mt_stream_t stream);

/*
 * Decode (T <= 4 new tokens, (Hq/Hkv) * T <= 16): mt_qk_norm_rope_cache followed
 * by causal GQA attention of the T rotated queries over the cache rows
 * 0..offset+T-1, in one launch (one CTA per kv head). The caches receive the
 * same rows as mt_qk_norm_rope_cache writes (bit-identical); o is
 * [T, Hq*D] (heads concatenated per token, the layout of the layer's o_proj
 * input). Replaces the qk_norm_rope_cache -> sdpa region pair of the
 * decoder-layer wrapper (examples/lfm2_5_1_2b_prefill/.../patch/wrappers.py:
 * 38-106) at decode; `scale` is the softmax scale (1/sqrt(D)).
 */
int mt_qk_norm_rope_sdpa_decode(const void* q, const void* k, const void* v,
                                int64_t q_stride, int64_t kv_stride,
                                const void* q_norm_w, const void* k_norm_w,
                                float eps, void* o, void* k_cache,
                                void* v_cache, int64_t T, int64_t Hq,
                                int64_t Hkv, int64_t D, int64_t cache_cap,
                                int64_t offset, float rope_base, float scale,
                                int dtype, mt_stream_t stream);

/* ------------------------------------------------------------------------ */
/* a-5: SwiGLU                                                               */
/* ------------------------------------------------------------------------ */
/* mlx_lm.models.activations.swiglu(gate, up) = silu(gate) * up with
 * sigmoid = 1/(1+exp(-x)) (autotuner/scaffold/lower.py:80), each op rounded
 * to dtype. */
int mt_swiglu(const void* gate, const void* up, void* y, int64_t n, int dtype,
              mt_stream_t stream);

/* y[i] = round(x[i] + r[i mod period]) in dtype (bf16 / f16 / f32): the `+`
 * of a residual branch, or the mlx-whisper encoder's `x + positional_embedding`
 * (models/whisper_large_v3_turbo_encoder.py:8-12) with the [n_ctx, n_state]
 * table repeated over the batch (period = n_ctx * n_state). n must be a
 * multiple of period; y may alias x. */
int mt_add(const void* x, const void* r, void* y, int64_t n, int64_t period,
           int dtype, mt_stream_t stream);

/* nn.Embedding: out[t, :] = table[tokens[t], :] for a dense [vocab, D] table
 * (mlx-lm mamba's embedding, models/mamba_370m.py:4-8). An id outside
 * [0, vocab) writes zeros and is reported through the device status. */
int mt_embedding(const int32_t* tokens, const void* table, void* out, int64_t T,
                 int64_t vocab, int64_t D, int dtype, mt_stream_t stream);

/* ------------------------------------------------------------------------ */
/* a-6: causal GQA scaled-dot-product attention                              */
/* ------------------------------------------------------------------------ */
/*
 * mx.fast.scaled_dot_product_attention(q, k, v, scale, mask="causal"|None)
 * (regions/build.py:28-34; FLOPs regions/roofline.py:60-65): softmax(q k^T *
 * scale + mask) v with KV head = q_head / (Hq / Hkv). Strides are in
 * elements: q[b,h,i,:] at q + b*qs_b + h*qs_h + i*qs_l (D contiguous), same
 * for k, v (key index) and o (query index). With `causal`, query i (absolute
 * position q_offset + i) sees keys 0..q_offset+i (MLX's bottom-right
 * alignment when q_offset = Lk - Lq). D must be 64 or 128.
 */
int mt_sdpa(const void* q, const void* k, const void* v, void* o, int64_t B,
            int64_t Hq, int64_t Hkv, int64_t Lq, int64_t Lk, int64_t D,
            float scale, int causal, int64_t q_offset, int64_t qs_b,
            int64_t qs_h, int64_t qs_l, int64_t ks_b, int64_t ks_h,
            int64_t ks_l, int64_t vs_b, int64_t vs_h, int64_t vs_l,
            int64_t os_b, int64_t os_h, int64_t os_l, int dtype,
            mt_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Either side of the layers (next row 1): quantized embedding, lm_head pick  */
/* ------------------------------------------------------------------------ */
/* mlx.nn.QuantizedEmbedding: out[t] = dequantize(w[tok[t]], scales[tok[t]],
 * biases[tok[t]]) with MLX's rounding (w = round(round(s*q)+b)). tokens int32;
 * an id outside [0, vocab) is an argument error reported through the device
 * status word and writes zeros. */
int mt_quantized_embedding(const int32_t* tokens, const uint32_t* w,
                           const void* scales, const void* biases, void* out,
                           int64_t T, int64_t vocab, int64_t D, int group_size,
                           int bits, int dtype, mt_stream_t stream);

/* Greedy pick from one row of logits (mlx-lm generate_step,
 * autotuner_runtime/inference.py:140-147): token = argmax(logits) (lowest
 * index on ties), lse = logsumexp(logits) in fp32, logprob = logits[token] -
 * lse rounded to dtype then widened to fp32. Single row of n logits. */
int mt_logits_pick(const void* logits, int64_t n, int dtype, int32_t* token,
                   float* logprob, float* lse, mt_stream_t stream);

/* ------------------------------------------------------------------------ */
/* a-10: output-diff reduction of the verification ladder                    */
/* ------------------------------------------------------------------------ */
/*
 * One pass over candidate `a` and reference `b` (n elements of dtype):
 * autotuner_runtime/numeric.py:50-107 (compare), :111-122 (check),
 * autotuner_runtime/exact.py:5-10 (bitwise_equal),
 * autotuner/ladder/numeric.py:22-35 (max_abs_diff),
 * autotuner/artifact/validate.py:64-103 (max abs diff, cosine).
 * Writes one mt_diff_stats to device memory `stats`.
 */
typedef struct mt_diff_stats {
  double max_excess;         /* worst |a-b| - max(atol + rtol|b|, wobble) over finite b */
  double max_abs;            /* worst |a-b| over positions where both are finite         */
  double dot_ab, dot_aa, dot_bb; /* fp64 sums for cosine, non-finite values taken as 0   */
  double amax_a, amax_b;     /* max |a|, max |b| over finite values (cosine's zero test)  */
  int64_t excess_index;      /* flat index of max_excess (lowest on ties), -1 if none    */
  int64_t over_count;        /* elements with excess > 0                                  */
  int64_t nonfinite_violations; /* elements breaking the non-finite pattern rule         */
  int64_t first_violation;   /* lowest flat index breaking the pattern, -1 if none       */
  int64_t bit_mismatches;    /* elements whose bit patterns differ                        */
  int64_t first_mismatch;    /* lowest flat index of a bit mismatch, -1 if none          */
  int64_t nan_excess;        /* elements whose excess evaluated to NaN                    */
} mt_diff_stats;

size_t mt_diff_workspace_bytes(int64_t n);

int mt_diff_reduce(const void* a, const void* b, int64_t n, int dtype,
                   float rtol, float atol, float wobble, mt_diff_stats* stats,
                   void* workspace, size_t workspace_bytes,
                   mt_stream_t stream);

/*
 * mt_diff_reduce without a workspace argument; it allocates nothing. No
 * counterpart in the reference: it exists for callers that must not
 * allocate device memory — a host binding of this C ABI that holds only
 * buffers lent to it and has no CUDA allocator of its own, or a verification
 * check that runs while the memory pool is deliberately filled with NaNs (the
 * reference's poisoned-pool gate), where allocating scratch would take memory
 * from, or add memory to, the very pool under test.
 *
 * Scratch lives in a static device array inside libmt.so (about 12 KB: a
 * counter and 128 block partials), held by every GPU that loads the library
 * until the process exits. n may be at most MT_DIFF_NOALLOC_MAX_ELEMS;
 * larger inputs are rejected with MT_ERR_INVALID_ARGUMENT (use
 * mt_diff_reduce). Same kernel and block partition as mt_diff_reduce, so the
 * statistics are identical. Every call looks up the array's device address
 * (cudaGetSymbolAddress) in the current context, so a call after a
 * cudaDeviceReset or a primary-context reset uses the array's new address;
 * the first call on a device also loads the library's module there, so make
 * that first call before any stream capture. Every call on a device shares the
 * array: calls whose kernels overlap on the GPU (other streams, other host
 * threads) race and must be serialised by the caller. Each call zeroes the
 * counter on its stream before its kernel runs.
 */
#define MT_DIFF_NOALLOC_MAX_ELEMS 1048576
int mt_diff_reduce_noalloc(const void* a, const void* b, int64_t n, int dtype,
                           float rtol, float atol, float wobble,
                           mt_diff_stats* stats, mt_stream_t stream);

/* ------------------------------------------------------------------------ */
/* a-7: dense linear (+bias, +GELU), the GELU-MLP region                     */
/* ------------------------------------------------------------------------ */
/*
 * y[M,N] = act(x[M,K] · w[N,K]^T + bias[N]) in fp32 with a sequential-k
 * fused-multiply-add order (the reference's matmul restatement,
 * autotuner/scaffold/lower.py:1109-1142), act 0 = identity, 1 = GELU exact
 * erf form 0.5 x (1 + erf(x / sqrt 2)) (mlx.nn.GELU default;
 * examples/tiny_mlp.py:5-6). Bit-reproducible against the CPU oracle.
 * bias may be NULL. dtype MT_F32; MT_BF16 / MT_F16 run the tensor-core
 * implicit GEMM of mt_conv1d (the Whisper MLP sizes: K a multiple of 32),
 * fp32 sums with the bias added before the one rounding (mx.addmm) and GELU
 * rounded after it (not bit-reproducible: the sums run in tiles). The 16-bit
 * path runs on the tcgen05 GEMM (tensor memory accumulators, TMA-staged
 * operands) when K is a multiple of 8: on pairs of SMs (cta_group::2,
 * 256 x 256 tiles) once there are at least as many such tiles as SM pairs,
 * else one SM per 128 x 256 tile; both give the same bits. The environment
 * variable MT_GEMM_PAIR=0 / 1 forces the choice (this and mt_conv1d,
 * mt_linear_residual and the quantized matmul from 1024 rows).
 */
int mt_linear(const void* x, const void* w, const void* bias, void* y,
              int64_t M, int64_t N, int64_t K, int act, int dtype,
              mt_stream_t stream);

/*
 * The residual branch of a pre-norm block (mlx-whisper ResidualAttentionBlock:
 * x + attn.out(...), x + mlp2(...); models/whisper_large_v3_turbo_encoder.py:
 * 8-12): y = round(round(x[M,K] · w[N,K]^T + bias[N]) + residual[M,N]) in
 * bf16 / f16 with fp32 sums (bias may be NULL), on the tcgen05 GEMM. K must
 * be a multiple of 8 (MT_ERR_UNSUPPORTED otherwise); y may alias residual.
 */
int mt_linear_residual(const void* x, const void* w, const void* bias,
                       const void* residual, void* y, int64_t M, int64_t N,
                       int64_t K, int dtype, mt_stream_t stream);

/* ------------------------------------------------------------------------ */
/* a-8: LayerNorm                                                            */
/* ------------------------------------------------------------------------ */
/*
 * mx.conv1d for the Whisper encoder's conv stem (mlx-whisper conv1 / conv2:
 * nn.Conv1d with bias, then GELU): channels-last x [N, L, Cin], w
 * [Cout, K, Cin] (mlx layouts), y [N, Lout, Cout] with
 * Lout = (L + 2*padding - K) / stride + 1, zero padding on both sides. The
 * conv sums in fp32; conv, + bias (NULL: none) and GELU (act = 1; 0: none)
 * are each rounded to dtype as the separate MLX ops would. Cin must be a
 * multiple of 32 (MT_ERR_UNSUPPORTED otherwise); bf16 or f16. Runs on the
 * tcgen05 implicit GEMM when Cin is a multiple of 64, the stride 1 or 2 with
 * L a multiple of it, and K <= 4 (both mlx-whisper stem convs); otherwise on
 * an mma.sync implicit GEMM.
 */
int mt_conv1d(const void* x, const void* w, const void* bias, void* y, int64_t N,
              int64_t L, int64_t Cin, int64_t Cout, int K, int stride,
              int padding, int act, int dtype, mt_stream_t stream);

/* mx.fast.layer_norm(x, w, b, eps): two-pass mean / centred variance, then
 * the optional affine (autotuner/scaffold/lower.py:448-466, :1357-1410).
 * w and b may be NULL. */
int mt_layer_norm(const void* x, const void* w, const void* b, float eps,
                  void* y, int64_t rows, int64_t dim, int dtype,
                  mt_stream_t stream);

/* ------------------------------------------------------------------------ */
/* a-9: Mamba selective scan                                                 */
/* ------------------------------------------------------------------------ */
/*
 * Mamba-1 selective scan (mlx-lm 0.31.3 mamba model; Gu & Dao 2023), one
 * batch element, over L steps and d_inner channels with d_state states:
 *   dt  = softplus(dt_raw[l,c] + dt_bias[c])
 *   h   = exp(dt * A[c,s]) * h + dt * B[l,s] * x[l,c]
 *   y   = sum_s C[l,s] h[s] + D[c] x[l,c];   y *= silu(z[l,c])
 * A = -exp(A_log) is passed in fp32 [d_inner, d_state]; x, dt_raw, z, y are
 * [L, d_inner] dtype; B, C are [L, d_state] dtype; dt_bias, D fp32
 * [d_inner]. h_state [d_inner, d_state] fp32 is read as the initial state
 * and overwritten with the final one (may be NULL for zero initial state
 * and no state output). Recurrence in fp32, sequential in l.
 */
int mt_mamba_scan(const void* x, const void* dt_raw, const float* dt_bias,
                  const float* A, const void* Bm, const void* Cm,
                  const float* Dv, const void* z, void* y, float* h_state,
                  int64_t L, int64_t d_inner, int64_t d_state, int dtype,
                  mt_stream_t stream);

/* Depthwise causal conv1d over [L, C] with kernel [C, width] and bias [C]
 * (mlx_lm mamba conv1d with groups = C and left padding width-1), then SiLU
 * when `silu` != 0. conv_state [C, width-1] holds the previous inputs (may be
 * NULL for zeros) and receives the last width-1 inputs afterwards. */
int mt_causal_conv1d(const void* x, const void* weight, const void* bias,
                     void* conv_state, void* y, int64_t L, int64_t C,
                     int width, int silu, int dtype, mt_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MT_H_ */
