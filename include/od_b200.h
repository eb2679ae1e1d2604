/*
 * od_b200.h - C ABI of libod_b200.so, the sm_100a kernels of the OpenDecider decision forward pass.
 *
 * Conventions (the same as the reference's own ctypes C ABI, deploy/llamacpp/od_llama.cpp:13-23 and
 * src/opendecider/llamacpp.py:37-52):
 *   - every entry point returns an int status: OD_OK (0) on success, a negative OD_E* code on error;
 *     od_last_error() returns a message for the calling thread's last error. No C++ exception crosses the ABI.
 *   - all pointers are DEVICE pointers unless the name says host; buffers are owned by the caller.
 *   - `stream` is a cudaStream_t passed as void* (NULL = the legacy default stream). No compute entry point
 *     synchronises the host or allocates device memory (od_gemm_w8a8 encodes its TMA descriptors on the host and
 *     passes them as kernel parameters).
 *   - dtype codes: OD_BF16, OD_F16, OD_F32 (see below).
 *   - shapes are int64; strides are in ELEMENTS.
 *
 * Layouts (the reference's, kept unchanged so the kernels read the reference's buffers as they are):
 *   int8 weight      qweight (N, K) int8 row-major + scale (N) in the weight dtype  (quant.py:122-127)
 *   int8 KV cache    q (S, Hkv, T, D) int8 + scale (S, Hkv, T) in the source dtype  (backbone.py:446, quant.py:37-41)
 *   activations      (M, K) row-major, bf16
 */
#ifndef OD_B200_H
#define OD_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define OD_API __attribute__((visibility("default")))
#else
#define OD_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  OD_OK = 0,
  OD_EINVAL = -1,      /* bad argument (shape, dtype, alignment, null pointer) */
  OD_ECUDA = -2,       /* a CUDA runtime/driver call failed */
  OD_EUNSUPPORTED = -3,/* a valid configuration this build does not implement */
  OD_ETIMEOUT = -4     /* a bounded device-side wait gave up (see od_device_error) */
};

enum { OD_BF16 = 0, OD_F16 = 1, OD_F32 = 2 };

/* Message of the calling thread's last error ("" if none). */
OD_API const char* od_last_error(void);

/* Library version string, e.g. "od_b200 0.1 sm_100a". */
OD_API const char* od_version(void);

/* Device-side error word written by kernels whose bounded waits give up (0 = none). Reads and clears it.
 * Synchronises `stream`. Not a hot-path call. */
OD_API int od_device_error(void* stream, int32_t* host_code);
/* No reference counterpart: a self-test of the kernels' failure detection. One thread waits on a barrier that nothing
 * completes, gives up after limit_cycles (at most the kernels' own limit), records 0x7F0001 in the device error word
 * and returns; od_device_error then reads it. Nothing faults or hangs. */
OD_API int od_selftest_bounded_wait(int64_t limit_cycles, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * A1 / A5 / A6: per-row symmetric int8 quantisation, Int8Tensor.quantize (quant.py:37-41) and the weight quantiser
 * of Int8Linear.__init__ (quant.py:124-127):
 *     s = max(max_k |x[m,k]|, 1e-8) / 127   (fp32, IEEE division)
 *     q = clamp(rint(x / s), -127, 127)     (fp32 IEEE division, round half to even)
 *     scale[m] = s rounded to `scale_dtype`
 * x (M, K) of `x_dtype` with row stride ldx (elements). Optional inv_s (K,) bf16: x is first multiplied by inv_s in
 * bf16 (SmoothedLinear.forward, quant.py:328-329: bf16(x * inv_s)) before quantising.
 * Replaces: Int8Tensor.quantize, Int8Linear.__init__'s quantiser, and GemLite A8W8's dynamic activation quant.
 */
OD_API int od_quant_rows_i8(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, const void* inv_s,
                     int8_t* q, void* scale, int scale_dtype, void* stream);

/* Row-wise dequantisation, Int8Tensor.dequantize (quant.py:43-45): y = out_dtype(out_dtype(q) * out_dtype(s)).
 * q (M, K) int8, scale (M) of scale_dtype, y (M, K) of out_dtype. */
OD_API int od_dequant_rows_i8(const int8_t* q, const void* scale, int scale_dtype, int64_t M, int64_t K,
                       void* y, int out_dtype, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * A6: int8 KV-cache append. New keys/values k, v of `t` tokens per state, bf16 or fp16, addressed as
 * k[s*ks_s + j*ks_t + h*ks_h + d] (any strides, d contiguous), are quantised per (state, head, token) over D exactly
 * as Int8Tensor.quantize and written at token offset t0 of the cache:
 *     kq[s, h, t0 + j, :], ksc[s, h, t0 + j]    (cache: (S, Hkv, T_cap, D) int8 + (S, Hkv, T_cap) scales)
 * Scales are stored in the dtype of k/v (as Int8Tensor does). kb, vb (optional, both or neither, 16-byte aligned,
 * (S, Hkv, T_cap, D) in the dtype of k/v) receive the same rows materialised, q * s rounded once as materialize()
 * computes it (quant.py:43-45), so a kept bf16 copy of the cache is extended without re-reading the int8 rows.
 * Replaces PackedCache.pack's per-layer maybe_quantize (backbone.py:446) and PrefixCache._take's new-slice
 * quantisation (state_cache.py:79).
 */
OD_API int od_kv_append_i8(const void* k, const void* v, int kv_dtype, int64_t S, int64_t t, int Hkv, int D,
                    int64_t ks_s, int64_t ks_t, int64_t ks_h, int64_t vs_s, int64_t vs_t, int64_t vs_h,
                    int8_t* kq, int8_t* vq, void* ksc, void* vsc, void* kb, void* vb, int64_t T_cap, int64_t t0,
                    void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * A3 + A4 + A5: residual add + Qwen3.5 RMSNorm + (optional SmoothQuant multiply) + per-token int8 quantisation.
 *     h   = res_in ? bf16(x + res_in) : x                    (decoder residual add, modeling_qwen3_5.py:768/781)
 *     y   = bf16(float(h) * rsqrt(mean(float(h)^2) + eps) * (1 + float(w)))   (Qwen3_5RMSNorm, :720-725)
 *     y'  = inv_s ? bf16(y * inv_s) : y                      (SmoothedLinear, quant.py:328-329)
 *     q,s = quantise(y') as od_quant_rows_i8 with fp32 scales
 * x, res_in, res_out, y_out: (M, H) bf16. res_out (may alias x) receives h when res_in is given. y_out (optional)
 * receives y' in bf16. q (M, H) int8 and s (M) fp32 are optional (both or neither).
 */
OD_API int od_rmsnorm_res_quant(const void* x, const void* res_in, void* res_out, const void* w, const void* inv_s,
                         float eps, int64_t M, int H, void* y_out, int8_t* q, float* s, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * A2: W8A8 GEMM on the 5th-generation tensor cores (tcgen05.mma kind::i8, int32 accumulators in TMEM, TMA loads).
 *     acc[m, n] = sum_k A[m, k] * W[n, k]          (int32, exact)
 * epilogue OD_EPI_BF16:   Y[m, n] = bf16((float(acc) * sa[m]) * float(sw[n]))            Y (M, N) bf16, ldy = N
 * epilogue OD_EPI_SWIGLU: W rows are interleaved in blocks of 128 (gate_0..127, up_0..127, gate_128.., ...);
 *                         g = bf16(acc_gate...), u = bf16(acc_up...), Y[m, j] = bf16(bf16(silu(g)) * u)
 *                         (Qwen3_5MLP.forward: act_fn(gate_proj(x)) * up_proj(x)), Y (M, N/2) bf16
 * epilogue OD_EPI_INT32:  Y[m, n] = acc (int32) - the bit-exact parity mode
 * A (M, K) int8 row-major, sa (M) fp32 (per-token activation scales), W (N, K) int8 row-major (Int8Linear.qweight),
 * sw (N) bf16 (Int8Linear.scale). K % 128 == 0, N % 32 == 0 (OD_EPI_SWIGLU: N % 256 == 0), M >= 0 (any).
 * A, W 16-byte aligned. Replaces GemLite A8W8 (quant.py:302-314) and the dequant+cuBLAS path (quant.py:149-157).
 */
enum { OD_EPI_BF16 = 0, OD_EPI_SWIGLU = 1, OD_EPI_INT32 = 2 };
OD_API int od_gemm_w8a8(const int8_t* A, const float* sa, const int8_t* W, const void* sw, void* Y,
                 int64_t M, int64_t N, int64_t K, int epilogue, void* stream);
/* od_gemm_w8a8 writing rows of Y ldy elements apart (ldy >= the output width, a multiple of one 16-byte store),
 * so several projections of one layer can fill column ranges of one stacked output: the SmoothQuant path's separate
 * q / k / v GEMMs (each input smoothed by its own vector, SmoothedLinear quant.py:317-329) write the same fused
 * (M, Hq*2D + 2*Hkv*D) layout the single stacked GEMM writes. */
OD_API int od_gemm_w8a8_ld(const int8_t* A, const float* sa, const int8_t* W, const void* sw, void* Y,
                    int64_t M, int64_t N, int64_t K, int epilogue, int64_t ldy, void* stream);
/* Split-K for small M (M < 1024, the single-CTA form): the K range of each 128 x 256 tile is divided among `splits`
 * work items (1..8, at most K / 128), each writing its int32 partial tile to `workspace` (tiles x splits x 128 x 256
 * int32, no initial contents needed); a second kernel sums the partials (exact integer addition) and runs the
 * epilogue: results identical to od_gemm_w8a8. Calls sharing a workspace must be stream-ordered.
 * od_gemm_w8a8_plan returns the split count this GPU's SM count favours (1: no split, no workspace) and the
 * workspace size. Same reference interfaces as od_gemm_w8a8. */
OD_API int od_gemm_w8a8_plan(int64_t M, int64_t N, int64_t K, int num_sms, int* splits, int64_t* workspace_bytes);
OD_API int od_gemm_w8a8_splitk(const int8_t* A, const float* sa, const int8_t* W, const void* sw, void* Y,
                        int64_t M, int64_t N, int64_t K, int epilogue, int64_t ldy, int splits, void* workspace,
                        int64_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Embedding lookup of an int8 table, Int8Embedding.forward (quant.py:199-200):
 *     out[i, :] = bf16(bf16(qweight[ids[i], :]) * scale[ids[i]])
 * ids (n) int64, qweight (V, H) int8, scale (V) bf16, out (n, H) bf16.
 */
OD_API int od_embed_i8(const int64_t* ids, int64_t n, const int8_t* qweight, const void* scale, int64_t V, int H,
                void* out, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Attention pre-processing on the fused q/k/v projection output (Qwen3_5Attention.forward, modeling_qwen3_5.py:
 * 647-668 and prefix_attn.py:84-90): per token, q_proj's gated layout [head h: q (D) | gate (D)] is split,
 * q and k get the per-head RMSNorm (1 + w), then rotate-half RoPE with the cos/sin tables:
 *     q' = bf16(bf16(q * cos) + bf16(rotate_half(q) * sin))   (bf16 tables, the HF rounding points)
 * qkv (M, Hq*2D + 2*Hkv*D) bf16 row-major; pos (M) int32 position of every token; cos, sin (P, D) bf16 tables.
 * Outputs: q_out (M, Hq, D), k_out (M, Hkv, D), v_out (M, Hkv, D) bf16. The gate stays in qkv.
 */
OD_API int od_qk_norm_rope(const void* qkv, const int32_t* pos, const void* cos, const void* sin, int64_t P,
                    const void* qnorm_w, const void* knorm_w, float eps, int64_t M, int Hq, int Hkv, int D,
                    void* q_out, void* k_out, void* v_out, void* stream);
/* (f.1) od_qk_norm_rope that also writes the pass's K/V into the int8 cache (the state pass's fused KV write,
 * replacing od_kv_append_i8 after it): token m = r * t + j of the pass is cache position t0 + j of state r;
 * kq/vq (S, Hkv, T_cap, D) int8, ksc/vsc (S, Hkv, T_cap) bf16, bytes and scales exactly as od_kv_append_i8 writes
 * them (PackedCache.pack's maybe_quantize, backbone.py:446; PrefixCache._take, state_cache.py:79); kb/vb (optional,
 * both or neither) the materialised bf16 rows. q/k/v outputs as od_qk_norm_rope. */
OD_API int od_qk_norm_rope_kv_i8(const void* qkv, const int32_t* pos, const void* cos, const void* sin, int64_t P,
                          const void* qnorm_w, const void* knorm_w, float eps, int64_t M, int Hq, int Hkv, int D,
                          void* q_out, void* k_out, void* v_out, int64_t t, int8_t* kq, int8_t* vq, void* ksc,
                          void* vsc, void* kb, void* vb, int64_t T_cap, int64_t t0, void* stream);

/* Output gate + per-token quantisation of the o_proj input (Qwen3_5Attention.forward :666-668):
 *     g = bf16(o * bf16(sigmoid(gate))),  g' = inv_s ? bf16(g * inv_s) : g,  then q, s = quantise(g') (fp32 scales)
 * o (M, Hq*D) bf16; gate read from qkv (M, ldqkv) at column h*2D + D + d for head h; inv_s (Hq*D) bf16 or NULL
 * (the o_proj SmoothedLinear multiply, quant.py:328-329). */
OD_API int od_gate_quant(const void* o, const void* qkv, int64_t ldqkv, int64_t M, int Hq, int D,
                  const void* inv_s, int8_t* q, float* s, void* stream);
/* SwiGLU of separate gate / up projections + the down projection's input quantisation (Qwen3_5MLP.forward, with a
 * SmoothedLinear on each of gate_proj, up_proj and down_proj, quant.py:317-350, whose vectors differ so gate and up
 * cannot share the interleaved SwiGLU GEMM):
 *     a = bf16(g / (1 + exp(-g))),  h = bf16(a * u),  h' = inv_s ? bf16(h * inv_s) : h,  q, s = quantise(h')
 * g, u (M, F) bf16 (F % 8 == 0), inv_s (F) bf16 or NULL, q (M, F) int8, s (M) fp32. Same rounding points as the
 * OD_EPI_SWIGLU epilogue. */
OD_API int od_swiglu_quant(const void* g, const void* u, int64_t M, int64_t F, const void* inv_s, int8_t* q,
                    float* s, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * A9/A10: branched shared-prefix attention (Hydragen split, prefix_attn.py:43-76, merged exactly by log-sum-exp).
 * Every query row r (a question or option row, t tokens, Hq heads) attends, in ONE online softmax:
 *   1. the state prefix of state st = row_state[r]: keys p in [p_lo[st], p_hi[st]) of Kp/Vp (S, Hkv, T, D); keys
 *      with pmask[st, p] == 0 are skipped (pmask may be NULL). Either int8 with per-token scales ksc/vsc
 *      (S, Hkv, T), dequantised in shared memory exactly as materialize() does (bf16(q * s); fp16 scales:
 *      bf16(fp16(q * s))), or (dims.prefix_bf16 = 1) the already materialised bf16 cache (prefix_attn.py:146-149),
 *      ksc/vsc unused.
 *   2. optionally a second bf16 prefix level (the question cache, prefix_attn.py:94-99): keys j < q_len[qr] of
 *      Kq/Vq (NQ, Lq, Hkv, D) for question qr = row_q[r].
 *   3. its own k/v (R, t, Hkv, D) bf16 causally: key j visible to query i iff j <= i and
 *      own_lo[r] <= j < own_hi[r] (own_lo / own_hi may be NULL: 0 / t; left-padded rows set own_lo).
 * Output o (R, t, Hq, D) bf16 and optionally lse (R, Hq, t) fp32 (natural log, -inf when no key is visible; such
 * rows output 0, wide_attention.py:62-67). q (R, t, Hq, D) bf16. GQA: query head h reads kv head h / (Hq / Hkv).
 * row_groups (G, 2) int32 [first row, rows] (optional; NULL = every row alone): consecutive rows that share their
 * state and question and are processed together by one CTA of up to two 128-slot tensor-core tiles
 * (rows x t x Hq/Hkv <= 256 when a group has more than one row); they still attend only their own keys.
 * dims.nsplit > 1 divides each state prefix among that many CTAs (for launches with fewer query tiles than SMs): each
 * writes its partial O / l and LSE (fp32) to `workspace` and a second kernel merges them by log-sum-exp; the
 * workspace (16-byte aligned) holds nsplit x R x t x Hq x (D + 1) floats. od_prefix_attn_plan picks nsplit for a
 * GPU of num_sms SMs and returns the workspace size; workspace may be NULL when nsplit <= 1.
 * Every row sees the same key layout whatever its index or group: outputs do not depend on row order.
 * Runs on tcgen05 (S = Q K^T and O += P V in TMEM); head_dim 64 or 128.
 * o and lse are undefined whenever od_device_error reports a code (a bounded wait gave up); with nsplit > 1 the
 * merge then writes NaN. An empty problem (R, t or G = 0) returns OD_OK without a launch or a workspace.
 */
typedef struct {
  int64_t R, t, S, T, NQ, Lq;   /* rows, tokens per row, states, prefix capacity, questions, question length */
  int Hq, Hkv, D;
  int scale_dtype;              /* dtype of ksc/vsc: OD_BF16 or OD_F16 */
  float sm_scale;               /* softmax scale (head_dim ** -0.5) */
  int64_t G;                    /* number of row groups (used when row_groups != NULL) */
  int max_group_rows;           /* largest group (used when row_groups != NULL) */
  int prefix_bf16;              /* 1: Kp/Vp are bf16 (materialised), 0: int8 + ksc/vsc */
  int nsplit;                   /* CTAs per state prefix (0 or 1: one) */
} od_attn_dims;

OD_API int od_prefix_attn(const void* q, const void* Kp, const void* Vp, const void* ksc, const void* vsc,
                          const int32_t* row_state, const int32_t* p_lo, const int32_t* p_hi, const uint8_t* pmask,
                          const void* Kq, const void* Vq, const int32_t* row_q, const int32_t* q_len,
                          const void* k_own, const void* v_own, const int32_t* own_lo, const int32_t* own_hi,
                          const int32_t* row_groups, void* o, float* lse, od_attn_dims dims, void* workspace,
                          int64_t workspace_bytes, void* stream);
/* The split count for od_prefix_attn on a GPU of num_sms SMs and its workspace size in bytes (0 for one split). */
OD_API int od_prefix_attn_plan(const od_attn_dims* dims, int num_sms, int* nsplit, int64_t* workspace_bytes);
/* No reference counterpart (an addition of this library, not a replacement of a reference interface): od_prefix_attn
 * whose split workspace is a static 16 MiB device array of the library instead of a caller buffer, so the call
 * allocates nothing. Requests needing more scratch are rejected (OD_EINVAL). The array is shared by all calls on a
 * device: calls on one device must be ordered (one stream or synchronised streams). */
OD_API int od_prefix_attn_noalloc(const void* q, const void* Kp, const void* Vp, const void* ksc, const void* vsc,
                                  const int32_t* row_state, const int32_t* p_lo, const int32_t* p_hi,
                                  const uint8_t* pmask, const void* Kq, const void* Vq, const int32_t* row_q,
                                  const int32_t* q_len, const void* k_own, const void* v_own, const int32_t* own_lo,
                                  const int32_t* own_hi, const int32_t* row_groups, void* o, float* lse,
                                  od_attn_dims dims, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * (f.2) LM-head log-probabilities of given tokens: Backbone.token_logprob (backbone.py:165-178), the V3 trunk's
 * option log-prob feature (v3_lm_feature, v3.py:437-442 and 527-532):
 *     lp[m] = float(h[m]) . (float(qW[tok[m]]) * float(sW[tok[m]])) - logsumexp_v float(bf16(h[m] . Wb[v]))
 * h (M, H) bf16 (the final normed hidden state of the position before each token), Wb (V, H) bf16 = bf16(qW * sW)
 * (the tied head as head_rows() dequantises it, quant.py:202-203), qW (V, H) int8 + sW (V,) bf16 the int8 head,
 * tok (M,) int64, lp (M,) fp32 (-inf for a token outside [0, V)). H must be a multiple of 64. The vocabulary is
 * divided into vsplit ranges (od_lm_logprob_plan); workspace holds 8 x M x vsplit bytes of per-split partials.
 */
OD_API int od_lm_logprob_plan(int64_t M, int64_t V, int num_sms, int* vsplit, int64_t* workspace_bytes);
OD_API int od_lm_logprob(const void* h, int64_t M, int H, const void* Wb, const int8_t* qW, const void* sW,
                         int64_t V, const int64_t* tok, float* lp, void* workspace, int64_t workspace_bytes,
                         int vsplit, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * A12: the V3 decision trunk in fp32 (V3.forward, v3.py:606-709). Every trunk linear (nn.Linear in fp32, v3.py's
 * MHA :82-100 and XATGLU :53-67, the input projections) runs through od_gemm_f32 on operands held as a pair
 * hi = x rounded to tf32, lo = x - hi ("3xTF32" on the tensor cores: fp32-level results); the kernels that produce
 * a linear's input write that pair directly.
 *
 * od_split_tf32: x (M, K) fp32 (row stride ldx) -> hi, lo (M, K) (row stride ldo). Used for weights, once.
 * od_scalenorm_split: ScaleNorm (v3.py:43-50) of each row, g * x / max(||x||_2, eps), g a device fp32 scalar; with
 *   mix_w (n_mix fp32 weights, the softmax of layer_mix) the row is first the mix of n_mix feature layers stored
 *   side by side (V3._mix_wide, v3.py:328-341: x = sum_l mix_w[l] * float(row[l * K:(l + 1) * K])). x in dtype
 *   OD_BF16 / OD_F16 / OD_F32, K <= 8192. Writes hi, lo (M, K).
 * od_gemm_f32: y[out_rows[r]] = x[r] . W^T (+ bias) (+ res[out_rows[r]]), x = x_hi + x_lo (M, K), W = w_hi + w_lo
 *   (N, K) (nn.Linear's layout), bias (N,) or NULL, res rows at res + out_row * ldres (ldres 0: one row for every
 *   output row; res may be y: x = x + layer(x)) or NULL, out_rows (M,) int64 or NULL (identity). With rope_pos (M,)
 *   int32 the columns [0, rope_cols) - the q and / or k of MHA's projections - leave RoPE'd (v3.py:70-79) at row r's
 *   position: pairs (2i, 2i+1) of each rope_dh-wide head rotated by the angle fp32(pos * rope_inv[i]), rope_inv
 *   (rope_dh / 2,) fp32 = 1 / 10000^(2i / rope_dh) as the reference's formula evaluates it. K % 4 == 0; row
 *   strides in elements, multiples of 4 for x and W; operands 16-byte aligned.
 * od_xatglu_split: zv (M, 2F) = [wg x + bg | wv x + bv] -> the XATGLU product (v3.py:65-66)
 *   (((atan z + pi/2) / pi) * (1 + 2a) - a) * value as hi, lo (M, F); alpha a device fp32 scalar.
 * od_trunk_attn: scaled_dot_product_attention (v3.py:97, scale 1/sqrt(Dh)) of one MHA call with its additive mask
 *   built from ids instead of an (N, h, P, T) tensor; q and k arrive RoPE'd (od_gemm_f32's rope_pos):
 *     OD_TRUNK_SELF  keys with k_grp < 0 masked, + bonus[h] where q_grp == k_grp >= 0 (the option self-attention:
 *                    same_bias * same, masked_fill of padded keys, V3.forward :676-681)
 *     OD_TRUNK_KEYS  keys with k_grp < 0 masked (the cross-attention to the question, c_pad)
 *     OD_TRUNK_CLS   query i sees only keys with k_grp == i (the CLS readout of option i, :690-697)
 *   q row (b, i) at q + b * q_bstride + i * ldq + h * Dh (q_bstride = ldq = 0: one row shared by every query),
 *   k / v row (b, j) at + b * kv_bstride + j * ldkv + h * Dh; groups (B, Lq) and (B, Lk) int32.
 *   Output row (b, i) at o + (b * Lq + i) * ldo + h * Dh (heads side by side, the layout of the o projection's
 *   input), as fp32 (o) and / or as the hi / lo pair. Dh in {16, 32, 64}. q_len / k_len (B,) int32 or NULL: the
 *   real queries / keys of each batch row are a prefix of that length (the rest padding: keys past k_len are not
 *   read, queries past q_len get zeros - the reference computes values there that reach no logit). A query with no
 *   visible key gets zeros (only padded CLS options, whose logits are masked).
 */
enum { OD_TRUNK_SELF = 0, OD_TRUNK_KEYS = 1, OD_TRUNK_CLS = 2 };
OD_API int od_split_tf32(const float* x, int64_t ldx, int64_t M, int64_t K, float* hi, float* lo, int64_t ldo,
                         void* stream);
OD_API int od_scalenorm_split(const void* x, int dtype, int64_t ldx, int64_t M, int64_t K, const float* mix_w,
                              int n_mix, const float* g, float eps, float* hi, float* lo, int64_t ldo, void* stream);
OD_API int od_gemm_f32(const float* x_hi, const float* x_lo, int64_t ldx, const float* w_hi, const float* w_lo,
                       int64_t ldw, const float* bias, const float* res, int64_t ldres, const int64_t* out_rows,
                       const int32_t* rope_pos, const float* rope_inv, int rope_cols, int rope_dh, float* y,
                       int64_t ldy, int64_t M, int64_t N, int64_t K, void* stream);
OD_API int od_xatglu_split(const float* zv, int64_t ldzv, int64_t M, int64_t F, const float* alpha, float* hi,
                           float* lo, int64_t ldo, void* stream);
OD_API int od_trunk_attn(const float* q, int64_t ldq, int64_t q_bstride, const float* k, const float* v, int64_t ldkv,
                         int64_t kv_bstride, const int32_t* q_grp, const int32_t* k_grp, const float* bonus,
                         const int32_t* q_len, const int32_t* k_len, int mode, int64_t B, int64_t Lq, int64_t Lk,
                         int H, int Dh, float* o, float* o_hi, float* o_lo, int64_t ldo, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * A13: option readout, Decider._probs (decider.py:255-257):
 *     p[i, :] = softmax(logits[i, :] / T[i] + bias[i, :]) * mask[i, :]
 * logits (N, K) fp32, T (N) fp32, bias (N, K) fp32 or NULL, mask (N, K) uint8; probs (N, K) fp32.
 * If none_col (N) int32 is given (the explicit `none` text option, decider.py:296-303; -1 = absent), also writes
 * renorm (N, K) fp64: the probabilities clamped at 0 and renormalised over the caller's options 0..none_col-1
 * (all K columns when none_col[i] == -1) in fp64 (decider._normalize, :26-29; other columns 0), and p_none (N) =
 * p[i, none_col] (or 0).
 */
OD_API int od_readout(const float* logits, const float* T, const float* bias, const uint8_t* mask,
               const int32_t* none_col, int64_t N, int64_t K, float* probs, double* renorm, float* p_none,
               void* stream);

#ifdef __cplusplus
}
#endif
#endif /* OD_B200_H */
