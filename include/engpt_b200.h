/*
 * engpt_b200 C ABI: the forward hot path of enGPT (carried-radius nGPT) on
 * B200 (sm_100a).
 *
 * Every entry point takes raw device pointers, element counts/strides and a
 * CUDA stream handle (cudaStream_t passed as void*), launches its kernels on
 * that stream and returns an engpt_status.  Nothing here allocates device
 * memory or synchronises the stream; outputs are written into caller-owned
 * buffers.  On a non-zero status engpt_last_error() returns a message for
 * the calling thread.
 *
 * Reference interface each entry point replaces is cited as
 * <file>:<lines> inside the Pi-Willie/enGPT project.
 */
#ifndef ENGPT_B200_H
#define ENGPT_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ENGPT_API __attribute__((visibility("default")))
#else
#define ENGPT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types accepted for activations. */
enum engpt_dtype {
  ENGPT_F32 = 0,
  ENGPT_BF16 = 1
};

enum engpt_status {
  ENGPT_OK = 0,
  ENGPT_ERR_SHAPE = 1,       /* sizes inconsistent or out of the supported range */
  ENGPT_ERR_DTYPE = 2,       /* dtype code not supported by this entry point     */
  ENGPT_ERR_ALIGN = 3,       /* pointer or stride misaligned for vector/TMA use  */
  ENGPT_ERR_LAUNCH = 4,      /* CUDA launch error                                */
  ENGPT_ERR_TIMEOUT = 5,     /* a device-side wait ran out (see engpt_device_status) */
  ENGPT_ERR_UNSUPPORTED = 6, /* no kernel for this configuration                  */
  ENGPT_ERR_ARG = 7          /* null pointer or invalid scalar argument          */
};

/* Auxiliary output of the carried residual (the next GEMM's operand). */
enum engpt_aux_mode {
  ENGPT_AUX_NONE = 0,
  ENGPT_AUX_BF16_Y = 1,  /* bf16(Y_out): input of the next block's QKV projection      */
  ENGPT_AUX_BF16_H = 2,  /* bf16(Y_out / rho_out): input of up/gate or output head     */
  ENGPT_AUX_F32_H = 3    /* fp32 Y_out / rho_out (fp32 mode)                            */
};

/* Output layout of engpt_qkv_postprocess. */
enum engpt_qkv_layout {
  ENGPT_QKV_BTHD = 0,     /* q, k, v as separate [B, T, H, Dh] tensors (the reference's return layout)  */
  ENGPT_QKV_BHTD = 1,     /* q, k, v as separate [B, H, T, Dh] tensors (head-major)                     */
  ENGPT_QKV_INPLACE = 2   /* written back over qkv [B, T, 3, H, Dh] (q_out/k_out/v_out: NULL or qkv) */
};

/* Attention kernel selection (engpt_causal_attention `impl`). */
enum engpt_attn_impl {
  ENGPT_ATTN_AUTO = 0,   /* tcgen05 kernel when bf16 and head_dim in {64,128}, else SIMT */
  ENGPT_ATTN_TCGEN05 = 1,
  ENGPT_ATTN_SIMT = 2,
  ENGPT_ATTN_TCGEN05_1TILE = 3  /* tcgen05 kernel with one 128-query tile per CTA (head_dim 64 comparison path) */
};

/* Message for the last failing call on this host thread ("" if none). */
ENGPT_API const char* engpt_last_error(void);

/* ABI version of this library (major * 100 + minor). */
ENGPT_API int engpt_abi_version(void);

/*
 * Device-side error word of the current device: 0 when no kernel has
 * recorded a failure; otherwise the first failure recorded, its engpt_status
 * code in bits 0-7 and its site in the upper bits: ENGPT_ERR_TIMEOUT for a
 * bounded wait that ran out, ENGPT_ERR_ARG for an out-of-range token id or
 * target.  Synchronises the device.  engpt_clear_device_status() resets it.
 * A set word does not change what later launches compute.
 */
ENGPT_API int engpt_device_status(void);
ENGPT_API int engpt_clear_device_status(void);

/*
 * Failure-path self-test (no counterpart in the reference, which has no
 * device-side waits): one CTA whose first wait, on an mbarrier nothing
 * arrives on, runs out after limit_ns (0 < limit_ns <= 1 s) and records
 * ENGPT_ERR_TIMEOUT with site 99 in the device status word; a second role
 * of the same CTA waiting on another such barrier leaves through the CTA's
 * abort word.  flags_out (2 device ints) receives 1 for each wait that
 * reported failure.  The kernel returns normally and the context stays
 * usable; the caller clears the status word afterwards.
 */
ENGPT_API int engpt_selftest_wait_timeout(int64_t limit_ns, int* flags_out, void* stream);

/*
 * qkv_postprocess_from_carried -- engpt/kernels.py:139-179.
 *
 * qkv: [B, T, 3, H, Dh] contiguous, dtype `dtype` (raw projection Y W^T).
 * rho: [B, T] fp32.  cos_tab/sin_tab: [T, rope_half] fp32 (rope_half = Dh/2
 * rounded down, as rotary_frequencies builds them).  qk_scale: [H, Dh] fp32;
 * the scale applied is qk_scale * qk_mult (pass 1.0 for an effective scale).
 * Outputs q, k, v in `dtype`, laid out as engpt_qkv_layout says: separate
 * [B, T, H, Dh] or [B, H, T, Dh] tensors, or in place over qkv (the layout
 * the reference's no-grad path leaves, engpt/kernels.py:174-178).
 */
ENGPT_API int engpt_qkv_postprocess(const void* qkv, int dtype, const float* rho,
                          const float* cos_tab, const float* sin_tab, int rope_half,
                          const float* qk_scale, float qk_mult, float norm_eps,
                          int B, int T, int H, int Dh,
                          void* q_out, void* k_out, void* v_out, int out_layout,
                          void* stream);

/*
 * causal_sdpa -- engpt/kernels.py:417-431 (softmax(scale * q k^T + causal) v).
 *
 * q, k, v, o: element strides (batch, token, head) given in `strides`
 * (12 int64: q_b, q_t, q_h, k_b, k_t, k_h, v_b, v_t, v_h, o_b, o_t, o_h); the
 * head_dim axis is contiguous.  dtype ENGPT_BF16 or ENGPT_F32 for all four.
 */
ENGPT_API int engpt_causal_attention(const void* q, const void* k, const void* v, void* o,
                           int dtype, int B, int T, int H, int Dh, float scale,
                           const int64_t* strides, int impl, void* stream);

/*
 * causal_sdpa as the nGPT block calls it -- engpt/models.py:143-151 (q, k from
 * qkv_postprocess_from_carried, engpt/kernels.py:139-179, then causal_sdpa
 * engpt/kernels.py:417-431 with scale sqrt(Dh), engpt/kernels.py:434-435).
 *
 * Same arguments as engpt_causal_attention plus the effective score scales:
 * q and k of head h must be unit vectors (per head) multiplied elementwise
 * by qk_scale[h, :] * qk_mult (qk_scale [H, Dh] fp32 on the device), which is
 * what the QKV post-process produces.  Then every score satisfies
 * |q.k| <= max_i (qk_scale[h, i] qk_mult)^2, and the bf16 kernels for head_dim
 * 64 and 128 exponentiate against that fixed per-head bound instead of a
 * running row maximum (no rescaling of P, l or O).  The bound is read on the
 * device (no host synchronisation).  A head whose bound exceeds 48 in log2
 * units (scale * log2(e) * max s^2) runs the running-max softmax, as do other
 * head dims and fp32 (the engpt_causal_attention kernels).
 */
ENGPT_API int engpt_ngpt_attention(const void* q, const void* k, const void* v, void* o, int dtype, int B, int T,
                                   int H, int Dh, float scale, const int64_t* strides, const float* qk_scale,
                                   float qk_mult, void* stream);

/*
 * carried_residual_gauge -- engpt/kernels.py:277-324 (with the unfused pair
 * carried_residual 232-274 + gauge_carried_state 327-338 as the
 * max_radius <= 0 / > 0 cases).
 *
 * y, y_out: [rows, d] fp32 (may alias); rho, rho_out: [rows] fp32 (may
 * alias); branch: [rows, d] in `branch_dtype`.  alpha: [d] fp32, the applied
 * alpha is (alpha_abs ? |alpha| : alpha) * alpha_mult.  aux_out receives the
 * engpt_aux_mode side output ([rows, d], bf16 or fp32) when aux_mode != 0.
 */
ENGPT_API int engpt_carried_residual_gauge(const float* y, const float* rho, const void* branch,
                                 int branch_dtype, const float* alpha, float alpha_mult,
                                 int alpha_abs, float branch_eps, float residual_eps,
                                 float max_radius, int64_t rows, int d,
                                 float* y_out, float* rho_out, void* aux_out, int aux_mode,
                                 void* stream);

/* rotary_frequencies -- engpt/kernels.py:355-374: fp32 cos/sin [T, Dh/2]. */
ENGPT_API int engpt_rotary_tables(int T, int Dh, float theta, float* cos_out, float* sin_out, void* stream);

/*
 * EfficientNGPT.forward embedding step -- engpt/models.py:263-268:
 * y = token_emb[idx] (fp32 [n, d]), rho = 1; aux_bf16 (optional) = bf16(y).
 * Out-of-range ids are reported through the device status word.
 */
ENGPT_API int engpt_embed_carried(const int64_t* idx, const float* emb, int64_t n_tokens, int d,
                        int64_t vocab, float* y_out, float* rho_out, void* aux_bf16,
                        void* stream);

/*
 * carried_up_gate_swiglu epilogue -- engpt/kernels.py:200-206: given the
 * up/gate projection ug [rows, 2W] (`dtype`), writes
 * out = (u * s_u * u_mult) * silu(gate * s_gate * gate_mult) in `out_dtype`.
 */
ENGPT_API int engpt_swiglu(const void* ug, int dtype, const float* s_u, const float* s_gate,
                 float u_mult, float gate_mult, int64_t rows, int width,
                 void* out, int out_dtype, void* stream);

/*
 * Row-scaled cast for the output head -- engpt/kernels.py:229 and
 * engpt/models.py:366-368: out[r, :] = src[r, :] * (scale[r] * mult),
 * written in out_dtype.  With scale == NULL it is a plain cast.
 */
ENGPT_API int engpt_scale_rows_cast(const float* src, const float* scale, float mult, int64_t rows,
                          int64_t cols, void* out, int out_dtype, void* stream);

/*
 * Batched fp32 -> bf16 cast of n tensors (src[i], dst[i], counts[i] elements)
 * in one launch per 64 tensors: the bf16 copies of the linear weights that
 * autocast makes on every forward (engpt/models.py:142,152,166,172 under
 * torch.autocast).  src/dst/counts are host arrays of device pointers.
 */
ENGPT_API int engpt_cast_f32_bf16_many(const void* const* src, void* const* dst, const int64_t* counts, int n,
                                       void* stream);

/*
 * Dense projection -- the bias-free F.linear of engpt/models.py:142,152,166,172
 * (nn.Linear under bf16 autocast): C[M, N] = A[M, K] * B[N, K]^T, bf16 A, B
 * (rows of K contiguous elements, row strides lda / ldb) and bf16 C (row
 * stride ldc), fp32 accumulation.  Persistent tcgen05 kernel; rows 16-byte
 * aligned, K a multiple of 8.
 */
ENGPT_API int engpt_gemm_bf16(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc, int M,
                              int N, int K, void* stream);

/*
 * QKV projection with the QKV post-process fused into the GEMM epilogue --
 * F.linear of engpt/models.py:142 followed by qkv_postprocess_from_carried
 * (engpt/kernels.py:139-179) on the fp32 accumulator: x [B*T, in_features]
 * bf16, w_qkv [3 * H * Dh, in_features] bf16 (the q rows of the H heads, then
 * their k rows, then their v rows; in_features = H * Dh for the whole model,
 * the model width for a head group of a head split); writes the
 * post-processed q | k | v rows into qkv_out [B*T, 3, H, Dh] bf16 (the layout
 * engpt_qkv_postprocess leaves in place).  head_dim 64 or 128, H * Dh a
 * multiple of 256, in_features a multiple of 8.
 */
ENGPT_API int engpt_qkv_projection(const void* x, int in_features, const void* w_qkv, const float* rho,
                                   const float* cos_tab, const float* sin_tab, int rope_half, const float* qk_scale,
                                   float qk_mult, float norm_eps, int B, int T, int H, int Dh, void* qkv_out,
                                   void* stream);

/*
 * Up/gate projection with SwiGLU fused into the GEMM epilogue --
 * carried_up_gate_swiglu (engpt/kernels.py:182-206) from x = bf16(Y / rho):
 * w_ug [2 * width, d] bf16 (u rows, then gate rows, as nn.Linear stores them),
 * hidden [rows, width] bf16 = (u * s_u * u_mult) * silu(gate * s_gate *
 * gate_mult), computed from the fp32 accumulator.  width a multiple of 128.
 */
ENGPT_API int engpt_up_gate_swiglu(const void* x, const void* w_ug, const float* s_u, const float* s_gate,
                                   float u_mult, float gate_mult, int64_t rows, int d, int width, void* hidden,
                                   void* stream);

/*
 * Output projection with the carried residual fused into the GEMM epilogue --
 * branch = self.out_proj(attn) / self.down_proj(hidden) (engpt/models.py:152,
 * 172 under bf16 autocast) followed by carried_residual_gauge
 * (engpt/kernels.py:277-324, call sites engpt/models.py:153-161, 173-181):
 * a [rows, K] bf16 (row stride lda), w [d, K] bf16 (row stride ldw); the
 * branch is rounded to bf16 as the autocast GEMM output is and never stored.
 * y, rho, alpha, the epsilons, y_out, rho_out, aux_out and aux_mode
 * (ENGPT_AUX_NONE, _BF16_Y or _BF16_H) mean what they mean for
 * engpt_carried_residual_gauge; y_out may be y and rho_out may be rho.
 * d in {256, 512, 768, 1024}; K a multiple of 8.
 */
ENGPT_API int engpt_gemm_carried_residual(const void* a, int64_t lda, const void* w, int64_t ldw, int K,
                                          const float* y, const float* rho, const float* alpha, float alpha_mult,
                                          int alpha_abs, float branch_eps, float residual_eps, float max_radius,
                                          int64_t rows, int d, float* y_out, float* rho_out, void* aux_out,
                                          int aux_mode, void* stream);

/*
 * Output head and token cross-entropy in one pass over the logits --
 * F.linear(x, w_head) of engpt/kernels.py:209-229 (x = bf16(Y / rho), w_head
 * = bf16(E_out * s_z_eff), [vocab, d]) followed by F.cross_entropy
 * (engpt/models.py:328-333, mean, ignore_index -100).  The tcgen05 GEMM
 * stores the bf16 logits [rows, vocab] (row stride ld) and, from the same
 * bf16 values, each row's log-sum-exp per 256-column tile into `partials`
 * (scratch of ceil(vocab / 256) * rows float pairs); a second kernel merges
 * them, subtracts the target's logit into row_loss [rows] (scratch) and
 * loss_out receives the fp32 mean.  d and ld multiples of 8.
 */
ENGPT_API int engpt_logits_cross_entropy(const void* x, const void* w_head, int64_t rows, int d, int64_t vocab,
                                         void* logits, int64_t ld, const int64_t* targets, void* partials,
                                         float* row_loss, float* loss_out, void* stream);

/*
 * Optimizer-side sphere operations of nGPT training (NGPTAdamW,
 * engpt/optim.py:74-109), in place on a [rows, cols] row-major matrix of
 * `dtype` (ENGPT_F32 or ENGPT_BF16), computed in fp32:
 *
 * normalize_rows_ -- engpt/kernels.py:98-105 (Triton _row_normalize_kernel
 *   32-42): x[r, :] /= max(|x[r, :]|, eps).
 * normalize_columns_ -- engpt/kernels.py:108-116 (_column_normalize_kernel
 *   44-55): x[:, c] /= max(|x[:, c]|, eps).
 * project_row_grad_ -- engpt/kernels.py:119-125 (_row_grad_project_kernel
 *   57-67): grad[r, :] -= (grad[r, :] . weight[r, :]) weight[r, :].
 * project_column_grad_ -- engpt/kernels.py:128-136
 *   (_column_grad_project_kernel 69-81): grad[:, c] -= (grad[:, c] .
 *   weight[:, c]) weight[:, c].
 *
 * weight and grad share the dtype and shape.  The column forms read each
 * column tile in row splits and take caller scratch of
 * engpt_column_scratch_floats(rows, cols) floats for the partial sums.
 */
ENGPT_API int engpt_normalize_rows(void* x, int dtype, int64_t rows, int64_t cols, float eps, void* stream);
ENGPT_API int engpt_normalize_columns(void* x, int dtype, int64_t rows, int64_t cols, float eps, float* scratch,
                                      void* stream);
ENGPT_API int engpt_project_row_grad(const void* weight, void* grad, int dtype, int64_t rows, int64_t cols,
                                     void* stream);
ENGPT_API int engpt_project_column_grad(const void* weight, void* grad, int dtype, int64_t rows, int64_t cols,
                                        float* scratch, void* stream);
ENGPT_API int64_t engpt_column_scratch_floats(int64_t rows, int64_t cols);

/*
 * Token cross-entropy -- engpt/models.py:328-333 (F.cross_entropy, mean).
 * logits [rows, vocab] with leading dimension ld (elements), `dtype`;
 * targets int64 [rows].  row_loss [rows] fp32 is caller-provided scratch;
 * loss_out receives the fp32 mean.
 */
ENGPT_API int engpt_cross_entropy(const void* logits, int dtype, int64_t rows, int64_t vocab, int64_t ld,
                        const int64_t* targets, float* row_loss, float* loss_out, void* stream);

/*
 * Token cross-entropy that allocates nothing and needs no scratch buffer from
 * the caller.  This entry point has no counterpart in the reference.
 *
 * It is for callers that cannot call cudaMalloc: a host that only owns the
 * logits, targets and loss buffers it was handed (an FFI or embedded runtime
 * with no device allocator of its own), or a serving loop that must not call
 * cudaMalloc because it can synchronise the device.  Same arguments and result
 * as engpt_cross_entropy, without `row_loss`: the per-row losses go to a
 * fixed array of ENGPT_CE_NOALLOC_MAX_ROWS floats (1 MiB) that lives in the
 * library's device memory; every GPU that loads the library holds it until the
 * process exits.  More rows than that are rejected with ENGPT_ERR_SHAPE.
 *
 * Every call looks up the array's device address on the current device (the
 * first call on a device may load the library's device code there); make
 * that first call before any stream capture.
 * All calls share the one array and it keeps the last call's contents; each
 * call writes every entry it reads, so nothing needs clearing.  Calls that
 * overlap on the GPU (other streams, other threads) race on the array.
 */
#define ENGPT_CE_NOALLOC_MAX_ROWS 262144
ENGPT_API int engpt_cross_entropy_noalloc(const void* logits, int dtype, int64_t rows, int64_t vocab,
                                          int64_t ld, const int64_t* targets, float* loss_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ENGPT_B200_H */
