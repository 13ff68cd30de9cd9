/*
 * flashmhc.h -- C ABI of the B200 (sm_100a) mHC-lite hot-path kernels.
 *
 * libflashmhc_sm100.so exports exactly the functions declared here.  Every
 * entry point:
 *   - takes raw device pointers, element counts and a cudaStream_t passed as
 *     `void *` (NULL = legacy default stream); no torch or C++ types;
 *   - launches asynchronously on that stream and never synchronises;
 *   - allocates no device memory (any scratch is passed in by the caller);
 *   - returns an fmhc_status; on failure fmhc_last_error() describes it
 *     (thread-local; valid until the next call on the same thread);
 *   - accepts T == 0 (returns FMHC_OK without launching).
 *
 * Tensor layouts are dense row-major.  n (number of residual streams) must be
 * 4.  "bf16" buffers hold IEEE bfloat16 values, "f32" buffers IEEE float32.
 * Coefficient buffers (h_pre, h_post, H_merged, their gradients, inv_rms) must
 * be 16-byte aligned; bf16 buffers must be at least 2-byte aligned (16-byte
 * alignment and C % 8 == 0 select the 128-bit vector path).
 *
 * Each function replaces one launch of the reference's Triton kernels; the
 * reference interface it stands in for is cited beside it (paths relative to
 * the alint77/flash-mHC project root).
 */
#ifndef FLASHMHC_H
#define FLASHMHC_H

#include <stdint.h>

#if defined(__GNUC__)
#define FMHC_API __attribute__((visibility("default")))
#else
#define FMHC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum fmhc_status {
  FMHC_OK = 0,
  FMHC_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, n != 4 ... */
  FMHC_ERR_UNSUPPORTED = 2,      /* shape the kernels do not implement      */
  FMHC_ERR_ALIGNMENT = 3,        /* a pointer violates the alignment rule   */
  FMHC_ERR_LAUNCH = 4,           /* the CUDA launch itself failed           */
  FMHC_ERR_CUDA = 5,             /* another CUDA runtime/driver call failed */
  FMHC_ERR_WORKSPACE = 6         /* caller-provided workspace too small     */
} fmhc_status;

/* Human-readable description of the last failure on this thread ("" if none). */
FMHC_API const char *fmhc_last_error(void);

/* Library version string, e.g. "flashmhc-sm100 0.1.0". */
FMHC_API const char *fmhc_version(void);

/* Failure detection for the tensor-core kernels.  Every wait of those kernels
 * on a barrier is bounded (about 1 s); a wait that expires makes the kernel
 * record a non-zero site code in a per-device error word, release its
 * resources and return early (its outputs are then invalid).  This call
 * synchronises the current device, stores the word in *code (0 = no expired
 * wait since the last call) and clears it.  No reference counterpart: the
 * reference's Triton kernels have no device-side failure reporting. */
FMHC_API int fmhc_check_device_error(int *code);

/* Test hook for the failure path above (not for production use): the
 * tensor-core K1 forward (x (T, nC) bf16, W (32, nC) bf16, 16-byte aligned,
 * nC % 64 == 0, T >= 1) in which the first CTA arms its first pipeline stage
 * for a copy that it never issues.  Its waits on that stage expire after the
 * bound (about 1 s each, two in a row), it records a site code in the error
 * word, frees its tensor memory and returns; the other CTAs finish normally.
 * The outputs are not meaningful; the context stays usable, so a following
 * fmhc_check_device_error reports the code and later calls run normally.
 * While the word is set, fmhc_k1_bwd and fmhc_k1_bwd_noalloc write grad_W as
 * NaN.  No reference counterpart. */
FMHC_API int fmhc_debug_k1_fwd_lost_copy(const void *x, const void *W, void *out,
                                         float *inv_rms, int64_t T, int64_t nC, void *stream);

/* ------------------------------------------------------------------------
 * K1 forward: fused RMSNorm + thin projection.
 *   inv_rms[t] = rsqrt(sum_k x[t,k]^2 / nC + 1e-6)                    (f32)
 *   out[t,d]   = bf16( (sum_k x[t,k] * W[d,k]) * inv_rms[t] )   f32 accumulate
 * x (T, nC) bf16, W (D, nC) bf16 -> out (T, D) bf16, inv_rms (T,) f32.  D <= 32.
 * Replaces op flash_mhc::fused_rmsnorm_project (src/flash_mhc/ops.py:24-26,
 * 205-264) and kernel _fused_rmsnorm_project_fwd_kernel
 * (src/flash_mhc/kernels.py:250-303).
 */
FMHC_API int fmhc_k1_fwd(const void *x, const void *W, void *out, float *inv_rms,
                int64_t T, int64_t nC, int64_t D, void *stream);

/* ------------------------------------------------------------------------
 * K1 backward, grad_x only.
 *   s[t]       = (sum_d go[t,d] * proj[t,d]) * inv_rms[t]^2 / nC
 *   grad_x[t,k]= bf16( inv_rms[t] * sum_d go[t,d] W[d,k] - s[t] * x[t,k] )
 * grad_out, proj (T, D) bf16; x (T, nC) bf16; W (D, nC) bf16; inv_rms (T,) f32
 * -> grad_x (T, nC) bf16.
 * Replaces op flash_mhc::fused_rmsnorm_project_bwd_dx (src/flash_mhc/ops.py:27-29,
 * 267-344) and kernel _fused_rmsnorm_project_bwd_dx_kernel
 * (src/flash_mhc/kernels.py:306-376).
 */
FMHC_API int fmhc_k1_bwd_dx(const void *grad_out, const void *x, const void *W,
                   const void *proj, const float *inv_rms, void *grad_x,
                   int64_t T, int64_t nC, int64_t D, void *stream);

/* ------------------------------------------------------------------------
 * K1 backward, grad_x AND grad_W in one pass over x.
 *   grad_x as fmhc_k1_bwd_dx;
 *   grad_W[d,k] = bf16( sum_t bf16(go[t,d] * inv_rms[t]) * x[t,k] )   f32 accumulate
 * -> grad_x (T, nC) bf16, grad_W (D, nC) bf16.
 * `workspace` is caller-owned device memory of at least
 * fmhc_k1_bwd_workspace_size(T, nC, D) bytes (256-byte aligned; the size
 * depends on the current device's SM count); its contents on entry do not
 * matter and the result does not depend on them (the grad_W reduction order
 * is fixed, so results are bitwise reproducible).  While the device error
 * word is set (a bounded wait expired; see fmhc_check_device_error), grad_W
 * is written as NaN instead of a sum of partials that were not all written.
 * Replaces the K1 autograd formula (src/flash_mhc/ops.py:678-685): the
 * bwd-dx op plus the separate cuBLAS matmul for grad_W (ops.py:683-684).
 */
FMHC_API int64_t fmhc_k1_bwd_workspace_size(int64_t T, int64_t nC, int64_t D);
FMHC_API int fmhc_k1_bwd(const void *grad_out, const void *x, const void *W,
                         const void *proj, const float *inv_rms, void *grad_x,
                         void *grad_W, void *workspace, int64_t workspace_bytes,
                         int64_t T, int64_t nC, int64_t D, void *stream);

/* ------------------------------------------------------------------------
 * K1 backward without a caller workspace: same inputs, outputs and results as
 * fmhc_k1_bwd, but the scratch comes from a fixed 32 MiB array inside the
 * library, so this call allocates no memory and needs none from the caller.
 * For callers that cannot allocate device memory: hosts that only hold
 * pointers handed to them and have no device allocator of their own (C, Go or
 * Java code calling through this ABI, plugins inside another framework's
 * memory pool), serving runtimes that reserve all HBM up front, and
 * latency-critical paths where cudaMalloc (which can synchronise the device)
 * is not allowed.
 * Limit: fmhc_k1_bwd_workspace_size(T, nC, D) must not exceed 32 MiB.  On
 * the tensor-core path (nC a multiple of 128) the workspace is the grad_W
 * partials alone, at most 18.5 MiB at any T; the CUDA-core path needs up to
 * 2 KiB x nC, so it fits up to nC = 16384.  Larger calls fail with
 * FMHC_ERR_WORKSPACE and should use fmhc_k1_bwd.  Every GPU that loads the
 * library holds the 32 MiB until the process exits.  The first call in each
 * CUDA context (once per device, and again after a device reset creates a new
 * context) looks up the array's device address; make the first call on each
 * device before any stream capture.  All calls share the array, so calls that
 * overlap on the same GPU race and must not be issued; when a call succeeds
 * the array's previous contents do not matter (after an expired wait grad_W
 * is NaN, as for fmhc_k1_bwd).
 * No counterpart in the reference (its ops always allocate through torch).
 */
FMHC_API int fmhc_k1_bwd_noalloc(const void *grad_out, const void *x, const void *W,
                                 const void *proj, const float *inv_rms, void *grad_x,
                                 void *grad_W, int64_t T, int64_t nC, int64_t D,
                                 void *stream);

/* ------------------------------------------------------------------------
 * K3 forward: pre-map of the n streams into the layer input.
 *   out[t,c] = bf16( sum_j h_pre[t,j] * x[t,j,c] )
 * x (T, n, C) bf16, h_pre (T, n) f32 -> out (T, C) bf16.
 * Replaces op flash_mhc::fused_pre_map (src/flash_mhc/ops.py:31, 347-414) and
 * kernel _fused_pre_map_fwd_kernel (src/flash_mhc/kernels.py:673-717).
 */
FMHC_API int fmhc_k3_fwd(const void *x, const float *h_pre, void *out,
                int64_t T, int64_t n, int64_t C, void *stream);

/* ------------------------------------------------------------------------
 * K3 backward (fused).
 *   grad_x[t,j,c] = bf16( h_pre[t,j] * go[t,c] )
 *   grad_h[t,j]   = sum_c x[t,j,c] * go[t,c]                         (f32)
 * grad_out (T, C) bf16, x (T, n, C) bf16, h_pre (T, n) f32
 * -> grad_x (T, n, C) bf16, grad_h (T, n) f32.  grad_x may be NULL: then only
 * grad_h is computed (grad_x is then formed by fmhc_mhc_grad_x_combine).
 * Replaces op flash_mhc::fused_pre_map_backward (src/flash_mhc/ops.py:32-34,
 * 417-493) and kernel _fused_pre_map_bwd_fused_kernel_n4
 * (src/flash_mhc/kernels.py:720-853).
 */
FMHC_API int fmhc_k3_bwd(const void *grad_out, const void *x, const float *h_pre,
                void *grad_x, float *grad_h,
                int64_t T, int64_t n, int64_t C, void *stream);

/* ------------------------------------------------------------------------
 * K4 forward: post-res mixing.
 *   out[t,i,c] = bf16( sum_j H[t,i,j] * x[t,j,c] + h_post[t,i] * lo[t,c] )
 * x (T, n, C) bf16, lo (T, C) bf16, H (T, n, n) f32, h_post (T, n) f32
 * -> out (T, n, C) bf16.
 * Replaces op flash_mhc::fused_post_res (src/flash_mhc/ops.py:36-38, 496-567)
 * and kernel _fused_post_res_fwd_kernel_n4 (src/flash_mhc/kernels.py:384-481).
 */
FMHC_API int fmhc_k4_fwd(const void *x, const void *lo, const float *H,
                const float *h_post, void *out,
                int64_t T, int64_t n, int64_t C, void *stream);

/* ------------------------------------------------------------------------
 * K4 backward (fused, one pass over grad_out, x and lo).
 *   grad_lo[t,c]  = bf16( sum_i h_post[t,i] * go[t,i,c] )
 *   grad_hp[t,i]  = sum_c go[t,i,c] * lo[t,c]                        (f32)
 *   grad_H[t,i,j] = sum_c go[t,i,c] * x[t,j,c]                       (f32)
 *   grad_x[t,j,c] = bf16( sum_i H[t,i,j] * go[t,i,c] )
 * grad_x may be NULL: then only grad_lo, grad_hp and grad_H are computed and
 * one (T, n, C) write is saved (fmhc_mhc_grad_x_combine_post forms K4's
 * grad_x later from go and H).
 * Replaces op flash_mhc::fused_post_res_backward (src/flash_mhc/ops.py:39-41,
 * 570-667) and kernel _fused_post_res_bwd_fused_kernel_n4
 * (src/flash_mhc/kernels.py:487-665).
 */
FMHC_API int fmhc_k4_bwd(const void *grad_out, const void *x, const void *lo,
                const float *H, const float *h_post,
                void *grad_x, void *grad_lo, float *grad_H, float *grad_hp,
                int64_t T, int64_t n, int64_t C, void *stream);

/* ------------------------------------------------------------------------
 * Gradient of the residual streams from the three paths that read them:
 *   grad_x[t,j,c] = bf16( gx1[t,j,c] + h_pre[t,j] * grad_li[t,c] + gx4[t,j,c] )
 * gx1: K1's grad_x (T, n, C) bf16; grad_li: the gradient of the layer input
 * (T, C) bf16 (K3's upstream gradient); gx4: K4's grad_x (T, n, C) bf16 or
 * NULL; h_pre (T, n) f32.  grad_x may alias gx1.  One pass instead of K3's
 * grad_x write plus two separate additions.
 * No counterpart in the reference (its autograd engine sums three tensors).
 */
FMHC_API int fmhc_mhc_grad_x_combine(const void *gx1, const void *grad_li, const float *h_pre,
                                     const void *gx4, void *grad_x, int64_t T, int64_t n,
                                     int64_t C, void *stream);

/* ------------------------------------------------------------------------
 * The same combination with K4's grad_x formed in place from K4's upstream
 * gradient instead of read back:
 *   grad_x[t,j,c] = bf16( gx1[t,j,c] + h_pre[t,j] * grad_li[t,c]
 *                         + sum_i H[t,i,j] * grad_out[t,i,c] )
 * grad_out: the gradient of the block output (T, n, C) bf16; H: H_merged
 * (T, n, n) f32.  With fmhc_k4_bwd(grad_x = NULL) this saves K4's (T, n, C)
 * grad_x write and its read here.  grad_x may alias gx1.
 * No counterpart in the reference (its autograd engine sums three tensors).
 */
FMHC_API int fmhc_mhc_grad_x_combine_post(const void *gx1, const void *grad_li,
                                          const float *h_pre, const void *grad_out,
                                          const float *H, void *grad_x, int64_t T, int64_t n,
                                          int64_t C, void *stream);

/* ------------------------------------------------------------------------
 * K2 forward: the per-token coefficient math on the 32 projection logits
 * (n = 4, D = 32), one launch.
 *   h_pre  = sigmoid(a_pre  * proj[:, 0:4]  + bias[0:4])
 *   h_post = 2 sigmoid(a_post * proj[:, 4:8] + bias[4:8])
 *   a      = softmax(a_res * proj[:, 8:32] + bias[8:32])
 *   H_merged[i][j] = sum_k a[k] perm[k][4i+j] - h_post[i] h_pre[j]
 * proj (T, 32) bf16; params (35,) f32 = [a_pre, a_post, a_res, bias[32]];
 * perm (24, 16) f32 -> h_pre, h_post (T, 4) f32, H_merged (T, 4, 4) f32.  The
 * parameters are rounded to bf16 as the reference's .to(dt) does; the
 * arithmetic and the outputs are f32 (the reference's bf16 eager K2 rounds
 * every op; f32 keeps the block within 2e-2 / 1e-2 of its float32 path).
 * Replaces the eager K2 of the caller (src/flash_mhc/block.py:150-170),
 * ~20 torch launches.
 */
FMHC_API int fmhc_k2_fwd(const void *proj, const float *params, const float *perm,
                         float *h_pre, float *h_post, float *H_merged, int64_t T,
                         void *stream);

/* Element types of fmhc_k2_fwd_typed's parameter pointers. */
enum fmhc_dtype { FMHC_DTYPE_F32 = 0, FMHC_DTYPE_BF16 = 1 };

/* ------------------------------------------------------------------------
 * The same K2 forward reading the parameters where they live, in their own
 * dtype (f32 or bf16, `param_dtype` for the three alphas and the 32 bias
 * entries, `perm_dtype` for perm (24, 16)): a module's alpha_pre, alpha_post,
 * alpha_res, W_all.bias and perm_mat tensors are passed as they are, so no
 * packing launch runs before it and a captured CUDA graph reads the live
 * values.  Results are identical to fmhc_k2_fwd on the packed f32 copy.
 * No counterpart in the reference (see fmhc_k2_fwd).
 */
FMHC_API int fmhc_k2_fwd_typed(const void *proj, const void *alpha_pre, const void *alpha_post,
                               const void *alpha_res, const void *bias, int param_dtype,
                               const void *perm, int perm_dtype, float *h_pre, float *h_post,
                               float *H_merged, int64_t T, void *stream);

/* ------------------------------------------------------------------------
 * The pre-block of an mHC-lite layer in one call: K1 (x (T, n, C) bf16 as
 * x_flat (T, nC), W (32, nC) bf16 -> proj (T, 32) bf16, inv_rms (T,) f32),
 * K2 on proj (parameters as in fmhc_k2_fwd_typed -> h_pre, h_post (T, 4),
 * H_merged (T, 4, 4) f32) and, when layer_input is not NULL, K3
 * (layer_input (T, C) bf16 = pre-map of x with h_pre).  K1 runs the kernel
 * fmhc_k1_fwd would run, with K2 in its epilogue (no launch and no read of
 * proj for K2); for T <= 888 with C % 8 == 0 and 16-byte aligned x, W and
 * layer_input, K3 runs in the same kernel too (one launch in all).  Every
 * output is bit-identical to fmhc_k1_fwd -> fmhc_k2_fwd_typed -> fmhc_k3_fwd.
 * proj, h_pre, h_post and H_merged 16-byte aligned; n == 4.
 * Replaces the reference's MHCLiteBlock._mhc_pre_map_triton
 * (src/flash_mhc/block.py:172-177 with _mhc_coeffs_triton, 150-170): its
 * fused_rmsnorm_project (ops.py:205-264), eager coefficient math and
 * fused_pre_map (ops.py:347-414) calls.
 */
FMHC_API int fmhc_mhc_pre_fwd(const void *x, const void *W, const void *alpha_pre,
                              const void *alpha_post, const void *alpha_res, const void *bias,
                              int param_dtype, const void *perm, int perm_dtype, void *proj,
                              float *inv_rms, float *h_pre, float *h_post, float *H_merged,
                              void *layer_input, int64_t T, int64_t n, int64_t C, void *stream);

/* ------------------------------------------------------------------------
 * K2 backward: given the f32 gradients of h_pre, h_post and H_merged, returns
 * grad_proj (T, 32) bf16 and grad_params (35,) f32 (summed over tokens in a
 * fixed order, deterministic).  `workspace` (256-byte aligned) holds per-block
 * partial sums; size from fmhc_k2_bwd_workspace_size(T).
 * Replaces the torch autograd backward of the eager K2 (src/flash_mhc/block.py:150-170).
 */
FMHC_API int64_t fmhc_k2_bwd_workspace_size(int64_t T);
FMHC_API int fmhc_k2_bwd(const void *proj, const float *params, const float *perm,
                         const float *grad_h_pre, const float *grad_h_post,
                         const float *grad_H_merged, void *grad_proj, float *grad_params,
                         void *workspace, int64_t workspace_bytes, int64_t T, void *stream);

/* ------------------------------------------------------------------------
 * The same K2 backward with the parameters read where they live (as
 * fmhc_k2_fwd_typed) and their gradients written in the parameters' own dtype
 * (`param_dtype`; bf16 gradients are rounded once from the f32 sums):
 * grad_alpha_pre, grad_alpha_post, grad_alpha_res one value each, grad_bias
 * 32.  So a module's parameter gradients need no packing before or casts
 * after.  Same workspace as fmhc_k2_bwd.  T == 0 writes zero gradients.
 * No counterpart in the reference (see fmhc_k2_bwd).
 */
FMHC_API int fmhc_k2_bwd_typed(const void *proj, const void *alpha_pre, const void *alpha_post,
                               const void *alpha_res, const void *bias, int param_dtype,
                               const void *perm, int perm_dtype, const float *grad_h_pre,
                               const float *grad_h_post, const float *grad_H_merged,
                               void *grad_proj, void *grad_alpha_pre, void *grad_alpha_post,
                               void *grad_alpha_res, void *grad_bias, void *workspace,
                               int64_t workspace_bytes, int64_t T, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASHMHC_H */
