// Internal (C++) launchers behind the C ABI in include/flashmhc.h.  They assume
// the arguments were validated by capi.cu and only enqueue kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fmhc {

// capi.cu -- sets this thread's fmhc_last_error() text, returns `code`.
int set_last_error(int code, const char *msg);

// k3k4_stream.cu -- `vec` is the bf16 chunk width (8, 4, 2 or 1).
void launch_k3_fwd(const void *x, const float *hp, void *out, int64_t T, int C, int vec,
                   cudaStream_t s);
void launch_k3_bwd(const void *go, const void *x, const float *hp, void *gx, float *gh,
                   int64_t T, int C, int vec, cudaStream_t s);
void launch_k4_fwd(const void *x, const void *lo, const float *H, const float *hp, void *out,
                   int64_t T, int C, int vec, cudaStream_t s);
void launch_grad_x_combine(const void *gx1, const void *gli, const float *hp, const void *gx4,
                           void *gx, int64_t T, int C, int vec, cudaStream_t s);
void launch_grad_x_combine_post(const void *gx1, const void *gli, const float *hp,
                                const void *go, const float *H, void *gx, int64_t T, int C,
                                int vec, cudaStream_t s);
void launch_k4_bwd(const void *go, const void *x, const void *lo, const float *H,
                   const float *hp, void *gx, void *glo, float *gH, float *ghp, int64_t T,
                   int C, int vec, cudaStream_t s);

// k1_simt.cu -- general-shape K1 (vec is 8 or 1).
void launch_k1_fwd_simt(const void *x, const void *W, void *out, float *inv_rms, int64_t T,
                        int nC, int D, int vec, cudaStream_t s);
// Small-T forward (block per 2 tokens, k split over the block); D == 32,
// nC % 8 == 0, x and W 16-byte aligned.  With `coeffs` non-null it also runs
// K2 (writing h_pre, h_post, H, 16-byte aligned), and with `pre_out` non-null
// also K3 into pre_out (T, nC / 4) bf16 (nC % 32 == 0, pre_out 16-byte aligned).
struct K2Params;
void launch_k1_fwd_rows(const void *x, const void *W, void *out, float *inv_rms, int64_t T,
                        int nC, int D, cudaStream_t s, const K2Params *coeffs = nullptr,
                        float *h_pre = nullptr, float *h_post = nullptr, float *H = nullptr,
                        void *pre_out = nullptr);
// Largest T for which fmhc_k1_fwd takes the small-T kernel: three waves of
// its one-block-per-SM grid on 148 SMs.  Measured at nC = 3072 (4096): 5.4
// (6.1) us up to T = 256, 10.2 (11.8) us at 512, 18.9 (22.0) us at 1024,
// against 18.6 (23.7) us for the tensor-core kernel at any T below ~9000.
#ifndef FMHC_K1_ROWS_MAX_T
#define FMHC_K1_ROWS_MAX_T 888
#endif
void launch_k1_bwd_dx_simt(const void *go, const void *x, const void *W, const void *proj,
                           const float *inv_rms, void *gx, int64_t T, int nC, int D, int vec,
                           cudaStream_t s);
int k1_dw_splits(int64_t T);
int64_t k1_dw_workspace_bytes(int64_t T, int64_t nC, int64_t D);
void launch_k1_dw_simt(const void *go, const void *x, const float *inv_rms, void *gW,
                       float *ws, int64_t T, int nC, int D, cudaStream_t s);

// k2_coeffs.cu -- coefficient math (n = 4, D = 32).
int64_t k2_bwd_workspace_bytes(int64_t T);
// The K2 parameters where they live: a_pre, a_post, a_res (one value each),
// bias (32) and the permutation rows perm (24 x 16), each f32 or bf16.
struct K2Params {
  const void *a_pre, *a_post, *a_res, *bias, *perm;
  int param_bf16, perm_bf16;
};
// params (35,) f32 = [a_pre, a_post, a_res, bias[32]], perm (24, 16) f32.
K2Params k2_packed_params(const float *params, const float *perm);
void launch_k2_fwd(const void *proj, const K2Params &P, float *h_pre, float *h_post, float *H,
                   int64_t T, cudaStream_t s);
// Where K2's backward writes the gradients of a_pre, a_post, a_res (one value
// each) and bias (32), in f32 (bf16 = 0) or bf16 (bf16 = 1).
struct K2ParamGrads {
  void *a_pre, *a_post, *a_res, *bias;
  int bf16;
};
// g_params (35,) f32 = [a_pre, a_post, a_res, bias[32]].
K2ParamGrads k2_packed_grads(float *g_params);
void launch_k2_bwd(const void *proj, const K2Params &P, const float *g_hpre, const float *g_hpost,
                   const float *g_H, void *g_proj, const K2ParamGrads &Gp, float *ws, int64_t T,
                   cudaStream_t s);

}  // namespace fmhc
