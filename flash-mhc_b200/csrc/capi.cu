// C ABI (include/flashmhc.h): argument validation, path selection, launch,
// error reporting.  No device memory is allocated here.
#include <cstdarg>
#include <cstdio>

#include "../../include/flashmhc.h"
#include "fmhc_launch.h"
#include "k1_tc.h"

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_err[0] = '\0';
  return FMHC_OK;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(FMHC_ERR_LAUNCH, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return ok();
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Largest bf16 chunk width v in {8,4,2,1} with C % v == 0 and every bf16
// pointer aligned to 2*v bytes.
int pick_vec(int64_t C, std::initializer_list<const void *> ptrs) {
  for (int v : {8, 4, 2, 1}) {
    if (C % v) continue;
    bool good = true;
    for (const void *p : ptrs) good = good && aligned(p, uintptr_t(2 * v));
    if (good) return v;
  }
  return 0;
}

int check_streams(const char *what, int64_t T, int64_t n, int64_t C) {
  if (T < 0) return fail(FMHC_ERR_INVALID_ARGUMENT, "%s: T must be >= 0 (got %lld)", what, (long long)T);
  if (n != 4) return fail(FMHC_ERR_INVALID_ARGUMENT, "%s: supports n=4 only (got n=%lld)", what, (long long)n);
  if (C < 1 || C > (int64_t(1) << 28))
    return fail(FMHC_ERR_INVALID_ARGUMENT, "%s: C must be in [1, 2^28] (got %lld)", what, (long long)C);
  return FMHC_OK;
}

#define FMHC_REQUIRE_PTR(what, p) \
  if ((p) == nullptr) return fail(FMHC_ERR_INVALID_ARGUMENT, "%s: %s is NULL", what, #p)
#define FMHC_REQUIRE_ALIGN16(what, p) \
  if (!aligned((p), 16)) return fail(FMHC_ERR_ALIGNMENT, "%s: %s must be 16-byte aligned", what, #p)
#define FMHC_REQUIRE_ALIGN2(what, p) \
  if (!aligned((p), 2)) return fail(FMHC_ERR_ALIGNMENT, "%s: %s must be 2-byte aligned", what, #p)

}  // namespace

namespace fmhc {
// Records `msg` as this thread's fmhc_last_error() text and returns `code`.
int set_last_error(int code, const char *msg) { return fail(code, "%s", msg); }
}  // namespace fmhc

extern "C" {

const char *fmhc_last_error(void) { return g_err; }

const char *fmhc_version(void) { return "flashmhc-sm100 0.1.0"; }

int fmhc_check_device_error(int *code) {
  if (code == nullptr) return fail(FMHC_ERR_INVALID_ARGUMENT, "fmhc_check_device_error: code is NULL");
  if (cudaDeviceSynchronize() != cudaSuccess)
    return fail(FMHC_ERR_CUDA, "fmhc_check_device_error: %s", cudaGetErrorString(cudaGetLastError()));
  unsigned v = 0;
  if (fmhc::read_device_error(&v)) return fail(FMHC_ERR_CUDA, "fmhc_check_device_error: symbol copy failed");
  *code = int(v);
  return ok();
}

int fmhc_k3_fwd(const void *x, const float *h_pre, void *out, int64_t T, int64_t n, int64_t C,
                void *stream) {
  const char *w = "fmhc_k3_fwd";
  if (int e = check_streams(w, T, n, C)) return e;
  if (T == 0) return ok();
  FMHC_REQUIRE_PTR(w, x); FMHC_REQUIRE_PTR(w, h_pre); FMHC_REQUIRE_PTR(w, out);
  FMHC_REQUIRE_ALIGN16(w, h_pre);
  FMHC_REQUIRE_ALIGN2(w, x); FMHC_REQUIRE_ALIGN2(w, out);
  const int vec = pick_vec(C, {x, out});
  fmhc::launch_k3_fwd(x, h_pre, out, T, int(C), vec, (cudaStream_t)stream);
  return check_launch(w);
}

int fmhc_k3_bwd(const void *grad_out, const void *x, const float *h_pre, void *grad_x,
                float *grad_h, int64_t T, int64_t n, int64_t C, void *stream) {
  const char *w = "fmhc_k3_bwd";
  if (int e = check_streams(w, T, n, C)) return e;
  if (T == 0) return ok();
  FMHC_REQUIRE_PTR(w, grad_out); FMHC_REQUIRE_PTR(w, x); FMHC_REQUIRE_PTR(w, h_pre);
  FMHC_REQUIRE_PTR(w, grad_h);
  FMHC_REQUIRE_ALIGN16(w, h_pre); FMHC_REQUIRE_ALIGN16(w, grad_h);
  FMHC_REQUIRE_ALIGN2(w, grad_out); FMHC_REQUIRE_ALIGN2(w, x);
  if (grad_x) FMHC_REQUIRE_ALIGN2(w, grad_x);
  const int vec = grad_x ? pick_vec(C, {grad_out, x, grad_x}) : pick_vec(C, {grad_out, x});
  fmhc::launch_k3_bwd(grad_out, x, h_pre, grad_x, grad_h, T, int(C), vec, (cudaStream_t)stream);
  return check_launch(w);
}

int fmhc_mhc_grad_x_combine(const void *gx1, const void *grad_li, const float *h_pre,
                            const void *gx4, void *grad_x, int64_t T, int64_t n, int64_t C,
                            void *stream) {
  const char *w = "fmhc_mhc_grad_x_combine";
  if (int e = check_streams(w, T, n, C)) return e;
  if (T == 0) return ok();
  FMHC_REQUIRE_PTR(w, gx1); FMHC_REQUIRE_PTR(w, grad_li); FMHC_REQUIRE_PTR(w, h_pre);
  FMHC_REQUIRE_PTR(w, grad_x);
  FMHC_REQUIRE_ALIGN16(w, h_pre);
  FMHC_REQUIRE_ALIGN2(w, gx1); FMHC_REQUIRE_ALIGN2(w, grad_li); FMHC_REQUIRE_ALIGN2(w, grad_x);
  if (gx4) FMHC_REQUIRE_ALIGN2(w, gx4);
  const int vec = gx4 ? pick_vec(C, {gx1, grad_li, gx4, grad_x}) : pick_vec(C, {gx1, grad_li, grad_x});
  fmhc::launch_grad_x_combine(gx1, grad_li, h_pre, gx4, grad_x, T, int(C), vec,
                              (cudaStream_t)stream);
  return check_launch(w);
}

int fmhc_mhc_grad_x_combine_post(const void *gx1, const void *grad_li, const float *h_pre,
                                 const void *grad_out, const float *H, void *grad_x, int64_t T,
                                 int64_t n, int64_t C, void *stream) {
  const char *w = "fmhc_mhc_grad_x_combine_post";
  if (int e = check_streams(w, T, n, C)) return e;
  if (T == 0) return ok();
  FMHC_REQUIRE_PTR(w, gx1); FMHC_REQUIRE_PTR(w, grad_li); FMHC_REQUIRE_PTR(w, h_pre);
  FMHC_REQUIRE_PTR(w, grad_out); FMHC_REQUIRE_PTR(w, H); FMHC_REQUIRE_PTR(w, grad_x);
  FMHC_REQUIRE_ALIGN16(w, h_pre); FMHC_REQUIRE_ALIGN16(w, H);
  FMHC_REQUIRE_ALIGN2(w, gx1); FMHC_REQUIRE_ALIGN2(w, grad_li); FMHC_REQUIRE_ALIGN2(w, grad_out);
  FMHC_REQUIRE_ALIGN2(w, grad_x);
  const int vec = pick_vec(C, {gx1, grad_li, grad_out, grad_x});
  fmhc::launch_grad_x_combine_post(gx1, grad_li, h_pre, grad_out, H, grad_x, T, int(C), vec,
                                   (cudaStream_t)stream);
  return check_launch(w);
}

int fmhc_k4_fwd(const void *x, const void *lo, const float *H, const float *h_post, void *out,
                int64_t T, int64_t n, int64_t C, void *stream) {
  const char *w = "fmhc_k4_fwd";
  if (int e = check_streams(w, T, n, C)) return e;
  if (T == 0) return ok();
  FMHC_REQUIRE_PTR(w, x); FMHC_REQUIRE_PTR(w, lo); FMHC_REQUIRE_PTR(w, H);
  FMHC_REQUIRE_PTR(w, h_post); FMHC_REQUIRE_PTR(w, out);
  FMHC_REQUIRE_ALIGN16(w, H); FMHC_REQUIRE_ALIGN16(w, h_post);
  FMHC_REQUIRE_ALIGN2(w, x); FMHC_REQUIRE_ALIGN2(w, lo); FMHC_REQUIRE_ALIGN2(w, out);
  const int vec = pick_vec(C, {x, lo, out});
  fmhc::launch_k4_fwd(x, lo, H, h_post, out, T, int(C), vec, (cudaStream_t)stream);
  return check_launch(w);
}

int fmhc_k4_bwd(const void *grad_out, const void *x, const void *lo, const float *H,
                const float *h_post, void *grad_x, void *grad_lo, float *grad_H,
                float *grad_hp, int64_t T, int64_t n, int64_t C, void *stream) {
  const char *w = "fmhc_k4_bwd";
  if (int e = check_streams(w, T, n, C)) return e;
  if (T == 0) return ok();
  FMHC_REQUIRE_PTR(w, grad_out); FMHC_REQUIRE_PTR(w, x); FMHC_REQUIRE_PTR(w, lo);
  FMHC_REQUIRE_PTR(w, H); FMHC_REQUIRE_PTR(w, h_post);
  FMHC_REQUIRE_PTR(w, grad_lo); FMHC_REQUIRE_PTR(w, grad_H); FMHC_REQUIRE_PTR(w, grad_hp);
  FMHC_REQUIRE_ALIGN16(w, H); FMHC_REQUIRE_ALIGN16(w, h_post);
  FMHC_REQUIRE_ALIGN16(w, grad_H); FMHC_REQUIRE_ALIGN16(w, grad_hp);
  FMHC_REQUIRE_ALIGN2(w, grad_out); FMHC_REQUIRE_ALIGN2(w, x); FMHC_REQUIRE_ALIGN2(w, lo);
  FMHC_REQUIRE_ALIGN2(w, grad_lo);
  if (grad_x) FMHC_REQUIRE_ALIGN2(w, grad_x);  // NULL: parameter gradients only
  const int vec = grad_x ? pick_vec(C, {grad_out, x, lo, grad_x, grad_lo})
                         : pick_vec(C, {grad_out, x, lo, grad_lo});
  fmhc::launch_k4_bwd(grad_out, x, lo, H, h_post, grad_x, grad_lo, grad_H, grad_hp, T, int(C),
                      vec, (cudaStream_t)stream);
  return check_launch(w);
}

static int check_k1(const char *w, int64_t T, int64_t nC, int64_t D) {
  if (T < 0) return fail(FMHC_ERR_INVALID_ARGUMENT, "%s: T must be >= 0 (got %lld)", w, (long long)T);
  if (nC < 1 || nC > (int64_t(1) << 28))
    return fail(FMHC_ERR_INVALID_ARGUMENT, "%s: nC must be in [1, 2^28] (got %lld)", w, (long long)nC);
  if (D < 1 || D > 32)
    return fail(FMHC_ERR_UNSUPPORTED, "%s: D (projection width) must be in [1, 32] (got %lld)", w,
                (long long)D);
  return FMHC_OK;
}

int fmhc_k1_fwd(const void *x, const void *W, void *out, float *inv_rms, int64_t T, int64_t nC,
                int64_t D, void *stream) {
  const char *w = "fmhc_k1_fwd";
  if (int e = check_k1(w, T, nC, D)) return e;
  if (T == 0) return ok();
  FMHC_REQUIRE_PTR(w, x); FMHC_REQUIRE_PTR(w, W); FMHC_REQUIRE_PTR(w, out);
  FMHC_REQUIRE_PTR(w, inv_rms);
  FMHC_REQUIRE_ALIGN2(w, x); FMHC_REQUIRE_ALIGN2(w, W); FMHC_REQUIRE_ALIGN2(w, out);
  if (!aligned(inv_rms, 4)) return fail(FMHC_ERR_ALIGNMENT, "%s: inv_rms must be 4-byte aligned", w);
  cudaStream_t s = (cudaStream_t)stream;
  if (T <= FMHC_K1_ROWS_MAX_T && D == 32 && nC % 8 == 0 && aligned(x, 16) && aligned(W, 16)) {
    // Few tokens: one pass over W per block of 2 tokens (split over a cluster
    // while the tokens are too few to fill the GPU) beats the tensor-core
    // kernel's serial k-loop per tile.
    const int rc = fmhc::launch_k1_fwd_rows_cluster(x, W, out, inv_rms, T, int(nC), s);
    if (rc > 0) return fail(rc, "%s: %s", w, fmhc::k1_tc_error());
    if (rc < 0) fmhc::launch_k1_fwd_rows(x, W, out, inv_rms, T, int(nC), int(D), s);
  } else if (fmhc::k1_tc_fwd_supported(x, W, out, inv_rms, T, nC, D)) {
    if (int e = fmhc::launch_k1_tc_fwd(x, W, out, inv_rms, T, int(nC), s))
      return fail(e, "%s: %s", w, fmhc::k1_tc_error());
  } else {
    const int vec = pick_vec(nC, {x, W});
    fmhc::launch_k1_fwd_simt(x, W, out, inv_rms, T, int(nC), int(D), vec == 8 ? 8 : 1, s);
  }
  return check_launch(w);
}

int fmhc_debug_k1_fwd_lost_copy(const void *x, const void *W, void *out, float *inv_rms,
                                int64_t T, int64_t nC, void *stream) {
  const char *w = "fmhc_debug_k1_fwd_lost_copy";
  if (int e = check_k1(w, T, nC, 32)) return e;
  if (T == 0) return fail(FMHC_ERR_INVALID_ARGUMENT, "%s: needs T >= 1", w);
  FMHC_REQUIRE_PTR(w, x); FMHC_REQUIRE_PTR(w, W); FMHC_REQUIRE_PTR(w, out);
  FMHC_REQUIRE_PTR(w, inv_rms);
  if (!fmhc::k1_tc_fwd_supported(x, W, out, inv_rms, T, nC, 32))
    return fail(FMHC_ERR_INVALID_ARGUMENT,
                "%s: needs the tensor-core K1 forward (nC %% 64 == 0, 16-byte aligned x, W, out, "
                "a B200)", w);
  if (int e = fmhc::launch_k1_tc_fwd_lost_copy(x, W, out, inv_rms, T, int(nC), (cudaStream_t)stream))
    return fail(e, "%s: %s", w, fmhc::k1_tc_error());
  return check_launch(w);
}

int fmhc_k1_bwd_dx(const void *grad_out, const void *x, const void *W, const void *proj,
                   const float *inv_rms, void *grad_x, int64_t T, int64_t nC, int64_t D,
                   void *stream) {
  const char *w = "fmhc_k1_bwd_dx";
  if (int e = check_k1(w, T, nC, D)) return e;
  if (T == 0) return ok();
  FMHC_REQUIRE_PTR(w, grad_out); FMHC_REQUIRE_PTR(w, x); FMHC_REQUIRE_PTR(w, W);
  FMHC_REQUIRE_PTR(w, proj); FMHC_REQUIRE_PTR(w, inv_rms); FMHC_REQUIRE_PTR(w, grad_x);
  FMHC_REQUIRE_ALIGN2(w, grad_out); FMHC_REQUIRE_ALIGN2(w, x); FMHC_REQUIRE_ALIGN2(w, W);
  FMHC_REQUIRE_ALIGN2(w, proj); FMHC_REQUIRE_ALIGN2(w, grad_x);
  if (!aligned(inv_rms, 4)) return fail(FMHC_ERR_ALIGNMENT, "%s: inv_rms must be 4-byte aligned", w);
  cudaStream_t s = (cudaStream_t)stream;
  if (fmhc::k1_tc_bwd_supported(grad_out, x, W, proj, grad_x, T, nC, D)) {
    if (int e = fmhc::launch_k1_tc_bwd(grad_out, x, W, proj, inv_rms, grad_x, nullptr, nullptr, 0,
                                       T, int(nC), s))
      return fail(e, "%s: %s", w, fmhc::k1_tc_error());
  } else {
    const int vec = pick_vec(nC, {x, W, grad_x});
    fmhc::launch_k1_bwd_dx_simt(grad_out, x, W, proj, inv_rms, grad_x, T, int(nC), int(D),
                                vec == 8 ? 8 : 1, s);
  }
  return check_launch(w);
}

int64_t fmhc_k1_bwd_workspace_size(int64_t T, int64_t nC, int64_t D) {
  if (T <= 0 || nC <= 0 || D <= 0 || D > 32) return 0;
  const int64_t a = fmhc::k1_tc_bwd_workspace_bytes(T, nC);
  const int64_t b = fmhc::k1_dw_workspace_bytes(T, nC, D);
  return a > b ? a : b;
}

int fmhc_k1_bwd(const void *grad_out, const void *x, const void *W, const void *proj,
                const float *inv_rms, void *grad_x, void *grad_W, void *workspace,
                int64_t workspace_bytes, int64_t T, int64_t nC, int64_t D, void *stream) {
  const char *w = "fmhc_k1_bwd";
  if (int e = check_k1(w, T, nC, D)) return e;
  FMHC_REQUIRE_PTR(w, grad_W);
  cudaStream_t s = (cudaStream_t)stream;
  if (T == 0) {
    // Empty batch: the weight gradient is exactly zero.
    if (cudaMemsetAsync(grad_W, 0, size_t(D * nC) * 2, s) != cudaSuccess)
      return fail(FMHC_ERR_CUDA, "%s: cudaMemsetAsync failed", w);
    return ok();
  }
  FMHC_REQUIRE_PTR(w, grad_out); FMHC_REQUIRE_PTR(w, x); FMHC_REQUIRE_PTR(w, W);
  FMHC_REQUIRE_PTR(w, proj); FMHC_REQUIRE_PTR(w, inv_rms); FMHC_REQUIRE_PTR(w, grad_x);
  FMHC_REQUIRE_PTR(w, workspace);
  FMHC_REQUIRE_ALIGN2(w, grad_out); FMHC_REQUIRE_ALIGN2(w, x); FMHC_REQUIRE_ALIGN2(w, W);
  FMHC_REQUIRE_ALIGN2(w, proj); FMHC_REQUIRE_ALIGN2(w, grad_x); FMHC_REQUIRE_ALIGN2(w, grad_W);
  if (!aligned(inv_rms, 4)) return fail(FMHC_ERR_ALIGNMENT, "%s: inv_rms must be 4-byte aligned", w);
  if (!aligned(workspace, 256)) return fail(FMHC_ERR_ALIGNMENT, "%s: workspace must be 256-byte aligned", w);
  const int64_t need = fmhc_k1_bwd_workspace_size(T, nC, D);
  if (workspace_bytes < need)
    return fail(FMHC_ERR_WORKSPACE, "%s: workspace of %lld bytes, %lld needed", w,
                (long long)workspace_bytes, (long long)need);
  if (fmhc::k1_tc_bwd_supported(grad_out, x, W, proj, grad_x, T, nC, D)) {
    if (int e = fmhc::launch_k1_tc_bwd(grad_out, x, W, proj, inv_rms, grad_x, grad_W, workspace,
                                       workspace_bytes, T, int(nC), s))
      return fail(e, "%s: %s", w, fmhc::k1_tc_error());
  } else {
    const int vec = pick_vec(nC, {x, W, grad_x});
    fmhc::launch_k1_bwd_dx_simt(grad_out, x, W, proj, inv_rms, grad_x, T, int(nC), int(D),
                                vec == 8 ? 8 : 1, s);
    fmhc::launch_k1_dw_simt(grad_out, x, inv_rms, grad_W, (float *)workspace, T, int(nC),
                            int(D), s);
  }
  return check_launch(w);
}

int fmhc_k2_fwd(const void *proj, const float *params, const float *perm, float *h_pre,
                float *h_post, float *H_merged, int64_t T, void *stream) {
  const char *w = "fmhc_k2_fwd";
  if (T < 0) return fail(FMHC_ERR_INVALID_ARGUMENT, "%s: T must be >= 0 (got %lld)", w, (long long)T);
  if (T == 0) return ok();
  FMHC_REQUIRE_PTR(w, proj); FMHC_REQUIRE_PTR(w, params); FMHC_REQUIRE_PTR(w, perm);
  FMHC_REQUIRE_PTR(w, h_pre); FMHC_REQUIRE_PTR(w, h_post); FMHC_REQUIRE_PTR(w, H_merged);
  FMHC_REQUIRE_ALIGN16(w, proj); FMHC_REQUIRE_ALIGN16(w, h_pre); FMHC_REQUIRE_ALIGN16(w, h_post);
  FMHC_REQUIRE_ALIGN16(w, H_merged);
  if (!aligned(params, 4) || !aligned(perm, 4)) return fail(FMHC_ERR_ALIGNMENT, "%s: params/perm must be 4-byte aligned", w);
  fmhc::launch_k2_fwd(proj, fmhc::k2_packed_params(params, perm), h_pre, h_post, H_merged, T,
                      (cudaStream_t)stream);
  return check_launch(w);
}

int fmhc_k2_fwd_typed(const void *proj, const void *alpha_pre, const void *alpha_post,
                      const void *alpha_res, const void *bias, int param_dtype, const void *perm,
                      int perm_dtype, float *h_pre, float *h_post, float *H_merged, int64_t T,
                      void *stream) {
  const char *w = "fmhc_k2_fwd_typed";
  if (T < 0) return fail(FMHC_ERR_INVALID_ARGUMENT, "%s: T must be >= 0 (got %lld)", w, (long long)T);
  const auto dt_ok = [](int d) { return d == FMHC_DTYPE_F32 || d == FMHC_DTYPE_BF16; };
  if (!dt_ok(param_dtype) || !dt_ok(perm_dtype))
    return fail(FMHC_ERR_UNSUPPORTED, "%s: parameter dtypes must be FMHC_DTYPE_F32 or FMHC_DTYPE_BF16", w);
  if (T == 0) return ok();
  FMHC_REQUIRE_PTR(w, proj); FMHC_REQUIRE_PTR(w, alpha_pre); FMHC_REQUIRE_PTR(w, alpha_post);
  FMHC_REQUIRE_PTR(w, alpha_res); FMHC_REQUIRE_PTR(w, bias); FMHC_REQUIRE_PTR(w, perm);
  FMHC_REQUIRE_PTR(w, h_pre); FMHC_REQUIRE_PTR(w, h_post); FMHC_REQUIRE_PTR(w, H_merged);
  FMHC_REQUIRE_ALIGN16(w, proj); FMHC_REQUIRE_ALIGN16(w, h_pre); FMHC_REQUIRE_ALIGN16(w, h_post);
  FMHC_REQUIRE_ALIGN16(w, H_merged);
  const uintptr_t pa = param_dtype == FMHC_DTYPE_BF16 ? 2 : 4;
  const uintptr_t qa = perm_dtype == FMHC_DTYPE_BF16 ? 2 : 4;
  if (!aligned(alpha_pre, pa) || !aligned(alpha_post, pa) || !aligned(alpha_res, pa) ||
      !aligned(bias, pa) || !aligned(perm, qa))
    return fail(FMHC_ERR_ALIGNMENT, "%s: parameters must be aligned to their element size", w);
  const fmhc::K2Params P{alpha_pre, alpha_post, alpha_res, bias, perm,
                         param_dtype == FMHC_DTYPE_BF16 ? 1 : 0,
                         perm_dtype == FMHC_DTYPE_BF16 ? 1 : 0};
  fmhc::launch_k2_fwd(proj, P, h_pre, h_post, H_merged, T, (cudaStream_t)stream);
  return check_launch(w);
}

int fmhc_mhc_pre_fwd(const void *x, const void *W, const void *alpha_pre, const void *alpha_post,
                     const void *alpha_res, const void *bias, int param_dtype, const void *perm,
                     int perm_dtype, void *proj, float *inv_rms, float *h_pre, float *h_post,
                     float *H_merged, void *layer_input, int64_t T, int64_t n, int64_t C,
                     void *stream) {
  const char *w = "fmhc_mhc_pre_fwd";
  if (int e = check_streams(w, T, n, C)) return e;
  const int64_t nC = n * C, D = 32;
  if (int e = check_k1(w, T, nC, D)) return e;
  const auto dt_ok = [](int d) { return d == FMHC_DTYPE_F32 || d == FMHC_DTYPE_BF16; };
  if (!dt_ok(param_dtype) || !dt_ok(perm_dtype))
    return fail(FMHC_ERR_UNSUPPORTED, "%s: parameter dtypes must be FMHC_DTYPE_F32 or FMHC_DTYPE_BF16", w);
  if (T == 0) return ok();
  FMHC_REQUIRE_PTR(w, x); FMHC_REQUIRE_PTR(w, W); FMHC_REQUIRE_PTR(w, alpha_pre);
  FMHC_REQUIRE_PTR(w, alpha_post); FMHC_REQUIRE_PTR(w, alpha_res); FMHC_REQUIRE_PTR(w, bias);
  FMHC_REQUIRE_PTR(w, perm); FMHC_REQUIRE_PTR(w, proj); FMHC_REQUIRE_PTR(w, inv_rms);
  FMHC_REQUIRE_PTR(w, h_pre); FMHC_REQUIRE_PTR(w, h_post); FMHC_REQUIRE_PTR(w, H_merged);
  FMHC_REQUIRE_ALIGN2(w, x); FMHC_REQUIRE_ALIGN2(w, W); FMHC_REQUIRE_ALIGN16(w, proj);
  FMHC_REQUIRE_ALIGN16(w, h_pre); FMHC_REQUIRE_ALIGN16(w, h_post); FMHC_REQUIRE_ALIGN16(w, H_merged);
  if (!aligned(inv_rms, 4)) return fail(FMHC_ERR_ALIGNMENT, "%s: inv_rms must be 4-byte aligned", w);
  if (layer_input) FMHC_REQUIRE_ALIGN2(w, layer_input);
  const uintptr_t pa = param_dtype == FMHC_DTYPE_BF16 ? 2 : 4;
  const uintptr_t qa = perm_dtype == FMHC_DTYPE_BF16 ? 2 : 4;
  if (!aligned(alpha_pre, pa) || !aligned(alpha_post, pa) || !aligned(alpha_res, pa) ||
      !aligned(bias, pa) || !aligned(perm, qa))
    return fail(FMHC_ERR_ALIGNMENT, "%s: parameters must be aligned to their element size", w);
  const fmhc::K2Params P{alpha_pre, alpha_post, alpha_res, bias, perm,
                         param_dtype == FMHC_DTYPE_BF16 ? 1 : 0,
                         perm_dtype == FMHC_DTYPE_BF16 ? 1 : 0};
  cudaStream_t s = (cudaStream_t)stream;
  bool pre_done = false;
  // K1 takes the kernel fmhc_k1_fwd would take for this call, with K2 (and
  // at few tokens K3) in its epilogue, so every output equals the separate
  // fmhc_k1_fwd -> fmhc_k2_fwd_typed -> fmhc_k3_fwd results bit for bit.
  if (T <= FMHC_K1_ROWS_MAX_T && nC % 8 == 0 && aligned(x, 16) && aligned(W, 16)) {
    const bool pre = layer_input && C % 8 == 0 && aligned(layer_input, 16);
    void *pre_out = pre ? layer_input : nullptr;
    const int rc = fmhc::launch_k1_fwd_rows_cluster(x, W, proj, inv_rms, T, int(nC), s, &P, h_pre,
                                                    h_post, H_merged, pre_out);
    if (rc > 0) return fail(rc, "%s: %s", w, fmhc::k1_tc_error());
    if (rc < 0)
      fmhc::launch_k1_fwd_rows(x, W, proj, inv_rms, T, int(nC), int(D), s, &P, h_pre, h_post,
                               H_merged, pre_out);
    pre_done = pre;
  } else if (fmhc::k1_tc_fwd_supported(x, W, proj, inv_rms, T, nC, D)) {
    if (int e = fmhc::launch_k1_tc_fwd(x, W, proj, inv_rms, T, int(nC), s, &P, h_pre, h_post,
                                       H_merged))
      return fail(e, "%s: %s", w, fmhc::k1_tc_error());
  } else {
    const int vec = pick_vec(nC, {x, W});
    fmhc::launch_k1_fwd_simt(x, W, proj, inv_rms, T, int(nC), int(D), vec == 8 ? 8 : 1, s);
    fmhc::launch_k2_fwd(proj, P, h_pre, h_post, H_merged, T, s);
  }
  if (layer_input && !pre_done) {
    const int vec = pick_vec(C, {x, layer_input});
    fmhc::launch_k3_fwd(x, h_pre, layer_input, T, int(C), vec, s);
  }
  return check_launch(w);
}

int64_t fmhc_k2_bwd_workspace_size(int64_t T) {
  if (T <= 0) return 0;
  return fmhc::k2_bwd_workspace_bytes(T);
}

int fmhc_k2_bwd(const void *proj, const float *params, const float *perm, const float *grad_h_pre,
                const float *grad_h_post, const float *grad_H_merged, void *grad_proj,
                float *grad_params, void *workspace, int64_t workspace_bytes, int64_t T,
                void *stream) {
  const char *w = "fmhc_k2_bwd";
  if (T < 0) return fail(FMHC_ERR_INVALID_ARGUMENT, "%s: T must be >= 0 (got %lld)", w, (long long)T);
  FMHC_REQUIRE_PTR(w, grad_params);
  cudaStream_t s = (cudaStream_t)stream;
  if (T == 0) {
    if (cudaMemsetAsync(grad_params, 0, 35 * sizeof(float), s) != cudaSuccess)
      return fail(FMHC_ERR_CUDA, "%s: cudaMemsetAsync failed", w);
    return ok();
  }
  FMHC_REQUIRE_PTR(w, proj); FMHC_REQUIRE_PTR(w, params); FMHC_REQUIRE_PTR(w, perm);
  FMHC_REQUIRE_PTR(w, grad_h_pre); FMHC_REQUIRE_PTR(w, grad_h_post);
  FMHC_REQUIRE_PTR(w, grad_H_merged); FMHC_REQUIRE_PTR(w, grad_proj); FMHC_REQUIRE_PTR(w, workspace);
  FMHC_REQUIRE_ALIGN16(w, proj); FMHC_REQUIRE_ALIGN16(w, grad_h_pre);
  FMHC_REQUIRE_ALIGN16(w, grad_h_post); FMHC_REQUIRE_ALIGN16(w, grad_H_merged);
  FMHC_REQUIRE_ALIGN16(w, grad_proj);
  if (!aligned(workspace, 256)) return fail(FMHC_ERR_ALIGNMENT, "%s: workspace must be 256-byte aligned", w);
  if (!aligned(params, 4) || !aligned(perm, 4) || !aligned(grad_params, 4))
    return fail(FMHC_ERR_ALIGNMENT, "%s: params/perm/grad_params must be 4-byte aligned", w);
  const int64_t need = fmhc::k2_bwd_workspace_bytes(T);
  if (workspace_bytes < need)
    return fail(FMHC_ERR_WORKSPACE, "%s: workspace of %lld bytes, %lld needed", w,
                (long long)workspace_bytes, (long long)need);
  fmhc::launch_k2_bwd(proj, fmhc::k2_packed_params(params, perm), grad_h_pre, grad_h_post,
                      grad_H_merged, grad_proj, fmhc::k2_packed_grads(grad_params),
                      (float *)workspace, T, s);
  return check_launch(w);
}

int fmhc_k2_bwd_typed(const void *proj, const void *alpha_pre, const void *alpha_post,
                      const void *alpha_res, const void *bias, int param_dtype, const void *perm,
                      int perm_dtype, const float *grad_h_pre, const float *grad_h_post,
                      const float *grad_H_merged, void *grad_proj, void *grad_alpha_pre,
                      void *grad_alpha_post, void *grad_alpha_res, void *grad_bias,
                      void *workspace, int64_t workspace_bytes, int64_t T, void *stream) {
  const char *w = "fmhc_k2_bwd_typed";
  if (T < 0) return fail(FMHC_ERR_INVALID_ARGUMENT, "%s: T must be >= 0 (got %lld)", w, (long long)T);
  const auto dt_ok = [](int d) { return d == FMHC_DTYPE_F32 || d == FMHC_DTYPE_BF16; };
  if (!dt_ok(param_dtype) || !dt_ok(perm_dtype))
    return fail(FMHC_ERR_UNSUPPORTED, "%s: parameter dtypes must be FMHC_DTYPE_F32 or FMHC_DTYPE_BF16", w);
  FMHC_REQUIRE_PTR(w, grad_alpha_pre); FMHC_REQUIRE_PTR(w, grad_alpha_post);
  FMHC_REQUIRE_PTR(w, grad_alpha_res); FMHC_REQUIRE_PTR(w, grad_bias);
  const uintptr_t pa = param_dtype == FMHC_DTYPE_BF16 ? 2 : 4;
  const uintptr_t qa = perm_dtype == FMHC_DTYPE_BF16 ? 2 : 4;
  if (!aligned(grad_alpha_pre, pa) || !aligned(grad_alpha_post, pa) ||
      !aligned(grad_alpha_res, pa) || !aligned(grad_bias, pa))
    return fail(FMHC_ERR_ALIGNMENT, "%s: parameter gradients must be aligned to their element size", w);
  const fmhc::K2ParamGrads G{grad_alpha_pre, grad_alpha_post, grad_alpha_res, grad_bias,
                             param_dtype == FMHC_DTYPE_BF16 ? 1 : 0};
  cudaStream_t s = (cudaStream_t)stream;
  if (T == 0) {
    fmhc::launch_k2_bwd(nullptr, fmhc::K2Params{}, nullptr, nullptr, nullptr, nullptr, G, nullptr,
                        0, s);
    return check_launch(w);
  }
  FMHC_REQUIRE_PTR(w, proj); FMHC_REQUIRE_PTR(w, alpha_pre); FMHC_REQUIRE_PTR(w, alpha_post);
  FMHC_REQUIRE_PTR(w, alpha_res); FMHC_REQUIRE_PTR(w, bias); FMHC_REQUIRE_PTR(w, perm);
  FMHC_REQUIRE_PTR(w, grad_h_pre); FMHC_REQUIRE_PTR(w, grad_h_post);
  FMHC_REQUIRE_PTR(w, grad_H_merged); FMHC_REQUIRE_PTR(w, grad_proj); FMHC_REQUIRE_PTR(w, workspace);
  FMHC_REQUIRE_ALIGN16(w, proj); FMHC_REQUIRE_ALIGN16(w, grad_h_pre);
  FMHC_REQUIRE_ALIGN16(w, grad_h_post); FMHC_REQUIRE_ALIGN16(w, grad_H_merged);
  FMHC_REQUIRE_ALIGN16(w, grad_proj);
  if (!aligned(alpha_pre, pa) || !aligned(alpha_post, pa) || !aligned(alpha_res, pa) ||
      !aligned(bias, pa) || !aligned(perm, qa))
    return fail(FMHC_ERR_ALIGNMENT, "%s: parameters must be aligned to their element size", w);
  if (!aligned(workspace, 256)) return fail(FMHC_ERR_ALIGNMENT, "%s: workspace must be 256-byte aligned", w);
  const int64_t need = fmhc::k2_bwd_workspace_bytes(T);
  if (workspace_bytes < need)
    return fail(FMHC_ERR_WORKSPACE, "%s: workspace of %lld bytes, %lld needed", w,
                (long long)workspace_bytes, (long long)need);
  const fmhc::K2Params P{alpha_pre, alpha_post, alpha_res, bias, perm,
                         param_dtype == FMHC_DTYPE_BF16 ? 1 : 0,
                         perm_dtype == FMHC_DTYPE_BF16 ? 1 : 0};
  fmhc::launch_k2_bwd(proj, P, grad_h_pre, grad_h_post, grad_H_merged, grad_proj, G,
                      (float *)workspace, T, s);
  return check_launch(w);
}

}  // extern "C"
