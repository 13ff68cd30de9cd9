// K1 on the 5th-generation tensor cores (TMA + tcgen05.mma + TMEM).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "fmhc_launch.h"

namespace fmhc {

// True when the tensor-core forward kernel handles this call (shape, alignment,
// device).  Otherwise the CUDA-core kernel in k1_simt.cu runs.
bool k1_tc_fwd_supported(const void *x, const void *W, const void *out, const float *inv_rms,
                         int64_t T, int64_t nC, int64_t D);
// Returns 0 or an fmhc_status code; k1_tc_error() then describes the failure.
// With `coeffs` non-null the epilogue also runs K2 (parameters *coeffs) and
// writes h_pre, h_post (T, 4) and H_merged (T, 4, 4), each 16-byte aligned.
int launch_k1_tc_fwd(const void *x, const void *W, void *out, float *inv_rms, int64_t T, int nC,
                     cudaStream_t s, const K2Params *coeffs = nullptr, float *h_pre = nullptr,
                     float *h_post = nullptr, float *H = nullptr);
const char *k1_tc_error();

// K1 forward for T <= 2 x (SMs / 2) tokens on the CUDA cores, each 2-token
// pair split over a cluster of 2-8 CTAs (same preconditions and options as
// launch_k1_fwd_rows).  Returns 0 when launched, -1 when T is too large for
// it (the caller then runs launch_k1_fwd_rows), or an fmhc_status code.
int launch_k1_fwd_rows_cluster(const void *x, const void *W, void *out, float *inv_rms, int64_t T,
                               int nC, cudaStream_t s, const K2Params *coeffs = nullptr,
                               float *h_pre = nullptr, float *h_post = nullptr, float *H = nullptr,
                               void *pre_out = nullptr);

// Backward (grad_x, and grad_W when gW != nullptr) on the tensor cores.
bool k1_tc_bwd_supported(const void *go, const void *x, const void *W, const void *proj,
                         const void *gx, int64_t T, int64_t nC, int64_t D);
// Caller workspace for the grad_W variant on the current device (0 if unsupported shape).
int64_t k1_tc_bwd_workspace_bytes(int64_t T, int64_t nC);
int launch_k1_tc_bwd(const void *go, const void *x, const void *W, const void *proj,
                     const float *inv_rms, void *gx, void *gW, void *ws, int64_t ws_bytes,
                     int64_t T, int nC, cudaStream_t s);

// Test hook: the persistent tensor-core forward in which CTA 0 loses its first
// copy, so its waits on that stage expire (see k1_fwd_tc_kernel's LOSE_COPY).
// Same preconditions as launch_k1_tc_fwd; the output is not meaningful.
int launch_k1_tc_fwd_lost_copy(const void *x, const void *W, void *out, float *inv_rms,
                               int64_t T, int nC, cudaStream_t s);

// Reads and clears the per-device error word set by expired bounded waits.
int read_device_error(unsigned *code);

}  // namespace fmhc
