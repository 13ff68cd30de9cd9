// fmhc_k1_bwd_noalloc: the K1 backward (grad_x and grad_W) for callers that
// cannot allocate device memory.
//
// Who needs it: a host that only receives device pointers from someone else
// and has no device allocator of its own (a C, Go or Java process calling this
// library through its C ABI, or a plugin inside another framework whose memory
// pool it may not touch); serving runtimes that reserve all of HBM up front
// and refuse further cudaMalloc; and latency-critical paths where cudaMalloc,
// which can synchronise the device, is not allowed.  fmhc_k1_bwd needs a
// caller-provided workspace; this variant uses a fixed scratch array that
// lives in the library instead.
//
// The scratch is a file-scope __device__ array of kScratchBytes (32 MiB).  Every
// GPU on which the library's device code is loaded holds that memory until the
// process exits.  In host code the array's name is only a host-side stand-in,
// so the device address is looked up with cudaGetSymbolAddress, once per
// device, with that device current, on the first call made on that device;
// make that first call before any stream capture begins.
//
// Calls share the one array: two calls whose kernels overlap on the same GPU
// (different streams, or different host threads) race on it and must not be
// issued.  Nothing in the array needs to start at zero: each call writes every
// scratch value it later reads, so the contents left by the previous call do
// not matter.
#include <cstdio>
#include <mutex>

#include "../../include/flashmhc.h"
#include "fmhc_launch.h"

namespace {

constexpr int64_t kScratchBytes = int64_t(32) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_k1_bwd_scratch[kScratchBytes];

std::mutex g_mu;
void *g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set-up on first use).
int scratch_for_current_device(void **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    return fmhc::set_last_error(FMHC_ERR_CUDA, "fmhc_k1_bwd_noalloc: no usable current device");
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_k1_bwd_scratch);
    if (e != cudaSuccess || p == nullptr) {
      char msg[256];
      snprintf(msg, sizeof(msg),
               "fmhc_k1_bwd_noalloc: cudaGetSymbolAddress of the scratch array failed on device "
               "%d: %s",
               dev, cudaGetErrorString(e));
      return fmhc::set_last_error(FMHC_ERR_CUDA, msg);
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return FMHC_OK;
}

}  // namespace

extern "C" int fmhc_k1_bwd_noalloc(const void *grad_out, const void *x, const void *W,
                                   const void *proj, const float *inv_rms, void *grad_x,
                                   void *grad_W, int64_t T, int64_t nC, int64_t D,
                                   void *stream) {
  const int64_t need = fmhc_k1_bwd_workspace_size(T, nC, D);
  if (need > kScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "fmhc_k1_bwd_noalloc: T=%lld, nC=%lld needs %lld bytes of scratch, above the "
             "built-in maximum of %lld bytes; call fmhc_k1_bwd with a workspace instead",
             (long long)T, (long long)nC, (long long)need, (long long)kScratchBytes);
    return fmhc::set_last_error(FMHC_ERR_WORKSPACE, msg);
  }
  void *scratch = nullptr;
  if (int e = scratch_for_current_device(&scratch)) return e;
  return fmhc_k1_bwd(grad_out, x, W, proj, inv_rms, grad_x, grad_W, scratch, kScratchBytes, T,
                     nC, D, stream);
}
