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
// so the device address is looked up with cudaGetSymbolAddress, with the
// device current, on the first call made in each CUDA context: once per
// device, and again after a device reset (cudaDeviceReset ends the primary
// context; the next one reloads the module, and the array may move).  The
// cache is keyed on the context's unique ID (cuCtxGetId), so a stale address
// is never reused.  Make the first call on each device before any stream
// capture begins.
//
// Calls share the one array: two calls whose kernels overlap on the same GPU
// (different streams, or different host threads) race on it and must not be
// issued.  Nothing in the array needs to start at zero: a call that succeeds
// writes every scratch value it later reads, so the contents left by the
// previous call do not matter.  When a bounded wait of the kernel expires
// (fmhc_check_device_error reports it), grad_W is written as NaN rather than
// summed from partials that were not all written.
#include <cstdio>
#include <mutex>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "../../include/flashmhc.h"
#include "fmhc_launch.h"

namespace {

constexpr int64_t kScratchBytes = int64_t(32) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_k1_bwd_scratch[kScratchBytes];

std::mutex g_mu;
struct Cached {
  unsigned long long ctx_id;
  void *ptr;
};
Cached g_cache[kMaxDevices] = {};

// Driver entry points, fetched through the runtime so the library needs no
// link-time dependency on libcuda.
PFN_cuCtxGetCurrent_v4000 g_ctx_current = nullptr;
PFN_cuCtxGetId_v12000 g_ctx_id = nullptr;

int driver_fns() {
  if (g_ctx_current && g_ctx_id) return FMHC_OK;
  void *a = nullptr, *b = nullptr;
  cudaDriverEntryPointQueryResult qa{}, qb{};
  if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &a, 4000, cudaEnableDefault, &qa) !=
          cudaSuccess || qa != cudaDriverEntryPointSuccess || a == nullptr ||
      cudaGetDriverEntryPointByVersion("cuCtxGetId", &b, 12000, cudaEnableDefault, &qb) !=
          cudaSuccess || qb != cudaDriverEntryPointSuccess || b == nullptr) {
    return fmhc::set_last_error(FMHC_ERR_CUDA,
                                "fmhc_k1_bwd_noalloc: driver entry points cuCtxGetCurrent / "
                                "cuCtxGetId unavailable");
  }
  g_ctx_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(a);
  g_ctx_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(b);
  return FMHC_OK;
}

// Unique ID of the context current on this thread (0 if none is current yet).
unsigned long long current_ctx_id() {
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (g_ctx_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (g_ctx_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of the scratch array in the current context (looked up on
// the first call in each context).
int scratch_for_current_device(void **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    return fmhc::set_last_error(FMHC_ERR_CUDA, "fmhc_k1_bwd_noalloc: no usable current device");
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (int e = driver_fns()) return e;
  unsigned long long id = current_ctx_id();
  if (id == 0 || g_cache[dev].ctx_id != id || g_cache[dev].ptr == nullptr) {
    // cudaGetSymbolAddress also makes the device's primary context current on
    // this thread if none was, so the context ID is read again afterwards.
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
    id = current_ctx_id();
    g_cache[dev] = Cached{id, p};
  }
  *out = g_cache[dev].ptr;
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
