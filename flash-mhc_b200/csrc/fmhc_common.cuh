// Shared device helpers for the mHC-lite kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
#include <utility>

namespace fmhc {

constexpr int kStreams = 4;   // n: residual streams (the kernels are specialised for 4)
constexpr int kWarp = 32;

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  Every kernel of this library is launched
// with launch() below, so the next kernel in the stream is scheduled as the
// CTAs of the previous one exit instead of after the whole grid has drained
// and flushed, hiding launch latency and the next kernel's prologue (barrier
// set-up, TMEM allocation, tensor-map prefetch).  The rule that makes this
// safe: every kernel calls pdl_wait() before its first global-memory access
// (read or write); it returns once the preceding grid has completed and its
// writes are visible.  No kernel triggers its dependents early: a trigger at
// kernel start let the whole step's kernels launch ahead and park CTAs on the
// SMs, 17% slower than none; without it a dependent cannot become resident
// beside a CTA of its predecessor, so TMEM and shared memory are never
// contended across kernels.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Barrier over `nthreads` threads (whole warps) of the block on barrier `id`
// (1..15; 0 is __syncthreads()).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// On unless the environment sets FLASH_MHC_PDL=0 (read once per process).
inline bool pdl_enabled() {
  static const bool on = [] {
    const char *e = std::getenv("FLASH_MHC_PDL");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t s, Args &&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// launch() with thread-block clusters of `cluster_x` CTAs along x.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                  cudaStream_t s, unsigned cluster_x, Args &&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// bf16 <-> f32 on packed 32-bit words.  bf16 -> f32 is exact (a shift);
// f32 -> bf16 uses the hardware round-to-nearest-even conversion.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

// A chunk of VEC consecutive bf16 values moved as one memory transaction.
template <int VEC> struct Chunk;
template <> struct Chunk<8> { uint4 v; };
template <> struct Chunk<4> { uint2 v; };
template <> struct Chunk<2> { uint32_t v; };
template <> struct Chunk<1> { uint16_t v; };

// Streaming (evict-first) loads for data read exactly once.
template <int VEC>
__device__ __forceinline__ void load_stream(const __nv_bfloat16 *p, float (&f)[VEC]) {
  if constexpr (VEC == 8) {
    uint4 u = __ldcs(reinterpret_cast<const uint4 *>(p));
    f[0] = bf16lo(u.x); f[1] = bf16hi(u.x); f[2] = bf16lo(u.y); f[3] = bf16hi(u.y);
    f[4] = bf16lo(u.z); f[5] = bf16hi(u.z); f[6] = bf16lo(u.w); f[7] = bf16hi(u.w);
  } else if constexpr (VEC == 4) {
    uint2 u = __ldcs(reinterpret_cast<const uint2 *>(p));
    f[0] = bf16lo(u.x); f[1] = bf16hi(u.x); f[2] = bf16lo(u.y); f[3] = bf16hi(u.y);
  } else if constexpr (VEC == 2) {
    uint32_t u = __ldcs(reinterpret_cast<const unsigned int *>(p));
    f[0] = bf16lo(u); f[1] = bf16hi(u);
  } else {
    unsigned short u = __ldcs(reinterpret_cast<const unsigned short *>(p));
    f[0] = __uint_as_float(uint32_t(u) << 16);
  }
}

// Raw streaming load (kept packed so several can be in flight before use).
template <int VEC>
__device__ __forceinline__ Chunk<VEC> ld_raw(const __nv_bfloat16 *p) {
  Chunk<VEC> c;
  if constexpr (VEC == 8) c.v = __ldcs(reinterpret_cast<const uint4 *>(p));
  else if constexpr (VEC == 4) c.v = __ldcs(reinterpret_cast<const uint2 *>(p));
  else if constexpr (VEC == 2) c.v = __ldcs(reinterpret_cast<const unsigned int *>(p));
  else c.v = __ldcs(reinterpret_cast<const unsigned short *>(p));
  return c;
}

template <int VEC>
__device__ __forceinline__ void unpack(const Chunk<VEC> &c, float (&f)[VEC]) {
  if constexpr (VEC == 8) {
    f[0] = bf16lo(c.v.x); f[1] = bf16hi(c.v.x); f[2] = bf16lo(c.v.y); f[3] = bf16hi(c.v.y);
    f[4] = bf16lo(c.v.z); f[5] = bf16hi(c.v.z); f[6] = bf16lo(c.v.w); f[7] = bf16hi(c.v.w);
  } else if constexpr (VEC == 4) {
    f[0] = bf16lo(c.v.x); f[1] = bf16hi(c.v.x); f[2] = bf16lo(c.v.y); f[3] = bf16hi(c.v.y);
  } else if constexpr (VEC == 2) {
    f[0] = bf16lo(c.v); f[1] = bf16hi(c.v);
  } else {
    f[0] = __uint_as_float(uint32_t(c.v) << 16);
  }
}

// Streaming store (no L2 write-allocate reuse expected).
template <int VEC>
__device__ __forceinline__ void store_stream(__nv_bfloat16 *p, const float (&f)[VEC]) {
  if constexpr (VEC == 8) {
    uint4 u;
    u.x = pack_bf16x2(f[0], f[1]); u.y = pack_bf16x2(f[2], f[3]);
    u.z = pack_bf16x2(f[4], f[5]); u.w = pack_bf16x2(f[6], f[7]);
    __stcs(reinterpret_cast<uint4 *>(p), u);
  } else if constexpr (VEC == 4) {
    uint2 u;
    u.x = pack_bf16x2(f[0], f[1]); u.y = pack_bf16x2(f[2], f[3]);
    __stcs(reinterpret_cast<uint2 *>(p), u);
  } else if constexpr (VEC == 2) {
    __stcs(reinterpret_cast<unsigned int *>(p), pack_bf16x2(f[0], f[1]));
  } else {
    __nv_bfloat16 b = __float2bfloat16_rn(f[0]);
    __stcs(reinterpret_cast<unsigned short *>(p), *reinterpret_cast<unsigned short *>(&b));
  }
}

// ---------------------------------------------------------------------------
// Warp "reduce-scatter": each lane holds N partial sums (N a power of two,
// N <= 32).  After the call, lane L holds in v[0] the warp-wide total of value
// index scatter_index<N>(L).  Costs N-1 + log2(32/N) shuffles instead of
// N*5 for N independent butterflies.
// ---------------------------------------------------------------------------
template <int N>
__device__ __forceinline__ int scatter_index(int lane) {
  // Step s (offset 16>>s) keeps the upper half of the live values when bit
  // (4-s) of the lane is set; the kept halves compose the index MSB-first.
  int idx = 0;
  int live = N;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    if (live > 1) {
      live >>= 1;
      if (lane & off) idx += live;
    }
  }
  return idx;
}

template <int N>
__device__ __forceinline__ void warp_reduce_scatter(float (&v)[N], int lane) {
  int live = N;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    if (live > 1) {
      const int half = live >> 1;
      const bool upper = (lane & off) != 0;
#pragma unroll
      for (int k = 0; k < half; ++k) {
        float send = upper ? v[k] : v[k + half];
        float keep = upper ? v[k + half] : v[k];
        v[k] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
      live = half;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    }
  }
}

}  // namespace fmhc
