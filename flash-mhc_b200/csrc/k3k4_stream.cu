// K3 (pre-map) and K4 (post-res) forward/backward: single-pass streaming
// kernels over the (T, 4, C) residual streams.
//
// Work mapping: one warp owns one token row at a time (a grid-stride loop over
// tokens), lanes walk the C dimension in chunks of VEC bf16 values (VEC = 8 ->
// 128-bit accesses), U chunks per lane are loaded before any is used so that
// every lane keeps U*(bytes per chunk) in flight.  The per-token coefficients
// (h_pre / h_post / H_merged) are warp-uniform loads (one broadcast request).
// Per-token reductions over C (grad_h, grad_H) are accumulated in registers
// and finished with a warp reduce-scatter, so lane L ends up owning one output
// value and the stores are one coalesced request per token.
//
// Semantics follow src/flash_mhc/kernels.py:384-853 of the reference: bf16
// inputs are widened to f32, all arithmetic is f32, bf16 outputs are rounded
// once (RNE), reductions are stored as f32.
#include "fmhc_common.cuh"
#include "fmhc_launch.h"

#include <mutex>

// Chunks per lane in flight (U) and minimum resident blocks per SM (MINB,
// bounds registers) of each kernel; chosen by measurement at T=65536, C=1024.
#ifndef FMHC_K3F_U
#define FMHC_K3F_U 2
#endif
#ifndef FMHC_K3F_MINB
#define FMHC_K3F_MINB 1
#endif
#ifndef FMHC_K3B_U
#define FMHC_K3B_U 2
#endif
#ifndef FMHC_K3B_MINB
#define FMHC_K3B_MINB 1
#endif
#ifndef FMHC_K4F_U
#define FMHC_K4F_U 2
#endif
#ifndef FMHC_K4F_MINB
#define FMHC_K4F_MINB 1
#endif
#ifndef FMHC_K4B_U
#define FMHC_K4B_U 1
#endif
#ifndef FMHC_K4B_MINB
#define FMHC_K4B_MINB 2
#endif

namespace fmhc {

using bf16 = __nv_bfloat16;

// ---------------------------------------------------------------- K3 forward
template <int VEC, int U, int MINB, bool REV>
__global__ void __launch_bounds__(256, MINB)
k3_fwd_kernel(const bf16 *__restrict__ x, const float4 *__restrict__ hp,
              bf16 *__restrict__ out, int64_t T, int C) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int nchunk = C / VEC;
  for (int64_t i = warp; i < T; i += nwarps) {
    const int64_t t = REV ? T - 1 - i : i;  // sweep direction (kRev* below)
    const float4 h = __ldg(hp + t);
    const bf16 *xr = x + t * 4 * C;
    bf16 *orow = out + t * C;
    for (int c0 = lane; c0 < nchunk; c0 += 32 * U) {
      Chunk<VEC> a[U][4];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * u;
        if (c < nchunk) {
#pragma unroll
          for (int j = 0; j < 4; ++j) a[u][j] = ld_raw<VEC>(xr + j * C + c * VEC);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * u;
        if (c < nchunk) {
          float f0[VEC], f1[VEC], f2[VEC], f3[VEC], o[VEC];
          unpack(a[u][0], f0); unpack(a[u][1], f1); unpack(a[u][2], f2); unpack(a[u][3], f3);
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            float acc = h.x * f0[e];
            acc = fmaf(h.y, f1[e], acc);
            acc = fmaf(h.z, f2[e], acc);
            o[e] = fmaf(h.w, f3[e], acc);
          }
          store_stream<VEC>(orow + c * VEC, o);
        }
      }
    }
  }
}

// --------------------------------------------------------------- K3 backward
template <int VEC, int U, int MINB, bool REV>
__global__ void __launch_bounds__(256, MINB)
k3_bwd_kernel(const bf16 *__restrict__ go, const bf16 *__restrict__ x,
              const float4 *__restrict__ hp, bf16 *__restrict__ gx,
              float *__restrict__ gh, int64_t T, int C) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int nchunk = C / VEC;
  for (int64_t i = warp; i < T; i += nwarps) {
    const int64_t t = REV ? T - 1 - i : i;  // sweep direction (kRev* below)
    const float4 h = __ldg(hp + t);
    const float hj[4] = {h.x, h.y, h.z, h.w};
    const bf16 *xr = x + t * 4 * C;
    const bf16 *gorow = go + t * C;
    bf16 *gxr = gx + t * 4 * C;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c0 = lane; c0 < nchunk; c0 += 32 * U) {
      Chunk<VEC> g[U], a[U][4];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * u;
        if (c < nchunk) {
          g[u] = ld_raw<VEC>(gorow + c * VEC);
#pragma unroll
          for (int j = 0; j < 4; ++j) a[u][j] = ld_raw<VEC>(xr + j * C + c * VEC);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * u;
        if (c < nchunk) {
          float fg[VEC];
          unpack(g[u], fg);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float fx[VEC], o[VEC];
            unpack(a[u][j], fx);
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              o[e] = hj[j] * fg[e];
              acc[j] = fmaf(fx[e], fg[e], acc[j]);
            }
            if (gx) store_stream<VEC>(gxr + j * C + c * VEC, o);
          }
        }
      }
    }
    warp_reduce_scatter<4>(acc, lane);
    if ((lane & 7) == 0) __stcs(gh + t * 4 + scatter_index<4>(lane), acc[0]);
  }
}

// ---------------------------------------------------------------- K4 forward
template <int VEC, int U, int MINB, bool REV>
__global__ void __launch_bounds__(256, MINB)
k4_fwd_kernel(const bf16 *__restrict__ x, const bf16 *__restrict__ lo,
              const float4 *__restrict__ H, const float4 *__restrict__ hpost,
              bf16 *__restrict__ out, int64_t T, int C) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int nchunk = C / VEC;
  for (int64_t i = warp; i < T; i += nwarps) {
    const int64_t t = REV ? T - 1 - i : i;  // sweep direction (kRev* below)
    float Hm[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 r = __ldg(H + t * 4 + i);
      Hm[i][0] = r.x; Hm[i][1] = r.y; Hm[i][2] = r.z; Hm[i][3] = r.w;
    }
    const float4 hp4 = __ldg(hpost + t);
    const float hp[4] = {hp4.x, hp4.y, hp4.z, hp4.w};
    const bf16 *xr = x + t * 4 * C;
    const bf16 *lor = lo + t * C;
    bf16 *orow = out + t * 4 * C;
    for (int c0 = lane; c0 < nchunk; c0 += 32 * U) {
      Chunk<VEC> a[U][4], l[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * u;
        if (c < nchunk) {
          l[u] = ld_raw<VEC>(lor + c * VEC);
#pragma unroll
          for (int j = 0; j < 4; ++j) a[u][j] = ld_raw<VEC>(xr + j * C + c * VEC);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * u;
        if (c < nchunk) {
          float fl[VEC], fx[4][VEC];
          unpack(l[u], fl);
#pragma unroll
          for (int j = 0; j < 4; ++j) unpack(a[u][j], fx[j]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float o[VEC];
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              // Same order as the reference kernel: hp*lo first, then j = 0..3.
              float acc = hp[i] * fl[e];
              acc = fmaf(Hm[i][0], fx[0][e], acc);
              acc = fmaf(Hm[i][1], fx[1][e], acc);
              acc = fmaf(Hm[i][2], fx[2][e], acc);
              o[e] = fmaf(Hm[i][3], fx[3][e], acc);
            }
            store_stream<VEC>(orow + i * C + c * VEC, o);
          }
        }
      }
    }
  }
}

// --------------------------------------------------------------- K4 backward
// WITH_GX = false computes only grad_lo, grad_H and grad_h_post (the fused
// block forms K4's grad_x later, inside its grad_x combination).
template <int VEC, int U, int MINB, bool WITH_GX, bool REV>
__global__ void __launch_bounds__(256, MINB)
k4_bwd_kernel(const bf16 *__restrict__ go, const bf16 *__restrict__ x,
              const bf16 *__restrict__ lo, const float4 *__restrict__ H,
              const float4 *__restrict__ hpost, bf16 *__restrict__ gx,
              bf16 *__restrict__ glo, float *__restrict__ gH,
              float *__restrict__ ghp, int64_t T, int C) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int nchunk = C / VEC;
  for (int64_t i = warp; i < T; i += nwarps) {
    const int64_t t = REV ? T - 1 - i : i;  // sweep direction (kRev* below)
    float Hm[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 r = __ldg(H + t * 4 + i);
      Hm[i][0] = r.x; Hm[i][1] = r.y; Hm[i][2] = r.z; Hm[i][3] = r.w;
    }
    const float4 hp4 = __ldg(hpost + t);
    const float hp[4] = {hp4.x, hp4.y, hp4.z, hp4.w};
    const bf16 *gor = go + t * 4 * C;
    const bf16 *xr = x + t * 4 * C;
    const bf16 *lor = lo + t * C;
    bf16 *gxr = WITH_GX ? gx + t * 4 * C : nullptr;
    bf16 *glor = glo + t * C;
    float accH[16];  // accH[i*4+j] = sum_c go_i * x_j
    float accP[4];   // accP[i]     = sum_c go_i * lo
#pragma unroll
    for (int k = 0; k < 16; ++k) accH[k] = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) accP[k] = 0.f;
    for (int c0 = lane; c0 < nchunk; c0 += 32 * U) {
      Chunk<VEC> g[U][4], a[U][4], l[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * u;
        if (c < nchunk) {
#pragma unroll
          for (int i = 0; i < 4; ++i) g[u][i] = ld_raw<VEC>(gor + i * C + c * VEC);
          l[u] = ld_raw<VEC>(lor + c * VEC);
#pragma unroll
          for (int j = 0; j < 4; ++j) a[u][j] = ld_raw<VEC>(xr + j * C + c * VEC);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * u;
        if (c < nchunk) {
          float fg[4][VEC];
#pragma unroll
          for (int i = 0; i < 4; ++i) unpack(g[u][i], fg[i]);
          {
            float fl[VEC], o[VEC];
            unpack(l[u], fl);
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              float s = hp[0] * fg[0][e];
              s = fmaf(hp[1], fg[1][e], s);
              s = fmaf(hp[2], fg[2][e], s);
              o[e] = fmaf(hp[3], fg[3][e], s);
#pragma unroll
              for (int i = 0; i < 4; ++i) accP[i] = fmaf(fg[i][e], fl[e], accP[i]);
            }
            store_stream<VEC>(glor + c * VEC, o);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float fx[VEC], o[VEC];
            unpack(a[u][j], fx);
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              if constexpr (WITH_GX) {
                float s = Hm[0][j] * fg[0][e];
                s = fmaf(Hm[1][j], fg[1][e], s);
                s = fmaf(Hm[2][j], fg[2][e], s);
                o[e] = fmaf(Hm[3][j], fg[3][e], s);
              }
#pragma unroll
              for (int i = 0; i < 4; ++i) accH[i * 4 + j] = fmaf(fg[i][e], fx[e], accH[i * 4 + j]);
            }
            if constexpr (WITH_GX) store_stream<VEC>(gxr + j * C + c * VEC, o);
          }
        }
      }
    }
    warp_reduce_scatter<16>(accH, lane);
    warp_reduce_scatter<4>(accP, lane);
    if ((lane & 1) == 0) __stcs(gH + t * 16 + scatter_index<16>(lane), accH[0]);
    if ((lane & 7) == 0) __stcs(ghp + t * 4 + scatter_index<4>(lane), accP[0]);
  }
}

// ------------------------------------------ combined grad_x of the block
// gx[t,j,c] = bf16( gx1[t,j,c] + h_pre[t,j] * g_li[t,c] + k4[t,j,c] )
// The three contributions to the gradient of the residual streams (K1's
// backward, K3's grad_x, K4's grad_x) in one pass.  MODE selects K4's term:
//   0: none;
//   1: k4 = gx4, K4's grad_x as written by its backward kernel (bf16);
//   2: k4 = sum_i H[t,i,j] * go[t,i,c], formed here from K4's upstream
//      gradient go (T, 4, C) and H_merged, in f32 and in the order K4's
//      backward uses, so K4's backward need not write its grad_x at all.
template <int VEC, int U, int MODE, bool REV>
__global__ void __launch_bounds__(256)
grad_x_combine_kernel(const bf16 *__restrict__ gx1, const bf16 *__restrict__ gli,
                      const float4 *__restrict__ hp, const bf16 *__restrict__ k4,
                      const float4 *__restrict__ H, bf16 *__restrict__ gx, int64_t T, int C) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int nchunk = C / VEC;
  for (int64_t i = warp; i < T; i += nwarps) {
    const int64_t t = REV ? T - 1 - i : i;  // sweep direction (kRev* below)
    const float4 h = __ldg(hp + t);
    const float hj[4] = {h.x, h.y, h.z, h.w};
    float Hm[4][4];
    if constexpr (MODE == 2) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 r = __ldg(H + t * 4 + i);
        Hm[i][0] = r.x; Hm[i][1] = r.y; Hm[i][2] = r.z; Hm[i][3] = r.w;
      }
    }
    const int64_t row = t * 4 * C;
    for (int c0 = lane; c0 < nchunk; c0 += 32 * U) {
      Chunk<VEC> g[U], a[U][4], b[U][4];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * u;
        if (c < nchunk) {
          g[u] = ld_raw<VEC>(gli + t * C + c * VEC);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            a[u][j] = ld_raw<VEC>(gx1 + row + j * C + c * VEC);
            if constexpr (MODE != 0) b[u][j] = ld_raw<VEC>(k4 + row + j * C + c * VEC);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + 32 * u;
        if (c < nchunk) {
          float fg[VEC];
          unpack(g[u], fg);
          float fo[4][VEC];  // MODE 2: the four go rows
          if constexpr (MODE == 2) {
#pragma unroll
            for (int i = 0; i < 4; ++i) unpack(b[u][i], fo[i]);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float fa[VEC], o[VEC];
            unpack(a[u][j], fa);
            if constexpr (MODE == 1) {
              float fb[VEC];
              unpack(b[u][j], fb);
#pragma unroll
              for (int e = 0; e < VEC; ++e) o[e] = fmaf(hj[j], fg[e], fa[e] + fb[e]);
            } else if constexpr (MODE == 2) {
#pragma unroll
              for (int e = 0; e < VEC; ++e) {
                float s4 = Hm[0][j] * fo[0][e];
                s4 = fmaf(Hm[1][j], fo[1][e], s4);
                s4 = fmaf(Hm[2][j], fo[2][e], s4);
                s4 = fmaf(Hm[3][j], fo[3][e], s4);
                o[e] = fmaf(hj[j], fg[e], fa[e] + s4);
              }
            } else {
#pragma unroll
              for (int e = 0; e < VEC; ++e) o[e] = fmaf(hj[j], fg[e], fa[e]);
            }
            store_stream<VEC>(gx + row + j * C + c * VEC, o);
          }
        }
      }
    }
  }
}

// ------------------------------------------------------------------ launchers
// Resident blocks per SM of `kernel` and the SM count, cached for the process
// (occupancy queries and attribute reads stay out of CUDA-graph captures and
// out of the per-launch cost).
template <class K>
int grid_for(K kernel, int64_t T, int threads) {
  struct Entry {
    const void *k;
    int dev, per_sm, sms;
  };
  static std::mutex mu;
  static Entry cache[64];
  static int used = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  int per_sm = 0, sms = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i)
      if (cache[i].k == reinterpret_cast<const void *>(kernel) && cache[i].dev == dev) {
        per_sm = cache[i].per_sm;
        sms = cache[i].sms;
      }
    if (sms == 0) {
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0);
      if (per_sm < 1) per_sm = 1;
      if (used < 64) cache[used++] = Entry{reinterpret_cast<const void *>(kernel), dev, per_sm, sms};
    }
  }
  const int64_t warps_per_block = threads / 32;
  const int64_t need = (T + warps_per_block - 1) / warps_per_block;
  const int64_t cap = int64_t(sms) * per_sm;
  return int(need < cap ? need : cap);
}

namespace {
constexpr int kThreads = 256;

// Token sweep direction of each streaming kernel.  Every kernel of the path
// reads x (T, 4, C), and at its end the L2 holds the tokens it touched last;
// the next kernel starting from that end reads them from L2 instead of HBM.
// The grid-stride loops sweep all tokens coherently (warp w handles the w-th
// token of the current window), so alternating directions between
// consecutive kernels of the step K1f, K3f, K4f, K4b, K3b, K1b gives every
// boundary that reuse: K3f forward, K4f backward, K4b forward, K3b backward
// (K1b sweeps forward; K1f gives each CTA a contiguous range, so it has no
// single direction).  In the block's backward the grad_x combination follows
// K1b and reads K1b's grad_x backward, from its most recently written end.
// Outputs are per token, so the direction changes no result bit.
#ifndef FMHC_SWEEP_ALT  // 0: every kernel sweeps forward (A/B measurements)
#define FMHC_SWEEP_ALT 1
#endif
// The direction is a template parameter: as a runtime argument the extra
// select in the token loop cost K4 bwd 7% (0.310 -> 0.332 ms at T = 65536,
// C = 1024, same box), while the forward instantiations here compile to the
// loop without it.
constexpr bool kRevK3Fwd = false;
constexpr bool kRevK4Fwd = FMHC_SWEEP_ALT != 0;
constexpr bool kRevK4Bwd = false;
constexpr bool kRevK3Bwd = FMHC_SWEEP_ALT != 0;
constexpr bool kRevCombine = FMHC_SWEEP_ALT != 0;

}  // namespace

#define FMHC_DISPATCH_VEC(VEC_RT, ...)                      \
  switch (VEC_RT) {                                         \
    case 8: { constexpr int VEC = 8; __VA_ARGS__; } break;  \
    case 4: { constexpr int VEC = 4; __VA_ARGS__; } break;  \
    case 2: { constexpr int VEC = 2; __VA_ARGS__; } break;  \
    default: { constexpr int VEC = 1; __VA_ARGS__; } break; \
  }

void launch_k3_fwd(const void *x, const float *hp, void *out, int64_t T, int C, int vec,
                   cudaStream_t s) {
  FMHC_DISPATCH_VEC(vec, {
    auto k = k3_fwd_kernel<VEC, FMHC_K3F_U, FMHC_K3F_MINB, kRevK3Fwd>;
    launch(k, dim3(grid_for(k, T, kThreads)), dim3(kThreads), 0, s, (const bf16 *)x,
           (const float4 *)hp, (bf16 *)out, T, C);
  });
}

void launch_k3_bwd(const void *go, const void *x, const float *hp, void *gx, float *gh,
                   int64_t T, int C, int vec, cudaStream_t s) {
  FMHC_DISPATCH_VEC(vec, {
    auto k = k3_bwd_kernel<VEC, FMHC_K3B_U, FMHC_K3B_MINB, kRevK3Bwd>;
    launch(k, dim3(grid_for(k, T, kThreads)), dim3(kThreads), 0, s, (const bf16 *)go,
           (const bf16 *)x, (const float4 *)hp, (bf16 *)gx, gh, T, C);
  });
}

void launch_k4_fwd(const void *x, const void *lo, const float *H, const float *hp, void *out,
                   int64_t T, int C, int vec, cudaStream_t s) {
  FMHC_DISPATCH_VEC(vec, {
    auto k = k4_fwd_kernel<VEC, FMHC_K4F_U, FMHC_K4F_MINB, kRevK4Fwd>;
    launch(k, dim3(grid_for(k, T, kThreads)), dim3(kThreads), 0, s, (const bf16 *)x,
           (const bf16 *)lo, (const float4 *)H, (const float4 *)hp, (bf16 *)out, T, C);
  });
}

void launch_grad_x_combine(const void *gx1, const void *gli, const float *hp, const void *gx4,
                           void *gx, int64_t T, int C, int vec, cudaStream_t s) {
  FMHC_DISPATCH_VEC(vec, {
    if (gx4) {
      auto k = grad_x_combine_kernel<VEC, 2, 1, kRevCombine>;
      launch(k, dim3(grid_for(k, T, kThreads)), dim3(kThreads), 0, s, (const bf16 *)gx1,
             (const bf16 *)gli, (const float4 *)hp, (const bf16 *)gx4, (const float4 *)nullptr,
             (bf16 *)gx, T, C);
    } else {
      auto k = grad_x_combine_kernel<VEC, 2, 0, kRevCombine>;
      launch(k, dim3(grid_for(k, T, kThreads)), dim3(kThreads), 0, s, (const bf16 *)gx1,
             (const bf16 *)gli, (const float4 *)hp, (const bf16 *)nullptr, (const float4 *)nullptr,
             (bf16 *)gx, T, C);
    }
  });
}

void launch_grad_x_combine_post(const void *gx1, const void *gli, const float *hp,
                                const void *go, const float *H, void *gx, int64_t T, int C,
                                int vec, cudaStream_t s) {
  FMHC_DISPATCH_VEC(vec, {
    auto k = grad_x_combine_kernel<VEC, 2, 2, kRevCombine>;
    launch(k, dim3(grid_for(k, T, kThreads)), dim3(kThreads), 0, s, (const bf16 *)gx1,
           (const bf16 *)gli, (const float4 *)hp, (const bf16 *)go, (const float4 *)H,
           (bf16 *)gx, T, C);
  });
}

void launch_k4_bwd(const void *go, const void *x, const void *lo, const float *H,
                   const float *hp, void *gx, void *glo, float *gH, float *ghp, int64_t T,
                   int C, int vec, cudaStream_t s) {
  FMHC_DISPATCH_VEC(vec, {
    if (gx) {
      auto k = k4_bwd_kernel<VEC, FMHC_K4B_U, FMHC_K4B_MINB, true, kRevK4Bwd>;
      launch(k, dim3(grid_for(k, T, kThreads)), dim3(kThreads), 0, s, (const bf16 *)go,
             (const bf16 *)x, (const bf16 *)lo, (const float4 *)H, (const float4 *)hp,
             (bf16 *)gx, (bf16 *)glo, gH, ghp, T, C);
    } else {
      auto k = k4_bwd_kernel<VEC, FMHC_K4B_U, FMHC_K4B_MINB, false, kRevK4Bwd>;
      launch(k, dim3(grid_for(k, T, kThreads)), dim3(kThreads), 0, s, (const bf16 *)go,
             (const bf16 *)x, (const bf16 *)lo, (const float4 *)H, (const float4 *)hp,
             (bf16 *)nullptr, (bf16 *)glo, gH, ghp, T, C);
    }
  });
}

}  // namespace fmhc
