// K1 (fused RMSNorm + thin projection) on the CUDA cores.
//
// These kernels cover every shape (any nC, D <= 32, any T) and are the
// general path; the tensor-core kernels in k1_tc.cu take the shapes they
// support.  One warp owns one token row; lanes walk nC in VEC-wide chunks.
//
//   fwd : inv_rms[t] = rsqrt(sum_k x^2 / nC + 1e-6); out[t,d] = bf16(acc_d * inv_rms)
//         (src/flash_mhc/kernels.py:250-303)
//   dx  : gx = bf16(inv_rms * (go @ W) - (go . proj) * inv_rms^2 / nC * x)
//         (src/flash_mhc/kernels.py:306-376)
//   dW  : gW = bf16(sum_t bf16(go * inv_rms) x), two kernels: per-split f32
//         partial sums into caller workspace, then a fixed-order reduction
//         (deterministic), replacing src/flash_mhc/ops.py:683-684.
#include "fmhc_common.cuh"
#include "fmhc_launch.h"
#include "k2_token.cuh"

#include <mutex>

namespace fmhc {

using bf16 = __nv_bfloat16;
constexpr float kK1Eps = 1e-6f;

template <int VEC>
__global__ void __launch_bounds__(256)
k1_fwd_simt_kernel(const bf16 *__restrict__ x, const bf16 *__restrict__ W,
                   bf16 *__restrict__ out, float *__restrict__ inv_rms, int64_t T, int nC,
                   int D) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int nchunk = nC / VEC;
  for (int64_t t = warp; t < T; t += nwarps) {
    const bf16 *xr = x + t * nC;
    float acc[32];
#pragma unroll
    for (int d = 0; d < 32; ++d) acc[d] = 0.f;
    float ss = 0.f;
    for (int c = lane; c < nchunk; c += 32) {
      float fx[VEC];
      load_stream<VEC>(xr + c * VEC, fx);
#pragma unroll
      for (int e = 0; e < VEC; ++e) ss = fmaf(fx[e], fx[e], ss);
#pragma unroll
      for (int d = 0; d < 32; ++d) {
        if (d < D) {
          float fw[VEC];
          // W is small and shared by every token: keep it in the caches.
          if constexpr (VEC == 8) {
            uint4 u = __ldg(reinterpret_cast<const uint4 *>(W + int64_t(d) * nC + c * VEC));
            fw[0] = bf16lo(u.x); fw[1] = bf16hi(u.x); fw[2] = bf16lo(u.y); fw[3] = bf16hi(u.y);
            fw[4] = bf16lo(u.z); fw[5] = bf16hi(u.z); fw[6] = bf16lo(u.w); fw[7] = bf16hi(u.w);
          } else {
#pragma unroll
            for (int e = 0; e < VEC; ++e) fw[e] = __bfloat162float(W[int64_t(d) * nC + c * VEC + e]);
          }
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[d] = fmaf(fx[e], fw[e], acc[d]);
        }
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float r = rsqrtf(ss / float(nC) + kK1Eps);
    warp_reduce_scatter<32>(acc, lane);
    const int d = scatter_index<32>(lane);
    if (d < D) out[t * D + d] = __float2bfloat16_rn(acc[0] * r);
    if (lane == 0) inv_rms[t] = r;
  }
}

// Small-T forward.  One block of 256 threads per 2 tokens; the threads split
// the nC columns into 16-byte chunks (chunk c belongs to thread c mod 256) and
// each accumulates, over its chunks, both tokens' sums of squares and 32 dot
// products with W.  The block then reduces them: a warp butterfly per value,
// then the 8 warp totals are added in warp order in shared memory.  A tile of
// the tensor-core kernel walks its nC / 64 k-steps one after another, ~18 us
// at nC = 3072 whatever T; here every block makes one pass over W.
// Needs D == 32, nC % 8 == 0 and 16-byte aligned x and W.
//
// COEFFS: thread tb of the block then runs K2 on token tb's stored logits
// (k2_token.cuh) and writes h_pre, h_post and H_merged.  PRE (with COEFFS):
// the block then also runs K3 on its tokens, layer_input[t, c] =
// bf16(sum_j h_pre[t, j] x[t, j, c]) with the arithmetic of k3_fwd_kernel,
// re-reading the token rows it has just read from the caches (C % 8 == 0,
// 16-byte aligned layer_input).  At a few tokens the whole pre-block of the
// layer is then one launch instead of three.
constexpr int kRowsTB = 2;
template <bool COEFFS, bool PRE>
__global__ void __launch_bounds__(256, 1)
k1_fwd_rows_kernel(const bf16 *__restrict__ x, const bf16 *__restrict__ W,
                   bf16 *__restrict__ out, float *__restrict__ inv_rms, int64_t T, int nC,
                   int D, const K2Params P, const k2tok::Out co, bf16 *__restrict__ pre_out) {
  static_assert(COEFFS || !PRE, "K3 needs the coefficients");
  pdl_wait();
  __shared__ float red[8][kRowsTB][33];
  __shared__ float tot[kRowsTB][33];
  __shared__ k2tok::ParamSmem k2s;
  __shared__ float4 hs[kRowsTB];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if constexpr (COEFFS) k2tok::stage_params(k2s, P, tid, 256);  // read after the next barrier
  const int64_t t0 = int64_t(blockIdx.x) * kRowsTB;
  const bool has1 = t0 + 1 < T;
  const int nchunk = nC / 8;
  float acc0[32], acc1[32], ss0 = 0.f, ss1 = 0.f;
#pragma unroll
  for (int d = 0; d < 32; ++d) acc0[d] = acc1[d] = 0.f;
  for (int c = tid; c < nchunk; c += 256) {
    const uint4 u0 = __ldcs(reinterpret_cast<const uint4 *>(x + t0 * nC + c * 8));
    uint4 u1 = make_uint4(0u, 0u, 0u, 0u);
    if (has1) u1 = __ldcs(reinterpret_cast<const uint4 *>(x + (t0 + 1) * nC + c * 8));
    const float f0[8] = {bf16lo(u0.x), bf16hi(u0.x), bf16lo(u0.y), bf16hi(u0.y),
                         bf16lo(u0.z), bf16hi(u0.z), bf16lo(u0.w), bf16hi(u0.w)};
    const float f1[8] = {bf16lo(u1.x), bf16hi(u1.x), bf16lo(u1.y), bf16hi(u1.y),
                         bf16lo(u1.z), bf16hi(u1.z), bf16lo(u1.w), bf16hi(u1.w)};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      ss0 = fmaf(f0[e], f0[e], ss0);
      ss1 = fmaf(f1[e], f1[e], ss1);
    }
    // W rows in two batches of 16 loads, all in flight before their FMAs
    // (loads behind a per-row condition were issued one round trip at a time).
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint4 wv[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        wv[i] = __ldg(reinterpret_cast<const uint4 *>(W + int64_t(16 * h + i) * nC + c * 8));
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint4 u = wv[i];
        const float fw[8] = {bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y),
                             bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w)};
        const int d = 16 * h + i;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          acc0[d] = fmaf(f0[e], fw[e], acc0[d]);
          acc1[d] = fmaf(f1[e], fw[e], acc1[d]);
        }
      }
    }
  }
  // Butterfly per value: with two 32-value reduce-scatters the accumulators
  // were placed in local memory.
#pragma unroll
  for (int d = 0; d < 32; ++d)
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      acc0[d] += __shfl_xor_sync(0xffffffffu, acc0[d], off);
      acc1[d] += __shfl_xor_sync(0xffffffffu, acc1[d], off);
    }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    ss0 += __shfl_xor_sync(0xffffffffu, ss0, off);
    ss1 += __shfl_xor_sync(0xffffffffu, ss1, off);
  }
  if (lane == 0) {
#pragma unroll
    for (int d = 0; d < 32; ++d) {
      red[warp][0][d] = acc0[d];
      red[warp][1][d] = acc1[d];
    }
    red[warp][0][32] = ss0;
    red[warp][1][32] = ss1;
  }
  __syncthreads();
  if (tid < kRowsTB * 33) {
    const int tb = tid / 33, j = tid - tb * 33;
    float v = red[0][tb][j];
#pragma unroll
    for (int w = 1; w < 8; ++w) v += red[w][tb][j];
    tot[tb][j] = v;
  }
  __syncthreads();
  if (tid < kRowsTB * 32) {
    const int tb = tid / 32, d = tid - tb * 32;
    const int64_t t = t0 + tb;
    if (t < T) {
      const float r = rsqrtf(tot[tb][32] / float(nC) + kK1Eps);
      out[t * 32 + d] = __float2bfloat16_rn(tot[tb][d] * r);
      if (d == 0) inv_rms[t] = r;
    }
  }
  if constexpr (COEFFS) {
    if (tid < kRowsTB && t0 + tid < T) {
      const int64_t t = t0 + tid;
      const float r = rsqrtf(tot[tid][32] / float(nC) + kK1Eps);
      float pv[32];  // the logits as stored above (bf16)
#pragma unroll
      for (int d = 0; d < 32; ++d) pv[d] = __bfloat162float(__float2bfloat16_rn(tot[tid][d] * r));
      hs[tid] = k2tok::store_coeffs(k2s, pv, co.h_pre, co.h_post, co.H, t);
    }
  }
  if constexpr (PRE) {
    __syncthreads();
    const int C = nC >> 2, nch = C >> 3;
    for (int tb = 0; tb < kRowsTB; ++tb) {
      const int64_t t = t0 + tb;
      if (t >= T) break;
      const float4 h = hs[tb];
      const bf16 *xr = x + t * nC;
      for (int c = tid; c < nch; c += 256) {
        float f0[8], f1[8], f2[8], f3[8], o[8];
        Chunk<8> a0, a1, a2, a3;
        a0.v = __ldg(reinterpret_cast<const uint4 *>(xr + c * 8));
        a1.v = __ldg(reinterpret_cast<const uint4 *>(xr + C + c * 8));
        a2.v = __ldg(reinterpret_cast<const uint4 *>(xr + 2 * C + c * 8));
        a3.v = __ldg(reinterpret_cast<const uint4 *>(xr + 3 * C + c * 8));
        unpack(a0, f0); unpack(a1, f1); unpack(a2, f2); unpack(a3, f3);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float acc = h.x * f0[e];
          acc = fmaf(h.y, f1[e], acc);
          acc = fmaf(h.z, f2[e], acc);
          o[e] = fmaf(h.w, f3[e], acc);
        }
        store_stream<8>(pre_out + t * C + c * 8, o);
      }
    }
  }
}

template <int VEC>
__global__ void __launch_bounds__(256)
k1_bwd_dx_simt_kernel(const bf16 *__restrict__ go, const bf16 *__restrict__ x,
                      const bf16 *__restrict__ W, const bf16 *__restrict__ proj,
                      const float *__restrict__ inv_rms, bf16 *__restrict__ gx, int64_t T,
                      int nC, int D) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int nchunk = nC / VEC;
  for (int64_t t = warp; t < T; t += nwarps) {
    const float r = inv_rms[t];
    float g_l = 0.f, p_l = 0.f;
    if (lane < D) {
      g_l = __bfloat162float(go[t * D + lane]);
      p_l = __bfloat162float(proj[t * D + lane]);
    }
    float dot = g_l * p_l;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    const float s = dot * (r * r) / float(nC);
    float gd[32];
#pragma unroll
    for (int d = 0; d < 32; ++d) gd[d] = __shfl_sync(0xffffffffu, g_l, d);
    const bf16 *xr = x + t * nC;
    bf16 *gr = gx + t * nC;
    for (int c = lane; c < nchunk; c += 32) {
      float o[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = 0.f;
#pragma unroll
      for (int d = 0; d < 32; ++d) {
        if (d < D) {
          float fw[VEC];
          if constexpr (VEC == 8) {
            uint4 u = __ldg(reinterpret_cast<const uint4 *>(W + int64_t(d) * nC + c * VEC));
            fw[0] = bf16lo(u.x); fw[1] = bf16hi(u.x); fw[2] = bf16lo(u.y); fw[3] = bf16hi(u.y);
            fw[4] = bf16lo(u.z); fw[5] = bf16hi(u.z); fw[6] = bf16lo(u.w); fw[7] = bf16hi(u.w);
          } else {
#pragma unroll
            for (int e = 0; e < VEC; ++e) fw[e] = __bfloat162float(W[int64_t(d) * nC + c * VEC + e]);
          }
#pragma unroll
          for (int e = 0; e < VEC; ++e) o[e] = fmaf(gd[d], fw[e], o[e]);
        }
      }
      float fx[VEC];
      load_stream<VEC>(xr + c * VEC, fx);
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = r * o[e] - s * fx[e];
      store_stream<VEC>(gr + c * VEC, o);
    }
  }
}

// dW partial sums: block (256 threads) owns 256 consecutive columns k and one
// token split; the split's scaled grads bf16(go*inv_rms) are staged 32 tokens
// at a time in shared memory.  ws layout: [split][d][k] f32.
constexpr int kDwTile = 32;
__global__ void __launch_bounds__(256)
k1_dw_partial_kernel(const bf16 *__restrict__ go, const bf16 *__restrict__ x,
                     const float *__restrict__ inv_rms, float *__restrict__ ws, int64_t T,
                     int nC, int D, int64_t tokens_per_split) {
  pdl_wait();
  __shared__ float gos[kDwTile][32];
  const int k = blockIdx.x * 256 + threadIdx.x;
  const int split = blockIdx.y;
  const int64_t t0 = int64_t(split) * tokens_per_split;
  int64_t t1 = t0 + tokens_per_split;
  if (t1 > T) t1 = T;
  float acc[32];
#pragma unroll
  for (int d = 0; d < 32; ++d) acc[d] = 0.f;
  for (int64_t tb = t0; tb < t1; tb += kDwTile) {
    __syncthreads();
    for (int i = threadIdx.x; i < kDwTile * 32; i += 256) {
      const int tt = i / 32, d = i % 32;
      const int64_t t = tb + tt;
      float v = 0.f;
      if (t < t1 && d < D) {
        v = __bfloat162float(go[t * D + d]) * inv_rms[t];
        v = __bfloat162float(__float2bfloat16_rn(v));  // the reference rounds to bf16
      }
      gos[tt][d] = v;
    }
    __syncthreads();
    if (k < nC) {
      const int nt = int((t1 - tb) < kDwTile ? (t1 - tb) : kDwTile);
      for (int tt = 0; tt < nt; ++tt) {
        const float xv = __bfloat162float(x[(tb + tt) * nC + k]);
#pragma unroll
        for (int d = 0; d < 32; ++d) acc[d] = fmaf(gos[tt][d], xv, acc[d]);
      }
    }
  }
  if (k < nC) {
    for (int d = 0; d < D; ++d) ws[(int64_t(split) * D + d) * nC + k] = acc[d];
  }
}

__global__ void k1_dw_reduce_kernel(const float *__restrict__ ws, bf16 *__restrict__ gW,
                                    int nsplit, int64_t n) {
  pdl_wait();
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float s = 0.f;
  for (int p = 0; p < nsplit; ++p) s += ws[int64_t(p) * n + i];
  gW[i] = __float2bfloat16_rn(s);
}

int k1_dw_splits(int64_t T) {
  int64_t s = (T + 1023) / 1024;
  if (s < 1) s = 1;
  if (s > 16) s = 16;
  return int(s);
}

int64_t k1_dw_workspace_bytes(int64_t T, int64_t nC, int64_t D) {
  return int64_t(k1_dw_splits(T)) * D * nC * int64_t(sizeof(float));
}

namespace {
int sm_count() {
  static std::mutex mu;
  static int cache[16] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 16) dev = 15;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
  return cache[dev];
}
int warp_grid(int64_t T) {
  const int64_t cap = int64_t(sm_count()) * 8;  // 8 blocks of 8 warps per SM
  const int64_t need = (T + 7) / 8;
  return int(need < cap ? need : cap);
}
}  // namespace

void launch_k1_fwd_simt(const void *x, const void *W, void *out, float *inv_rms, int64_t T,
                        int nC, int D, int vec, cudaStream_t s) {
  if (vec == 8)
    launch(k1_fwd_simt_kernel<8>, dim3(warp_grid(T)), dim3(256), 0, s, (const bf16 *)x,
           (const bf16 *)W, (bf16 *)out, inv_rms, T, nC, D);
  else
    launch(k1_fwd_simt_kernel<1>, dim3(warp_grid(T)), dim3(256), 0, s, (const bf16 *)x,
           (const bf16 *)W, (bf16 *)out, inv_rms, T, nC, D);
}

void launch_k1_fwd_rows(const void *x, const void *W, void *out, float *inv_rms, int64_t T,
                        int nC, int D, cudaStream_t s, const K2Params *coeffs, float *h_pre,
                        float *h_post, float *H, void *pre_out) {
  const K2Params P = coeffs ? *coeffs : K2Params{};
  const k2tok::Out co{(float4 *)h_pre, (float4 *)h_post, (float4 *)H};
  auto k = !coeffs ? k1_fwd_rows_kernel<false, false>
         : pre_out ? k1_fwd_rows_kernel<true, true> : k1_fwd_rows_kernel<true, false>;
  launch(k, dim3(unsigned((T + kRowsTB - 1) / kRowsTB)), dim3(256), 0, s, (const bf16 *)x,
         (const bf16 *)W, (bf16 *)out, inv_rms, T, nC, D, P, co, (bf16 *)pre_out);
}

void launch_k1_bwd_dx_simt(const void *go, const void *x, const void *W, const void *proj,
                           const float *inv_rms, void *gx, int64_t T, int nC, int D, int vec,
                           cudaStream_t s) {
  if (vec == 8)
    launch(k1_bwd_dx_simt_kernel<8>, dim3(warp_grid(T)), dim3(256), 0, s, (const bf16 *)go,
           (const bf16 *)x, (const bf16 *)W, (const bf16 *)proj, inv_rms, (bf16 *)gx, T, nC, D);
  else
    launch(k1_bwd_dx_simt_kernel<1>, dim3(warp_grid(T)), dim3(256), 0, s, (const bf16 *)go,
           (const bf16 *)x, (const bf16 *)W, (const bf16 *)proj, inv_rms, (bf16 *)gx, T, nC, D);
}

void launch_k1_dw_simt(const void *go, const void *x, const float *inv_rms, void *gW,
                       float *ws, int64_t T, int nC, int D, cudaStream_t s) {
  const int nsplit = k1_dw_splits(T);
  const int64_t per = (T + nsplit - 1) / nsplit;
  dim3 grid((nC + 255) / 256, nsplit);
  launch(k1_dw_partial_kernel, dim3(grid), dim3(256), 0, s, (const bf16 *)go, (const bf16 *)x,
         inv_rms, ws, T, nC, D, per);
  const int64_t n = int64_t(D) * nC;
  launch(k1_dw_reduce_kernel, dim3(int((n + 255) / 256)), dim3(256), 0, s, ws, (bf16 *)gW, nsplit,
         n);
}

}  // namespace fmhc
