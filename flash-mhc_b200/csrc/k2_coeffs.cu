// K2: the per-token coefficient math of mHC-lite, forward and backward, as one
// kernel each (the reference runs it as ~20 eager torch launches in the
// caller, src/flash_mhc/block.py:150-170).  The per-token forward and its
// rounding rules live in k2_token.cuh (shared with the K1 forward kernels
// that run it in their epilogue).
//
// The backward takes the f32 gradients of h_pre (from K3's backward), h_post
// and H_merged (from K4's backward), recomputes the forward intermediates from
// proj and returns grad_proj (bf16, the dtype of proj) plus the parameter
// gradients (3 alphas, 32 bias entries) summed over tokens in a fixed order.
#include "k2_token.cuh"

namespace fmhc {

using bf16 = __nv_bfloat16;

namespace {

using k2tok::kP;
using k2tok::kNF;
using K2Smem = k2tok::ParamSmem;
using K2Tok = k2tok::Tok;

__device__ __forceinline__ void load_params(K2Smem &sm, const K2Params &P) {
  k2tok::stage_params(sm, P, threadIdx.x, blockDim.x);
  __syncthreads();
}

__device__ __forceinline__ void load_proj(const bf16 *proj, int64_t t, float (&v)[32]) {
  const uint4 *p4 = reinterpret_cast<const uint4 *>(proj + t * 32);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 u = __ldg(p4 + c);
    v[8 * c + 0] = bf16lo(u.x); v[8 * c + 1] = bf16hi(u.x);
    v[8 * c + 2] = bf16lo(u.y); v[8 * c + 3] = bf16hi(u.y);
    v[8 * c + 4] = bf16lo(u.z); v[8 * c + 5] = bf16hi(u.z);
    v[8 * c + 6] = bf16lo(u.w); v[8 * c + 7] = bf16hi(u.w);
  }
}

}  // namespace

__global__ void __launch_bounds__(256)
k2_fwd_kernel(const bf16 *__restrict__ proj, const K2Params P, float4 *__restrict__ h_pre,
              float4 *__restrict__ h_post, float4 *__restrict__ H, int64_t T) {
  pdl_wait();
  __shared__ K2Smem sm;
  const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  float v[32];
  if (t < T) load_proj(proj, t, v);  // in flight while the parameters are staged
  load_params(sm, P);
  if (t >= T) return;
  k2tok::store_coeffs(sm, v, h_pre, h_post, H, t);
}

// One thread per token; each block writes the sums of its tokens' parameter
// gradients to part[blockIdx.x][35].
__global__ void __launch_bounds__(256)
k2_bwd_kernel(const bf16 *__restrict__ proj, const K2Params P, const float4 *__restrict__ g_hpre,
              const float4 *__restrict__ g_hpost, const float4 *__restrict__ g_H,
              bf16 *__restrict__ g_proj, float *__restrict__ part, int64_t T) {
  pdl_wait();
  __shared__ K2Smem sm;
  __shared__ float red[8][kP];
  load_params(sm, P);
  const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  float gp[kP];  // this token's contribution to the 35 parameter gradients
#pragma unroll
  for (int i = 0; i < kP; ++i) gp[i] = 0.f;
  if (t < T) {
    float v[32];
    load_proj(proj, t, v);
    K2Tok k;
    k2tok::forward_token(sm, v, k);
    const float4 a4 = g_hpre[t], b4 = g_hpost[t];
    float ghpre[4] = {a4.x, a4.y, a4.z, a4.w};
    float ghpost[4] = {b4.x, b4.y, b4.z, b4.w};
    float gH[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 r = g_H[t * 4 + i];
      gH[4 * i + 0] = r.x; gH[4 * i + 1] = r.y; gH[4 * i + 2] = r.z; gH[4 * i + 3] = r.w;
    }
    // H_merged = H_res - h_post (outer) h_pre
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ghpost[i] = fmaf(-gH[4 * i + j], k.hpre[j], ghpost[i]);
        ghpre[j] = fmaf(-gH[4 * i + j], k.hpost[i], ghpre[j]);
      }
    }
    // H_res = sum_k a_k perm_k ; softmax backward
    float ga[kNF], dot = 0.f;
#pragma unroll
    for (int j = 0; j < kNF; ++j) {
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) acc = fmaf(gH[e], sm.perm[j * 16 + e], acc);
      ga[j] = acc;
      dot = fmaf(acc, k.a[j], dot);
    }
    const float ap = sm.par[0], aq = sm.par[1], ar = sm.par[2];
    float g[32];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float zpre = ghpre[i] * k.spre[i] * (1.f - k.spre[i]);
      const float zpost = ghpost[i] * 2.f * k.spost[i] * (1.f - k.spost[i]);
      g[i] = zpre * ap;
      g[4 + i] = zpost * aq;
      gp[0] = fmaf(zpre, v[i], gp[0]);
      gp[1] = fmaf(zpost, v[4 + i], gp[1]);
      gp[3 + i] = zpre;
      gp[7 + i] = zpost;
    }
#pragma unroll
    for (int j = 0; j < kNF; ++j) {
      const float zr = k.a[j] * (ga[j] - dot);
      g[8 + j] = zr * ar;
      gp[2] = fmaf(zr, v[8 + j], gp[2]);
      gp[11 + j] = zr;
    }
    uint4 *o = reinterpret_cast<uint4 *>(g_proj + t * 32);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint4 w;
      w.x = pack_bf16x2(g[8 * c + 0], g[8 * c + 1]);
      w.y = pack_bf16x2(g[8 * c + 2], g[8 * c + 3]);
      w.z = pack_bf16x2(g[8 * c + 4], g[8 * c + 5]);
      w.w = pack_bf16x2(g[8 * c + 6], g[8 * c + 7]);
      o[c] = w;
    }
  }
  // Block sum of the 35 parameter gradients: warp butterflies, then the 8
  // warp sums in warp order.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < kP; ++i) {
    float s = gp[i];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) red[warp][i] = s;
  }
  __syncthreads();
  if (threadIdx.x < kP) {
    float s = 0.f;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) s += red[w][threadIdx.x];
    part[int64_t(blockIdx.x) * kP + threadIdx.x] = s;
  }
}

// One warp per parameter: lane l sums blocks l, l+32, ... then a fixed
// butterfly (deterministic).  The sum is written in the parameter's dtype
// (rounded once from the f32 total when that is bf16).
__global__ void k2_param_reduce_kernel(const float *__restrict__ part, const K2ParamGrads G,
                                       int nblocks) {
  pdl_wait();
  const int i = blockIdx.x, lane = threadIdx.x;
  float s = 0.f;
  for (int b = lane; b < nblocks; b += 32) s += part[int64_t(b) * kP + i];
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) {
    void *dst = i == 0 ? G.a_pre : i == 1 ? G.a_post : i == 2 ? G.a_res : G.bias;
    const int idx = i < 3 ? 0 : i - 3;
    if (G.bf16) reinterpret_cast<bf16 *>(dst)[idx] = __float2bfloat16_rn(s);
    else reinterpret_cast<float *>(dst)[idx] = s;
  }
}

int64_t k2_bwd_workspace_bytes(int64_t T) {
  const int64_t nb = (T + 255) / 256;
  return ((nb * kP * 4) + 255) & ~int64_t(255);
}

K2Params k2_packed_params(const float *params, const float *perm) {
  return K2Params{params, params + 1, params + 2, params + 3, perm, 0, 0};
}

void launch_k2_fwd(const void *proj, const K2Params &P, float *h_pre, float *h_post, float *H,
                   int64_t T, cudaStream_t s) {
  const unsigned nb = unsigned((T + 255) / 256);
  launch(k2_fwd_kernel, dim3(nb), dim3(256), 0, s, (const bf16 *)proj, P, (float4 *)h_pre,
         (float4 *)h_post, (float4 *)H, T);
}

K2ParamGrads k2_packed_grads(float *g_params) {
  return K2ParamGrads{g_params, g_params + 1, g_params + 2, g_params + 3, 0};
}

void launch_k2_bwd(const void *proj, const K2Params &P, const float *g_hpre, const float *g_hpost,
                   const float *g_H, void *g_proj, const K2ParamGrads &Gp, float *ws, int64_t T,
                   cudaStream_t s) {
  const unsigned nb = unsigned((T + 255) / 256);
  if (T == 0) {  // empty batch: the parameter gradients are zero
    launch(k2_param_reduce_kernel, dim3(kP), dim3(32), 0, s, (const float *)nullptr, Gp, 0);
    return;
  }
  launch(k2_bwd_kernel, dim3(nb), dim3(256), 0, s, (const bf16 *)proj, P, (const float4 *)g_hpre, (const float4 *)g_hpost, (const float4 *)g_H, (bf16 *)g_proj, ws,
         T);
  launch(k2_param_reduce_kernel, dim3(kP), dim3(32), 0, s, ws, Gp, int(nb));
}

}  // namespace fmhc
