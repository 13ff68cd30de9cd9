// K2 forward for one token, shared by the stand-alone K2 kernel
// (k2_coeffs.cu) and the K1 forward kernels that run it in their epilogue
// (k1_tc.cu, k1_simt.cu), so every path computes the coefficients with the
// same instructions and gives the same bits.
//
// From the 32 projection logits proj = [p (4) | q (4) | r (24)] of a token
// (the bf16 values K1 stores):
//   h_pre   = sigmoid(a_pre * p + b[0:4])
//   h_post  = 2 * sigmoid(a_post * q + b[4:8])
//   a       = softmax(a_res * r + b[8:32])              (over the 24 entries)
//   H_res   = sum_k a[k] * perm[k]                      (4x4, perm rows are the
//                                                        flattened permutation matrices)
//   H_merged= H_res - h_post (outer) h_pre
// (reference: src/flash_mhc/block.py:150-170).  The reference evaluates this
// in the input dtype (bf16): alphas and bias are cast to bf16, every
// intermediate op rounds to bf16, and h_pre, h_post, H_merged are stored as
// bf16 before the f32 copies that K3/K4 consume.  Here the parameters are
// rounded to bf16 the same way (the reference's `.to(dt)`), the logits are
// the bf16 values K1 stores, and everything after that runs and is stored in
// f32: the coefficients are those of the reference's float32 path on the same
// logits, to f32 rounding.  (Rounding them to bf16 as the bf16 eager code does
// costs up to 2^-9 of each coefficient, which the post-mix multiplies by
// |x| + |layer_output|; in f32 they stay within 1e-4 of the float32 block.)
#pragma once

#include "fmhc_common.cuh"
#include "fmhc_launch.h"

namespace fmhc {
namespace k2tok {

constexpr int kP = 35;  // a_pre, a_post, a_res, bias[32]
constexpr int kNF = 24; // permutations of 4

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
__device__ __forceinline__ float sigm(float z) { return 1.f / (1.f + __expf(-z)); }

// The parameters, rounded to bf16, staged in shared memory.
struct ParamSmem {
  float par[kP];
  float perm[kNF * 16];
};

__device__ __forceinline__ float ld_param(const void *p, int i, int is_bf16) {
  return is_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i])
                 : reinterpret_cast<const float *>(p)[i];
}

// Threads tid = 0 .. nthreads-1 of the caller's group stage the parameters;
// the caller synchronises the group before the first read.
__device__ __forceinline__ void stage_params(ParamSmem &sm, const K2Params &P, int tid,
                                             int nthreads) {
  for (int i = tid; i < kP; i += nthreads) {
    const float v = i == 0 ? ld_param(P.a_pre, 0, P.param_bf16)
                  : i == 1 ? ld_param(P.a_post, 0, P.param_bf16)
                  : i == 2 ? ld_param(P.a_res, 0, P.param_bf16)
                           : ld_param(P.bias, i - 3, P.param_bf16);
    sm.par[i] = bf16r(v);
  }
  for (int i = tid; i < kNF * 16; i += nthreads)
    sm.perm[i] = bf16r(ld_param(P.perm, i, P.perm_bf16));
}

// Forward intermediates of one token.
struct Tok {
  float spre[4], spost[4];  // sigmoids (unrounded)
  float hpre[4], hpost[4];  // outputs
  float a[kNF];             // softmax
};

__device__ __forceinline__ void forward_token(const ParamSmem &sm, const float (&v)[32], Tok &k) {
  const float ap = sm.par[0], aq = sm.par[1], ar = sm.par[2];
  const float *b = sm.par + 3;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    k.spre[i] = sigm(ap * v[i] + b[i]);
    k.hpre[i] = k.spre[i];
    k.spost[i] = sigm(aq * v[4 + i] + b[4 + i]);
    k.hpost[i] = 2.f * k.spost[i];
  }
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < kNF; ++j) {
    k.a[j] = ar * v[8 + j] + b[8 + j];
    m = fmaxf(m, k.a[j]);
  }
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kNF; ++j) {
    k.a[j] = __expf(k.a[j] - m);
    s += k.a[j];
  }
  const float inv = 1.f / s;
#pragma unroll
  for (int j = 0; j < kNF; ++j) k.a[j] *= inv;
}

// h_pre, h_post (T, 4) and H_merged (T, 4, 4) of token t, in f32.  Returns the h_pre written.
__device__ __forceinline__ float4 store_coeffs(const ParamSmem &sm, const float (&v)[32],
                                             float4 *__restrict__ h_pre,
                                             float4 *__restrict__ h_post,
                                             float4 *__restrict__ H, int64_t t) {
  Tok k;
  forward_token(sm, v, k);
  float Hm[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    float acc = 0.f;  // softmax output times the permutation rows, f32 accumulate
#pragma unroll
    for (int j = 0; j < kNF; ++j) acc = fmaf(k.a[j], sm.perm[j * 16 + e], acc);
    Hm[e] = fmaf(-k.hpost[e >> 2], k.hpre[e & 3], acc);
  }
  const float4 hp = make_float4(k.hpre[0], k.hpre[1], k.hpre[2], k.hpre[3]);
  h_pre[t] = hp;
  h_post[t] = make_float4(k.hpost[0], k.hpost[1], k.hpost[2], k.hpost[3]);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    H[t * 4 + i] = make_float4(Hm[4 * i + 0], Hm[4 * i + 1], Hm[4 * i + 2], Hm[4 * i + 3]);
  return hp;
}

// Where a fused K1 forward writes the coefficients (all null: K1 only).
struct Out {
  float4 *h_pre, *h_post, *H;
};

}  // namespace k2tok
}  // namespace fmhc
