// K1 forward on the 5th-generation tensor cores.
//
//   inv_rms[t] = rsqrt(sum_k x[t,k]^2 / nC + 1e-6)
//   out[t,d]   = bf16( (sum_k x[t,k] W[d,k]) * inv_rms[t] )        (D = 32)
//
// (src/flash_mhc/kernels.py:250-303 of the reference.)  At ~32 FLOP/byte the
// projection needs ~210 TFLOP/s to keep up with HBM, beyond the CUDA cores, so
// the (T, nC) x (nC, 32) contraction runs as tcgen05.mma with the accumulator
// in TMEM while the sum of squares is taken by CUDA cores from the same
// shared-memory tiles.
//
// Persistent kernel, FMHC_K1F_CTAS_PER_SM resident CTAs per SM, 6 warps:
//   warp 0     TMA producer: x tile (<=128 rows x 64 k, four 32-row boxes,
//              128-byte swizzle) + W chunk (32 x 64) per pipeline stage;
//   warp 1     MMA issuer: 4 x tcgen05.mma M128 N32 K16 per stage into one of
//              two TMEM accumulators (64 columns allocated);
//   warps 2-5  one thread per tile row: sum of squares from shared memory,
//              then the epilogue (tcgen05.ld of the row's 32 f32 columns,
//              scale by inv_rms, bf16 store).  These threads read the stage
//              with ordinary (generic-proxy) loads while its refill is a TMA
//              (async-proxy) write, so each thread issues fence.proxy.async
//              before its release arrive; without it, loads still pending at
//              the arrive were seen returning the next fill's data.
// Each CTA owns a contiguous token range in 32-row units (balanced to within
// 32 rows across CTAs); partial tiles load only the 32-row boxes they need.
// Every mbarrier wait is bounded (sm100_ptx.cuh): on expiry the kernel records
// an error code, drains its copies and MMAs (bounded), frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>

#include "fmhc_common.cuh"
#include "k1_tc.h"
#include "k2_token.cuh"
#include "sm100_ptx.cuh"

namespace fmhc {
namespace k1tc {

using namespace sm100;

// A stage holds kColBoxes column boxes of 64 k (one 128-byte swizzled row
// each) for up to 128 rows, so every x row is read kColBoxes * 128 contiguous
// bytes at a time.
// Defaults measured at T=65536, nC=4096: two resident CTAs per SM, each with
// four 20 KiB stages, reach ~92% of the HBM copy bandwidth (one CTA with five
// 40 KiB stages: ~84%).
#ifndef FMHC_K1F_COLBOXES
#define FMHC_K1F_COLBOXES 1
#endif
#ifndef FMHC_K1F_STAGES
#define FMHC_K1F_STAGES 4
#endif
// Resident CTAs per SM (each with its own pipeline and token range).
#ifndef FMHC_K1F_CTAS_PER_SM
#define FMHC_K1F_CTAS_PER_SM 2
#endif
constexpr int kBM = 128;            // tile rows (MMA M)
constexpr int kColBoxes = FMHC_K1F_COLBOXES;
constexpr int kBK = 64 * kColBoxes; // k per stage
constexpr int kND = 32;             // projection width (MMA N)
constexpr int kBoxRows = 32;        // TMA box rows for x
constexpr int kStages = FMHC_K1F_STAGES;
constexpr int kColABytes = kBM * 64 * 2;       // 16 KiB: one column box, 128 rows
constexpr int kColBBytes = kND * 64 * 2;       // 4 KiB: one W column box
constexpr int kABytes = kColBoxes * kColABytes;
constexpr int kBBytes = kColBoxes * kColBBytes;
constexpr int kBoxBytes = kBoxRows * 64 * 2;   // 4 KiB: 32 rows of one column box
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 192;
constexpr int kRowThreads = 128;    // warps 2-5: sumsq + epilogue
constexpr uint32_t kTmemCols = 64;  // two 32-column accumulators
constexpr float kEps = 1e-6f;

struct alignas(1024) FwdSmem {
  uint8_t stage[kStages][kStageBytes];  // kColBoxes x 20 KiB each, 1 KiB aligned
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  k2tok::ParamSmem k2;  // K2 parameters (coefficient epilogue only)
};

// Error sites recorded in g_device_error.
enum : unsigned { kSiteProdEmpty = 0x101, kSiteMmaFull = 0x102, kSiteMmaTempty = 0x103,
                  kSiteEpiFull = 0x104, kSiteEpiTfull = 0x105, kSiteDrain = 0x106 };

// COEFFS: the epilogue also runs K2 on each token's stored (bf16) logits and
// writes h_pre, h_post and H_merged (k2_token.cuh), saving K2's launch and
// its read of proj.
// LOSE_COPY (test hook only, fmhc_debug_k1_fwd_lost_copy): CTA 0 arms its
// first stage's barrier for the copy's bytes but issues no copy, so the waits
// on that stage can only end by expiring.  This exercises the failure path:
// the first waiter to expire records its site code and raises the abort flag,
// the other roles leave their loops, the producer's drain wait on the same
// stage expires too (bounded), TMEM is freed and the CTA returns.  No copy is
// left in flight.  The production instantiations have LOSE_COPY = false.
template <bool COEFFS, bool LOSE_COPY = false>
__global__ void __launch_bounds__(kThreads, FMHC_K1F_CTAS_PER_SM)
k1_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmap_x,
                 const __grid_constant__ CUtensorMap tmap_w, __nv_bfloat16 *__restrict__ out,
                 float *__restrict__ inv_rms, int64_t T, int nC, int64_t units,
                 const K2Params P, const k2tok::Out co) {
  extern __shared__ uint8_t smem_raw[];
  FwdSmem &sm = *reinterpret_cast<FwdSmem *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int *abort = &sm.abort;

  // Contiguous token range of this CTA, in 32-row units.
  const int64_t u0 = int64_t(blockIdx.x) * units / gridDim.x;
  const int64_t u1 = int64_t(blockIdx.x + 1) * units / gridDim.x;
  const int64_t t_begin = u0 * kBoxRows;
  const int64_t t_end = (u1 * kBoxRows < T) ? u1 * kBoxRows : T;
  const int ntiles = t_end > t_begin ? int((t_end - t_begin + kBM - 1) / kBM) : 0;
  const int nk = nC / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&sm.full[s]), 1);
      // MMA commit + every row-warp thread: each thread fences and releases
      // its own shared-memory reads before the TMA may refill the stage.
      mbar_init(smem_u32(&sm.empty[s]), 1 + kRowThreads);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&sm.tfull[b]), 1);
      mbar_init(smem_u32(&sm.tempty[b]), 4);
    }
    mbar_init(smem_u32(&sm.mma_done), 1);
    sm.abort = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&sm.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  // No global memory is touched before this point (see pdl_wait()).
  pdl_wait();

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int tile = 0; tile < ntiles && !*abort; ++tile) {
        const int64_t row0 = t_begin + int64_t(tile) * kBM;
        const int64_t rows = (t_end - row0) < kBM ? (t_end - row0) : kBM;
        const int nbox = int((rows + kBoxRows - 1) / kBoxRows);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(smem_u32(&sm.empty[stage]), phase ^ 1, abort, kSiteProdEmpty)) break;
          const uint32_t full = smem_u32(&sm.full[stage]);
          mbar_arrive_expect_tx(full, uint32_t(kColBoxes * (nbox * kBoxBytes + kColBBytes)));
          const uint32_t a = smem_u32(sm.stage[stage]);
          const bool lose = LOSE_COPY && blockIdx.x == 0 && issued == 0;
          for (int cb = 0; cb < kColBoxes && !lose; ++cb) {
            const int32_t k0 = kb * kBK + cb * 64;
            for (int b = 0; b < nbox; ++b)
              tma_load_2d(a + cb * kColABytes + b * kBoxBytes, &tmap_x, full, k0,
                          int32_t(row0 + b * kBoxRows));
            tma_load_2d(a + kABytes + cb * kColBBytes, &tmap_w, full, k0, 0);
          }
          ++issued;
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: the last min(issued, kStages) loads must have landed before exit.
      int n = issued < kStages ? issued : kStages;
      int s = stage;
      uint32_t ph = phase;
      for (int i = 0; i < n; ++i) {
        if (--s < 0) { s = kStages - 1; ph ^= 1; }
        mbar_wait(smem_u32(&sm.full[s]), ph, abort, kSiteDrain, true);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kBM, kND, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = 0; tile < ntiles && !*abort; ++tile) {
        if (!mbar_wait(smem_u32(&sm.tempty[acc]), acc_phase ^ 1, abort, kSiteMmaTempty)) break;
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(acc * kND);
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(smem_u32(&sm.full[stage]), phase, abort, kSiteMmaFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = smem_u32(sm.stage[stage]);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const int cb = k / 4, kk = k % 4;
            const uint64_t ad = smem_desc(a + cb * kColABytes + kk * 32, 16, 1024, 2);
            const uint64_t bd = smem_desc(a + kABytes + cb * kColBBytes + kk * 32, 16, 1024, 2);
            mma_bf16_ss(d, ad, bd, idesc, (kb | k) != 0);
          }
          mma_commit(smem_u32(&sm.empty[stage]));
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit(smem_u32(&sm.tfull[acc]));
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      // All MMAs issued by this thread complete before TMEM is freed.
      mma_commit(smem_u32(&sm.mma_done));
      mbar_wait(smem_u32(&sm.mma_done), 0, abort, kSiteDrain, true);
    }
  } else {
    // ------------------------------------------ row warps: sumsq + epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int r = q * 32 + lane;
    if constexpr (COEFFS) {
      k2tok::stage_params(sm.k2, P, int(threadIdx.x) - 64, kRowThreads);
      named_bar_sync(1, kRowThreads);
    }
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = 0; tile < ntiles && !*abort; ++tile) {
      const int64_t row0 = t_begin + int64_t(tile) * kBM;
      const int64_t rows = (t_end - row0) < kBM ? (t_end - row0) : kBM;
      // Eight independent partial sums (one per bf16 lane of a 16-byte chunk)
      // keep the FMA pipe busy instead of one serial chain per thread.
      float ss8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        if (!mbar_wait(smem_u32(&sm.full[stage]), phase, abort, kSiteEpiFull)) { ok = false; break; }
#pragma unroll
        for (int cb = 0; cb < kColBoxes; ++cb) {
          const uint8_t *row = sm.stage[stage] + cb * kColABytes + r * 128;
          uint4 u[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)  // rotate by r: the 8 rows of a swizzle atom hit distinct banks
            u[i] = *reinterpret_cast<const uint4 *>(row + (((i + r) & 7) << 4));
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float f;
            f = bf16lo(u[i].x); ss8[0] = fmaf(f, f, ss8[0]); f = bf16hi(u[i].x); ss8[1] = fmaf(f, f, ss8[1]);
            f = bf16lo(u[i].y); ss8[2] = fmaf(f, f, ss8[2]); f = bf16hi(u[i].y); ss8[3] = fmaf(f, f, ss8[3]);
            f = bf16lo(u[i].z); ss8[4] = fmaf(f, f, ss8[4]); f = bf16hi(u[i].z); ss8[5] = fmaf(f, f, ss8[5]);
            f = bf16lo(u[i].w); ss8[6] = fmaf(f, f, ss8[6]); f = bf16hi(u[i].w); ss8[7] = fmaf(f, f, ss8[7]);
          }
        }
        // The refill is a TMA (async-proxy) write: order this thread's
        // generic-proxy reads of the stage before it, then release.
        fence_proxy_async_smem();
        mbar_arrive(smem_u32(&sm.empty[stage]));
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      if (!mbar_wait(smem_u32(&sm.tfull[acc]), acc_phase, abort, kSiteEpiTfull)) break;
      tc_fence_after();
      uint32_t v[32];
      tmem_ld_32x32b_x32(tmem + (uint32_t(q * 32) << 16) + uint32_t(acc * kND), v);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sm.tempty[acc]));
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      if (r < rows) {
        const int64_t t = row0 + r;
        const float ss = ((ss8[0] + ss8[1]) + (ss8[2] + ss8[3])) + ((ss8[4] + ss8[5]) + (ss8[6] + ss8[7]));
        const float inv = rsqrtf(ss / float(nC) + kEps);
        uint4 *o = reinterpret_cast<uint4 *>(out + t * kND);
        float pv[32];  // the stored bf16 logits, for the coefficient epilogue
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(v[8 * c + 0]) * inv, __uint_as_float(v[8 * c + 1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(v[8 * c + 2]) * inv, __uint_as_float(v[8 * c + 3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(v[8 * c + 4]) * inv, __uint_as_float(v[8 * c + 5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(v[8 * c + 6]) * inv, __uint_as_float(v[8 * c + 7]) * inv);
          __stcs(o + c, w);
          pv[8 * c + 0] = bf16lo(w.x); pv[8 * c + 1] = bf16hi(w.x);
          pv[8 * c + 2] = bf16lo(w.y); pv[8 * c + 3] = bf16hi(w.y);
          pv[8 * c + 4] = bf16lo(w.z); pv[8 * c + 5] = bf16hi(w.z);
          pv[8 * c + 6] = bf16lo(w.w); pv[8 * c + 7] = bf16hi(w.w);
        }
        __stcs(inv_rms + t, inv);
        if constexpr (COEFFS) k2tok::store_coeffs(sm.k2, pv, co.h_pre, co.h_post, co.H, t);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// K1 forward, split-K over a thread-block cluster (a few thousand tokens).
//
// With few token tiles, each CTA of the persistent kernel above walks all
// nC / 64 k-steps of a small tile one after another and the launch is
// latency-bound (~29 us at T = 8192, nC = 4096).  Here a cluster of S CTAs
// (S = 2 or 4) takes one 128-row tile; CTA r of the cluster runs the k-steps
// [r nk / S, (r + 1) nk / S) with the same pipeline (TMA producer, tcgen05
// MMA into TMEM, row warps taking the sum of squares from the stages).  The S
// partials of each row (32 projections and the sum of squares) are then added
// up a binary tree through distributed shared memory, in a fixed order:
// first level, rank r + 1 -> rank r for even r; second level (S = 4), rank 2 -> rank 0,
// so rank 0 holds (p0 + p1) + (p2 + p3).  A sender's row threads store their
// 33 values into the receiver's buffer for that level and arrive (release,
// cluster scope) on the receiver's mbarrier; the receiver waits (bounded,
// acquire) and adds.  Senders then exit: no CTA reads another's buffer after
// its owner may have left.  Rank 0 finishes: inv_rms = rsqrt(ss / nC + eps),
// out = bf16(proj * inv_rms).  Nothing here addresses another GPU.
//
// Pipeline depth ST: with at most one CTA per SM (clusters x S <= SMs) each
// CTA streams its k-steps through kSkStagesDeep stages (160 KiB in flight:
// the k-loop is bound by the TMA round trip, not by bandwidth); with more CTAs
// two share an SM and each gets kSkStagesShallow.
constexpr int kSkStagesShallow = 3;
constexpr int kSkStagesDeep = 8;
constexpr int kSkRows = 128;
template <int ST>
struct alignas(1024) SkSmem {
  uint8_t stage[ST][kStageBytes];
  float recv[2][kSkRows][33];  // partials received at the first and second level
  uint64_t full[ST];
  uint64_t empty[ST];
  uint64_t tfull;
  uint64_t rfull[2];           // 128 remote arrivals (one per sender row thread)
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  k2tok::ParamSmem k2;         // K2 parameters (coefficient epilogue, rank 0 only)
};

enum : unsigned { kSiteSkProdEmpty = 0x111, kSiteSkMmaFull = 0x112, kSiteSkRowFull = 0x113,
                  kSiteSkTfull = 0x114, kSiteSkRecv = 0x115, kSiteSkDrain = 0x116 };

template <int ST>
__device__ __forceinline__ void sk_send(SkSmem<ST> &sm, const float (&acc)[33], int r, int slot,
                                        uint32_t dst) {
  const uint32_t base = mapa_shared(smem_u32(&sm.recv[slot][r][0]), dst);
#pragma unroll
  for (int j = 0; j < 33; ++j) st_cluster_f32(base + 4 * j, acc[j]);
  mbar_arrive_remote(mapa_shared(smem_u32(&sm.rfull[slot]), dst));
}

// COEFFS: as in k1_fwd_tc_kernel, rank 0's epilogue also runs K2.
template <bool COEFFS, int ST>
__global__ void __launch_bounds__(kThreads, FMHC_K1F_CTAS_PER_SM)
k1_fwd_tc_splitk_kernel(const __grid_constant__ CUtensorMap tmap_x,
                        const __grid_constant__ CUtensorMap tmap_w,
                        __nv_bfloat16 *__restrict__ out, float *__restrict__ inv_rms, int64_t T,
                        int nC, int S, const K2Params P, const k2tok::Out co) {
  extern __shared__ uint8_t smem_raw[];
  SkSmem<ST> &sm = *reinterpret_cast<SkSmem<ST> *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int *abort = &sm.abort;
  const uint32_t rank = cluster_ctarank();
  const int64_t row0 = int64_t(blockIdx.x / S) * kSkRows;
  const int64_t rows = (T - row0) < kSkRows ? (T - row0) : kSkRows;
  const int nbox = int((rows + kBoxRows - 1) / kBoxRows);
  const int nk = nC / kBK;
  const int kb0 = int(rank) * nk / S, kb1 = (int(rank) + 1) * nk / S;

  if (threadIdx.x == 0) {
    for (int st = 0; st < ST; ++st) {
      mbar_init(smem_u32(&sm.full[st]), 1);
      mbar_init(smem_u32(&sm.empty[st]), 1 + kRowThreads);
    }
    mbar_init(smem_u32(&sm.tfull), 1);
    mbar_init(smem_u32(&sm.rfull[0]), kRowThreads);
    mbar_init(smem_u32(&sm.rfull[1]), kRowThreads);
    mbar_init(smem_u32(&sm.mma_done), 1);
    sm.abort = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&sm.tmem_base), 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Every CTA's barriers exist before any peer arrives on them.
  cluster_sync_all();
  const uint32_t tmem = sm.tmem_base;
  // No global memory is touched before this point (see pdl_wait()).
  pdl_wait();

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1 && !*abort; ++kb) {
        if (!mbar_wait(smem_u32(&sm.empty[stage]), phase ^ 1, abort, kSiteSkProdEmpty)) break;
        const uint32_t full = smem_u32(&sm.full[stage]);
        mbar_arrive_expect_tx(full, uint32_t(kColBoxes * (nbox * kBoxBytes + kColBBytes)));
        const uint32_t a = smem_u32(sm.stage[stage]);
        for (int cb = 0; cb < kColBoxes; ++cb) {
          const int32_t k0 = kb * kBK + cb * 64;
          for (int b = 0; b < nbox; ++b)
            tma_load_2d(a + cb * kColABytes + b * kBoxBytes, &tmap_x, full, k0,
                        int32_t(row0 + b * kBoxRows));
          tma_load_2d(a + kABytes + cb * kColBBytes, &tmap_w, full, k0, 0);
        }
        ++issued;
        if (++stage == ST) { stage = 0; phase ^= 1; }
      }
      int n = issued < ST ? issued : ST;
      int st = stage;
      uint32_t ph = phase;
      for (int i = 0; i < n; ++i) {
        if (--st < 0) { st = ST - 1; ph ^= 1; }
        mbar_wait(smem_u32(&sm.full[st]), ph, abort, kSiteSkDrain, true);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kBM, kND, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(smem_u32(&sm.full[stage]), phase, abort, kSiteSkMmaFull)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a = smem_u32(sm.stage[stage]);
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          const int cb = k / 4, kk = k % 4;
          const uint64_t ad = smem_desc(a + cb * kColABytes + kk * 32, 16, 1024, 2);
          const uint64_t bd = smem_desc(a + kABytes + cb * kColBBytes + kk * 32, 16, 1024, 2);
          mma_bf16_ss(tmem, ad, bd, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
        }
        mma_commit(smem_u32(&sm.empty[stage]));
        if (++stage == ST) { stage = 0; phase ^= 1; }
      }
      if (ok) mma_commit(smem_u32(&sm.tfull));
      mma_commit(smem_u32(&sm.mma_done));
      mbar_wait(smem_u32(&sm.mma_done), 0, abort, kSiteSkDrain, true);
    }
  } else {
    // ---------------------------------- row warps: sumsq, partial, tree
    const int q = warp & 3;
    const int r = q * 32 + lane;
    if constexpr (COEFFS) {
      if (rank == 0) {
        k2tok::stage_params(sm.k2, P, int(threadIdx.x) - 64, kRowThreads);
        named_bar_sync(1, kRowThreads);
      }
    }
    int stage = 0;
    uint32_t phase = 0;
    float ss8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    bool ok = true;
    for (int kb = kb0; kb < kb1; ++kb) {
      if (!mbar_wait(smem_u32(&sm.full[stage]), phase, abort, kSiteSkRowFull)) { ok = false; break; }
#pragma unroll
      for (int cb = 0; cb < kColBoxes; ++cb) {
        const uint8_t *row = sm.stage[stage] + cb * kColABytes + r * 128;
        uint4 u[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) u[i] = *reinterpret_cast<const uint4 *>(row + (((i + r) & 7) << 4));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float f;
          f = bf16lo(u[i].x); ss8[0] = fmaf(f, f, ss8[0]); f = bf16hi(u[i].x); ss8[1] = fmaf(f, f, ss8[1]);
          f = bf16lo(u[i].y); ss8[2] = fmaf(f, f, ss8[2]); f = bf16hi(u[i].y); ss8[3] = fmaf(f, f, ss8[3]);
          f = bf16lo(u[i].z); ss8[4] = fmaf(f, f, ss8[4]); f = bf16hi(u[i].z); ss8[5] = fmaf(f, f, ss8[5]);
          f = bf16lo(u[i].w); ss8[6] = fmaf(f, f, ss8[6]); f = bf16hi(u[i].w); ss8[7] = fmaf(f, f, ss8[7]);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(smem_u32(&sm.empty[stage]));
      if (++stage == ST) { stage = 0; phase ^= 1; }
    }
    if (ok && mbar_wait(smem_u32(&sm.tfull), 0, abort, kSiteSkTfull)) {
      tc_fence_after();
      uint32_t v[32];
      tmem_ld_32x32b_x32(tmem + (uint32_t(q * 32) << 16), v);
      tmem_wait_ld();
      float acc[33];
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] = __uint_as_float(v[j]);
      acc[32] = ((ss8[0] + ss8[1]) + (ss8[2] + ss8[3])) + ((ss8[4] + ss8[5]) + (ss8[6] + ss8[7]));
      bool done = false;
      // First level: odd ranks send to rank - 1.
      if (rank & 1u) {
        sk_send(sm, acc, r, 0, rank - 1);
        done = true;
      } else if (mbar_wait_cluster(smem_u32(&sm.rfull[0]), 0, abort, kSiteSkRecv)) {
#pragma unroll
        for (int j = 0; j < 33; ++j) acc[j] += sm.recv[0][r][j];
      } else {
        done = true;
      }
      // Second level (S = 4): rank 2 sends to rank 0.
      if (!done && S == 4) {
        if (rank == 2) {
          sk_send(sm, acc, r, 1, 0);
          done = true;
        } else if (mbar_wait_cluster(smem_u32(&sm.rfull[1]), 0, abort, kSiteSkRecv)) {
#pragma unroll
          for (int j = 0; j < 33; ++j) acc[j] += sm.recv[1][r][j];
        } else {
          done = true;
        }
      }
      if (!done && rank == 0 && r < rows) {
        const int64_t t = row0 + r;
        const float inv = rsqrtf(acc[32] / float(nC) + kEps);
        uint4 *o = reinterpret_cast<uint4 *>(out + t * kND);
        float pv[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint4 w;
          w.x = pack_bf16x2(acc[8 * c + 0] * inv, acc[8 * c + 1] * inv);
          w.y = pack_bf16x2(acc[8 * c + 2] * inv, acc[8 * c + 3] * inv);
          w.z = pack_bf16x2(acc[8 * c + 4] * inv, acc[8 * c + 5] * inv);
          w.w = pack_bf16x2(acc[8 * c + 6] * inv, acc[8 * c + 7] * inv);
          __stcs(o + c, w);
          pv[8 * c + 0] = bf16lo(w.x); pv[8 * c + 1] = bf16hi(w.x);
          pv[8 * c + 2] = bf16lo(w.y); pv[8 * c + 3] = bf16hi(w.y);
          pv[8 * c + 4] = bf16lo(w.z); pv[8 * c + 5] = bf16hi(w.z);
          pv[8 * c + 6] = bf16lo(w.w); pv[8 * c + 7] = bf16hi(w.w);
        }
        __stcs(inv_rms + t, inv);
        if constexpr (COEFFS) k2tok::store_coeffs(sm.k2, pv, co.h_pre, co.h_post, co.H, t);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

// ---------------------------------------------------------------------------
// K1 forward for very few tokens, split over a thread-block cluster.
//
// With T <= 2 x (SMs / 2) tokens the one-block-per-2-tokens CUDA-core kernel
// (k1_simt.cu) leaves most SMs idle and each block walks all of W (nC x 32
// bf16) itself.  Here the 2-token pair gets a cluster of S CTAs (S = 8, 4 or
// 2, the largest that keeps the grid within one wave); CTA r of the cluster
// takes the 16-byte chunks [r nch / S, (r + 1) nch / S) of the row.  Inside a
// CTA the four warp pairs split W's 32 rows into groups of 8 (warps 2g, 2g+1
// take rows 8g .. 8g+7) and the 64 threads of a pair walk the chunks, so a
// thread issues its x load and 8 W loads in one batch.  Per value a warp
// butterfly, then the two warps of a group are added in warp order; the
// CTA's 66 partials (2 tokens x (32 projections + sum of squares)) go to rank 0
// through distributed shared memory (st.shared::cluster, then an arrive with
// release at cluster scope on rank 0's mbarrier), and rank 0 adds them in
// rank order after a bounded wait.  Rank 0 then writes proj and inv_rms and,
// as k1_fwd_rows_kernel, runs K2 (COEFFS) and K3 (PRE) for its tokens.  The
// other ranks exit after sending; rank 0 never touches their memory.  Only the
// barrier set-up uses the cluster-wide hardware barrier.  Same preconditions
// as the CUDA-core small-T kernel: D == 32, nC % 8 == 0, x and W 16-byte
// aligned (PRE: nC % 32 == 0 and 16-byte aligned pre_out).
constexpr int kRcTokens = 2;
constexpr int kRcThreads = 256;
constexpr int kRcMaxS = 8;
constexpr int kRcVals = kRcTokens * 33;
enum : unsigned { kSiteRcRecv = 0x121 };

template <bool COEFFS, bool PRE>
__global__ void __launch_bounds__(kRcThreads, 1)
k1_fwd_rows_cluster_kernel(const __nv_bfloat16 *__restrict__ x, const __nv_bfloat16 *__restrict__ W,
                           __nv_bfloat16 *__restrict__ out, float *__restrict__ inv_rms, int64_t T,
                           int nC, int S, const K2Params P, const k2tok::Out co,
                           __nv_bfloat16 *__restrict__ pre_out) {
  static_assert(COEFFS || !PRE, "K3 needs the coefficients");
  __shared__ float red[8][kRcTokens][9];
  __shared__ float recv[kRcMaxS][kRcVals];  // rank 0: slot r holds rank r's partials
  __shared__ float tot[kRcTokens][33];
  __shared__ alignas(8) uint64_t rfull;
  __shared__ k2tok::ParamSmem k2s;
  __shared__ float4 hs[kRcTokens];
  __shared__ int abort_flag;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t rank = cluster_ctarank();
  if (tid == 0) {
    if (rank == 0) mbar_init(smem_u32(&rfull), uint32_t(S - 1) * kRcVals);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // rank 0's barrier exists before any peer arrives on it
  cluster_sync_all();
  // No global memory is touched before this point (see pdl_wait()).
  pdl_wait();
  if (COEFFS && rank == 0) k2tok::stage_params(k2s, P, tid, kRcThreads);

  const int64_t t0 = int64_t(blockIdx.x / S) * kRcTokens;
  const bool has1 = t0 + 1 < T;
  const int nch = nC >> 3;
  const int c0 = int(rank) * nch / S, c1 = (int(rank) + 1) * nch / S;
  const int g = warp >> 1;    // W rows 8g .. 8g+7
  const int j = tid & 63;     // thread within the warp pair
  float acc0[8], acc1[8], ss0 = 0.f, ss1 = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) acc0[i] = acc1[i] = 0.f;
  for (int c = c0 + j; c < c1; c += 64) {
    const uint4 u0 = __ldg(reinterpret_cast<const uint4 *>(x + t0 * nC + c * 8));
    uint4 u1 = make_uint4(0u, 0u, 0u, 0u);
    if (has1) u1 = __ldg(reinterpret_cast<const uint4 *>(x + (t0 + 1) * nC + c * 8));
    uint4 wv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      wv[i] = __ldg(reinterpret_cast<const uint4 *>(W + int64_t(8 * g + i) * nC + c * 8));
    const float f0[8] = {bf16lo(u0.x), bf16hi(u0.x), bf16lo(u0.y), bf16hi(u0.y),
                         bf16lo(u0.z), bf16hi(u0.z), bf16lo(u0.w), bf16hi(u0.w)};
    const float f1[8] = {bf16lo(u1.x), bf16hi(u1.x), bf16lo(u1.y), bf16hi(u1.y),
                         bf16lo(u1.z), bf16hi(u1.z), bf16lo(u1.w), bf16hi(u1.w)};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      ss0 = fmaf(f0[e], f0[e], ss0);
      ss1 = fmaf(f1[e], f1[e], ss1);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 u = wv[i];
      const float fw[8] = {bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y),
                           bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w)};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        acc0[i] = fmaf(f0[e], fw[e], acc0[i]);
        acc1[i] = fmaf(f1[e], fw[e], acc1[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      acc0[i] += __shfl_xor_sync(0xffffffffu, acc0[i], off);
      acc1[i] += __shfl_xor_sync(0xffffffffu, acc1[i], off);
    }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    ss0 += __shfl_xor_sync(0xffffffffu, ss0, off);
    ss1 += __shfl_xor_sync(0xffffffffu, ss1, off);
  }
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      red[warp][0][i] = acc0[i];
      red[warp][1][i] = acc1[i];
    }
    red[warp][0][8] = ss0;  // every group sums the squares; group 0's are used
    red[warp][1][8] = ss1;
  }
  __syncthreads();
  if (tid < kRcVals) {
    const int tb = tid / 33, d = tid - tb * 33;
    const int gg = d < 32 ? d >> 3 : 0, i = d < 32 ? d & 7 : 8;
    const float v = red[2 * gg][tb][i] + red[2 * gg + 1][tb][i];
    if (rank != 0) {
      st_cluster_f32(mapa_shared(smem_u32(&recv[rank][tid]), 0), v);
      mbar_arrive_remote(mapa_shared(smem_u32(&rfull), 0));
    } else {
      recv[0][tid] = v;
    }
  }
  if (rank != 0) return;
  __syncthreads();
  if (tid < kRcVals) {
    if (S == 1 || mbar_wait_cluster(smem_u32(&rfull), 0, &abort_flag, kSiteRcRecv)) {
      float v = recv[0][tid];
      for (int r = 1; r < S; ++r) v += recv[r][tid];
      tot[tid / 33][tid % 33] = v;
    }
  }
  __syncthreads();
  if (abort_flag) return;
  if (tid < kRcTokens * 32) {
    const int tb = tid / 32, d = tid - tb * 32;
    const int64_t t = t0 + tb;
    if (t < T) {
      const float r = rsqrtf(tot[tb][32] / float(nC) + kEps);
      out[t * 32 + d] = __float2bfloat16_rn(tot[tb][d] * r);
      if (d == 0) inv_rms[t] = r;
    }
  }
  if constexpr (COEFFS) {
    if (tid < kRcTokens && t0 + tid < T) {
      const int64_t t = t0 + tid;
      const float r = rsqrtf(tot[tid][32] / float(nC) + kEps);
      float pv[32];  // the logits as stored above (bf16)
#pragma unroll
      for (int d = 0; d < 32; ++d) pv[d] = __bfloat162float(__float2bfloat16_rn(tot[tid][d] * r));
      hs[tid] = k2tok::store_coeffs(k2s, pv, co.h_pre, co.h_post, co.H, t);
    }
  }
  if constexpr (PRE) {
    __syncthreads();
    const int C = nC >> 2, n3 = C >> 3;
    for (int it = tid; it < kRcTokens * n3; it += kRcThreads) {
      const int tb = it / n3, c = it - tb * n3;
      const int64_t t = t0 + tb;
      if (t >= T) continue;
      const float4 h = hs[tb];
      const __nv_bfloat16 *xr = x + t * nC;
      Chunk<8> a0, a1, a2, a3;
      a0.v = __ldg(reinterpret_cast<const uint4 *>(xr + c * 8));
      a1.v = __ldg(reinterpret_cast<const uint4 *>(xr + C + c * 8));
      a2.v = __ldg(reinterpret_cast<const uint4 *>(xr + 2 * C + c * 8));
      a3.v = __ldg(reinterpret_cast<const uint4 *>(xr + 3 * C + c * 8));
      float f0[8], f1[8], f2[8], f3[8], o[8];
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

}  // namespace k1tc
}  // namespace fmhc

#include "k1_tc_bwd.cuh"

namespace fmhc {
namespace k1tc {

// ------------------------------------------------------------------- host side
namespace {

thread_local char g_msg[256] = "";

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D bf16 tensor map: inner dimension `inner` (contiguous), `outer` rows of
// `row_bytes` stride, box inner x outer_box, 128-byte swizzle, zero fill.
bool make_map(CUtensorMap *m, const void *base, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int device_sms() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

// Opt in to the kernel's dynamic shared memory once per (kernel, device) for
// the whole process (not per thread: autograd runs backward ops on its own
// threads, and a first-time attribute call must not land inside a CUDA-graph
// capture made on another thread).
int set_smem_attr(const void *kernel, size_t bytes) {
  static std::mutex mu;
  static const void *done_kernel[8][16] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 16) dev = 15;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < 8; ++i) {
    if (done_kernel[i][dev] == kernel) return 0;
    if (done_kernel[i][dev] == nullptr) {
      if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes)) !=
          cudaSuccess) {
        snprintf(g_msg, sizeof(g_msg), "cudaFuncSetAttribute(smem=%zu) failed", bytes);
        return 5;
      }
      done_kernel[i][dev] = kernel;
      return 0;
    }
  }
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes)) ==
                 cudaSuccess ? 0 : 5;
}

bool device_is_sm100() {
  int dev = 0, major = 0, minor = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return major == 10 && minor == 0;
}

}  // namespace
}  // namespace k1tc

const char *k1_tc_error() { return k1tc::g_msg; }

static_assert(sizeof(k1tc::BwdSmem) + 1024 <= 232448, "K1 backward shared memory");
static_assert((sizeof(k1tc::FwdSmem) + 1024) * FMHC_K1F_CTAS_PER_SM <= 232448,
              "K1 forward shared memory");
static_assert((sizeof(k1tc::SkSmem<k1tc::kSkStagesShallow>) + 1024) * FMHC_K1F_CTAS_PER_SM <= 232448,
              "split-K K1 forward shared memory");
static_assert(sizeof(k1tc::SkSmem<k1tc::kSkStagesDeep>) + 1024 <= 232448,
              "split-K K1 forward shared memory (one CTA per SM)");

int launch_k1_fwd_rows_cluster(const void *x, const void *W, void *out, float *inv_rms, int64_t T,
                               int nC, cudaStream_t s, const K2Params *coeffs, float *h_pre,
                               float *h_post, float *H, void *pre_out) {
  using namespace k1tc;
#ifndef FMHC_K1F_ROWS_CLUSTER  // 0 keeps the one-block-per-2-tokens kernel (A/B measurements)
#define FMHC_K1F_ROWS_CLUSTER 1
#endif
  if (!FMHC_K1F_ROWS_CLUSTER || T < 1 || !device_is_sm100()) return -1;
  const int64_t pairs = (T + kRcTokens - 1) / kRcTokens;
  const int64_t sms = device_sms();
  int S = 0;
  for (int c : {8, 4, 2})
    if (pairs * c <= sms) { S = c; break; }
  if (S == 0) return -1;
  const K2Params P = coeffs ? *coeffs : K2Params{};
  const k2tok::Out co{reinterpret_cast<float4 *>(h_pre), reinterpret_cast<float4 *>(h_post),
                      reinterpret_cast<float4 *>(H)};
  auto kern = !coeffs ? k1_fwd_rows_cluster_kernel<false, false>
            : pre_out ? k1_fwd_rows_cluster_kernel<true, true>
                      : k1_fwd_rows_cluster_kernel<true, false>;
  if (launch_cluster(kern, dim3(unsigned(pairs * S)), dim3(kRcThreads), 0, s, unsigned(S),
                     reinterpret_cast<const __nv_bfloat16 *>(x),
                     reinterpret_cast<const __nv_bfloat16 *>(W),
                     reinterpret_cast<__nv_bfloat16 *>(out), inv_rms, T, nC, S, P, co,
                     reinterpret_cast<__nv_bfloat16 *>(pre_out)) != cudaSuccess) {
    snprintf(g_msg, sizeof(g_msg), "cluster launch of the small-T K1 forward failed");
    return 4;
  }
  return 0;
}

bool k1_tc_fwd_supported(const void *x, const void *W, const void *out, const float *inv_rms,
                         int64_t T, int64_t nC, int64_t D) {
  if (D != k1tc::kND || nC % k1tc::kBK != 0 || T < 1 || T > (int64_t(1) << 31)) return false;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(W)) & 15) return false;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(inv_rms) & 3))
    return false;
  return k1tc::device_is_sm100() && k1tc::encode_fn() != nullptr;
}

int launch_k1_tc_fwd(const void *x, const void *W, void *out, float *inv_rms, int64_t T, int nC,
                     cudaStream_t s, const K2Params *coeffs, float *h_pre, float *h_post,
                     float *H) {
  using namespace k1tc;
  const K2Params P = coeffs ? *coeffs : K2Params{};
  const k2tok::Out co{reinterpret_cast<float4 *>(h_pre), reinterpret_cast<float4 *>(h_post),
                      reinterpret_cast<float4 *>(H)};
  // Few 128-row tiles: split k over clusters of S CTAs.  Measured (profiler
  // kernel times, nC = 4096; nC = 3072 alike): S = 4 while the clusters fit
  // one CTA per SM (T <= 4736: 24 -> 18.6 us at T = 1024..4096); S = 2 while
  // they fill at most 3/4 of the two-CTA-per-SM slots (T <= 14208: 31.5 ->
  // 22.0 us at T = 8192; S = 4 there, two CTAs per SM, 28.1 us); beyond that
  // the persistent kernel (S = 2 at T = 16384: 34.1 against 33.6 us).
  {
    const int64_t tiles = (T + kSkRows - 1) / kSkRows;
    const int64_t sms = device_sms();
    const int64_t slots = sms * FMHC_K1F_CTAS_PER_SM;
    const int nk = nC / kBK;
    int S = 0;
#ifndef FMHC_K1F_SPLITK  // 0 disables the split-K path (A/B measurements)
#define FMHC_K1F_SPLITK 1
#endif
#ifndef FMHC_K1F_SK_DEEP  // 0 keeps the shallow pipeline everywhere (A/B measurements)
#define FMHC_K1F_SK_DEEP 1
#endif
    if (FMHC_K1F_SPLITK && tiles * 4 <= sms && nk >= 8) S = 4;
    else if (FMHC_K1F_SPLITK && tiles * 2 * 4 <= slots * 3 && nk >= 4) S = 2;
    if (S) {
      CUtensorMap mx, mw;
      if (!make_map(&mx, x, uint64_t(nC), uint64_t(T), uint64_t(nC) * 2, 64, kBoxRows,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
          !make_map(&mw, W, uint64_t(nC), kND, uint64_t(nC) * 2, 64, kND,
                    CU_TENSOR_MAP_SWIZZLE_128B)) {
        snprintf(g_msg, sizeof(g_msg), "cuTensorMapEncodeTiled failed");
        return 5;
      }
      // One CTA per SM when the clusters fit: the deep pipeline.
      const bool deep = tiles * S <= sms && FMHC_K1F_SK_DEEP;
      const size_t smem = (deep ? sizeof(SkSmem<kSkStagesDeep>) : sizeof(SkSmem<kSkStagesShallow>)) + 1024;
      auto kern = deep ? (coeffs ? k1_fwd_tc_splitk_kernel<true, kSkStagesDeep>
                                 : k1_fwd_tc_splitk_kernel<false, kSkStagesDeep>)
                       : (coeffs ? k1_fwd_tc_splitk_kernel<true, kSkStagesShallow>
                                 : k1_fwd_tc_splitk_kernel<false, kSkStagesShallow>);
      if (int e = set_smem_attr(reinterpret_cast<const void *>(kern), smem)) return e;
      if (launch_cluster(kern, dim3(unsigned(tiles * S)), dim3(kThreads), smem, s, unsigned(S), mx,
                         mw, reinterpret_cast<__nv_bfloat16 *>(out), inv_rms, T, nC, S, P,
                         co) != cudaSuccess) {
        snprintf(g_msg, sizeof(g_msg), "cluster launch of the split-K K1 forward failed");
        return 4;
      }
      return 0;
    }
  }
  CUtensorMap mx, mw;
  if (!make_map(&mx, x, uint64_t(nC), uint64_t(T), uint64_t(nC) * 2, 64, kBoxRows,
                CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mw, W, uint64_t(nC), kND, uint64_t(nC) * 2, 64, kND,
                CU_TENSOR_MAP_SWIZZLE_128B)) {
    snprintf(g_msg, sizeof(g_msg), "cuTensorMapEncodeTiled failed");
    return 5;
  }
  const int64_t units = (T + kBoxRows - 1) / kBoxRows;
  int64_t grid = int64_t(device_sms()) * FMHC_K1F_CTAS_PER_SM;
  if (grid > units) grid = units;
  const size_t smem = sizeof(FwdSmem) + 1024;
  auto kern = coeffs ? k1_fwd_tc_kernel<true> : k1_fwd_tc_kernel<false>;
  if (int e = set_smem_attr(reinterpret_cast<const void *>(kern), smem)) return e;
  launch(kern, dim3(unsigned(grid)), dim3(kThreads), smem, s, mx, mw,
         reinterpret_cast<__nv_bfloat16 *>(out), inv_rms, T, nC, units, P, co);
  return 0;
}

// ---------------------------------------------------------------- K1 backward
namespace k1tc {
namespace {

struct BwdPlan {
  int ntt, nkc, G, ngroups, grid, base, rem;
  int64_t part_bytes;
};

int64_t round256(int64_t b) { return (b + 255) & ~int64_t(255); }

// Work split of the backward kernel (see k1_tc_bwd.cuh): the nkc k-chunks form
// nkc / G groups, the grid's CTAs are spread over the groups as evenly as
// possible (the first `rem` groups get base + 1 CTAs, the rest base), and CTA
// i of a group of ng takes the token tiles i, i + ng, ...  G (a divisor of
// nkc, at most 8) minimises an estimate of the kernel time fitted to
// measurements at nC = 4096 (T = 8192 and 65536, G = 2, 4, 8):
//   1.56 us per unit of the busiest CTA (64 KiB of HBM traffic)
// + 0.28 us per token tile of the busiest CTA (slot load and tile prep)
// + the grad_W partials, G x 16 KiB per CTA written and read back, at 6 TB/s.
// Large T favours G = 8 (fewest tile switches); small T, where the partials
// weigh more, favours smaller G.
BwdPlan bwd_plan(int64_t T, int64_t nC) {
  BwdPlan p{};
  p.ntt = int((T + kBwdBT - 1) / kBwdBT);
  p.nkc = int(nC / kBwdBK);
  const int sms = device_sms();
  double best_cost = -1.0;
  for (int G = kBwdMaxG; G >= 1; G >>= 1) {
    if (p.nkc % G) continue;
    const int ngroups = p.nkc / G;
    int64_t grid = int64_t(ngroups) * p.ntt;
    if (grid > sms) grid = sms;
    if (grid < ngroups) continue;  // every group needs a CTA
    const int base = int(grid / ngroups);
    const int64_t tiles = (p.ntt + base - 1) / base;
    const double part_us = double(grid) * G * kND * kBwdBK * 4 * 2 / 6.0e6;
    const double cost = 1.56 * double(G * tiles) + 0.28 * double(tiles) + part_us;
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      p.G = G;
      p.ngroups = ngroups;
      p.grid = int(grid);
      p.base = base;
      p.rem = int(grid % ngroups);
    }
  }
  p.part_bytes = round256(int64_t(p.grid) * p.G * kND * kBwdBK * 4);
  return p;
}

}  // namespace
}  // namespace k1tc

bool k1_tc_bwd_supported(const void *go, const void *x, const void *W, const void *proj,
                         const void *gx, int64_t T, int64_t nC, int64_t D) {
  if (D != k1tc::kND || nC % k1tc::kBwdBK != 0 || T < 1 || T > (int64_t(1) << 31)) return false;
  // Each group of at most 8 k-chunks needs its own CTA.
  if (nC / k1tc::kBwdBK > int64_t(k1tc::kBwdMaxG) * k1tc::device_sms()) return false;
  const uintptr_t m = reinterpret_cast<uintptr_t>(go) | reinterpret_cast<uintptr_t>(x) |
                      reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(proj) |
                      reinterpret_cast<uintptr_t>(gx);
  if (m & 15) return false;
  return k1tc::device_is_sm100() && k1tc::encode_fn() != nullptr;
}

int64_t k1_tc_bwd_workspace_bytes(int64_t T, int64_t nC) {
  if (T < 1 || nC < k1tc::kBwdBK || nC % k1tc::kBwdBK) return 0;
  if (nC / k1tc::kBwdBK > int64_t(k1tc::kBwdMaxG) * k1tc::device_sms()) return 0;
  const k1tc::BwdPlan p = k1tc::bwd_plan(T, nC);
  return p.part_bytes;
}

int launch_k1_tc_bwd(const void *go, const void *x, const void *W, const void *proj,
                     const float *inv_rms, void *gx, void *gW, void *ws, int64_t ws_bytes,
                     int64_t T, int nC, cudaStream_t s) {
  using namespace k1tc;
  const BwdPlan p = bwd_plan(T, nC);
  const bool with_dw = gW != nullptr;
  float *part = nullptr;
  if (with_dw) {
    if (ws == nullptr || ws_bytes < p.part_bytes || (reinterpret_cast<uintptr_t>(ws) & 255)) {
      snprintf(g_msg, sizeof(g_msg), "workspace of %lld bytes (need %lld, 256-byte aligned)",
               (long long)ws_bytes, (long long)p.part_bytes);
      return 6;
    }
    part = static_cast<float *>(ws);
  }
  CUtensorMap mx, mgx, mgo, mproj, mw;
  bool ok = make_map(&mx, x, uint64_t(nC), uint64_t(T), uint64_t(nC) * 2, 64, kBwdBT,
                     CU_TENSOR_MAP_SWIZZLE_128B) &&
            make_map(&mgx, gx, uint64_t(nC), uint64_t(T), uint64_t(nC) * 2, 64, kBwdBT,
                     CU_TENSOR_MAP_SWIZZLE_128B) &&
            make_map(&mgo, go, kND, uint64_t(T), kND * 2, kND, kBwdBT, CU_TENSOR_MAP_SWIZZLE_64B) &&
            make_map(&mproj, proj, kND, uint64_t(T), kND * 2, kND, kBwdBT,
                     CU_TENSOR_MAP_SWIZZLE_64B) &&
            make_map(&mw, W, uint64_t(nC), kND, uint64_t(nC) * 2, 64, kND,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (!ok) {
    snprintf(g_msg, sizeof(g_msg), "cuTensorMapEncodeTiled failed");
    return 5;
  }
  const size_t smem = sizeof(BwdSmem) + 1024;
  if (int e = set_smem_attr(reinterpret_cast<const void *>(k1_bwd_tc_kernel), smem)) return e;
  BwdArgs args;
  args.inv_rms = inv_rms;
  args.dw_part = part;
  args.T = T;
  args.nC = nC;
  args.ntt = p.ntt;
  args.G = p.G;
  args.base = p.base;
  args.rem = p.rem;
  args.with_dw = with_dw ? 1 : 0;
  launch(k1_bwd_tc_kernel, dim3(unsigned(p.grid)), dim3(kBwdThreads), smem, s, mx, mgx, mgo, mproj,
         mw, args);
  if (with_dw) {
    launch(k1_bwd_dw_reduce_kernel, dim3(unsigned(p.nkc), kND), dim3(kBwdBK), 0, s, part,
           static_cast<__nv_bfloat16 *>(gW), nC, p.ntt, p.G, p.base, p.rem);
  }
  return 0;
}

int launch_k1_tc_fwd_lost_copy(const void *x, const void *W, void *out, float *inv_rms,
                               int64_t T, int nC, cudaStream_t s) {
  using namespace k1tc;
  CUtensorMap mx, mw;
  if (!make_map(&mx, x, uint64_t(nC), uint64_t(T), uint64_t(nC) * 2, 64, kBoxRows,
                CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map(&mw, W, uint64_t(nC), kND, uint64_t(nC) * 2, 64, kND,
                CU_TENSOR_MAP_SWIZZLE_128B)) {
    snprintf(g_msg, sizeof(g_msg), "cuTensorMapEncodeTiled failed");
    return 5;
  }
  const int64_t units = (T + kBoxRows - 1) / kBoxRows;
  int64_t grid = int64_t(device_sms()) * FMHC_K1F_CTAS_PER_SM;
  if (grid > units) grid = units;
  const size_t smem = sizeof(FwdSmem) + 1024;
  auto kern = k1_fwd_tc_kernel<false, true>;
  if (int e = set_smem_attr(reinterpret_cast<const void *>(kern), smem)) return e;
  launch(kern, dim3(unsigned(grid)), dim3(kThreads), smem, s, mx, mw,
         reinterpret_cast<__nv_bfloat16 *>(out), inv_rms, T, nC, units, K2Params{},
         k2tok::Out{nullptr, nullptr, nullptr});
  return 0;
}

int read_device_error(unsigned *code) {
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, sm100::g_device_error, sizeof(v)) != cudaSuccess) return 5;
  if (v && cudaMemcpyToSymbol(sm100::g_device_error, &zero, sizeof(zero)) != cudaSuccess) return 5;
  *code = v;
  return 0;
}

}  // namespace fmhc
