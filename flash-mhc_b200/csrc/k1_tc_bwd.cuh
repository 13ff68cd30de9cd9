// K1 backward on the tensor cores: grad_x and (optionally) grad_W in one pass
// over x.  Included by k1_tc.cu (same translation unit as the forward kernel,
// sharing its PTX helpers and device error word).
//
//   s[t]        = (sum_d go[t,d] proj[t,d]) * inv_rms[t]^2 / nC
//   grad_x[t,k] = bf16( inv_rms[t] * sum_d go[t,d] W[d,k] - s[t] * x[t,k] )
//   grad_W[d,k] = bf16( sum_t gos[t,d] x[t,k] ),  gos = bf16(go * inv_rms)
//
// (src/flash_mhc/kernels.py:306-376 and src/flash_mhc/ops.py:683-684 of the
// reference.)  Work unit = (k-chunk of 128 columns, tile of 128 tokens); the
// units are ordered k-chunk-major and each persistent CTA takes a contiguous
// run of them, so it sweeps token tiles for one k-chunk at a time:
//
//   warp 0     TMA producer: per unit x[128 t x 128 k] (two 64-column boxes,
//              128-byte swizzle), go[128 t x 32] and gos[128 t x 32] (64-byte
//              swizzle); per k-chunk segment the W chunk [32 x 128 k].
//   warp 1     MMA issuer, per unit:
//                grad_W: D2[k, d] += x^T (MN-major A) * gos (MN-major B),
//                        8 x M128 N32 K16, accumulated over the segment;
//                grad_x: D1[t, k]  = go (K-major A) * W^T (MN-major B),
//                        2 x M128 N128 K16 into one of two TMEM buffers.
//   warps 2-9  epilogue, two warps per TMEM lane quarter: thread = token row,
//              warps 2-5 columns 0-63, warps 6-9 columns 64-127 of the unit:
//              grad_x = inv*D1 - s*x written over x in the stage buffer; at a
//              segment end warps 2-5 move the grad_W partial D2 (thread per
//              k row) to the workspace.
//   warp 10    store: TMA-stores each unit's grad_x from its stage and frees
//              the stage as soon as the store has read it, so a stage is held
//              only for its load, its epilogue and its store read.
// A prep kernel computes per token s and inv_rms (float2) and the grad_W
// operand gos; the producer brings the unit's 128 (s, inv) pairs into the
// stage with a bulk copy, so the epilogue reads them from shared memory.  A
// final small kernel reduces the per-CTA grad_W partials in a fixed order
// (deterministic) and rounds to bf16.  Without a workspace (grad_x only) the
// epilogue computes s itself from go and proj.
#pragma once

namespace fmhc {
namespace k1tc {

#ifndef FMHC_K1B_STAGES
#define FMHC_K1B_STAGES 4
#endif
#ifndef FMHC_K1B_CTAS_PER_SM
#define FMHC_K1B_CTAS_PER_SM 1
#endif
#ifndef FMHC_K1B_ACC_BUFS   // grad_x TMEM accumulators (1 or 2)
#define FMHC_K1B_ACC_BUFS 2
#endif
#ifndef FMHC_K1B_STORES_IN_FLIGHT  // grad_x TMA stores outstanding per CTA (1 or 2)
#define FMHC_K1B_STORES_IN_FLIGHT 2
#endif
#ifndef FMHC_K1B_W_BUFS     // W chunk buffers (1 or 2)
#define FMHC_K1B_W_BUFS 2
#endif
constexpr int kBwdBT = 128;                       // tokens per unit (MMA M of grad_x)
constexpr int kBwdBK = 128;                       // k per unit (MMA N of grad_x, M of grad_W)
constexpr int kBwdStages = FMHC_K1B_STAGES;
constexpr int kBwdAcc = FMHC_K1B_ACC_BUFS;
constexpr int kBwdWBufs = FMHC_K1B_W_BUFS;
static_assert(kBwdAcc == 1 || kBwdAcc == 2, "one or two grad_x accumulators");
constexpr int kBwdXBytes = kBwdBT * kBwdBK * 2;   // 32 KiB (two 16 KiB boxes)
constexpr int kBwdXBox = kBwdBT * 64 * 2;         // 16 KiB
constexpr int kBwdGBytes = kBwdBT * kND * 2;      // 8 KiB  (go or gos tile)
constexpr int kBwdSBytes = kBwdBT * 8;            // 1 KiB  ((s, inv_rms) per token)
constexpr int kBwdStageBytes = kBwdXBytes + 2 * kBwdGBytes + kBwdSBytes;  // 49 KiB
constexpr int kBwdThreads = 352;                  // producer, MMA, 8 epilogue warps, store
constexpr int kBwdEpiWarps = 8;
constexpr int kBwdStoreWarp = 2 + kBwdEpiWarps;
constexpr int kBwdWBytes = kND * kBwdBK * 2;      // 8 KiB  (two 4 KiB boxes)
// kBwdAcc x 128 (grad_x) + 32 (grad_W) columns, rounded up to a power of two.
constexpr uint32_t kBwdTmemCols = kBwdAcc == 2 ? 512 : 256;
constexpr uint32_t kBwdDwCol = kBwdAcc * 128;

struct alignas(1024) BwdSmem {
  uint8_t stage[kBwdStages][kBwdStageBytes];
  uint8_t wbuf[kBwdWBufs][kBwdWBytes];
  uint64_t full[kBwdStages];
  uint64_t empty[kBwdStages];
  uint64_t tfull[kBwdAcc];
  uint64_t tempty[kBwdAcc];
  uint64_t wfull[kBwdWBufs];
  uint64_t wempty[kBwdWBufs];
  uint64_t dwfull;
  uint64_t dwempty;
  // epi[s]: the 8 epilogue warps finished writing grad_x into stage s.  One
  // barrier per stage: its next phase belongs to the next unit in that stage,
  // which cannot be loaded before the store warp has waited on this phase and
  // freed the stage, so phases never alias and each counts one unit's arrivals.
  uint64_t epi[kBwdStages];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

enum : unsigned { kSiteBProdEmpty = 0x201, kSiteBProdW = 0x202, kSiteBMmaFull = 0x203,
                  kSiteBMmaTempty = 0x204, kSiteBMmaW = 0x205, kSiteBMmaDw = 0x206,
                  kSiteBEpiFull = 0x207, kSiteBEpiTfull = 0x208, kSiteBEpiDw = 0x209,
                  kSiteBDrain = 0x20a, kSiteBEpiStore = 0x20b };

struct BwdArgs {
  const __nv_bfloat16 *go;    // (T, 32)
  const __nv_bfloat16 *proj;  // (T, 32)
  const float *inv_rms;       // (T,)
  const float2 *sinv;         // (ntt*128,) (s, inv_rms) per token, or nullptr
  float *dw_part;             // [grid][maxseg][32][128] f32 (only with_dw)
  int64_t T;
  int nC;
  int ntt;                    // token tiles
  int64_t units;              // (nC / 128) * ntt
  int maxseg;
  int with_dw;
};

// Unit u -> (k-chunk, token tile).
__device__ __forceinline__ void bwd_unit(int64_t u, int ntt, int &kc, int &tt) {
  kc = int(u / ntt);
  tt = int(u - int64_t(kc) * ntt);
}

// Partial dot product of one 16-byte chunk (8 of the 32 d) of go and proj.
// The full dot product is (p0 + p1) + (p2 + p3) over the four chunks, in this
// order in both places that compute it (prep kernel, no-workspace epilogue),
// so grad_x is identical whichever entry point computed it.
__device__ __forceinline__ float go_proj_chunk_dot(const uint4 g, const uint4 p) {
  float dot = 0.f;
  dot = fmaf(bf16lo(g.x), bf16lo(p.x), dot); dot = fmaf(bf16hi(g.x), bf16hi(p.x), dot);
  dot = fmaf(bf16lo(g.y), bf16lo(p.y), dot); dot = fmaf(bf16hi(g.y), bf16hi(p.y), dot);
  dot = fmaf(bf16lo(g.z), bf16lo(p.z), dot); dot = fmaf(bf16hi(g.z), bf16hi(p.z), dot);
  dot = fmaf(bf16lo(g.w), bf16lo(p.w), dot); dot = fmaf(bf16hi(g.w), bf16hi(p.w), dot);
  return dot;
}

__global__ void __launch_bounds__(kBwdThreads, FMHC_K1B_CTAS_PER_SM)
k1_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmap_x,
                 const __grid_constant__ CUtensorMap tmap_gx,
                 const __grid_constant__ CUtensorMap tmap_go,
                 const __grid_constant__ CUtensorMap tmap_gos,
                 const __grid_constant__ CUtensorMap tmap_w, const BwdArgs a) {
  extern __shared__ uint8_t smem_raw[];
  BwdSmem &sm = *reinterpret_cast<BwdSmem *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int *abort = &sm.abort;

  const int64_t u0 = int64_t(blockIdx.x) * a.units / gridDim.x;
  const int64_t u1 = int64_t(blockIdx.x + 1) * a.units / gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kBwdStages; ++s) {
      mbar_init(smem_u32(&sm.full[s]), 1);
      mbar_init(smem_u32(&sm.empty[s]), 1);  // released by the store warp after its store read
      mbar_init(smem_u32(&sm.epi[s]), kBwdEpiWarps);
    }
    for (int b = 0; b < kBwdAcc; ++b) {
      mbar_init(smem_u32(&sm.tfull[b]), 1);
      mbar_init(smem_u32(&sm.tempty[b]), kBwdEpiWarps);
    }
    for (int b = 0; b < kBwdWBufs; ++b) {
      mbar_init(smem_u32(&sm.wfull[b]), 1);
      mbar_init(smem_u32(&sm.wempty[b]), 1);
    }
    mbar_init(smem_u32(&sm.dwfull), 1);
    mbar_init(smem_u32(&sm.dwempty), 4);  // warps 2-5 read the grad_W partial
    mbar_init(smem_u32(&sm.mma_done), 1);
    sm.abort = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_gx);
    prefetch_tmap(&tmap_go);
    prefetch_tmap(&tmap_gos);
    prefetch_tmap(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&sm.tmem_base), kBwdTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  // No global memory is touched before this point (see pdl_wait()).
  pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0, issued = 0, seg = -1, kc_prev = -1;
      uint32_t phase = 0;
      const uint32_t tx = uint32_t(kBwdXBytes + (a.with_dw ? 2 : 1) * kBwdGBytes +
                                   (a.sinv ? kBwdSBytes : 0));
      for (int64_t u = u0; u < u1 && !*abort; ++u) {
        int kc, tt;
        bwd_unit(u, a.ntt, kc, tt);
        if (kc != kc_prev) {  // new segment: W chunk into wbuf[seg % kBwdWBufs]
          ++seg;
          kc_prev = kc;
          const int wb = seg % kBwdWBufs;
          if (!mbar_wait(smem_u32(&sm.wempty[wb]), ((seg / kBwdWBufs) & 1) ^ 1, abort, kSiteBProdW))
            break;
          const uint32_t wf = smem_u32(&sm.wfull[wb]);
          mbar_arrive_expect_tx(wf, kBwdWBytes);
          tma_load_2d(smem_u32(sm.wbuf[wb]), &tmap_w, wf, kc * kBwdBK, 0);
          tma_load_2d(smem_u32(sm.wbuf[wb]) + kBwdWBytes / 2, &tmap_w, wf, kc * kBwdBK + 64, 0);
        }
        if (!mbar_wait(smem_u32(&sm.empty[stage]), phase ^ 1, abort, kSiteBProdEmpty)) break;
        const uint32_t f = smem_u32(&sm.full[stage]);
        const uint32_t base = smem_u32(sm.stage[stage]);
        const int32_t row0 = tt * kBwdBT;
        mbar_arrive_expect_tx(f, tx);
        tma_load_2d(base, &tmap_x, f, kc * kBwdBK, row0);
        tma_load_2d(base + kBwdXBox, &tmap_x, f, kc * kBwdBK + 64, row0);
        tma_load_2d(base + kBwdXBytes, &tmap_go, f, 0, row0);
        if (a.with_dw) tma_load_2d(base + kBwdXBytes + kBwdGBytes, &tmap_gos, f, 0, row0);
        if (a.sinv) bulk_load(base + kBwdXBytes + 2 * kBwdGBytes, a.sinv + row0, kBwdSBytes, f);
        ++issued;
        if (++stage == kBwdStages) { stage = 0; phase ^= 1; }
      }
      const int n = issued < kBwdStages ? issued : kBwdStages;
      int s = stage;
      uint32_t ph = phase;
      for (int i = 0; i < n; ++i) {
        if (--s < 0) { s = kBwdStages - 1; ph ^= 1; }
        mbar_wait(smem_u32(&sm.full[s]), ph, abort, kSiteBDrain, true);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_dx = idesc_bf16_f32(kBwdBT, kBwdBK, 0, 1);
      constexpr uint32_t idesc_dw = idesc_bf16_f32(kBwdBK, kND, 1, 1);
      int stage = 0, acc = 0, seg = -1, kc_prev = -1;
      uint32_t phase = 0, acc_phase = 0;
      bool first_in_seg = false;
      for (int64_t u = u0; u < u1 && !*abort; ++u) {
        int kc, tt;
        bwd_unit(u, a.ntt, kc, tt);
        if (kc != kc_prev) {
          ++seg;
          kc_prev = kc;
          first_in_seg = true;
          if (a.with_dw && seg > 0 &&
              !mbar_wait(smem_u32(&sm.dwempty), (seg - 1) & 1, abort, kSiteBMmaDw))
            break;
          if (!mbar_wait(smem_u32(&sm.wfull[seg % kBwdWBufs]), (seg / kBwdWBufs) & 1, abort,
                         kSiteBMmaW))
            break;
        }
        int kc_next = -1, tt_next;
        if (u + 1 < u1) bwd_unit(u + 1, a.ntt, kc_next, tt_next);
        const bool last_in_seg = kc_next != kc;
        if (!mbar_wait(smem_u32(&sm.tempty[acc]), acc_phase ^ 1, abort, kSiteBMmaTempty)) break;
        if (!mbar_wait(smem_u32(&sm.full[stage]), phase, abort, kSiteBMmaFull)) break;
        tc_fence_after();
        const uint32_t base = smem_u32(sm.stage[stage]);
        if (a.with_dw) {
          // grad_W: M = k (two 64-wide MN blocks 16 KiB apart), N = d, K = tokens.
#pragma unroll
          for (int k = 0; k < kBwdBT / 16; ++k) {
            const uint64_t ad = smem_desc(base + k * 2048, kBwdXBox, 1024, 2);
            const uint64_t bd = smem_desc(base + kBwdXBytes + kBwdGBytes + k * 1024, 512, 512, 4);
            mma_bf16_ss(tmem + kBwdDwCol, ad, bd, idesc_dw, (first_in_seg && k == 0) ? 0u : 1u);
          }
        }
        {
          // grad_x: M = tokens, N = 128 k (two 64-wide MN blocks 4 KiB apart), K = d.
          const uint32_t wb = smem_u32(sm.wbuf[seg % kBwdWBufs]);
#pragma unroll
          for (int k = 0; k < kND / 16; ++k) {
            const uint64_t ad = smem_desc(base + kBwdXBytes + k * 32, 16, 512, 4);
            const uint64_t bd = smem_desc(wb + k * 2048, kBwdWBytes / 2, 1024, 2);
            mma_bf16_ss(tmem + uint32_t(acc * kBwdBK), ad, bd, idesc_dx, k != 0);
          }
        }
        mma_commit(smem_u32(&sm.tfull[acc]));
        if (last_in_seg) {
          if (a.with_dw) mma_commit(smem_u32(&sm.dwfull));
          mma_commit(smem_u32(&sm.wempty[seg % kBwdWBufs]));
        }
        first_in_seg = false;
        if (++acc == kBwdAcc) { acc = 0; acc_phase ^= 1; }
        if (++stage == kBwdStages) { stage = 0; phase ^= 1; }
      }
      mma_commit(smem_u32(&sm.mma_done));
      mbar_wait(smem_u32(&sm.mma_done), 0, abort, kSiteBDrain, true);
    }
  } else if (warp < kBwdStoreWarp) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;           // TMEM lane quarter
    const int h = (warp - 2) >> 2;    // column half of the unit (0: 0-63, 1: 64-127)
    const int r = q * 32 + lane;      // token row of the unit / k row of the grad_W partial
    int stage = 0, acc = 0, seg = -1, kc_prev = -1;
    uint32_t phase = 0, acc_phase = 0;
    for (int64_t u = u0; u < u1 && !*abort; ++u) {
      int kc, tt;
      bwd_unit(u, a.ntt, kc, tt);
      if (kc != kc_prev) { ++seg; kc_prev = kc; }
      int kc_next = -1, tt_next;
      if (u + 1 < u1) bwd_unit(u + 1, a.ntt, kc_next, tt_next);
      const bool last_in_seg = kc_next != kc;

      const int64_t t = int64_t(tt) * kBwdBT + r;
      float s = 0.f, inv = 0.f;
      if (!a.sinv && t < a.T) {
        // No workspace: s = (go . proj) * inv^2 / nC from the stored forward output.
        inv = a.inv_rms[t];
        const uint4 *g4 = reinterpret_cast<const uint4 *>(a.go + t * kND);
        const uint4 *p4 = reinterpret_cast<const uint4 *>(a.proj + t * kND);
        float pc[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) pc[c] = go_proj_chunk_dot(__ldg(g4 + c), __ldg(p4 + c));
        const float dot = (pc[0] + pc[1]) + (pc[2] + pc[3]);
        s = dot * (inv * inv) / float(a.nC);
      }
      if (!mbar_wait(smem_u32(&sm.full[stage]), phase, abort, kSiteBEpiFull)) break;
      uint8_t *xs = sm.stage[stage];
      if (a.sinv) {
        const float2 si = reinterpret_cast<const float2 *>(xs + kBwdXBytes + 2 * kBwdGBytes)[r];
        s = si.x;
        inv = si.y;
      }
      if (!mbar_wait(smem_u32(&sm.tfull[acc]), acc_phase, abort, kSiteBEpiTfull)) break;
      tc_fence_after();
      uint32_t v[2][32];
      const uint32_t tl = tmem + (uint32_t(q * 32) << 16) + uint32_t(acc * kBwdBK + 64 * h);
      tmem_ld_32x32b_x32(tl, v[0]);
      tmem_ld_32x32b_x32(tl + 32, v[1]);
      tmem_wait_ld();
      // Columns 64h .. 64h+63 of row r are one 128-byte row of x box h; read
      // all eight 16-byte chunks before the math so the loads overlap.
      uint8_t *rowp = xs + h * kBwdXBox + r * 128;
      uint4 xv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) xv[i] = *reinterpret_cast<const uint4 *>(rowp + ((i ^ (r & 7)) << 4));
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float *dv = reinterpret_cast<const float *>(v[i >> 2] + 8 * (i & 3));
        uint4 o;
        o.x = pack_bf16x2(fmaf(-s, bf16lo(xv[i].x), inv * dv[0]), fmaf(-s, bf16hi(xv[i].x), inv * dv[1]));
        o.y = pack_bf16x2(fmaf(-s, bf16lo(xv[i].y), inv * dv[2]), fmaf(-s, bf16hi(xv[i].y), inv * dv[3]));
        o.z = pack_bf16x2(fmaf(-s, bf16lo(xv[i].z), inv * dv[4]), fmaf(-s, bf16hi(xv[i].z), inv * dv[5]));
        o.w = pack_bf16x2(fmaf(-s, bf16lo(xv[i].w), inv * dv[6]), fmaf(-s, bf16hi(xv[i].w), inv * dv[7]));
        *reinterpret_cast<uint4 *>(rowp + ((i ^ (r & 7)) << 4)) = o;
      }
      // Every writer makes its grad_x visible to the TMA (async proxy), then
      // one arrive per warp on epi[stage] for the store warp and on tempty.
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&sm.epi[stage]));
        mbar_arrive(smem_u32(&sm.tempty[acc]));
      }
      if (a.with_dw && last_in_seg && h == 0) {
        // grad_W partial of this segment: thread r owns k row r, 32 d columns.
        if (!mbar_wait(smem_u32(&sm.dwfull), seg & 1, abort, kSiteBEpiDw)) break;
        tc_fence_after();
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + (uint32_t(q * 32) << 16) + kBwdDwCol, v);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&sm.dwempty));
        const int sidx = seg < a.maxseg ? seg : a.maxseg - 1;
        float *dst = a.dw_part + (int64_t(blockIdx.x) * a.maxseg + sidx) * (kND * kBwdBK) + r;
#pragma unroll
        for (int d = 0; d < kND; ++d) __stcg(dst + d * kBwdBK, __uint_as_float(v[d]));
      }
      if (++acc == kBwdAcc) { acc = 0; acc_phase ^= 1; }
      if (++stage == kBwdStages) { stage = 0; phase ^= 1; }
    }
  } else {
    // --------------------------------------------------------------- store
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int prev = -1;
      (void)prev;
      for (int64_t u = u0; u < u1 && !*abort; ++u) {
        int kc, tt;
        bwd_unit(u, a.ntt, kc, tt);
        if (!mbar_wait(smem_u32(&sm.epi[stage]), phase, abort, kSiteBEpiStore)) break;
        const uint32_t base = smem_u32(sm.stage[stage]);
        tma_store_2d(&tmap_gx, base, kc * kBwdBK, tt * kBwdBT);
        tma_store_2d(&tmap_gx, base + kBwdXBox, kc * kBwdBK + 64, tt * kBwdBT);
        tma_store_commit();
#if FMHC_K1B_STORES_IN_FLIGHT == 2
        // Free the previous unit's stage once its store has read it, keeping
        // this unit's store in flight.
        tma_store_wait_read<1>();
        if (prev >= 0) mbar_arrive(smem_u32(&sm.empty[prev]));
        prev = stage;
#else
        // Free the stage once this store has read it (the global writes may
        // still be in flight).
        tma_store_wait_read<0>();
        mbar_arrive(smem_u32(&sm.empty[stage]));
#endif
        if (++stage == kBwdStages) { stage = 0; phase ^= 1; }
      }
      tma_store_wait_all<0>();
#if FMHC_K1B_STORES_IN_FLIGHT == 2
      if (prev >= 0) mbar_arrive(smem_u32(&sm.empty[prev]));
#endif
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kBwdTmemCols);
  }
}

// Per token: sinv[t] = (s, inv_rms) with s = (go . proj) * inv_rms^2 / nC,
// and (when gos != nullptr) gos[t, :] = bf16(go[t, :] * inv_rms[t]), the
// grad_W operand, rounded like the reference's (grad_out * inv_rms).to(x.dtype).
// Four threads per token, one 16-byte chunk of go and proj each; the chunk
// dot products are combined with two shuffles.  Rows T .. T_pad-1 of sinv
// are zeroed.  The grid covers exactly 4 * T_pad threads (T_pad is a multiple
// of 128), so every warp is whole.
__global__ void __launch_bounds__(256)
k1_bwd_prep_kernel(const __nv_bfloat16 *__restrict__ go, const __nv_bfloat16 *__restrict__ proj,
                   const float *__restrict__ inv_rms, __nv_bfloat16 *__restrict__ gos,
                   float2 *__restrict__ sinv, int64_t T, int64_t T_pad, int nC) {
  pdl_wait();
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t t = i >> 2;
  const int c = int(i & 3);
  if (t >= T_pad) return;  // never splits a warp (see above)
  const bool valid = t < T;
  float r = 0.f, dot = 0.f;
  uint4 g = make_uint4(0, 0, 0, 0);
  if (valid) {
    r = inv_rms[t];
    g = __ldg(reinterpret_cast<const uint4 *>(go + t * kND) + c);
    const uint4 p = __ldg(reinterpret_cast<const uint4 *>(proj + t * kND) + c);
    dot = go_proj_chunk_dot(g, p);
  }
  dot += __shfl_xor_sync(0xffffffffu, dot, 1);
  dot += __shfl_xor_sync(0xffffffffu, dot, 2);
  if (valid && gos) {
    uint4 o;
    o.x = pack_bf16x2(bf16lo(g.x) * r, bf16hi(g.x) * r);
    o.y = pack_bf16x2(bf16lo(g.y) * r, bf16hi(g.y) * r);
    o.z = pack_bf16x2(bf16lo(g.z) * r, bf16hi(g.z) * r);
    o.w = pack_bf16x2(bf16lo(g.w) * r, bf16hi(g.w) * r);
    reinterpret_cast<uint4 *>(gos + t * kND)[c] = o;
  }
  if (c == 0) sinv[t] = valid ? make_float2(dot * (r * r) / float(nC), r) : make_float2(0.f, 0.f);
}

// grad_W[d, k] = bf16(sum of the partials of every CTA whose unit range
// touches k-chunk k / 128), in increasing CTA order (deterministic).
// Block (kc, d): row d of k-chunk kc, one thread per column.  CTA c owns units
// [c*units/grid, (c+1)*units/grid) and grid <= units, so no CTA is empty and
// the contributors of the chunk's units [lo, hi) are exactly the CTAs from the
// owner of lo to the owner of hi - 1, where owner(u) = ((u+1)*grid - 1) / units.
// Their partials are loaded eight at a time and added in CTA order.
__global__ void __launch_bounds__(kBwdBK)
k1_bwd_dw_reduce_kernel(const float *__restrict__ part, __nv_bfloat16 *__restrict__ gW, int nC,
                        int ntt, int64_t units, int grid, int maxseg) {
  pdl_wait();
  const int kc = blockIdx.x, d = blockIdx.y, kl = threadIdx.x;
  const int64_t lo = int64_t(kc) * ntt, hi = lo + ntt;
  const int c_first = int(((lo + 1) * grid - 1) / units);
  const int c_last = int((hi * grid - 1) / units);
  const float *col = part + int64_t(d) * kBwdBK + kl;
  float acc = 0.f;
  for (int c = c_first; c <= c_last; c += 8) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int cc = c + i;
      v[i] = 0.f;
      if (cc <= c_last) {
        const int seg = kc - int((int64_t(cc) * units / grid) / ntt);
        v[i] = __ldg(col + (int64_t(cc) * maxseg + seg) * (kND * kBwdBK));
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (c + i <= c_last) acc += v[i];
  }
  gW[int64_t(d) * nC + int64_t(kc) * kBwdBK + kl] = __float2bfloat16_rn(acc);
}

}  // namespace k1tc
}  // namespace fmhc
