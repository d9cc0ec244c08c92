// Forward for 64 < D <= 256 on CTA pairs: O = act(X @ W1) @ W2 with M = 256 tcgen05.mma
// (cta_group::2). Same math and rounding points as the other forward kernels, which
// replace flashmlp_fwd_kernel (flashmlp.py:63-158): Z accumulates in fp32, H = act(Z) is
// rounded to the input dtype before the second product (flashmlp.py:140-147), O
// accumulates in fp32 over E chunks and is rounded once (flashmlp.py:150, :157).
//
// A cluster of two CTAs (ranks 0 and 1, one per SM) owns 256 rows of one head: CTA r the
// rows [256 p + 128 r, 256 p + 128 r + 128). Per E chunk c of 128 columns:
//   GEMM1  Z[zb]  = X @ W1c      M = 256, N = 128, K = DP   (A: X, 128 rows per CTA;
//                                 B: W1c, e columns 64 r .. 64 r + 63 held by CTA r)
//   act    H = round(act(Z))     each CTA's 16 activation warps on its own TMEM rows,
//                                 H packed back into Z's columns
//   GEMM2  O[ob] += H @ W2c      M = 256, N = DP, K = 128   (A: H in TMEM;
//                                 B: W2c, d columns DP/2 r .. DP/2 (r+1) - 1 held by CTA r)
// Why pairs: each SM stages only half of every weight chunk (the weight stream per FLOP is
// halved, as with two row tiles per CTA) and reads 6 KB of operands per 64-cycle K-step of
// GEMM1 instead of 8 KB, while TMEM keeps room for several Z buffers: GEMM1 runs NZ - 1
// chunks ahead of GEMM2 (NZ = 3 for DP = 128), so the activation warps never wait for a
// GEMM1 queued behind the GEMM2 of the chunk they have just finished, and the tensor pipe
// has the next GEMM2 as soon as a chunk is activated.
//
// Roles (18 warps per CTA): warp 0 loads this CTA's tiles (TMA; transaction bytes counted
// on CTA 0's barriers), warp 1 of CTA 0 issues every MMA of the pair and commits to both
// CTAs' barriers (warp 1 of CTA 1 only takes part in the TMEM allocation), warps 2..17
// activate and run the epilogue, arriving on CTA 0's barriers. All waits are bounded.
//
// TMEM per CTA: O [0, DP), Z buffers [DP, DP + NZ*128): NZ = 3 (DP = 128), 2 (DP = 256).
// Shared memory per CTA: X (own 128 rows) x XB, WS stages of the own halves of the W1 and
// W2 chunks.
#include "fmlp_act.cuh"
#include "fmlp_kernels.h"
#include "fmlp_ptx.cuh"

namespace fmlp {

template <int DP>
struct Fwd2Cfg {
  static_assert(DP == 128 || DP == 256, "pair forward covers 64 < D <= 256");
  static constexpr int BM = kRows;  // rows per CTA
  static constexpr int ET = 128;    // E chunk (GEMM1 N across the pair)
  static constexpr int XB = DP <= 128 ? 2 : 1;
  static constexpr int NO = 1;                 // O accumulators in TMEM
  static constexpr int NZ = DP <= 128 ? 3 : 2;  // Z buffers: GEMM1 runs NZ - 1 chunks ahead
  static constexpr int WS = DP <= 128 ? 4 : 2;
  static constexpr int X_BYTES = BM * DP * 2;
  static constexpr int W1H_BYTES = DP * (ET / 2) * 2;  // own half of a W1 chunk: DP rows x 64 e
  static constexpr int W2H_BYTES = ET * (DP / 2) * 2;  // own half of a W2 chunk: 128 e rows x DP/2 d
  static constexpr int OFF_X = 0;
  static constexpr int OFF_W1 = OFF_X + XB * X_BYTES;
  static constexpr int OFF_W2 = OFF_W1 + WS * W1H_BYTES;
  static constexpr int OFF_BAR = OFF_W2 + WS * W2H_BYTES;
  // x_full[XB] x_empty[XB] w1_full[WS] w1_empty[WS] w2_full[WS] w2_empty[WS]
  // z_full[NZ] h_full[NZ] o_full[NO] o_empty[NO] done
  static constexpr int NBAR = 2 * XB + 4 * WS + 2 * NZ + 2 * NO + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16 + 1024;
  static constexpr int SMEM = SMEM_USED > 120 * 1024 ? SMEM_USED : 120 * 1024;
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr int TMEM_O = 0;
  static constexpr int TMEM_Z = NO * DP;
  static constexpr int TMEM_COLS = 512;
  static_assert(TMEM_Z + NZ * ET <= TMEM_COLS, "TMEM budget");
  static constexpr int NUM_ACT_WARPS = 16;
  static constexpr int NUM_THREADS = 32 * (2 + NUM_ACT_WARPS);
  static constexpr int ARRIVALS = 2 * NUM_ACT_WARPS;  // activation warps of both CTAs
  static constexpr int SW = ET / 4;  // Z columns per activation warp
  static constexpr int OW = DP / 4;  // O columns per activation warp
};

template <int DP, typename T, int ACT>
__global__ void __launch_bounds__(576, 1)
    fmlp_fwd2sm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w1,
                       const __grid_constant__ CUtensorMap tm_w2, T* __restrict__ O, int H, int B, int D, int E,
                       uint32_t* status) {
  using C = Fwd2Cfg<DP>;
  constexpr int ET = C::ET, XB = C::XB, NO = C::NO, NZ = C::NZ, WS = C::WS, BM = C::BM, SW = C::SW, OW = C::OW;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzle atoms; the same offset in both CTAs (same
  // kernel), as the pair MMA requires of its operands.
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sX = smem + C::OFF_X;
  uint8_t* sW1 = smem + C::OFF_W1;
  uint8_t* sW2 = smem + C::OFF_W2;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* x_full = bars;
  uint64_t* x_empty = x_full + XB;
  uint64_t* w1_full = x_empty + XB;
  uint64_t* w1_empty = w1_full + WS;
  uint64_t* w2_full = w1_empty + WS;
  uint64_t* w2_empty = w2_full + WS;
  uint64_t* z_full = w2_empty + WS;
  uint64_t* h_full = z_full + NZ;
  uint64_t* o_full = h_full + NZ;
  uint64_t* o_empty = o_full + NO;
  uint64_t* done_bar = o_empty + NO;
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_flag = misc + 1;  // misc[2] stays 0: "never abort" flag for drains
  const WaitCtx ctx{abort_flag, status};
  const WaitCtx drain{misc + 2, status};

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cid = int(cluster_index()), ncl = int(cluster_count());
  const int nB = (B + BM - 1) / BM;
  const int nP = (nB + 1) / 2;  // 256-row blocks per head
  const int nE = (E + ET - 1) / ET;
  const int nitems = H * nP;

  if (threadIdx.x == 0) {
    misc[1] = 0;
    misc[2] = 0;
    for (int i = 0; i < XB; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
    }
    for (int i = 0; i < WS; ++i) {
      mbar_init(&w1_full[i], 1);
      mbar_init(&w1_empty[i], 1);
      mbar_init(&w2_full[i], 1);
      mbar_init(&w2_empty[i], 1);
    }
    for (int i = 0; i < NZ; ++i) {
      mbar_init(&z_full[i], 1);
      mbar_init(&h_full[i], C::ARRIVALS);
    }
    for (int i = 0; i < NO; ++i) {
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], C::ARRIVALS);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w1);
    tma_prefetch_desc(&tm_w2);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers exist before any arrival or transaction byte
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (each CTA)
    if (lane == 0) {
      // CTA 0's producer announces the bytes of both CTAs on CTA 0's full barriers; CTA 1
      // only issues its loads there. Each CTA learns that a stage is free from its own
      // empty barrier (the pair MMA's commit reaches both).
      const bool lead = rank == 0;
      uint32_t c1 = 0, c2 = 0, xl = 0;
      bool ok = true;
      for (int item = cid; item < nitems && ok; item += ncl) {
        const int h = item / nP, pr = item % nP;
        {
          const int xb = xl % XB;
          if (!(ok = mbar_wait(&x_empty[xb], ((xl / XB) & 1) ^ 1, ctx))) break;
          if (lead) mbar_arrive_expect_tx(&x_full[xb], 2 * C::X_BYTES);
          const uint32_t bar = mapa_shared(smem_u32(&x_full[xb]), 0);
          for (int r = 0; r < DP / 64; ++r)
            tma_load_3d_pair(sX + xb * C::X_BYTES + r * BM * 128, &tm_x, bar, 64 * r, (2 * pr + int(rank)) * BM, h);
          ++xl;
        }
        for (int c = 0; c < nE && ok; ++c) {
          {
            const int s = c1 % WS;
            if (!(ok = mbar_wait(&w1_empty[s], ((c1 / WS) & 1) ^ 1, ctx))) break;
            if (lead) mbar_arrive_expect_tx(&w1_full[s], 2 * C::W1H_BYTES);
            tma_load_3d_pair(sW1 + s * C::W1H_BYTES, &tm_w1, mapa_shared(smem_u32(&w1_full[s]), 0),
                             c * ET + 64 * int(rank), 0, h);
            ++c1;
          }
          {
            const int s = c2 % WS;
            if (!(ok = mbar_wait(&w2_empty[s], ((c2 / WS) & 1) ^ 1, ctx))) break;
            if (lead) mbar_arrive_expect_tx(&w2_full[s], 2 * C::W2H_BYTES);
            const uint32_t bar = mapa_shared(smem_u32(&w2_full[s]), 0);
            for (int r = 0; r < DP / 128; ++r)
              tma_load_3d_pair(sW2 + s * C::W2H_BYTES + r * ET * 128, &tm_w2, bar, (DP / 2) * int(rank) + 64 * r,
                               c * ET, h);
            ++c2;
          }
        }
      }
      // Drain (matters only after an abort): CTA 0 waits for the full barriers of what it
      // issued, which also count CTA 1's bytes of the same stages; CTA 1 gives its own
      // in-flight loads time to land before the final cluster barrier.
      if (lead) {
        for (uint32_t s = 0; s < WS; ++s) {
          if (c1 > s) mbar_wait(&w1_full[s], ((c1 - 1 - s) / WS) & 1, drain);
          if (c2 > s) mbar_wait(&w2_full[s], ((c2 - 1 - s) / WS) & 1, drain);
        }
        for (uint32_t b = 0; b < XB; ++b)
          if (xl > b) mbar_wait(&x_full[b], ((xl - 1 - b) / XB) & 1, drain);
      } else if (!ok) {
        __nanosleep(100000);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (CTA 0)
    // One flat sequence of this pair's chunks g = (item, c) over all its items. GEMM1 runs
    // up to NZ - 1 chunks ahead of GEMM2: GEMM1(g) writes Z[g % NZ], which held H of chunk
    // g - NZ, read by GEMM2(g - NZ) issued before it (MMAs of one thread run in order).
    // So GEMM1 of the chunks the activation warps take next is never queued behind the
    // GEMM2 that waits for the chunk they are on.
    if (rank == 0) {
      constexpr bool kBF = Pack<T>::kBF16;
      constexpr uint32_t idesc1 = make_idesc_f16(kBF, 2 * BM, ET, false, true);
      constexpr uint32_t idesc2 = make_idesc_f16(kBF, 2 * BM, DP, false, true);
      constexpr uint16_t kBoth = 0x3;
      const int my_items = cid < nitems ? (nitems - 1 - cid) / ncl + 1 : 0;
      const uint32_t total = uint32_t(my_items) * uint32_t(nE);
      const uint32_t sX_a = smem_u32(sX), sW1_a = smem_u32(sW1), sW2_a = smem_u32(sW2);
      uint32_t c1 = 0, c2 = 0, g1 = 0;
      bool ok = true;

      auto gemm1 = [&](uint32_t g) -> bool {  // GEMM1 of chunk g into Z[g % NZ]
        const uint32_t it = g / uint32_t(nE), c = g % uint32_t(nE);
        const int xb = int(it % XB);
        if (c == 0) {
          if (!warp_wait(&x_full[xb], (it / XB) & 1, ctx)) return false;
        }
        const int s = c1 % WS;
        const uint32_t n = c1 / WS;
        ++c1;
        if (!warp_wait(&w1_full[s], n & 1, ctx)) return false;
        tc_fence_after();
        const uint32_t zb = g % NZ;
        if (elect_one()) {
          const uint64_t xdesc = make_sdesc_sw128(sX_a + xb * C::X_BYTES, 16, 1024);
          const uint32_t d_tmem = tmem + C::TMEM_Z + zb * ET;
          // own half of the chunk: one 64-wide MN group (LBO unused), 16 K rows per step
          const uint64_t wdesc = make_sdesc_sw128(sW1_a + s * C::W1H_BYTES, C::W1H_BYTES, 1024);
#pragma unroll
          for (int k = 0; k < DP / 16; ++k)
            mma_ss_pair(d_tmem, sdesc_add(xdesc, (k >> 2) * (BM * 128) + (k & 3) * 32), sdesc_add(wdesc, k * 2048),
                        idesc1, k > 0 ? 1u : 0u);
          mma_commit_pair(&z_full[zb], kBoth);
          mma_commit_pair(&w1_empty[s], kBoth);
          if (c + 1 == uint32_t(nE)) mma_commit_pair(&x_empty[xb], kBoth);  // every reader of X issued
        }
        __syncwarp();
        return true;
      };

      for (uint32_t g = 0; g < total && ok; ++g) {
        for (; g1 < total && g1 < g + NZ && ok; ++g1) ok = gemm1(g1);
        if (!ok) break;
        const uint32_t it = g / uint32_t(nE), c = g % uint32_t(nE);
        const int ob = int(it % NO);
        if (c == 0 && !(ok = warp_wait(&o_empty[ob], ((it / NO) & 1) ^ 1, ctx))) break;
        const uint32_t zb = g % NZ;
        if (!(ok = warp_wait(&h_full[zb], (g / NZ) & 1, ctx))) break;
        const int s = c2 % WS;
        const uint32_t n = c2 / WS;
        ++c2;
        if (!(ok = warp_wait(&w2_full[s], n & 1, ctx))) break;
        tc_fence_after();
        if (elect_one()) {
          // own half of the chunk: DP/2 d columns in 64-wide groups 128 rows x 128 B apart
          const uint64_t wdesc = make_sdesc_sw128(sW2_a + s * C::W2H_BYTES, ET * 128, 1024);
          const uint32_t o_tmem = tmem + C::TMEM_O + ob * DP;
          const uint32_t h_base = tmem + C::TMEM_Z + zb * ET;
          const uint32_t acc0 = c > 0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < ET / 16; ++k) {
            // H of E columns [16k, 16k+16) was packed by the activation warp owning that
            // column slice, at the start of its slice
            const int sl = (16 * k) / SW;
            const int within = 16 * k - sl * SW;
            mma_ts_pair(o_tmem, h_base + sl * SW + within / 2, sdesc_add(wdesc, k * 2048), idesc2, k > 0 ? 1u : acc0);
          }
          mma_commit_pair(&w2_empty[s], kBoth);
          if (c + 1 == uint32_t(nE)) mma_commit_pair(&o_full[ob], kBoth);
        }
        __syncwarp();
      }
      // Every MMA issued by this warp has completed before TMEM is released.
      if (elect_one()) mma_commit_pair(done_bar, 0x1);
      __syncwarp();
      warp_wait(done_bar, 0, drain);
    }
  } else {
    // ------------------------------------------------------------------ activation + epilogue
    // 16 warps per CTA: warp (q, j) owns TMEM lanes [32q, 32q+32) and column slice j of
    // every Z chunk and of the O tile; arrivals go to CTA 0's barriers.
    const int q = warp & 3;
    const int j = (warp - 2) >> 2;
    const uint32_t lane_off = uint32_t(q * 32) << 16;
    // CTA 0's h_full / o_empty barriers (consecutive 8-byte words)
    const uint32_t h_bar0 = mapa_shared(smem_u32(&h_full[0]), 0);
    const uint32_t o_bar0 = mapa_shared(smem_u32(&o_empty[0]), 0);
    uint32_t g = 0, it = 0;
    bool ok = true;
    for (int item = cid; item < nitems && ok; item += ncl, ++it) {
      const int h = item / nP, pr = item % nP;
      const int ob = it % NO;
      for (int c = 0; c < nE; ++c, ++g) {
        const uint32_t zb = g % NZ;
        if (!(ok = mbar_wait(&z_full[zb], (g / NZ) & 1, ctx))) break;
        tc_fence_after();
        const uint32_t zaddr = tmem + lane_off + C::TMEM_Z + zb * ET + j * SW;
        // H for these SW columns is packed two per column into the first SW/2 columns of
        // the slice, which this warp has just read.
        uint32_t v[SW], p[SW / 2];
        tmem_ld32_sync(zaddr, v);
        act_pack<T, ACT, SW / 2>(v, p);
        tmem_st16(zaddr, p);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(h_bar0 + 8 * zb);
      }
      if (!ok) break;
      // Epilogue: O (fp32, TMEM) -> input dtype -> global, 16-byte stores per row.
      if (!(ok = mbar_wait(&o_full[ob], (it / NO) & 1, ctx))) break;
      tc_fence_after();
      const int row = (2 * pr + int(rank)) * BM + q * 32 + lane;
      T* orow = O + (size_t(h) * B + row) * D;
      const uint32_t oaddr = tmem + lane_off + C::TMEM_O + ob * DP + j * OW;
#pragma unroll
      for (int u = 0; u < OW / 32; ++u) {
        const int col0 = j * OW + u * 32;
        uint32_t v[32], p[16];
        tmem_ld32_sync(oaddr + u * 32, v);
        plain_pack<T, 16>(v, p);
        if (u + 1 == OW / 32) {  // the whole slice of O is in registers: release it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(o_bar0 + 8 * ob);
        }
        if (row < B) {
          uint4* dst = reinterpret_cast<uint4*>(orow + col0);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (col0 + 8 * (i + 1) <= D) dst[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no arrival, load or MMA of the pair still targets either CTA
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, C::TMEM_COLS);
}

template <int DP, typename T, int ACT>
static cudaError_t launch_fwd2sm_t(const FwdLaunch& a) {
  using C = Fwd2Cfg<DP>;
  auto kern = fmlp_fwd2sm_kernel<DP, T, ACT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(C::NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = a.stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // persistent: as many pairs as fit at once (one CTA per SM), at most one per work item
  static int max_pairs[64] = {};
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (max_pairs[dev] == 0) {
    cfg.gridDim = dim3(2 * (a.sm_count / 2), 1, 1);
    int n = 0;
    if ((e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg)) != cudaSuccess) return e;
    max_pairs[dev] = n > 0 ? n : 1;
  }
  const long long nB = (a.B + kRows - 1) / kRows;
  const long long items = (long long)a.H * ((nB + 1) / 2);
  const int pairs = int(items < max_pairs[dev] ? items : max_pairs[dev]);
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  e = cudaLaunchKernelEx(&cfg, kern, a.tm_x, a.tm_w1, a.tm_w2, reinterpret_cast<T*>(a.o), a.H, a.B, a.D, a.E,
                         a.status);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <int DP, typename T>
static cudaError_t launch_fwd2sm_act(const FwdLaunch& a) {
  switch (a.act) {
    case kLeakyRelu: return launch_fwd2sm_t<DP, T, kLeakyRelu>(a);
    case kSilu: return launch_fwd2sm_t<DP, T, kSilu>(a);
    case kSigmoid: return launch_fwd2sm_t<DP, T, kSigmoid>(a);
    default: return launch_fwd2sm_t<DP, T, kLinear>(a);
  }
}

cudaError_t launch_fwd2sm(const FwdLaunch& a) {
  switch (a.dp) {
    case 128: return a.bf16 ? launch_fwd2sm_act<128, __nv_bfloat16>(a) : launch_fwd2sm_act<128, __half>(a);
    case 256: return a.bf16 ? launch_fwd2sm_act<256, __nv_bfloat16>(a) : launch_fwd2sm_act<256, __half>(a);
  }
  return cudaErrorInvalidValue;
}

}  // namespace fmlp
