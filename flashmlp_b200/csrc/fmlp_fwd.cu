// Fused multi-head MLP forward for sm_100a:  O[h] = act(X[h] @ W1[h]) @ W2[h].
//
// Replaces the Triton kernel `flashmlp_fwd_kernel` (flashmlp.py:63-158). Same math and
// rounding points: Z = X@W1 accumulates in fp32, H = act(Z) is rounded to the input dtype
// before the second product (flashmlp.py:140-147), O accumulates in fp32 over E chunks and
// is rounded once at the end (flashmlp.py:150,157).
//
// Design (one CTA per SM, persistent over (head, 128-row tile) work items):
//   warp 0      TMA producer: X tile (double-buffered), W1/W2 E-chunks (2-stage rings)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..17 activation + epilogue (4 per TMEM lane quadrant): Z (fp32, TMEM) -> act
//               -> H (16-bit, written back into the same TMEM columns) ; O (TMEM) -> global
// GEMM1  Z[zb]  = X[smem]  @ W1c[smem]     (SS, M=128, N=ET,  K=D)
// GEMM2  O[ob] += H[tmem]  @ W2c[smem]     (TS, M=128, N=DP,  K=ET)
// Z is double-buffered so GEMM1 of chunk c+1 runs while chunk c is activated; O is
// double-buffered (DP<=128) so the epilogue of one tile overlaps the next tile.
#include "fmlp_kernels.h"
#include "fmlp_act.cuh"
#include "fmlp_ptx.cuh"

namespace fmlp {

template <int DP>
struct FwdCfg {
  static constexpr int BM = kRows;
  static constexpr int ET = DP <= 128 ? 128 : 64;
  static constexpr int XB = DP <= 128 ? 2 : 1;  // X smem buffers
  static constexpr int NO = DP <= 128 ? 2 : 1;  // O accumulators in TMEM
  static constexpr int WS = DP <= 64 ? 4 : 2;   // W ring stages
  static constexpr int X_BYTES = BM * DP * 2;
  static constexpr int W1_BYTES = DP * ET * 2;
  static constexpr int W2_BYTES = ET * DP * 2;
  static constexpr int OFF_X = 0;
  static constexpr int OFF_W1 = OFF_X + XB * X_BYTES;
  static constexpr int OFF_W2 = OFF_W1 + WS * W1_BYTES;
  static constexpr int OFF_BAR = OFF_W2 + WS * W2_BYTES;
  // barriers: x_full[XB] x_empty[XB] w1_full[WS] w1_empty[WS] w2_full[WS] w2_empty[WS]
  //           z_full[2] h_full[2] o_full[NO] o_empty[NO] done
  static constexpr int NBAR = 2 * XB + 4 * WS + 4 + 2 * NO + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  // + alignment slack; at least 120 KB so that only one CTA (and one 512-column TMEM
  // allocation) is ever resident per SM.
  static constexpr int SMEM_USED = OFF_MISC + 16 + 1024;
  static constexpr int SMEM = SMEM_USED > 120 * 1024 ? SMEM_USED : 120 * 1024;
  static constexpr int TMEM_O = 0;
  static constexpr int TMEM_Z = NO * DP;
  static constexpr int TMEM_COLS = 512;
  static_assert(TMEM_Z + 2 * ET <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr int NUM_ACT_WARPS = 16;  // 4 per TMEM lane quadrant
  static constexpr int NUM_THREADS = 32 * (2 + NUM_ACT_WARPS);
  static constexpr int SW = ET / 4;  // Z columns per activation warp
  static constexpr int OW = DP / 4;  // O columns per activation warp
};

template <int DP, typename T, int ACT>
__global__ void __launch_bounds__(576, 1)
    fmlp_fwd_kernel(const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_w1,
                    const __grid_constant__ CUtensorMap tm_w2, T* __restrict__ O, int H, int B,
                    int D, int E, uint32_t* status) {
  using C = FwdCfg<DP>;
  constexpr int ET = C::ET, XB = C::XB, NO = C::NO, WS = C::WS, BM = C::BM;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzle atoms.
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
  uint64_t* h_full = z_full + 2;
  uint64_t* o_full = h_full + 2;
  uint64_t* o_empty = o_full + NO;
  uint64_t* done_bar = o_empty + NO;
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_flag = misc + 1;  // misc[2] stays 0: "never abort" flag for drains

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nB = (B + BM - 1) / BM;
  const int nE = (E + ET - 1) / ET;
  const int ntiles = H * nB;
  const WaitCtx ctx{abort_flag, status};

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
    for (int i = 0; i < 2; ++i) {
      mbar_init(&z_full[i], 1);
      mbar_init(&h_full[i], C::NUM_ACT_WARPS);
    }
    for (int i = 0; i < NO; ++i) {
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], C::NUM_ACT_WARPS);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w1);
    tma_prefetch_desc(&tm_w2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      // c1/c2/xl count loads actually issued into the W1 ring, W2 ring and X buffers.
      uint32_t c1 = 0, c2 = 0, xl = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int h = tile / nB, bt = tile % nB;
        {
          const int xb = xl % XB;
          const uint32_t xn = xl / XB;
          if (!(ok = mbar_wait(&x_empty[xb], (xn & 1) ^ 1, ctx))) break;
          mbar_arrive_expect_tx(&x_full[xb], C::X_BYTES);
          for (int r = 0; r < DP / 64; ++r)
            tma_load_3d(sX + xb * C::X_BYTES + r * BM * 128, &tm_x, &x_full[xb], 64 * r, bt * BM, h);
          ++xl;
        }
        for (int c = 0; c < nE && ok; ++c) {
          {
            const int s = c1 % WS;
            const uint32_t n = c1 / WS;
            if (!(ok = mbar_wait(&w1_empty[s], (n & 1) ^ 1, ctx))) break;
            mbar_arrive_expect_tx(&w1_full[s], C::W1_BYTES);
            for (int r = 0; r < ET / 64; ++r)
              tma_load_3d(sW1 + s * C::W1_BYTES + r * DP * 128, &tm_w1, &w1_full[s],
                          c * ET + 64 * r, 0, h);
            ++c1;
          }
          {
            const int s = c2 % WS;
            const uint32_t n = c2 / WS;
            if (!(ok = mbar_wait(&w2_empty[s], (n & 1) ^ 1, ctx))) break;
            mbar_arrive_expect_tx(&w2_full[s], C::W2_BYTES);
            for (int r = 0; r < DP / 64; ++r)
              tma_load_3d(sW2 + s * C::W2_BYTES + r * ET * 128, &tm_w2, &w2_full[s], 64 * r,
                          c * ET, h);
            ++c2;
          }
        }
      }
      // Drain: no TMA write may still be in flight when the CTA exits (matters only
      // after an abort; in a normal run every load has already been consumed).
      const WaitCtx drain{misc + 2, status};
      for (uint32_t s = 0; s < WS; ++s) {
        if (c1 > s) mbar_wait(&w1_full[s], ((c1 - 1 - s) / WS) & 1, drain);
        if (c2 > s) mbar_wait(&w2_full[s], ((c2 - 1 - s) / WS) & 1, drain);
      }
      for (uint32_t b = 0; b < XB; ++b)
        if (xl > b) mbar_wait(&x_full[b], ((xl - 1 - b) / XB) & 1, drain);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp runs the schedule (warp-uniform waits); one elected lane issues
    // each unrolled burst of MMAs and the commits that follow it.
    constexpr bool kBF = Pack<T>::kBF16;
    constexpr uint32_t idesc1 = make_idesc_f16(kBF, BM, ET, false, true);
    constexpr uint32_t idesc2 = make_idesc_f16(kBF, BM, DP, false, true);
    uint32_t c1 = 0, c2 = 0, zc = 0, it = 0;
    bool ok = true;
    const uint32_t sX_a = smem_u32(sX), sW1_a = smem_u32(sW1), sW2_a = smem_u32(sW2);

    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
      const int xb = it % XB;
      const uint32_t xn = it / XB;
      const int ob = it % NO;
      const uint32_t on = it / NO;
      if (!(ok = warp_wait(&x_full[xb], xn & 1, ctx))) break;
      tc_fence_after();
      const uint64_t xdesc = make_sdesc_sw128(sX_a + xb * C::X_BYTES, 16, 1024);

      // GEMM1 of one E chunk into Z buffer (zidx & 1). K runs over the padded DP: the
      // columns of X and rows of W1 beyond D are zero-filled by TMA.
      auto gemm1 = [&](uint32_t zidx) -> bool {
        const int s = c1 % WS;
        const uint32_t n = c1 / WS;
        ++c1;
        if (!warp_wait(&w1_full[s], n & 1, ctx)) return false;
        tc_fence_after();
        const uint32_t zb = zidx & 1;
        if (elect_one()) {
          const uint32_t d_tmem = tmem + C::TMEM_Z + zb * ET;
          const uint64_t wdesc = make_sdesc_sw128(sW1_a + s * C::W1_BYTES, DP * 128, 1024);
#pragma unroll
          for (int k = 0; k < DP / 16; ++k)
            mma_ss(d_tmem, sdesc_add(xdesc, (k >> 2) * (BM * 128) + (k & 3) * 32),
                   sdesc_add(wdesc, k * 2048), idesc1, k > 0 ? 1u : 0u);
          mma_commit(&z_full[zb]);
          mma_commit(&w1_empty[s]);
        }
        __syncwarp();
        return true;
      };

      if (!(ok = gemm1(zc))) break;
      for (int c = 0; c < nE; ++c) {
        const uint32_t zcur = zc + c;
        if (c + 1 < nE) {
          if (!(ok = gemm1(zcur + 1))) break;
        } else {
          if (elect_one()) mma_commit(&x_empty[xb]);  // every reader of this X buffer issued
          __syncwarp();
        }
        if (c == 0) {
          if (!(ok = warp_wait(&o_empty[ob], (on & 1) ^ 1, ctx))) break;
        }
        const uint32_t zb = zcur & 1;
        if (!(ok = warp_wait(&h_full[zb], (zcur >> 1) & 1, ctx))) break;
        const int s = c2 % WS;
        const uint32_t n = c2 / WS;
        ++c2;
        if (!(ok = warp_wait(&w2_full[s], n & 1, ctx))) break;
        tc_fence_after();
        if (elect_one()) {
          const uint64_t wdesc = make_sdesc_sw128(sW2_a + s * C::W2_BYTES, ET * 128, 1024);
          const uint32_t o_tmem = tmem + C::TMEM_O + ob * DP;
          const uint32_t h_base = tmem + C::TMEM_Z + zb * ET;
          const uint32_t acc0 = c > 0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < ET / 16; ++k) {
            // H of E columns [16k, 16k+16) was packed by the activation warp that owns
            // that column slice, at the start of its slice (see the activation loop below).
            const int sl = (16 * k) / C::SW;
            const int within = 16 * k - sl * C::SW;
            mma_ts(o_tmem, h_base + sl * C::SW + within / 2, sdesc_add(wdesc, k * 2048), idesc2,
                   k > 0 ? 1u : acc0);
          }
          mma_commit(&w2_empty[s]);
          if (c + 1 == nE) mma_commit(&o_full[ob]);
        }
        __syncwarp();
      }
      zc += nE;
    }
    // Drain every MMA issued by this warp before TMEM is released.
    if (elect_one()) mma_commit(done_bar);
    __syncwarp();
    warp_wait(done_bar, 0, WaitCtx{misc + 2, status});
  } else {
    // ------------------------------------------------------------------ activation + epilogue
    // 16 warps: warp (q, j) owns TMEM lanes [32q, 32q+32) (its hardware quadrant) and
    // column slice j of every Z chunk and of the O tile.
    const int q = warp & 3;
    const int j = (warp - 2) >> 2;
    constexpr int SW = C::SW, OW = C::OW;
    const uint32_t lane_off = uint32_t(q * 32) << 16;
    uint32_t zc = 0, it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
      const int h = tile / nB, bt = tile % nB;
      const int ob = it % NO;
      const uint32_t on = it / NO;
      for (int c = 0; c < nE; ++c, ++zc) {
        const uint32_t zb = zc & 1;
        if (!(ok = mbar_wait(&z_full[zb], (zc >> 1) & 1, ctx))) break;
        tc_fence_after();
        const uint32_t zaddr = tmem + lane_off + C::TMEM_Z + zb * ET + j * SW;
        // H for these SW columns is packed two per column into the first SW/2 columns of
        // the slice, which this warp has just read.
        if constexpr (SW == 32) {
          uint32_t v[32], p[16];
          tmem_ld32_sync(zaddr, v);
#pragma unroll
          for (int i = 0; i < 16; ++i)
            p[i] = Pack<T>::pack(act_fwd<T, ACT>(__uint_as_float(v[2 * i])),
                                 act_fwd<T, ACT>(__uint_as_float(v[2 * i + 1])));
          tmem_st16(zaddr, p);
        } else {
          uint32_t v[16], p[8];
          tmem_ld16_sync(zaddr, v);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            p[i] = Pack<T>::pack(act_fwd<T, ACT>(__uint_as_float(v[2 * i])),
                                 act_fwd<T, ACT>(__uint_as_float(v[2 * i + 1])));
          tmem_st8(zaddr, p);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&h_full[zb]);
      }
      if (!ok) break;
      // Epilogue: O (fp32, TMEM) -> input dtype -> global, 16-byte stores per row.
      if (!(ok = mbar_wait(&o_full[ob], on & 1, ctx))) break;
      tc_fence_after();
      const int row = bt * BM + q * 32 + lane;
      T* orow = O + (size_t(h) * B + row) * D;
      const uint32_t oaddr = tmem + lane_off + C::TMEM_O + ob * DP + j * OW;
#pragma unroll
      for (int u = 0; u < (OW + 31) / 32; ++u) {
        constexpr int NC = OW < 32 ? OW : 32;
        const int col0 = j * OW + u * NC;
        uint32_t p[NC / 2];
        if constexpr (NC == 32) {
          uint32_t v[32];
          tmem_ld32_sync(oaddr + u * 32, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) p[i] = Pack<T>::pack(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
        } else {
          uint32_t v[16];
          tmem_ld16_sync(oaddr, v);
#pragma unroll
          for (int i = 0; i < 8; ++i) p[i] = Pack<T>::pack(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
        }
        if (row < B) {
          uint4* dst = reinterpret_cast<uint4*>(orow + col0);
#pragma unroll
          for (int i = 0; i < NC / 8; ++i)
            if (col0 + 8 * (i + 1) <= D) dst[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[ob]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

template <int DP, typename T, int ACT>
static cudaError_t launch_fwd_t(const FwdLaunch& a) {
  using C = FwdCfg<DP>;
  auto kern = fmlp_fwd_kernel<DP, T, ACT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  kern<<<a.grid, C::NUM_THREADS, C::SMEM, a.stream>>>(a.tm_x, a.tm_w1, a.tm_w2,
                                                      reinterpret_cast<T*>(a.o), a.H, a.B, a.D,
                                                      a.E, a.status);
  return cudaGetLastError();
}

template <int DP, typename T>
static cudaError_t launch_fwd_act(const FwdLaunch& a) {
  switch (a.act) {
    case kLeakyRelu: return launch_fwd_t<DP, T, kLeakyRelu>(a);
    case kSilu: return launch_fwd_t<DP, T, kSilu>(a);
    case kSigmoid: return launch_fwd_t<DP, T, kSigmoid>(a);
    default: return launch_fwd_t<DP, T, kLinear>(a);
  }
}

template <int DP>
static cudaError_t launch_fwd_dt(const FwdLaunch& a) {
  return a.bf16 ? launch_fwd_act<DP, __nv_bfloat16>(a) : launch_fwd_act<DP, __half>(a);
}

int fwd_smem_bytes(int dp) {
  switch (dp) {
    case 64: return FwdCfg<64>::SMEM;
    case 128: return FwdCfg<128>::SMEM;
    case 256: return FwdCfg<256>::SMEM;
  }
  return -1;
}

cudaError_t launch_fwd(const FwdLaunch& a) {
  switch (a.dp) {
    case 64:
    case 128: return launch_fwd_pair(a);
    case 256: return a.shared_x ? cudaErrorNotSupported : launch_fwd_dt<256>(a);
  }
  return cudaErrorInvalidValue;
}

}  // namespace fmlp
