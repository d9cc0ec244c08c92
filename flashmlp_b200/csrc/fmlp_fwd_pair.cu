// Forward for D <= 128: two 128-row tiles (A, B) of one head per CTA share every W1/W2
// chunk, O = act(X @ W1) @ W2 (same math and rounding points as fmlp_fwd.cu, which
// replaces flashmlp_fwd_kernel, flashmlp.py:63-158).
//
// Why pairs: with one 128-row tile per CTA, each E chunk streams 2*ET*DP*2 bytes of
// weights through TMA for 4*128*ET*DP FLOPs, and the weight stream (not the tensor pipe
// or the activation) set the pace. Two tiles per chunk halve the bytes per FLOP and give
// the loads twice the time to land. They also give the tensor pipe independent work while
// one tile is being activated:
//   per tile t and chunk c, one MMA warp per tile issues:  G2_t(c)  G1_t(c+1)
//   activation warps alternate act_A(c), act_B(c), ...; while tile A is activated the
//   tensor pipe runs tile B's products and vice versa.
// G1_t(c+1) overwrites Z_t, which holds H_t(c) read by G2_t(c) issued just before by the
// same warp (MMAs from one thread execute in issue order).
//
// TMEM (DP=128): O_A [0,128) O_B [128,256) Z_A [256,384) Z_B [384,512).
// smem: X_A, X_B tiles + 2-stage W1 and W2 rings (DP=64: 4 stages).
//
// SX = true (shared input): X is one (B, D) matrix used by every head and the output is
// the mean over heads, O = (1/H) sum_h act(X @ W1[h]) @ W2[h] -- what the reference's
// FlashMLP computes for a 2-D input by expanding X to (H, B, D) and averaging the per-head
// outputs (flashmlp.py:603-614), without the H copies of X and of O. A work item is a
// pair of row tiles; its chunk loop runs over (head, E chunk), X stays in shared memory
// for all heads and O accumulates over all heads in TMEM; the epilogue scales by 1/H.
#include "fmlp_act.cuh"
#include "fmlp_kernels.h"
#include "fmlp_ptx.cuh"

namespace fmlp {

template <int DP>
struct FwdPairCfg {
  static_assert(DP == 64 || DP == 128, "pair kernel covers D <= 128");
  static constexpr int BM = kRows;
  static constexpr int ET = 128;
  static constexpr int WS = DP <= 64 ? 4 : 2;
  static constexpr int X_BYTES = BM * DP * 2;
  static constexpr int W1_BYTES = DP * ET * 2;
  static constexpr int W2_BYTES = ET * DP * 2;
  static constexpr int OFF_X = 0;
  static constexpr int OFF_W1 = OFF_X + 2 * X_BYTES;
  static constexpr int OFF_W2 = OFF_W1 + WS * W1_BYTES;
  static constexpr int OFF_BAR = OFF_W2 + WS * W2_BYTES;
  // x_full[2] x_empty[2] w1_full[WS] w1_empty[WS] w2_full[WS] w2_empty[WS]
  // z_full[2] h_full[2] o_full[2] o_empty[2] done[2]
  static constexpr int NBAR = 4 + 4 * WS + 8 + 2;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16 + 1024;
  static constexpr int SMEM = SMEM_USED > 120 * 1024 ? SMEM_USED : 120 * 1024;
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr int TMEM_O = 0;        // O_t at TMEM_O + t*DP
  static constexpr int TMEM_Z = 2 * DP;   // Z_t at TMEM_Z + t*ET
  static constexpr int TMEM_COLS = 512;
  static_assert(TMEM_Z + 2 * ET <= TMEM_COLS, "TMEM budget");
  static constexpr int NUM_ACT_WARPS = 16;
  static constexpr int FIRST_ACT_WARP = 3;  // warp 0 TMA, warps 1-2 MMA (tile A, tile B)
  static constexpr int NUM_THREADS = 32 * (FIRST_ACT_WARP + NUM_ACT_WARPS);
  static constexpr int SW = ET / 4;  // Z columns per activation warp
  static constexpr int OW = DP / 4;  // O columns per activation warp
};

template <int DP, typename T, int ACT, bool SX>
__global__ void __launch_bounds__(608, 1)
    fmlp_fwd_pair_kernel(const __grid_constant__ CUtensorMap tm_x,
                         const __grid_constant__ CUtensorMap tm_w1,
                         const __grid_constant__ CUtensorMap tm_w2, T* __restrict__ O, int H,
                         int B, int D, int E, uint32_t* status) {
  using C = FwdPairCfg<DP>;
  constexpr int ET = C::ET, WS = C::WS, BM = C::BM, SW = C::SW, OW = C::OW;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sX = smem + C::OFF_X;
  uint8_t* sW1 = smem + C::OFF_W1;
  uint8_t* sW2 = smem + C::OFF_W2;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* x_full = bars;
  uint64_t* x_empty = x_full + 2;
  uint64_t* w1_full = x_empty + 2;
  uint64_t* w1_empty = w1_full + WS;
  uint64_t* w2_full = w1_empty + WS;
  uint64_t* w2_empty = w2_full + WS;
  uint64_t* z_full = w2_empty + WS;
  uint64_t* h_full = z_full + 2;
  uint64_t* o_full = h_full + 2;
  uint64_t* o_empty = o_full + 2;
  uint64_t* done_bar = o_empty + 2;
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_flag = misc + 1;  // misc[2] stays 0: "never abort" flag for drains
  const WaitCtx ctx{abort_flag, status};
  const WaitCtx drain{misc + 2, status};

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nB = (B + BM - 1) / BM;
  const int nP = (nB + 1) / 2;  // row pairs per head
  const int nE = (E + ET - 1) / ET;
  const int nEv = SX ? H * nE : nE;  // chunks per work item: (head, chunk) pairs when SX
  const int nitems = SX ? nP : H * nP;

  if (threadIdx.x == 0) {
    misc[1] = 0;
    misc[2] = 0;
    for (int i = 0; i < 2; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
      mbar_init(&z_full[i], 1);
      mbar_init(&h_full[i], C::NUM_ACT_WARPS);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], C::NUM_ACT_WARPS);
    }
    for (int i = 0; i < WS; ++i) {
      mbar_init(&w1_full[i], 1);
      mbar_init(&w1_empty[i], 2);  // released by both MMA warps
      mbar_init(&w2_full[i], 1);
      mbar_init(&w2_empty[i], 2);
    }
    mbar_init(&done_bar[0], 1);
    mbar_init(&done_bar[1], 1);
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
      uint32_t c1 = 0, c2 = 0, it = 0;  // loads issued (W1, W2), pairs started
      uint32_t xl[2] = {0, 0};          // X loads issued per tile slot
      bool ok = true;
      for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x, ++it) {
        const int h = SX ? 0 : item / nP, pr = SX ? item : item % nP;
        for (int t = 0; t < 2 && ok; ++t) {
          if (!(ok = mbar_wait(&x_empty[t], (it & 1) ^ 1, ctx))) break;
          mbar_arrive_expect_tx(&x_full[t], C::X_BYTES);
          for (int r = 0; r < DP / 64; ++r)
            tma_load_3d(sX + t * C::X_BYTES + r * BM * 128, &tm_x, &x_full[t], 64 * r,
                        (2 * pr + t) * BM, h);
          ++xl[t];
        }
        for (int cv = 0; cv < nEv && ok; ++cv) {
          const int hw = SX ? cv / nE : h;  // head of the weights
          const int c = SX ? cv % nE : cv;
          {
            const int s = c1 % WS;
            if (!(ok = mbar_wait(&w1_empty[s], ((c1 / WS) & 1) ^ 1, ctx))) break;
            mbar_arrive_expect_tx(&w1_full[s], C::W1_BYTES);
            for (int r = 0; r < ET / 64; ++r)
              tma_load_3d(sW1 + s * C::W1_BYTES + r * DP * 128, &tm_w1, &w1_full[s], c * ET + 64 * r, 0, hw);
            ++c1;
          }
          {
            const int s = c2 % WS;
            if (!(ok = mbar_wait(&w2_empty[s], ((c2 / WS) & 1) ^ 1, ctx))) break;
            mbar_arrive_expect_tx(&w2_full[s], C::W2_BYTES);
            for (int r = 0; r < DP / 64; ++r)
              tma_load_3d(sW2 + s * C::W2_BYTES + r * ET * 128, &tm_w2, &w2_full[s], 64 * r, c * ET, hw);
            ++c2;
          }
        }
      }
      // Drain in-flight loads (matters only after an abort).
      for (uint32_t s = 0; s < WS; ++s) {
        if (c1 > s) mbar_wait(&w1_full[s], ((c1 - 1 - s) / WS) & 1, drain);
        if (c2 > s) mbar_wait(&w2_full[s], ((c2 - 1 - s) / WS) & 1, drain);
      }
      for (int t = 0; t < 2; ++t)
        if (xl[t] > 0) mbar_wait(&x_full[t], (xl[t] - 1) & 1, drain);
    }
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------------ MMA issuers
    // Warp 1 drives tile A, warp 2 tile B: while one waits for its activation warps, the
    // other keeps the tensor pipe fed. Their TMEM columns are disjoint; the weight stages
    // they share are released by both (count-2 empty barriers).
    const int t = warp - 1;
    constexpr bool kBF = Pack<T>::kBF16;
    constexpr uint32_t idesc1 = make_idesc_f16(kBF, BM, ET, false, true);
    constexpr uint32_t idesc2 = make_idesc_f16(kBF, BM, DP, false, true);
    const uint64_t xd = make_sdesc_sw128(smem_u32(sX) + t * C::X_BYTES, 16, 1024);
    const uint32_t sW1_a = smem_u32(sW1), sW2_a = smem_u32(sW2);
    const uint32_t z_tmem = tmem + C::TMEM_Z + t * ET;
    const uint32_t o_tmem = tmem + C::TMEM_O + t * DP;
    uint32_t c1 = 0, c2 = 0, it = 0;
    bool ok = true;

    // GEMM1 of this tile for the next W1 chunk (K over the padded DP, zero-filled).
    auto gemm1 = [&](bool last) -> bool {  // last: final GEMM1 of this pair for tile t
      const int s1 = c1 % WS;
      if (!warp_wait(&w1_full[s1], (c1 / WS) & 1, ctx)) return false;
      ++c1;
      tc_fence_after();
      if (elect_one()) {
        const uint64_t wd = make_sdesc_sw128(sW1_a + s1 * C::W1_BYTES, DP * 128, 1024);
#pragma unroll
        for (int k = 0; k < DP / 16; ++k)
          mma_ss(z_tmem, sdesc_add(xd, (k >> 2) * (BM * 128) + (k & 3) * 32), sdesc_add(wd, k * 2048),
                 idesc1, k > 0 ? 1u : 0u);
        mma_commit(&z_full[t]);
        mma_commit(&w1_empty[s1]);
        if (last) mma_commit(&x_empty[t]);  // every reader of X_t has been issued
      }
      __syncwarp();
      return true;
    };

    for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x, ++it) {
      if (!(ok = warp_wait(&x_full[t], it & 1, ctx))) break;
      if (!(ok = gemm1(nEv == 1))) break;
      for (int c = 0; c < nEv && ok; ++c) {
        const uint32_t zc = it * nEv + c;  // chunk index, for the z/h barrier parities
        const int s2 = c2 % WS;
        if (!(ok = warp_wait(&w2_full[s2], (c2 / WS) & 1, ctx))) break;
        ++c2;
        if (c == 0 && !(ok = warp_wait(&o_empty[t], (it & 1) ^ 1, ctx))) break;
        if (!(ok = warp_wait(&h_full[t], zc & 1, ctx))) break;
        tc_fence_after();
        if (elect_one()) {
          // GEMM2: O_t += H_t @ W2c. H of E columns [16k, 16k+16) was packed by the
          // activation warp owning that column slice, at the start of its slice.
          const uint64_t wd = make_sdesc_sw128(sW2_a + s2 * C::W2_BYTES, ET * 128, 1024);
          const uint32_t acc0 = c > 0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < ET / 16; ++k) {
            const int sl = (16 * k) / SW;
            const int within = 16 * k - sl * SW;
            mma_ts(o_tmem, z_tmem + sl * SW + within / 2, sdesc_add(wd, k * 2048), idesc2, k > 0 ? 1u : acc0);
          }
          mma_commit(&w2_empty[s2]);
          if (c + 1 == nEv) mma_commit(&o_full[t]);
        }
        __syncwarp();
        if (c + 1 < nEv && !(ok = gemm1(c + 2 == nEv))) break;  // overwrites Z_t after GEMM2 read H_t
      }
    }
    if (elect_one()) mma_commit(&done_bar[t]);
    __syncwarp();
    warp_wait(&done_bar[t], 0, drain);
  } else {
    // ------------------------------------------------------------------ activation + epilogue
    // 16 warps: warp (q, j) owns TMEM lanes [32q, 32q+32) and column slice j.
    const int q = warp & 3;
    const int j = (warp - C::FIRST_ACT_WARP) >> 2;
    const uint32_t lane_off = uint32_t(q * 32) << 16;
    uint32_t it = 0;
    bool ok = true;
    const float inv_h = SX ? 1.0f / float(H) : 1.0f;
    for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x, ++it) {
      const int h = SX ? 0 : item / nP, pr = SX ? item : item % nP;
      for (int c = 0; c < nEv && ok; ++c) {
        const uint32_t zc = it * nEv + c;
        for (int t = 0; t < 2; ++t) {
          if (!(ok = mbar_wait(&z_full[t], zc & 1, ctx))) break;
          tc_fence_after();
          const uint32_t za = tmem + lane_off + C::TMEM_Z + t * ET + j * SW;
          // H for these SW columns is packed two per column into the first SW/2 columns
          // of the slice, which this warp has just read.
          uint32_t v[SW], p[SW / 2];
          tmem_ld32_sync(za, v);
          act_pack<T, ACT, SW / 2>(v, p);
          tmem_st16(za, p);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&h_full[t]);
        }
      }
      // Epilogue per tile: O_t (fp32, TMEM) -> input dtype -> global.
      for (int t = 0; t < 2 && ok; ++t) {
        if (!(ok = mbar_wait(&o_full[t], it & 1, ctx))) break;
        tc_fence_after();
        const int row = (2 * pr + t) * BM + q * 32 + lane;
        T* orow = O + (size_t(h) * B + row) * D;
        const uint32_t oa = tmem + lane_off + C::TMEM_O + t * DP + j * OW;
        uint32_t v[OW], p[OW / 2];
        if constexpr (OW == 32) {
          tmem_ld32_sync(oa, v);
        } else {
          tmem_ld16_sync(oa, v);
        }
        if constexpr (SX) {
#pragma unroll
          for (int i = 0; i < OW; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * inv_h);
        }
        plain_pack<T, OW / 2>(v, p);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_empty[t]);  // O_t may be overwritten from here on
        if (row < B) {
          const int col0 = j * OW;
          uint4* dst = reinterpret_cast<uint4*>(orow + col0);
#pragma unroll
          for (int i = 0; i < OW / 8; ++i)
            if (col0 + 8 * (i + 1) <= D) dst[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

template <int DP, typename T, int ACT, bool SX>
static cudaError_t launch_pair_sx(const FwdLaunch& a) {
  using C = FwdPairCfg<DP>;
  auto kern = fmlp_fwd_pair_kernel<DP, T, ACT, SX>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const long long nB = (a.B + kRows - 1) / kRows;
  const long long items = (SX ? 1LL : (long long)a.H) * ((nB + 1) / 2);
  const int grid = int(items < a.sm_count ? items : a.sm_count);
  kern<<<grid, C::NUM_THREADS, C::SMEM, a.stream>>>(a.tm_x, a.tm_w1, a.tm_w2, reinterpret_cast<T*>(a.o),
                                                    a.H, a.B, a.D, a.E, a.status);
  return cudaGetLastError();
}

template <int DP, typename T, int ACT>
static cudaError_t launch_pair_t(const FwdLaunch& a) {
  return a.shared_x ? launch_pair_sx<DP, T, ACT, true>(a) : launch_pair_sx<DP, T, ACT, false>(a);
}

template <int DP, typename T>
static cudaError_t launch_pair_act(const FwdLaunch& a) {
  switch (a.act) {
    case kLeakyRelu: return launch_pair_t<DP, T, kLeakyRelu>(a);
    case kSilu: return launch_pair_t<DP, T, kSilu>(a);
    case kSigmoid: return launch_pair_t<DP, T, kSigmoid>(a);
    default: return launch_pair_t<DP, T, kLinear>(a);
  }
}

cudaError_t launch_fwd_pair(const FwdLaunch& a) {
  switch (a.dp) {
    case 64: return a.bf16 ? launch_pair_act<64, __nv_bfloat16>(a) : launch_pair_act<64, __half>(a);
    case 128: return a.bf16 ? launch_pair_act<128, __nv_bfloat16>(a) : launch_pair_act<128, __half>(a);
  }
  return cudaErrorInvalidValue;
}

}  // namespace fmlp
