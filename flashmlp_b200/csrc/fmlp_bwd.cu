// Unified fused multi-head MLP backward for sm_100a.
//
// Replaces the Triton kernel `flashmlp_bwd_kernel` (flashmlp.py:341-421) and its helpers
// `_flashmlp_bwd_dx` (flashmlp.py:165-244) and `_flashmlp_bwd_dw1w2` (flashmlp.py:247-329).
// One launch holds two kinds of programs, split by program id as in the reference:
//   * dW programs, one per (head, 128-wide E chunk): own dW1[h,:,chunk] and dW2[h,chunk,:]
//     and loop over every B tile of the head (deterministic, no atomics on outputs);
//   * dX programs, one per (head, 128-row B tile): own dX[h,tile,:] and loop over E.
// All dW programs come first in program-id order so the long ones start first.
// Both recompute Z = X@W1 and H = act(Z) per chunk and form dH = dO@W2^T and
// dZ = dH * act'(Z) in fp32; H and dZ are rounded to the input dtype before they enter
// the next products (flashmlp.py:212-235, :294-320).
//
// dW program (transposed so H^T and dZ^T land in TMEM as K-major A operands):
//   Z^T  = W1c^T[smem] @ X_b^T[smem]     SS  M=128(e) N=128(b) K=DP
//   dH^T = W2c  [smem] @ dO_b^T[smem]    SS  M=128(e) N=128(b) K=DP
//   dW2   += H^T [tmem] @ dO_b[smem]     TS  M=128(e) N=DP     K=128(b)
//   dW1^T += dZ^T[tmem] @ X_b [smem]     TS  M=128(e) N=DP     K=128(b)
// The activation runs in two phases so the tensor pipe is not idle while it runs:
// H^T = act(Z^T) as soon as Z^T is done (dW2 can start), then dZ^T once dH^T is done.
// dX program (X_b and dO_b are copied once into TMEM, so every MMA reads only weights
// from shared memory):
//   Z  = X_b [tmem] @ W1c [smem]         TS  M=128(b) N=64(e)  K=DP
//   dH = dO_b[tmem] @ W2c^T[smem]        TS  M=128(b) N=64(e)  K=DP
//   dX += dZ[tmem] @ W1c^T[smem]         TS  M=128(b) N=DP     K=64(e)
#include "fmlp_kernels.h"
#include "fmlp_act.cuh"
#include "fmlp_ptx.cuh"

namespace fmlp {

template <int DP>
struct BwdCfg {
  static constexpr int BM = kRows;
  static constexpr int TILE_BYTES = BM * DP * 2;  // one 128-row tile of X or dO
  // dX program
  static constexpr int ETX = kBwdEtX;
  static constexpr int WSX = 4;
  static constexpr int W1X_BYTES = DP * ETX * 2;
  static constexpr int W2X_BYTES = ETX * DP * 2;
  static constexpr int X_OFF_X = 0;
  static constexpr int X_OFF_DO = TILE_BYTES;
  static constexpr int X_OFF_W1 = 2 * TILE_BYTES;
  static constexpr int X_OFF_W2 = X_OFF_W1 + WSX * W1X_BYTES;
  static constexpr int X_END = X_OFF_W2 + WSX * W2X_BYTES;
  // dW program
  static constexpr int ETW = kBwdEtW;
  static constexpr int XDS = 2;
  static constexpr int W1W_BYTES = DP * ETW * 2;
  static constexpr int W2W_BYTES = ETW * DP * 2;
  static constexpr int W_OFF_W1 = 0;
  static constexpr int W_OFF_W2 = W1W_BYTES;
  static constexpr int W_OFF_X = W1W_BYTES + W2W_BYTES;
  static constexpr int W_OFF_DO = W_OFF_X + XDS * TILE_BYTES;
  static constexpr int W_END = W_OFF_DO + XDS * TILE_BYTES;
  static constexpr int OFF_BAR = X_END > W_END ? X_END : W_END;
  static constexpr int NBAR = 24;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  // + alignment slack; at least 120 KB so that only one CTA (and one 512-column TMEM
  // allocation) is ever resident per SM.
  static constexpr int SMEM_USED = OFF_MISC + 16 + 1024;
  static constexpr int SMEM = SMEM_USED > 120 * 1024 ? SMEM_USED : 120 * 1024;
  static constexpr int TMEM_COLS = 512;
  // TMEM columns, dX program
  static constexpr int X_TM_X = 0;            // X_b packed, DP/2 columns
  static constexpr int X_TM_DO = DP / 2;      // dO_b packed, DP/2 columns
  static constexpr int X_TM_DX = DP;          // dX accumulator, DP columns
  static constexpr int X_TM_Z = 2 * DP;       // 2 buffers x (Z 64 | dH 64)
  // TMEM columns, dW program
  static constexpr int W_TM_DW1 = 0;             // dW1^T accumulator, DP columns
  static constexpr int W_TM_DW2 = DP;            // dW2 accumulator, DP columns
  static constexpr int W_TM_ZT = 2 * DP;         // Z^T 128 columns (H^T packed in place)
  static constexpr int W_TM_DHT = 2 * DP + 128;  // dH^T 128 columns (dZ^T packed in place)
  static_assert(X_TM_Z + 2 * 128 <= TMEM_COLS, "TMEM budget (dX)");
  static_assert(W_TM_DHT + 128 <= TMEM_COLS, "TMEM budget (dW)");
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr int NUM_ACT_WARPS = 16;  // 4 per TMEM lane quadrant
  static constexpr int FIRST_ACT_WARP = 3;  // warp 0 TMA, warps 1-2 MMA
  static constexpr int NUM_THREADS = 32 * (FIRST_ACT_WARP + NUM_ACT_WARPS);
};

template <int DP, typename T, int ACT>
__global__ void __launch_bounds__(608, 1)
    fmlp_bwd_kernel(const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_w1,
                    const __grid_constant__ CUtensorMap tm_w2,
                    const __grid_constant__ CUtensorMap tm_w2w, T* __restrict__ dX,
                    T* __restrict__ dW1, T* __restrict__ dW2, int H, int B, int D, int E,
                    uint32_t* status) {
  using C = BwdCfg<DP>;
  using St = ActState<T, ACT>;
  constexpr int BM = C::BM;
  constexpr int NACT = C::NUM_ACT_WARPS;
  constexpr bool kBF = Pack<T>::kBF16;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_flag = misc + 1;  // misc[2] stays 0: "never abort" flag for drains
  const WaitCtx ctx{abort_flag, status};
  const WaitCtx drain{misc + 2, status};

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nB = (B + BM - 1) / BM;
  const int nEw = (E + C::ETW - 1) / C::ETW;
  const int nEx = (E + C::ETX - 1) / C::ETX;
  const bool is_dw = int(blockIdx.x) < H * nEw;
  int h, idx;
  if (is_dw) {
    h = blockIdx.x / nEw;
    idx = blockIdx.x % nEw;  // E chunk
  } else {
    const int p = blockIdx.x - H * nEw;
    h = p / nB;
    idx = p % nB;  // B tile
  }

  // Barriers (both program kinds use the same slots differently).
  uint64_t* in_full = bars + 0;     // dX: X_b+dO_b loaded ; dW: W1c+W2c loaded
  uint64_t* ring_full = bars + 1;   // 4: dX: W stages ; dW: X/dO stages
  uint64_t* ring_empty = bars + 5;  // 4
  uint64_t* p_full = bars + 9;      // 2: dX: Z,dH of chunk ready ; dW: [0] Z^T, [1] dH^T ready
  uint64_t* a_full = bars + 11;     // 2: dX: dZ packed ; dW: [0] H^T packed, [1] dZ^T packed
  uint64_t* acc_full = bars + 13;   // accumulators final
  uint64_t* xt_full = bars + 14;    // dX: X_b, dO_b copied into TMEM
  uint64_t* done_bar = bars + 15;   // 2: all MMAs of MMA warp 1 / 2 retired
  uint64_t* zfree = bars + 17;      // 2: dX: dZ of buffer read by its dX product

  if (threadIdx.x == 0) {
    misc[1] = 0;
    misc[2] = 0;
    mbar_init(in_full, 1);
    for (int i = 0; i < 4; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], 2);  // released by both MMA warps
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], 1);
      mbar_init(&a_full[i], NACT);
      mbar_init(&done_bar[i], 1);
      mbar_init(&zfree[i], 1);
    }
    mbar_init(acc_full, is_dw ? 2 : 1);  // dW: dW2 (warp 1) and dW1^T (warp 2)
    mbar_init(xt_full, NACT);
    fence_mbar_init();
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_w1);
    tma_prefetch_desc(is_dw ? &tm_w2w : &tm_w2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Activation warps: warp (q, j) owns TMEM lanes [32q, 32q+32) and column slice j.
  const int q = warp & 3;
  const int j = (warp - C::FIRST_ACT_WARP) >> 2;
  const uint32_t lane_off = uint32_t(q * 32) << 16;

  if (is_dw) {
    // ==================================================================== dW program
    const int c = idx;
    uint8_t* sW1 = smem + C::W_OFF_W1;
    uint8_t* sW2 = smem + C::W_OFF_W2;
    uint8_t* sX = smem + C::W_OFF_X;
    uint8_t* sDO = smem + C::W_OFF_DO;
    constexpr int XDS = C::XDS;
    if (warp == 0) {
      if (lane == 0) {
        mbar_arrive_expect_tx(in_full, C::W1W_BYTES + C::W2W_BYTES);
        for (int r = 0; r < 2; ++r)
          tma_load_3d(sW1 + r * DP * 128, &tm_w1, in_full, c * 128 + 64 * r, 0, h);
        for (int r = 0; r < DP / 64; ++r)
          tma_load_3d(sW2 + r * 128 * 128, &tm_w2w, in_full, 64 * r, c * 128, h);
        uint32_t nl = 0;  // X/dO stages issued
        for (int bt = 0; bt < nB; ++bt) {
          const int s = bt % XDS;
          const uint32_t n = bt / XDS;
          if (!mbar_wait(&ring_empty[s], (n & 1) ^ 1, ctx)) break;
          mbar_arrive_expect_tx(&ring_full[s], 2 * C::TILE_BYTES);
          for (int r = 0; r < DP / 64; ++r) {
            tma_load_3d(sX + s * C::TILE_BYTES + r * BM * 128, &tm_x, &ring_full[s], 64 * r, bt * BM, h);
            tma_load_3d(sDO + s * C::TILE_BYTES + r * BM * 128, &tm_do, &ring_full[s], 64 * r, bt * BM, h);
          }
          ++nl;
        }
        mbar_wait(in_full, 0, drain);
        for (uint32_t s = 0; s < XDS; ++s)
          if (nl > s) mbar_wait(&ring_full[s], ((nl - 1 - s) / XDS) & 1, drain);
      }
    } else if (warp == 1 || warp == 2) {
      // Two MMA warps, each owning one pair of products and its TMEM columns:
      //   warp 1: dW2(i) += H^T(i) @ dO_i, then Z^T(i+1)   (columns of Z^T and dW2)
      //   warp 2: dW1^T(i) += dZ^T(i) @ X_i, then dH^T(i+1) (columns of dH^T and dW1^T)
      // so while the activation warps compute H^T(i+1) the tensor pipe runs dW1^T(i) and
      // dH^T(i+1), and while they compute dZ^T(i) it runs dW2(i) and Z^T(i+1). Each warp's
      // overwrite of a TMEM region follows its own read of it (same-thread MMA order).
      const int m = warp - 1;
      constexpr uint32_t idesc_s = make_idesc_f16(kBF, 128, 128, true, false);   // A MN, B K
      constexpr uint32_t idesc_s2 = make_idesc_f16(kBF, 128, 128, false, false); // A K, B K
      constexpr uint32_t idesc_w = make_idesc_f16(kBF, 128, DP, false, true);    // A tmem, B MN
      // warp 1: A = W1c^T (MN-major), B = X tile (K-major), products into Z^T
      // warp 2: A = W2c (K-major),    B = dO tile (K-major), products into dH^T
      const uint64_t wdesc = m == 0 ? make_sdesc_sw128(smem_u32(sW1), DP * 128, 1024)
                                    : make_sdesc_sw128(smem_u32(sW2), 16, 1024);
      uint8_t* const sIn = m == 0 ? sX : sDO;    // tile read by this warp's first product
      uint8_t* const sAcc = m == 0 ? sDO : sX;   // tile read by this warp's dW product
      const uint32_t prod_col = m == 0 ? C::W_TM_ZT : C::W_TM_DHT;
      const uint32_t acc_col = m == 0 ? C::W_TM_DW2 : C::W_TM_DW1;
      auto issue_prod = [&](int bt) -> bool {  // Z^T(bt) or dH^T(bt)
        const int s = bt % XDS;
        if (!warp_wait(&ring_full[s], (bt / XDS) & 1, ctx)) return false;
        tc_fence_after();
        if (elect_one()) {
          const uint64_t bk = make_sdesc_sw128(smem_u32(sIn + s * C::TILE_BYTES), 16, 1024);
#pragma unroll
          for (int k = 0; k < DP / 16; ++k) {
            const uint32_t aoff = m == 0 ? k * 2048 : (k >> 2) * (128 * 128) + (k & 3) * 32;
            mma_ss(tmem + prod_col, sdesc_add(wdesc, aoff), sdesc_add(bk, (k >> 2) * (BM * 128) + (k & 3) * 32),
                   m == 0 ? idesc_s : idesc_s2, k > 0 ? 1u : 0u);
          }
          mma_commit(&p_full[m]);
        }
        __syncwarp();
        return true;
      };
      bool ok = warp_wait(in_full, 0, ctx);
      tc_fence_after();
      if (ok && nB > 0) ok = issue_prod(0);
      for (int bt = 0; bt < nB && ok; ++bt) {
        const int s = bt % XDS;
        // dW2 += H^T @ dO_b (warp 1) / dW1^T += dZ^T @ X_b (warp 2), K = the 128 tile rows;
        // the packed operand of B columns [16k, 16k+16) sits in slice k/2 at offset 8*(k%2).
        if (!(ok = warp_wait(&a_full[m], bt & 1, ctx))) break;
        tc_fence_after();
        if (elect_one()) {
          const uint64_t bm = make_sdesc_sw128(smem_u32(sAcc + s * C::TILE_BYTES), BM * 128, 1024);
          const uint32_t acc0 = bt > 0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < BM / 16; ++k)
            mma_ts(tmem + acc_col, tmem + prod_col + (k >> 1) * 32 + (k & 1) * 8, sdesc_add(bm, k * 2048),
                   idesc_w, k > 0 ? 1u : acc0);
          mma_commit(&ring_empty[s]);  // this warp is done with stage s
          if (bt + 1 == nB) mma_commit(acc_full);
        }
        __syncwarp();
        if (bt + 1 < nB && !(ok = issue_prod(bt + 1))) break;
      }
      if (elect_one()) mma_commit(&done_bar[m]);
      __syncwarp();
      warp_wait(&done_bar[m], 0, drain);
    } else {
      // Activation warps: slice j = B columns [32j, 32j+32) of Z^T / dH^T.
      const uint32_t zt = tmem + lane_off + C::W_TM_ZT + 32 * j;
      const uint32_t dt = tmem + lane_off + C::W_TM_DHT + 32 * j;
      bool ok = true;
      for (int bt = 0; bt < nB && ok; ++bt) {
        St st[32];
        // phase 1: H^T = act(Z^T), packed in place
        if (!(ok = mbar_wait(&p_full[0], bt & 1, ctx))) break;
        tc_fence_after();
        {
          uint32_t v[32], ph[16];
          tmem_ld32_sync(zt, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float h0 = act_forward<T, ACT>(__uint_as_float(v[2 * i]), st[2 * i]);
            const float h1 = act_forward<T, ACT>(__uint_as_float(v[2 * i + 1]), st[2 * i + 1]);
            ph[i] = Pack<T>::pack(h0, h1);
          }
          tmem_st16(zt, ph);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[0]);
        // phase 2: dZ^T = dH^T * act'(Z^T), packed in place (two halves of 16 columns)
        if (!(ok = mbar_wait(&p_full[1], bt & 1, ctx))) break;
        tc_fence_after();
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          uint32_t v[16], pd[8];
          tmem_ld16_sync(dt + 16 * u, v);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            pd[i] = Pack<T>::pack(act_grad<T, ACT>(__uint_as_float(v[2 * i]), st[16 * u + 2 * i]),
                                  act_grad<T, ACT>(__uint_as_float(v[2 * i + 1]), st[16 * u + 2 * i + 1]));
          tmem_st8(dt + 8 * u, pd);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[1]);
      }
      if (ok && (ok = mbar_wait(acc_full, 0, ctx))) {
        tc_fence_after();
        const int e = c * 128 + q * 32 + lane;
        constexpr int OW = DP / 4;  // accumulator columns per warp
        const int col0 = j * OW;
        // dW1^T rows are E, columns D: dW1[h, d, e]. Lanes hold consecutive e, so each
        // column d is one coalesced 64-byte store across the warp.
#pragma unroll
        for (int u = 0; u < OW / 16; ++u) {
          uint32_t v[16];
          tmem_ld16_sync(tmem + lane_off + C::W_TM_DW1 + col0 + 16 * u, v);
          if (e < E) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int d = col0 + 16 * u + i;
              if (d < D) {
                const uint32_t pk = Pack<T>::pack(__uint_as_float(v[i]), 0.f);
                reinterpret_cast<uint16_t*>(dW1)[(size_t(h) * D + d) * E + e] = uint16_t(pk & 0xFFFFu);
              }
            }
          }
        }
        T* w2row = dW2 + (size_t(h) * E + e) * D;
#pragma unroll
        for (int u = 0; u < OW / 16; ++u) {
          uint32_t v[16], p[8];
          tmem_ld16_sync(tmem + lane_off + C::W_TM_DW2 + col0 + 16 * u, v);
#pragma unroll
          for (int i = 0; i < 8; ++i) p[i] = Pack<T>::pack(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
          const int cc = col0 + 16 * u;
          if (e < E) {
            uint4* dst = reinterpret_cast<uint4*>(w2row + cc);
            if (cc + 8 <= D) dst[0] = make_uint4(p[0], p[1], p[2], p[3]);
            if (cc + 16 <= D) dst[1] = make_uint4(p[4], p[5], p[6], p[7]);
          }
        }
      }
    }
  } else {
    // ==================================================================== dX program
    const int bt = idx;
    constexpr int WSX = C::WSX;
    uint8_t* sX = smem + C::X_OFF_X;
    uint8_t* sDO = smem + C::X_OFF_DO;
    uint8_t* sW1 = smem + C::X_OFF_W1;
    uint8_t* sW2 = smem + C::X_OFF_W2;
    if (warp == 0) {
      if (lane == 0) {
        mbar_arrive_expect_tx(in_full, 2 * C::TILE_BYTES);
        for (int r = 0; r < DP / 64; ++r) {
          tma_load_3d(sX + r * BM * 128, &tm_x, in_full, 64 * r, bt * BM, h);
          tma_load_3d(sDO + r * BM * 128, &tm_do, in_full, 64 * r, bt * BM, h);
        }
        uint32_t nl = 0;
        for (int c = 0; c < nEx; ++c) {
          const int s = c % WSX;
          const uint32_t n = c / WSX;
          if (!mbar_wait(&ring_empty[s], (n & 1) ^ 1, ctx)) break;
          mbar_arrive_expect_tx(&ring_full[s], C::W1X_BYTES + C::W2X_BYTES);
          tma_load_3d(sW1 + s * C::W1X_BYTES, &tm_w1, &ring_full[s], c * 64, 0, h);
          for (int r = 0; r < DP / 64; ++r)
            tma_load_3d(sW2 + s * C::W2X_BYTES + r * 64 * 128, &tm_w2, &ring_full[s], 64 * r, c * 64, h);
          ++nl;
        }
        mbar_wait(in_full, 0, drain);
        for (uint32_t s = 0; s < WSX; ++s)
          if (nl > s) mbar_wait(&ring_full[s], ((nl - 1 - s) / WSX) & 1, drain);
      }
    } else if (warp == 1) {
      // MMA warp 1: Z(c) = X_b @ W1c and dH(c) = dO_b @ W2c^T into buffer c%2, running
      // ahead of warp 2; before reusing a buffer it waits until warp 2's dX product has
      // read the dZ packed there (zfree).
      constexpr uint32_t idesc_z = make_idesc_f16(kBF, 128, 64, false, true);   // A tmem, B MN
      constexpr uint32_t idesc_h = make_idesc_f16(kBF, 128, 64, false, false);  // A tmem, B K
      bool ok = warp_wait(xt_full, 0, ctx);  // X_b, dO_b are in TMEM
      tc_fence_after();
      for (int c = 0; c < nEx && ok; ++c) {
        const int s = c % WSX;
        if (!(ok = warp_wait(&ring_full[s], (c / WSX) & 1, ctx))) break;
        if (c >= 2 && !(ok = warp_wait(&zfree[c & 1], ((c >> 1) - 1) & 1, ctx))) break;
        tc_fence_after();
        if (elect_one()) {
          const uint32_t zbase = tmem + C::X_TM_Z + (c & 1) * 128;
          const uint64_t w1m = make_sdesc_sw128(smem_u32(sW1 + s * C::W1X_BYTES), DP * 128, 1024);
          const uint64_t w2k = make_sdesc_sw128(smem_u32(sW2 + s * C::W2X_BYTES), 16, 1024);
#pragma unroll
          for (int k = 0; k < DP / 16; ++k)
            mma_ts(zbase, tmem + C::X_TM_X + 8 * k, sdesc_add(w1m, k * 2048), idesc_z, k > 0 ? 1u : 0u);
#pragma unroll
          for (int k = 0; k < DP / 16; ++k)
            mma_ts(zbase + 64, tmem + C::X_TM_DO + 8 * k,
                   sdesc_add(w2k, (k >> 2) * (64 * 128) + (k & 3) * 32), idesc_h, k > 0 ? 1u : 0u);
          mma_commit(&p_full[c & 1]);
          mma_commit(&ring_empty[s]);  // warp 1 is done with stage s
        }
        __syncwarp();
      }
      if (elect_one()) mma_commit(&done_bar[0]);
      __syncwarp();
      warp_wait(&done_bar[0], 0, drain);
    } else if (warp == 2) {
      // MMA warp 2: dX += dZ(c) @ W1c^T once the activation warps have packed dZ(c).
      constexpr uint32_t idesc_x = make_idesc_f16(kBF, 128, DP, false, false);  // A tmem, B K
      bool ok = true;
      for (int c = 0; c < nEx && ok; ++c) {
        const uint32_t zb = c & 1;
        if (!(ok = warp_wait(&a_full[zb], (c >> 1) & 1, ctx))) break;
        tc_fence_after();
        if (elect_one()) {
          const int s = c % WSX;
          const uint64_t wk = make_sdesc_sw128(smem_u32(sW1 + s * C::W1X_BYTES), 16, 1024);
          const uint32_t zbase = tmem + C::X_TM_Z + zb * 128;
          const uint32_t acc0 = c > 0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < 4; ++k)  // dZ of E columns [16k, 16k+16) is in slice k
            mma_ts(tmem + C::X_TM_DX, zbase + 16 * k, sdesc_add(wk, k * 32), idesc_x, k > 0 ? 1u : acc0);
          mma_commit(&zfree[zb]);
          mma_commit(&ring_empty[s]);  // warp 2 is done with stage s
          if (c + 1 == nEx) mma_commit(acc_full);
        }
        __syncwarp();
      }
      if (elect_one()) mma_commit(&done_bar[1]);
      __syncwarp();
      warp_wait(&done_bar[1], 0, drain);
    } else {
      bool ok = mbar_wait(in_full, 0, ctx);
      // Copy this warp's share of X_b and dO_b from the swizzled smem tiles into TMEM as
      // packed K-major A operands (column w holds elements 2w, 2w+1 of the row).
      if (ok) {
        const int r = q * 32 + lane;  // tile row == TMEM lane
        constexpr int WPW = DP / 8;   // 32-bit words per warp slice (DP/2 words per row)
        const int e0 = j * WPW * 2;   // first element of the slice
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const uint8_t* tile = t == 0 ? sX : sDO;
          uint32_t w[WPW];
#pragma unroll
          for (int g = 0; g < WPW / 4; ++g) {  // 16-byte chunks of 8 elements
            const int el = e0 + 8 * g;
            const int region = el >> 6, chunk = (el & 63) >> 3;
            const uint4 v = *reinterpret_cast<const uint4*>(tile + region * (BM * 128) + r * 128 +
                                                            ((chunk ^ (r & 7)) << 4));
            w[4 * g] = v.x, w[4 * g + 1] = v.y, w[4 * g + 2] = v.z, w[4 * g + 3] = v.w;
          }
          const uint32_t dst = tmem + lane_off + (t == 0 ? C::X_TM_X : C::X_TM_DO) + j * WPW;
          if constexpr (WPW == 16) {
            tmem_st16(dst, w);
          } else {
            tmem_st8(dst, w);
          }
        }
        tmem_wait_st();
        tc_fence_before();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(xt_full);
      // Per E chunk: slice j = E columns [16j, 16j+16) of Z and dH.
      for (int c = 0; c < nEx && ok; ++c) {
        const uint32_t zb = c & 1;
        if (!(ok = mbar_wait(&p_full[zb], (c >> 1) & 1, ctx))) break;
        tc_fence_after();
        const uint32_t za = tmem + lane_off + C::X_TM_Z + zb * 128 + 16 * j;
        uint32_t vz[16], vd[16], pd[8];
        tmem_ld16_sync(za, vz);
        tmem_ld16_sync(za + 64, vd);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          St s0, s1;
          act_forward<T, ACT>(__uint_as_float(vz[2 * i]), s0);
          act_forward<T, ACT>(__uint_as_float(vz[2 * i + 1]), s1);
          pd[i] = Pack<T>::pack(act_grad<T, ACT>(__uint_as_float(vd[2 * i]), s0),
                                act_grad<T, ACT>(__uint_as_float(vd[2 * i + 1]), s1));
        }
        tmem_st8(za, pd);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[zb]);
      }
      if (ok && (ok = mbar_wait(acc_full, 0, ctx))) {
        tc_fence_after();
        const int row = bt * BM + q * 32 + lane;
        T* xrow = dX + (size_t(h) * B + row) * D;
        constexpr int OW = DP / 4;
        const int col0 = j * OW;
#pragma unroll
        for (int u = 0; u < OW / 16; ++u) {
          uint32_t v[16], p[8];
          tmem_ld16_sync(tmem + lane_off + C::X_TM_DX + col0 + 16 * u, v);
#pragma unroll
          for (int i = 0; i < 8; ++i) p[i] = Pack<T>::pack(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
          const int cc = col0 + 16 * u;
          if (row < B) {
            uint4* dst = reinterpret_cast<uint4*>(xrow + cc);
            if (cc + 8 <= D) dst[0] = make_uint4(p[0], p[1], p[2], p[3]);
            if (cc + 16 <= D) dst[1] = make_uint4(p[4], p[5], p[6], p[7]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

template <int DP, typename T, int ACT>
static cudaError_t launch_bwd_t(const BwdLaunch& a) {
  using C = BwdCfg<DP>;
  auto kern = fmlp_bwd_kernel<DP, T, ACT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int nB = (a.B + kRows - 1) / kRows;
  const int nEw = (a.E + C::ETW - 1) / C::ETW;
  const long long grid = (long long)a.H * (nEw + nB);
  if (grid <= 0 || grid > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  kern<<<unsigned(grid), C::NUM_THREADS, C::SMEM, a.stream>>>(
      a.tm_x, a.tm_do, a.tm_w1, a.tm_w2, a.tm_w2w, reinterpret_cast<T*>(a.dx),
      reinterpret_cast<T*>(a.dw1), reinterpret_cast<T*>(a.dw2), a.H, a.B, a.D, a.E, a.status);
  return cudaGetLastError();
}

template <int DP, typename T>
static cudaError_t launch_bwd_act(const BwdLaunch& a) {
  switch (a.act) {
    case kLeakyRelu: return launch_bwd_t<DP, T, kLeakyRelu>(a);
    case kSilu: return launch_bwd_t<DP, T, kSilu>(a);
    case kSigmoid: return launch_bwd_t<DP, T, kSigmoid>(a);
    default: return launch_bwd_t<DP, T, kLinear>(a);
  }
}

template <int DP>
static cudaError_t launch_bwd_dt(const BwdLaunch& a) {
  return a.bf16 ? launch_bwd_act<DP, __nv_bfloat16>(a) : launch_bwd_act<DP, __half>(a);
}

int bwd_smem_bytes(int dp) {
  switch (dp) {
    case 64: return BwdCfg<64>::SMEM;
    case 128: return BwdCfg<128>::SMEM;
  }
  return -1;
}

cudaError_t launch_bwd(const BwdLaunch& a) {
  switch (a.dp) {
    case 64: return launch_bwd_dt<64>(a);
    case 128: return launch_bwd_dt<128>(a);
  }
  return cudaErrorNotSupported;
}

}  // namespace fmlp
