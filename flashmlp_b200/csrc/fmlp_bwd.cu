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
//   Z^T  = W1c^T[smem] @ X_b^T[smem]     SS  M=128(e) N=128(b) K=D
//   dH^T = W2c  [smem] @ dO_b^T[smem]    SS  M=128(e) N=128(b) K=D
//   dW2   += H^T [tmem] @ dO_b[smem]     TS  M=128(e) N=DP     K=128(b)
//   dW1^T += dZ^T[tmem] @ X_b [smem]     TS  M=128(e) N=DP     K=128(b)
// dX program:
//   Z  = X_b [smem] @ W1c [smem]         SS  M=128(b) N=64(e)  K=D
//   dH = dO_b[smem] @ W2c^T[smem]        SS  M=128(b) N=64(e)  K=D
//   dX += dZ[tmem] @ W1c^T[smem]         TS  M=128(b) N=DP     K=64(e)
#include "fmlp_kernels.h"
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
  // TMEM columns
  static constexpr int X_TM_DX = 0;        // dX accumulator, DP columns
  static constexpr int X_TM_Z = DP;        // 2 buffers x (Z 64 | dH 64)
  static constexpr int W_TM_DW1 = 0;       // dW1^T accumulator, DP columns
  static constexpr int W_TM_DW2 = DP;      // dW2 accumulator, DP columns
  static constexpr int W_TM_ZT = 2 * DP;   // Z^T 128 columns (H^T packed in place)
  static constexpr int W_TM_DHT = 2 * DP + 128;  // dH^T 128 columns (dZ^T packed in place)
  static_assert(X_TM_Z + 2 * 128 <= TMEM_COLS, "TMEM budget (dX)");
  static_assert(W_TM_DHT + 128 <= TMEM_COLS, "TMEM budget (dW)");
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr int NUM_THREADS = 320;
};

template <typename T, int ACT>
__device__ __forceinline__ float act_h(float z) {
  if constexpr (ACT == kLeakyRelu) {
    return fmaxf(z, 0.01f * z);
  } else if constexpr (ACT == kSilu) {
    return z * sigmoid_fast(z);
  } else if constexpr (ACT == kSigmoid) {
    return sigmoid_fast(z);
  } else {
    return z;
  }
}

// Given z and dh (fp32), returns h = act(z) and dz = dh * act'(z) (both unrounded fp32,
// except that the derivative is formed from the rounded h where the reference does so).
template <typename T, int ACT>
__device__ __forceinline__ void act_bwd(float z, float dh, float& h, float& dz) {
  if constexpr (ACT == kLeakyRelu) {
    h = fmaxf(z, 0.01f * z);
    dz = dh * (z >= 0.f ? 1.0f : 0.01f);  // flashmlp.py:33-34, :227-228
  } else if constexpr (ACT == kSilu) {
    const float s = sigmoid_fast(z);
    h = z * s;
    const float hr = Pack<T>::round(h);
    dz = dh * (s + hr * (1.0f - s));  // d_silu(z, h) with rounded h, flashmlp.py:43-46
  } else if constexpr (ACT == kSigmoid) {
    h = sigmoid_fast(z);
    const float hr = Pack<T>::round(h);
    // dh * sig * (1 - sig) with sig the rounded h; (1 - sig) is formed in the input dtype
    // as in flashmlp.py:232-233.
    dz = (dh * hr) * Pack<T>::round(1.0f - hr);
  } else {
    h = z;
    dz = dh;
  }
}

template <int DP, typename T, int ACT>
__global__ void __launch_bounds__(320, 1)
    fmlp_bwd_kernel(const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_w1,
                    const __grid_constant__ CUtensorMap tm_w2,
                    const __grid_constant__ CUtensorMap tm_w2w, T* __restrict__ dX,
                    T* __restrict__ dW1, T* __restrict__ dW2, int H, int B, int D, int E,
                    uint32_t* status) {
  using C = BwdCfg<DP>;
  constexpr int BM = C::BM;
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

  // Barrier assignment (both program kinds use the same slots differently).
  uint64_t* in_full = bars + 0;        // dX: X_b+dO_b ; dW: W1c+W2c
  uint64_t* ring_full = bars + 1;      // up to 4: dX: W stages ; dW: X/dO stages
  uint64_t* ring_empty = bars + 5;     // up to 4
  uint64_t* s_full = bars + 9;         // 2: products ready for the activation warps
  uint64_t* hz_full = bars + 11;       // 2: packed operands written back to TMEM
  uint64_t* acc_full = bars + 13;      // accumulators final
  uint64_t* done_bar = bars + 14;      // all MMAs retired

  if (threadIdx.x == 0) {
    misc[1] = 0;
    misc[2] = 0;
    mbar_init(in_full, 1);
    for (int i = 0; i < 4; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&hz_full[i], 8);
    }
    mbar_init(acc_full, 1);
    mbar_init(done_bar, 1);
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
    } else if (warp == 1) {
      if (lane == 0) {
        constexpr uint32_t idesc_s = make_idesc_f16(kBF, 128, 128, true, false);  // A MN, B K
        constexpr uint32_t idesc_s2 = make_idesc_f16(kBF, 128, 128, false, false); // A K, B K
        constexpr uint32_t idesc_w = make_idesc_f16(kBF, 128, DP, false, true);   // A tmem, B MN
        const int nK = (D + 15) / 16;
        const uint32_t w1a = smem_u32(sW1), w2a = smem_u32(sW2);
        bool ok = mbar_wait(in_full, 0, ctx);
        tc_fence_after();
        for (int bt = 0; bt < nB && ok; ++bt) {
          const int s = bt % XDS;
          if (!(ok = mbar_wait(&ring_full[s], (bt / XDS) & 1, ctx))) break;
          tc_fence_after();
          const uint32_t xa = smem_u32(sX + s * C::TILE_BYTES);
          const uint32_t da = smem_u32(sDO + s * C::TILE_BYTES);
          // Z^T = W1c^T @ X_b^T ; dH^T = W2c @ dO_b^T
          for (int k = 0; k < nK; ++k) {
            const uint64_t a1 = make_sdesc_sw128(w1a + k * 2048, DP * 128, 1024);
            const uint64_t bx = make_sdesc_sw128(xa + (k >> 2) * (BM * 128) + (k & 3) * 32, 16, 1024);
            mma_ss(tmem + C::W_TM_ZT, a1, bx, idesc_s, k > 0 ? 1u : 0u);
          }
          for (int k = 0; k < nK; ++k) {
            const uint64_t a2 = make_sdesc_sw128(w2a + (k >> 2) * (128 * 128) + (k & 3) * 32, 16, 1024);
            const uint64_t bd = make_sdesc_sw128(da + (k >> 2) * (BM * 128) + (k & 3) * 32, 16, 1024);
            mma_ss(tmem + C::W_TM_DHT, a2, bd, idesc_s2, k > 0 ? 1u : 0u);
          }
          mma_commit(&s_full[0]);
          if (!(ok = mbar_wait(&hz_full[0], bt & 1, ctx))) break;
          tc_fence_after();
          // dW2 += H^T @ dO_b ; dW1^T += dZ^T @ X_b   (K = 128 rows of the tile)
          for (int k = 0; k < BM / 16; ++k) {
            const int hf = k >> 2;
            const uint32_t acol = hf * 64 + (k & 3) * 8;
            const uint64_t bd = make_sdesc_sw128(da + k * 2048, BM * 128, 1024);
            const uint64_t bx = make_sdesc_sw128(xa + k * 2048, BM * 128, 1024);
            const uint32_t acc = (bt > 0 || k > 0) ? 1u : 0u;
            mma_ts(tmem + C::W_TM_DW2, tmem + C::W_TM_ZT + acol, bd, idesc_w, acc);
            mma_ts(tmem + C::W_TM_DW1, tmem + C::W_TM_DHT + acol, bx, idesc_w, acc);
          }
          mma_commit(&ring_empty[s]);
        }
        if (ok) mma_commit(acc_full);
        mma_commit(done_bar);
        mbar_wait(done_bar, 0, drain);
      }
    } else {
      const int q = warp & 3;
      const int hf = (warp - 2) >> 2;
      const uint32_t lane_off = uint32_t(q * 32) << 16;
      bool ok = true;
      for (int bt = 0; bt < nB && ok; ++bt) {
        if (!(ok = mbar_wait(&s_full[0], bt & 1, ctx))) break;
        tc_fence_after();
        const uint32_t zt = tmem + lane_off + C::W_TM_ZT + 64 * hf;
        const uint32_t dt = tmem + lane_off + C::W_TM_DHT + 64 * hf;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint32_t vz[32], vd[32];
          tmem_ld32_sync(zt + 32 * j, vz);
          tmem_ld32_sync(dt + 32 * j, vd);
          uint32_t ph[16], pd[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float h0, h1, d0, d1;
            act_bwd<T, ACT>(__uint_as_float(vz[2 * i]), __uint_as_float(vd[2 * i]), h0, d0);
            act_bwd<T, ACT>(__uint_as_float(vz[2 * i + 1]), __uint_as_float(vd[2 * i + 1]), h1, d1);
            ph[i] = Pack<T>::pack(h0, h1);
            pd[i] = Pack<T>::pack(d0, d1);
          }
          tmem_st16(zt + 16 * j, ph);
          tmem_st16(dt + 16 * j, pd);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&hz_full[0]);
      }
      if (ok && (ok = mbar_wait(acc_full, 0, ctx))) {
        tc_fence_after();
        const int e = c * 128 + q * 32 + lane;
        // dW1^T rows are E, columns D: dW1[h, d, e]. Lanes hold consecutive e, so each
        // column d is one coalesced 64-byte store across the warp.
#pragma unroll
        for (int j = 0; j < (DP / 2) / 32; ++j) {
          const int col0 = hf * (DP / 2) + 32 * j;
          uint32_t v[32];
          tmem_ld32_sync(tmem + lane_off + C::W_TM_DW1 + col0, v);
          if (e < E) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int d = col0 + i;
              if (d < D) {
                const uint32_t pk = Pack<T>::pack(__uint_as_float(v[i]), 0.f);
                reinterpret_cast<uint16_t*>(dW1)[(size_t(h) * D + d) * E + e] = uint16_t(pk & 0xFFFFu);
              }
            }
          }
        }
        T* w2row = dW2 + (size_t(h) * E + e) * D;
#pragma unroll
        for (int j = 0; j < (DP / 2) / 32; ++j) {
          const int col0 = hf * (DP / 2) + 32 * j;
          uint32_t v[32];
          tmem_ld32_sync(tmem + lane_off + C::W_TM_DW2 + col0, v);
          if (e < E && col0 < D) {
            uint32_t p[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              p[i] = Pack<T>::pack(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
            uint4* dst = reinterpret_cast<uint4*>(w2row + col0);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (col0 + 8 * (i + 1) <= D) dst[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
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
      if (lane == 0) {
        constexpr uint32_t idesc_z = make_idesc_f16(kBF, 128, 64, false, true);   // A K, B MN
        constexpr uint32_t idesc_h = make_idesc_f16(kBF, 128, 64, false, false);  // A K, B K
        constexpr uint32_t idesc_x = make_idesc_f16(kBF, 128, DP, false, false);  // A tmem, B K
        const int nK = (D + 15) / 16;
        const uint32_t xa = smem_u32(sX), da = smem_u32(sDO);
        bool ok = mbar_wait(in_full, 0, ctx);
        tc_fence_after();
        auto dx_step = [&](int cc) -> bool {
          const uint32_t zb = cc & 1;
          if (!mbar_wait(&hz_full[zb], (cc >> 1) & 1, ctx)) return false;
          tc_fence_after();
          const int s = cc % WSX;
          const uint32_t wa = smem_u32(sW1 + s * C::W1X_BYTES);
          const uint32_t zbase = tmem + C::X_TM_Z + zb * 128;
          for (int k = 0; k < 4; ++k) {
            const uint32_t acol = (k >> 1) * 32 + (k & 1) * 8;
            const uint64_t bd = make_sdesc_sw128(wa + k * 32, 16, 1024);
            mma_ts(tmem + C::X_TM_DX, zbase + acol, bd, idesc_x, (cc > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&ring_empty[s]);
          return true;
        };
        for (int c = 0; c < nEx && ok; ++c) {
          const int s = c % WSX;
          if (!(ok = mbar_wait(&ring_full[s], (c / WSX) & 1, ctx))) break;
          tc_fence_after();
          const uint32_t zb = c & 1;
          const uint32_t zbase = tmem + C::X_TM_Z + zb * 128;
          const uint32_t w1a = smem_u32(sW1 + s * C::W1X_BYTES);
          const uint32_t w2a = smem_u32(sW2 + s * C::W2X_BYTES);
          for (int k = 0; k < nK; ++k) {
            const uint64_t ad = make_sdesc_sw128(xa + (k >> 2) * (BM * 128) + (k & 3) * 32, 16, 1024);
            const uint64_t bd = make_sdesc_sw128(w1a + k * 2048, DP * 128, 1024);
            mma_ss(zbase, ad, bd, idesc_z, k > 0 ? 1u : 0u);
          }
          for (int k = 0; k < nK; ++k) {
            const uint64_t ad = make_sdesc_sw128(da + (k >> 2) * (BM * 128) + (k & 3) * 32, 16, 1024);
            const uint64_t bd = make_sdesc_sw128(w2a + (k >> 2) * (64 * 128) + (k & 3) * 32, 16, 1024);
            mma_ss(zbase + 64, ad, bd, idesc_h, k > 0 ? 1u : 0u);
          }
          mma_commit(&s_full[zb]);
          if (c > 0) ok = dx_step(c - 1);
        }
        if (ok && nEx > 0) ok = dx_step(nEx - 1);
        if (ok) mma_commit(acc_full);
        mma_commit(done_bar);
        mbar_wait(done_bar, 0, drain);
      }
    } else {
      const int q = warp & 3;
      const int hf = (warp - 2) >> 2;
      const uint32_t lane_off = uint32_t(q * 32) << 16;
      bool ok = true;
      for (int c = 0; c < nEx && ok; ++c) {
        const uint32_t zb = c & 1;
        if (!(ok = mbar_wait(&s_full[zb], (c >> 1) & 1, ctx))) break;
        tc_fence_after();
        const uint32_t za = tmem + lane_off + C::X_TM_Z + zb * 128 + 32 * hf;
        uint32_t vz[32], vd[32];
        tmem_ld32_sync(za, vz);
        tmem_ld32_sync(za + 64, vd);
        uint32_t pd[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float h0, h1, d0, d1;
          act_bwd<T, ACT>(__uint_as_float(vz[2 * i]), __uint_as_float(vd[2 * i]), h0, d0);
          act_bwd<T, ACT>(__uint_as_float(vz[2 * i + 1]), __uint_as_float(vd[2 * i + 1]), h1, d1);
          pd[i] = Pack<T>::pack(d0, d1);
        }
        tmem_st16(za, pd);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&hz_full[zb]);
      }
      if (ok && (ok = mbar_wait(acc_full, 0, ctx))) {
        tc_fence_after();
        const int row = bt * BM + q * 32 + lane;
        T* xrow = dX + (size_t(h) * B + row) * D;
#pragma unroll
        for (int j = 0; j < (DP / 2) / 32; ++j) {
          const int col0 = hf * (DP / 2) + 32 * j;
          uint32_t v[32];
          tmem_ld32_sync(tmem + lane_off + C::X_TM_DX + col0, v);
          if (row < B && col0 < D) {
            uint32_t p[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              p[i] = Pack<T>::pack(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
            uint4* dst = reinterpret_cast<uint4*>(xrow + col0);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (col0 + 8 * (i + 1) <= D) dst[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
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
