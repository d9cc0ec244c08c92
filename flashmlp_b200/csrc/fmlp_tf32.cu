// fp32 inputs: forward and unified backward with TF32 tensor-core products, D <= 128.
//
// The reference runs its Triton kernels on fp32 tensors too (flashmlp.py:63-158, 341-421);
// `tl.dot` then multiplies at TF32 precision and everything between the products stays
// fp32: H = act(Z) and dZ are not rounded (the `.to(dtype)` casts are no-ops). These
// kernels do the same with tcgen05.mma kind::tf32: operands are fp32 in shared memory or
// TMEM and are used at TF32 precision, accumulation is fp32, and H / dZ are written back
// into TMEM as fp32 in place of Z / dH (one element per 32-bit column, the layout a TMEM A
// operand of a TF32 MMA has), so no packing is needed. Outputs are fp32.
//
// Layouts: a TF32 operand read K-major uses the usual 128-byte swizzle; read MN-major it
// must use the 128-byte swizzle with 32-byte atoms (4-row atoms, descriptor layout type 1,
// TMA CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B) -- the only MN-major layout TF32 operands have.
// The forward reads its weight chunks only MN-major. The backward reads some tiles both
// ways (X and dO in the dW programs, W1c in the dX programs), so those are loaded twice,
// once per layout, with 32-wide tiles to fit shared memory.
// An fp32 tile of 128 rows x 128 columns is 64 KB, twice a 16-bit one; the stationary
// operand of each backward program (W1c^T of a dW program, X_b of a dX program) sits in
// TMEM, as in the D = 256 kernels.
//
// Forward, one CTA per SM, persistent over (head, 128-row tile) work items:
//   Z(c)   = X[smem] @ W1c[smem]       SS M=128(b) N=64(e) K=DP     (Z double-buffered)
//   H(c)   = act(Z(c)) in place (fp32)
//   O     += H(c)[tmem] @ W2c[smem]    TS M=128(b) N=DP    K=64(e)
// TMEM: O [0,DP) Z [DP, DP+128). smem: X tile + 2-stage W1c and W2c rings (192 KB at DP 128).
//
// Backward, dW programs (head, 128-wide E chunk) first, then dX programs (head, 128-row
// tile), the reference's program split:
//   dW:  Z^T(t)  = W1c^T[tmem] @ X_t^T[smem]   TS M=128(e) N=32(b) K=DP   (X_t K-major)
//        dH^T(t) = W2c[smem] @ dO_t^T[smem]    SS M=128(e) N=32(b) K=DP   (dO_t K-major)
//        H^T, dZ^T in place;  dW2 += H^T @ dO_t,  dW1^T += dZ^T @ X_t   TS N=DP K=32(b)
//        (dO_t, X_t MN-major copies)
//        TMEM: dW1^T [0,DP) dW2 [DP,2DP) W1c^T [2DP,3DP) Z^T +32 dH^T +32
//        smem: W2c + 2 stages of {X_t, dO_t} x {K-major, MN-major} (192 KB at DP 128)
//   dX:  Z(c)  = X_b[tmem] @ W1c[smem]        TS M=128(b) N=32(e) K=DP   (W1c MN-major)
//        dH(c) = dO_b[smem] @ W2c^T[smem]     SS M=128(b) N=32(e) K=DP
//        dX   += dZ(c)[tmem] @ W1c^T[smem]    TS M=128(b) N=DP    K=32(e) (W1c K-major)
//        TMEM: dX [0,DP) X_b [DP,2DP) Z +32 dH +32
//        smem: dO_b + 3 stages of W1c in both layouts + 2-stage W2c ring (192 KB at DP 128)
// Issue orders as in fmlp_bwd256.cu. Every wait is bounded (fmlp_ptx.cuh).
#include "fmlp_act.cuh"
#include "fmlp_kernels.h"
#include "fmlp_ptx.cuh"

namespace fmlp {

// fp32 tiles in 128-byte swizzled rows hold 32 elements; a TMA box is {32, rows}.
constexpr int kF32Row = 32;

// ============================================================================ forward
template <int DP>
struct FwdTf32Cfg {
  static_assert(DP == 64 || DP == 128, "fp32 kernels cover D <= 128");
  static constexpr int BM = kRows;
  static constexpr int ET = 64;
  static constexpr int WS = 2;
  static constexpr int X_BYTES = BM * DP * 4;   // DP/32 regions of [128 rows][128 B]
  static constexpr int W1_BYTES = DP * ET * 4;  // 2 regions (32 e) of [DP rows][128 B]
  static constexpr int W2_BYTES = ET * DP * 4;  // DP/32 regions of [64 rows][128 B]
  static constexpr int OFF_X = 0;
  static constexpr int OFF_W1 = X_BYTES;
  static constexpr int OFF_W2 = OFF_W1 + WS * W1_BYTES;
  static constexpr int OFF_BAR = OFF_W2 + WS * W2_BYTES;
  // x_full x_empty w1_full[2] w1_empty[2] w2_full[2] w2_empty[2] z_full[2] h_full[2]
  // o_full o_empty done
  static constexpr int NBAR = 2 + 4 * WS + 4 + 3;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16 + 1024;
  static constexpr int SMEM = SMEM_USED > 120 * 1024 ? SMEM_USED : 120 * 1024;
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr int TMEM_O = 0;
  static constexpr int TMEM_Z = DP;
  static constexpr int TMEM_COLS = 512;
  static constexpr int NUM_ACT_WARPS = 16;
  static constexpr int NUM_THREADS = 32 * (2 + NUM_ACT_WARPS);
  static constexpr int SW = ET / 4;  // Z columns per activation warp (16)
  static constexpr int OW = DP / 4;  // O columns per activation warp (16 or 32)
};

template <int DP, int ACT>
__global__ void __launch_bounds__(576, 1)
    fmlp_fwd_tf32_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w1,
                         const __grid_constant__ CUtensorMap tm_w2, float* __restrict__ O, int H, int B, int D,
                         int E, uint32_t* status) {
  using C = FwdTf32Cfg<DP>;
  constexpr int ET = C::ET, WS = C::WS, BM = C::BM, SW = C::SW, OW = C::OW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sX = smem + C::OFF_X;
  uint8_t* sW1 = smem + C::OFF_W1;
  uint8_t* sW2 = smem + C::OFF_W2;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* x_full = bars;
  uint64_t* x_empty = bars + 1;
  uint64_t* w1_full = bars + 2;
  uint64_t* w1_empty = w1_full + WS;
  uint64_t* w2_full = w1_empty + WS;
  uint64_t* w2_empty = w2_full + WS;
  uint64_t* z_full = w2_empty + WS;
  uint64_t* h_full = z_full + 2;
  uint64_t* o_full = h_full + 2;
  uint64_t* o_empty = o_full + 1;
  uint64_t* done_bar = o_empty + 1;
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_flag = misc + 1;  // misc[2] stays 0: "never abort" flag for drains
  const WaitCtx ctx{abort_flag, status};
  const WaitCtx drain{misc + 2, status};

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nB = (B + BM - 1) / BM;
  const int nE = (E + ET - 1) / ET;
  const int ntiles = H * nB;

  if (threadIdx.x == 0) {
    misc[1] = 0;
    misc[2] = 0;
    mbar_init(x_full, 1);
    mbar_init(x_empty, 1);
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
    mbar_init(o_full, 1);
    mbar_init(o_empty, C::NUM_ACT_WARPS);
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
    if (lane == 0) {
      uint32_t c1 = 0, c2 = 0, xl = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int h = tile / nB, bt = tile % nB;
        if (!(ok = mbar_wait(x_empty, (xl & 1) ^ 1, ctx))) break;
        mbar_arrive_expect_tx(x_full, C::X_BYTES);
        for (int r = 0; r < DP / kF32Row; ++r)
          tma_load_3d(sX + r * BM * 128, &tm_x, x_full, kF32Row * r, bt * BM, h);
        ++xl;
        for (int c = 0; c < nE && ok; ++c) {
          {
            const int s = c1 % WS;
            if (!(ok = mbar_wait(&w1_empty[s], ((c1 / WS) & 1) ^ 1, ctx))) break;
            mbar_arrive_expect_tx(&w1_full[s], C::W1_BYTES);
            for (int r = 0; r < ET / kF32Row; ++r)
              tma_load_3d(sW1 + s * C::W1_BYTES + r * DP * 128, &tm_w1, &w1_full[s], c * ET + kF32Row * r, 0, h);
            ++c1;
          }
          {
            const int s = c2 % WS;
            if (!(ok = mbar_wait(&w2_empty[s], ((c2 / WS) & 1) ^ 1, ctx))) break;
            mbar_arrive_expect_tx(&w2_full[s], C::W2_BYTES);
            for (int r = 0; r < DP / kF32Row; ++r)
              tma_load_3d(sW2 + s * C::W2_BYTES + r * ET * 128, &tm_w2, &w2_full[s], kF32Row * r, c * ET, h);
            ++c2;
          }
        }
      }
      for (uint32_t s = 0; s < WS; ++s) {
        if (c1 > s) mbar_wait(&w1_full[s], ((c1 - 1 - s) / WS) & 1, drain);
        if (c2 > s) mbar_wait(&w2_full[s], ((c2 - 1 - s) / WS) & 1, drain);
      }
      if (xl > 0) mbar_wait(x_full, (xl - 1) & 1, drain);
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc1 = make_idesc_tf32(BM, ET, false, true);  // A K-major, B MN-major
    constexpr uint32_t idesc2 = make_idesc_tf32(BM, DP, false, true);  // A tmem, B MN-major
    const uint64_t xdesc = make_sdesc_sw128(smem_u32(sX), 16, 1024);
    const uint32_t sW1_a = smem_u32(sW1), sW2_a = smem_u32(sW2);
    uint32_t c1 = 0, c2 = 0, zc = 0, it = 0;
    bool ok = true;
    auto gemm1 = [&](uint32_t zidx) -> bool {  // Z[zidx & 1] = X @ W1c, K over the padded DP
      const int s = c1 % WS;
      if (!warp_wait(&w1_full[s], (c1 / WS) & 1, ctx)) return false;
      ++c1;
      tc_fence_after();
      if (elect_one()) {
        const uint64_t wdesc = make_sdesc_mn32(sW1_a + s * C::W1_BYTES, DP * 128);
#pragma unroll
        for (int k = 0; k < DP / 8; ++k)
          mma_ss_tf32(tmem + C::TMEM_Z + (zidx & 1) * ET, sdesc_add(xdesc, (k >> 2) * (BM * 128) + (k & 3) * 32),
                      sdesc_add(wdesc, k * 1024), idesc1, k > 0 ? 1u : 0u);
        mma_commit(&z_full[zidx & 1]);
        mma_commit(&w1_empty[s]);
      }
      __syncwarp();
      return true;
    };
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
      if (!(ok = warp_wait(x_full, it & 1, ctx))) break;
      tc_fence_after();
      if (!(ok = gemm1(zc))) break;
      for (int c = 0; c < nE && ok; ++c) {
        const uint32_t zcur = zc + c;
        if (c + 1 < nE) {
          if (!(ok = gemm1(zcur + 1))) break;
        } else {
          if (elect_one()) mma_commit(x_empty);  // every reader of X issued
          __syncwarp();
        }
        if (c == 0 && !(ok = warp_wait(o_empty, (it & 1) ^ 1, ctx))) break;
        if (!(ok = warp_wait(&h_full[zcur & 1], (zcur >> 1) & 1, ctx))) break;
        const int s = c2 % WS;
        if (!(ok = warp_wait(&w2_full[s], (c2 / WS) & 1, ctx))) break;
        ++c2;
        tc_fence_after();
        if (elect_one()) {
          const uint64_t wdesc = make_sdesc_mn32(sW2_a + s * C::W2_BYTES, ET * 128);
          const uint32_t hb = tmem + C::TMEM_Z + (zcur & 1) * ET;
#pragma unroll
          for (int k = 0; k < ET / 8; ++k)
            mma_ts_tf32(tmem + C::TMEM_O, hb + 8 * k, sdesc_add(wdesc, k * 1024), idesc2, (c > 0 || k > 0) ? 1u : 0u);
          mma_commit(&w2_empty[s]);
          if (c + 1 == nE) mma_commit(o_full);
        }
        __syncwarp();
      }
      zc += nE;
    }
    if (elect_one()) mma_commit(done_bar);
    __syncwarp();
    warp_wait(done_bar, 0, drain);
  } else {
    const int q = warp & 3;
    const int j = (warp - 2) >> 2;
    const uint32_t lane_off = uint32_t(q * 32) << 16;
    uint32_t zc = 0, it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
      const int h = tile / nB, bt = tile % nB;
      for (int c = 0; c < nE; ++c, ++zc) {
        if (!(ok = mbar_wait(&z_full[zc & 1], (zc >> 1) & 1, ctx))) break;
        tc_fence_after();
        const uint32_t za = tmem + lane_off + C::TMEM_Z + (zc & 1) * ET + j * SW;
        uint32_t v[16];
        tmem_ld16_sync(za, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(act_fwd<float, ACT>(__uint_as_float(v[i])));
        tmem_st16(za, v);  // H (fp32) in place of Z
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&h_full[zc & 1]);
      }
      if (!ok) break;
      if (!(ok = mbar_wait(o_full, it & 1, ctx))) break;
      tc_fence_after();
      const int row = bt * BM + q * 32 + lane;
      float* orow = O + (size_t(h) * B + row) * D;
#pragma unroll
      for (int u = 0; u < OW / 16; ++u) {
        uint32_t v[16];
        tmem_ld16_sync(tmem + lane_off + C::TMEM_O + j * OW + 16 * u, v);
        const int cc = j * OW + 16 * u;
        if (row < B && cc < D) {  // D % 16 == 0: all 16 columns are inside
          float4* dst = reinterpret_cast<float4*>(orow + cc);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]), __uint_as_float(v[4 * i + 2]),
                                 __uint_as_float(v[4 * i + 3]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ============================================================================ backward
template <int DP>
struct BwdTf32Cfg {
  static_assert(DP == 64 || DP == 128, "fp32 kernels cover D <= 128");
  static constexpr int BM = kRows;  // rows of a dX program's B tile, M of every MMA
  static constexpr int T = 32;      // B rows per dW tile, E columns per dX chunk
  static constexpr int EW = 128;    // E rows per dW program
  // dW program smem
  static constexpr int W2C_BYTES = EW * DP * 4;  // DP/32 regions of [128 rows][128 B]
  static constexpr int WT_BYTES = T * DP * 4;    // DP/32 regions of [32 rows][128 B]
  static constexpr int WS = 2;
  static constexpr int W_OFF_W2 = 0;
  static constexpr int W_OFF_STAGE = W2C_BYTES;  // per stage: X_K, X_MN, dO_K, dO_MN
  static constexpr int W_STAGE = 4 * WT_BYTES;
  static constexpr int W_END = W_OFF_STAGE + WS * W_STAGE;
  // dX program smem
  static constexpr int DOB_BYTES = BM * DP * 4;  // DP/32 regions of [128 rows][128 B]
  static constexpr int W1X_BYTES = DP * T * 4;   // one region [DP rows][128 B] (32 e)
  static constexpr int W2X_BYTES = T * DP * 4;   // DP/32 regions of [32 rows][128 B]
  static constexpr int S1 = 3, S2 = 2;
  static constexpr int X_OFF_DO = 0;
  static constexpr int X_OFF_W1 = DOB_BYTES;     // per stage: W1c MN-major, W1c K-major
  static constexpr int X_OFF_W2 = X_OFF_W1 + S1 * 2 * W1X_BYTES;
  static constexpr int X_END = X_OFF_W2 + S2 * W2X_BYTES;
  static constexpr int OFF_BAR = X_END > W_END ? X_END : W_END;
  static constexpr int NBAR = 24;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16 + 1024;
  static constexpr int SMEM = SMEM_USED > 120 * 1024 ? SMEM_USED : 120 * 1024;
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr int TMEM_COLS = 512;
  // TMEM columns, dW program
  static constexpr int W_TM_DW1 = 0, W_TM_DW2 = DP, W_TM_W1T = 2 * DP, W_TM_ZT = 3 * DP, W_TM_DHT = 3 * DP + T;
  // TMEM columns, dX program
  static constexpr int X_TM_DX = 0, X_TM_XB = DP, X_TM_Z = 2 * DP, X_TM_DH = 2 * DP + T;
  static_assert(W_TM_DHT + T <= TMEM_COLS, "TMEM budget");
  static constexpr int NUM_ACT_WARPS = 16;
  static constexpr int NUM_THREADS = 32 * (2 + NUM_ACT_WARPS);
};

template <int DP, int ACT>
__global__ void __launch_bounds__(576, 1)
    fmlp_bwd_tf32_kernel(const __grid_constant__ Tf32BwdMaps tm, const float* __restrict__ X,
                         const float* __restrict__ W1, float* __restrict__ dX, float* __restrict__ dW1,
                         float* __restrict__ dW2, float* __restrict__ part, float* __restrict__ dzt, int splits,
                         int H, int B, int D, int E, uint32_t* status) {
  using C = BwdTf32Cfg<DP>;
  using St = ActState<float, ACT>;
  constexpr int BM = C::BM, T = C::T;
  constexpr int NACT = C::NUM_ACT_WARPS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_flag = misc + 1;  // misc[2] stays 0: "never abort" flag for drains
  const WaitCtx ctx{abort_flag, status};
  const WaitCtx drain{misc + 2, status};

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nEw = (E + C::EW - 1) / C::EW;  // dW programs per head and B range
  // dW programs: (head, split, E chunk), chunk fastest; with splits > 1 each covers a
  // contiguous range of the 32-row B tiles and writes fp32 partial sums to `part`
  // (part[split][0] = dW1 (H,D,E), part[split][1] = dW2 (H,E,D)), added in split order by
  // fmlp_dw_reduce_f32_kernel
  const bool is_dw = int(blockIdx.x) < H * nEw * splits;
  int h, idx, t0 = 0, t1 = 0;
  if (is_dw) {
    h = blockIdx.x / (nEw * splits);
    const int r = blockIdx.x % (nEw * splits);
    const int split = r / nEw;
    idx = r % nEw;  // E chunk
    const int nTt = (B + T - 1) / T;
    t0 = int((long long)split * nTt / splits);
    t1 = int((long long)(split + 1) * nTt / splits);
    if (part != nullptr) {
      const size_t n = size_t(H) * D * E;
      dW1 = part + size_t(split) * 2 * n;
      dW2 = dW1 + n;
    }
  } else {
    const int nBx = (B + BM - 1) / BM;
    const int p = blockIdx.x - H * nEw * splits;
    h = p / nBx;
    idx = p % nBx;  // B tile
  }

  uint64_t* in_full = bars + 0;     // dW: W2c loaded ; dX: dO_b loaded
  uint64_t* tin_full = bars + 1;    // W1c^T / X_b written into TMEM by the activation warps
  uint64_t* ring_full = bars + 2;   // 3: dW: X+dO stages ; dX: W1c stages
  uint64_t* ring_empty = bars + 5;  // 3
  uint64_t* w2_full = bars + 8;     // 2: dX: W2c stages
  uint64_t* w2_empty = bars + 10;   // 2
  uint64_t* p_full = bars + 12;     // 2: [0] Z^T / Z, [1] dH^T / dH
  uint64_t* a_full = bars + 14;     // 2: [0] phase 1 done, [1] phase 2 done
  uint64_t* acc_full = bars + 16;   // accumulators final
  uint64_t* done_bar = bars + 17;   // all MMAs retired
  uint64_t* x_free = bars + 18;     // 2: dW: dW1^T(t) read the stage's X tiles
  uint64_t* do_free = bars + 20;    // 2: dW: dW2(t) read the stage's dO tiles

  if (threadIdx.x == 0) {
    misc[1] = 0;
    misc[2] = 0;
    mbar_init(in_full, 1);
    mbar_init(tin_full, NACT);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&w2_full[i], 1);
      mbar_init(&w2_empty[i], 1);
      mbar_init(&p_full[i], 1);
      mbar_init(&a_full[i], NACT);
      mbar_init(&x_free[i], 1);
      mbar_init(&do_free[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(done_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int q = warp & 3;
  const int j = (warp - 2) >> 2;
  const uint32_t lane_off = uint32_t(q * 32) << 16;
  constexpr int TW = DP / 4;  // TMEM columns of a stationary operand or accumulator per warp

  // Phase 1 over the 8 product columns at `col` (column slice j of a 32-wide product):
  // derivative state; if `store_h`, H (fp32) in place of Z.
  auto phase1 = [&](uint32_t col, St (&st)[8], bool store_h) {
    uint32_t v[8];
    tmem_ld8_sync(col, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __float_as_uint(act_forward<float, ACT>(__uint_as_float(v[i]), st[i]));
    if (store_h) tmem_st8(col, v);
  };
  // Phase 2 over the 8 dH columns at `col`: dZ (fp32) in place and, if `g` is set, also
  // stored to g[0], g[row], ..., g[7 * row] (the dZ-store workspace, one value per b row).
  auto phase2 = [&](uint32_t col, const St (&st)[8], float* g, uint32_t row) {
    uint32_t v[8];
    tmem_ld8_sync(col, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __float_as_uint(act_grad<float, ACT>(__uint_as_float(v[i]), st[i]));
    tmem_st8(col, v);
    if (g != nullptr) {
#pragma unroll
      for (int i = 0; i < 8; ++i) g[i * row] = __uint_as_float(v[i]);
    }
  };
  auto signal = [&](uint64_t* bar, bool wrote_tmem) {
    if (wrote_tmem) tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
  };

  if (is_dw) {
    // ==================================================================== dW program
    const int c = idx;
    const int nT = t1 - t0;  // 32-row tiles of this program; tile t of the loops is t0 + t
    uint8_t* sW2 = smem + C::W_OFF_W2;
    constexpr int WS = C::WS;
    // stage s: X_K, X_MN, dO_K, dO_MN
    auto tile = [&](int s, int which) { return smem + C::W_OFF_STAGE + s * C::W_STAGE + which * C::WT_BYTES; };
    if (warp == 0) {
      if (lane == 0) {
        mbar_arrive_expect_tx(in_full, C::W2C_BYTES);
        for (int r = 0; r < DP / kF32Row; ++r)
          for (int eq = 0; eq < C::EW / T; ++eq)
            tma_load_3d(sW2 + r * (C::EW * 128) + eq * (T * 128), &tm.w2_k, in_full, kF32Row * r, c * C::EW + T * eq, h);
        uint32_t nl = 0;
        for (int t = 0; t < nT; ++t) {
          const int s = t % WS;
          const uint32_t par = ((t / WS) & 1) ^ 1;
          // the stage is free once dW1^T(t-2) read its X tiles and dW2(t-2) its dO tiles
          if (!mbar_wait(&x_free[s], par, ctx) || !mbar_wait(&do_free[s], par, ctx)) break;
          mbar_arrive_expect_tx(&ring_full[s], C::W_STAGE);
          for (int r = 0; r < DP / kF32Row; ++r) {
            const int off = r * (T * 128);
            tma_load_3d(tile(s, 0) + off, &tm.x_k, &ring_full[s], kF32Row * r, (t0 + t) * T, h);
            tma_load_3d(tile(s, 1) + off, &tm.x_mn, &ring_full[s], kF32Row * r, (t0 + t) * T, h);
            tma_load_3d(tile(s, 2) + off, &tm.do_k, &ring_full[s], kF32Row * r, (t0 + t) * T, h);
            tma_load_3d(tile(s, 3) + off, &tm.do_mn, &ring_full[s], kF32Row * r, (t0 + t) * T, h);
          }
          ++nl;
        }
        mbar_wait(in_full, 0, drain);
        for (uint32_t i = 0; i < WS; ++i)
          if (nl > i) mbar_wait(&ring_full[(nl - 1 - i) % WS], ((nl - 1 - i) / WS) & 1, drain);
      }
    } else if (warp == 1) {
      constexpr uint32_t idesc_p = make_idesc_tf32(128, T, false, false);  // A K / tmem, B K
      constexpr uint32_t idesc_w = make_idesc_tf32(128, DP, false, true);  // A tmem, B MN
      const uint64_t w2k = make_sdesc_sw128(smem_u32(sW2), 16, 1024);
      // Z^T(t) (m = 0) or dH^T(t) (m = 1); K over the padded DP (zero-filled).
      auto issue_prod = [&](int m, int t) {
        const int s = t % WS;
        if (elect_one()) {
          const uint64_t bk = make_sdesc_sw128(smem_u32(tile(s, m == 0 ? 0 : 2)), 16, 1024);
          const uint32_t d = tmem + (m == 0 ? C::W_TM_ZT : C::W_TM_DHT);
#pragma unroll
          for (int k = 0; k < DP / 8; ++k) {
            const uint64_t bkk = sdesc_add(bk, (k >> 2) * (T * 128) + (k & 3) * 32);
            if (m == 0)
              mma_ts_tf32(d, tmem + C::W_TM_W1T + 8 * k, bkk, idesc_p, k > 0 ? 1u : 0u);
            else
              mma_ss_tf32(d, sdesc_add(w2k, (k >> 2) * (C::EW * 128) + (k & 3) * 32), bkk, idesc_p, k > 0 ? 1u : 0u);
          }
          mma_commit(&p_full[m]);
        }
        __syncwarp();
      };
      // dW2 += H^T(t) @ dO_t (m = 0) or dW1^T += dZ^T(t) @ X_t (m = 1): B = the MN-major copy,
      // DP columns in 32-wide regions (LBO = region stride), K = the tile's 32 rows.
      auto issue_dw = [&](int m, int t) {
        const int s = t % WS;
        if (elect_one()) {
          const uint64_t bm = make_sdesc_mn32(smem_u32(tile(s, m == 0 ? 3 : 1)), T * 128);
          const uint32_t d = tmem + (m == 0 ? C::W_TM_DW2 : C::W_TM_DW1);
          const uint32_t a = tmem + (m == 0 ? C::W_TM_ZT : C::W_TM_DHT);
          const uint32_t acc0 = t > 0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < T / 8; ++k)
            mma_ts_tf32(d, a + 8 * k, sdesc_add(bm, k * 1024), idesc_w, k > 0 ? 1u : acc0);
          mma_commit(m == 0 ? &do_free[s] : &x_free[s]);
        }
        __syncwarp();
      };
      auto wait_tile = [&](int t) { return warp_wait(&ring_full[t % WS], (t / WS) & 1, ctx); };
      bool ok = warp_wait(in_full, 0, ctx) && warp_wait(tin_full, 0, ctx) && nT > 0 && wait_tile(0);
      tc_fence_after();
      if (ok) {
        issue_prod(0, 0);
        issue_prod(1, 0);
      }
      for (int t = 0; t < nT && ok; ++t) {
        const bool more = t + 1 < nT;
        if (!(ok = warp_wait(&a_full[0], t & 1, ctx))) break;  // H^T(t) in place of Z^T(t)
        tc_fence_after();
        issue_dw(0, t);
        if (more) {  // overwrites H^T(t) after dW2(t) read it
          if (!(ok = wait_tile(t + 1))) break;
          tc_fence_after();
          issue_prod(0, t + 1);
        }
        if (!(ok = warp_wait(&a_full[1], t & 1, ctx))) break;  // dZ^T(t) in place of dH^T(t)
        tc_fence_after();
        issue_dw(1, t);
        if (more) issue_prod(1, t + 1);  // overwrites dZ^T(t) after dW1^T(t) read it
      }
      if (ok) {
        if (elect_one()) mma_commit(acc_full);
        __syncwarp();
      }
      if (elect_one()) mma_commit(done_bar);
      __syncwarp();
      warp_wait(done_bar, 0, drain);
    } else {
      // W1c^T into TMEM: lane e of quadrant q holds W1[h, d, c*128 + 32q + lane] for d in
      // [TW*j, TW*j + TW) as fp32 columns at W1T + TW*j (zero outside D and E); for each d
      // the warp's 32 lanes read 32 consecutive e (128 bytes).
      {
        const int e = c * C::EW + q * 32 + lane;
        const float* col = W1 + size_t(h) * D * E + e;
#pragma unroll 1
        for (int u = 0; u < TW / 16; ++u) {
          uint32_t v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int d = TW * j + 16 * u + i;
            v[i] = (e < E && d < D) ? __float_as_uint(col[size_t(d) * E]) : 0u;
          }
          tmem_st16(tmem + lane_off + C::W_TM_W1T + TW * j + 16 * u, v);
        }
        signal(tin_full, true);
      }
      const uint32_t zt = tmem + lane_off + C::W_TM_ZT + 8 * j;
      const uint32_t dt = tmem + lane_off + C::W_TM_DHT + 8 * j;
      // dZ-store mode: dZ (not transposed) in the workspace as (H, nB*128, nE*128) fp32,
      // e contiguous, the K-major operand fmlp_dx_gemm_tf32_kernel reads by TMA. This
      // thread (e = 128c + 32q + lane) stores b = 32(t0 + t) + 8j + i, i < 8; for each i the
      // warp's 32 lanes write 128 contiguous bytes. 32-bit element offsets (the workspace
      // holds at most 2^31 fp32 values).
      const uint32_t dz_ld = uint32_t(nEw * C::EW);  // row length of the workspace
      const uint32_t dz_off = uint32_t(size_t(h) * ((B + BM - 1) / BM) * BM * dz_ld) +
                              uint32_t(T * t0 + 8 * j) * dz_ld + uint32_t(c * C::EW + q * 32 + lane);
      bool ok = true;
      for (int t = 0; t < nT && ok; ++t) {
        St st[8];
        if (!(ok = mbar_wait(&p_full[0], t & 1, ctx))) break;
        tc_fence_after();
        phase1(zt, st, true);  // H^T in place of Z^T
        signal(&a_full[0], true);
        if (!(ok = mbar_wait(&p_full[1], t & 1, ctx))) break;
        tc_fence_after();
        phase2(dt, st, dzt != nullptr ? dzt + (dz_off + uint32_t(t * T) * dz_ld) : nullptr, dz_ld);  // dZ^T in place of dH^T
        signal(&a_full[1], true);
      }
      if (ok && (ok = mbar_wait(acc_full, 0, ctx))) {
        tc_fence_after();
        const int e = c * C::EW + q * 32 + lane;
        // dW1^T rows are E, columns D: dW1[h, d, e]; each column d is one coalesced
        // 128-byte store across the warp.
#pragma unroll 1
        for (int u = 0; u < TW / 16; ++u) {
          uint32_t v[16];
          tmem_ld16_sync(tmem + lane_off + C::W_TM_DW1 + TW * j + 16 * u, v);
          if (e < E) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int d = TW * j + 16 * u + i;
              if (d < D) dW1[(size_t(h) * D + d) * E + e] = __uint_as_float(v[i]);
            }
          }
        }
        float* w2row = dW2 + (size_t(h) * E + e) * D;
#pragma unroll 1
        for (int u = 0; u < TW / 16; ++u) {
          uint32_t v[16];
          tmem_ld16_sync(tmem + lane_off + C::W_TM_DW2 + TW * j + 16 * u, v);
          const int cc = TW * j + 16 * u;
          if (e < E && cc < D) {
            float4* dst = reinterpret_cast<float4*>(w2row + cc);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dst[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                   __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
          }
        }
      }
    }
  } else {
    // ==================================================================== dX program
    const int bt = idx;
    const int nE = (E + T - 1) / T;
    uint8_t* sDO = smem + C::X_OFF_DO;
    uint8_t* sW1 = smem + C::X_OFF_W1;  // stage s: MN-major copy, then K-major copy
    uint8_t* sW2 = smem + C::X_OFF_W2;
    if (warp == 0) {
      if (lane == 0) {
        mbar_arrive_expect_tx(in_full, C::DOB_BYTES);
        for (int r = 0; r < DP / kF32Row; ++r)  // the dO map's box is 32 rows (the dW tiles)
          for (int rq = 0; rq < BM / T; ++rq)
            tma_load_3d(sDO + r * (BM * 128) + rq * (T * 128), &tm.do_k, in_full, kF32Row * r, bt * BM + T * rq, h);
        uint32_t n1 = 0, n2 = 0;
        for (int c = 0; c < nE; ++c) {  // the order the MMA warp consumes them
          const int s1 = c % C::S1, s2 = c % C::S2;
          if (!mbar_wait(&ring_empty[s1], ((c / C::S1) & 1) ^ 1, ctx)) break;
          mbar_arrive_expect_tx(&ring_full[s1], 2 * C::W1X_BYTES);
          tma_load_3d(sW1 + s1 * 2 * C::W1X_BYTES, &tm.w1_mn, &ring_full[s1], c * T, 0, h);
          tma_load_3d(sW1 + s1 * 2 * C::W1X_BYTES + C::W1X_BYTES, &tm.w1_k, &ring_full[s1], c * T, 0, h);
          ++n1;
          if (!mbar_wait(&w2_empty[s2], ((c / C::S2) & 1) ^ 1, ctx)) break;
          mbar_arrive_expect_tx(&w2_full[s2], C::W2X_BYTES);
          for (int r = 0; r < DP / kF32Row; ++r)
            tma_load_3d(sW2 + s2 * C::W2X_BYTES + r * (T * 128), &tm.w2_k, &w2_full[s2], kF32Row * r, c * T, h);
          ++n2;
        }
        mbar_wait(in_full, 0, drain);
        for (uint32_t i = 0; i < C::S1; ++i)
          if (n1 > i) mbar_wait(&ring_full[(n1 - 1 - i) % C::S1], ((n1 - 1 - i) / C::S1) & 1, drain);
        for (uint32_t i = 0; i < C::S2; ++i)
          if (n2 > i) mbar_wait(&w2_full[(n2 - 1 - i) % C::S2], ((n2 - 1 - i) / C::S2) & 1, drain);
      }
    } else if (warp == 1) {
      constexpr uint32_t idesc_z = make_idesc_tf32(128, T, false, true);   // A tmem, B MN
      constexpr uint32_t idesc_h = make_idesc_tf32(128, T, false, false);  // A K, B K
      constexpr uint32_t idesc_x = make_idesc_tf32(128, DP, false, false); // A tmem, B K
      const uint64_t dk = make_sdesc_sw128(smem_u32(sDO), 16, 1024);
      auto issue_z = [&](int c) {  // Z(c) = X_b @ W1c (MN-major copy: rows D, 32 E per row)
        if (elect_one()) {
          const uint64_t w1m = make_sdesc_mn32(smem_u32(sW1 + (c % C::S1) * 2 * C::W1X_BYTES), DP * 128);
#pragma unroll
          for (int k = 0; k < DP / 8; ++k)
            mma_ts_tf32(tmem + C::X_TM_Z, tmem + C::X_TM_XB + 8 * k, sdesc_add(w1m, k * 1024), idesc_z,
                        k > 0 ? 1u : 0u);
          mma_commit(&p_full[0]);
        }
        __syncwarp();
      };
      auto issue_dh = [&](int c) {  // dH(c) = dO_b @ W2c^T
        const int s = c % C::S2;
        if (elect_one()) {
          const uint64_t w2k = make_sdesc_sw128(smem_u32(sW2 + s * C::W2X_BYTES), 16, 1024);
#pragma unroll
          for (int k = 0; k < DP / 8; ++k)
            mma_ss_tf32(tmem + C::X_TM_DH, sdesc_add(dk, (k >> 2) * (BM * 128) + (k & 3) * 32),
                        sdesc_add(w2k, (k >> 2) * (T * 128) + (k & 3) * 32), idesc_h, k > 0 ? 1u : 0u);
          mma_commit(&p_full[1]);
          mma_commit(&w2_empty[s]);  // dH(c) is the W2c stage's only reader
        }
        __syncwarp();
      };
      auto issue_dx = [&](int c) {  // dX += dZ(c) @ W1c^T (K-major copy: rows D, K = 32 E)
        const int s = c % C::S1;
        if (elect_one()) {
          const uint64_t w1k = make_sdesc_sw128(smem_u32(sW1 + s * 2 * C::W1X_BYTES + C::W1X_BYTES), 16, 1024);
          const uint32_t acc0 = c > 0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < T / 8; ++k)
            mma_ts_tf32(tmem + C::X_TM_DX, tmem + C::X_TM_DH + 8 * k, sdesc_add(w1k, k * 32), idesc_x,
                        k > 0 ? 1u : acc0);
          mma_commit(&ring_empty[s]);  // dX(c) is the W1c stage's last reader
        }
        __syncwarp();
      };
      auto wait_w1 = [&](int c) { return warp_wait(&ring_full[c % C::S1], (c / C::S1) & 1, ctx); };
      auto wait_w2 = [&](int c) { return warp_wait(&w2_full[c % C::S2], (c / C::S2) & 1, ctx); };
      bool ok = warp_wait(in_full, 0, ctx) && warp_wait(tin_full, 0, ctx) && nE > 0 && wait_w1(0) && wait_w2(0);
      tc_fence_after();
      if (ok) {
        issue_z(0);
        issue_dh(0);
      }
      for (int c = 0; c < nE && ok; ++c) {
        const bool more = c + 1 < nE;
        if (!(ok = warp_wait(&a_full[0], c & 1, ctx))) break;  // phase 1(c) has read Z(c)
        if (more) {
          if (!(ok = wait_w1(c + 1))) break;
          tc_fence_after();
          issue_z(c + 1);
        }
        if (!(ok = warp_wait(&a_full[1], c & 1, ctx))) break;  // dZ(c) in place of dH(c)
        tc_fence_after();
        issue_dx(c);
        if (more) {  // overwrites dZ(c) after dX(c) read it
          if (!(ok = wait_w2(c + 1))) break;
          tc_fence_after();
          issue_dh(c + 1);
        }
      }
      if (ok) {
        if (elect_one()) mma_commit(acc_full);
        __syncwarp();
      }
      if (elect_one()) mma_commit(done_bar);
      __syncwarp();
      warp_wait(done_bar, 0, drain);
    } else {
      const int row = bt * BM + q * 32 + lane;
      // X_b into TMEM: lane b of quadrant q holds X[h, row, d] for d in [TW*j, TW*j + TW)
      // as fp32 columns at XB + TW*j (zero outside B and D).
      {
        const float4* src = reinterpret_cast<const float4*>(X + (size_t(h) * B + row) * D + TW * j);
#pragma unroll 1
        for (int u = 0; u < TW / 16; ++u) {
          uint32_t v[16];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
            if (row < B && TW * j + 16 * u + 4 * i < D) f = src[4 * u + i];
            v[4 * i] = __float_as_uint(f.x), v[4 * i + 1] = __float_as_uint(f.y);
            v[4 * i + 2] = __float_as_uint(f.z), v[4 * i + 3] = __float_as_uint(f.w);
          }
          tmem_st16(tmem + lane_off + C::X_TM_XB + TW * j + 16 * u, v);
        }
        signal(tin_full, true);
      }
      // Per E chunk: E columns [8j, 8j+8) of Z and dH.
      const uint32_t za = tmem + lane_off + C::X_TM_Z + 8 * j;
      const uint32_t da = tmem + lane_off + C::X_TM_DH + 8 * j;
      bool ok = true;
      for (int c = 0; c < nE && ok; ++c) {
        St st[8];
        if (!(ok = mbar_wait(&p_full[0], c & 1, ctx))) break;
        tc_fence_after();
        phase1(za, st, false);  // derivative state only
        signal(&a_full[0], false);
        if (!(ok = mbar_wait(&p_full[1], c & 1, ctx))) break;
        tc_fence_after();
        phase2(da, st, nullptr, 0);  // dZ in place of dH
        signal(&a_full[1], true);
      }
      if (ok && (ok = mbar_wait(acc_full, 0, ctx))) {
        tc_fence_after();
        float* xrow = dX + (size_t(h) * B + row) * D;
#pragma unroll 1
        for (int u = 0; u < TW / 16; ++u) {
          uint32_t v[16];
          tmem_ld16_sync(tmem + lane_off + C::X_TM_DX + TW * j + 16 * u, v);
          const int cc = TW * j + 16 * u;
          if (row < B && cc < D) {
            float4* dst = reinterpret_cast<float4*>(xrow + cc);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dst[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                   __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
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

// ============================================================================ launchers
template <int DP, int ACT>
static cudaError_t launch_fwd_tf32_t(const FwdLaunch& a) {
  using C = FwdTf32Cfg<DP>;
  auto kern = fmlp_fwd_tf32_kernel<DP, ACT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  kern<<<a.grid, C::NUM_THREADS, C::SMEM, a.stream>>>(a.tm_x, a.tm_w1, a.tm_w2, reinterpret_cast<float*>(a.o), a.H,
                                                      a.B, a.D, a.E, a.status);
  return cudaGetLastError();
}

// dX of the dZ-store mode for fp32 inputs: dX[h, b, :] = sum over e of dZ[h, b, e] *
// W1[h, :, e] with TF32 products and fp32 accumulation -- the dX programs' last product on
// the dZ the dW programs stored (fp32, as the dX programs keep it). One CTA per (128-row B
// tile, head); warp 0 issues TMA loads, warp 1 the MMAs, warps 2-5 store dX. K steps of
// 32 e, both operands K-major with the ordinary 128-byte swizzle:
//   dX(b, d) += dZ(b, e) [smem, box {32 e, 128 b}] @ W1^T(e, d) [smem, box {32 e, DP d}]
//   kind::tf32 M=128(b) N=DP K=8, four per stage; 3 stages of 32 KB (DP = 128), two CTAs
//   per SM. HBM-bound: 4*E bytes of dZ per output row.
template <int DP>
struct DxGemmTf32Cfg {
  static constexpr int BM = kRows;
  static constexpr int KT = 32;
  static constexpr int A_BYTES = BM * KT * 4;
  static constexpr int B_BYTES = DP * KT * 4;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int NST = DP == 64 ? 4 : 3;
  static constexpr int OFF_BAR = NST * STAGE;
  static constexpr int OFF_MISC = OFF_BAR + (2 * NST + 2) * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;
  static constexpr int NUM_THREADS = 192;
  static_assert(2 * (SMEM + 1024) <= 233472, "two CTAs per SM");
};

template <int DP>
__global__ void __launch_bounds__(192)
    fmlp_dx_gemm_tf32_kernel(const __grid_constant__ CUtensorMap tm_dz, const __grid_constant__ CUtensorMap tm_w1,
                             float* __restrict__ dX, int B, int D, int E, uint32_t* status) {
  using C = DxGemmTf32Cfg<DP>;
  constexpr int BM = C::BM;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty = full + C::NST;
  uint64_t* acc_full = empty + C::NST;
  uint64_t* done_bar = acc_full + 1;
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile uint32_t* abort_flag = misc + 1;
  const WaitCtx ctx{abort_flag, status};
  const WaitCtx drain{misc + 2, status};  // misc[2] stays 0: drains never abort early
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bt = blockIdx.x;
  const int h = blockIdx.y;
  const int nK = (E + C::KT - 1) / C::KT;
  if (threadIdx.x == 0) {
    misc[1] = 0;
    misc[2] = 0;
    for (int i = 0; i < C::NST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(done_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tm_dz);
    tma_prefetch_desc(&tm_w1);
  }
  if (warp == 1) {
    tmem_alloc(misc, DP);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  if (warp == 0) {
    if (lane == 0) {
      uint32_t n = 0;
      for (int k = 0; k < nK; ++k) {
        const int s = k % C::NST;
        if (!mbar_wait(&empty[s], ((k / C::NST) & 1) ^ 1, ctx)) break;
        uint8_t* st = smem + s * C::STAGE;
        mbar_arrive_expect_tx(&full[s], C::STAGE);
        tma_load_3d(st, &tm_dz, &full[s], k * C::KT, bt * BM, h);
        tma_load_3d(st + C::A_BYTES, &tm_w1, &full[s], k * C::KT, 0, h);
        ++n;
      }
      for (uint32_t k = 0; k < uint32_t(C::NST); ++k)
        if (n > k) mbar_wait(&full[(n - 1 - k) % C::NST], ((n - 1 - k) / C::NST) & 1, drain);
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = make_idesc_tf32(128, DP, false, false);  // A K, B K
    bool ok = true;
    for (int k = 0; k < nK && ok; ++k) {
      const int s = k % C::NST;
      if (!(ok = warp_wait(&full[s], (k / C::NST) & 1, ctx))) break;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t st = smem_u32(smem + s * C::STAGE);
        const uint64_t ad = make_sdesc_sw128(st, 16, 1024);
        const uint64_t bd = make_sdesc_sw128(st + C::A_BYTES, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < C::KT / 8; ++kk)  // K = 8 tf32 = 32 bytes per MMA
          mma_ss_tf32(tmem, sdesc_add(ad, kk * 32), sdesc_add(bd, kk * 32), idesc, (k > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&empty[s]);
      }
      __syncwarp();
    }
    if (ok) {
      if (elect_one()) mma_commit(acc_full);
      __syncwarp();
    }
    if (elect_one()) mma_commit(done_bar);
    __syncwarp();
    warp_wait(done_bar, 0, drain);
  } else {
    const int q = warp & 3;
    if (mbar_wait(acc_full, 0, ctx)) {
      tc_fence_after();
      const int row = bt * BM + q * 32 + lane;
      float* xrow = dX + (size_t(h) * B + row) * D;
      const uint32_t ta = tmem + (uint32_t(q * 32) << 16);
#pragma unroll
      for (int u = 0; u < DP / 16; ++u) {
        uint32_t v[16];
        tmem_ld16_sync(ta + 16 * u, v);
        const int cc = 16 * u;
        if (row < B && cc < D) {  // D % 16 == 0
          float4* dst = reinterpret_cast<float4*>(xrow + cc);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]), __uint_as_float(v[4 * i + 2]),
                                 __uint_as_float(v[4 * i + 3]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, DP);
}

template <int DP>
static cudaError_t launch_dx_gemm_tf32(const BwdLaunch& a) {
  using C = DxGemmTf32Cfg<DP>;
  auto kern = fmlp_dx_gemm_tf32_kernel<DP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const long long nB = (a.B + kRows - 1) / kRows;
  if (nB <= 0 || nB > 0x7FFFFFFFLL || a.H <= 0 || a.H > 65535 || a.tf32_maps == nullptr) return cudaErrorInvalidValue;
  kern<<<dim3(unsigned(nB), unsigned(a.H)), C::NUM_THREADS, C::SMEM, a.stream>>>(
      a.tf32_maps->dz, a.tf32_maps->w1_k, reinterpret_cast<float*>(a.dx), a.B, a.D, a.E, a.status);
  return cudaGetLastError();
}

// dW1 / dW2 of split fp32 dW programs: out[i] = sum over s = 0..S-1, in that order, of
// part[s][which][i] (which = blockIdx.y: 0 = dW1 into o1, 1 = dW2 into o2), four elements
// per step (H*D*E is a multiple of 4). Deterministic, no atomics.
__global__ void __launch_bounds__(256)
    fmlp_dw_reduce_f32_kernel(const float* __restrict__ part, float* __restrict__ o1, float* __restrict__ o2,
                              long long n4, int splits) {
  const long long n = n4 * 4;
  const float4* src = reinterpret_cast<const float4*>(part + blockIdx.y * n);
  float4* dst = reinterpret_cast<float4*>(blockIdx.y ? o2 : o1);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    float4 acc = __ldcs(src + i);
    for (int sp = 1; sp < splits; ++sp) {
      const float4 v = __ldcs(src + size_t(sp) * 2 * n4 + i);
      acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
    }
    dst[i] = acc;
  }
}

template <int DP, int ACT>
static cudaError_t launch_bwd_tf32_t(const BwdLaunch& a) {
  using C = BwdTf32Cfg<DP>;
  auto kern = fmlp_bwd_tf32_kernel<DP, ACT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int nBx = (a.B + kRows - 1) / kRows;
  const int nEw = (a.E + C::EW - 1) / C::EW;
  const int splits = a.splits < 1 ? 1 : a.splits;
  if (splits > 1 && (a.part == nullptr || splits > (a.B + C::T - 1) / C::T)) return cudaErrorInvalidValue;
  // dZ-store mode: dW programs only (they store dZ), then fmlp_dx_gemm_tf32_kernel
  const bool dz = a.dzt != nullptr;
  const long long grid = (long long)a.H * ((long long)nEw * splits + (dz ? 0 : nBx));
  if (grid <= 0 || grid > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  // dW as fp32 into dw_f32 (dW1 (H,D,E) then dW2 (H,E,D)) when given, else into dw1 / dw2
  float* d1 = a.dw_f32 ? a.dw_f32 : reinterpret_cast<float*>(a.dw1);
  float* d2 = a.dw_f32 ? a.dw_f32 + size_t(a.H) * a.D * a.E : reinterpret_cast<float*>(a.dw2);
  if (a.tf32_maps == nullptr) return cudaErrorInvalidValue;
  kern<<<unsigned(grid), C::NUM_THREADS, C::SMEM, a.stream>>>(
      *a.tf32_maps, reinterpret_cast<const float*>(a.x), reinterpret_cast<const float*>(a.w1),
      reinterpret_cast<float*>(a.dx), d1, d2, splits > 1 ? a.part : nullptr, reinterpret_cast<float*>(a.dzt), splits,
      a.H, a.B, a.D, a.E, a.status);
  cudaError_t le = cudaGetLastError();
  if (le == cudaSuccess && dz) le = launch_dx_gemm_tf32<DP>(a);
  if (le != cudaSuccess || splits == 1) return le;
  const long long n4 = (long long)a.H * a.D * a.E / 4;  // E % 8 == 0
  long long blocks = (n4 + 255) / 256;
  const long long cap = (long long)a.sm_count * 4;
  if (blocks > cap) blocks = cap;
  fmlp_dw_reduce_f32_kernel<<<dim3(unsigned(blocks), 2), 256, 0, a.stream>>>(a.part, d1, d2, n4, splits);
  return cudaGetLastError();
}

template <int DP>
static cudaError_t launch_fwd_tf32_dp(const FwdLaunch& a) {
  switch (a.act) {
    case kLeakyRelu: return launch_fwd_tf32_t<DP, kLeakyRelu>(a);
    case kSilu: return launch_fwd_tf32_t<DP, kSilu>(a);
    case kSigmoid: return launch_fwd_tf32_t<DP, kSigmoid>(a);
    default: return launch_fwd_tf32_t<DP, kLinear>(a);
  }
}

template <int DP>
static cudaError_t launch_bwd_tf32_dp(const BwdLaunch& a) {
  switch (a.act) {
    case kLeakyRelu: return launch_bwd_tf32_t<DP, kLeakyRelu>(a);
    case kSilu: return launch_bwd_tf32_t<DP, kSilu>(a);
    case kSigmoid: return launch_bwd_tf32_t<DP, kSigmoid>(a);
    default: return launch_bwd_tf32_t<DP, kLinear>(a);
  }
}

cudaError_t launch_fwd_tf32(const FwdLaunch& a) {
  switch (a.dp) {
    case 64: return launch_fwd_tf32_dp<64>(a);
    case 128: return launch_fwd_tf32_dp<128>(a);
  }
  return cudaErrorNotSupported;
}

int bwd_dw_splits_tf32(int H, int B, int D, int E, int sm_count) {
  if (D > 128 || H <= 0 || B <= 0 || E <= 0 || sm_count <= 0) return 1;
  constexpr int T = 32;
  const long long nT = (B + T - 1) / T, nBx = (B + kRows - 1) / kRows, nEw = (E + 127) / 128, nEx = (E + T - 1) / T;
  // Work in units of one 128 x 32 x DP product: a dW program does 4 per 32-row tile, a dX
  // program 3 per 32-wide E chunk. Split until one dW program is at most 0.8 of an SM's
  // share of the launch, keeping at least 2 tiles per split and at most 8 splits.
  const long long work = 4LL * H * nEw * nT + 3LL * H * nBx * nEx;
  const long long max_s = nT / 2 < 8 ? nT / 2 : 8;
  for (long long s = 1; s <= max_s; ++s) {
    const long long lw = 4 * ((nT + s - 1) / s);
    if (5 * lw * sm_count <= 4 * work) return int(s);
  }
  return max_s < 1 ? 1 : int(max_s);
}

int bwd_dz_splits_tf32(int H, int B, int D, int E, int sm_count) {
  if (D > 128 || H <= 0 || B <= 0 || E <= 0 || sm_count <= 0) return 1;
  constexpr int T = 32;
  const long long nT = (B + T - 1) / T, nEw = (E + 127) / 128;
  // dZ-store mode: the launch holds dW programs only, all of the same length, so it runs
  // in whole waves (as bwd_dz_splits): S in 1..16 minimising waves * (tiles per program +
  // 2) * tile time + the fp32 reduce of the partials.
  const int dp = D <= 64 ? 64 : 128;
  const double tile_s = 8.0 * 128 * T * dp / (0.5e15 / sm_count);  // 4 TF32 products of 128x32xDP
  const double hde = double(H) * D * E;
  const long long max_s = nT / 2 < 16 ? nT / 2 : 16;
  int best = 1;
  double best_t = 0;
  for (long long s = 1; s <= (max_s < 1 ? 1 : max_s); ++s) {
    const long long waves = (H * nEw * s + sm_count - 1) / sm_count;
    double t = double(waves) * double((nT + s - 1) / s + 2) * tile_s;
    if (s > 1) t += (8.0 * s + 8.0) * hde / 6.0e12 + 5e-6;
    if (s == 1 || t < best_t) best = int(s), best_t = t;
  }
  return best;
}

size_t bwd_workspace_bytes_tf32(int H, int B, int D, int E, int sm_count) {
  const int s = bwd_dw_splits_tf32(H, B, D, E, sm_count);
  return s > 1 ? size_t(2) * s * size_t(H) * D * E * sizeof(float) : 0;
}

cudaError_t launch_bwd_tf32(const BwdLaunch& a) {
  switch (a.dp) {
    case 64: return launch_bwd_tf32_dp<64>(a);
    case 128: return launch_bwd_tf32_dp<128>(a);
  }
  return cudaErrorNotSupported;
}

}  // namespace fmlp
