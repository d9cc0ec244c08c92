// Unified fused multi-head MLP backward for 128 < D <= 256 (DP = 256) on sm_100a.
//
// Same math, rounding points and program-id split as fmlp_bwd.cu (which replaces
// `flashmlp_bwd_kernel`, flashmlp.py:341-421): dW programs first, then dX programs; Z, H,
// dH and dZ never leave the SM, dW is reduced over B inside one program (no atomics).
//
// At D = 256 the D <= 128 layout does not fit: the dW1^T and dW2 accumulators of a
// 128-wide E chunk alone take all 512 TMEM columns, and a 128-row tile of X or dO is
// 64 KB. The two program kinds are therefore shaped differently:
//
// dW program, one per (head, 128-wide E chunk, D half g): owns dW1[h, 128g:128g+128, chunk]
// and dW2[h, chunk, 128g:128g+128] and loops over 64-row B tiles i. W1c^T is loaded into
// TMEM once (it is the A operand of Z^T), W2c stays in smem:
//   Z^T(i)  = W1c^T[tmem] @ X_i^T[smem]       TS M=128(e) N=64(b) K=256
//   dH^T(i) = W2c[smem] @ dO_i^T[smem]        SS M=128(e) N=64(b) K=256
//   dW2   += H^T(i)[tmem] @ dO_i[:, g][smem]  TS M=128(e) N=128(d) K=64(b)
//   dW1^T += dZ^T(i)[tmem] @ X_i[:, g][smem]  TS M=128(e) N=128(d) K=64(b)
// Both D halves recompute Z^T and dH^T. Issue order per tile as in fmlp_bwd.cu:
//   after phase 1(i): dW2(i)  Z^T(i+1)        after phase 2(i): dW1^T(i)  dH^T(i+1)
// TMEM: dW1^T [0,128) dW2 [128,256) W1c^T [256,384) Z^T [384,448) dH^T [448,512).
// smem: W2c 64 KB + X and dO through 2-stage rings of 32 KB tiles = 192 KB.
//
// dX program, one per (head, 128-row B tile), loops over 64-wide E chunks c. X_b is loaded
// into TMEM once (A operand of Z), dO_b stays in smem:
//   Z(c)   = X_b[tmem] @ W1c[smem]            TS M=128(b) N=64(e) K=256
//   dH(c)  = dO_b[smem] @ W2c^T[smem]         SS M=128(b) N=64(e) K=256
//   dX    += dZ(c)[tmem] @ W1c^T[smem]        TS M=128(b) N=256(d) K=64(e)
// Phase 1 keeps the derivative state in registers and frees Z; phase 2 packs dZ over dH.
// Issue order: after phase 1(c): Z(c+1); after phase 2(c): dX(c) dH(c+1).
// TMEM: dX [0,256) X_b [256,384) Z [384,448) dH [448,512).
// smem: dO_b 64 KB + a 3-stage W1c ring + a 2-stage W2c ring of 32 KB chunks = 224 KB.
//
// Warp roles as in fmlp_bwd.cu: warp 0 TMA, warp 1 MMA, warps 2..17 activation (warp
// (q, j) owns TMEM lanes [32q, 32q+32) and 16-column slice j of each 64-column product).
//
// dZ-store mode: the launch holds only the dW programs of D half 0, which also store their
// packed dZ^T and H^T tiles; fmlp_dw_gemm256_kernel forms the D-half-1 dW from those tiles
// (the same operands and order as a half-1 program, without its recompute of Z^T and dH^T)
// and fmlp_dx_gemm_kernel (N = 256) forms dX.
#include "fmlp_act.cuh"
#include "fmlp_kernels.h"
#include "fmlp_ptx.cuh"

namespace fmlp {

struct Bwd256Cfg {
  static constexpr int DP = 256;
  static constexpr int BM = kRows;  // rows of a dX program's B tile, M of every MMA
  static constexpr int BT = 64;     // B rows per dW tile
  static constexpr int ET = 64;     // E columns per dX chunk
  static constexpr int EW = 128;    // E rows per dW program
  // dW program smem
  static constexpr int W2C_BYTES = EW * DP * 2;  // W2 chunk, 4 regions (64 D) of 128 rows
  static constexpr int WT_BYTES = BT * DP * 2;   // 64-row tile of X or dO, 4 regions of 8 KB
  static constexpr int WS = 2;
  static constexpr int W_OFF_W2 = 0;
  static constexpr int W_OFF_X = W2C_BYTES;
  static constexpr int W_OFF_DO = W_OFF_X + WS * WT_BYTES;
  static constexpr int W_END = W_OFF_DO + WS * WT_BYTES;
  // dX program smem
  static constexpr int DOB_BYTES = BM * DP * 2;  // dO_b, 4 regions of 16 KB
  static constexpr int W1X_BYTES = DP * ET * 2;  // W1 chunk: 256 D rows x 64 E (one region)
  static constexpr int W2X_BYTES = ET * DP * 2;  // W2 chunk: 4 regions (64 D) of 64 E rows
  static constexpr int S1 = 3, S2 = 2;
  static constexpr int X_OFF_DO = 0;
  static constexpr int X_OFF_W1 = DOB_BYTES;
  static constexpr int X_OFF_W2 = X_OFF_W1 + S1 * W1X_BYTES;
  static constexpr int X_END = X_OFF_W2 + S2 * W2X_BYTES;
  static constexpr int OFF_BAR = X_END > W_END ? X_END : W_END;
  static constexpr int NBAR = 24;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr int TMEM_COLS = 512;
  // TMEM columns, dW program
  static constexpr int W_TM_DW1 = 0, W_TM_DW2 = 128, W_TM_W1T = 256, W_TM_ZT = 384, W_TM_DHT = 448;
  // TMEM columns, dX program
  static constexpr int X_TM_DX = 0, X_TM_XB = 256, X_TM_Z = 384, X_TM_DH = 448;
  static constexpr int NUM_ACT_WARPS = 16;
  static constexpr int NUM_THREADS = 32 * (2 + NUM_ACT_WARPS);
};

template <typename T, int ACT>
__global__ void __launch_bounds__(576, 1)
    fmlp_bwd256_kernel(const __grid_constant__ CUtensorMap tm_x,
                       const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_w1,
                       const __grid_constant__ CUtensorMap tm_w2, const T* __restrict__ X,
                       const T* __restrict__ W1, T* __restrict__ dX, T* __restrict__ dW1,
                       T* __restrict__ dW2, float* __restrict__ dwf, float* __restrict__ part,
                       T* __restrict__ dzt, T* __restrict__ hts, int halves, int splits, int H, int B, int D,
                       int E, uint32_t* status) {
  using C = Bwd256Cfg;
  using St = ActState<T, ACT>;
  constexpr int DP = C::DP;
  constexpr int BM = C::BM;
  constexpr int NACT = C::NUM_ACT_WARPS;
  constexpr bool kBF = Pack<T>::kBF16;
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
  const int nEw = (E + C::EW - 1) / C::EW;  // dW programs per head, D half and B range
  // halves = 2: programs for both D halves; 1 (dZ-store mode): D half 0 only
  const int nW = H * nEw * halves * splits;
  const bool is_dw = int(blockIdx.x) < nW;
  int h, idx, g = 0, split = 0;
  if (is_dw) {  // (head, B range, E chunk, D half), D half fastest
    const int per_h = nEw * halves * splits;
    h = blockIdx.x / per_h;
    const int r = blockIdx.x % per_h;
    split = r / (nEw * halves);
    const int rr = r % (nEw * halves);
    idx = rr / halves;  // E chunk
    g = rr % halves;    // D half
  } else {
    const int nBx = (B + BM - 1) / BM;
    const int p = blockIdx.x - nW;
    h = p / nBx;
    idx = p % nBx;  // B tile
  }

  // Every barrier completes at most one phase ahead of each of its waiters.
  uint64_t* in_full = bars + 0;     // dW: W2c loaded ; dX: dO_b loaded
  uint64_t* tin_full = bars + 1;    // W1c^T / X_b written into TMEM by the activation warps
  uint64_t* ring_full = bars + 2;   // 3: dW: X stages ; dX: W1c stages
  uint64_t* ring_empty = bars + 5;  // 3
  uint64_t* w2_full = bars + 8;     // 2: dW: dO stages ; dX: W2c stages
  uint64_t* w2_empty = bars + 10;   // 2
  uint64_t* p_full = bars + 12;     // 2: [0] Z^T / Z, [1] dH^T / dH
  uint64_t* a_full = bars + 14;     // 2: [0] phase 1 done, [1] phase 2 done
  uint64_t* acc_full = bars + 16;   // accumulators final
  uint64_t* done_bar = bars + 17;   // all MMAs retired

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
    }
    mbar_init(acc_full, 1);
    mbar_init(done_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_do);
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

  const int q = warp & 3;
  const int j = (warp - 2) >> 2;
  const uint32_t lane_off = uint32_t(q * 32) << 16;

  // Phase 1 over the 16 product columns at `col`: derivative state and the packed H in p;
  // if `pack_h`, also written to the first 8 of those columns.
  auto phase1 = [&](uint32_t col, St (&st)[16], bool pack_h, uint32_t (&p)[8]) {
    uint32_t v[16];
    tmem_ld16_sync(col, v);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      p[i] = act_pair<T, ACT>(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]), st[2 * i], st[2 * i + 1]);
    if (pack_h) tmem_st8(col, p);
  };
  auto signal = [&](uint64_t* bar, bool wrote_tmem) {
    if (wrote_tmem) tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
  };
  // Phase 2 over the 16 dH columns at `col`: dZ packed into the first 8 of them, `done`
  // signalled, and then, if `gz` is set, the values stored to the dZ-store workspace as
  // two 8-value pieces at gz and gz + 512 (off the chain of the products waiting on `done`).
  auto phase2 = [&](uint32_t col, const St (&st)[16], T* gz, uint64_t* done) {
    uint32_t v[16], p[8];
    tmem_ld16_sync(col, v);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      p[i] = grad_pair<T, ACT>(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]), st[2 * i], st[2 * i + 1]);
    tmem_st8(col, p);
    signal(done, true);
    if (gz != nullptr) {
      *reinterpret_cast<uint4*>(gz) = make_uint4(p[0], p[1], p[2], p[3]);
      *reinterpret_cast<uint4*>(gz + 512) = make_uint4(p[4], p[5], p[6], p[7]);
    }
  };
  // Packed operand with K = 64: the 16-bit values of K-step k sit in the first 8 columns
  // of 16-column slice k.
  auto packed_col = [](int k) -> uint32_t { return uint32_t(k) * 16; };

  if (is_dw) {
    // ==================================================================== dW program
    const int c = idx;
    // this program's 64-row tiles [t0, t0 + nT): the 128-row B tiles of its range
    const int nB128 = (B + BM - 1) / BM;
    const int bt0 = int((long long)split * nB128 / splits);
    const int bt1 = int((long long)(split + 1) * nB128 / splits);
    const int t0 = 2 * bt0;
    const int nT64 = (B + C::BT - 1) / C::BT;
    const int nT = (2 * bt1 < nT64 ? 2 * bt1 : nT64) - t0;
    uint8_t* sW2 = smem + C::W_OFF_W2;
    uint8_t* sX = smem + C::W_OFF_X;
    uint8_t* sDO = smem + C::W_OFF_DO;
    constexpr int WS = C::WS;
    if (warp == 0) {
      if (lane == 0) {
        mbar_arrive_expect_tx(in_full, C::W2C_BYTES);
        for (int r = 0; r < 4; ++r)
          for (int eh = 0; eh < 2; ++eh)
            tma_load_3d(sW2 + r * (C::EW * 128) + eh * (64 * 128), &tm_w2, in_full, 64 * r, c * C::EW + 64 * eh, h);
        uint32_t nx = 0, nd = 0;
        for (int t = 0; t < nT; ++t) {
          const int s = t % WS;
          const uint32_t par = ((t / WS) & 1) ^ 1;
          if (!mbar_wait(&ring_empty[s], par, ctx)) break;
          mbar_arrive_expect_tx(&ring_full[s], C::WT_BYTES);
          for (int r = 0; r < 4; ++r)
            tma_load_3d(sX + s * C::WT_BYTES + r * (C::BT * 128), &tm_x, &ring_full[s], 64 * r, (t0 + t) * C::BT, h);
          ++nx;
          if (!mbar_wait(&w2_empty[s], par, ctx)) break;
          mbar_arrive_expect_tx(&w2_full[s], C::WT_BYTES);
          for (int r = 0; r < 4; ++r)
            tma_load_3d(sDO + s * C::WT_BYTES + r * (C::BT * 128), &tm_do, &w2_full[s], 64 * r, (t0 + t) * C::BT, h);
          ++nd;
        }
        mbar_wait(in_full, 0, drain);
        for (uint32_t i = 0; i < WS; ++i) {
          if (nx > i) mbar_wait(&ring_full[(nx - 1 - i) % WS], ((nx - 1 - i) / WS) & 1, drain);
          if (nd > i) mbar_wait(&w2_full[(nd - 1 - i) % WS], ((nd - 1 - i) / WS) & 1, drain);
        }
      }
    } else if (warp == 1) {
      constexpr uint32_t idesc_p = make_idesc_f16(kBF, 128, C::BT, false, false);  // A K / tmem, B K
      constexpr uint32_t idesc_w = make_idesc_f16(kBF, 128, 128, false, true);     // A tmem, B MN
      const uint64_t w2k = make_sdesc_sw128(smem_u32(sW2), 16, 1024);
      // Z^T(t) (m = 0) or dH^T(t) (m = 1); K over the padded 256 (zero-filled).
      auto issue_prod = [&](int m, int t) {
        const int s = t % WS;
        if (elect_one()) {
          const uint64_t bk = make_sdesc_sw128(smem_u32((m == 0 ? sX : sDO) + s * C::WT_BYTES), 16, 1024);
          const uint32_t d = tmem + (m == 0 ? C::W_TM_ZT : C::W_TM_DHT);
#pragma unroll
          for (int k = 0; k < DP / 16; ++k) {
            const uint64_t bkk = sdesc_add(bk, (k >> 2) * (C::BT * 128) + (k & 3) * 32);
            if (m == 0)
              mma_ts(d, tmem + C::W_TM_W1T + 8 * k, bkk, idesc_p, k > 0 ? 1u : 0u);
            else
              mma_ss(d, sdesc_add(w2k, (k >> 2) * (C::EW * 128) + (k & 3) * 32), bkk, idesc_p, k > 0 ? 1u : 0u);
          }
          mma_commit(&p_full[m]);
        }
        __syncwarp();
      };
      // dW2[:, g] += H^T(t) @ dO_t[:, g] (m = 0) or dW1^T[:, g] += dZ^T(t) @ X_t[:, g] (m = 1);
      // the D half of the tile is two 64-column regions (MN-major B, LBO = region stride).
      auto issue_dw = [&](int m, int t) {
        const int s = t % WS;
        if (elect_one()) {
          const uint8_t* tile = (m == 0 ? sDO : sX) + s * C::WT_BYTES + (2 * g) * (C::BT * 128);
          const uint64_t bm = make_sdesc_sw128(smem_u32(tile), C::BT * 128, 1024);
          const uint32_t d = tmem + (m == 0 ? C::W_TM_DW2 : C::W_TM_DW1);
          const uint32_t a = tmem + (m == 0 ? C::W_TM_ZT : C::W_TM_DHT);
          const uint32_t acc0 = t > 0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < C::BT / 16; ++k)
            mma_ts(d, a + packed_col(k), sdesc_add(bm, k * 2048), idesc_w, k > 0 ? 1u : acc0);
          mma_commit(m == 0 ? &w2_empty[s] : &ring_empty[s]);  // last reader of dO_t / X_t
        }
        __syncwarp();
      };
      auto wait_x = [&](int t) { return warp_wait(&ring_full[t % WS], (t / WS) & 1, ctx); };
      auto wait_do = [&](int t) { return warp_wait(&w2_full[t % WS], (t / WS) & 1, ctx); };
      bool ok = warp_wait(in_full, 0, ctx) && warp_wait(tin_full, 0, ctx) && nT > 0 && wait_x(0) && wait_do(0);
      tc_fence_after();
      if (ok) {
        issue_prod(0, 0);
        issue_prod(1, 0);
      }
      for (int t = 0; t < nT && ok; ++t) {
        const bool more = t + 1 < nT;
        if (!(ok = warp_wait(&a_full[0], t & 1, ctx))) break;  // H^T(t) packed
        tc_fence_after();
        issue_dw(0, t);
        if (more) {  // overwrites H^T(t) after dW2(t) read it
          if (!(ok = wait_x(t + 1))) break;
          tc_fence_after();
          issue_prod(0, t + 1);
        }
        if (!(ok = warp_wait(&a_full[1], t & 1, ctx))) break;  // dZ^T(t) packed
        tc_fence_after();
        issue_dw(1, t);
        if (more) {  // overwrites dZ^T(t) after dW1^T(t) read it
          if (!(ok = wait_do(t + 1))) break;
          tc_fence_after();
          issue_prod(1, t + 1);
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
      // W1c^T into TMEM: lane e of quadrant q holds W1[h, d, c*128 + 32q + lane] for
      // d in [64j, 64j+64) as 32 packed columns at W1T + 32j (zero outside D and E).
      {
        const int e = c * C::EW + q * 32 + lane;
        uint32_t p[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int d0 = 64 * j + 2 * i;
          uint32_t lo = 0, hi = 0;
          if (e < E) {
            const uint16_t* col = reinterpret_cast<const uint16_t*>(W1) + size_t(h) * D * E + e;
            if (d0 < D) lo = col[size_t(d0) * E];
            if (d0 + 1 < D) hi = col[size_t(d0 + 1) * E];
          }
          p[i] = lo | (hi << 16);
        }
        const uint32_t base = tmem + lane_off + C::W_TM_W1T + 32 * j;
        tmem_st16(base, *reinterpret_cast<const uint32_t(*)[16]>(&p[0]));
        tmem_st16(base + 16, *reinterpret_cast<const uint32_t(*)[16]>(&p[16]));
        signal(tin_full, true);
      }
      // Activation warps: B columns [16j, 16j+16) of Z^T / dH^T.
      const uint32_t zt = tmem + lane_off + C::W_TM_ZT + 16 * j;
      const uint32_t dt = tmem + lane_off + C::W_TM_DHT + 16 * j;
      // dZ-store mode (the D-half-0 programs; both halves compute the same dZ^T): the tiled
      // workspace of fmlp_bwd.cu, one 128 x 128 tile per (head, 128-wide E chunk, 128-row B
      // tile) laid out [e / 64][b / 8][e % 64][b % 8]. A 64-row tile t is half (t % 2) of
      // B tile t / 2; this thread (e = 32q + lane) owns b = 64(t%2) + 16j + 0..15: 8-b
      // groups 8(t%2) + 2j and the next. 32-bit element offsets (the workspace holds at
      // most 2^32 elements).
      const uint32_t dz_off = uint32_t(((size_t(h) * nEw + c) * nB128 + bt0) * (BM * 128)) + (q >> 1) * 8192 +
                              (2 * j) * 512 + ((q & 1) * 32 + lane) * 8;
      T* const dz = (g == 0) ? dzt : nullptr;
      // H^T tiles (dZ-store mode, for fmlp_dw_gemm256_kernel): one 128 x 128 tile per (head,
      // E chunk, 128-row B tile) laid out [b / 8][e][b % 8], the K-major no-swizzle operand
      // layout, so a 64-row half tile is 16 KB of contiguous memory; this thread writes the
      // 8-b groups 8(t%2) + 2j and the next of row e.
      const uint32_t h_off = uint32_t(((size_t(h) * nEw + c) * nB128 + bt0) * (BM * 128)) + (2 * j) * 1024 +
                             (q * 32 + lane) * 8;
      T* const hs = (g == 0) ? hts : nullptr;
      bool ok = true;
      for (int t = 0; t < nT && ok; ++t) {
        St st[16];
        uint32_t ph[8];
        if (!(ok = mbar_wait(&p_full[0], t & 1, ctx))) break;
        tc_fence_after();
        phase1(zt, st, true, ph);  // H^T packed over Z^T
        signal(&a_full[0], true);
        if (hs != nullptr) {  // off the chain of the products waiting on a_full[0]
          T* hp = hs + (h_off + uint32_t(t >> 1) * (BM * 128) + uint32_t(t & 1) * 8192);
          *reinterpret_cast<uint4*>(hp) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
          *reinterpret_cast<uint4*>(hp + 1024) = make_uint4(ph[4], ph[5], ph[6], ph[7]);
        }
        if (!(ok = mbar_wait(&p_full[1], t & 1, ctx))) break;
        tc_fence_after();
        phase2(dt, st, dz != nullptr ? dz + (dz_off + uint32_t(t >> 1) * (BM * 128) + uint32_t(t & 1) * 4096) : nullptr,
               &a_full[1]);
      }
      if (ok && (ok = mbar_wait(acc_full, 0, ctx))) {
        tc_fence_after();
        const int e = c * C::EW + q * 32 + lane;
        const int d0 = g * 128 + 32 * j;  // this warp's 32 accumulator columns
        // fp32 sums: this B range's partials (fmlp_dw_reduce_kernel adds the ranges in
        // order), or the unrounded fp32 output
        float* fout = part != nullptr ? part + size_t(split) * 2 * (size_t(H) * D * E) : dwf;
        if (fout != nullptr) {
          // dW1 laid out (H, D, E), then dW2 laid out (H, E, D)
          float* f1 = fout;
          float* f2 = fout + size_t(H) * D * E;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            uint32_t v[16];
            tmem_ld16_sync(tmem + lane_off + C::W_TM_DW1 + 32 * j + 16 * u, v);
            if (e < E) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int d = d0 + 16 * u + i;
                if (d < D) f1[(size_t(h) * D + d) * E + e] = __uint_as_float(v[i]);
              }
            }
          }
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            uint32_t v[16];
            tmem_ld16_sync(tmem + lane_off + C::W_TM_DW2 + 32 * j + 16 * u, v);
            const int cc = d0 + 16 * u;
            if (e < E && cc < D) {  // D % 16 == 0: all 16 columns are inside
              float4* dst = reinterpret_cast<float4*>(f2 + (size_t(h) * E + e) * D + cc);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                dst[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                     __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
            }
          }
        } else {
          // dW1^T rows are E, columns D: dW1[h, d, e]; lanes hold consecutive e, so each
          // column d is one coalesced 64-byte store across the warp.
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            uint32_t v[16];
            tmem_ld16_sync(tmem + lane_off + C::W_TM_DW1 + 32 * j + 16 * u, v);
            if (e < E) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int d = d0 + 16 * u + i;
                if (d < D) {
                  const uint32_t pk = Pack<T>::pack(__uint_as_float(v[i]), 0.f);
                  reinterpret_cast<uint16_t*>(dW1)[(size_t(h) * D + d) * E + e] = uint16_t(pk & 0xFFFFu);
                }
              }
            }
          }
          T* w2row = dW2 + (size_t(h) * E + e) * D;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            uint32_t v[16], p[8];
            tmem_ld16_sync(tmem + lane_off + C::W_TM_DW2 + 32 * j + 16 * u, v);
            plain_pack<T, 8>(v, p);
            const int cc = d0 + 16 * u;
            if (e < E) {
              uint4* dst = reinterpret_cast<uint4*>(w2row + cc);
              if (cc + 8 <= D) dst[0] = make_uint4(p[0], p[1], p[2], p[3]);
              if (cc + 16 <= D) dst[1] = make_uint4(p[4], p[5], p[6], p[7]);
            }
          }
        }
      }
    }
  } else {
    // ==================================================================== dX program
    const int bt = idx;
    const int nE = (E + C::ET - 1) / C::ET;
    uint8_t* sDO = smem + C::X_OFF_DO;
    uint8_t* sW1 = smem + C::X_OFF_W1;
    uint8_t* sW2 = smem + C::X_OFF_W2;
    if (warp == 0) {
      if (lane == 0) {
        mbar_arrive_expect_tx(in_full, C::DOB_BYTES);
        for (int r = 0; r < 4; ++r)
          for (int rh = 0; rh < 2; ++rh)
            tma_load_3d(sDO + r * (BM * 128) + rh * (64 * 128), &tm_do, in_full, 64 * r, bt * BM + 64 * rh, h);
        uint32_t n1 = 0, n2 = 0;
        for (int c = 0; c < nE; ++c) {  // the order the MMA warp consumes them
          const int s1 = c % C::S1, s2 = c % C::S2;
          if (!mbar_wait(&ring_empty[s1], ((c / C::S1) & 1) ^ 1, ctx)) break;
          mbar_arrive_expect_tx(&ring_full[s1], C::W1X_BYTES);
          tma_load_3d(sW1 + s1 * C::W1X_BYTES, &tm_w1, &ring_full[s1], c * C::ET, 0, h);
          ++n1;
          if (!mbar_wait(&w2_empty[s2], ((c / C::S2) & 1) ^ 1, ctx)) break;
          mbar_arrive_expect_tx(&w2_full[s2], C::W2X_BYTES);
          for (int r = 0; r < 4; ++r)
            tma_load_3d(sW2 + s2 * C::W2X_BYTES + r * (C::ET * 128), &tm_w2, &w2_full[s2], 64 * r, c * C::ET, h);
          ++n2;
        }
        mbar_wait(in_full, 0, drain);
        for (uint32_t i = 0; i < C::S1; ++i)
          if (n1 > i) mbar_wait(&ring_full[(n1 - 1 - i) % C::S1], ((n1 - 1 - i) / C::S1) & 1, drain);
        for (uint32_t i = 0; i < C::S2; ++i)
          if (n2 > i) mbar_wait(&w2_full[(n2 - 1 - i) % C::S2], ((n2 - 1 - i) / C::S2) & 1, drain);
      }
    } else if (warp == 1) {
      constexpr uint32_t idesc_z = make_idesc_f16(kBF, 128, C::ET, false, true);   // A tmem, B MN
      constexpr uint32_t idesc_h = make_idesc_f16(kBF, 128, C::ET, false, false);  // A K, B K
      constexpr uint32_t idesc_x = make_idesc_f16(kBF, 128, DP, false, false);     // A tmem, B K
      const uint64_t dk = make_sdesc_sw128(smem_u32(sDO), 16, 1024);
      auto issue_z = [&](int c) {  // Z(c) = X_b @ W1c; W1c rows are K (D), 64 E per row
        if (elect_one()) {
          const uint64_t w1m = make_sdesc_sw128(smem_u32(sW1 + (c % C::S1) * C::W1X_BYTES), C::W1X_BYTES, 1024);
#pragma unroll
          for (int k = 0; k < DP / 16; ++k)
            mma_ts(tmem + C::X_TM_Z, tmem + C::X_TM_XB + 8 * k, sdesc_add(w1m, k * 2048), idesc_z, k > 0 ? 1u : 0u);
          mma_commit(&p_full[0]);
        }
        __syncwarp();
      };
      auto issue_dh = [&](int c) {  // dH(c) = dO_b @ W2c^T
        const int s = c % C::S2;
        if (elect_one()) {
          const uint64_t w2k = make_sdesc_sw128(smem_u32(sW2 + s * C::W2X_BYTES), 16, 1024);
#pragma unroll
          for (int k = 0; k < DP / 16; ++k)
            mma_ss(tmem + C::X_TM_DH, sdesc_add(dk, (k >> 2) * (BM * 128) + (k & 3) * 32),
                   sdesc_add(w2k, (k >> 2) * (C::ET * 128) + (k & 3) * 32), idesc_h, k > 0 ? 1u : 0u);
          mma_commit(&p_full[1]);
          mma_commit(&w2_empty[s]);  // dH(c) is the W2c stage's only reader
        }
        __syncwarp();
      };
      auto issue_dx = [&](int c) {  // dX += dZ(c) @ W1c^T; the same W1c tile, K-major (rows D)
        const int s = c % C::S1;
        if (elect_one()) {
          const uint64_t w1k = make_sdesc_sw128(smem_u32(sW1 + s * C::W1X_BYTES), 16, 1024);
          const uint32_t acc0 = c > 0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < C::ET / 16; ++k)
            mma_ts(tmem + C::X_TM_DX, tmem + C::X_TM_DH + packed_col(k), sdesc_add(w1k, k * 32), idesc_x,
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
        if (!(ok = warp_wait(&a_full[1], c & 1, ctx))) break;  // dZ(c) packed over dH(c)
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
      // X_b into TMEM: lane b of quadrant q holds X[h, row, d] for d in [64j, 64j+64) as 32
      // packed columns at XB + 32j (zero outside B and D; D % 16 == 0, so an 8-element
      // group is entirely inside or outside D).
      {
        uint32_t p[32];
        const uint4* src = reinterpret_cast<const uint4*>(X + (size_t(h) * B + row) * D + 64 * j);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          uint4 v = make_uint4(0, 0, 0, 0);
          if (row < B && 64 * j + 8 * i < D) v = src[i];
          p[4 * i] = v.x, p[4 * i + 1] = v.y, p[4 * i + 2] = v.z, p[4 * i + 3] = v.w;
        }
        const uint32_t base = tmem + lane_off + C::X_TM_XB + 32 * j;
        tmem_st16(base, *reinterpret_cast<const uint32_t(*)[16]>(&p[0]));
        tmem_st16(base + 16, *reinterpret_cast<const uint32_t(*)[16]>(&p[16]));
        signal(tin_full, true);
      }
      // Per E chunk: E columns [16j, 16j+16) of Z and dH.
      const uint32_t za = tmem + lane_off + C::X_TM_Z + 16 * j;
      const uint32_t da = tmem + lane_off + C::X_TM_DH + 16 * j;
      bool ok = true;
      for (int c = 0; c < nE && ok; ++c) {
        St st[16];
        uint32_t ph[8];
        if (!(ok = mbar_wait(&p_full[0], c & 1, ctx))) break;
        tc_fence_after();
        phase1(za, st, false, ph);  // derivative state only
        signal(&a_full[0], false);
        if (!(ok = mbar_wait(&p_full[1], c & 1, ctx))) break;
        tc_fence_after();
        phase2(da, st, nullptr, &a_full[1]);  // dZ packed over dH
      }
      if (ok && (ok = mbar_wait(acc_full, 0, ctx))) {
        tc_fence_after();
        T* xrow = dX + (size_t(h) * B + row) * D;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint32_t v[16], p[8];
          tmem_ld16_sync(tmem + lane_off + C::X_TM_DX + 64 * j + 16 * u, v);
          plain_pack<T, 8>(v, p);
          const int cc = 64 * j + 16 * u;
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

template <typename T, int ACT>
static cudaError_t launch_bwd256_t(const BwdLaunch& a) {
  using C = Bwd256Cfg;
  auto kern = fmlp_bwd256_kernel<T, ACT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int nBx = (a.B + kRows - 1) / kRows;
  const int nEw = (a.E + C::EW - 1) / C::EW;
  // dZ-store mode: the D-half-0 dW programs only (they store dZ^T and H^T), then
  // fmlp_dw_gemm256_kernel forms the D-half-1 dW and fmlp_dx_gemm_kernel dX
  const bool dz = a.dzt != nullptr;
  const int halves = dz ? 1 : 2;
  T* const hts = dz ? reinterpret_cast<T*>(a.dzt) + dz_tile_elems(a.H, a.B, a.E) : nullptr;
  // dW programs over `splits` B ranges (fp32 partials reduced afterwards) when there are
  // too few (head, E chunk, D half) programs for the SMs
  const int splits = a.splits < 1 ? 1 : a.splits;
  if (splits > 1 && (a.part == nullptr || splits > nBx)) return cudaErrorInvalidValue;
  const long long grid = (long long)a.H * ((long long)halves * nEw * splits + (dz ? 0 : nBx));
  if (grid <= 0 || grid > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  kern<<<unsigned(grid), C::NUM_THREADS, C::SMEM, a.stream>>>(
      a.tm_x, a.tm_do, a.tm_w1, a.tm_w2, reinterpret_cast<const T*>(a.x), reinterpret_cast<const T*>(a.w1),
      reinterpret_cast<T*>(a.dx), reinterpret_cast<T*>(a.dw1), reinterpret_cast<T*>(a.dw2), a.dw_f32,
      splits > 1 ? a.part : nullptr, reinterpret_cast<T*>(a.dzt), hts, halves, splits, a.H, a.B, a.D, a.E,
      a.status);
  cudaError_t le = cudaGetLastError();
  if (le == cudaSuccess && dz) le = launch_dw_gemm256(a);
  if (le == cudaSuccess && dz) le = launch_dx_gemm(a);
  if (le != cudaSuccess || splits == 1) return le;
  return launch_dw_reduce(a);
}

template <typename T>
static cudaError_t launch_bwd256_act(const BwdLaunch& a) {
  switch (a.act) {
    case kLeakyRelu: return launch_bwd256_t<T, kLeakyRelu>(a);
    case kSilu: return launch_bwd256_t<T, kSilu>(a);
    case kSigmoid: return launch_bwd256_t<T, kSigmoid>(a);
    default: return launch_bwd256_t<T, kLinear>(a);
  }
}

int bwd256_smem_bytes() { return Bwd256Cfg::SMEM; }

cudaError_t launch_bwd256(const BwdLaunch& a) {
  return a.bf16 ? launch_bwd256_act<__nv_bfloat16>(a) : launch_bwd256_act<__half>(a);
}

}  // namespace fmlp
