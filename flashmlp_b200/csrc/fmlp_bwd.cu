// Unified fused multi-head MLP backward for sm_100a.
//
// Replaces the Triton kernel `flashmlp_bwd_kernel` (flashmlp.py:341-421) and its helpers
// `_flashmlp_bwd_dx` (flashmlp.py:165-244) and `_flashmlp_bwd_dw1w2` (flashmlp.py:247-329).
// One launch holds two kinds of programs, split by program id as in the reference:
//   * dW programs, one per (head, 128-wide E chunk): own dW1[h,:,chunk] and dW2[h,chunk,:]
//     and loop over every B tile of the head (deterministic, no atomics on outputs);
//   * dX programs, one per (head, 128-row B tile): own dX[h,tile,:] and loop over E.
// All dW programs come first in program-id order so the long ones start first.
// When a launch has too few dW programs to keep the SMs busy (few heads and E chunks,
// e.g. 4 heads per GPU when 32 heads are sharded over 8 GPUs), each (head, E chunk) is
// split into S dW programs over contiguous B ranges; they write fp32 partial sums to the
// caller's workspace and fmlp_dw_reduce_kernel adds them in the fixed order s = 0..S-1
// (deterministic, still no atomics).
// With SX (shared input: X, dO and dX are (B, D) matrices used by every head, the
// backward of the reference's FlashMLP on a 2-D input, flashmlp.py:603-614), the dW
// programs read the shared X/dO tiles, there is one dX program per B tile that loops over
// (head, E chunk) pairs and accumulates dX over all heads in TMEM (the sum the expand's
// backward takes), and the 1/H of the head mean is applied to dH (and so to dZ and dW1)
// and to dW2 in fp32.
// Both recompute Z = X@W1 and H = act(Z) per chunk and form dH = dO@W2^T and
// dZ = dH * act'(Z) in fp32; H and dZ are rounded to the input dtype before they enter
// the next products (flashmlp.py:212-235, :294-320).
//
// Both programs use the same shape of pipeline: one TMA warp, one MMA warp and 16
// activation warps that work in two phases per chunk: phase 1 reads Z (the SFU-heavy
// activation), phase 2 reads dH and forms dZ. The 16-bit operands the next products need
// are packed into TMEM columns whose fp32 contents have already been read. TMEM columns
// are overwritten only after the MMA that reads them (MMAs from one thread run in order).
// All 512 TMEM columns are in use, so the issue order below is what overlaps the SFU work
// with the tensor work.
//
// dW program (transposed so H^T and dZ^T land in TMEM as K-major A operands). Phase 1
// packs H^T over Z^T, phase 2 packs dZ^T over dH^T. Issue order per B tile i:
//   after phase 1(i): dW2(i)  Z^T(i+1)        after phase 2(i): dW1^T(i)  dH^T(i+1)
//   Z^T(i)  = W1c^T[smem] @ X_i^T[smem]   SS M=128(e) N=128(b) K=DP
//   dH^T(i) = W2c[smem] @ dO_i^T[smem]    SS M=128(e) N=128(b) K=DP
//   dW2    += H^T(i)[tmem] @ dO_i[smem]   TS M=128(e) N=DP     K=128(b)
//   dW1^T  += dZ^T(i)[tmem] @ X_i[smem]   TS M=128(e) N=DP     K=128(b)
// X and dO tiles stream through separate 2-stage rings: dW2(i) frees dO_i, dW1^T(i) frees
// X_i, so X_{i+1} lands while phase 2(i) runs.
// Fused-phase schedule (every activation but sigmoid): the activation warps load Z^T(i)
// into registers and release its columns at once (z_free), so Z^T(i+1) is computed while
// they are still on the SFU, where they also form the factor dH is multiplied by; after
// loading dH^T(i) they pack H^T(i) into the first 16 and dZ^T(i) into the last 16
// columns of each 32-column dH^T slice. Issue order: after z_free(i): Z^T(i+1);
// after both are packed: dW2(i) dW1^T(i) dH^T(i+1). X_{i+1} is read before dW1^T(i) frees
// X_i, so the X ring has 3 stages in this schedule.
//
// dX program (Z double-buffered). Phase 1 keeps the derivative state in registers, phase 2
// packs dZ(c) over the Z(c) buffer, so the dH columns are free as soon as phase 2 has read
// them and dH(c+1) runs while phase 1(c+1) does; the activation warps never wait on the
// dZ -> dX -> dH chain. Issue order after phase 2(c):  dH(c+1)  dX(c)  Z(c+2)
//   Z(c)   = X_b[smem] @ W1c[smem]        SS M=128(b) N=128(e) K=DP
//   dH(c)  = dO_b[smem] @ W2c^T[smem]     SS M=128(b) N=128(e) K=DP
//   dX    += dZ(c)[tmem] @ W1c^T[smem]    TS M=128(b) N=DP     K=128(e)
// W1 chunks stream through a 3-stage ring (read by Z(c) and dX(c), with Z(c+1) and Z(c+2)
// in between), W2 chunks through a 2-stage ring (read by dH(c) only).
#include "fmlp_act.cuh"
#include "fmlp_kernels.h"
#include "fmlp_ptx.cuh"

namespace fmlp {

template <int DP>
struct BwdCfg {
  static constexpr int BM = kRows;
  static constexpr int ET = 128;                  // E chunk of both program kinds
  static constexpr int TILE_BYTES = BM * DP * 2;  // one 128-row tile of X or dO
  static constexpr int W1C_BYTES = DP * ET * 2;   // one E chunk of W1 (DP rows x 128)
  static constexpr int W2C_BYTES = ET * DP * 2;   // one E chunk of W2 (128 rows x DP)
  // dX program: X_b, dO_b, a 3-stage W1c ring and a 2-stage W2c ring
  static constexpr int WS1 = 3, WS2 = 2;
  static constexpr int X_OFF_X = 0;
  static constexpr int X_OFF_DO = TILE_BYTES;
  static constexpr int X_OFF_W1 = 2 * TILE_BYTES;
  static constexpr int X_OFF_W2 = X_OFF_W1 + WS1 * W1C_BYTES;
  static constexpr int X_END = X_OFF_W2 + WS2 * W2C_BYTES;
  // dW program: W1c, W2c, X ring (room for 3 stages), 2-stage dO ring
  static constexpr int XDS = 2;   // dO stages (and X stages of the two-phase schedule)
  static constexpr int XS_MAX = 3;
  static constexpr int W_OFF_W1 = 0;
  static constexpr int W_OFF_W2 = W1C_BYTES;
  static constexpr int W_OFF_X = W1C_BYTES + W2C_BYTES;
  static constexpr int W_OFF_DO = W_OFF_X + XS_MAX * TILE_BYTES;
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
  static constexpr int X_TM_DX = 0;             // dX accumulator, DP columns
  static constexpr int X_TM_Z = DP;             // Z, 2 buffers x 128 columns (dZ packed in)
  static constexpr int X_TM_DH = DP + 256;      // dH, 128 columns
  // TMEM columns, dW program
  static constexpr int W_TM_DW1 = 0;             // dW1^T accumulator, DP columns
  static constexpr int W_TM_DW2 = DP;            // dW2 accumulator, DP columns
  static constexpr int W_TM_ZT = 2 * DP;         // Z^T 128 columns (H^T packed in place)
  static constexpr int W_TM_DHT = 2 * DP + 128;  // dH^T 128 columns (dZ^T packed in place)
  static_assert(X_TM_DH + 128 <= TMEM_COLS, "TMEM budget (dX)");
  static_assert(W_TM_DHT + 128 <= TMEM_COLS, "TMEM budget (dW)");
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr int NUM_ACT_WARPS = 16;  // 4 per TMEM lane quadrant
  static constexpr int FIRST_ACT_WARP = 2;  // warp 0 TMA, warp 1 MMA
  static constexpr int NUM_THREADS = 32 * (FIRST_ACT_WARP + NUM_ACT_WARPS);
};

template <int DP, typename T, int ACT, bool SX>
__global__ void __launch_bounds__(576, 1)
    fmlp_bwd_kernel(const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_w1,
                    const __grid_constant__ CUtensorMap tm_w2, T* __restrict__ dX,
                    T* __restrict__ dW1, T* __restrict__ dW2, float* __restrict__ part,
                    T* __restrict__ dzt, int splits, int H, int B, int D, int E, uint32_t* status) {
  using C = BwdCfg<DP>;
  using St = ActState<T, ACT>;
  constexpr int BM = C::BM;
  constexpr int NACT = C::NUM_ACT_WARPS;
  // dW programs run the fused-phase schedule (see the dW notes) for every activation but
  // sigmoid, whose two recorded factors per element make it spill and measured 5-10 %
  // slower (C4 silu bf16 -2 % against the two-phase schedule, fp16 -3 %, leaky_relu and
  // linear -2 to -3 %)
  constexpr bool kFused = ACT != kSigmoid;
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
  const int nE = (E + C::ET - 1) / C::ET;
  const int nW = H * nE * splits;  // dW programs: (head, split, E chunk), chunk fastest
  // dX programs loop over E chunks of their head, or (SX) over (head, E chunk) pairs
  const int nEv = SX ? H * nE : nE;
  const float inv_h = SX ? 1.0f / float(H) : 1.0f;
  const bool is_dw = int(blockIdx.x) < nW;
  int h, idx, bt0 = 0, bt1 = nB, split = 0;
  if (is_dw) {
    h = blockIdx.x / (nE * splits);
    const int r = blockIdx.x % (nE * splits);
    split = r / nE;
    idx = r % nE;  // E chunk
    bt0 = int((long long)split * nB / splits);  // this program's B tiles [bt0, bt1)
    bt1 = int((long long)(split + 1) * nB / splits);
  } else {
    const int p = blockIdx.x - nW;
    h = SX ? 0 : p / nB;  // SX: one program per B tile for all heads
    idx = SX ? p : p % nB;  // B tile
  }

  // Every barrier below completes at most one phase ahead of each of its waiters, so
  // parity waits cannot alias.
  uint64_t* in_full = bars + 0;     // dX: X_b+dO_b loaded ; dW: W1c+W2c loaded
  uint64_t* ring_full = bars + 1;   // 3: dX: W1c stages ; dW: X stages
  uint64_t* ring_empty = bars + 4;  // 3
  uint64_t* w2_full = bars + 7;     // 2: dX: W2c stages ; dW: dO stages
  uint64_t* w2_empty = bars + 17;   // 2
  uint64_t* p_full = bars + 9;      // 3: [0] Z^T / Z buffer 0, [1] dH^T / dH, [2] Z buffer 1
  uint64_t* a_full = bars + 12;     // 2: [0] phase 1 done (dW only), [1] phase 2 done
  uint64_t* acc_full = bars + 15;   // accumulators final
  uint64_t* done_bar = bars + 16;   // all MMAs retired
  uint64_t* z_free = bars + 19;     // dW, fused schedule: Z^T(i) has been read into registers

  if (threadIdx.x == 0) {
    misc[1] = 0;
    misc[2] = 0;
    mbar_init(in_full, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&w2_full[i], 1);
      mbar_init(&w2_empty[i], 1);
    }
    for (int i = 0; i < 3; ++i) mbar_init(&p_full[i], 1);
    for (int i = 0; i < 2; ++i) mbar_init(&a_full[i], NACT);
    mbar_init(acc_full, 1);
    mbar_init(done_bar, 1);
    mbar_init(z_free, NACT);
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

  // Activation warps: warp (q, j) owns TMEM lanes [32q, 32q+32) and column slice j
  // (32 columns of every 128-column product).
  const int q = warp & 3;
  const int j = (warp - C::FIRST_ACT_WARP) >> 2;
  const uint32_t lane_off = uint32_t(q * 32) << 16;

  // Phase 1 over the 32 Z columns at `col`: the derivative state in registers and, if
  // `pack_h`, the packed H in the first 16 of those columns. Loads are pipelined in halves.
  auto phase1 = [&](uint32_t col, St (&st)[32], bool pack_h) {
    uint32_t va[16], vb[16], ph[8];
    tmem_ld16_async(col, va);
    tmem_wait_ld_dep(va);
    tmem_ld16_async(col + 16, vb);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      ph[i] = act_pair<T, ACT>(__uint_as_float(va[2 * i]), __uint_as_float(va[2 * i + 1]), st[2 * i], st[2 * i + 1]);
    if (pack_h) tmem_st8(col, ph);
    tmem_wait_ld_dep(vb);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      ph[i] = act_pair<T, ACT>(__uint_as_float(vb[2 * i]), __uint_as_float(vb[2 * i + 1]), st[16 + 2 * i],
                               st[17 + 2 * i]);
    if (pack_h) tmem_st8(col + 8, ph);
  };
  // 16 packed 16-bit values (16 consecutive b of this thread's dZ^T row) to the dZ-store
  // workspace: two 16-byte pieces, 8 b each, which the tiled layout keeps 512 elements
  // (one 8-b group of 64 e rows) apart
  auto store_dz = [](T* g, const uint32_t (&p)[8]) {
    *reinterpret_cast<uint4*>(g) = make_uint4(p[0], p[1], p[2], p[3]);
    *reinterpret_cast<uint4*>(g + 512) = make_uint4(p[4], p[5], p[6], p[7]);
  };
  // dH as phase 2 uses it: with a shared input the upstream gradient of the head mean is
  // dO / H, applied here in fp32 (dH is linear in dO).
  auto dh_in = [&](uint32_t v) -> float {
    if constexpr (SX) return __uint_as_float(v) * inv_h;
    return __uint_as_float(v);
  };
  auto signal = [&](uint64_t* bar, bool wrote_tmem) {
    if (wrote_tmem) tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
  };
  // Phase 2 over the 32 dH columns at `src`: dZ packed into the 16 columns at `dst`
  // (`dst` == `src`, or columns this warp has already read in phase 1), `done` signalled
  // once they are in TMEM, and then, if `g` is set, the same 32 16-bit values stored to
  // the dZ-store workspace at g (off the chain of the products waiting on `done`).
  auto phase2 = [&](uint32_t src, uint32_t dst, const St (&st)[32], T* g, uint64_t* done) {
    uint32_t va[16], vb[16], pd[8], pe[8];
    tmem_ld16_async(src, va);
    tmem_wait_ld_dep(va);
    tmem_ld16_async(src + 16, vb);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      pd[i] = grad_pair<T, ACT>(dh_in(va[2 * i]), dh_in(va[2 * i + 1]), st[2 * i], st[2 * i + 1]);
    tmem_st8(dst, pd);
    tmem_wait_ld_dep(vb);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      pe[i] = grad_pair<T, ACT>(dh_in(vb[2 * i]), dh_in(vb[2 * i + 1]), st[16 + 2 * i],
                                st[17 + 2 * i]);
    tmem_st8(dst + 8, pe);
    signal(done, true);
    if (g != nullptr) {
      store_dz(g, pd);
      store_dz(g + 1024, pe);
    }
  };

  // Packed operands with K = 128 rows/columns: the 16-bit values of columns [16k, 16k+16)
  // sit in the first 16 columns of slice k/2 (32 columns per slice) at offset 8*(k%2).
  auto packed_col = [](int k) -> uint32_t { return (k >> 1) * 32 + (k & 1) * 8; };

  if (is_dw) {
    // ==================================================================== dW program
    const int c = idx;
    uint8_t* sW1 = smem + C::W_OFF_W1;
    uint8_t* sW2 = smem + C::W_OFF_W2;
    uint8_t* sX = smem + C::W_OFF_X;
    uint8_t* sDO = smem + C::W_OFF_DO;
    constexpr int XDS = C::XDS;
    // X stages: the fused schedule issues Z^T(i+1) before dW1^T(i) frees X_i's stage
    constexpr int XS = kFused ? C::XS_MAX : XDS;
    const int nT = bt1 - bt0;  // B tiles of this program; tile i of the loops is bt0 + i
    if (warp == 0) {
      if (lane == 0) {
        mbar_arrive_expect_tx(in_full, C::W1C_BYTES + C::W2C_BYTES);
        for (int r = 0; r < 2; ++r) tma_load_3d(sW1 + r * DP * 128, &tm_w1, in_full, c * 128 + 64 * r, 0, h);
        for (int r = 0; r < DP / 64; ++r) tma_load_3d(sW2 + r * 128 * 128, &tm_w2, in_full, 64 * r, c * 128, h);
        uint32_t nx = 0, nd = 0;  // X / dO stages issued
        for (int i = 0; i < nT; ++i) {
          const int sx = i % XS, sd = i % XDS;
          const int row = (bt0 + i) * BM;
          if (!mbar_wait(&ring_empty[sx], ((i / XS) & 1) ^ 1, ctx)) break;
          mbar_arrive_expect_tx(&ring_full[sx], C::TILE_BYTES);
          for (int r = 0; r < DP / 64; ++r)
            tma_load_3d(sX + sx * C::TILE_BYTES + r * BM * 128, &tm_x, &ring_full[sx], 64 * r, row, SX ? 0 : h);
          ++nx;
          if (!mbar_wait(&w2_empty[sd], ((i / XDS) & 1) ^ 1, ctx)) break;
          mbar_arrive_expect_tx(&w2_full[sd], C::TILE_BYTES);
          for (int r = 0; r < DP / 64; ++r)
            tma_load_3d(sDO + sd * C::TILE_BYTES + r * BM * 128, &tm_do, &w2_full[sd], 64 * r, row, SX ? 0 : h);
          ++nd;
        }
        mbar_wait(in_full, 0, drain);
        for (uint32_t k = 0; k < uint32_t(XS); ++k)
          if (nx > k) mbar_wait(&ring_full[(nx - 1 - k) % XS], ((nx - 1 - k) / XS) & 1, drain);
        for (uint32_t k = 0; k < uint32_t(XDS); ++k)
          if (nd > k) mbar_wait(&w2_full[(nd - 1 - k) % XDS], ((nd - 1 - k) / XDS) & 1, drain);
      }
    } else if (warp == 1) {
      constexpr uint32_t idesc_s = make_idesc_f16(kBF, 128, 128, true, false);   // A MN, B K
      constexpr uint32_t idesc_s2 = make_idesc_f16(kBF, 128, 128, false, false); // A K, B K
      constexpr uint32_t idesc_w = make_idesc_f16(kBF, 128, DP, false, true);    // A tmem, B MN
      const uint64_t w1m = make_sdesc_sw128(smem_u32(sW1), DP * 128, 1024);  // W1c^T, MN-major A
      const uint64_t w2k = make_sdesc_sw128(smem_u32(sW2), 16, 1024);        // W2c, K-major A
      // Z^T(bt) = W1c^T @ X^T (m = 0) or dH^T(bt) = W2c @ dO^T (m = 1); K over the padded
      // DP (zero-filled).
      auto issue_prod = [&](int m, int bt) {
        const int s = m == 0 ? bt % XS : bt % XDS;
        if (elect_one()) {
          const uint64_t bk = make_sdesc_sw128(smem_u32((m == 0 ? sX : sDO) + s * C::TILE_BYTES), 16, 1024);
          const uint32_t d = tmem + (m == 0 ? C::W_TM_ZT : C::W_TM_DHT);
#pragma unroll
          for (int k = 0; k < DP / 16; ++k) {
            const uint64_t bkk = sdesc_add(bk, (k >> 2) * (BM * 128) + (k & 3) * 32);
            if (m == 0)
              mma_ss(d, sdesc_add(w1m, k * 2048), bkk, idesc_s, k > 0 ? 1u : 0u);
            else
              mma_ss(d, sdesc_add(w2k, (k >> 2) * (128 * 128) + (k & 3) * 32), bkk, idesc_s2, k > 0 ? 1u : 0u);
          }
          mma_commit(&p_full[m]);
        }
        __syncwarp();
      };
      // dW2 += H^T(bt) @ dO (m = 0) or dW1^T += dZ^T(bt) @ X (m = 1); K = the tile's 128
      // rows.
      auto issue_dw = [&](int m, int bt) {
        const int s = m == 0 ? bt % XDS : bt % XS;
        if (elect_one()) {
          const uint64_t bm = make_sdesc_sw128(smem_u32((m == 0 ? sDO : sX) + s * C::TILE_BYTES), BM * 128, 1024);
          const uint32_t d = tmem + (m == 0 ? C::W_TM_DW2 : C::W_TM_DW1);
          // H^T / dZ^T: packed over Z^T / dH^T, or (fused) both in the dH^T columns
          const uint32_t a = tmem + (kFused ? C::W_TM_DHT + (m == 0 ? 0 : 16) : (m == 0 ? C::W_TM_ZT : C::W_TM_DHT));
          const uint32_t acc0 = bt > 0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < BM / 16; ++k)
            mma_ts(d, a + packed_col(k), sdesc_add(bm, k * 2048), idesc_w, k > 0 ? 1u : acc0);
          mma_commit(m == 0 ? &w2_empty[s] : &ring_empty[s]);  // last reader of dO_bt / X_bt
        }
        __syncwarp();
      };
      auto wait_x = [&](int bt) { return warp_wait(&ring_full[bt % XS], (bt / XS) & 1, ctx); };
      auto wait_do = [&](int bt) { return warp_wait(&w2_full[bt % XDS], (bt / XDS) & 1, ctx); };
      bool ok = warp_wait(in_full, 0, ctx) && nT > 0 && wait_x(0) && wait_do(0);
      tc_fence_after();
      if (ok) {
        issue_prod(0, 0);
        issue_prod(1, 0);
      }
      for (int bt = 0; bt < nT && ok && kFused; ++bt) {
        // fused schedule: Z^T(bt+1) as soon as every activation warp has read Z^T(bt);
        // dW2(bt), dW1^T(bt) and dH^T(bt+1) once H^T(bt) and dZ^T(bt) are packed in the
        // dH^T columns
        const bool more = bt + 1 < nT;
        if (more) {
          if (!(ok = warp_wait(z_free, bt & 1, ctx) && wait_x(bt + 1))) break;
          tc_fence_after();
          issue_prod(0, bt + 1);
        }
        if (!(ok = warp_wait(&a_full[1], bt & 1, ctx))) break;
        tc_fence_after();
        issue_dw(0, bt);
        issue_dw(1, bt);
        if (more) {  // overwrites H^T(bt), dZ^T(bt) after dW2(bt), dW1^T(bt) read them
          if (!(ok = wait_do(bt + 1))) break;
          tc_fence_after();
          issue_prod(1, bt + 1);
        }
      }
      for (int bt = 0; bt < nT && ok && !kFused; ++bt) {
        const bool more = bt + 1 < nT;
        if (!(ok = warp_wait(&a_full[0], bt & 1, ctx))) break;  // H^T(bt) packed
        tc_fence_after();
        issue_dw(0, bt);
        if (more) {  // overwrites H^T(bt) after dW2(bt) read it
          if (!(ok = wait_x(bt + 1))) break;
          tc_fence_after();
          issue_prod(0, bt + 1);
        }
        if (!(ok = warp_wait(&a_full[1], bt & 1, ctx))) break;  // dZ^T(bt) packed
        tc_fence_after();
        issue_dw(1, bt);
        if (more) {  // overwrites dZ^T(bt) after dW1^T(bt) read it
          if (!(ok = wait_do(bt + 1))) break;
          tc_fence_after();
          issue_prod(1, bt + 1);
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
      // Activation warps: B columns [32j, 32j+32) of Z^T / dH^T.
      const uint32_t zt = tmem + lane_off + C::W_TM_ZT + 32 * j;
      const uint32_t dt = tmem + lane_off + C::W_TM_DHT + 32 * j;
      // dZ-store mode: the dZ^T tile of (head h, E chunk c, B tile t) is 128 x 128 values
      // at tile index (h*nE + c)*nB + t, laid out [e / 64][b / 8][e % 64][b % 8]: a warp's
      // 32 lanes (consecutive e) store 512 contiguous bytes per 8-b group, and each half
      // (64 e) is the no-swizzle MN-major operand layout the dX GEMM reads with one bulk
      // copy. This thread (e = 32q + lane) owns b = 32j..32j+31: 8-b groups 4j..4j+3. The
      // workspace holds at most 2^32 elements, so a 32-bit element offset addresses it.
      const uint32_t dz_off = uint32_t(((size_t(h) * nE + c) * nB + bt0) * (BM * 128)) + (q >> 1) * 8192 +
                              (4 * j) * 512 + ((q & 1) * 32 + lane) * 8;
      auto dz_at = [&](int bt) -> T* { return dzt == nullptr ? nullptr : dzt + (dz_off + uint32_t(bt) * (BM * 128)); };
      bool ok = true;
      for (int bt = 0; bt < nT && ok && kFused; ++bt) {
        // Phase 1 also forms the factors dH is multiplied by (grad_fac), while dH^T(bt)
        // is still being computed, so phase 2 -- on the path to the next dH^T -- is one
        // or two multiplies per element.
        GradFac<T, ACT> fac[32];
        uint32_t hp[16];
        if (!(ok = mbar_wait(&p_full[0], bt & 1, ctx))) break;
        tc_fence_after();
        {
          uint32_t va[16], vb[16];
          tmem_ld16_async(zt, va);
          tmem_ld16_async(zt + 16, vb);
          tmem_wait_ld_dep2(va, vb);
          signal(z_free, false);  // Z^T(bt) is in registers: Z^T(bt+1) may overwrite it
#pragma unroll
          for (int i = 0; i < 8; ++i)
            hp[i] = act_pair_fac<T, ACT>(__uint_as_float(va[2 * i]), __uint_as_float(va[2 * i + 1]), fac[2 * i],
                                         fac[2 * i + 1]);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            hp[8 + i] = act_pair_fac<T, ACT>(__uint_as_float(vb[2 * i]), __uint_as_float(vb[2 * i + 1]), fac[16 + 2 * i],
                                             fac[17 + 2 * i]);
        }
        if (!(ok = mbar_wait(&p_full[1], bt & 1, ctx))) break;
        tc_fence_after();
        {
          // dH^T columns [0,32) of this slice -> registers (one wait); H^T packed over
          // columns [0,16), dZ^T over [16,32)
          // The dZ-store writes follow the signal: the dW products and dH^T(bt+1) need
          // only the TMEM copy, so the global stores stay off their chain.
          uint32_t va[16], vb[16], pd[8], pe[8];
          T* g = dz_at(bt);
          tmem_ld16_async(dt, va);
          tmem_ld16_async(dt + 16, vb);
          tmem_wait_ld_dep2(va, vb);
          tmem_st16(dt, hp);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            pd[i] = grad_pair_fac<T, ACT>(dh_in(va[2 * i]), dh_in(va[2 * i + 1]), fac[2 * i], fac[2 * i + 1]);
          tmem_st8(dt + 16, pd);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            pe[i] = grad_pair_fac<T, ACT>(dh_in(vb[2 * i]), dh_in(vb[2 * i + 1]), fac[16 + 2 * i], fac[17 + 2 * i]);
          tmem_st8(dt + 24, pe);
          signal(&a_full[1], true);
          if (g != nullptr) {
            store_dz(g, pd);
            store_dz(g + 1024, pe);
          }
        }
      }
      for (int bt = 0; bt < nT && ok && !kFused; ++bt) {
        St st[32];
        if (!(ok = mbar_wait(&p_full[0], bt & 1, ctx))) break;
        tc_fence_after();
        phase1(zt, st, true);  // H^T packed over Z^T
        signal(&a_full[0], true);
        if (!(ok = mbar_wait(&p_full[1], bt & 1, ctx))) break;
        tc_fence_after();
        phase2(dt, dt, st, dz_at(bt), &a_full[1]);  // dZ^T packed over dH^T
      }
      if (ok && (ok = mbar_wait(acc_full, 0, ctx))) {
        tc_fence_after();
        const int e = c * 128 + q * 32 + lane;
        constexpr int OW = DP / 4;  // accumulator columns per warp
        const int col0 = j * OW;
        // dW2 = H^T dO_h with dO_h = dO / H for a shared input (dW1 already carries 1/H
        // through dZ)
        auto scale_dw2 = [&](uint32_t (&v)[16]) {
          if constexpr (SX) {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * inv_h);
          }
        };
        if (part != nullptr) {
          // fp32 sums of this B range: part[split][0] is dW1 laid out (H, D, E),
          // part[split][1] is dW2 laid out (H, E, D); with several splits
          // fmlp_dw_reduce_kernel adds them, with one it is the fp32 output itself.
          const size_t n = size_t(H) * D * E;
          float* p1 = part + size_t(split) * 2 * n;
          float* p2 = p1 + n;
#pragma unroll
          for (int u = 0; u < OW / 16; ++u) {
            uint32_t v[16];
            tmem_ld16_sync(tmem + lane_off + C::W_TM_DW1 + col0 + 16 * u, v);
            if (e < E) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int d = col0 + 16 * u + i;
                if (d < D) p1[(size_t(h) * D + d) * E + e] = __uint_as_float(v[i]);
              }
            }
          }
#pragma unroll
          for (int u = 0; u < OW / 16; ++u) {
            uint32_t v[16];
            tmem_ld16_sync(tmem + lane_off + C::W_TM_DW2 + col0 + 16 * u, v);
            scale_dw2(v);
            const int cc = col0 + 16 * u;
            if (e < E && cc < D) {  // D % 16 == 0: all 16 columns are inside
              float4* dst = reinterpret_cast<float4*>(p2 + (size_t(h) * E + e) * D + cc);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                dst[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                     __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
            }
          }
        } else {
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
            scale_dw2(v);
            plain_pack<T, 8>(v, p);
            const int cc = col0 + 16 * u;
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
        // Same order as the MMA warp consumes them: W1c(c), W2c(c), W1c(c+1), ...
        uint32_t n1 = 0, n2 = 0;
        auto load_w1 = [&](int c) -> bool {
          const int s = c % C::WS1;
          if (!mbar_wait(&ring_empty[s], ((c / C::WS1) & 1) ^ 1, ctx)) return false;
          mbar_arrive_expect_tx(&ring_full[s], C::W1C_BYTES);
          for (int r = 0; r < 2; ++r)
            tma_load_3d(sW1 + s * C::W1C_BYTES + r * DP * 128, &tm_w1, &ring_full[s], (c % nE) * 128 + 64 * r, 0, SX ? c / nE : h);
          ++n1;
          return true;
        };
        auto load_w2 = [&](int c) -> bool {
          const int s = c % C::WS2;
          if (!mbar_wait(&w2_empty[s], ((c / C::WS2) & 1) ^ 1, ctx)) return false;
          mbar_arrive_expect_tx(&w2_full[s], C::W2C_BYTES);
          for (int r = 0; r < DP / 64; ++r)
            tma_load_3d(sW2 + s * C::W2C_BYTES + r * 128 * 128, &tm_w2, &w2_full[s], 64 * r, (c % nE) * 128, SX ? c / nE : h);
          ++n2;
          return true;
        };
        for (int c = 0; c < nEv; ++c)
          if (!load_w1(c) || !load_w2(c)) break;
        mbar_wait(in_full, 0, drain);
        for (uint32_t s = 0; s < C::WS1; ++s)
          if (n1 > s) mbar_wait(&ring_full[s], ((n1 - 1 - s) / C::WS1) & 1, drain);
        for (uint32_t s = 0; s < C::WS2; ++s)
          if (n2 > s) mbar_wait(&w2_full[s], ((n2 - 1 - s) / C::WS2) & 1, drain);
      }
    } else if (warp == 1) {
      constexpr uint32_t idesc_z = make_idesc_f16(kBF, 128, 128, false, true);   // A K, B MN
      constexpr uint32_t idesc_h = make_idesc_f16(kBF, 128, 128, false, false);  // A K, B K
      constexpr uint32_t idesc_x = make_idesc_f16(kBF, 128, DP, false, false);   // A tmem, B K
      const uint64_t xk = make_sdesc_sw128(smem_u32(sX), 16, 1024);
      const uint64_t dk = make_sdesc_sw128(smem_u32(sDO), 16, 1024);
      auto issue_z = [&](int c) {  // Z(c) = X_b @ W1c into buffer c%2
        const int s = c % C::WS1;
        if (elect_one()) {
          const uint64_t w1m = make_sdesc_sw128(smem_u32(sW1 + s * C::W1C_BYTES), DP * 128, 1024);
#pragma unroll
          for (int k = 0; k < DP / 16; ++k)
            mma_ss(tmem + C::X_TM_Z + (c & 1) * 128, sdesc_add(xk, (k >> 2) * (BM * 128) + (k & 3) * 32),
                   sdesc_add(w1m, k * 2048), idesc_z, k > 0 ? 1u : 0u);
          mma_commit(&p_full[(c & 1) ? 2 : 0]);
        }
        __syncwarp();
      };
      auto issue_dh = [&](int c) {  // dH(c) = dO_b @ W2c^T
        const int s = c % C::WS2;
        if (elect_one()) {
          const uint64_t w2k = make_sdesc_sw128(smem_u32(sW2 + s * C::W2C_BYTES), 16, 1024);
#pragma unroll
          for (int k = 0; k < DP / 16; ++k)
            mma_ss(tmem + C::X_TM_DH, sdesc_add(dk, (k >> 2) * (BM * 128) + (k & 3) * 32),
                   sdesc_add(w2k, (k >> 2) * (128 * 128) + (k & 3) * 32), idesc_h, k > 0 ? 1u : 0u);
          mma_commit(&p_full[1]);
          mma_commit(&w2_empty[s]);  // dH(c) is the W2c stage's only reader
        }
        __syncwarp();
      };
      auto wait_w1 = [&](int c) { return warp_wait(&ring_full[c % C::WS1], (c / C::WS1) & 1, ctx); };
      auto wait_w2 = [&](int c) { return warp_wait(&w2_full[c % C::WS2], (c / C::WS2) & 1, ctx); };
      bool ok = warp_wait(in_full, 0, ctx) && nEv > 0 && wait_w1(0) && wait_w2(0);
      tc_fence_after();
      if (ok) {
        issue_z(0);
        issue_dh(0);
        if (nEv > 1 && (ok = wait_w1(1))) {
          tc_fence_after();
          issue_z(1);
        }
      }
      for (int c = 0; c < nEv && ok; ++c) {
        // Phase 2(c) has read dH(c) and packed dZ(c) over the Z(c) buffer.
        if (!(ok = warp_wait(&a_full[1], c & 1, ctx))) break;
        tc_fence_after();
        if (c + 1 < nEv) {
          if (!(ok = wait_w2(c + 1))) break;
          tc_fence_after();
          issue_dh(c + 1);
        }
        if (elect_one()) {
          const int s = c % C::WS1;
          const uint64_t w1k = make_sdesc_sw128(smem_u32(sW1 + s * C::W1C_BYTES), 16, 1024);
          const uint32_t dz = tmem + C::X_TM_Z + (c & 1) * 128;
          const uint32_t acc0 = c > 0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < 8; ++k)  // K = the 128 E columns of the chunk (2 regions of 64)
            mma_ts(tmem + C::X_TM_DX, dz + packed_col(k), sdesc_add(w1k, (k >> 2) * (DP * 128) + (k & 3) * 32),
                   idesc_x, k > 0 ? 1u : acc0);
          mma_commit(&ring_empty[s]);  // dX(c) is the W1c stage's last reader
        }
        __syncwarp();
        if (c + 2 < nEv) {  // overwrites dZ(c) after dX(c) read it
          if (!(ok = wait_w1(c + 2))) break;
          tc_fence_after();
          issue_z(c + 2);
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
      // Per E chunk: E columns [32j, 32j+32) of Z (buffer c%2) and dH.
      const uint32_t da = tmem + lane_off + C::X_TM_DH + 32 * j;
      bool ok = true;
      for (int c = 0; c < nEv && ok; ++c) {
        St st[32];
        const uint32_t zc = tmem + lane_off + C::X_TM_Z + (c & 1) * 128 + 32 * j;
        if (!(ok = mbar_wait(&p_full[(c & 1) ? 2 : 0], (c >> 1) & 1, ctx))) break;
        tc_fence_after();
        phase1(zc, st, false);  // derivative state only
        if (!(ok = mbar_wait(&p_full[1], c & 1, ctx))) break;
        tc_fence_after();
        phase2(da, zc, st, nullptr, &a_full[1]);  // dZ packed over this warp's Z columns
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
          plain_pack<T, 8>(v, p);
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

// dW1 / dW2 of split dW programs: out[i] = sum over s = 0..S-1, in that order, of
// part[s][which][i] with which = blockIdx.y (0: dW1 (H,D,E), 1: dW2 (H,E,D)), rounded into
// dW1 / dW2, or stored unrounded into out_f32[which][i] when out_f32 is set; four elements
// per step (H*D*E is a multiple of 4). HBM-bound: 4*S bytes read, 2 (or 4) written per
// element.
template <typename T>
__global__ void __launch_bounds__(256)
    fmlp_dw_reduce_kernel(const float* __restrict__ part, T* __restrict__ dW1, T* __restrict__ dW2,
                          float* __restrict__ out_f32, long long n4, int splits) {
  const size_t n = size_t(n4) * 4;
  const float4* src = reinterpret_cast<const float4*>(part + blockIdx.y * n);
  const size_t stride4 = 2 * size_t(n4);  // float4s between consecutive splits
  uint2* dst = reinterpret_cast<uint2*>(blockIdx.y ? dW2 : dW1);
  float4* dstf = out_f32 ? reinterpret_cast<float4*>(out_f32 + blockIdx.y * n) : nullptr;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    float4 acc = __ldcs(src + i);
    for (int s = 1; s < splits; ++s) {
      const float4 v = __ldcs(src + s * stride4 + i);
      acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
    }
    if (dstf)
      dstf[i] = acc;
    else
      dst[i] = make_uint2(Pack<T>::pack(acc.x, acc.y), Pack<T>::pack(acc.z, acc.w));
  }
}

template <int DP, typename T, int ACT, bool SX>
static cudaError_t launch_bwd_sx(const BwdLaunch& a) {
  using C = BwdCfg<DP>;
  auto kern = fmlp_bwd_kernel<DP, T, ACT, SX>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int nB = (a.B + kRows - 1) / kRows;
  const int nE = (a.E + C::ET - 1) / C::ET;
  const int splits = a.splits < 1 ? 1 : a.splits;
  if (splits > 1 && (a.part == nullptr || splits > nB)) return cudaErrorInvalidValue;
  // dZ-store mode: dW programs only; their dZ^T feeds fmlp_dx_gemm_kernel
  const bool dz = a.dzt != nullptr;
  const long long grid = (long long)a.H * nE * splits + (dz ? 0LL : (SX ? 1LL : (long long)a.H) * nB);
  if (grid <= 0 || grid > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  // the dW programs' fp32 target: the split partials, or the fp32 output itself
  float* kpart = splits > 1 ? a.part : a.dw_f32;
  kern<<<unsigned(grid), C::NUM_THREADS, C::SMEM, a.stream>>>(
      a.tm_x, a.tm_do, a.tm_w1, a.tm_w2, reinterpret_cast<T*>(a.dx), reinterpret_cast<T*>(a.dw1),
      reinterpret_cast<T*>(a.dw2), kpart, reinterpret_cast<T*>(a.dzt), splits, a.H, a.B, a.D, a.E, a.status);
  cudaError_t le = cudaGetLastError();
  if (le == cudaSuccess && dz) le = launch_dx_gemm(a);
  if (le != cudaSuccess || splits == 1) return le;
  return launch_dw_reduce(a);
}

template <typename T>
static cudaError_t launch_dw_reduce_t(const BwdLaunch& a) {
  const long long n4 = (long long)a.H * a.D * a.E / 4;  // E % 8 == 0
  long long blocks = (n4 + 255) / 256;
  const long long cap = (long long)a.sm_count * 4;
  if (blocks > cap) blocks = cap;
  fmlp_dw_reduce_kernel<T><<<dim3(unsigned(blocks), 2), 256, 0, a.stream>>>(
      a.part, reinterpret_cast<T*>(a.dw1), reinterpret_cast<T*>(a.dw2), a.dw_f32, n4, a.splits);
  return cudaGetLastError();
}

cudaError_t launch_dw_reduce(const BwdLaunch& a) {
  return a.bf16 ? launch_dw_reduce_t<__nv_bfloat16>(a) : launch_dw_reduce_t<__half>(a);
}

template <int DP, typename T, int ACT>
static cudaError_t launch_bwd_t(const BwdLaunch& a) {
  return a.shared_x ? launch_bwd_sx<DP, T, ACT, true>(a) : launch_bwd_sx<DP, T, ACT, false>(a);
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

int bwd_dw_splits(int H, int B, int D, int E, int sm_count) {
  if (D > 128 || H <= 0 || B <= 0 || E <= 0 || sm_count <= 0) return 1;
  const long long nB = (B + kRows - 1) / kRows, nE = (E + kBwdEt - 1) / kBwdEt;
  // Work in units of one 128x128x128 product: a dW program does 4 per B tile, a dX
  // program 3 per E chunk. Split until one dW program is at most 0.8 of an SM's share of
  // the launch, keeping at least 2 B tiles per split and at most 8 splits.
  const long long work = 7LL * H * nE * nB;
  const long long max_s = nB / 2 < 8 ? nB / 2 : 8;
  for (long long s = 1; s <= max_s; ++s) {
    const long long lw = 4 * ((nB + s - 1) / s);
    if (5 * lw * sm_count <= 4 * work) return int(s);
  }
  return max_s < 1 ? 1 : int(max_s);
}

size_t bwd_workspace_bytes(int H, int B, int D, int E, int sm_count) {
  const int s = bwd_dw_splits(H, B, D, E, sm_count);
  return s > 1 ? size_t(2) * s * size_t(H) * D * E * sizeof(float) : 0;
}

size_t bwd_dz_bytes(int H, int B, int D, int E, int sm_count, int elem_bytes) {
  if (D > (elem_bytes == 4 ? 128 : 256) || H <= 0 || B <= 0 || E <= 0 || sm_count <= 0) return 0;
  // dZ^T tiles; for 128 < D <= 256 (16-bit) the H^T tiles of the D-half-1 GEMM follow
  const size_t regions = (D > 128 && elem_bytes == 2) ? 2 : 1;
  const size_t bytes = dz_tile_elems(H, B, E) * elem_bytes * regions;
  return bytes <= kDzCapBytes ? bytes : 0;
}

int bwd_dz_splits(int H, int B, int D, int E, int sm_count) {
  if (D > 256 || H <= 0 || B <= 0 || E <= 0 || sm_count <= 0) return 1;
  const long long nB = (B + kRows - 1) / kRows, nE = (E + kBwdEt - 1) / kBwdEt;
  // The launch holds dW programs only, all of the same length, so it runs in whole waves
  // of sm_count programs: pick S (1..16, at least 2 B tiles per split) minimising
  // waves * (tiles per program + 2 for a program's fill and drain) * tile time + the fp32
  // reduce of the partials (S > 1). For 128 < D <= 256 (fmlp_bwd256.cu) the launch holds
  // the D-half-0 programs, each forming Z^T and dH^T over all of D, and the D-half-1 GEMM
  // (fmlp_dwgemm256.cu) has as many programs, HBM-bound on the 64 KB of stored dZ^T and
  // H^T tiles per 128-row tile.
  const int dp = D <= 64 ? 64 : (D <= 128 ? 128 : 256);
  const double tile_flop = dp == 256 ? 4.0 * 128 * 128 * 256 + 4.0 * 128 * 128 * 128  // Z^T, dH^T, two half dW
                                     : 8.0 * 128 * 128 * dp;                          // 4 products of 128x128xDP
  const double tile_s = tile_flop / (1.2e15 / sm_count) + (dp == 256 ? 65536.0 / (6.0e12 / sm_count) : 0.0);
  const double hde = double(H) * D * E;
  const long long max_s = nB / 2 < 16 ? nB / 2 : 16;
  int best = 1;
  double best_t = 0;
  for (long long s = 1; s <= (max_s < 1 ? 1 : max_s); ++s) {
    const long long progs = (long long)H * nE * s;
    const long long waves = (progs + sm_count - 1) / sm_count;
    double t = double(waves) * double((nB + s - 1) / s + 2) * tile_s;
    if (s > 1) t += (8.0 * s + 4.0) * hde / 6.0e12 + 5e-6;
    if (s == 1 || t < best_t) best = int(s), best_t = t;
  }
  return best;
}

size_t bwd_dz_workspace_bytes(int H, int B, int D, int E, int sm_count, int elem_bytes) {
  const size_t dz = bwd_dz_bytes(H, B, D, E, sm_count, elem_bytes);
  if (dz == 0) return 0;
  const int s = elem_bytes == 4 ? bwd_dz_splits_tf32(H, B, D, E, sm_count) : bwd_dz_splits(H, B, D, E, sm_count);
  return dz + (s > 1 ? size_t(2) * s * size_t(H) * D * E * sizeof(float) : 0);
}

int bwd_dz_group_heads(int H, int B, int D, int E, int sm_count, int elem_bytes, size_t workspace_bytes) {
  if (H <= 0) return 0;
  const size_t one = bwd_dz_bytes(1, B, D, E, sm_count, elem_bytes);
  if (one == 0) return 0;  // the mode does not apply, or one head alone exceeds the cap
  long long g = H;
  if ((long long)(kDzCapBytes / one) < g) g = (long long)(kDzCapBytes / one);
  if ((long long)(workspace_bytes / one) < g) g = (long long)(workspace_bytes / one);
  const long long floor_g = H < kDzMinGroupHeads ? H : kDzMinGroupHeads;
  for (; g >= floor_g && g >= 1; --g) {
    if (bwd_dz_workspace_bytes(int(g), B, D, E, sm_count, elem_bytes) > workspace_bytes) continue;
    // as many groups as this size needs, with the heads spread evenly over them
    const long long n = (H + g - 1) / g, even = (H + n - 1) / n;
    if (even < g && bwd_dz_workspace_bytes(int(even), B, D, E, sm_count, elem_bytes) <= workspace_bytes)
      return int(even);
    return int(g);
  }
  return 0;
}

int bwd_smem_bytes(int dp) {
  switch (dp) {
    case 64: return BwdCfg<64>::SMEM;
    case 128: return BwdCfg<128>::SMEM;
    case 256: return bwd256_smem_bytes();
  }
  return -1;
}

cudaError_t launch_bwd(const BwdLaunch& a) {
  switch (a.dp) {
    case 64: return launch_bwd_dt<64>(a);
    case 128: return launch_bwd_dt<128>(a);
    case 256: return a.shared_x ? cudaErrorNotSupported : launch_bwd256(a);
  }
  return cudaErrorNotSupported;
}

}  // namespace fmlp
