// dX programs of the backward when the dW programs have stored dZ: a GEMM over E.
//
// In the reference's unified backward (flashmlp.py:341-421) the dX programs
// (`_flashmlp_bwd_dx`, flashmlp.py:165-244) recompute Z = X@W1 and dH = dO@W2^T for every
// E chunk to form dZ = dH * act'(Z), round it to the input dtype (flashmlp.py:232-235) and
// accumulate dX += dZ @ W1^T. The dW programs compute the same dZ (transposed, per E
// chunk and B tile). In the dZ-store mode of fmlp_bwd the dW programs also write their
// rounded dZ^T tiles to the caller's workspace, and the dX programs become this kernel:
//   dX[h, b, :] = sum over e of dZ^T[h, e, b] * W1[h, :, e]
// with the same 16-bit dZ values and fp32 accumulation, i.e. two of the three products of
// a dX program and the activation are not recomputed. The kernel reads 2*E bytes of dZ
// per output row: HBM-bound (E FLOP per byte, below the B200 ridge of ~250).
// With a shared input (X, dO, dX are (B, D) for every head) one program sums over
// (head, e): dZ already carries the head mean's 1/H.
//
// One CTA per (B tile of 128 rows, head); warp 0 issues the loads, warp 1 the MMAs,
// warps 2-5 read the fp32 accumulator out of TMEM and store dX. K steps of 64 e:
//   dX(b, d) += dZ(b, e) [smem, MN-major, no swizzle: 8 x 8 core matrices, 8 b by 8 e]
//             @ W1^T(e, d) [smem, K-major: W1 rows d, 64 e per 128-byte row, TMA]
//   SS M=128(b) N=DP K=16, four per stage.
// The dW programs store each dZ^T tile (128 e x 128 b of one head, E chunk and B tile) as
// [e / 64][b / 8][e % 64][b % 8], so the 64 e of a K step for all 128 b are 16 KB of
// contiguous memory already in that operand layout: one untiled bulk copy per stage.
// Three to four stages of 24-32 KB (two of 48 KB for D = 256, N = 256) keep ~100 KB of
// loads in flight per CTA; two CTAs fit on an SM (shared memory and TMEM), so one CTA's
// epilogue overlaps the other's loads.
#include "fmlp_act.cuh"
#include "fmlp_kernels.h"
#include "fmlp_ptx.cuh"

namespace fmlp {

template <int DP>
struct DxGemmCfg {
  static constexpr int BM = kRows;
  static constexpr int KT = 64;                    // e per stage (one 128-byte swizzle row)
  static constexpr int A_BYTES = KT * BM * 2;      // dZ^T: 64 e x 128 b, [b / 8][e][b % 8]
  static constexpr int TILE_ELEMS = BM * 128;      // one stored dZ^T tile (128 e x 128 b)
  static constexpr int B_BYTES = DP * KT * 2;      // W1: DP d rows x 64 e
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int NST = DP == 64 ? 4 : (DP == 128 ? 3 : 2);
  static constexpr int OFF_BAR = NST * STAGE;
  static constexpr int OFF_MISC = OFF_BAR + (2 * NST + 2) * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;  // + alignment slack
  static constexpr int TMEM_COLS = DP;               // fp32 accumulator, DP columns
  static constexpr int NUM_THREADS = 192;
  static_assert(2 * (SMEM + 1024) <= 233472, "two CTAs per SM");
};

template <int DP, typename T, bool SX>
__global__ void __launch_bounds__(192)
    fmlp_dx_gemm_kernel(const T* __restrict__ dzt, const __grid_constant__ CUtensorMap tm_w1,
                        T* __restrict__ dX, int H, int B, int D, int E, uint32_t* status) {
  using C = DxGemmCfg<DP>;
  constexpr int BM = C::BM;
  constexpr bool kBF = Pack<T>::kBF16;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty = full + C::NST;
  uint64_t* acc_full = empty + C::NST;
  uint64_t* done_bar = acc_full + 1;
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_flag = misc + 1;
  const WaitCtx ctx{abort_flag, status};
  const WaitCtx drain{misc + 2, status};  // misc[2] stays 0: drains never abort early

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bt = blockIdx.x;
  const int h = SX ? 0 : int(blockIdx.y);
  const int nKh = (E + C::KT - 1) / C::KT;  // K steps per head
  const int nK = SX ? H * nKh : nKh;
  const int nB = (B + BM - 1) / BM;
  const int nE = (E + 127) / 128;  // 128-wide E chunks of the stored tiles

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
    tma_prefetch_desc(&tm_w1);
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
      uint32_t n = 0;  // stages issued
      for (int k = 0; k < nK; ++k) {
        const int s = k % C::NST;
        const int hk = SX ? k / nKh : h;
        const int kh = SX ? k % nKh : k;  // K step within the head: E chunk kh / 2, half kh % 2
        if (!mbar_wait(&empty[s], ((k / C::NST) & 1) ^ 1, ctx)) break;
        uint8_t* st = smem + s * C::STAGE;
        mbar_arrive_expect_tx(&full[s], C::STAGE);
        const size_t tile = (size_t(hk) * nE + (kh >> 1)) * nB + bt;
        bulk_load(st, dzt + tile * C::TILE_ELEMS + (kh & 1) * (C::TILE_ELEMS / 2), C::A_BYTES, &full[s]);
        tma_load_3d(st + C::A_BYTES, &tm_w1, &full[s], kh * C::KT, 0, hk);
        ++n;
      }
      // no bulk copy may still be writing shared memory when the CTA exits
      for (uint32_t k = 0; k < uint32_t(C::NST); ++k)
        if (n > k) mbar_wait(&full[(n - 1 - k) % C::NST], ((n - 1 - k) / C::NST) & 1, drain);
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = make_idesc_f16(kBF, 128, DP, true, false);  // A MN, B K
    bool ok = true;
    for (int k = 0; k < nK && ok; ++k) {
      const int s = k % C::NST;
      if (!(ok = warp_wait(&full[s], (k / C::NST) & 1, ctx))) break;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t st = smem_u32(smem + s * C::STAGE);
        // dZ stage [b / 8][e][b % 8]: core matrices 128 B apart along K (8 e), 1 KB
        // apart along M (8 b); a K step of 16 e is +256 B
        const uint64_t ad = make_sdesc_noswz(st, 128, C::KT * 16);
        const uint64_t bd = make_sdesc_sw128(st + C::A_BYTES, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < C::KT / 16; ++kk)
          mma_ss(tmem, sdesc_add(ad, kk * 256), sdesc_add(bd, kk * 32), idesc, (k > 0 || kk > 0) ? 1u : 0u);
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
    // warps 2..5: TMEM lane quadrant warp % 4 holds rows [32q, 32q+32) of the tile
    const int q = warp & 3;
    if (mbar_wait(acc_full, 0, ctx)) {
      tc_fence_after();
      const int row = bt * BM + q * 32 + lane;
      T* xrow = dX + (size_t(h) * B + row) * D;
      const uint32_t ta = tmem + (uint32_t(q * 32) << 16);
#pragma unroll
      for (int u = 0; u < DP / 16; ++u) {
        uint32_t v[16], p[8];
        tmem_ld16_sync(ta + 16 * u, v);
        plain_pack<T, 8>(v, p);
        const int cc = 16 * u;
        if (row < B && cc < D) {  // D % 16 == 0
          uint4* dst = reinterpret_cast<uint4*>(xrow + cc);
          dst[0] = make_uint4(p[0], p[1], p[2], p[3]);
          dst[1] = make_uint4(p[4], p[5], p[6], p[7]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

template <int DP, typename T, bool SX>
static cudaError_t launch_dx_gemm_t(const BwdLaunch& a) {
  using C = DxGemmCfg<DP>;
  auto kern = fmlp_dx_gemm_kernel<DP, T, SX>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const long long nB = (a.B + kRows - 1) / kRows;
  const long long nH = SX ? 1 : a.H;
  if (nB <= 0 || nB > 0x7FFFFFFFLL || nH > 65535) return cudaErrorInvalidValue;
  kern<<<dim3(unsigned(nB), unsigned(nH)), C::NUM_THREADS, C::SMEM, a.stream>>>(
      reinterpret_cast<const T*>(a.dzt), a.tm_w1, reinterpret_cast<T*>(a.dx), a.H, a.B, a.D, a.E, a.status);
  return cudaGetLastError();
}

template <int DP, typename T>
static cudaError_t launch_dx_gemm_dt(const BwdLaunch& a) {
  return a.shared_x ? launch_dx_gemm_t<DP, T, true>(a) : launch_dx_gemm_t<DP, T, false>(a);
}

cudaError_t launch_dx_gemm(const BwdLaunch& a) {
  switch (a.dp) {
    case 64: return a.bf16 ? launch_dx_gemm_dt<64, __nv_bfloat16>(a) : launch_dx_gemm_dt<64, __half>(a);
    case 128: return a.bf16 ? launch_dx_gemm_dt<128, __nv_bfloat16>(a) : launch_dx_gemm_dt<128, __half>(a);
    case 256: return a.shared_x ? cudaErrorNotSupported
                                : (a.bf16 ? launch_dx_gemm_t<256, __nv_bfloat16, false>(a) : launch_dx_gemm_t<256, __half, false>(a));
  }
  return cudaErrorNotSupported;
}

}  // namespace fmlp
