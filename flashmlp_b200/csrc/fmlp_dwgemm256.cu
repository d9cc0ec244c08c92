// D half 1 of the dW programs for 128 < D <= 256 in the dZ-store mode: a GEMM over B.
//
// In the reference's unified backward the dW programs (`_flashmlp_bwd_dw1w2`,
// flashmlp.py:247-338) recompute Z = X@W1, H = act(Z), dH = dO@W2^T and dZ = dH * act'(Z)
// for every B tile, round H and dZ to the input dtype and accumulate dW1 += X^T dZ,
// dW2 += H^T dO in fp32. For D = 256 fmlp_bwd256.cu runs one such program per (head,
// 128-wide E chunk, D half, B range); each half forms Z^T and dH^T over all of D, a 128 x
// 64 x 256 product each per 64-row tile, for 128 x 64 x 128 products of its own. In the
// dZ-store mode the D-half-0 programs also store the rounded dZ^T and H^T tiles, and the
// D-half-1 outputs come from them without the recompute:
//   dW1^T[e, d] += sum over b of dZ^T[e, b] X[b, d]       d in [128, D)
//   dW2[e, d]   += sum over b of H^T[e, b] dO[b, d]
// The operands are the same 16-bit values, taken in the same 64-row K steps in the same
// order into the same fp32 accumulators as in the half-1 program this replaces, so every
// sum has the same bits. Per 64-row step the kernel reads 32 KB of stored tiles (HBM) and
// 32 KB of X / dO (shared by the E chunks of one B range through L2) for 2 x 128 x 128 x 64
// multiply-adds: HBM-bound (2H*B*E*2 bytes per launch).
//
// One CTA per (head, B range, E chunk), E chunk fastest, so the chunks that read the same X
// and dO rows run together. Warp 0 issues the loads, warp 1 the MMAs, warps 2-5 store the
// accumulators. Per 64-row step (one stage of 64 KB, three stages):
//   dZ^T: 16 untiled bulk copies of 1 KB from the stored layout [e/64][b/8][e%64][b%8]
//         into [b/8][e][b%8] (K-major, no swizzle: core matrices 128 B apart along e,
//         2 KB apart along b);
//   H^T:  one 16 KB bulk copy (stored as [b/8][e][b%8] already);
//   X, dO columns [128, 256): two 64 x 64 TMA boxes each (128-byte swizzle, MN-major).
//   dW1^T += dZ^T @ X[:, 128:]   SS M=128(e) N=128(d) K=16, four per step
//   dW2   += H^T  @ dO[:, 128:]  SS M=128(e) N=128(d) K=16, four per step
// TMEM: dW1^T [0,128) dW2 [128,256).
#include "fmlp_act.cuh"
#include "fmlp_kernels.h"
#include "fmlp_ptx.cuh"

namespace fmlp {

struct DwGemmCfg {
  static constexpr int BT = 64;                        // B rows per K step (a stored half tile)
  static constexpr int A_BYTES = 128 * BT * 2;         // 128 e x 64 b, [b / 8][e][b % 8]
  static constexpr int B_BYTES = BT * 128 * 2;         // 64 b rows x 128 d, two 64-d regions
  static constexpr int REGION = BT * 128;              // one 64 x 64 box, 128-byte rows
  static constexpr int STAGE = 2 * A_BYTES + 2 * B_BYTES;  // dZ^T, H^T, X, dO
  static constexpr int NST = 3;
  static constexpr int TILE_ELEMS = kRows * 128;       // one stored 128 x 128 tile
  static constexpr int OFF_BAR = NST * STAGE;
  static constexpr int OFF_MISC = OFF_BAR + (2 * NST + 2) * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;    // + alignment slack
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr int TMEM_COLS = 256;
  static constexpr int TM_DW1 = 0, TM_DW2 = 128;
  static constexpr int NUM_THREADS = 192;
};

template <typename T>
__global__ void __launch_bounds__(192, 1)
    fmlp_dw_gemm256_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_do,
                           const T* __restrict__ dzt, const T* __restrict__ hts, T* __restrict__ dW1,
                           T* __restrict__ dW2, float* __restrict__ dwf, float* __restrict__ part, int splits,
                           int H, int B, int D, int E, uint32_t* status) {
  using C = DwGemmCfg;
  constexpr bool kBF = Pack<T>::kBF16;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
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
  const int nEw = (E + 127) / 128;
  const int nB128 = (B + kRows - 1) / kRows;
  const int h = blockIdx.x / (splits * nEw);
  const int r = blockIdx.x % (splits * nEw);
  const int split = r / nEw;
  const int c = r % nEw;
  // the 64-row steps of this B range: those the D-half-0 program of the same range stored
  const int bt0 = int((long long)split * nB128 / splits);
  const int bt1 = int((long long)(split + 1) * nB128 / splits);
  const int t0 = 2 * bt0;
  const int nT64 = (B + C::BT - 1) / C::BT;
  const int nT = (2 * bt1 < nT64 ? 2 * bt1 : nT64) - t0;
  const size_t tiles0 = (size_t(h) * nEw + c) * nB128 + bt0;  // first stored tile of the range

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
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_do);
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
      for (int t = 0; t < nT; ++t) {
        const int s = t % C::NST;
        if (!mbar_wait(&empty[s], ((t / C::NST) & 1) ^ 1, ctx)) break;
        uint8_t* st = smem + s * C::STAGE;
        mbar_arrive_expect_tx(&full[s], C::STAGE);
        const size_t tile = (tiles0 + size_t(t >> 1)) * C::TILE_ELEMS;
        const int u = t & 1;  // half of the 128-row tile: b / 8 in [8u, 8u + 8)
        for (int kb = 0; kb < 8; ++kb)
          for (int eh = 0; eh < 2; ++eh)
            bulk_load(st + kb * 2048 + eh * 1024, dzt + tile + eh * 8192 + (8 * u + kb) * 512, 1024, &full[s]);
        bulk_load(st + C::A_BYTES, hts + tile + u * 8192, C::A_BYTES, &full[s]);
        const int row = (t0 + t) * C::BT;
        for (int rg = 0; rg < 2; ++rg) {
          tma_load_3d(st + 2 * C::A_BYTES + rg * C::REGION, &tm_x, &full[s], 128 + 64 * rg, row, h);
          tma_load_3d(st + 2 * C::A_BYTES + C::B_BYTES + rg * C::REGION, &tm_do, &full[s], 128 + 64 * rg, row, h);
        }
        ++n;
      }
      // no copy may still be writing shared memory when the CTA exits
      for (uint32_t k = 0; k < uint32_t(C::NST); ++k)
        if (n > k) mbar_wait(&full[(n - 1 - k) % C::NST], ((n - 1 - k) / C::NST) & 1, drain);
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = make_idesc_f16(kBF, 128, 128, false, true);  // A K-major, B MN-major
    bool ok = true;
    for (int t = 0; t < nT && ok; ++t) {
      const int s = t % C::NST;
      if (!(ok = warp_wait(&full[s], (t / C::NST) & 1, ctx))) break;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t st = smem_u32(smem + s * C::STAGE);
        // A [b / 8][e][b % 8]: core matrices (8 e x 8 b) 128 B apart along M (e), 2 KB
        // apart along K (b); a K step of 16 b is +4 KB
        const uint64_t a1 = make_sdesc_noswz(st, 2048, 128);
        const uint64_t a2 = make_sdesc_noswz(st + C::A_BYTES, 2048, 128);
        // B: rows b of 64 d (128 B, swizzled), the second 64 d one region further
        const uint64_t b1 = make_sdesc_sw128(st + 2 * C::A_BYTES, C::REGION, 1024);
        const uint64_t b2 = make_sdesc_sw128(st + 2 * C::A_BYTES + C::B_BYTES, C::REGION, 1024);
        const uint32_t acc0 = t > 0 ? 1u : 0u;
#pragma unroll
        for (int k = 0; k < C::BT / 16; ++k)
          mma_ss(tmem + C::TM_DW2, sdesc_add(a2, k * 4096), sdesc_add(b2, k * 2048), idesc, k > 0 ? 1u : acc0);
#pragma unroll
        for (int k = 0; k < C::BT / 16; ++k)
          mma_ss(tmem + C::TM_DW1, sdesc_add(a1, k * 4096), sdesc_add(b1, k * 2048), idesc, k > 0 ? 1u : acc0);
        mma_commit(&empty[s]);
      }
      __syncwarp();
    }
    if (ok && nT > 0) {
      if (elect_one()) mma_commit(acc_full);
      __syncwarp();
    }
    if (elect_one()) mma_commit(done_bar);
    __syncwarp();
    warp_wait(done_bar, 0, drain);
  } else {
    // warps 2..5: TMEM lane quadrant warp % 4 holds E rows [32q, 32q+32) of the chunk
    const int q = warp & 3;
    if (nT > 0 && mbar_wait(acc_full, 0, ctx)) {
      tc_fence_after();
      const int e = c * 128 + q * 32 + lane;
      const uint32_t ta = tmem + (uint32_t(q * 32) << 16);
      // fp32 sums: this B range's partials (fmlp_dw_reduce_kernel adds the ranges in
      // order), or the unrounded fp32 output; else the rounded outputs
      float* fout = part != nullptr ? part + size_t(split) * 2 * (size_t(H) * D * E) : dwf;
      if (fout != nullptr) {
        float* f1 = fout;                         // dW1 laid out (H, D, E)
        float* f2 = fout + size_t(H) * D * E;     // dW2 laid out (H, E, D)
#pragma unroll 1
        for (int u = 0; u < 8; ++u) {
          uint32_t v[16];
          tmem_ld16_sync(ta + C::TM_DW1 + 16 * u, v);
          if (e < E) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int d = 128 + 16 * u + i;
              if (d < D) f1[(size_t(h) * D + d) * E + e] = __uint_as_float(v[i]);
            }
          }
        }
#pragma unroll 1
        for (int u = 0; u < 8; ++u) {
          uint32_t v[16];
          tmem_ld16_sync(ta + C::TM_DW2 + 16 * u, v);
          const int cc = 128 + 16 * u;
          if (e < E && cc < D) {  // D % 16 == 0: all 16 columns are inside
            float4* dst = reinterpret_cast<float4*>(f2 + (size_t(h) * E + e) * D + cc);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dst[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                   __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
          }
        }
      } else {
        // dW1^T rows are E, columns D: each column d is one coalesced store across the warp
#pragma unroll 1
        for (int u = 0; u < 8; ++u) {
          uint32_t v[16];
          tmem_ld16_sync(ta + C::TM_DW1 + 16 * u, v);
          if (e < E) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int d = 128 + 16 * u + i;
              if (d < D) {
                const uint32_t pk = Pack<T>::pack(__uint_as_float(v[i]), 0.f);
                reinterpret_cast<uint16_t*>(dW1)[(size_t(h) * D + d) * E + e] = uint16_t(pk & 0xFFFFu);
              }
            }
          }
        }
        T* w2row = dW2 + (size_t(h) * E + e) * D;
#pragma unroll 1
        for (int u = 0; u < 8; ++u) {
          uint32_t v[16], p[8];
          tmem_ld16_sync(ta + C::TM_DW2 + 16 * u, v);
          plain_pack<T, 8>(v, p);
          const int cc = 128 + 16 * u;
          if (e < E) {
            uint4* dst = reinterpret_cast<uint4*>(w2row + cc);
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

template <typename T>
static cudaError_t launch_dw_gemm256_t(const BwdLaunch& a) {
  using C = DwGemmCfg;
  auto kern = fmlp_dw_gemm256_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int nB = (a.B + kRows - 1) / kRows;
  const int nEw = (a.E + 127) / 128;
  const int splits = a.splits < 1 ? 1 : a.splits;
  if (a.dzt == nullptr || (splits > 1 && (a.part == nullptr || splits > nB))) return cudaErrorInvalidValue;
  const long long grid = (long long)a.H * nEw * splits;
  if (grid <= 0 || grid > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  const T* dzt = reinterpret_cast<const T*>(a.dzt);
  kern<<<unsigned(grid), C::NUM_THREADS, C::SMEM, a.stream>>>(
      a.tm_x, a.tm_do, dzt, dzt + dz_tile_elems(a.H, a.B, a.E), reinterpret_cast<T*>(a.dw1),
      reinterpret_cast<T*>(a.dw2), a.dw_f32, splits > 1 ? a.part : nullptr, splits, a.H, a.B, a.D, a.E, a.status);
  return cudaGetLastError();
}

cudaError_t launch_dw_gemm256(const BwdLaunch& a) {
  if (a.dp != 256 || a.shared_x || a.f32) return cudaErrorNotSupported;
  return a.bf16 ? launch_dw_gemm256_t<__nv_bfloat16>(a) : launch_dw_gemm256_t<__half>(a);
}

}  // namespace fmlp
