// FP8 (e4m3) forward for D <= 128: O = act(X W1) W2 per head with 8-bit operands on
// tcgen05.mma kind::f8f6f4 and fp32 accumulation. Not in the reference (flashmlp.py has
// 16-bit and fp32 paths only); its forward kernel `flashmlp_fwd_kernel` (flashmlp.py:63-158)
// sets the structure this follows: E in chunks, Z and H never leave the SM.
//
// Scaling (per tensor, the usual FP8 inference recipe): the caller passes e4m3 tensors X8,
// W1^T_8, W2^T_8 and scales sx, sw1, sw2, sh with X ~ sx X8 etc.;
//   Z  = (X8 @ W1_8) * (sx sw1)                       fp32 (products of e4m3 are exact)
//   H8 = e4m3(act(Z) / sh)                            round to nearest even, saturating
//   O  = (H8 @ W2_8) * (sh sw2)                       fp32, rounded once to bf16/fp16
// The weights come transposed (W1^T (H,E,D), W2^T (H,D,E)): then both shared-memory
// operands of both products are K-major, the layout every operand type supports, and a
// 128-byte swizzled row holds a whole K-step group (128 e4m3 values).
//
// Same pipeline as the 16-bit row-pair kernel (fmlp_fwd_pair.cu): two 128-row tiles of
// one head per CTA share each weight chunk; warp 0 TMA, warps 1-2 issue the products of
// tile A / tile B, warps 3-18 activate. Per tile t and 128-wide E chunk c:
//   G1_t(c): Z_t = X_t[smem] @ W1c[smem]     SS M=128(b) N=128(e) K=128(d)  4 MMAs
//   activation: Z_t -> H8_t, 32 values per warp slice packed into its first 8 columns
//   G2_t(c): O_t += H8_t[tmem] @ W2c[smem]   TS M=128(b) N=128(d) K=128(e)  4 MMAs
// TMEM: O_A [0,128) O_B [128,256) Z_A [256,384) Z_B [384,512). smem: X_A, X_B (16 KB
// each) + 4-stage rings of W1c and W2c chunks (16 KB each) = 160 KB.
#include <cuda_fp8.h>

#include "fmlp_act.cuh"
#include "fmlp_kernels.h"
#include "fmlp_ptx.cuh"

namespace fmlp {

struct FwdFp8Cfg {
  static constexpr int BM = kRows;
  static constexpr int ET = 128;     // E chunk
  static constexpr int DB = 128;     // D padded: one 128-byte row of e4m3 values
  static constexpr int WS = 4;       // weight stages
  static constexpr int X_BYTES = BM * DB;
  static constexpr int W1_BYTES = ET * DB;  // W1^T chunk: 128 e rows x 128 d
  static constexpr int W2_BYTES = DB * ET;  // W2^T chunk: 128 d rows x 128 e
  static constexpr int OFF_X = 0;
  static constexpr int OFF_W1 = OFF_X + 2 * X_BYTES;
  static constexpr int OFF_W2 = OFF_W1 + WS * W1_BYTES;
  static constexpr int OFF_BAR = OFF_W2 + WS * W2_BYTES;
  static constexpr int NBAR = 4 + 4 * WS + 8 + 2;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_USED = OFF_MISC + 16 + 1024;
  static constexpr int SMEM = SMEM_USED > 120 * 1024 ? SMEM_USED : 120 * 1024;
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr int TMEM_O = 0;    // O_t at TMEM_O + t*DB
  static constexpr int TMEM_Z = 256;  // Z_t at TMEM_Z + t*ET
  static constexpr int TMEM_COLS = 512;
  static constexpr int NUM_ACT_WARPS = 16;
  static constexpr int FIRST_ACT_WARP = 3;
  static constexpr int NUM_THREADS = 32 * (FIRST_ACT_WARP + NUM_ACT_WARPS);
  static constexpr int SW = ET / 4;  // Z columns per activation warp (one K-step of G2)
  static constexpr int OW = DB / 4;  // O columns per activation warp
};

// Four e4m3 values, saturating round to nearest even, a0 in the lowest byte.
__device__ __forceinline__ uint32_t pack_e4m3x4(float a0, float a1, float a2, float a3) {
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a0, a1), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(a2, a3), __NV_SATFINITE, __NV_E4M3);
  return lo | (hi << 16);
}

// act(z * z_scale) * h_inv_scale for the pair (v0, v1), two elements per instruction
// (sm_100's packed fp32 forms). The SFU is this kernel's bound (75 % busy against 35 % for
// the tensor pipe at 8 bits), so pairs with pair % FMLP_FP8_FMA_EVERY ==
// FMLP_FP8_FMA_EVERY - 1 evaluate the sigmoid on the FMA pipe instead (sigmoid2_fma, max
// relative error 8.1e-5, below tanh.approx's); measured at C4: every 8th pair 1.37 ->
// 1.34 ms, every 6th the same, every 4th 1.49 ms (the FMA/ALU pipes fill), 0 = never.
#ifndef FMLP_FP8_FMA_EVERY
#define FMLP_FP8_FMA_EVERY 8
#endif
template <int ACT>
__device__ __forceinline__ uint64_t act_fwd_scaled_pair(uint32_t v0, uint32_t v1, uint64_t zs2, uint64_t his2,
                                                        int pair) {
  const uint64_t z = mul2(f2(__uint_as_float(v0), __uint_as_float(v1)), zs2);
  uint64_t h;
  if constexpr (ACT == kSilu || ACT == kSigmoid) {
    const uint64_t half = f2(0.5f, 0.5f);
    if (FMLP_FP8_FMA_EVERY > 0 && pair % (FMLP_FP8_FMA_EVERY > 0 ? FMLP_FP8_FMA_EVERY : 1) == FMLP_FP8_FMA_EVERY - 1) {
      const uint64_t sg = sigmoid2_fma(z);
      h = ACT == kSilu ? mul2(z, sg) : sg;
    } else {
      const uint64_t u = mul2(half, z);
      const uint64_t t = f2(tanh_approx(f2_lo(u)), tanh_approx(f2_hi(u)));
      h = ACT == kSilu ? fma2(u, t, u) : fma2(half, t, half);  // u tanh(u) + u, or sigma
    }
  } else if constexpr (ACT == kLeakyRelu) {
    const uint64_t m = mul2(f2(0.01f, 0.01f), z);
    h = f2(fmaxf(f2_lo(z), f2_lo(m)), fmaxf(f2_hi(z), f2_hi(m)));
  } else {
    h = z;
  }
  return mul2(h, his2);
}

template <typename TO, int ACT>
__global__ void __launch_bounds__(608, 1)
    fmlp_fwd_fp8_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w1t,
                        const __grid_constant__ CUtensorMap tm_w2t, TO* __restrict__ O, int H, int B, int D, int E,
                        float z_scale, float h_inv_scale, float o_scale, uint32_t* status) {
  using C = FwdFp8Cfg;
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
  const int nitems = H * nP;

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
    tma_prefetch_desc(&tm_w1t);
    tma_prefetch_desc(&tm_w2t);
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
        const int h = item / nP, pr = item % nP;
        for (int t = 0; t < 2 && ok; ++t) {
          if (!(ok = mbar_wait(&x_empty[t], (it & 1) ^ 1, ctx))) break;
          mbar_arrive_expect_tx(&x_full[t], C::X_BYTES);
          tma_load_3d(sX + t * C::X_BYTES, &tm_x, &x_full[t], 0, (2 * pr + t) * BM, h);
          ++xl[t];
        }
        for (int c = 0; c < nE && ok; ++c) {
          {
            const int s = c1 % WS;
            if (!(ok = mbar_wait(&w1_empty[s], ((c1 / WS) & 1) ^ 1, ctx))) break;
            mbar_arrive_expect_tx(&w1_full[s], C::W1_BYTES);
            tma_load_3d(sW1 + s * C::W1_BYTES, &tm_w1t, &w1_full[s], 0, c * ET, h);
            ++c1;
          }
          {
            const int s = c2 % WS;
            if (!(ok = mbar_wait(&w2_empty[s], ((c2 / WS) & 1) ^ 1, ctx))) break;
            mbar_arrive_expect_tx(&w2_full[s], C::W2_BYTES);
            tma_load_3d(sW2 + s * C::W2_BYTES, &tm_w2t, &w2_full[s], c * ET, 0, h);
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
    // Warp 1 drives tile A, warp 2 tile B (disjoint TMEM columns; the weight stages they
    // share are released by both).
    const int t = warp - 1;
    // e4m3 x e4m3 (format code 0 for both), fp32 accumulation, both operands K-major
    constexpr uint32_t idesc = make_idesc_f16(false, BM, 128, false, false);
    const uint64_t xd = make_sdesc_sw128(smem_u32(sX) + t * C::X_BYTES, 16, 1024);
    const uint32_t sW1_a = smem_u32(sW1), sW2_a = smem_u32(sW2);
    const uint32_t z_tmem = tmem + C::TMEM_Z + t * ET;
    const uint32_t o_tmem = tmem + C::TMEM_O + t * C::DB;
    uint32_t c1 = 0, c2 = 0, it = 0;
    bool ok = true;

    // G1 of this tile for the next W1 chunk (K over the padded 128 d, zero-filled).
    auto gemm1 = [&](bool last) -> bool {  // last: final G1 of this pair for tile t
      const int s1 = c1 % WS;
      if (!warp_wait(&w1_full[s1], (c1 / WS) & 1, ctx)) return false;
      ++c1;
      tc_fence_after();
      if (elect_one()) {
        const uint64_t wd = make_sdesc_sw128(sW1_a + s1 * C::W1_BYTES, 16, 1024);
#pragma unroll
        for (int k = 0; k < C::DB / 32; ++k)
          mma_ss_f8(z_tmem, sdesc_add(xd, k * 32), sdesc_add(wd, k * 32), idesc, k > 0 ? 1u : 0u);
        mma_commit(&z_full[t]);
        mma_commit(&w1_empty[s1]);
        if (last) mma_commit(&x_empty[t]);  // every reader of X_t has been issued
      }
      __syncwarp();
      return true;
    };

    for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x, ++it) {
      if (!(ok = warp_wait(&x_full[t], it & 1, ctx))) break;
      if (!(ok = gemm1(nE == 1))) break;
      for (int c = 0; c < nE && ok; ++c) {
        const uint32_t zc = it * nE + c;  // chunk index, for the z/h barrier parities
        const int s2 = c2 % WS;
        if (!(ok = warp_wait(&w2_full[s2], (c2 / WS) & 1, ctx))) break;
        ++c2;
        if (c == 0 && !(ok = warp_wait(&o_empty[t], (it & 1) ^ 1, ctx))) break;
        if (!(ok = warp_wait(&h_full[t], zc & 1, ctx))) break;
        tc_fence_after();
        if (elect_one()) {
          // G2: O_t += H8_t @ W2c; the 32 H8 values of E columns [32k, 32k+32) sit in the
          // first 8 columns of slice k
          const uint64_t wd = make_sdesc_sw128(sW2_a + s2 * C::W2_BYTES, 16, 1024);
          const uint32_t acc0 = c > 0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < ET / 32; ++k)
            mma_ts_f8(o_tmem, z_tmem + k * SW, sdesc_add(wd, k * 32), idesc, k > 0 ? 1u : acc0);
          mma_commit(&w2_empty[s2]);
          if (c + 1 == nE) mma_commit(&o_full[t]);
        }
        __syncwarp();
        if (c + 1 < nE && !(ok = gemm1(c + 2 == nE))) break;  // overwrites Z_t after G2 read H8_t
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
    const uint64_t zs2 = f2(z_scale, z_scale), his2 = f2(h_inv_scale, h_inv_scale);
    for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x, ++it) {
      const int h = item / nP, pr = item % nP;
      for (int c = 0; c < nE && ok; ++c) {
        const uint32_t zc = it * nE + c;
        for (int t = 0; t < 2; ++t) {
          if (!(ok = mbar_wait(&z_full[t], zc & 1, ctx))) break;
          tc_fence_after();
          const uint32_t za = tmem + lane_off + C::TMEM_Z + t * ET + j * SW;
          uint32_t v[SW], p[SW / 4];
          tmem_ld32_sync(za, v);
#pragma unroll
          for (int i = 0; i < SW / 4; ++i) {
            const uint64_t q0 = act_fwd_scaled_pair<ACT>(v[4 * i], v[4 * i + 1], zs2, his2, 2 * i);
            const uint64_t q1 = act_fwd_scaled_pair<ACT>(v[4 * i + 2], v[4 * i + 3], zs2, his2, 2 * i + 1);
            p[i] = pack_e4m3x4(f2_lo(q0), f2_hi(q0), f2_lo(q1), f2_hi(q1));
          }
          tmem_st8(za, p);  // H8 over the first 8 columns of the slice, just read
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&h_full[t]);
        }
      }
      // Epilogue per tile: O_t (fp32, TMEM) * o_scale -> output dtype -> global.
      for (int t = 0; t < 2 && ok; ++t) {
        if (!(ok = mbar_wait(&o_full[t], it & 1, ctx))) break;
        tc_fence_after();
        const int row = (2 * pr + t) * BM + q * 32 + lane;
        TO* orow = O + (size_t(h) * B + row) * D;
        const uint32_t oa = tmem + lane_off + C::TMEM_O + t * C::DB + j * OW;
        uint32_t v[OW], p[OW / 2];
        tmem_ld32_sync(oa, v);
#pragma unroll
        for (int i = 0; i < OW; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * o_scale);
        plain_pack<TO, OW / 2>(v, p);
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

template <typename TO, int ACT>
static cudaError_t launch_fp8_t(const Fp8FwdLaunch& a) {
  using C = FwdFp8Cfg;
  auto kern = fmlp_fwd_fp8_kernel<TO, ACT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const long long nB = (a.B + kRows - 1) / kRows;
  const long long items = (long long)a.H * ((nB + 1) / 2);
  const int grid = int(items < a.sm_count ? items : a.sm_count);
  kern<<<grid, C::NUM_THREADS, C::SMEM, a.stream>>>(a.tm_x, a.tm_w1t, a.tm_w2t, reinterpret_cast<TO*>(a.o), a.H,
                                                    a.B, a.D, a.E, a.z_scale, a.h_inv_scale, a.o_scale,
                                                    a.status);
  return cudaGetLastError();
}

template <typename TO>
static cudaError_t launch_fp8_act(const Fp8FwdLaunch& a) {
  switch (a.act) {
    case kLeakyRelu: return launch_fp8_t<TO, kLeakyRelu>(a);
    case kSilu: return launch_fp8_t<TO, kSilu>(a);
    case kSigmoid: return launch_fp8_t<TO, kSigmoid>(a);
    default: return launch_fp8_t<TO, kLinear>(a);
  }
}

cudaError_t launch_fwd_fp8(const Fp8FwdLaunch& a) {
  return a.out_bf16 ? launch_fp8_act<__nv_bfloat16>(a) : launch_fp8_act<__half>(a);
}

}  // namespace fmlp
