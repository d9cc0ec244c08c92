// Host-side launch interface shared by the kernel translation units and the C ABI.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace fmlp {

struct FwdLaunch {
  CUtensorMap tm_x;   // X  (H,B,D)  viewed 3-D {D, B, H}, box {64, 128, 1}
  CUtensorMap tm_w1;  // W1 (H,D,E)  viewed 3-D {E, D, H}, box {64, DP, 1}
  CUtensorMap tm_w2;  // W2 (H,E,D)  viewed 3-D {D, E, H}, box {64, ET, 1}
  void* o;            // O  (H,B,D)  row-major, written directly
  int H, B, D, E;
  int dp;             // D rounded up to a multiple of 64 (64, 128 or 256)
  int bf16;           // 1 = bfloat16, 0 = float16 (fp32 inputs: f32 = 1)
  int f32;            // 1 = float32 inputs and outputs (TF32 products)
  int act;            // fmlp::Act
  int shared_x;       // 1: X is (B,D) for every head and o is the (B,D) mean over heads
  int grid;           // persistent CTAs (single-tile kernel)
  int sm_count;       // SMs of the device
  uint32_t* status;   // device status word
  cudaStream_t stream;
};

// FP8 (e4m3) forward (fmlp_fwd_fp8.cu): per-tensor scales, the weights pre-transposed
// so that every shared-memory operand is K-major.
struct Fp8FwdLaunch {
  CUtensorMap tm_x;    // X   (H,B,D) e4m3 viewed {D, B, H}, box {128, 128, 1}
  CUtensorMap tm_w1t;  // W1^T (H,E,D) e4m3 viewed {D, E, H}, box {128, 128, 1}
  CUtensorMap tm_w2t;  // W2^T (H,D,E) e4m3 viewed {E, D, H}, box {128, 128, 1}
  void* o;             // O (H,B,D) in bf16 or fp16
  int H, B, D, E;
  float z_scale;       // x_scale * w1_scale: Z = (X8 @ W1_8) * z_scale
  float h_inv_scale;   // 1 / h_scale: H8 = e4m3(act(Z) / h_scale), saturating
  float o_scale;       // h_scale * w2_scale: O = (H8 @ W2_8) * o_scale
  int act;
  int out_bf16;        // 1 = bfloat16 output, 0 = float16
  int sm_count;
  uint32_t* status;
  cudaStream_t stream;
};
cudaError_t launch_fwd_fp8(const Fp8FwdLaunch& a);

// Tensor maps of the fp32 (TF32) backward: *_k with the 128-byte swizzle (tiles read
// K-major), *_mn with the 128-byte swizzle of 32-byte atoms (tiles read MN-major, the
// only MN-major layout of TF32 operands). Boxes {32 elements, rows}: X, dO and W2 32 rows,
// W1 DP rows.
struct Tf32BwdMaps {
  CUtensorMap x_k, x_mn, do_k, do_mn, w1_k, w1_mn, w2_k;
  CUtensorMap dz;  // dZ-store mode: dZ workspace {nE*128, nB*128, H} fp32, box {32, 128}
};

struct BwdLaunch {
  CUtensorMap tm_x;    // X  {D, B, H}, box {64, 128, 1} (DP = 256: {64, 64, 1})
  CUtensorMap tm_do;   // dO {D, B, H}, box {64, 128, 1} (DP = 256: {64, 64, 1})
  CUtensorMap tm_w1;   // W1 {E, D, H}, box {64, DP, 1}
  CUtensorMap tm_w2;   // W2 {D, E, H}, box {64, 128, 1} (DP = 256: {64, 64, 1})
  const void* x;       // X and W1 as plain pointers (DP = 256 loads them into TMEM)
  const void* w1;
  void* dx;
  void* dw1;
  void* dw2;
  float* part;         // fp32 dW partial sums of split dW programs (splits > 1), else null
  float* dw_f32;       // if set: dW1 (H,D,E) then dW2 (H,E,D) as unrounded fp32, not dw1/dw2
  void* dzt;           // dZ-store mode: dZ^T tiles (H, nE, nB) x 128 x 128 in the input dtype
  const Tf32BwdMaps* tf32_maps;  // fp32 inputs only
  int splits;          // dW programs per (head, E chunk); 1 = no split (DP <= 128 only)
  int sm_count;
  int H, B, D, E;
  int dp, bf16, act;
  int f32;             // 1 = float32 inputs and outputs (TF32 products)
  int shared_x;        // 1: X, dO, dX are (B,D) shared by every head (mean over heads)
  uint32_t* status;
  cudaStream_t stream;
};

// Tile constants shared by host and device.
constexpr int kRows = 128;  // rows of a B tile (tcgen05 M)

inline int fwd_et(int dp) { return dp <= 128 ? 128 : 64; }
constexpr int kBwdEt = 128;  // E chunk of both backward program kinds

// Elements of one launch's stored dZ^T tiles (dZ-store mode): a 128 x 128 tile per (head,
// 128-wide E chunk, 128-row B tile). For 128 < D <= 256 the H^T tiles follow, as many.
inline size_t dz_tile_elems(int H, int B, int E) {
  return size_t(H) * ((size_t(E) + kBwdEt - 1) / kBwdEt) * kBwdEt * ((size_t(B) + kRows - 1) / kRows) * kRows;
}

// Forward on CTA pairs (fmlp_fwd2sm.cu): 16-bit inputs, per-head X, DP in {128, 256};
// a.tm_w2 must have boxes of 128 E rows.
cudaError_t launch_fwd2sm(const FwdLaunch& a);
int bwd_smem_bytes(int dp);
cudaError_t launch_fwd(const FwdLaunch& a);       // D <= 128: the row-pair kernel
cudaError_t launch_fwd_pair(const FwdLaunch& a);  // two row tiles per CTA, D <= 128
cudaError_t launch_bwd(const BwdLaunch& a);     // picks the kernel for a.dp
cudaError_t launch_bwd256(const BwdLaunch& a);  // 128 < D <= 256
cudaError_t launch_dx_gemm(const BwdLaunch& a);  // dX from the stored dZ^T (dZ-store mode)
// D half 1 of dW for 128 < D <= 256 from the stored dZ^T and H^T tiles (dZ-store mode)
cudaError_t launch_dw_gemm256(const BwdLaunch& a);
// fixed-order sum of the a.splits fp32 dW partials at a.part into dw1/dw2 (or a.dw_f32)
cudaError_t launch_dw_reduce(const BwdLaunch& a);
cudaError_t launch_fwd_tf32(const FwdLaunch& a);  // fp32 inputs, TF32 products, D <= 128
cudaError_t launch_bwd_tf32(const BwdLaunch& a);
int bwd256_smem_bytes();
// SM count and device status word of the current device (fails if it is not an sm_100).
int current_device_status(int* sm_count, uint32_t** status);
void* current_context();  // the calling thread's current CUDA context (CUcontext), or nullptr

// Split factor of the dW programs for a backward launch (1 = none) and the fp32 workspace
// bytes it needs: 2 * splits * H * D * E * 4 when splits > 1.
int bwd_dw_splits(int H, int B, int D, int E, int sm_count);
size_t bwd_workspace_bytes(int H, int B, int D, int E, int sm_count);
// The same for the fp32 (TF32) backward, whose dW programs walk 32-row B tiles.
int bwd_dw_splits_tf32(int H, int B, int D, int E, int sm_count);
size_t bwd_workspace_bytes_tf32(int H, int B, int D, int E, int sm_count);
int bwd_dz_splits_tf32(int H, int B, int D, int E, int sm_count);  // dZ-store mode, fp32

// dZ-store mode of the backward (16-bit inputs with D <= 256, fp32 inputs with D <= 128):
// the dW programs also store dZ and a GEMM over E forms dX from it (fmlp_dxgemm.cu; fp32:
// fmlp_tf32.cu); for 128 < D <= 256 they store H^T as well, and a GEMM over B forms the
// second D half of dW from the two (fmlp_dwgemm256.cu). bwd_dz_bytes is the dZ (and H^T)
// workspace of one launch over H heads for elements
// of elem_bytes (0 when the mode does not apply or would need more than kDzCapBytes: the
// kernels address a launch's dZ tiles with 32-bit element offsets); bwd_dz_splits the dW
// split factor of that launch, whose fp32 partials follow the dZ region
// (bwd_dz_workspace_bytes is the total). A backward call whose heads do not fit one such
// launch, or whose caller gives a smaller workspace, runs the mode in head groups that
// reuse the workspace: bwd_dz_group_heads is the group size for a workspace (0: the mode
// does not apply, or fewer than min(H, kDzMinGroupHeads) heads fit, where the recompute
// mode in one launch is the better choice).
constexpr size_t kDzCapBytes = size_t(8) << 30;
constexpr int kDzMinGroupHeads = 4;
size_t bwd_dz_bytes(int H, int B, int D, int E, int sm_count, int elem_bytes = 2);
int bwd_dz_splits(int H, int B, int D, int E, int sm_count);
size_t bwd_dz_workspace_bytes(int H, int B, int D, int E, int sm_count, int elem_bytes = 2);
int bwd_dz_group_heads(int H, int B, int D, int E, int sm_count, int elem_bytes, size_t workspace_bytes);

// Body of fmlp_bwd; allow_dz = 0 keeps the recompute mode whatever the workspace size
// (fmlp_bwd_noalloc).
int bwd_entry(const void* x, const void* w1, const void* w2, const void* dO, void* dx, void* dw1, void* dw2,
              void* workspace, size_t workspace_bytes, int H, int B, int D, int E, int dtype, int act,
              void* stream, int allow_dz);

}  // namespace fmlp
