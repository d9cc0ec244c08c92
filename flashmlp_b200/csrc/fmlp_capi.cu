// C ABI of libflashmlp_b200.so: argument checks, TMA tensor maps, launches.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/flashmlp_b200.h"
#include "fmlp_kernels.h"
#include "fmlp_ptx.cuh"

namespace fmlp {

// Per-device kernel status word (see fmlp_ptx.cuh, mbar_wait).
__device__ uint32_t g_fmlp_status;

namespace {

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  bool init = false;
  void* ctx = nullptr;  // the context the cached device addresses belong to
  int sm_count = 0;
  int cc_major = 0;
  uint32_t* status = nullptr;
};

std::mutex g_mu;
DeviceInfo g_dev[kMaxDevices];
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

}  // namespace

// The calling thread's current CUDA context (cuCtxGetCurrent through the runtime's
// driver entry point), or nullptr if there is none or the lookup fails. Device addresses
// of __device__ symbols belong to a context: after cudaDeviceReset the primary context
// is a new one, and addresses cached for the old one would dangle.
void* current_context() {
  static PFN_cuCtxGetCurrent_v4000 fn = []() -> PFN_cuCtxGetCurrent_v4000 {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f);
  }();
  CUcontext c = nullptr;
  if (fn == nullptr || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

namespace {

int device_info(DeviceInfo** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return FMLP_ERR_CUDA;
  void* ctx = current_context();
  if (ctx == nullptr) {  // no context yet on this thread: make the device's primary one current
    cudaFree(nullptr);
    ctx = current_context();
  }
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.init || d.ctx != ctx) {
    d.init = false;
    if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return FMLP_ERR_CUDA;
    if (cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return FMLP_ERR_CUDA;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fmlp_status) != cudaSuccess) return FMLP_ERR_CUDA;
    d.status = static_cast<uint32_t*>(p);
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
              cudaSuccess ||
          q != cudaDriverEntryPointSuccess || fn == nullptr)
        return FMLP_ERR_TMA;
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    d.ctx = ctx;
    d.init = true;
  }
  if (d.cc_major != 10) return FMLP_ERR_DEVICE;
  *out = &d;
  return FMLP_OK;
}

// 3-D tiled map over a contiguous (d2, d1, d0) row-major tensor of `dtype` elements
// (FMLP_DTYPE_*), 128-byte swizzle, zero fill out of bounds.
int encode3d(CUtensorMap* m, const void* ptr, int dtype, uint64_t d0, uint64_t d1, uint64_t d2,
             uint32_t b0, uint32_t b1, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  const uint64_t esz = dtype == FMLP_DTYPE_F32 ? 4 : 2;
  const CUtensorMapDataType dt = dtype == FMLP_DTYPE_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == FMLP_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * esz, d0 * d1 * esz};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FMLP_OK : FMLP_ERR_TMA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 3-D map of a byte tensor (e4m3 values) {d0, d1, d2} with 128 x 128-byte boxes.
int encode3d_u8(CUtensorMap* m, const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2) {
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0, d0 * d1};
  cuuint32_t box[3] = {128, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FMLP_OK : FMLP_ERR_TMA;
}

int check_common(int H, int B, int D, int E, int dtype) {
  if (H < 0 || B < 0 || D < 0 || E < 0) return FMLP_ERR_INVALID_SHAPE;
  if (dtype != FMLP_DTYPE_F16 && dtype != FMLP_DTYPE_BF16 && dtype != FMLP_DTYPE_F32)
    return FMLP_ERR_UNSUPPORTED_DTYPE;
  const long long hb = (long long)H * B, hd = (long long)H * D;
  if (hb * D >= (1LL << 40) || hd * E >= (1LL << 40)) return FMLP_ERR_INVALID_SHAPE;
  if (B > (1 << 30) || E > (1 << 30)) return FMLP_ERR_INVALID_SHAPE;
  return FMLP_OK;
}

int round_dp(int D) { return D <= 64 ? 64 : (D <= 128 ? 128 : 256); }

size_t elem_bytes(int dtype) { return dtype == FMLP_DTYPE_F32 ? 4 : 2; }

int cuda_rc(cudaError_t e) { return e == cudaSuccess ? FMLP_OK : FMLP_ERR_CUDA; }

// What a backward call runs for a given workspace: the dZ-store mode when the workspace
// holds the dZ^T tiles (and their split-dW partials) of a group of at least
// min(H, kDzMinGroupHeads) heads and the mode applies, otherwise the recompute mode,
// which needs `need` bytes (0 unless its dW programs split). In the dZ-store mode the
// heads run in groups of `group` that reuse the workspace (one group when it holds all
// heads). One rule for fmlp_bwd and fmlp_bwd_plan. `usable`: the workspace pointer is
// non-null and 16-byte aligned (fmlp_bwd_plan assumes it is). `grouping`: the call may run
// in head groups (not the shared-input form, whose dX sums over heads, nor the fp32-dW
// form, whose dW2 block follows all heads' dW1).
struct BwdPlan {
  bool dz = false;
  int splits = 1;
  int group = 0;        // heads per launch: H, or the group size in the dZ-store mode
  size_t dz_bytes = 0;  // dZ^T region at the start of the workspace (dZ-store mode)
};

int plan_bwd(int H, int B, int D, int E, bool f32, bool allow_dz, bool grouping, int sm_count,
             size_t workspace_bytes, bool usable, BwdPlan* p) {
  const size_t need = f32 ? bwd_workspace_bytes_tf32(H, B, D, E, sm_count) : bwd_workspace_bytes(H, B, D, E, sm_count);
  const int esz = f32 ? 4 : 2;  // dZ is stored in the input dtype (fp32 stays fp32)
  p->group = H;
  if (allow_dz && usable) {
    const int g = bwd_dz_group_heads(H, B, D, E, sm_count, esz, workspace_bytes);
    if (g > 0 && (grouping || g == H)) {
      p->dz = true;
      p->group = g;
      p->splits = f32 ? bwd_dz_splits_tf32(g, B, D, E, sm_count) : bwd_dz_splits(g, B, D, E, sm_count);
      p->dz_bytes = bwd_dz_bytes(g, B, D, E, sm_count, esz);
      return FMLP_OK;
    }
  }
  if (workspace_bytes < need || (need && !usable)) return FMLP_ERR_WORKSPACE;
  p->splits = need ? (f32 ? bwd_dw_splits_tf32(H, B, D, E, sm_count) : bwd_dw_splits(H, B, D, E, sm_count)) : 1;
  return FMLP_OK;
}

// w - lr * g is formed with two roundings (no FMA contraction), the same arithmetic as the
// fused all-reduce + SGD kernel and as `w.float() - lr * g` in PyTorch.
__global__ void sgd_kernel_bf16(__nv_bfloat16* w, const float* g, long long n, float lr) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    w[i] = __float2bfloat16_rn(__fsub_rn(__bfloat162float(w[i]), __fmul_rn(lr, g[i])));
}
__global__ void sgd_kernel_f16(__half* w, const float* g, long long n, float lr) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    w[i] = __float2half_rn(__fsub_rn(__half2float(w[i]), __fmul_rn(lr, g[i])));
}

}  // namespace

int current_device_status(int* sm_count, uint32_t** status) {
  DeviceInfo* d = nullptr;
  const int rc = device_info(&d);
  if (rc) return rc;
  *sm_count = d->sm_count;
  *status = d->status;
  return FMLP_OK;
}

}  // namespace fmlp

using namespace fmlp;

extern "C" {

int fmlp_abi_version(void) { return 100; }

const char* fmlp_error_string(int code) {
  switch (code) {
    case FMLP_OK: return "ok";
    case FMLP_ERR_INVALID_SHAPE: return "invalid shape (negative size or too large)";
    case FMLP_ERR_UNSUPPORTED_DTYPE:
      return "unsupported dtype (float16, bfloat16; float32 only for the per-head fmlp_fwd/fmlp_bwd)";
    case FMLP_ERR_UNSUPPORTED_D:
      return "unsupported hidden dim D (needs D % 16 == 0 and D <= 256; D <= 128 for float32 and for the "
             "shared-input entry points)";
    case FMLP_ERR_UNSUPPORTED_E: return "unsupported intermediate dim E (needs E % 8 == 0)";
    case FMLP_ERR_MISALIGNED: return "tensor data pointer is not 16-byte aligned";
    case FMLP_ERR_CUDA: return "CUDA runtime error";
    case FMLP_ERR_TMA: return "TMA tensor-map encoding failed";
    case FMLP_ERR_DEVICE: return "current device is not an sm_100 (B200-class) GPU";
    case FMLP_ERR_WORKSPACE: return "workspace too small";
    case FMLP_ERR_DEVICE_TIMEOUT: return "a kernel pipeline wait timed out on the device";
    case FMLP_ERR_SCRATCH_LIMIT:
      return "shape needs more scratch than fmlp_bwd_noalloc's static device buffer "
             "(FMLP_NOALLOC_SCRATCH_BYTES); call fmlp_bwd with a workspace";
    case FMLP_ERR_PEER_ABORT:
      return "a rank of the fused all-reduce group gave up on a barrier (now or in an earlier call); "
             "every rank should stop";
    case FMLP_ERR_INVALID_SCALE: return "fmlp_fwd_fp8: every scale must be finite and > 0";
  }
  return "unknown error";
}

}  // extern "C"

namespace {

// Shared body of fmlp_fwd (X, O per head) and fmlp_fwd_shared_x (X, O (B,D), O the mean
// over heads).
int fwd_impl(const void* x, const void* w1, const void* w2, void* o, int H, int B, int D, int E, int dtype,
             int act, int shared_x, void* stream) {
  int rc = check_common(H, B, D, E, dtype);
  if (rc) return rc;
  const bool f32 = dtype == FMLP_DTYPE_F32;
  if (f32 && shared_x) return FMLP_ERR_UNSUPPORTED_DTYPE;
  if (D % 16 != 0 || D > (shared_x || f32 ? 128 : 256)) return FMLP_ERR_UNSUPPORTED_D;
  if (E % 8 != 0) return FMLP_ERR_UNSUPPORTED_E;
  if (shared_x && H == 0) return FMLP_ERR_INVALID_SHAPE;  // no mean over zero heads
  DeviceInfo* dev = nullptr;
  if ((rc = device_info(&dev))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t o_elems = size_t(shared_x ? 1 : H) * B * D;
  if (o_elems == 0) return FMLP_OK;
  if (E == 0) return cuda_rc(cudaMemsetAsync(o, 0, o_elems * elem_bytes(dtype), st));
  if (!aligned16(x) || !aligned16(w1) || !aligned16(w2) || !aligned16(o)) return FMLP_ERR_MISALIGNED;
  FwdLaunch a{};
  a.dp = round_dp(D);
  // 64 < D <= 256 (16-bit, per-head X): CTA-pair kernel, W2 chunks of 128 E rows
  const bool pair = !f32 && !shared_x && a.dp >= 128;
  const int et = f32 ? 64 : (pair ? 128 : fwd_et(a.dp));
  const uint32_t inner = f32 ? 32 : 64;  // elements per 128-byte swizzled row
  // fp32: the weight chunks are read MN-major only, which needs the 32-byte-atom swizzle
  const CUtensorMapSwizzle wswz = f32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  if ((rc = encode3d(&a.tm_x, x, dtype, D, B, shared_x ? 1 : H, inner, kRows))) return rc;
  if ((rc = encode3d(&a.tm_w1, w1, dtype, E, D, H, inner, a.dp, wswz))) return rc;
  if ((rc = encode3d(&a.tm_w2, w2, dtype, D, E, H, inner, et, wswz))) return rc;
  const int bf = dtype == FMLP_DTYPE_BF16;
  a.f32 = f32;
  a.o = o;
  a.H = H, a.B = B, a.D = D, a.E = E;
  a.bf16 = bf;
  a.act = act;
  a.shared_x = shared_x;
  const long long tiles = (long long)H * ((B + kRows - 1) / kRows);
  a.grid = int(tiles < dev->sm_count ? tiles : dev->sm_count);
  a.sm_count = dev->sm_count;
  a.status = dev->status;
  a.stream = st;
  return cuda_rc(f32 ? launch_fwd_tf32(a) : (pair ? launch_fwd2sm(a) : launch_fwd(a)));
}

}  // namespace

extern "C" {

int fmlp_fwd(const void* x, const void* w1, const void* w2, void* o, int H, int B, int D, int E,
             int dtype, int act, void* stream) {
  return fwd_impl(x, w1, w2, o, H, B, D, E, dtype, act, 0, stream);
}

int fmlp_fwd_shared_x(const void* x, const void* w1, const void* w2, void* o, int H, int B, int D, int E,
                      int dtype, int act, void* stream) {
  return fwd_impl(x, w1, w2, o, H, B, D, E, dtype, act, 1, stream);
}

int fmlp_fwd_fp8(const void* x, const void* w1t, const void* w2t, void* o, int H, int B, int D, int E,
                 float x_scale, float w1_scale, float w2_scale, float h_scale, int act, int out_dtype,
                 void* stream) {
  if (H < 0 || B < 0 || D < 0 || E < 0 || B > (1 << 30) || E > (1 << 30)) return FMLP_ERR_INVALID_SHAPE;
  if ((long long)H * B * D >= (1LL << 40) || (long long)H * D * E >= (1LL << 40)) return FMLP_ERR_INVALID_SHAPE;
  if (out_dtype != FMLP_DTYPE_BF16 && out_dtype != FMLP_DTYPE_F16) return FMLP_ERR_UNSUPPORTED_DTYPE;
  if (D % 16 != 0 || D > 128) return FMLP_ERR_UNSUPPORTED_D;
  if (E % 16 != 0) return FMLP_ERR_UNSUPPORTED_E;  // W2^T rows of E bytes: 16-byte strides
  const float sc[4] = {x_scale, w1_scale, w2_scale, h_scale};
  for (float v : sc)
    if (!(v > 0.f) || !(v < 3.0e38f)) return FMLP_ERR_INVALID_SCALE;  // also rejects NaN
  DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (size_t(H) * B * D == 0) return FMLP_OK;
  if (E == 0) return cuda_rc(cudaMemsetAsync(o, 0, size_t(H) * B * D * 2, st));
  if (!aligned16(x) || !aligned16(w1t) || !aligned16(w2t) || !aligned16(o)) return FMLP_ERR_MISALIGNED;
  Fp8FwdLaunch a{};
  // e4m3 tensors as bytes; boxes of 128 x 128 bytes, 128-byte swizzle (all K-major)
  if ((rc = encode3d_u8(&a.tm_x, x, D, B, H))) return rc;
  if ((rc = encode3d_u8(&a.tm_w1t, w1t, D, E, H))) return rc;
  if ((rc = encode3d_u8(&a.tm_w2t, w2t, E, D, H))) return rc;
  a.o = o;
  a.H = H, a.B = B, a.D = D, a.E = E;
  a.z_scale = x_scale * w1_scale;
  a.h_inv_scale = 1.0f / h_scale;
  a.o_scale = h_scale * w2_scale;
  a.act = act;
  a.out_bf16 = out_dtype == FMLP_DTYPE_BF16;
  a.sm_count = dev->sm_count;
  a.status = dev->status;
  a.stream = st;
  return cuda_rc(launch_fwd_fp8(a));
}

size_t fmlp_bwd_workspace_size_min(int H, int B, int D, int E, int dtype) {
  if (check_common(H, B, D, E, dtype) || D % 16 != 0 || D > 256 || E % 8 != 0) return 0;
  DeviceInfo* dev = nullptr;
  if (device_info(&dev)) return 0;
  return dtype == FMLP_DTYPE_F32 ? bwd_workspace_bytes_tf32(H, B, D, E, dev->sm_count)
                                 : bwd_workspace_bytes(H, B, D, E, dev->sm_count);
}

size_t fmlp_bwd_workspace_size(int H, int B, int D, int E, int dtype) {
  const size_t least = fmlp_bwd_workspace_size_min(H, B, D, E, dtype);
  if (D > 256 || check_common(H, B, D, E, dtype) || D % 16 != 0 || E % 8 != 0) return least;
  DeviceInfo* dev = nullptr;
  if (device_info(&dev)) return 0;
  const int esz = dtype == FMLP_DTYPE_F32 ? 4 : 2;
  // the largest head group the cap allows (all heads when they fit one launch)
  const int g = bwd_dz_group_heads(H, B, D, E, dev->sm_count, esz, ~size_t(0));
  const size_t dz = g > 0 ? bwd_dz_workspace_bytes(g, B, D, E, dev->sm_count, esz) : 0;
  return dz > least ? dz : least;
}

int fmlp_bwd_plan(int H, int B, int D, int E, int dtype, size_t workspace_bytes, int* mode, int* splits,
                  int* launches) {
  int rc = check_common(H, B, D, E, dtype);
  if (rc) return rc;
  const bool f32 = dtype == FMLP_DTYPE_F32;
  if (D % 16 != 0 || D > (f32 ? 128 : 256)) return FMLP_ERR_UNSUPPORTED_D;
  if (E % 8 != 0) return FMLP_ERR_UNSUPPORTED_E;
  DeviceInfo* dev = nullptr;
  if ((rc = device_info(&dev))) return rc;
  BwdPlan p;  // the choice fmlp_bwd makes for a non-null, 16-byte aligned workspace
  if ((rc = plan_bwd(H, B, D, E, f32, true, true, dev->sm_count, workspace_bytes, true, &p))) return rc;
  const bool empty = H == 0 || B == 0 || D == 0 || E == 0;
  const int groups = p.dz ? (H + p.group - 1) / p.group : 1;
  if (mode) *mode = p.dz ? 1 : 0;
  if (splits) *splits = p.splits;
  // dW programs, [D-half-1 dW GEMM (dZ-store mode, 128 < D <= 256)], [dX GEMM (dZ-store
  // mode)], [ordered reduce of the split dW partials]
  const int dw_gemm = (p.dz && !f32 && D > 128) ? 1 : 0;
  if (launches) *launches = empty ? 0 : groups * (1 + dw_gemm + (p.dz ? 1 : 0) + (p.splits > 1 ? 1 : 0));
  return FMLP_OK;
}

}  // extern "C"

namespace {

// One backward launch sequence over Hg heads whose tensors start at the given pointers.
int bwd_launch_group(const void* x, const void* w1, const void* w2, const void* dO, void* dx, void* dw1, void* dw2,
                     float* dwf, void* workspace, const BwdPlan& plan, int H, int B, int D, int E, int dtype, int act,
                     int shared_x, const DeviceInfo* dev, cudaStream_t st) {
  int rc = FMLP_OK;
  const bool f32 = dtype == FMLP_DTYPE_F32;
  BwdLaunch a{};
  a.dp = round_dp(D);
  const int bf = dtype == FMLP_DTYPE_BF16;
  // B rows and W2 E rows per TMA box: 128 for 16-bit D <= 128; 64 for D = 256 and fp32
  const int rows = (a.dp == 256 || f32) ? 64 : kRows;
  const uint32_t inner = f32 ? 32 : 64;  // elements per 128-byte swizzled row
  const int hx = shared_x ? 1 : H;       // heads of X / dO
  Tf32BwdMaps tm32;
  if (f32) {  // 32-row boxes; tiles read MN-major get a second map with 32-byte atoms
    const CUtensorMapSwizzle mn = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
    if ((rc = encode3d(&tm32.x_k, x, dtype, D, B, H, 32, 32))) return rc;
    if ((rc = encode3d(&tm32.x_mn, x, dtype, D, B, H, 32, 32, mn))) return rc;
    if ((rc = encode3d(&tm32.do_k, dO, dtype, D, B, H, 32, 32))) return rc;
    if ((rc = encode3d(&tm32.do_mn, dO, dtype, D, B, H, 32, 32, mn))) return rc;
    if ((rc = encode3d(&tm32.w1_k, w1, dtype, E, D, H, 32, a.dp))) return rc;
    if ((rc = encode3d(&tm32.w1_mn, w1, dtype, E, D, H, 32, a.dp, mn))) return rc;
    if ((rc = encode3d(&tm32.w2_k, w2, dtype, D, E, H, 32, 32))) return rc;
    if (plan.dz) {  // the dZ workspace (H, nB*128, nE*128) fp32, read K-major by the dX GEMM
      const uint64_t bp = uint64_t((B + kRows - 1) / kRows) * kRows, ep = uint64_t((E + kBwdEt - 1) / kBwdEt) * kBwdEt;
      if ((rc = encode3d(&tm32.dz, workspace, dtype, ep, bp, H, 32, kRows))) return rc;
    }
    a.tf32_maps = &tm32;
  } else {
    if ((rc = encode3d(&a.tm_x, x, dtype, D, B, hx, inner, rows))) return rc;
    if ((rc = encode3d(&a.tm_do, dO, dtype, D, B, hx, inner, rows))) return rc;
    if ((rc = encode3d(&a.tm_w1, w1, dtype, E, D, H, inner, a.dp))) return rc;
    if ((rc = encode3d(&a.tm_w2, w2, dtype, D, E, H, inner, rows))) return rc;
  }
  a.f32 = f32;
  a.x = x, a.w1 = w1;
  a.dx = dx, a.dw1 = dw1, a.dw2 = dw2;
  a.dw_f32 = dwf;
  a.splits = plan.splits;
  a.dzt = plan.dz ? workspace : nullptr;
  a.part = plan.splits > 1 ? reinterpret_cast<float*>(static_cast<char*>(workspace) + plan.dz_bytes) : nullptr;
  a.sm_count = dev->sm_count;
  a.H = H, a.B = B, a.D = D, a.E = E;
  a.bf16 = bf;
  a.act = act;
  a.shared_x = shared_x;
  a.status = dev->status;
  a.stream = st;
  return cuda_rc(f32 ? launch_bwd_tf32(a) : launch_bwd(a));
}

// Shared body of fmlp_bwd (dW rounded into dw1/dw2) and fmlp_bwd_dw_f32 (dW as unrounded
// fp32 into dwf = dW1 (H,D,E) followed by dW2 (H,E,D)).
int bwd_impl(const void* x, const void* w1, const void* w2, const void* dO, void* dx, void* dw1, void* dw2,
             float* dwf, void* workspace, size_t workspace_bytes, int H, int B, int D, int E, int dtype, int act,
             int shared_x, void* stream, bool allow_dz = true) {
  int rc = check_common(H, B, D, E, dtype);
  if (rc) return rc;
  const bool f32 = dtype == FMLP_DTYPE_F32;
  if (f32 && shared_x) return FMLP_ERR_UNSUPPORTED_DTYPE;
  if (D % 16 != 0 || D > (shared_x || f32 ? 128 : 256)) return FMLP_ERR_UNSUPPORTED_D;
  if (E % 8 != 0) return FMLP_ERR_UNSUPPORTED_E;
  if (shared_x && H == 0) return FMLP_ERR_INVALID_SHAPE;
  DeviceInfo* dev = nullptr;
  if ((rc = device_info(&dev))) return rc;
  // dZ-store mode when the workspace holds dZ^T (the size fmlp_bwd_workspace_size asks
  // for); otherwise the dX programs recompute Z and dH
  BwdPlan plan;
  if ((rc = plan_bwd(H, B, D, E, f32, allow_dz, !shared_x && dwf == nullptr, dev->sm_count, workspace_bytes,
                     workspace != nullptr && aligned16(workspace), &plan)))
    return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (H == 0 || D == 0) return FMLP_OK;
  const size_t esz = elem_bytes(dtype);
  if (E == 0) return cuda_rc(cudaMemsetAsync(dx, 0, size_t(shared_x ? 1 : H) * B * D * esz, st));
  if (B == 0) {
    if (dwf) return cuda_rc(cudaMemsetAsync(dwf, 0, size_t(2) * H * D * E * sizeof(float), st));
    if ((rc = cuda_rc(cudaMemsetAsync(dw1, 0, size_t(H) * D * E * esz, st)))) return rc;
    return cuda_rc(cudaMemsetAsync(dw2, 0, size_t(H) * E * D * esz, st));
  }
  if (!aligned16(x) || !aligned16(w1) || !aligned16(w2) || !aligned16(dO) || !aligned16(dx))
    return FMLP_ERR_MISALIGNED;
  if (dwf ? !aligned16(dwf) : (!aligned16(dw1) || !aligned16(dw2))) return FMLP_ERR_MISALIGNED;
  // one launch sequence per head group (one group unless the dZ-store mode runs in groups)
  const int G = plan.group > 0 ? plan.group : H;
  for (int g0 = 0; g0 < H; g0 += G) {
    const int Hg = H - g0 < G ? H - g0 : G;
    const size_t xo = shared_x ? 0 : size_t(g0) * B * D * esz, wo = size_t(g0) * D * E * esz;
    rc = bwd_launch_group(static_cast<const char*>(x) + xo, static_cast<const char*>(w1) + wo,
                          static_cast<const char*>(w2) + wo, static_cast<const char*>(dO) + xo,
                          static_cast<char*>(dx) + xo, dw1 ? static_cast<char*>(dw1) + wo : nullptr,
                          dw2 ? static_cast<char*>(dw2) + wo : nullptr, dwf, workspace, plan, Hg, B, D, E, dtype,
                          act, shared_x, dev, st);
    if (rc) return rc;
  }
  return FMLP_OK;
}

}  // namespace

extern "C" {

int fmlp_bwd(const void* x, const void* w1, const void* w2, const void* dO, void* dx, void* dw1,
             void* dw2, void* workspace, size_t workspace_bytes, int H, int B, int D, int E,
             int dtype, int act, void* stream) {
  return bwd_impl(x, w1, w2, dO, dx, dw1, dw2, nullptr, workspace, workspace_bytes, H, B, D, E, dtype, act, 0,
                  stream);
}

}  // extern "C"

namespace fmlp {
int bwd_entry(const void* x, const void* w1, const void* w2, const void* dO, void* dx, void* dw1, void* dw2,
              void* workspace, size_t workspace_bytes, int H, int B, int D, int E, int dtype, int act,
              void* stream, int allow_dz) {
  return bwd_impl(x, w1, w2, dO, dx, dw1, dw2, nullptr, workspace, workspace_bytes, H, B, D, E, dtype, act, 0,
                  stream, allow_dz != 0);
}
}  // namespace fmlp

extern "C" {

int fmlp_bwd_shared_x(const void* x, const void* w1, const void* w2, const void* dO, void* dx, void* dw1,
                      void* dw2, void* workspace, size_t workspace_bytes, int H, int B, int D, int E, int dtype,
                      int act, void* stream) {
  return bwd_impl(x, w1, w2, dO, dx, dw1, dw2, nullptr, workspace, workspace_bytes, H, B, D, E, dtype, act, 1,
                  stream);
}

int fmlp_bwd_dw_f32(const void* x, const void* w1, const void* w2, const void* dO, void* dx, float* dw_f32,
                    void* workspace, size_t workspace_bytes, int H, int B, int D, int E, int dtype, int act,
                    void* stream) {
  return bwd_impl(x, w1, w2, dO, dx, nullptr, nullptr, dw_f32, workspace, workspace_bytes, H, B, D, E, dtype,
                  act, 0, stream);
}

int fmlp_sgd_update(void* w, const float* g, long long n, float lr, int dtype, void* stream) {
  if (n < 0) return FMLP_ERR_INVALID_SHAPE;
  if (dtype != FMLP_DTYPE_F16 && dtype != FMLP_DTYPE_BF16) return FMLP_ERR_UNSUPPORTED_DTYPE;
  DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  if (n == 0) return FMLP_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  long long blocks = (n + 255) / 256;
  const long long cap = (long long)dev->sm_count * 8;
  if (blocks > cap) blocks = cap;
  if (dtype == FMLP_DTYPE_BF16)
    sgd_kernel_bf16<<<unsigned(blocks), 256, 0, st>>>(static_cast<__nv_bfloat16*>(w), g, n, lr);
  else
    sgd_kernel_f16<<<unsigned(blocks), 256, 0, st>>>(static_cast<__half*>(w), g, n, lr);
  return cuda_rc(cudaGetLastError());
}

int fmlp_device_status(int reset) {
  DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  if (cudaDeviceSynchronize() != cudaSuccess) return FMLP_ERR_CUDA;
  uint32_t v = 0;
  if (cudaMemcpy(&v, dev->status, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return FMLP_ERR_CUDA;
  if (reset) {
    const uint32_t z = 0;
    if (cudaMemcpy(dev->status, &z, sizeof(z), cudaMemcpyHostToDevice) != cudaSuccess) return FMLP_ERR_CUDA;
  }
  return v ? FMLP_ERR_DEVICE_TIMEOUT : FMLP_OK;
}

}  // extern "C"
