// fmlp_bwd_noalloc: the unified backward for callers that cannot allocate device memory.
//
// Some hosts of this kernel own every byte of device memory themselves: an inference or
// training engine whose memory planner hands each custom operator only its input and
// output buffers and forbids allocation inside the operator, or a process whose caching
// allocator already holds nearly all of HBM, so that a cudaMalloc from a library would
// fail or fragment its pool. Such callers cannot provide the fp32 workspace fmlp_bwd asks
// for when it splits its dW programs over B ranges (launches with few (head, E chunk)
// pairs, e.g. 4 heads with E = 2048 on a 148-SM B200). This entry point takes the same
// inputs and outputs as fmlp_bwd but keeps that scratch in a fixed, file-scope device
// array instead of a caller allocation.
//
// The array is kNoAllocScratchBytes (32 MiB) on every GPU that loads the library, held
// until the process exits. With D <= 128 the split rule needs at most about 28 MB on a
// 148-SM GPU, and shapes that do not split need none; a shape that would need more is
// rejected with FMLP_ERR_SCRATCH_LIMIT.
//
// All calls on one device share the one array, and it keeps whatever the last call left
// in it. Nothing in it has to start at zero: every partial sum the reduction reads is
// written earlier in the same call. Two calls whose kernels overlap on the GPU (e.g. on
// two streams of one device) race on the array and corrupt each other's dW; serialise
// them.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/flashmlp_b200.h"
#include "fmlp_kernels.h"

namespace fmlp {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // FMLP_NOALLOC_SCRATCH_BYTES

__device__ __align__(256) float g_fmlp_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch[kMaxDevices] = {};      // device address of the array, per device
void* g_scratch_ctx[kMaxDevices] = {};  // the context that address belongs to

// Device address of this device's copy of the array. In host code the array's name only
// stands in for the symbol; a kernel given it would read host memory or fault, so the
// address comes from cudaGetSymbolAddress, once per device and context, with that device
// current. A new context on the device (after cudaDeviceReset) gets a new array, whose
// address is looked up again.
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return FMLP_ERR_CUDA;
  void* ctx = current_context();
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch[dev] == nullptr || g_scratch_ctx[dev] != ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fmlp_noalloc_scratch) != cudaSuccess || p == nullptr)
      return FMLP_ERR_CUDA;
    g_scratch[dev] = p;
    g_scratch_ctx[dev] = current_context();  // the symbol lookup made the context current
  }
  *out = g_scratch[dev];
  return FMLP_OK;
}

}  // namespace
}  // namespace fmlp

extern "C" int fmlp_bwd_noalloc(const void* x, const void* w1, const void* w2, const void* dO,
                                void* dx, void* dw1, void* dw2, int H, int B, int D, int E,
                                int dtype, int act, void* stream) {
  static_assert(fmlp::kNoAllocScratchBytes == FMLP_NOALLOC_SCRATCH_BYTES, "header and array agree");
  const size_t need = fmlp_bwd_workspace_size_min(H, B, D, E, dtype);
  if (need > fmlp::kNoAllocScratchBytes) return FMLP_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = fmlp::scratch_for_current_device(&scratch);
    if (rc) return rc;
  }
  return fmlp::bwd_entry(x, w1, w2, dO, dx, dw1, dw2, scratch, need > 0 ? fmlp::kNoAllocScratchBytes : 0, H, B,
                         D, E, dtype, act, stream, 0);
}
