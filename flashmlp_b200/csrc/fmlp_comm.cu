// Fused gradient all-reduce + SGD for the batch-sharded training step, over NVLink peer
// memory (one process per GPU; buffers mapped into every rank with CUDA IPC).
//
// The reference has no multi-GPU path; its batch-sharded use would be an NCCL all-reduce
// of dW1 || dW2 followed by an optimizer step. Here one launch sequence does both, reading
// and writing the other GPUs' memory directly:
//
//   barrier(e)      every rank's fp32 gradient buffer is complete (its backward finished)
//   reduce + SGD    rank r owns slice r of the n weights (shard_range over 4-element
//                   groups): g = g_0 + g_1 + ... + g_{N-1} in that fixed rank order (fp32,
//                   read over NVLink), w = round(w - lr * g), and the new w is stored into
//                   every rank's replica (peer stores)
//   barrier(e + 1)  every slice of every replica is written
//
// Each element is summed once, by one rank, in a fixed order, and copied to all replicas,
// so the replicas are bit-identical and the result does not depend on timing. NVLink
// traffic per rank: (N-1)/N * n * 4 bytes read and (N-1)/N * n * 2 bytes written.
//
// The barriers are epoch counters: rank r writes the call's epoch into slot r of every
// rank's flag array (st.release.sys) and waits until each slot of its own array has
// reached it (ld.acquire.sys). Every wait is bounded (FMLP_WAIT_LIMIT_NS).
//
// Failure: a rank whose wait runs out (a peer never arrived) or that sees a peer's abort
// mark gives up. It writes a nonzero abort mark into its own abort slot of every rank's
// flag array, records the reason in its own call-status word, skips its reduce slice and
// publishes no further epoch. The abort marks are sticky: a peer that arrives late, or
// calls again, finds the mark before it waits, fails at once with FMLP_ERR_PEER_ABORT and
// touches no peer memory. So a call that returns a clean call status on a rank was
// completed by every rank: each rank published epoch + 1 only after its own first barrier
// passed and its slice was written. The call status belongs to the call (the first
// barrier resets it); the device-wide status word of other kernels is not consulted, so
// a timeout elsewhere in the process does not stop a later reduction. A group with an
// abort mark set must be rebuilt (fresh, zeroed flag arrays); every rank should stop.
// Only plain peer loads and stores are used (no multicast).
#include <cuda_runtime.h>

#include <cstring>

#include "../../include/flashmlp_b200.h"
#include "fmlp_kernels.h"
#include "fmlp_ptx.cuh"

namespace fmlp {
namespace {

static_assert(FMLP_PEER_STATUS_WORD >= 2 * FMLP_MAX_PEERS && FMLP_PEER_STATUS_WORD < FMLP_PEER_FLAG_WORDS,
              "flag array: epoch slots, abort slots, then the call status");

struct PeerSet {
  void* p[FMLP_MAX_PEERS];
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t* flag_words(const PeerSet& f, int k) { return static_cast<uint32_t*>(f.p[k]); }

// One warp, lane k < world speaks for rank k. `first`: the call's first barrier, which
// starts the call status afresh; the second one keeps the first one's verdict.
//   clean so far: publish `epoch` in slot `rank` of every rank's epoch slots, then wait
//     until every epoch slot of this rank's array has reached `epoch` (wrap-safe), an
//     abort mark appears, or the wait limit passes;
//   failed (now or before): publish this rank's abort mark in every rank's array.
__global__ void fmlp_peer_barrier_kernel(PeerSet flags, int world, int rank, uint32_t epoch, int first,
                                         uint32_t* dev_status) {
  const int k = threadIdx.x;
  uint32_t* own = flag_words(flags, rank);
  volatile uint32_t* call_status = own + FMLP_PEER_STATUS_WORD;
  uint32_t st = first ? 0u : *call_status;
  const bool marked = k < world && ld_acquire_sys(own + FMLP_MAX_PEERS + k) != 0u;
  if (__any_sync(0xffffffffu, marked) && st == 0u) st = FMLP_ERR_PEER_ABORT;
  if (st == 0u) {
    if (k < world) {
      __threadfence_system();  // this GPU's earlier writes to peers are visible first
      st_release_sys(flag_words(flags, k) + rank, epoch);
    }
    __syncwarp();
    bool done = k >= world, timed_out = false, aborted = false;
    const uint64_t t0 = global_timer_ns();
    while (!__all_sync(0xffffffffu, done)) {
      if (!done) {
        if (ld_acquire_sys(own + FMLP_MAX_PEERS + k) != 0u) {
          aborted = done = true;
        } else if (static_cast<int32_t>(ld_acquire_sys(own + k) - epoch) >= 0) {
          done = true;
        } else if (global_timer_ns() - t0 > FMLP_WAIT_LIMIT_NS) {
          timed_out = done = true;
        } else {
          __nanosleep(64);
        }
      }
    }
    if (__any_sync(0xffffffffu, timed_out))
      st = FMLP_ERR_DEVICE_TIMEOUT;
    else if (__any_sync(0xffffffffu, aborted))
      st = FMLP_ERR_PEER_ABORT;
  }
  if (st != 0u) {
    if (k < world) st_release_sys(flag_words(flags, k) + FMLP_MAX_PEERS + rank, 1u);
    if (k == 0 && st == FMLP_ERR_DEVICE_TIMEOUT) atomicOr(dev_status, kDevTimeout);
  }
  if (k == 0) *call_status = st;
}

// Slice [lo4, hi4) of 4-element groups: fixed-order fp32 sum of every rank's gradient,
// SGD step on this rank's replica, new values stored to every replica.
template <typename T>
__global__ void __launch_bounds__(256)
    fmlp_allreduce_sgd_kernel(PeerSet w, PeerSet g, int world, int rank, long long lo4, long long hi4, float lr,
                              const uint32_t* call_status) {
  // The call's first barrier failed (a rank did not arrive or gave up): touch no peer memory.
  if (*reinterpret_cast<const volatile uint32_t*>(call_status) != 0u) return;
  const uint2* wl = static_cast<const uint2*>(w.p[rank]);
  for (long long i = lo4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < hi4;
       i += (long long)gridDim.x * blockDim.x) {
    float4 acc = __ldcg(static_cast<const float4*>(g.p[0]) + i);
    for (int k = 1; k < world; ++k) {
      const float4 v = __ldcg(static_cast<const float4*>(g.p[k]) + i);
      acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
    }
    const uint2 wv = __ldcg(wl + i);
    // w - lr * g with two roundings (no FMA contraction), as fmlp_sgd_update computes it
    const float n0 = __fsub_rn(Pack<T>::lo(wv.x), __fmul_rn(lr, acc.x));
    const float n1 = __fsub_rn(Pack<T>::hi(wv.x), __fmul_rn(lr, acc.y));
    const float n2 = __fsub_rn(Pack<T>::lo(wv.y), __fmul_rn(lr, acc.z));
    const float n3 = __fsub_rn(Pack<T>::hi(wv.y), __fmul_rn(lr, acc.w));
    const uint2 out = make_uint2(Pack<T>::pack(n0, n1), Pack<T>::pack(n2, n3));
    for (int k = 0; k < world; ++k) static_cast<uint2*>(w.p[k])[i] = out;
  }
  __threadfence_system();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace fmlp

using namespace fmlp;

extern "C" {

int fmlp_peer_alloc(size_t bytes, void** dev_ptr) {
  if (dev_ptr == nullptr) return FMLP_ERR_INVALID_SHAPE;
  *dev_ptr = nullptr;
  if (bytes == 0) return FMLP_ERR_INVALID_SHAPE;
  if (cudaMalloc(dev_ptr, bytes) != cudaSuccess) return FMLP_ERR_CUDA;
  if (cudaMemset(*dev_ptr, 0, bytes) != cudaSuccess) return FMLP_ERR_CUDA;
  return FMLP_OK;
}

int fmlp_peer_free(void* dev_ptr) { return cudaFree(dev_ptr) == cudaSuccess ? FMLP_OK : FMLP_ERR_CUDA; }

int fmlp_ipc_get_handle(const void* dev_ptr, void* handle) {
  if (dev_ptr == nullptr || handle == nullptr) return FMLP_ERR_INVALID_SHAPE;
  static_assert(sizeof(cudaIpcMemHandle_t) == FMLP_IPC_HANDLE_BYTES, "handle size");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)) != cudaSuccess) return FMLP_ERR_CUDA;
  memcpy(handle, &h, sizeof(h));
  return FMLP_OK;
}

int fmlp_ipc_open_handle(const void* handle, void** dev_ptr) {
  if (dev_ptr == nullptr || handle == nullptr) return FMLP_ERR_INVALID_SHAPE;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *dev_ptr = nullptr;
  if (cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return FMLP_ERR_CUDA;
  return FMLP_OK;
}

int fmlp_ipc_close_handle(void* dev_ptr) {
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? FMLP_OK : FMLP_ERR_CUDA;
}

int fmlp_grad_allreduce_sgd(void* const* peer_w, const float* const* peer_g, uint32_t* const* peer_flags,
                            int world, int rank, long long n, float lr, int dtype, unsigned epoch, void* stream) {
  if (world < 1 || world > FMLP_MAX_PEERS || rank < 0 || rank >= world) return FMLP_ERR_INVALID_SHAPE;
  if (n < 0 || n % 4 != 0) return FMLP_ERR_INVALID_SHAPE;
  if (dtype != FMLP_DTYPE_F16 && dtype != FMLP_DTYPE_BF16) return FMLP_ERR_UNSUPPORTED_DTYPE;
  if (peer_w == nullptr || peer_g == nullptr || peer_flags == nullptr) return FMLP_ERR_INVALID_SHAPE;
  PeerSet w{}, g{}, f{};
  for (int k = 0; k < world; ++k) {
    if (!aligned16(peer_w[k]) || !aligned16(peer_g[k]) || peer_flags[k] == nullptr || peer_w[k] == nullptr ||
        peer_g[k] == nullptr)
      return FMLP_ERR_MISALIGNED;
    w.p[k] = peer_w[k];
    g.p[k] = const_cast<float*>(peer_g[k]);
    f.p[k] = peer_flags[k];
  }
  int sm_count = 0;
  uint32_t* status = nullptr;
  int rc = current_device_status(&sm_count, &status);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // this rank's slice of the n / 4 groups: the first (n/4) % world ranks get one extra
  const long long n4 = n / 4, base = n4 / world, extra = n4 % world;
  const long long lo4 = rank * base + (rank < extra ? rank : extra);
  const long long hi4 = lo4 + base + (rank < extra ? 1 : 0);
  const uint32_t* call_status = static_cast<const uint32_t*>(f.p[rank]) + FMLP_PEER_STATUS_WORD;
  fmlp_peer_barrier_kernel<<<1, 32, 0, st>>>(f, world, rank, epoch, 1, status);
  if (cudaGetLastError() != cudaSuccess) return FMLP_ERR_CUDA;
  if (hi4 > lo4) {
    long long blocks = (hi4 - lo4 + 255) / 256;
    const long long cap = (long long)sm_count * 4;
    if (blocks > cap) blocks = cap;
    if (dtype == FMLP_DTYPE_BF16)
      fmlp_allreduce_sgd_kernel<__nv_bfloat16><<<unsigned(blocks), 256, 0, st>>>(w, g, world, rank, lo4, hi4, lr,
                                                                                  call_status);
    else
      fmlp_allreduce_sgd_kernel<__half><<<unsigned(blocks), 256, 0, st>>>(w, g, world, rank, lo4, hi4, lr,
                                                                         call_status);
    if (cudaGetLastError() != cudaSuccess) return FMLP_ERR_CUDA;
  }
  fmlp_peer_barrier_kernel<<<1, 32, 0, st>>>(f, world, rank, epoch + 1u, 0, status);
  if (cudaGetLastError() != cudaSuccess) return FMLP_ERR_CUDA;
  return FMLP_OK;
}

}  // extern "C"
