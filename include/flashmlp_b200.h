/*
 * flashmlp_b200 — C ABI of the B200 (sm_100a) fused multi-head MLP.
 *
 *   O[h] = act(X[h] @ W1[h]) @ W2[h]          X, O: (H,B,D)  W1: (H,D,E)  W2: (H,E,D)
 *
 * These entry points are the drop-in boundary for the two Triton launches of the
 * reference (dtadpole/flashMLP, flashmlp.py): every argument is a plain pointer or size,
 * all pointers are DEVICE pointers to contiguous row-major tensors with exactly the
 * reference's layouts, and the caller owns every allocation. Work is enqueued
 * asynchronously on `stream` (a cudaStream_t; NULL = legacy default stream) of the
 * current device. Every function returns 0 on success or one of the FMLP_ERR_* codes.
 */
#ifndef FLASHMLP_B200_H_
#define FLASHMLP_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes */
#define FMLP_DTYPE_F16 0
#define FMLP_DTYPE_BF16 1
#define FMLP_DTYPE_F32 2 /* fp32 in and out, TF32 tensor-core products (the reference's fp32
                            path: tl.dot on fp32 tensors); fmlp_fwd / fmlp_bwd /
                            fmlp_bwd_dw_f32 with D <= 128 */

/* activation codes; the reference treats any unknown activation string as linear
 * (flashmlp.py:146-147, :682-683) and so does the Python layer of this library. */
#define FMLP_ACT_LINEAR 0
#define FMLP_ACT_LEAKY_RELU 1 /* slope 0.01, z >= 0 takes the identity branch */
#define FMLP_ACT_SILU 2
#define FMLP_ACT_SIGMOID 3

/* error codes */
#define FMLP_OK 0
#define FMLP_ERR_INVALID_SHAPE 1    /* negative size or size overflow                  */
#define FMLP_ERR_UNSUPPORTED_DTYPE 2 /* fp16, bf16; fp32 only where noted           */
#define FMLP_ERR_UNSUPPORTED_D 3    /* D % 16 != 0, or D > 256 (> 128: fp32, shared x)  */
#define FMLP_ERR_UNSUPPORTED_E 4    /* E % 8 != 0 (row stride of W1 must be 16 bytes)  */
#define FMLP_ERR_MISALIGNED 5       /* a pointer is not 16-byte aligned                */
#define FMLP_ERR_CUDA 6             /* CUDA runtime / launch error                     */
#define FMLP_ERR_TMA 7              /* tensor-map encoding failed                      */
#define FMLP_ERR_DEVICE 8           /* current device is not an sm_100 (B200) GPU       */
#define FMLP_ERR_WORKSPACE 9        /* workspace smaller than fmlp_bwd_workspace_size,
                                       null or not 16-byte aligned                     */
#define FMLP_ERR_DEVICE_TIMEOUT 10  /* a kernel's bounded pipeline wait ran out        */
#define FMLP_ERR_SCRATCH_LIMIT 11   /* fmlp_bwd_noalloc: shape needs more scratch than
                                       FMLP_NOALLOC_SCRATCH_BYTES                      */
#define FMLP_ERR_PEER_ABORT 12      /* fmlp_grad_allreduce_sgd: a rank of the group gave
                                       up on a barrier (now or in an earlier call)     */
#define FMLP_ERR_INVALID_SCALE 13   /* fmlp_fwd_fp8: a scale is not finite and > 0      */

/*
 * Forward. Replaces flashmlp_fwd + flashmlp_fwd_kernel (flashmlp.py:428-477, :63-158).
 * o (H,B,D) is fully written (the reference zero-fills it first, flashmlp.py:462).
 */
int fmlp_fwd(const void* x, const void* w1, const void* w2, void* o, int H, int B, int D, int E,
             int dtype, int act, void* stream);

/*
 * Unified backward. Replaces flashmlp_bwd + flashmlp_bwd_kernel (flashmlp.py:480-538,
 * :341-421). dO must be contiguous (the reference makes it so, flashmlp.py:508).
 * dx (H,B,D), dw1 (H,D,E) and dw2 (H,E,D) are fully written. `workspace` is device
 * scratch of at least fmlp_bwd_workspace_size(...) bytes (may be NULL when that is 0).
 */
int fmlp_bwd(const void* x, const void* w1, const void* w2, const void* dO, void* dx, void* dw1,
             void* dw2, void* workspace, size_t workspace_bytes, int H, int B, int D, int E,
             int dtype, int act, void* stream);

/*
 * Shared-input forward: x is ONE (B,D) matrix used by every head and o (B,D) receives the
 * mean over heads, o = (1/H) * sum_h act(x @ W1[h]) @ W2[h]. This is what the reference's
 * FlashMLP.forward computes for a 2-D input (flashmlp.py:603-614: x expanded to (H,B,D),
 * FlashMLPFunction, o.mean(0)) without materialising the H copies of x and of o; the head
 * sum is accumulated in fp32 and rounded once. Needs H >= 1 and D <= 128.
 */
int fmlp_fwd_shared_x(const void* x, const void* w1, const void* w2, void* o, int H, int B, int D,
                      int E, int dtype, int act, void* stream);

/*
 * FP8 (e4m3) forward with per-tensor scales. No counterpart in the reference, which has
 * 16-bit and fp32 paths only; it is the forward of fmlp_fwd with 8-bit operands:
 *   Z  = (x @ W1) * x_scale * w1_scale                 fp32 accumulation
 *   H8 = e4m3(act(Z) / h_scale)                        round to nearest even, saturating
 *   o  = (H8 @ W2) * h_scale * w2_scale                rounded to out_dtype (F16 / BF16)
 * x (H,B,D) holds e4m3 bytes; the weights come TRANSPOSED, w1t (H,E,D) = W1^T and
 * w2t (H,D,E) = W2^T, also e4m3 bytes (prepare them once per weight update); o (H,B,D)
 * in out_dtype is fully written. Needs D % 16 == 0, D <= 128, E % 16 == 0, 16-byte
 * aligned pointers and finite positive scales.
 */
int fmlp_fwd_fp8(const void* x, const void* w1t, const void* w2t, void* o, int H, int B, int D, int E,
                 float x_scale, float w1_scale, float w2_scale, float h_scale, int act, int out_dtype,
                 void* stream);

/*
 * Backward of fmlp_fwd_shared_x: dO (B,D) is the gradient of the head mean, dx (B,D) the
 * gradient of the shared input (summed over heads, as the expand's backward does), dw1
 * (H,D,E) and dw2 (H,E,D) per head. Workspace as for fmlp_bwd (fmlp_bwd_workspace_size
 * with the same H, B, D, E). Needs H >= 1 and D <= 128.
 */
int fmlp_bwd_shared_x(const void* x, const void* w1, const void* w2, const void* dO, void* dx,
                      void* dw1, void* dw2, void* workspace, size_t workspace_bytes, int H, int B,
                      int D, int E, int dtype, int act, void* stream);

/*
 * The same backward with dW left as unrounded fp32 sums over this call's B rows:
 * dw_f32 holds dW1 laid out (H,D,E) followed by dW2 laid out (H,E,D), 2*H*D*E floats.
 * dx is written as in fmlp_bwd; the workspace rule is fmlp_bwd's. Used by the batch-
 * sharded step, whose ranks add their fp32 partials before rounding (no reference
 * counterpart: flashmlp.py:480-538 returns dW in the input dtype).
 */
int fmlp_bwd_dw_f32(const void* x, const void* w1, const void* w2, const void* dO, void* dx,
                    float* dw_f32, void* workspace, size_t workspace_bytes, int H, int B, int D,
                    int E, int dtype, int act, void* stream);

/* Device scratch bytes for fmlp_bwd on the current device (no reference counterpart; the
 * reference allocates its outputs with torch.zeros_like, flashmlp.py:516-518).
 *
 * fmlp_bwd_workspace_size: the workspace of the fastest mode. For 16-bit inputs with
 * D <= 256 and fp32 inputs with D <= 128 that is the dZ-store mode: the dW programs also
 * store their dZ (H * ceil(E/128)*128 * ceil(B/128)*128 values of the input dtype, at
 * most 8 GiB) and dX becomes a GEMM over E of those values instead of programs that
 * recompute Z and dH; for 128 < D <= 256 they also store H = act(Z) (as many values),
 * from which with dZ a GEMM over B forms the second half of dW's D columns; plus the fp32
 * dW partial sums below when that launch splits its dW programs.
 *
 * fmlp_bwd_workspace_size_min: the least workspace fmlp_bwd accepts (the recompute mode).
 * Nonzero only when the launch has too few (head, E chunk) pairs to fill the GPU (e.g. 4
 * heads with E = 2048 on a 148-SM B200): the dW programs are then split over B ranges and
 * their fp32 partial sums (2 * splits * H * D * E floats) are added in a fixed order by a
 * second kernel.
 *
 * fmlp_bwd picks the dZ-store mode when workspace_bytes >= fmlp_bwd_workspace_size and
 * the mode applies, otherwise the recompute mode. Both return 0 for invalid arguments. */
size_t fmlp_bwd_workspace_size(int H, int B, int D, int E, int dtype);
size_t fmlp_bwd_workspace_size_min(int H, int B, int D, int E, int dtype);

/* What fmlp_bwd runs for this shape and workspace size on the current device (no reference
 * counterpart): *mode 1 = dZ-store mode, 0 = recompute mode; *splits = dW programs per
 * (head, E chunk); *launches = kernels per call (the backward kernel, the dX GEMM in the
 * dZ-store mode, the dW partial reduction when *splits > 1). Any output may be NULL.
 * Returns FMLP_ERR_WORKSPACE when workspace_bytes is below fmlp_bwd_workspace_size_min. */
int fmlp_bwd_plan(int H, int B, int D, int E, int dtype, size_t workspace_bytes, int* mode, int* splits,
                  int* launches);

/*
 * Unified backward that allocates nothing: same arguments and results as fmlp_bwd, minus
 * the workspace. No counterpart in the reference. It is for callers that cannot allocate
 * device memory: engines whose memory planner gives a custom operator only its inputs and
 * outputs, or processes whose allocator already holds the GPU's memory. The fp32 dW
 * partial sums that fmlp_bwd keeps in the caller's workspace live instead in a static
 * device array of FMLP_NOALLOC_SCRATCH_BYTES, which every GPU that loads the library holds
 * until the process exits; a shape whose fmlp_bwd_workspace_size_min exceeds it returns
 * FMLP_ERR_SCRATCH_LIMIT (no D <= 256 shape does on a 148-SM B200). It always runs the
 * recompute mode (dX programs recompute Z and dH), never the dZ-store mode.
 * The first call on a device whose shape needs scratch looks up the array's device
 * address (cudaGetSymbolAddress); make that first call before any stream capture on the
 * device. All calls on a device share the array: calls whose kernels overlap on the GPU
 * (e.g. on two streams) race on it, so serialise them. It calls no cudaMalloc/cudaFree.
 */
#define FMLP_NOALLOC_SCRATCH_BYTES (32u << 20)
int fmlp_bwd_noalloc(const void* x, const void* w1, const void* w2, const void* dO, void* dx,
                     void* dw1, void* dw2, int H, int B, int D, int E, int dtype, int act,
                     void* stream);

/*
 * In-place SGD step w[i] -= lr * g[i] for n elements, g in fp32 (e.g. the all-reduced
 * sum of dW shards) and w in `dtype`. Used by the batch-sharded multi-GPU training step;
 * the reference has no optimizer (no counterpart).
 */
int fmlp_sgd_update(void* w, const float* g, long long n, float lr, int dtype, void* stream);

/*
 * Fused gradient all-reduce + SGD of the batch-sharded training step over NVLink peer
 * memory; no reference counterpart (it replaces an NCCL all-reduce of dW1 || dW2 followed
 * by fmlp_sgd_update). One process per GPU, world <= FMLP_MAX_PEERS ranks on distinct GPUs
 * of one node. peer_w[k] (n 16-bit weights, rank k's replica), peer_g[k] (n fp32
 * gradients of rank k's rows) and peer_flags[k] (FMLP_PEER_FLAG_WORDS uint32 words,
 * zero-initialised when the group is formed) are rank k's buffers as mapped into this
 * process (fmlp_ipc_open_handle; the own rank's entries are its plain device pointers);
 * the arrays themselves are host memory. Every rank calls with the same n, lr, dtype and
 * epoch, and a fresh epoch per call (two counter values are used per call: epoch and
 * epoch + 1). Rank r sums slice r of the gradients over ranks 0..world-1 in that order in
 * fp32, applies w = round(w - lr * g) and stores the result into every replica; barriers
 * before and after make every replica complete when the call's work on `stream` ends.
 * n % 4 == 0.
 *
 * Failure reporting: when the call's work on `stream` has ended, word
 * FMLP_PEER_STATUS_WORD of this rank's own flag array holds the call's status: FMLP_OK
 * (every rank completed the call), FMLP_ERR_DEVICE_TIMEOUT (a peer did not arrive within
 * the wait limit; also recorded in fmlp_device_status) or FMLP_ERR_PEER_ABORT (a rank
 * gave up, in this call or an earlier one). A rank that fails skips its slice and marks
 * the failure in every rank's flag array (words FMLP_MAX_PEERS..2*FMLP_MAX_PEERS-1), so
 * every later call of the group fails at once on every rank: all ranks should stop.
 */
#define FMLP_PEER_FLAG_WORDS 32
#define FMLP_PEER_STATUS_WORD 16
#define FMLP_MAX_PEERS 8
int fmlp_grad_allreduce_sgd(void* const* peer_w, const float* const* peer_g,
                            uint32_t* const* peer_flags, int world, int rank, long long n, float lr,
                            int dtype, unsigned epoch, void* stream);

/* CUDA IPC plumbing for the buffers above (no reference counterpart). fmlp_peer_alloc
 * returns a zeroed cudaMalloc allocation of its own, so its IPC handle maps exactly that
 * buffer; fmlp_ipc_get_handle writes FMLP_IPC_HANDLE_BYTES bytes that another process on
 * the same node passes to fmlp_ipc_open_handle to map the buffer. */
#define FMLP_IPC_HANDLE_BYTES 64
int fmlp_peer_alloc(size_t bytes, void** dev_ptr);
int fmlp_peer_free(void* dev_ptr);
int fmlp_ipc_get_handle(const void* dev_ptr, void* handle);
int fmlp_ipc_open_handle(const void* handle, void** dev_ptr);
int fmlp_ipc_close_handle(void* dev_ptr);

/* Reads the current device's kernel status word (FMLP_OK or FMLP_ERR_DEVICE_TIMEOUT),
 * optionally clearing it. Synchronises the device. */
int fmlp_device_status(int reset);

/* Static description of an error code. */
const char* fmlp_error_string(int code);

/* ABI version (major*100 + minor). */
int fmlp_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FLASHMLP_B200_H_ */
