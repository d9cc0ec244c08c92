"""Multi-GPU wrappers for the fused multi-head MLP (one process per GPU).

The reference has no multi-GPU code; these wrappers add the two ways the path shards:

* head-sharded: heads are independent, so rank r of n owns a contiguous block of heads
  (dim 0 of X, W1, W2, O) and runs the kernels on it with no communication;
* batch-sharded: rank r owns a contiguous block of batch rows (dim 1 of X and dO) and a
  replica of W1/W2. After the local backward, dW1 and dW2 are summed over ranks with
  one NCCL all-reduce (in fp32, over one flattened buffer) and every rank applies the
  same SGD step W <- W - lr * dW with the library's update kernel, so replicas stay equal
  (`batch_sharded_train_step`);
* batch-sharded, fused (`FusedBatchShardedTrainer`): the backward leaves dW as unrounded
  fp32 in a buffer every rank can read over NVLink, and one library call
  (fmlp_grad_allreduce_sgd) sums each weight's gradient over ranks in a fixed order,
  applies the SGD step and writes the new weight into every replica, in place of the
  copy, the NCCL all-reduce and the two update kernels.

Process-group plumbing is torch.distributed; compute is libflashmlp_b200.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .api import _dtype_code, flashmlp_bwd, flashmlp_bwd_dw_f32, flashmlp_fwd


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) block of n items for `rank` of `world`; the first
    n % world ranks get one extra item."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_heads(t: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    a, b = shard_range(t.shape[0], world, rank)
    return t[a:b].contiguous()


def shard_batch(t: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    a, b = shard_range(t.shape[1], world, rank)
    return t[:, a:b].contiguous()


def sgd_update_(w: torch.Tensor, g: torch.Tensor, lr: float) -> None:
    """In-place w -= lr * g on the GPU (g fp32, w bf16/fp16), via fmlp_sgd_update."""
    if w.device.type != "cuda" or g.device != w.device:
        raise RuntimeError("sgd_update_ needs CUDA tensors on one device")
    if g.dtype != torch.float32 or g.numel() != w.numel() or not (w.is_contiguous() and g.is_contiguous()):
        raise ValueError("g must be a contiguous fp32 tensor with w's number of elements")
    with torch.cuda.device(w.device):
        stream = torch.cuda.current_stream(w.device).cuda_stream
        rc = _lib.lib().fmlp_sgd_update(ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(g.data_ptr()),
                                        w.numel(), float(lr), _dtype_code(w), ctypes.c_void_p(stream))
    _lib.check(rc, "fmlp_sgd_update")


@dataclass
class Compute:
    """The per-rank compute used by the wrappers; tests substitute a CPU checker."""
    fwd: Callable = flashmlp_fwd
    bwd: Callable = flashmlp_bwd
    update: Callable = sgd_update_


def head_sharded_fwd_bwd(x, w1, w2, do, activation: str = "", compute: Optional[Compute] = None):
    """Forward + backward of this rank's heads. Inputs are the local head blocks (see
    shard_heads); returns (o, dx, dw1, dw2) for those heads. No communication."""
    c = compute or Compute()
    o = c.fwd(x, w1, w2, activation)
    dx, dw1, dw2 = c.bwd(x, w1, w2, do, activation)
    return o, dx, dw1, dw2


def gather_heads(local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gathers head blocks (possibly uneven) into the full (H, ...) tensor."""
    world = dist.get_world_size(group)
    n = torch.tensor([local.shape[0]], device=local.device)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(s.item()) for s in sizes]
    mx = max(sizes)
    pad = torch.zeros((mx,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[:s] for p, s in zip(parts, sizes)], dim=0)


def batch_sharded_train_step(x_local, do_local, w1, w2, activation: str = "", lr: float = 1e-3,
                             group=None, compute: Optional[Compute] = None):
    """One data-parallel training step on this rank's batch rows.

    x_local, do_local: (H, B_local, D); w1 (H, D, E), w2 (H, E, D) replicated and updated
    in place. Returns (o_local, dx_local, dw1_sum, dw2_sum) where dw*_sum are the fp32
    gradients summed over all ranks (the gradient of the full batch).
    """
    c = compute or Compute()
    o = c.fwd(x_local, w1, w2, activation)
    dx, dw1, dw2 = c.bwd(x_local, w1, w2, do_local, activation)
    n1 = dw1.numel()
    flat = torch.empty(n1 + dw2.numel(), dtype=torch.float32, device=dw1.device)
    flat[:n1].copy_(dw1.reshape(-1))
    flat[n1:].copy_(dw2.reshape(-1))
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    g1, g2 = flat[:n1], flat[n1:]
    c.update(w1, g1, lr)
    c.update(w2, g2, lr)
    return o, dx, g1.view(dw1.shape), g2.view(dw2.shape)


# ----------------------------------------------------------------------------- fused path
class _DeviceView:
    """Zero-copy torch view of raw device memory (via __cuda_array_interface__)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}


def _typestr(dtype: torch.dtype) -> str:
    return {torch.float32: "<f4", torch.float16: "<f2", torch.uint32: "<u4", torch.int32: "<i4",
            torch.bfloat16: "<V2"}[dtype]


class PeerBuffer:
    """One device buffer per rank, mapped into every rank's address space with CUDA IPC.

    `ptrs[k]` is rank k's buffer as this process addresses it (the own rank's entry is its
    plain device pointer). Ranks must sit on distinct GPUs of one node. Allocated with the
    library's own cudaMalloc (zeroed), so an IPC handle maps exactly this buffer."""

    def __init__(self, nbytes: int, group=None):
        L = _lib.lib()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nbytes = int(nbytes)
        p = ctypes.c_void_p()
        _lib.check(L.fmlp_peer_alloc(self.nbytes, ctypes.byref(p)), "fmlp_peer_alloc")
        self.local = p.value
        h = (ctypes.c_char * _lib.FMLP_IPC_HANDLE_BYTES)()
        _lib.check(L.fmlp_ipc_get_handle(ctypes.c_void_p(self.local), h), "fmlp_ipc_get_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(h), group=group)
        self.ptrs, self._opened = [], []
        for k, hk in enumerate(handles):
            if k == self.rank:
                self.ptrs.append(self.local)
                continue
            q = ctypes.c_void_p()
            buf = ctypes.create_string_buffer(hk, len(hk))
            _lib.check(L.fmlp_ipc_open_handle(buf, ctypes.byref(q)), "fmlp_ipc_open_handle")
            self.ptrs.append(q.value)
            self._opened.append(q.value)

    def view(self, offset: int, shape, dtype: torch.dtype, device) -> torch.Tensor:
        """Tensor view of this rank's buffer at byte `offset`."""
        n = 1
        for s_ in shape:
            n *= s_
        esz = torch.empty((), dtype=dtype).element_size()
        if offset < 0 or offset + n * esz > self.nbytes or offset % 16:
            raise ValueError("view outside the buffer or not 16-byte aligned")
        if dtype == torch.bfloat16:  # no typestr for bfloat16: view 16-bit words, reinterpret
            t = torch.as_tensor(_DeviceView(self.local + offset, shape, "<i2"), device=device)
            return t.view(torch.bfloat16)
        return torch.as_tensor(_DeviceView(self.local + offset, shape, _typestr(dtype)), device=device)

    def close(self):
        L = _lib.lib()
        for q in self._opened:
            L.fmlp_ipc_close_handle(ctypes.c_void_p(q))
        self._opened = []
        if self.local:
            L.fmlp_peer_free(ctypes.c_void_p(self.local))
            self.local = None


def _align16(n: int) -> int:
    return (n + 15) // 16 * 16


class FusedBatchShardedTrainer:
    """Batch-sharded (data-parallel) training step with the fused gradient all-reduce + SGD.

    Holds this rank's replica of W1 (H, D, E) and W2 (H, E, D) in peer-mapped memory:
    `w1` and `w2` are views of it, initialised from the given tensors (equal on every
    rank). `step(x_local, do_local, activation, lr)` runs the forward and the backward on
    this rank's rows, with dW as fp32 sums into the peer-mapped gradient buffer, then
    fmlp_grad_allreduce_sgd: every weight's gradient is summed over ranks 0..N-1 in that
    order in fp32, w = round(w - lr * g) is applied once and stored into every replica.
    All ranks must call `step` together (it contains two cross-GPU barriers). Unlike
    `batch_sharded_train_step`, the per-rank gradients are not rounded to 16 bits before
    they are added. Call `close()` on every rank before destroying the process group."""

    def __init__(self, w1: torch.Tensor, w2: torch.Tensor, group=None):
        if w1.device.type != "cuda" or w2.device != w1.device or w1.dtype != w2.dtype:
            raise RuntimeError("w1 and w2 must be CUDA tensors on one device with one dtype")
        self.dtype_code = _dtype_code(w1)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _lib.FMLP_MAX_PEERS:
            raise ValueError(f"at most {_lib.FMLP_MAX_PEERS} ranks (GPUs of one node)")
        dev = w1.device
        # every rank on its own GPU: kernels that wait on each other must not share one
        ids = [None] * self.world
        dist.all_gather_object(ids, str(torch.cuda.get_device_properties(dev).uuid), group=group)
        if len(set(ids)) != self.world:
            raise RuntimeError("FusedBatchShardedTrainer needs one GPU per rank")
        self.n1, self.n2 = w1.numel(), w2.numel()
        self.n = self.n1 + self.n2
        self.shape1, self.shape2 = tuple(w1.shape), tuple(w2.shape)
        self.device = dev
        with torch.cuda.device(dev):
            self._w = PeerBuffer(_align16(2 * self.n), group)
            self._g = PeerBuffer(_align16(4 * self.n), group)
            self._f = PeerBuffer(_align16(4 * _lib.FMLP_PEER_FLAG_WORDS), group)
        wflat = self._w.view(0, (self.n,), w1.dtype, dev)
        self.w1 = wflat[: self.n1].view(self.shape1)
        self.w2 = wflat[self.n1:].view(self.shape2)
        self.w1.copy_(w1)
        self.w2.copy_(w2)
        self.grad = self._g.view(0, (self.n,), torch.float32, dev)  # this rank's fp32 dW1 || dW2
        # this rank's flag array: epoch slots, abort marks, then the last call's status
        self.flags = self._f.view(0, (_lib.FMLP_PEER_FLAG_WORDS,), torch.int32, dev)
        self.epoch = 0
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)  # every rank's buffers and zeroed flags exist before any use

    def _ptr_array(self, ptrs):
        return (ctypes.c_void_p * len(ptrs))(*[ctypes.c_void_p(p) for p in ptrs])

    def allreduce_sgd_(self, lr: float) -> None:
        """Sums `grad` over ranks, applies the SGD step and refreshes every replica."""
        L = _lib.lib()
        self.epoch += 2
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            rc = L.fmlp_grad_allreduce_sgd(self._ptr_array(self._w.ptrs), self._ptr_array(self._g.ptrs),
                                           self._ptr_array(self._f.ptrs), self.world, self.rank, self.n,
                                           float(lr), self.dtype_code, (self.epoch - 1) & 0xFFFFFFFF,
                                           ctypes.c_void_p(stream))
        _lib.check(rc, "fmlp_grad_allreduce_sgd")

    def status(self) -> int:
        """Status of the last fused all-reduce call on this rank (waits for it to finish):
        FMLP_OK, FMLP_ERR_DEVICE_TIMEOUT (a peer did not arrive in time) or
        FMLP_ERR_PEER_ABORT (a rank gave up, in that call or an earlier one)."""
        torch.cuda.current_stream(self.device).synchronize()
        return int(self.flags[_lib.FMLP_PEER_STATUS_WORD].item())

    def check(self) -> None:
        """Raises FlashMLPError if the last fused all-reduce call failed on this rank. After
        a failure the group's flag arrays carry an abort mark and every later call fails on
        every rank: all ranks must stop (and rebuild the trainer to continue)."""
        _lib.check(self.status(), "fmlp_grad_allreduce_sgd (device status of the call)")

    def step(self, x_local, do_local, activation: str = "", lr: float = 1e-3, check: bool = True):
        """Forward + backward on this rank's rows, then the fused all-reduce + SGD.
        Returns (o_local, dx_local). With check=True (the default) it waits for the step
        and raises FlashMLPError if the all-reduce failed on any rank (a peer timed out or
        gave up); with check=False the caller calls check() later, e.g. once after a
        timed loop (a failure is sticky, so no failed step goes unnoticed)."""
        o = flashmlp_fwd(x_local, self.w1, self.w2, activation)
        dx, _ = flashmlp_bwd_dw_f32(x_local, self.w1, self.w2, do_local, activation, dw_out=self.grad)
        self.allreduce_sgd_(lr)
        if check:
            self.check()
        return o, dx

    def close(self):
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no rank still reads or writes a peer's buffers
        for b in (self._w, self._g, self._f):
            b.close()
