"""Multi-GPU wrappers for the fused multi-head MLP (one process per GPU).

The reference has no multi-GPU code; these wrappers add the two ways the path shards:

* head-sharded: heads are independent, so rank r of n owns a contiguous block of heads
  (dim 0 of X, W1, W2, O) and runs the kernels on it with no communication;
* batch-sharded: rank r owns a contiguous block of batch rows (dim 1 of X and dO) and a
  replica of W1/W2. After the local backward, dW1 and dW2 are summed over ranks with
  one NCCL all-reduce (in fp32, over one flattened buffer) and every rank applies the
  same SGD step W <- W - lr * dW with the library's update kernel, so replicas stay equal.

Process-group plumbing is torch.distributed; compute is libflashmlp_b200.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .api import flashmlp_bwd, flashmlp_fwd, _dtype_code


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
