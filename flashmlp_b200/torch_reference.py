"""Plain-PyTorch counterparts that the reference module exports next to its kernels.

dtadpole/flashMLP's `flashmlp` module also exports a bmm-based module (`PyTorchMLP`,
flashmlp.py:619-664) and explicit forward/backward functions (`flashmlp_torch_fwd`,
`flashmlp_torch_bwd`, flashmlp.py:671-723) that its example script compares against.
They are re-provided here so `import flashmlp` keeps working for such scripts. They are
NOT used by flashmlp_fwd / flashmlp_bwd / FlashMLP, whose only compute path is the CUDA
library.
"""
from __future__ import annotations

from typing import Tuple

import numpy as np
import torch
import torch.nn.functional as F


def _activate(z: torch.Tensor, activation: str) -> torch.Tensor:
    if activation == "leaky_relu":
        return F.leaky_relu(z, negative_slope=0.01)
    if activation == "silu":
        return F.silu(z)
    if activation == "sigmoid":
        return torch.sigmoid(z)
    return z


def flashmlp_torch_fwd(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                       activation: str = "") -> torch.Tensor:
    """O = act(X @ W1) @ W2 with batched matmuls (materialises the (H,B,E) intermediate)."""
    return torch.bmm(_activate(torch.bmm(x, w1), activation), w2)


def flashmlp_torch_bwd(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                       do: torch.Tensor, activation: str = ""
                       ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Explicit gradients (dx, dw1, dw2) of sum(O * dO), recomputing the forward."""
    z = torch.bmm(x, w1)
    h = _activate(z, activation)
    dh = torch.bmm(do, w2.transpose(-1, -2))
    dw2 = torch.bmm(h.transpose(-1, -2), do)
    if activation == "leaky_relu":
        dz = dh * torch.where(z >= 0, 1.0, 0.01).to(dh.dtype)
    elif activation == "silu":
        s = torch.sigmoid(z)
        dz = dh * (s + z * s * (1 - s))
    elif activation == "sigmoid":
        dz = dh * h * (1 - h)
    else:
        dz = dh
    dx = torch.bmm(dz, w1.transpose(-1, -2))
    dw1 = torch.bmm(x.transpose(-1, -2), dz)
    return dx, dw1, dw2


class PyTorchMLP(torch.nn.Module):
    """bmm-based multi-head MLP with the same interface and init as FlashMLP."""

    def __init__(self, num_heads: int, hidden_dim: int, intermediate_dim: int,
                 activation: str = "silu", dtype=torch.float16, device="cuda"):
        super().__init__()
        self.num_heads = num_heads
        self.hidden_dim = hidden_dim
        self.intermediate_dim = intermediate_dim
        self.activation = activation
        self.w1 = torch.nn.Parameter(
            torch.randn(num_heads, hidden_dim, intermediate_dim, dtype=dtype, device=device)
            / np.sqrt(intermediate_dim)
        )
        self.w2 = torch.nn.Parameter(
            torch.randn(num_heads, intermediate_dim, hidden_dim, dtype=dtype, device=device)
            / np.sqrt(hidden_dim)
        )

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        squeeze_output = x.dim() == 2
        if squeeze_output:
            x = x.unsqueeze(0).expand(self.num_heads, -1, -1)
        o = flashmlp_torch_fwd(x, self.w1, self.w2, self.activation)
        if squeeze_output:
            o = o.mean(dim=0)
        return o
