"""flashmlp_b200 — B200 (sm_100a) fused multi-head MLP, a drop-in for dtadpole/flashMLP.

Public names match the reference module `flashmlp` (flashmlp.py): flashmlp_fwd,
flashmlp_bwd, FlashMLPFunction, FlashMLP, plus the plain-PyTorch PyTorchMLP,
flashmlp_torch_fwd and flashmlp_torch_bwd it also exports. Multi-GPU wrappers live in
flashmlp_b200.sharding; the FP8 (e4m3) forward, which the reference does not have, in
flashmlp_b200.fp8.
"""
from .api import (FlashMLP, FlashMLPFunction, FlashMLPSharedInputFunction, activation_code,
                  backward_workspace_limit, flashmlp_bwd, flashmlp_bwd_dw_f32, flashmlp_bwd_shared_x, flashmlp_fwd,
                  flashmlp_fwd_shared_x, low_memory_backward)
from .torch_reference import PyTorchMLP, flashmlp_torch_bwd, flashmlp_torch_fwd
from ._lib import FlashMLPError
from .fp8 import Fp8Weights, flashmlp_fwd_fp8, prepare_fp8_weights, quantize_e4m3

__all__ = [
    "low_memory_backward",
    "backward_workspace_limit",
    "flashmlp_fwd",
    "flashmlp_bwd",
    "FlashMLPFunction",
    "FlashMLP",
    "PyTorchMLP",
    "flashmlp_torch_fwd",
    "flashmlp_torch_bwd",
    "FlashMLPError",
    "activation_code",
    "flashmlp_bwd_dw_f32",
    "flashmlp_fwd_shared_x",
    "flashmlp_bwd_shared_x",
    "FlashMLPSharedInputFunction",
    "flashmlp_fwd_fp8",
    "prepare_fp8_weights",
    "quantize_e4m3",
    "Fp8Weights",
]
