"""Generates the golden fixtures in tests/golden/*.npz from the reference itself.

Run where a checkout of the reference (dtadpole/flashMLP) is available; the fixtures are
committed, so tests never need it:

    python tests/golden/make_golden.py REF_DIR      # REF_DIR holds the reference's flashmlp.py

For every case the reference's own code produces the expected outputs:
  * "torch_*": the reference's PyTorch path flashmlp_torch_fwd / flashmlp_torch_bwd
    (flashmlp.py:671-723) on CPU in float32, inputs upcast from the 16-bit values;
  * "triton_*": the reference's Triton kernels flashmlp_fwd_kernel / flashmlp_bwd_kernel
    (flashmlp.py:63-158, :341-421) under the Triton CPU interpreter (TRITON_INTERPRET=1)
    in float16, launched through the reference's own wrapper logic (flashmlp.py:449-477,
    :501-538) with explicit block sizes, since the autotuner needs a GPU driver.
    The interpreter cannot run bfloat16 and the reference's kernels require a power-of-two
    D (and its forward needs B and E to be multiples of its tiles: the B/E tails are
    handled wrongly there), so those cases carry only the "torch_*" outputs.
    The float32 case runs the Triton kernels on float32 tensors: the interpreter evaluates
    tl.dot in full fp32 (on a GPU it would use TF32).
Inputs are seeded (numpy default_rng) with X ~ N(0,1), W1 ~ N(0,1/D), W2 ~ N(0,1/E),
dO ~ N(0,1) and rounded to the 16-bit dtype (float32 inputs are not rounded).

    python tests/golden/make_golden.py REF_DIR [CASE ...]   # only the named cases
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

from oracle import flashmlp_oracle as orc  # noqa: E402

ACTS = ["", "leaky_relu", "silu", "sigmoid"]

# name, (H, B, D, E), dtype, activations, triton fwd tiles or None, triton bwd tiles or None
CASES = [
    ("f16_main", (2, 64, 64, 128), "f16", ACTS, (32, 32), (32, 32)),
    ("f16_tail", (2, 100, 32, 96), "f16", ACTS, None, (32, 64)),
    ("f16_c1", (2, 128, 64, 256), "f16", ["silu"], (64, 64), (64, 64)),
    ("bf16_main", (2, 64, 64, 128), "bf16", ACTS, None, None),
    ("bf16_c3", (1, 200, 96, 200), "bf16", ["", "sigmoid"], None, None),
    ("f32_main", (2, 64, 64, 128), "f32", ACTS, (32, 32), (32, 32)),
]


def _store_inputs(out: dict, arrs, dtype: str) -> None:
    for k, a in zip(("x", "w1", "w2", "do"), arrs):
        if dtype == "f16":
            out[k] = a.astype(np.float16)
        elif dtype == "f32":
            out[k] = a.astype(np.float32)
        else:
            out[k] = orc.bf16_bits(a)


def main(ref_dir: str, only=()) -> None:
    sys.path.insert(0, ref_dir)
    import torch
    import triton
    import flashmlp as ref  # the reference module (flashmlp.py)

    for seed, (name, (H, B, D, E), dtype, acts, ftiles, btiles) in enumerate(CASES):
        if only and name not in only:
            continue
        x, w1, w2, do = orc.make_inputs(H, B, D, E, dtype, seed=100 + seed)
        out = {"shape": np.array([H, B, D, E]), "dtype": np.array(dtype), "acts": np.array(acts)}
        _store_inputs(out, (x, w1, w2, do), dtype)
        tx, tw1, tw2, tdo = (torch.from_numpy(a) for a in (x, w1, w2, do))
        for act in acts:
            tag = act or "linear"
            o = ref.flashmlp_torch_fwd(tx, tw1, tw2, act)
            dx, dw1, dw2 = ref.flashmlp_torch_bwd(tx, tw1, tw2, tdo, act)
            out[f"torch_o_{tag}"] = o.numpy()
            out[f"torch_dx_{tag}"] = dx.numpy()
            out[f"torch_dw1_{tag}"] = dw1.numpy()
            out[f"torch_dw2_{tag}"] = dw2.numpy()
            if dtype == "bf16":
                continue
            cast = (lambda t: t.half()) if dtype == "f16" else (lambda t: t.float())
            hx, hw1, hw2, hdo = (cast(t) for t in (tx, tw1, tw2, tdo))
            xr, w1r, w2r = hx.reshape(H * B, D), hw1.reshape(D * H, E), hw2.reshape(E * H, D)
            if ftiles is not None:
                bb, be = ftiles
                o16 = torch.zeros_like(xr)
                ref.flashmlp_fwd_kernel.fn[(triton.cdiv(B, bb) * H,)](
                    xr, w1r, w2r, o16, H, B, D, E,
                    xr.stride(0), xr.stride(1), w1r.stride(0), w1r.stride(1),
                    w2r.stride(0), w2r.stride(1), o16.stride(0), o16.stride(1),
                    BLOCK_SIZE_B=bb, BLOCK_SIZE_E=be, ACTIVATION=act)
                out[f"triton_o_{tag}"] = o16.reshape(H, B, D).numpy()
            if btiles is not None:
                bb, be = btiles
                dor = hdo.reshape(H * B, D).contiguous()
                gx, g1, g2 = torch.zeros_like(xr), torch.zeros_like(w1r), torch.zeros_like(w2r)
                grid = ((triton.cdiv(B, bb) + triton.cdiv(E, be)) * H,)
                ref.flashmlp_bwd_kernel.fn[grid](
                    xr, w1r, w2r, gx, g1, g2, dor, H, B, D, E,
                    xr.stride(0), xr.stride(1), w1r.stride(0), w1r.stride(1),
                    w2r.stride(0), w2r.stride(1), gx.stride(0), gx.stride(1),
                    g1.stride(0), g1.stride(1), g2.stride(0), g2.stride(1),
                    dor.stride(0), dor.stride(1),
                    BLOCK_SIZE_B=bb, BLOCK_SIZE_E=be, ACTIVATION=act)
                out[f"triton_dx_{tag}"] = gx.reshape(H, B, D).numpy()
                out[f"triton_dw1_{tag}"] = g1.reshape(H, D, E).numpy()
                out[f"triton_dw2_{tag}"] = g2.reshape(H, E, D).numpy()
        path = HERE / f"{name}.npz"
        np.savez_compressed(path, **out)
        print(f"wrote {path.name}: {path.stat().st_size / 1024:.0f} KiB")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        raise SystemExit("usage: make_golden.py REF_DIR [CASE ...]")
    main(sys.argv[1], tuple(sys.argv[2:]))
