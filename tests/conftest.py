import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"
GOLDEN_CASES = ["f16_main", "f16_tail", "f16_c1", "bf16_main", "bf16_c3", "f32_main"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built CUDA library")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs")


def load_golden(name: str) -> dict:
    """Loads tests/golden/<name>.npz; inputs are returned as float32 arrays holding the
    16-bit values, outputs as float32."""
    from oracle import flashmlp_oracle as orc

    z = np.load(GOLDEN / f"{name}.npz")
    dtype = str(z["dtype"])
    out = {"shape": tuple(int(v) for v in z["shape"]), "dtype": dtype,
           "acts": [str(a) for a in z["acts"]]}
    for k in ("x", "w1", "w2", "do"):
        a = z[k]
        out[k] = a.astype(np.float32) if dtype in ("f16", "f32") else orc.bf16_from_bits(a)
    for k in z.files:
        if k.startswith(("torch_", "triton_")):
            out[k] = z[k].astype(np.float32)
    return out


@pytest.fixture(scope="session")
def golden():
    return {n: load_golden(n) for n in GOLDEN_CASES}


def pytest_terminal_summary(terminalreporter):
    """Largest norm-wise relative error ||a - r||_F / ||r||_F per (dtype, kind) that the
    parity checks saw in this session, next to the bound each one is held to."""
    try:
        import _refcheck
    except Exception:
        return
    for line in _refcheck.INFO:
        terminalreporter.write_line(line)
    if not _refcheck.NORM_SEEN:
        return
    terminalreporter.write_line("norm-wise parity (worst head slice seen / bound):")
    for (dt, kind), v in sorted(_refcheck.NORM_SEEN.items()):
        import torch

        c = _refcheck.NORM_C[getattr(torch, dt)]
        terminalreporter.write_line(f"  {dt:9s} {kind:4s} {v:.3e} / {c:g}")
