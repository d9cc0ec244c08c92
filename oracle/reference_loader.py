"""Loader of the unmodified reference module (dtadpole/flashMLP, flashmlp.py) — TEST
INFRASTRUCTURE ONLY.

The reference is installed, unmodified, into the git-ignored `baseline/_ref/` of this
repository (a pip install of a temporary copy of the reference with a minimal
pyproject.toml, since the reference ships no packaging metadata), so that it travels to
the GPU box with the working tree. Only tests/ and bench.py's reference leg load it, as
the checker (its Triton kernels on the B200, its PyTorch path on the host cores) and as
the timed reference arm; the product path (flashmlp_b200) never does.

The repository root also has a `flashmlp.py` (the drop-in module name of the B200
implementation), so the reference is loaded from its file path under the module name
`flashmlp_reference`, never as `flashmlp`.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path
from typing import Optional

REF_PATH = Path(__file__).resolve().parent.parent / "baseline" / "_ref" / "flashmlp.py"
MODULE_NAME = "flashmlp_reference"


def reference_available() -> bool:
    return REF_PATH.is_file()


def load_reference() -> Optional[object]:
    """The reference module, or None when baseline/_ref holds no install. Importing it
    imports torch and triton (the Triton kernels compile on first launch)."""
    if MODULE_NAME in sys.modules:
        return sys.modules[MODULE_NAME]
    if not reference_available():
        return None
    spec = importlib.util.spec_from_file_location(MODULE_NAME, REF_PATH)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[MODULE_NAME] = mod  # triton.jit inspects the defining module's source
    try:
        spec.loader.exec_module(mod)
    except Exception:
        del sys.modules[MODULE_NAME]
        raise
    return mod
