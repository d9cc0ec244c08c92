"""Drop-in module name: `import flashmlp` / `from flashmlp import FlashMLP, PyTorchMLP`
resolve to the B200 implementation in the flashmlp_b200 package."""
from flashmlp_b200 import *  # noqa: F401,F403
from flashmlp_b200 import __all__  # noqa: F401
