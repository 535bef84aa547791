"""The public API under the module path nvdiffrast uses: ``import diffrast_b200.torch as dr``."""

if __name__ == "torch":
    raise ImportError(
        "'import torch' found diffrast_b200/torch.py instead of PyTorch, because the package "
        "directory is the working directory or on sys.path. Run from another directory."
    )

from diffrast_b200 import *  # noqa: E402,F403
from diffrast_b200 import __all__ as __all__  # noqa: E402
