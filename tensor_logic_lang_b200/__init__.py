"""B200-native (sm_100a) execution backend for Tensor Logic programs.

The package holds the C-ABI runtime (csrc/ → libtl_cuda.so) and its host-side
mirror: `lang` reads `.tl` source into ABI statements, `runtime` drives the
library.  There is no CPU fallback: importing `runtime` requires the built
CUDA library.
"""
from . import abi, lang  # noqa: F401

__all__ = ["abi", "lang"]
