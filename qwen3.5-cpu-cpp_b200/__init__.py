"""Python side of the B200 Qwen3.5 hybrid forward pass.

The product is the C-ABI shared library ``libqwen_cuda.so`` built from ``csrc/`` (CUDA
kernels + engine) and ``host/`` (the C++ QwenModel / QwenForward / SafeTensors /
ModelConfig / memory-budget mirror of the reference API).  This package holds the
ctypes binding of that C ABI (``abi``) and the seeded synthetic checkpoint writer
(``synth``).  The directory name is not a Python identifier, so callers load it with
``__graft_entry__.load_package()`` which registers it as ``qwen35_b200``.
"""
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libqwen_cuda.so")

from . import synth  # noqa: E402,F401
from . import abi  # noqa: E402,F401
