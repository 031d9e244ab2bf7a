"""B200-native attention + KV-cache hot path of tampajohn/fpga-qwen's Qwen3-0.6B engine.

The product is ``libqattn.so`` (C ABI in ``include/qattn.h``); this package holds its CUDA
sources (``csrc/``), the build recipe (``build.py``), a ctypes binding (``qattn.py``), the
host-side mirror of the reference's model API for this path (``engine.py``), and the
canonical prefix-reuse policy (``prefix.py``).
"""
from .qattn import Context, QAttnError, lib  # noqa: F401
