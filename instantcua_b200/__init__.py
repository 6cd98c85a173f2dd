"""B200 (sm_100a) engine for the Qwen3VLTextModel token loop of instantcua.

The compute path is the in-tree CUDA library ``libicua_cuda.so`` behind the C ABI in
``include/icua.h``; this package holds the build script and the Python mirror of the reference
``Engine``.
"""
from ._lib import IcuaError, lib  # noqa: F401
from .engine import Engine, Timing  # noqa: F401
