"""A numpy stand-in for the part of ``mlx.core`` that the reference oracle uses (TEST INFRASTRUCTURE).

The reference's oracle (``tools/reference/qwen3vl_ref.py`` in the reference project) is written
against MLX, which is Apple-only and not installed here.  It uses a small surface of
``mlx.core``: ``array``, ``float32`` / ``int32``, ``eval``, ``load``, ``mean``, ``square``,
``rsqrt``, ``concatenate``, ``transpose``, ``repeat``, ``softmax``, ``sigmoid``, ``tanh``,
``erf``, ``triu``, ``full`` and ``argmax``.  :func:`install` registers a module with those names
in ``sys.modules`` under ``mlx`` / ``mlx.core``, each a numpy fp32 operation, so that the
reference file can be imported and run unmodified.  What this pins is the reference's own
algorithm (its order of operations, masks, GQA repeat, M-RoPE and rope_delta logic, DeepStack
scatter, decode loop); the elementwise and matmul arithmetic is numpy's fp32 in place of MLX's
fp32 kernels.

``argmax`` also appends its input to :data:`ARGMAX_LOG`, which is how the fixture generator reads
the reference's per-step decode logits (the reference returns only the first step's).
"""
from __future__ import annotations

import sys
import types

import numpy as np

F32 = np.float32
ARGMAX_LOG: list = []


def _f(x):
    """fp32 view of a float operand; integer arrays pass through."""
    a = np.asarray(x)
    return a.astype(F32, copy=False) if a.dtype.kind == "f" else a


def array(x, dtype=None):
    a = np.asarray(x)
    if dtype is not None:
        return np.array(a, dtype=dtype)
    return a.astype(F32) if a.dtype.kind == "f" and a.dtype != F32 else np.array(a)


def eval(*args):  # noqa: A001 - MLX's name; arrays here are already computed
    return None


def load(path):
    raise RuntimeError("mlx_numpy: weights are supplied by the fixture generator, not loaded from files")


def mean(x, axis=None, keepdims=False):
    return np.mean(_f(x), axis=axis, keepdims=keepdims, dtype=F32)


def square(x):
    x = _f(x)
    return x * x


def rsqrt(x):
    return (F32(1) / np.sqrt(_f(x))).astype(F32)


def concatenate(xs, axis=0):
    return np.concatenate([np.asarray(a) for a in xs], axis=axis)


def transpose(x, axes=None):
    return np.transpose(np.asarray(x), axes)


def repeat(x, repeats, axis=None):
    return np.repeat(np.asarray(x), repeats, axis=axis)


def softmax(x, axis=-1):
    x = _f(x)
    e = np.exp(x - np.max(x, axis=axis, keepdims=True))
    return (e / np.sum(e, axis=axis, keepdims=True, dtype=F32)).astype(F32)


def sigmoid(x):
    x = _f(x)
    return (F32(1) / (F32(1) + np.exp(-x))).astype(F32)


def tanh(x):
    return np.tanh(_f(x)).astype(F32)


def erf(x):
    from scipy.special import erf as _erf

    return _erf(_f(x)).astype(F32)


def triu(x, k=0):
    return np.triu(np.asarray(x), k=k)


def full(shape, value, dtype=None):
    return np.full(shape, value, dtype=dtype if dtype is not None else F32)


def argmax(x, axis=None):
    a = np.asarray(x)
    ARGMAX_LOG.append(np.array(a, dtype=F32))
    return np.argmax(a, axis=axis)


def install() -> types.ModuleType:
    """Registers this stand-in as ``mlx.core`` (and a parent ``mlx`` package) in sys.modules."""
    core = types.ModuleType("mlx.core")
    for name in ("array", "eval", "load", "mean", "square", "rsqrt", "concatenate", "transpose", "repeat",
                 "softmax", "sigmoid", "tanh", "erf", "triu", "full", "argmax"):
        setattr(core, name, globals()[name])
    core.float32 = np.float32
    core.int32 = np.int32
    core.ARGMAX_LOG = ARGMAX_LOG
    pkg = types.ModuleType("mlx")
    pkg.__path__ = []  # a package, so that "import mlx.core" resolves
    pkg.core = core
    sys.modules["mlx"] = pkg
    sys.modules["mlx.core"] = core
    return core
