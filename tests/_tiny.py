"""The tiny test model shared by the fixture generator and the tests.

Two decoder layers at full width (hidden 2048, 16/8 heads, FFN 6144) and a 1024-row vocabulary;
matrices N(0, 0.02) from the seeded stream of ``oracle.qwen3vl_oracle.generate_fp32_weights``,
norm weights 1 + 0.1 N(0, 1) so that the norm paths are exercised.
"""
from __future__ import annotations

import numpy as np

SEED = 7
N_LAYERS = 2
VOCAB = 1024


def tiny_fp32():
    """{oracle name: fp32 array}"""
    from oracle import qwen3vl_oracle as O

    w = dict(O.generate_fp32_weights(seed=SEED, n_layers=N_LAYERS, vocab=VOCAB))
    rng = np.random.default_rng(SEED + 1)
    for k in list(w):
        if w[k].ndim == 1:
            w[k] = (1.0 + 0.1 * rng.standard_normal(w[k].shape)).astype(np.float32)
    return w


def oracle_name_to_tid(name: str):
    """Maps an oracle tensor name to the reference TensorID(s) (codes id, SB id) or id."""
    from instantcua_b200 import _lib as L

    if name == "embed":
        return (L.TID_EMBED, L.TID_EMBED_SB)
    if name == "final_norm":
        return L.TID_FINAL_NORM
    l, nm = name[1:].split(".", 1)
    base = L.TID_LAYER_BASE + int(l) * L.TID_PER_LAYER
    if nm in ("wqkv", "wo", "wgu", "wd"):
        return (base + L.SLOT[nm], base + L.SLOT[nm + "_sb"])
    return base + L.SLOT[nm]


def fp32_stream(w: dict):
    for name, arr in w.items():
        yield oracle_name_to_tid(name), arr


def engine_tensors(w: dict | None = None) -> dict:
    """Quantized .icua tensors of the tiny model, produced by the product's C++ quantizers."""
    from instantcua_b200 import model

    return model.quantize_stream(fp32_stream(w if w is not None else tiny_fp32()))
