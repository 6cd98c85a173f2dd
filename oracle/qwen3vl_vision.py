"""CPU oracle for the Qwen3-VL vision encoder and mergers (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` may import this module, as the
checker; the CUDA vision path in ``instantcua_b200`` never routes through it.

Restates in numpy fp32, from the reference project (paths inside that project):

* ``tools/reference/qwen3vl_ref.py:25-38``   ``load_image_patches`` (from an RGB array) -> :func:`patchify`
* ``tools/reference/qwen3vl_ref.py:41-68``   ``compute_vision_pos_embed`` -> :func:`pos_embed_interp`
* ``tools/reference/qwen3vl_ref.py:71-84``   ``compute_vision_rope``      -> :func:`vision_rope`
* ``tools/reference/qwen3vl_ref.py:142-163`` ``layernorm`` / ``gelu_tanh`` / ``gelu_exact``
* ``tools/reference/qwen3vl_ref.py:165-216`` ``encode_vision`` (24 blocks, DeepStack mergers after
  blocks 5, 11, 17, final merger)           -> :func:`encode_vision`
* ``Sources/Engine/Convert.swift:99-152``    tensor storage: matrices fp16, biases / norms / the
  position table fp32, the two temporal patch frames folded into one 768-column patch matrix.

Dimensions are parameters (``VisionDims``) so that the restatement can be pinned against
Hugging Face ``Qwen3VLVisionModel`` on a narrow configuration (``tests/golden/make_golden_vision.py``);
the engine's kernels are built for the reference's dimensions (``REFERENCE``).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

F32 = np.float32


@dataclass(frozen=True)
class VisionDims:
    layers: int = 24
    hidden: int = 1024
    ff: int = 4096
    heads: int = 16
    head_dim: int = 64
    patch: int = 16
    merge: int = 2
    pos_side: int = 48
    deepstack: tuple = (5, 11, 17)
    out_hidden: int = 2048
    theta: float = 10000.0
    eps: float = 1e-6

    @property
    def patch_dim(self) -> int:
        return 3 * self.patch * self.patch

    @property
    def merged(self) -> int:
        return self.hidden * self.merge * self.merge


REFERENCE = VisionDims()


def patchify(rgb: np.ndarray, d: VisionDims = REFERENCE):
    """RGB uint8 [H, W, 3] -> patches [n, 3*p*p] in 2x2 merge-block order, values 2x/255 - 1
    (qwen3vl_ref.py:25-38; the device rounds them to fp16, Shaders.swift:82-110)."""
    arr = np.asarray(rgb, dtype=F32) * F32(2.0 / 255.0) - F32(1.0)
    H, W, C = arr.shape
    p, m = d.patch, d.merge
    assert H % (p * m) == 0 and W % (p * m) == 0
    gh, gw = H // p, W // p
    chw = np.transpose(arr, (2, 0, 1)).reshape(C, gh // m, m, p, gw // m, m, p)
    patches = np.transpose(chw, (1, 4, 2, 5, 0, 3, 6)).reshape(gh * gw, C * p * p)
    return np.ascontiguousarray(patches), gh, gw


def _merge_order_rc(gh: int, gw: int, m: int):
    """(row, col) of each patch in merge-block order."""
    idx = np.arange(gh * gw)
    bw = gw // m
    in_col = idx % m
    in_row = (idx // m) % m
    b_col = (idx // (m * m)) % bw
    b_row = idx // (m * m * bw)
    return b_row * m + in_row, b_col * m + in_col


def pos_embed_interp(table: np.ndarray, gh: int, gw: int, d: VisionDims = REFERENCE) -> np.ndarray:
    """Bilinear (align_corners) resampling of the [side*side, hidden] position table to the patch
    grid, rows in merge-block order (qwen3vl_ref.py:41-68)."""
    side = d.pos_side
    t = table.reshape(side, side, -1).astype(F32)
    row, col = _merge_order_rc(gh, gw, d.merge)
    src_h = row.astype(F32) * F32(side - 1) / F32(max(gh - 1, 1))
    src_w = col.astype(F32) * F32(side - 1) / F32(max(gw - 1, 1))
    h0 = np.floor(src_h).astype(np.int32)
    w0 = np.floor(src_w).astype(np.int32)
    h1 = np.minimum(h0 + 1, side - 1)
    w1 = np.minimum(w0 + 1, side - 1)
    dh = (src_h - h0)[:, None].astype(F32)
    dw = (src_w - w0)[:, None].astype(F32)
    return ((F32(1) - dh) * ((F32(1) - dw) * t[h0, w0] + dw * t[h0, w1]) +
            dh * ((F32(1) - dw) * t[h1, w0] + dw * t[h1, w1])).astype(F32)


def vision_rope(gh: int, gw: int, d: VisionDims = REFERENCE):
    """2-D axial RoPE cos / sin [n, head_dim]: the first quarter of the frequencies rotate by the
    patch row, the second by the column, repeated for the rotate-half pairs (qwen3vl_ref.py:71-84)."""
    spatial = d.head_dim // 2
    inv = (1.0 / (d.theta ** (np.arange(0, spatial, 2, dtype=F32) / spatial))).astype(F32)
    row, col = _merge_order_rc(gh, gw, d.merge)
    fh = row.astype(F32)[:, None] * inv[None, :]
    fw = col.astype(F32)[:, None] * inv[None, :]
    ang = np.concatenate([fh, fw, fh, fw], axis=-1).astype(F32)
    return np.cos(ang).astype(F32), np.sin(ang).astype(F32)


def layernorm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float) -> np.ndarray:
    mean = x.mean(axis=-1, keepdims=True, dtype=F32)
    var = np.square(x - mean).mean(axis=-1, keepdims=True, dtype=F32)
    return ((x - mean) / np.sqrt(var + F32(eps)) * w + b).astype(F32)


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    return (F32(0.5) * x * (F32(1) + np.tanh(F32(np.sqrt(2.0 / np.pi)) * (x + F32(0.044715) * x * x * x)))).astype(F32)


def gelu_exact(x: np.ndarray) -> np.ndarray:
    from scipy.special import erf

    return (F32(0.5) * x * (F32(1) + erf(x / F32(np.sqrt(2.0))).astype(F32))).astype(F32)


def _rotate_half(x: np.ndarray) -> np.ndarray:
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def weight_names(d: VisionDims = REFERENCE):
    """Oracle tensor names in the reference's TensorID order (ModelFile.swift:73-99)."""
    names = ["patch_w", "patch_b", "pos"]
    for l in range(d.layers):
        names += [f"v{l}.{k}" for k in ("norm1_w", "norm1_b", "qkv_w", "qkv_b", "proj_w", "proj_b", "norm2_w",
                                         "norm2_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b")]
    for m in range(len(d.deepstack) + 1):
        names += [f"m{m}.{k}" for k in ("norm_w", "norm_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b")]
    return names


def weight_shape(name: str, d: VisionDims = REFERENCE):
    k = name.split(".")[-1]
    if name == "patch_w":
        return (d.hidden, d.patch_dim)
    if name == "patch_b":
        return (d.hidden,)
    if name == "pos":
        return (d.pos_side * d.pos_side, d.hidden)
    if name.startswith("v"):
        return {"norm1_w": (d.hidden,), "norm1_b": (d.hidden,), "qkv_w": (3 * d.hidden, d.hidden),
                "qkv_b": (3 * d.hidden,), "proj_w": (d.hidden, d.hidden), "proj_b": (d.hidden,),
                "norm2_w": (d.hidden,), "norm2_b": (d.hidden,), "fc1_w": (d.ff, d.hidden), "fc1_b": (d.ff,),
                "fc2_w": (d.hidden, d.ff), "fc2_b": (d.hidden,)}[k]
    final = name.startswith(f"m{len(d.deepstack)}.")
    norm = d.hidden if final else d.merged  # final merger: LN per patch before the 2x2 shuffle
    return {"norm_w": (norm,), "norm_b": (norm,), "fc1_w": (d.merged, d.merged), "fc1_b": (d.merged,),
            "fc2_w": (d.out_hidden, d.merged), "fc2_b": (d.out_hidden,)}[k]


def is_matrix(name: str) -> bool:
    return name.endswith("_w") and name.split(".")[-1] in ("patch_w", "qkv_w", "proj_w", "fc1_w", "fc2_w")


def generate_weights(seed: int = 11, d: VisionDims = REFERENCE, std: float = 0.02):
    """Seeded synthetic weights: matrices N(0, std) rounded to fp16 (their storage type), biases
    N(0, std), norm weights 1 + 0.1 N(0, 1), norm biases 0.1 N(0, 1), position table N(0, 0.5)."""
    rng = np.random.default_rng(seed)
    w = {}
    for n in weight_names(d):
        shp = weight_shape(n, d)
        k = n.split(".")[-1]
        if is_matrix(n) or n == "patch_w":
            a = (rng.standard_normal(shp, dtype=F32) * F32(std)).astype(np.float16).astype(F32)
        elif n == "pos":
            a = rng.standard_normal(shp, dtype=F32) * F32(0.5)
        elif k.startswith("norm") and k.endswith("_w"):
            a = F32(1) + F32(0.1) * rng.standard_normal(shp, dtype=F32)
        elif k.startswith("norm"):
            a = F32(0.1) * rng.standard_normal(shp, dtype=F32)
        else:
            a = rng.standard_normal(shp, dtype=F32) * F32(std)
        w[n] = a.astype(F32)
    return w


def encode_vision(w: dict, patches: np.ndarray, gh: int, gw: int, d: VisionDims = REFERENCE):
    """Vision encoder + mergers (qwen3vl_ref.py:165-216).  Returns (pooler [n/4, out_hidden],
    [deepstack_0, deepstack_1, deepstack_2] each [n/4, out_hidden])."""
    n = gh * gw
    nv = n // (d.merge * d.merge)
    pos = pos_embed_interp(w["pos"], gh, gw, d)
    cos, sin = vision_rope(gh, gw, d)
    cos, sin = cos[:, None, :], sin[:, None, :]
    x = (patches.astype(F32) @ w["patch_w"].T + w["patch_b"] + pos).astype(F32)
    ds_out = []
    scale = F32(d.head_dim ** -0.5)
    for l in range(d.layers):
        p = f"v{l}."
        h = layernorm(x, w[p + "norm1_w"], w[p + "norm1_b"], d.eps)
        qkv = (h @ w[p + "qkv_w"].T + w[p + "qkv_b"]).reshape(n, 3, d.heads, d.head_dim)
        q = qkv[:, 0] * cos + _rotate_half(qkv[:, 0]) * sin
        k = qkv[:, 1] * cos + _rotate_half(qkv[:, 1]) * sin
        v = qkv[:, 2]
        qt, kt, vt = (np.transpose(a, (1, 0, 2)) for a in (q, k, v))
        s = (qt @ np.transpose(kt, (0, 2, 1))) * scale
        s = s - s.max(axis=-1, keepdims=True)
        e = np.exp(s)
        probs = e / e.sum(axis=-1, keepdims=True)
        att = np.transpose(probs @ vt, (1, 0, 2)).reshape(n, d.hidden)
        x = (x + att @ w[p + "proj_w"].T + w[p + "proj_b"]).astype(F32)
        h2 = layernorm(x, w[p + "norm2_w"], w[p + "norm2_b"], d.eps)
        f1 = gelu_tanh(h2 @ w[p + "fc1_w"].T + w[p + "fc1_b"])
        x = (x + f1 @ w[p + "fc2_w"].T + w[p + "fc2_b"]).astype(F32)
        if l in d.deepstack:
            m = f"m{d.deepstack.index(l)}."
            xm = layernorm(x.reshape(nv, d.merged), w[m + "norm_w"], w[m + "norm_b"], d.eps)
            xm = gelu_exact(xm @ w[m + "fc1_w"].T + w[m + "fc1_b"])
            ds_out.append((xm @ w[m + "fc2_w"].T + w[m + "fc2_b"]).astype(F32))
    m = f"m{len(d.deepstack)}."
    xm = layernorm(x, w[m + "norm_w"], w[m + "norm_b"], d.eps).reshape(nv, d.merged)
    xm = gelu_exact(xm @ w[m + "fc1_w"].T + w[m + "fc1_b"])
    pooler = (xm @ w[m + "fc2_w"].T + w[m + "fc2_b"]).astype(F32)
    return pooler, ds_out
