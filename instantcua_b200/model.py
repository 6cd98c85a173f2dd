"""Model tensors for the engine: seeded synthetic weights, quantization through the C ABI and the
``.icua`` container (reference ``Sources/Engine/ModelFile.swift``).

Synthetic weights follow the BASELINE configs: matrices N(0, 0.02) drawn from one
``np.random.default_rng(seed)`` stream in reference TensorID order (embed, then per layer wqkv,
wo, wgu, wd), norm weights 1.0; decoder matrices quantized q4s (symmetric int4, groups of 32,
fp16 scale), the tied embedding / lm_head q8.
"""
from __future__ import annotations

import ctypes as C
import os
import struct

import numpy as np

from . import _lib as L

H, FF, QKV_ROWS, GU_ROWS, HD = 2048, 6144, 4096, 12288, 128
MAGIC = 0x31554349  # "ICU1"
HEADER = 16384


def layer_tid(l: int, slot: str) -> int:
    return L.TID_LAYER_BASE + l * L.TID_PER_LAYER + L.SLOT[slot]


def quantize_q8(w: np.ndarray):
    """Reference q8 (Convert.swift:215-241) through the C ABI: int8 codes, fp16 scale bits."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    codes = np.empty((rows, cols), np.int8)
    scales = np.empty((rows, cols // 32), np.uint16)
    L.check(L.lib().icua_quantize_q8(w.ctypes.data_as(L._FP), rows, cols, codes.ctypes.data, scales.ctypes.data))
    return codes, scales


def quantize_q4s(w: np.ndarray):
    """BASELINE q4s through the C ABI: packed nibbles (u = q + 8), fp16 scale bits."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    packed = np.empty((rows, cols // 2), np.uint8)
    scales = np.empty((rows, cols // 32), np.uint16)
    L.check(L.lib().icua_quantize_q4s(w.ctypes.data_as(L._FP), rows, cols, packed.ctypes.data, scales.ctypes.data))
    return packed, scales


def synthetic_fp32(seed: int = 0, n_layers: int = 28, vocab: int = 151936, std: float = 0.02):
    """Yields (tensor id(s), fp32 array) in TensorID order; matrices N(0, std), norms 1.0."""
    rng = np.random.default_rng(seed)
    sd = np.float32(std)

    def mat(r, c):
        return rng.standard_normal((r, c), dtype=np.float32) * sd

    yield (L.TID_EMBED, L.TID_EMBED_SB), mat(vocab, H)
    yield L.TID_FINAL_NORM, np.ones(H, np.float32)
    for l in range(n_layers):
        yield layer_tid(l, "attn_norm"), np.ones(H, np.float32)
        yield (layer_tid(l, "wqkv"), layer_tid(l, "wqkv_sb")), mat(QKV_ROWS, H)
        yield layer_tid(l, "q_norm"), np.ones(HD, np.float32)
        yield layer_tid(l, "k_norm"), np.ones(HD, np.float32)
        yield (layer_tid(l, "wo"), layer_tid(l, "wo_sb")), mat(H, H)
        yield layer_tid(l, "mlp_norm"), np.ones(H, np.float32)
        yield (layer_tid(l, "wgu"), layer_tid(l, "wgu_sb")), mat(GU_ROWS, H)
        yield (layer_tid(l, "wd"), layer_tid(l, "wd_sb")), mat(H, FF)


def synthetic_fp32_fast(seed: int = 0, n_layers: int = 28, vocab: int = 151936, std: float = 0.02, device: int = 0):
    """Same shapes and distribution as :func:`synthetic_fp32` (seeded N(0, std), norms 1.0), drawn
    with torch's CUDA generator, for benchmarks where generating 1.7e9 numpy normals on the host
    would dominate the run.  The values differ from the numpy stream; parity tests use the latter."""
    import torch

    g = torch.Generator(device=f"cuda:{device}")
    g.manual_seed(seed)

    def mat(r, c):
        t = torch.randn((r, c), generator=g, device=f"cuda:{device}", dtype=torch.float32)
        return (t * std).cpu().numpy()

    yield (L.TID_EMBED, L.TID_EMBED_SB), mat(vocab, H)
    yield L.TID_FINAL_NORM, np.ones(H, np.float32)
    for l in range(n_layers):
        yield layer_tid(l, "attn_norm"), np.ones(H, np.float32)
        yield (layer_tid(l, "wqkv"), layer_tid(l, "wqkv_sb")), mat(QKV_ROWS, H)
        yield layer_tid(l, "q_norm"), np.ones(HD, np.float32)
        yield layer_tid(l, "k_norm"), np.ones(HD, np.float32)
        yield (layer_tid(l, "wo"), layer_tid(l, "wo_sb")), mat(H, H)
        yield layer_tid(l, "mlp_norm"), np.ones(H, np.float32)
        yield (layer_tid(l, "wgu"), layer_tid(l, "wgu_sb")), mat(GU_ROWS, H)
        yield (layer_tid(l, "wd"), layer_tid(l, "wd_sb")), mat(H, FF)


def quantize_stream(fp32_stream, keep_fp32: bool = False, fmt: int = L.FMT_Q4S):
    """Quantizes a (tid, array) stream to {tensor id: bytes} in the .icua tensor layout.

    ``fmt``: decoder-layer format, L.FMT_Q4S (BASELINE: symmetric int4 g32), L.FMT_Q8 (the
    reference's q8 files, Convert.swift:215-241; the tied embedding is q8 in both) or L.FMT_F16
    (the reference converter's default: every matrix fp16).
    ``keep_fp32`` also returns the fp32 arrays (by tensor id of the codes) for checkers.
    """
    if fmt not in (L.FMT_Q4S, L.FMT_Q8, L.FMT_F16):
        raise ValueError(f"unsupported layer format {fmt}")
    out, raw = {}, {}
    for tid, w in fp32_stream:
        if isinstance(tid, tuple):
            codes_id, sb_id = tid
            if fmt == L.FMT_F16:  # reference f16 files: fp16 values, no scale tensors
                out[codes_id] = np.ascontiguousarray(w, np.float32).astype(np.float16).tobytes()
                if keep_fp32:
                    raw[codes_id] = w
                continue
            if codes_id == L.TID_EMBED or fmt == L.FMT_Q8:
                codes, scales = quantize_q8(w)
            else:
                codes, scales = quantize_q4s(w)
            out[codes_id] = codes.tobytes()
            out[sb_id] = scales.tobytes()
            if keep_fp32:
                raw[codes_id] = w
        else:
            out[tid] = np.ascontiguousarray(w, np.float32).tobytes()
            if keep_fp32:
                raw[tid] = w
    return (out, raw) if keep_fp32 else out


VISION_TENSORS = 315  # reference TensorID 0..314 (ModelFile.swift:73-99)


def vision_shapes():
    """(shape, dtype) of each vision tensor by reference id (ModelFile.swift:73-99, storage types of
    Convert.swift:99-152): patch matrix, patch bias, position table; 24 blocks of (norm1 w/b, qkv
    w/b, proj w/b, norm2 w/b, fc1 w/b, fc2 w/b); 3 DeepStack mergers and the final merger of
    (norm w/b, fc1 w/b, fc2 w/b)."""
    f16, f32 = np.float16, np.float32
    out = [((1024, 768), f16), ((1024,), f32), ((2304, 1024), f32)]
    for _ in range(24):
        out += [((1024,), f32), ((1024,), f32), ((3072, 1024), f16), ((3072,), f32), ((1024, 1024), f16),
                ((1024,), f32), ((1024,), f32), ((1024,), f32), ((4096, 1024), f16), ((4096,), f32),
                ((1024, 4096), f16), ((1024,), f32)]
    for m in range(4):
        norm = 1024 if m == 3 else 4096
        out += [((norm,), f32), ((norm,), f32), ((4096, 4096), f16), ((4096,), f32), ((2048, 4096), f16),
                ((2048,), f32)]
    assert len(out) == VISION_TENSORS
    return out


def synthetic_vision_fast(seed: int = 0, device: int = 0, std: float = 0.02) -> dict:
    """Seeded synthetic vision tensors drawn on the GPU (torch) in their storage types: matrices and
    biases N(0, std), norm weights 1, norm biases 0, position table N(0, 0.5).  {id: bytes}."""
    import torch

    g = torch.Generator(device=f"cuda:{device}").manual_seed(seed)
    out = {}
    for tid, (shape, dt) in enumerate(vision_shapes()):
        if tid == 2:
            a = torch.randn(shape, generator=g, device=f"cuda:{device}") * 0.5
        elif len(shape) == 1 and ((tid >= 3 and tid < 291 and (tid - 3) % 12 in (0, 6)) or
                                  (tid >= 291 and (tid - 291) % 6 == 0)):
            a = torch.ones(shape, device=f"cuda:{device}")
        elif len(shape) == 1 and ((tid >= 3 and tid < 291 and (tid - 3) % 12 in (1, 7)) or
                                  (tid >= 291 and (tid - 291) % 6 == 1)):
            a = torch.zeros(shape, device=f"cuda:{device}")
        else:
            a = torch.randn(shape, generator=g, device=f"cuda:{device}") * std
        a = a.half() if dt == np.float16 else a.float()
        out[tid] = a.cpu().numpy().tobytes()
    return out


def vision_tensors(named: dict) -> dict:
    """Vision encoder tensors in the file's storage types (Convert.swift:99-152) keyed by reference
    tensor id: the matrices (patch embedding [1024, 768] with the temporal frames folded, QKV,
    projection, MLP, merger layers) as fp16 [out, in], biases, norms and the position table fp32.
    ``named``: fp32 arrays under the names of ``oracle.qwen3vl_vision.weight_names`` order, which
    is the id order."""
    shapes = vision_shapes()
    assert len(named) == VISION_TENSORS, len(named)
    out = {}
    for tid, arr in enumerate(named.values()):
        shape, dt = shapes[tid]
        a = np.ascontiguousarray(arr, dt)
        assert a.shape == shape, (tid, a.shape, shape)
        out[tid] = a.tobytes()
    return out


def write_icua(path: str, tensors: dict, fmt: int = L.FMT_Q4S) -> None:
    """Writes an .icua file (ModelFile.swift:164-195 layout): 16 KiB header with magic, version 1,
    format, tensor count and an (offset, size) u64 table; tensors 256-byte aligned; the file
    padded to a multiple of 16 KiB."""
    table = [(0, 0)] * L.TENSOR_COUNT
    cursor = HEADER
    layout = []
    for tid in sorted(tensors):
        data = tensors[tid]
        cursor = (cursor + 255) & ~255
        table[tid] = (cursor, len(data))
        layout.append((cursor, data))
        cursor += len(data)
    total = (cursor + HEADER - 1) // HEADER * HEADER
    with open(path, "wb") as f:
        hdr = bytearray(HEADER)
        struct.pack_into("<IIII", hdr, 0, MAGIC, 1, fmt, L.TENSOR_COUNT)
        for i, (o, s) in enumerate(table):
            struct.pack_into("<QQ", hdr, 16 + 16 * i, o, s)
        f.write(hdr)
        pos = HEADER
        for off, data in layout:
            if off > pos:
                f.write(b"\0" * (off - pos))
            f.write(data)
            pos = off + len(data)
        if total > pos:
            f.write(b"\0" * (total - pos))
