"""CPU tests of the C ABI library: it loads, exports every declared symbol, its host quantizers
match the oracle bit for bit, and its tile packing decodes back to the same values."""
import ctypes as C
import os
import re
import struct

import numpy as np
import pytest

from instantcua_b200 import _lib as L
from instantcua_b200 import model
from oracle import qwen3vl_oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "icua.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(icua_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    names = header_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(L.PROTOTYPES), set(names) ^ set(L.PROTOTYPES)


@pytest.mark.parametrize("shape", [(64, 256), (48, 2048)])
def test_host_quantizers_bit_exact(shape):
    rng = np.random.default_rng(shape[0])
    w = (rng.standard_normal(shape) * 0.02).astype(np.float32)
    w[0, :32] = 0.0
    w[1, 5] = 0.75
    c_ref, s_ref = O.quantize_q8(w)
    c, s = model.quantize_q8(w)
    assert np.array_equal(c, c_ref) and np.array_equal(s, s_ref.view(np.uint16))
    p_ref, s_ref = O.quantize_q4s(w)
    p, s = model.quantize_q4s(w)
    assert np.array_equal(p, p_ref) and np.array_equal(s, s_ref.view(np.uint16))


def test_host_quantizers_known_answers(golden):
    kat = golden["kat_in"]
    c, s = model.quantize_q8(kat)
    assert np.array_equal(c, golden["kat_q8_codes"]) and np.array_equal(s, golden["kat_q8_scales"].view(np.uint16))
    p, s = model.quantize_q4s(kat)
    assert np.array_equal(p, golden["kat_q4s_packed"]) and np.array_equal(s, golden["kat_q4s_scales"].view(np.uint16))


def test_tiny_model_tensors_match_pinned_hashes(golden):
    import hashlib

    from _tiny import engine_tensors, oracle_name_to_tid, tiny_fp32

    w = tiny_fp32()
    t = engine_tensors(w)
    for name, h in zip(golden["weight_names"], golden["weight_sha256"]):
        tid = oracle_name_to_tid(str(name))
        d = hashlib.sha256()
        for i in (tid if isinstance(tid, tuple) else (tid,)):
            d.update(t[i])
        assert d.hexdigest() == str(h), name


def decode_tiles(fmt, packed, n_rows, k):
    """numpy decoder of the device tile layout (independent of the CUDA value functions).

    Units of 16 rows x 64 columns, stored slice-major: K is split into `slices` slices (16 for
    q4s, 8 for q8); unit (tile, kk) of slice w = kk // ku lives at ((w * tiles + tile) * ku + kk % ku).
    """
    q4 = fmt in (L.FMT_Q4S, L.FMT_Q4)
    ub = 576 if q4 else 1088
    wb = 512 if q4 else 1024
    slices = 16 if q4 else 8
    upt, tiles = k // 64, n_rows // 16
    ku = upt // slices
    raw = packed.reshape(slices, tiles, ku, ub)
    units = raw.transpose(1, 0, 2, 3).reshape(tiles, upt, ub)  # [tile][kk]
    out = np.zeros((n_rows, k), np.float32)
    lanes = np.arange(32)
    g, t = lanes >> 2, lanes & 3
    for step in range(4):
        for (dk, rowoff) in ((0, 0), (1, 0), (8, 0), (9, 0), (0, 8), (1, 8), (8, 8), (9, 8)):
            kin = step * 16 + 2 * t + dk
            if q4:
                words = units[:, :, :wb].reshape(tiles, upt, 32, 4, 4)[:, :, :, step, :].copy().view(np.uint32)[..., 0]
                shift = (dk & 1) * 16 + (dk >> 3) * 8 + (rowoff >> 3) * 4
                u = ((words >> shift) & 0xF).astype(np.int32) - (8 if fmt == L.FMT_Q4S else 0)
            else:
                grp16 = units[:, :, (step >> 1) * 512:(step >> 1) * 512 + 512].reshape(tiles, upt, 32, 16)
                byte = (step & 1) * 8 + (dk >> 3) * 4 + (dk & 1) * 2 + (rowoff >> 3)
                u = grp16[..., byte].astype(np.int32) - 128
            rows = (np.arange(tiles)[:, None, None] * 16 + g[None, None, :] + rowoff)
            cols = np.arange(upt)[None, :, None] * 64 + kin[None, None, :]
            if fmt == L.FMT_Q4:  # affine: (scale, bias) of rows g, g+8 for the unit's 64 columns
                sb = units[:, :, wb:wb + 64].reshape(tiles, upt, 8, 2, 4).copy().view(np.float16)
                sb = sb.reshape(tiles, upt, 8, 2, 2)[:, :, g, rowoff >> 3, :].astype(np.float32)
                val = sb[..., 0] * u + sb[..., 1]
            else:
                sc = units[:, :, wb:wb + 64].reshape(tiles, upt, 8, 2, 4).copy().view(np.float16)
                grp = kin >> 5
                s = sc[:, :, g, grp, (rowoff >> 3)]  # [tiles, upt, 32]
                val = s.astype(np.float32) * u
            out[np.broadcast_to(rows, u.shape), np.broadcast_to(cols, u.shape)] = val
    return out


@pytest.mark.parametrize("fmt", [L.FMT_Q4S, L.FMT_Q8, L.FMT_Q4])
def test_pack_layout_roundtrip(fmt):
    rows, k = 48, 2048
    w = (np.random.default_rng(3).standard_normal((rows, k)) * 0.02).astype(np.float32)
    if fmt == L.FMT_Q4S:
        codes, scales = model.quantize_q4s(w)
        ref = O.dequant_q4s(codes, scales.view(np.float16))
    elif fmt == L.FMT_Q4:  # reference affine q4 (the oracle's quantizer makes the test codes)
        codes, sb = O.quantize_q4_affine(w)
        scales = np.ascontiguousarray(sb).view(np.uint16)
        ref = O.dequant_q4_affine(codes, sb)
    else:
        codes, scales = model.quantize_q8(w)
        ref = O.dequant_q8(codes, scales.view(np.float16))
    nbytes = L.lib().icua_packed_bytes(fmt, rows, k)
    assert nbytes == rows // 16 * k // 64 * (1088 if fmt == L.FMT_Q8 else 576)
    out = np.zeros(nbytes, np.uint8)
    L.check(L.lib().icua_pack_matrix(fmt, rows, k, codes.ctypes.data, scales.ctypes.data, out.ctypes.data))
    assert np.array_equal(decode_tiles(fmt, out, rows, k), ref)


def test_icua_file_layout(tmp_path):
    tensors = {L.TID_FINAL_NORM: np.arange(2048, dtype=np.float32).tobytes(), 400: b"\x01" * 100}
    p = tmp_path / "m.icua"
    model.write_icua(str(p), tensors)
    raw = p.read_bytes()
    assert len(raw) % 16384 == 0
    magic, ver, fmt, count = struct.unpack_from("<IIII", raw, 0)
    assert (magic, ver, fmt, count) == (0x31554349, 1, L.FMT_Q4S, 710)
    off, size = struct.unpack_from("<QQ", raw, 16 + 16 * L.TID_FINAL_NORM)
    assert off % 256 == 0 and size == 8192 and raw[off:off + size] == tensors[L.TID_FINAL_NORM]
    off2, size2 = struct.unpack_from("<QQ", raw, 16 + 16 * 400)
    assert off2 % 256 == 0 and off2 >= off + size and size2 == 100


def test_invalid_arguments_are_errors_not_crashes():
    lib = L.lib()
    assert lib.icua_quantize_q8(None, 1, 32, None, None) == L.ERR_INVALID
    assert lib.icua_packed_bytes(L.FMT_Q4S, 15, 1024) == 0
    assert lib.icua_packed_bytes(L.FMT_Q4S, 16, 512) == 0  # K must split into the 16 slices
    assert lib.icua_packed_bytes(L.FMT_F16, 16, 64) == 0
    cfg = L.IcuaConfig()
    lib.icua_default_config(C.byref(cfg))
    assert (cfg.n_layers, cfg.vocab, cfg.max_context, cfg.max_pass, cfg.max_steps) == (28, 151936, 2048, 512, 256)
    cfg.format = 7  # no such weight format (0 f16, 1 q8, 2 affine q4, 3 q4s are all loadable)
    h = C.c_void_p()
    assert lib.icua_engine_create(C.byref(cfg), C.byref(h)) == L.ERR_UNSUPPORTED
    assert b"format" in lib.icua_global_error()
