"""GPU tests of the tensor-core prefill path (tcgen05 dequant-GEMM, causal prefill attention).

GEMM bar: y within 1e-5 of max|y| of a float64 product of the same fp16 operands (the kernel's
weights are half(q) * half(scale), its activations fp16, its accumulation fp32 over K up to 6144:
about sqrt(K) * 2^-24 relative), and every
one-hot activation row reproduces that fp16 weight column exactly.  Engine bar (BASELINE):
logits within max-abs 2e-2 and cosine >= 0.999 of the oracle, identical greedy tokens on the
tiny model, and the tensor-core and row-by-row prefill paths within the same bar of each other.
"""
import ctypes as C

import numpy as np
import pytest

from instantcua_b200 import Engine
from instantcua_b200 import _lib as L
from instantcua_b200 import model
from oracle import qwen3vl_oracle as O
from oracle.qwen3vl_oracle import cos_sim

pytestmark = pytest.mark.gpu

ATOL = 2e-2
COS = 0.999
GEMM_TOL = 1e-5


@pytest.fixture(scope="module")
def torch_cuda(require_gpu):
    import torch

    torch.cuda.init()
    return torch


def _packed_q4s(n, k, seed):
    w = (np.random.default_rng(seed).standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float32)
    codes, scales = model.quantize_q4s(w)
    exact = O.dequant_q4s(codes, scales.view(np.float16))  # float(scale) * q, exact in fp32
    buf = np.empty(L.lib().icua_packed_bytes(L.FMT_Q4S, n, k), np.uint8)
    L.check(L.lib().icua_pack_matrix(L.FMT_Q4S, n, k, codes.ctypes.data, scales.ctypes.data, buf.ctypes.data))
    return buf, exact.astype(np.float16)  # the kernel's weight values: one fp16 rounding of q * scale


def _gemm(torch, n, k, m, dev_w, x16, err=None):
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    L.check(L.lib().icua_gemm_q4s(n, k, m, C.c_void_p(dev_w.data_ptr()), C.c_void_p(x16.data_ptr()),
                                  C.c_void_p(y.data_ptr()), C.c_void_p(err.data_ptr()) if err is not None else None,
                                  None))
    torch.cuda.synchronize()
    return y


@pytest.mark.parametrize("n,k,m", [(4096, 2048, 200), (2048, 2048, 1), (12288, 2048, 128), (2048, 6144, 300),
                                   (256, 1024, 129)])
def test_gemm_matches_fp64(torch_cuda, n, k, m):
    torch = torch_cuda
    buf, w16 = _packed_q4s(n, k, seed=n + k + m)
    dev_w = torch.from_numpy(buf).cuda()
    x = np.random.default_rng(m).standard_normal((m, k), dtype=np.float32).astype(np.float16)
    x16 = torch.from_numpy(x).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = _gemm(torch, n, k, m, dev_w, x16, err).cpu().numpy()
    assert int(err.item()) == 0
    want = x.astype(np.float64) @ w16.astype(np.float64).T
    rel = np.abs(y - want).max() / np.abs(want).max()
    print(f"gemm {m}x{n}x{k}: max rel err {rel:.2e}")
    assert rel <= GEMM_TOL
    y2 = _gemm(torch, n, k, m, dev_w, x16).cpu().numpy()
    assert np.array_equal(y, y2)  # deterministic


@pytest.mark.parametrize("n,k", [(4096, 2048), (2048, 6144)])
def test_dequant_f16_bit_exact(torch_cuda, n, k):
    """The prefill path's dequantised operand equals fp16(float(scale) * q) element for element."""
    torch = torch_cuda
    buf, w16 = _packed_q4s(n, k, seed=5)
    dev_w = torch.from_numpy(buf).cuda()
    out = torch.empty((n, k), dtype=torch.float16, device="cuda")
    L.check(L.lib().icua_dequant_q4s_f16(n, k, C.c_void_p(dev_w.data_ptr()), C.c_void_p(out.data_ptr()), None))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint16), w16.view(np.uint16))


@pytest.mark.parametrize("n,k,m", [(4096, 2048, 1255), (2048, 6144, 300), (12288, 2048, 64)])
def test_gemm_f16_route_matches(torch_cuda, n, k, m):
    """Dequantise-then-TMA GEMM (the prefill route) against the fused-dequant GEMM and float64."""
    torch = torch_cuda
    buf, w16 = _packed_q4s(n, k, seed=n + m)
    dev_w = torch.from_numpy(buf).cuda()
    x = np.random.default_rng(m).standard_normal((m, k), dtype=np.float32).astype(np.float16)
    x16 = torch.from_numpy(x).cuda()
    wd = torch.empty((n, k), dtype=torch.float16, device="cuda")
    L.check(L.lib().icua_dequant_q4s_f16(n, k, C.c_void_p(dev_w.data_ptr()), C.c_void_p(wd.data_ptr()), None))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    L.check(L.lib().icua_gemm_f16(n, k, m, C.c_void_p(wd.data_ptr()), C.c_void_p(x16.data_ptr()),
                                  C.c_void_p(y.data_ptr()), C.c_void_p(err.data_ptr()), None))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    y = y.cpu().numpy()
    want = x.astype(np.float64) @ w16.astype(np.float64).T
    rel = np.abs(y - want).max() / np.abs(want).max()
    fused = _gemm(torch, n, k, m, dev_w, x16).cpu().numpy()
    print(f"gemm_f16 {m}x{n}x{k}: max rel err {rel:.2e}, max |f16 route - fused| {np.abs(y - fused).max():.2e}")
    assert rel <= GEMM_TOL
    assert np.array_equal(y, fused)


def test_gemm_one_hot_rows_exact(torch_cuda):
    """Activation row t = e_j gives output row t = fp16 weight column j, exactly."""
    torch = torch_cuda
    n, k = 512, 2048
    buf, w16 = _packed_q4s(n, k, seed=3)
    dev_w = torch.from_numpy(buf).cuda()
    cols = [0, 1, 7, 8, 15, 16, 31, 32, 63, 64, 100, 511, 1024, 2047]
    x = np.zeros((len(cols), k), np.float16)
    for t, j in enumerate(cols):
        x[t, j] = 1.0
    y = _gemm(torch, n, k, len(cols), dev_w, torch.from_numpy(x).cuda()).cpu().numpy()
    for t, j in enumerate(cols):
        assert np.array_equal(y[t], w16[:, j].astype(np.float32)), j


def test_gemm_rejects_bad_shapes(torch_cuda):
    torch = torch_cuda
    w = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    x = torch.zeros(4096, dtype=torch.float16, device="cuda")
    y = torch.zeros(4096, dtype=torch.float32, device="cuda")
    for n, k, m in [(100, 2048, 1), (128, 1000, 1), (128, 2048, 0), (128, 8192, 1)]:
        assert L.lib().icua_gemm_q4s(n, k, m, C.c_void_p(w.data_ptr()), C.c_void_p(x.data_ptr()),
                                     C.c_void_p(y.data_ptr()), None, None) == L.ERR_INVALID


# ---- engine: tiny model through the tensor-core prefill ----------------------------------------
@pytest.fixture(scope="module")
def tensors():
    from _tiny import engine_tensors

    return engine_tensors()


def make_engine(tensors, kv="f16", gemm_min=1, **kw):
    args = dict(n_layers=2, vocab=1024, max_context=512, max_pass=256, max_steps=64, kv_dtype=kv, steps_per_graph=4,
                prefill_gemm_min=gemm_min)
    args.update(kw)
    e = Engine(tensors=tensors, **args)
    e.stop_on_eos = False
    return e


def check_logits(got, want, tag):
    for i, (a, b) in enumerate(zip(got, want)):
        err = float(np.abs(a - b).max())
        c = cos_sim(a, b)
        assert err <= ATOL and c >= COS, f"{tag} step {i}: max|d|={err} cos={c}"
    return max(float(np.abs(a - b).max()) for a, b in zip(got, want))


@pytest.mark.parametrize("kv", ["f16", "bf16"])
def test_text_prefill_gemm_matches_oracle(golden, tensors, kv):
    e = make_engine(tensors, kv=kv)
    steps = len(golden[f"text_{kv}_gen"])
    cap = e.capture_step_logits(steps)
    first = e.prefill(golden["text_tokens"], write_logits=True)
    first_logits = cap[0].copy()
    rest = e.decode(steps - 1)
    assert [first] + rest == golden[f"text_{kv}_gen"].tolist()
    got = np.concatenate([first_logits[None], cap[: steps - 1]])
    err = check_logits(got, golden[f"text_{kv}_logits"], kv)
    print(f"tensor-core prefill ({kv}): max|d| vs oracle {err:.3e}")
    e.close()


def test_multimodal_prefill_gemm_matches_oracle(golden, tensors):
    e = make_engine(tensors)
    steps = len(golden["mm_gen"])
    cap = e.capture_step_logits(steps)
    first = e.prefill(golden["mm_tokens"], pooler=golden["mm_pooler"], deepstack=list(golden["mm_deepstack"]),
                      grid=tuple(golden["mm_grid"].tolist()), write_logits=True)
    first_logits = cap[0].copy()
    rest = e.decode(steps - 1)
    assert [first] + rest == golden["mm_gen"].tolist()
    got = np.concatenate([first_logits[None], cap[: steps - 1]])
    err = check_logits(got, golden["mm_logits"], "multimodal")
    print(f"tensor-core prefill (multimodal): max|d| vs oracle {err:.3e}")
    e.close()


@pytest.mark.parametrize("kv", ["f16", "bf16"])
def test_gemm_and_row_prefill_agree_long_prompt(tensors, kv):
    """A 200-token prompt after a 40-token first turn (cache slots 40..239: the attention reads
    earlier turns and crosses several 64-row blocks), through both prefill paths."""
    rng = np.random.default_rng(9)
    turn1 = rng.integers(0, 1024, 40).astype(np.int32)
    turn2 = rng.integers(0, 1024, 200).astype(np.int32)
    outs = []
    for gemm_min in (1, 0):
        e = make_engine(tensors, kv=kv, gemm_min=gemm_min)
        e.prefill(turn1)
        cap = e.capture_step_logits(4)
        e.prefill(turn2, write_logits=True)
        first = cap[0].copy()
        rest = e.decode(3)
        outs.append((first, np.concatenate([first[None], cap[:3]]), rest))
        e.close()
    (fa, la, ta), (fb, lb, tb) = outs
    err = check_logits(la, lb, f"gemm vs rows ({kv})")
    print(f"gemm vs row prefill ({kv}): max|d| {err:.3e}")
    assert ta == tb
