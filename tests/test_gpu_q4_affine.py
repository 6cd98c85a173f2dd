"""GPU parity of a model in the reference's q4 format (FMT 2, Convert.swift:246-320): codes 0..15
with an fp16 (scale, bias) per 64 columns for every matrix, the tied embedding / lm_head
included.  Batch-1 decode (q4a GEMV, q4a lm_head), the tensor-core prefill (affine dequant to
fp16) and the batched step (fused affine dequant-GEMM) against the numpy oracle on the same
dequantized weights (value = scale * q + bias, Shaders.swift:471-476).

The test's codes come from a plain min / max affine fit (fast); the engine only reads the format,
so the reference converter's MSE clip search (oracle.quantize_q4_affine) is not needed here.
Bar (BASELINE): logits max-abs <= 2e-2, cosine >= 0.999; identical greedy tokens.
"""
import numpy as np
import pytest

from instantcua_b200 import Engine
from instantcua_b200 import _lib as L
from oracle import qwen3vl_oracle as O
from oracle.qwen3vl_oracle import cos_sim

pytestmark = pytest.mark.gpu

ATOL = 2e-2
COS = 0.999


def affine_q4(w):
    rows, cols = w.shape
    g = w.reshape(rows, cols // 64, 64)
    lo, hi = g.min(axis=2), g.max(axis=2)
    s = ((hi - lo) / 15).astype(np.float16)
    b = lo.astype(np.float16)
    sf = np.where(s.astype(np.float32) > 0, s.astype(np.float32), 1.0)[..., None]
    u = np.clip(np.rint((g - b.astype(np.float32)[..., None]) / sf), 0, 15).astype(np.uint8).reshape(rows, cols)
    packed = (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)
    sb = np.stack([s, b], axis=-1)  # [rows, cols / 64, 2] fp16
    return packed, sb


@pytest.fixture(scope="module")
def q4a_model(require_gpu):
    from _tiny import oracle_name_to_tid, tiny_fp32

    w32 = tiny_fp32()
    tensors, wq = {}, {}
    for name, arr in w32.items():
        tid = oracle_name_to_tid(name)
        if arr.ndim == 1:
            tensors[tid] = np.ascontiguousarray(arr, np.float32).tobytes()
            wq[name] = arr
        else:
            packed, sb = affine_q4(arr)
            tensors[tid[0]] = packed.tobytes()
            tensors[tid[1]] = np.ascontiguousarray(sb).tobytes()
            wq[name] = O.dequant_q4_affine(packed, sb)
    return tensors, wq


def make(tensors, **kw):
    args = dict(n_layers=2, vocab=1024, max_context=512, max_pass=128, max_steps=64, kv_dtype="f16",
                steps_per_graph=4, weight_format="q4")
    args.update(kw)
    e = Engine(tensors=tensors, **args)
    e.stop_on_eos = False
    return e


@pytest.mark.parametrize("gemm_min", [0, 1])
def test_q4_affine_generation_matches_oracle(q4a_model, gemm_min):
    tensors, wq = q4a_model
    prompt = np.random.default_rng(3).integers(0, 1024, 40).astype(np.int32)
    steps = 6
    e = make(tensors, prefill_gemm_min=gemm_min)
    cap = e.capture_step_logits(steps)
    first = e.prefill(prompt, write_logits=True)
    first_logits = cap[0].copy()
    rest = e.decode(steps - 1)
    toks = [first] + rest
    got = np.concatenate([first_logits[None], cap[: steps - 1]])
    e.close()
    ref = O.TextModel(wq, kv_dtype="f16")
    want_tok, want_logits = ref.generate(prompt, steps, teacher=toks)
    worst = 0.0
    for i, (a, b) in enumerate(zip(got, want_logits)):
        err = float(np.abs(a - b).max())
        worst = max(worst, err)
        assert err <= ATOL and cos_sim(a, b) >= COS, f"step {i}: max|d|={err}"
    print(f"q4 affine, prefill_gemm_min {gemm_min}: max|d| {worst:.3e}")
    assert want_tok == toks


def test_q4_affine_batched_step(q4a_model):
    tensors, _ = q4a_model
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, 1024, int(rng.integers(5, 30))).astype(np.int32) for _ in range(3)]
    eb, e1 = make(tensors, max_sessions=3), make(tensors, max_sessions=3)
    first = []
    for s, p in enumerate(prompts):
        eb.prefill(p, session=s)
        first.append(e1.prefill(p, session=s))
    cap = eb.capture_batch_logits(3)
    got = eb.decode_batch([0, 1, 2], 1, in_tokens=first)[:, 0]
    for s in range(3):
        t = e1.decode_step(first[s], session=s)
        want = e1.logits()
        err = float(np.abs(cap[s] - want).max())
        assert err <= ATOL and cos_sim(cap[s], want) >= COS, f"session {s}: max|d|={err}"
        assert got[s] == t or abs(want[got[s]] - want[t]) <= 2 * ATOL
    eb.close()
    e1.close()
