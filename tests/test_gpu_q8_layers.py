"""GPU parity of a model whose decoder layers are q8 (the reference's `--format q8` files, FMT 1:
int8 codes + fp16 scale per 32 columns, Convert.swift:215-241): batch-1 decode through the
streaming q8 GEMV, the tensor-core prefill (q8 dequantised to fp16), and the batched step (fused
q8 dequant-GEMM), each against the numpy oracle on the same dequantized weights.
Bar (BASELINE): logits max-abs <= 2e-2, cosine >= 0.999; identical greedy tokens.
"""
import numpy as np
import pytest

from instantcua_b200 import Engine, model
from instantcua_b200 import _lib as L
from oracle import qwen3vl_oracle as O
from oracle.qwen3vl_oracle import cos_sim

pytestmark = pytest.mark.gpu

ATOL = 2e-2
COS = 0.999


@pytest.fixture(scope="module")
def q8_model(require_gpu):
    from _tiny import fp32_stream, tiny_fp32

    w32 = tiny_fp32()
    tensors = model.quantize_stream(fp32_stream(w32), fmt=L.FMT_Q8)
    wq = {}
    for name, arr in w32.items():
        if arr.ndim == 1:
            wq[name] = arr
        else:
            wq[name] = O.dequant_q8(*O.quantize_q8(arr))
    return tensors, wq


def make(tensors, **kw):
    args = dict(n_layers=2, vocab=1024, max_context=512, max_pass=128, max_steps=64, kv_dtype="f16",
                steps_per_graph=4, weight_format="q8")
    args.update(kw)
    e = Engine(tensors=tensors, **args)
    e.stop_on_eos = False
    return e


def check(got, want, tag):
    for i, (a, b) in enumerate(zip(got, want)):
        err = float(np.abs(a - b).max())
        assert err <= ATOL and cos_sim(a, b) >= COS, f"{tag} step {i}: max|d|={err}"
    return max(float(np.abs(a - b).max()) for a, b in zip(got, want))


@pytest.mark.parametrize("gemm_min", [0, 1])
def test_q8_layers_generation_matches_oracle(q8_model, gemm_min):
    tensors, wq = q8_model
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
    err = check(got, want_logits, f"q8 (gemm_min {gemm_min})")
    print(f"q8 layers, prefill_gemm_min {gemm_min}: max|d| {err:.3e}")
    assert want_tok == toks


def test_q8_layers_batched_matches_one_at_a_time(q8_model):
    tensors, _ = q8_model
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, 1024, int(rng.integers(5, 30))).astype(np.int32) for _ in range(3)]
    e = make(tensors, max_sessions=3)
    for s, p in enumerate(prompts):
        e.prefill(p, session=s)
    cap = e.capture_batch_logits(3)
    got = e.decode_batch([0, 1, 2], 4)
    gl = cap.copy()
    e.close()
    e = make(tensors, max_sessions=3)
    want, wl = [], []
    for s, p in enumerate(prompts):
        e.prefill(p, session=s)
        c = e.capture_step_logits(4)
        want.append(e.decode(4, session=s))
        wl.append(c[3].copy())
    e.close()
    check(gl, wl, "q8 batched")
    assert np.array_equal(np.array(want), got)
