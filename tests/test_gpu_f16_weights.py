"""GPU parity of a model in the reference converter's default format (FMT 0: every matrix fp16,
no scales).  Such engines run every matrix on the tensor-core GEMM (fp16 operands straight from
the file, TMA-fed): prefill rows, and batch-1 decode as a one-row batched step.  Against the numpy
oracle on the same fp16-rounded weights; bar (BASELINE): logits max-abs <= 2e-2, cosine >= 0.999
per step, identical greedy tokens (teacher-forced).
"""
import numpy as np
import pytest

from instantcua_b200 import Engine, IcuaError, model
from instantcua_b200 import _lib as L
from oracle import qwen3vl_oracle as O
from oracle.qwen3vl_oracle import cos_sim

pytestmark = pytest.mark.gpu

ATOL = 2e-2
COS = 0.999


@pytest.fixture(scope="module")
def f16_model(require_gpu):
    from _tiny import fp32_stream, tiny_fp32

    w32 = tiny_fp32()
    tensors = model.quantize_stream(fp32_stream(w32), fmt=L.FMT_F16)
    wq = {k: (v if v.ndim == 1 else v.astype(np.float16).astype(np.float32)) for k, v in w32.items()}
    return tensors, wq


def make(tensors, **kw):
    args = dict(n_layers=2, vocab=1024, max_context=512, max_pass=128, max_steps=64, kv_dtype="f16",
                steps_per_graph=4, weight_format="f16")
    args.update(kw)
    e = Engine(tensors=tensors, **args)
    e.stop_on_eos = False
    return e


def test_f16_weights_generation_matches_oracle(f16_model):
    tensors, wq = f16_model
    prompt = np.random.default_rng(3).integers(0, 1024, 40).astype(np.int32)
    steps = 6
    e = make(tensors)
    toks = [e.prefill(prompt, write_logits=True)]
    logits = [e.logits()]
    for _ in range(steps - 1):
        toks.append(e.decode_step(toks[-1]))
        logits.append(e.logits())
    cont = e.decode(3)  # the graph-launched loop continues the same session
    assert len(cont) == 3
    e.close()
    ref = O.TextModel(wq, kv_dtype="f16")
    want_tok, want_logits = ref.generate(prompt, steps, teacher=toks)
    worst = 0.0
    for i, (a, b) in enumerate(zip(logits, want_logits)):
        err = float(np.abs(a - b).max())
        worst = max(worst, err)
        assert err <= ATOL and cos_sim(a, b) >= COS, f"step {i}: max|d|={err}"
    print(f"f16 weights: max|d| {worst:.3e}")
    assert want_tok == toks


def test_f16_weights_reject_visual_last_token(f16_model):
    tensors, _ = f16_model
    e = make(tensors)
    with pytest.raises(IcuaError):
        e.prefill(np.array([1, 2, 151655], np.int32), pooler=np.zeros((1, 2048), np.float32), grid=(1, 1))
    e.close()
