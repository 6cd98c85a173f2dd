"""GPU parity of the persistent decode kernel (decode_mk_kernel: every decoder layer of a step in one
cooperative launch; opt-in with ICUA_DECODE=mk when the weights are loaded).

The same bars as the launch-chain path: the engine against the reference's own oracle on the pin
model (teacher-forced logits within max-abs 2e-2 / cosine 0.999, the reference's argmax at every
step; see tests/test_gpu_refpin.py), and a long-context decode at 2048 cached bf16 positions
against the numpy oracle through the CUDA-graph path.
"""
import os

import numpy as np
import pytest

import _refpin as P
from instantcua_b200 import Engine
from oracle import qwen3vl_oracle as O

pytestmark = pytest.mark.gpu
FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_ref.npz")


def _mk_engine(monkeypatch, tensors, **kw):
    monkeypatch.setenv("ICUA_DECODE", "mk")
    e = Engine(tensors=tensors, **kw)
    monkeypatch.delenv("ICUA_DECODE")
    assert e.kernels_per_step == 3, "the persistent kernel is not in use on this device"
    return e


def test_persistent_kernel_matches_reference(require_gpu, monkeypatch):
    fx = dict(np.load(FIXTURE))
    e = _mk_engine(monkeypatch, P.engine_tensors(), max_context=256, max_pass=64, max_steps=16, kv_dtype="f16")
    e.stop_on_eos = False
    ids = fx["sample_ids"]
    for case in P.CASES:
        prefix, suffix, pooler, deepstack = P.case_inputs(case)
        gh, gw = P.CASES[case]["grid"]
        n_vis = gh * gw
        ref = fx[f"{case}.gen_tokens"].tolist()
        e.reset()
        first = e.prefill(np.asarray(fx[f"{case}.input_ids"], np.int32), pooler=pooler if n_vis else None,
                          deepstack=deepstack if n_vis else None, grid=(gh, gw), write_logits=True)
        toks = [first]
        for s in range(len(ref)):
            lg = e.logits()
            top = fx[f"{case}.top_ids"][s]
            got = np.concatenate([lg[ids], lg[top]])
            want = np.concatenate([fx[f"{case}.sampled"][s], fx[f"{case}.top_vals"][s]])
            err, cos = float(np.abs(got - want).max()), O.cos_sim(got, want)
            assert err <= 2e-2 and cos >= 0.999, (case, s, err, cos)
            if s + 1 < len(ref):
                toks.append(e.decode_step(ref[s]))
        assert toks == ref, case
    e.close()


def test_persistent_kernel_long_context_graph_decode(require_gpu, monkeypatch):
    from _tiny import engine_tensors, tiny_fp32

    w32 = tiny_fp32()
    wq = {k: (v if v.ndim == 1 else (O.dequant_q8(*O.quantize_q8(v)) if k == "embed" else O.dequant_q4s(*O.quantize_q4s(v))))
          for k, v in w32.items()}
    ctx, steps = 2048, 12
    rng = np.random.default_rng(9)
    k = rng.standard_normal((2, ctx, 8, 128), dtype=np.float32)
    v = rng.standard_normal((2, ctx, 8, 128), dtype=np.float32)
    e = _mk_engine(monkeypatch, engine_tensors(w32), n_layers=2, vocab=1024, max_context=ctx + 64, max_pass=16,
                   max_steps=64, kv_dtype="bf16", steps_per_graph=4)
    e.stop_on_eos = False
    e.inject_kv(k, v)
    cur = 17
    t1 = e.decode_step(cur)
    lg1 = e.logits()
    cap = e.capture_step_logits(steps - 1)
    rest = e.decode(steps - 1)
    e.close()
    toks = [t1] + rest
    logits = np.concatenate([lg1[None], cap])
    m = O.TextModel(wq, kv_dtype="bf16")
    m.inject_kv(list(k), list(v))
    x = m.prefill(np.asarray([cur] + toks[:-1]), return_hidden=True)
    want = m.logits(x)
    err = np.abs(logits - want).max()
    assert err <= 2e-2, err
    assert (want.argmax(axis=1) == np.asarray(toks)).mean() >= 0.99
