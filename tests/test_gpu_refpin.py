"""The CUDA engine against the reference's own oracle (GPU).

``tests/golden/golden_ref.npz`` holds what ``tools/reference/qwen3vl_ref.py`` (the reference's
Qwen3VLRef.generate, qwen3vl_ref.py:218-336, run unmodified through a numpy stand-in for
``mlx.core``) produced on the pin model of ``tests/_refpin.py``: 28 full-width layers, the full
151936-row tied embedding, q4s decoder / q8 embedding values, a text prompt and two multimodal
prompts with DeepStack and 3-D M-RoPE.  The engine loads the same quantized model.

* Teacher-forced: the prompt through ``icua_prefill``, then each of the reference's tokens through
  ``icua_decode_step``; every step's logits must be within max-abs 2e-2 and cosine 0.999 of the
  reference's (at the fixture's 4096 sampled ids and each step's top 32) and the argmax must be the
  reference's token.
* Free-running: ``icua_generate`` (prefill + the decode graph) must produce the reference's tokens;
  a step where the two differ is accepted only when the reference's own top-1 / top-2 margin there
  is below twice the logit tolerance (a near tie), and the comparison ends at that step.
"""
import os

import numpy as np
import pytest

import _refpin as P
from instantcua_b200 import Engine
from oracle import qwen3vl_oracle as O

pytestmark = pytest.mark.gpu

ATOL = 2e-2
COS = 0.999
FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_ref.npz")


@pytest.fixture(scope="module")
def pinned(require_gpu):
    fx = dict(np.load(FIXTURE))
    e = Engine(tensors=P.engine_tensors(), max_context=256, max_pass=64, max_steps=16, kv_dtype="f16")
    yield e, fx
    e.close()


def _check_step(lg, fx, case, s):
    ids = fx["sample_ids"]
    top = fx[f"{case}.top_ids"][s]
    got = np.concatenate([lg[ids], lg[top]])
    want = np.concatenate([fx[f"{case}.sampled"][s], fx[f"{case}.top_vals"][s]])
    err = float(np.abs(got - want).max())
    cos = O.cos_sim(got, want)
    return err, cos


@pytest.mark.parametrize("case", list(P.CASES))
def test_teacher_forced_matches_reference(pinned, case):
    e, fx = pinned
    prefix, suffix, pooler, deepstack = P.case_inputs(case)
    gh, gw = P.CASES[case]["grid"]
    n_vis = gh * gw
    tokens = np.asarray(fx[f"{case}.input_ids"], np.int32)
    ref = fx[f"{case}.gen_tokens"].tolist()
    e.stop_on_eos = False
    e.reset()
    first = e.prefill(tokens, pooler=pooler if n_vis else None, deepstack=deepstack if n_vis else None,
                      grid=(gh, gw), write_logits=True)
    errs, coss, agree = [], [], [first == ref[0]]
    err, cos = _check_step(e.logits(), fx, case, 0)
    errs.append(err)
    coss.append(cos)
    for s in range(1, len(ref)):
        t = e.decode_step(ref[s - 1])
        agree.append(t == ref[s])
        err, cos = _check_step(e.logits(), fx, case, s)
        errs.append(err)
        coss.append(cos)
    print(f"{case}: max|d| {max(errs):.3e}, min cos {min(coss):.6f}, argmax agreement {np.mean(agree):.3f}")
    assert max(errs) <= ATOL and min(coss) >= COS
    assert all(agree)


@pytest.mark.parametrize("case", list(P.CASES))
def test_free_running_generate_matches_reference(pinned, case):
    e, fx = pinned
    prefix, suffix, pooler, deepstack = P.case_inputs(case)
    gh, gw = P.CASES[case]["grid"]
    n_vis = gh * gw
    tokens = np.asarray(fx[f"{case}.input_ids"], np.int32)
    ref = fx[f"{case}.gen_tokens"].tolist()
    e.stop_on_eos = True  # the reference stops on its EOS pair (qwen3vl_ref.py:304, 335)
    e.use_prefix_cache = False
    got = e.generate_vision(tokens, len(ref), pooler=pooler if n_vis else None,
                            deepstack=deepstack if n_vis else None, grid=(gh, gw))
    for s, (a, b) in enumerate(zip(got, ref)):
        if a != b:
            vals = fx[f"{case}.top_vals"][s]
            margin = float(vals[0] - vals[1])
            print(f"{case}: step {s} engine {a} reference {b}, reference top-1/top-2 margin {margin:.4f}")
            assert margin < 2 * ATOL
            return
    assert len(got) == len(ref)
