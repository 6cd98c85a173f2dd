"""The oracle against the reference's own oracle (CPU).

``tests/golden/golden_ref.npz`` holds the outputs of the reference's ``qwen3vl_ref.py`` itself
(``Qwen3VLRef.generate``, tools/reference/qwen3vl_ref.py:218-336), run unmodified on the pin model
of ``tests/_refpin.py`` through a numpy stand-in for ``mlx.core`` (``tests/golden/make_golden_ref.py``).
This test re-runs ``oracle/qwen3vl_oracle.py`` on the same model and prompts and requires the
reference's tokens, input ids and rope_delta exactly, and its logits within 1e-5 at the sampled ids
and the top 32 of every step.
"""
import os

import numpy as np
import pytest

import _refpin as P
from oracle import qwen3vl_oracle as O

FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_ref.npz")


@pytest.fixture(scope="module")
def pin():
    return P.pin_dequantized(), dict(np.load(FIXTURE))


@pytest.mark.parametrize("case", list(P.CASES))
def test_oracle_reproduces_reference(pin, case):
    w, fx = pin
    ids = fx["sample_ids"]
    assert np.array_equal(ids, P.sample_ids())
    prefix, suffix, pooler, deepstack = P.case_inputs(case)
    gh, gw = P.CASES[case]["grid"]
    n_vis = gh * gw
    tokens = prefix + [O.IMAGE_PAD] * n_vis + suffix
    assert np.array_equal(np.asarray(tokens), fx[f"{case}.input_ids"])
    m = O.TextModel(w)
    toks, logits = m.generate(tokens, P.CASES[case]["new"], stop_on_eos=True, pooler=pooler if n_vis else None,
                              deepstack=deepstack if n_vis else None, llm_hw=(gh, gw))
    assert toks == fx[f"{case}.gen_tokens"].tolist()
    assert m.rope_delta == int(fx[f"{case}.rope_delta"])
    for s, lg in enumerate(logits):
        assert np.abs(lg[ids] - fx[f"{case}.sampled"][s]).max() <= 1e-5
        top = fx[f"{case}.top_ids"][s]
        assert np.abs(lg[top] - fx[f"{case}.top_vals"][s]).max() <= 1e-5
        l64 = lg.astype(np.float64)
        assert np.allclose([l64.sum(), (l64 * l64).sum()], fx[f"{case}.sums"][s], rtol=1e-5, atol=1e-3)
