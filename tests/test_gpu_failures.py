"""Failure paths of the token loop that must end in an error status, not in an invalid memory
access: a step whose logits have no finite value (here: an all-NaN final norm weight) stops the
session with ICUA_ERR_STATE before the next step could embed an id outside the vocabulary."""
import numpy as np
import pytest

from instantcua_b200 import Engine
from instantcua_b200 import _lib as L

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nan_tensors(require_gpu):
    from _tiny import engine_tensors, tiny_fp32

    w = tiny_fp32()
    w["final_norm"] = np.full_like(w["final_norm"], np.nan)
    return engine_tensors(w)


def make(tensors, **kw):
    args = dict(n_layers=2, vocab=1024, max_context=256, max_pass=64, max_steps=16, steps_per_graph=4)
    args.update(kw)
    e = Engine(tensors=tensors, **args)
    e.stop_on_eos = False
    return e


def test_nan_logits_stop_batch1_decode(nan_tensors):
    e = make(nan_tensors)
    prompt = np.arange(20, dtype=np.int32)
    with pytest.raises(L.IcuaError, match="no finite logit"):
        e.generate_vision(prompt, 4)
    e.close()


def test_nan_logits_stop_batched_decode(nan_tensors):
    e = make(nan_tensors, max_sessions=4)
    with pytest.raises(L.IcuaError, match="no finite logit"):
        e.decode_batch([0, 1, 2, 3], 3, in_tokens=np.array([1, 2, 3, 4], np.int32))
    e.close()
