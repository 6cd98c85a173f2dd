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


def test_wait_timeout_reports_and_engine_stays_failed(require_gpu):
    """A bounded device wait that gives up is reported, not hidden: with the GEMV's norm-weight wait
    limited to 0 polls the decode kernels flag the step (after still waiting, with the default
    bound, for their copies), the call returns ICUA_ERR_TIMEOUT, the engine refuses later calls
    with ICUA_ERR_STATE, and a new engine works once the limit is back (the context is usable)."""
    from _tiny import engine_tensors

    tensors = engine_tensors()
    lib = L.lib()
    prompt = np.arange(20, dtype=np.int32)
    e = make(tensors)
    try:
        L.check(lib.icua_set_wait_limit(0))
        with pytest.raises(L.IcuaError) as ei:
            e.generate_vision(prompt, 4)
        assert ei.value.status == L.ERR_TIMEOUT
        assert "bounded device wait" in str(ei.value)
    finally:
        L.check(lib.icua_set_wait_limit(1 << 22))
    with pytest.raises(L.IcuaError) as ei:
        e.generate_vision(prompt, 4)
    assert ei.value.status == L.ERR_STATE
    e.close()
    e2 = make(tensors)
    assert len(e2.generate_vision(prompt, 4)) == 4
    e2.close()
