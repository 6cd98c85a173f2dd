"""GPU parity of the whole token loop (prefill + greedy decode) against the oracle fixtures.

Tiny model (2 layers, full width, 1024-row vocabulary).  Bars: identical greedy tokens; per-step
logits within max-abs 2e-2 and cosine >= 0.999 of the oracle run with the same KV storage type
(BASELINE tolerance), and within 2e-2 of the fp32-KV oracle as well.
"""
import numpy as np
import pytest

from instantcua_b200 import Engine, IcuaError
from instantcua_b200 import _lib as L
from oracle.qwen3vl_oracle import cos_sim

pytestmark = pytest.mark.gpu

ATOL = 2e-2
COS = 0.999


@pytest.fixture(scope="module")
def tensors():
    from _tiny import engine_tensors

    return engine_tensors()


def make_engine(tensors, kv="f16", **kw):
    args = dict(n_layers=2, vocab=1024, max_context=512, max_pass=64, max_steps=64, kv_dtype=kv, steps_per_graph=4)
    args.update(kw)
    e = Engine(tensors=tensors, **args)
    e.stop_on_eos = False
    return e


def check_logits(got, want, tag):
    for i, (a, b) in enumerate(zip(got, want)):
        err = float(np.abs(a - b).max())
        c = cos_sim(a, b)
        assert err <= ATOL and c >= COS, f"{tag} step {i}: max|d|={err} cos={c}"


@pytest.mark.parametrize("kv", ["f16", "bf16"])
def test_text_generation_matches_oracle(require_gpu, golden, tensors, kv):
    e = make_engine(tensors, kv=kv)
    steps = len(golden[f"text_{kv}_gen"])
    cap = e.capture_step_logits(steps)
    first = e.prefill(golden["text_tokens"], write_logits=True)
    first_logits = cap[0].copy()
    rest = e.decode(steps - 1)
    toks = [first] + rest
    assert toks == golden[f"text_{kv}_gen"].tolist()
    got = np.concatenate([first_logits[None], cap[: steps - 1]])
    check_logits(got, golden[f"text_{kv}_logits"], kv)
    check_logits(got, golden["text_f32_logits"], kv + " vs fp32-KV oracle")
    np.testing.assert_array_equal(e.logits(), first_logits)
    print(kv, "max|d| vs oracle:", float(np.abs(got - golden[f"text_{kv}_logits"]).max()))
    e.close()


def test_generate_vision_api_and_determinism(require_gpu, golden, tensors):
    e = make_engine(tensors)
    n = len(golden["text_f16_gen"])
    a = e.generate_vision(golden["text_tokens"], max_new_tokens=n, write_first_logits=True)
    la = e.logits()
    b = e.generate_vision(golden["text_tokens"], max_new_tokens=n, write_first_logits=True)
    assert a == b == golden["text_f16_gen"].tolist()
    assert np.array_equal(la, e.logits())
    t = e.last_timing
    assert t.prefill_tokens == len(golden["text_tokens"]) and t.generated_tokens == n and t.prefill_ms > 0
    e.close()


def test_multimodal_deepstack_matches_oracle(require_gpu, golden, tensors):
    e = make_engine(tensors)
    steps = len(golden["mm_gen"])
    cap = e.capture_step_logits(steps)
    first = e.prefill(golden["mm_tokens"], pooler=golden["mm_pooler"], deepstack=list(golden["mm_deepstack"]),
                      grid=tuple(golden["mm_grid"].tolist()), write_logits=True)
    first_logits = cap[0].copy()
    rest = e.decode(steps - 1)
    assert [first] + rest == golden["mm_gen"].tolist()
    got = np.concatenate([first_logits[None], cap[: steps - 1]])
    # the fixture's oracle kept fp32 K/V; the engine stores fp16
    check_logits(got, golden["mm_logits"], "multimodal")
    e.close()


def test_decode_step_matches_decode(require_gpu, golden, tensors):
    e = make_engine(tensors)
    first = e.prefill(golden["text_tokens"])
    want = golden["text_f16_gen"].tolist()
    assert first == want[0]
    toks = [first]
    for _ in range(len(want) - 1):
        toks.append(e.decode_step(toks[-1]))
    assert toks == want
    assert e.position() == len(golden["text_tokens"]) + len(want) - 1
    e.close()


def test_eos_stop_truncates(require_gpu, golden, tensors):
    e = make_engine(tensors)
    want = golden["text_f16_gen"].tolist()
    e.stop_on_eos = True
    e.eos = (want[3], want[3])
    got = e.generate_vision(golden["text_tokens"], max_new_tokens=len(want))
    assert got == want[:3]
    e.close()


def test_error_paths(require_gpu, golden, tensors):
    e = make_engine(tensors)
    with pytest.raises(IcuaError) as ex:
        e.prefill([5, 2000, 7])  # token beyond the 1024-row vocabulary
    assert ex.value.status == L.ERR_INVALID
    with pytest.raises(IcuaError) as ex:
        e.prefill(list(range(65)))  # longer than max_pass
    assert ex.value.status == L.ERR_CAPACITY
    with pytest.raises(IcuaError) as ex:
        e.decode(4)  # nothing prefilled yet
    assert ex.value.status == L.ERR_STATE
    with pytest.raises(IcuaError) as ex:
        e.prefill([1, 151655, 3])  # IMAGE_PAD without visual rows
    assert ex.value.status == L.ERR_INVALID
    # the engine stays usable after rejected calls
    assert e.generate_vision(golden["text_tokens"], max_new_tokens=2) == golden["text_f16_gen"].tolist()[:2]
    e.close()


def test_missing_tensor_is_reported(require_gpu, tensors):
    part = {k: v for k, v in tensors.items() if k != L.TID_FINAL_NORM}
    e = Engine(n_layers=2, vocab=1024, max_context=64, max_pass=16, max_steps=8)
    with pytest.raises(IcuaError) as ex:
        e.set_tensors(part)
    assert ex.value.status == L.ERR_STATE
    with pytest.raises(IcuaError):
        e.prefill([1, 2, 3])
    e.close()


def test_model_file_roundtrip(require_gpu, golden, tensors, tmp_path):
    from instantcua_b200 import model

    p = tmp_path / "tiny.icua"
    model.write_icua(str(p), tensors)
    e = Engine(str(p), n_layers=2, vocab=1024, max_context=256, max_pass=64, max_steps=32)
    e.stop_on_eos = False
    assert e.generate_vision(golden["text_tokens"], max_new_tokens=4) == golden["text_f16_gen"].tolist()[:4]
    e.close()
    bad = tmp_path / "bad.icua"
    bad.write_bytes(b"XXXX" + bytes(16384 - 4))
    with pytest.raises(IcuaError) as ex:
        Engine(str(bad), n_layers=2, vocab=1024, max_context=64, max_pass=16, max_steps=8)
    assert ex.value.status == L.ERR_FORMAT


def test_prefix_cache_reuses_system_prompt(require_gpu, golden, tensors):
    """Engine.usePrefixCache (Engine.swift:719-738): a second generate with the same tokens before
    the image prefills only from the visual block on, with the same tokens and first logits."""
    args = dict(pooler=golden["mm_pooler"], deepstack=list(golden["mm_deepstack"]),
                grid=tuple(golden["mm_grid"].tolist()), write_first_logits=True)
    toks = golden["mm_tokens"]
    n_prefix = int(np.argmax(toks == 151655))
    e = make_engine(tensors)
    a = e.generate_vision(toks, max_new_tokens=4, **args)
    la = e.logits()
    assert e.last_timing.prefill_tokens == len(toks)
    b = e.generate_vision(toks, max_new_tokens=4, **args)
    lb = e.logits()
    assert e.last_timing.prefill_tokens == len(toks) - n_prefix  # prefix rows reused
    assert a == b == golden["mm_gen"].tolist()
    assert float(np.abs(la - lb).max()) <= 1e-4
    # a different prefix misses; turning the cache off prefills everything
    other = toks.copy()
    other[0] = (int(other[0]) + 1) % 1024
    e.generate_vision(other, max_new_tokens=2, **args)
    assert e.last_timing.prefill_tokens == len(toks)
    e.use_prefix_cache = False
    e.generate_vision(other, max_new_tokens=2, **args)
    assert e.last_timing.prefill_tokens == len(toks)
    e.close()


@pytest.mark.parametrize("kv", ["f16", "bf16"])
def test_folded_oproj_matches_launch_chain(require_gpu, golden, tensors, kv, monkeypatch):
    """q4s engines fold the o-projection into the decode attention (one cluster of 8 or 16 CTAs per
    kv head, 4 launches per layer instead of 5).  On the B200 it must be active; its tokens and
    logits match the five-launch chain (ICUA_ATTN_O=0) and the oracle."""
    steps = len(golden[f"text_{kv}_gen"])
    runs = {}
    for fold in ("1", "0"):
        monkeypatch.setenv("ICUA_ATTN_O", fold)
        e = make_engine(tensors, kv=kv)
        want_k = 4 * 2 + 2 if fold == "1" else 5 * 2 + 2
        assert e.kernels_per_step == want_k, (fold, e.kernels_per_step, e.attn_o_cluster)
        assert (e.attn_o_cluster in (8, 16)) if fold == "1" else e.attn_o_cluster == 0
        print(f"{kv}: ICUA_ATTN_O={fold}, cluster {e.attn_o_cluster}")
        cap = e.capture_step_logits(steps)
        first = e.prefill(golden["text_tokens"], write_logits=True)
        first_logits = cap[0].copy()
        toks = [first] + e.decode(steps - 1)
        runs[fold] = (toks, np.concatenate([first_logits[None], cap[: steps - 1]]))
        e.close()
    assert runs["1"][0] == runs["0"][0] == golden[f"text_{kv}_gen"].tolist()
    check_logits(runs["1"][1], golden[f"text_{kv}_logits"], kv + " folded o-proj")
    err = float(np.abs(runs["1"][1] - runs["0"][1]).max())
    print(f"{kv}: folded o-proj vs launch chain max|d| {err:.2e}")
    assert err <= 1e-3
