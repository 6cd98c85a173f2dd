"""GPU parity of the grammar-guided 2-token commit (reference k_commit, Shaders.swift:1497-1571).

The engine's two-token passes (both tokens through one read of the weights, the second token's
query attending the first's new K/V row) against the oracle's restatement of the same rule, which
feeds the pair as two single-token steps.  Bar (BASELINE): identical tokens, logits of every
model-predicted output within max-abs 2e-2 and cosine 0.999 of the oracle.  With the rule never
firing, the two-token kernels must reproduce the single-token kernels bit for bit.

The tiny model's vocabulary (1024) does not hold the reference's action-word ids, so the rules
here take ids that the model actually produces; the reference's own ids are checked on the host.
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
NEVER = -5  # an id no step produces (oracle-side placeholder while a rule is being chosen)


@pytest.fixture(scope="module")
def tiny(require_gpu):
    from _tiny import engine_tensors, tiny_fp32

    w32 = tiny_fp32()
    wq = {}
    for name, arr in w32.items():
        if arr.ndim == 1:
            wq[name] = arr
        elif name == "embed":
            wq[name] = O.dequant_q8(*O.quantize_q8(arr))
        else:
            wq[name] = O.dequant_q4s(*O.quantize_q4s(arr))
    return engine_tensors(w32), wq


def make(tensors, kv="f16", **kw):
    args = dict(n_layers=2, vocab=1024, max_context=512, max_pass=128, max_steps=64, kv_dtype=kv, steps_per_graph=4)
    args.update(kw)
    e = Engine(tensors=tensors, **args)
    e.stop_on_eos = False
    return e


def oracle_run(wq, kv, prompt, n, rule):
    return O.TextModel(wq, kv_dtype=kv).generate_grammar(prompt, n, rule=rule)


def engine_run(tensors, kv, prompt, n, rule, gemm_min=None):
    """(tokens, {output index: logits}) of prefill + decode with the rule (None: grammar off)."""
    e = make(tensors, kv=kv, prefill_gemm_min=gemm_min)
    if rule is not None:
        e.set_grammar_commit(True, actions=rule["actions"], comma=rule["comma"], space=rule["space"],
                             open_=rule["open"], close=rule["close"])
    cap = e.capture_step_logits(n)
    first = e.prefill(prompt, write_logits=True)
    logits = {0: cap[0].copy()}
    rest = e.decode(n - 1)
    for i in range(len(rest)):
        logits[1 + i] = cap[i].copy()
    e.close()
    return [first] + rest, logits


def choose_rule(wq, kv, prompt, n):
    """A rule that fires on this prompt: the first output is an action word, a later output is
    the comma, and a model-predicted token after the first comma pair is the closing token."""
    plain, _ = O.TextModel(wq, kv_dtype=kv).generate(prompt, n)
    act = plain[0]
    rule = {"actions": (act,), "comma": NEVER, "space": 220, "open": 7, "close": NEVER}
    out1, _ = oracle_run(wq, kv, prompt, n, rule)
    assert out1[1] == 7
    rule["comma"] = next(t for i, t in enumerate(out1) if i >= 3 and t not in (act, 7, 220))
    out2, _ = oracle_run(wq, kv, prompt, n, rule)
    c = out2.index(rule["comma"])
    later = [i for i in range(c + 3, len(out2))
             if i not in forced_indices(rule, out2) and out2[i] not in (act, rule["comma"], 7, 220)]
    if later:
        rule["close"] = out2[later[len(later) // 2]]
    else:
        rule["close"] = next(t for t in range(1023, 0, -1) if t not in out2)
    return rule


def forced_indices(rule, toks):
    """Outputs the rule appended (the token before them had a syntax token)."""
    return {i for i in range(1, len(toks)) if O.grammar_syntax(rule, toks[i - 1], i) is not None}


@pytest.mark.parametrize("kv", ["f16", "bf16"])
def test_grammar_rule_never_firing_is_bit_identical(tiny, kv, monkeypatch):
    """Two-token kernels with one-token passes == the single-token launch-chain kernels they are
    built from, bit for bit (grammar engines always decode by the five-launch chain, so the
    single-token engine runs it too: no persistent kernel, no o-projection folded into the
    attention)."""
    tensors, _ = tiny
    prompt = np.random.default_rng(11).integers(0, 1024, 40).astype(np.int32)
    n = 16
    monkeypatch.delenv("ICUA_DECODE", raising=False)
    monkeypatch.setenv("ICUA_ATTN_O", "0")
    base, lb = engine_run(tensors, kv, prompt, n, None)
    unused = [t for t in range(1024) if t not in base][:4]
    rule = {"actions": (unused[0],), "comma": unused[1], "space": 220, "open": 7, "close": unused[2]}
    got, lg = engine_run(tensors, kv, prompt, n, rule)
    assert got == base
    for i in lb:
        assert np.array_equal(lg[i], lb[i]), i


@pytest.mark.parametrize("kv,gemm_min", [("f16", None), ("bf16", None), ("f16", 0)])
def test_grammar_pairs_match_oracle(tiny, kv, gemm_min):
    tensors, wq = tiny
    prompt = np.random.default_rng(5).integers(0, 1024, 40).astype(np.int32)
    n = 24
    rule = choose_rule(wq, kv, prompt, n)
    want, want_lg = oracle_run(wq, kv, prompt, n, rule)
    got, got_lg = engine_run(tensors, kv, prompt, n, rule, gemm_min=gemm_min)
    forced = forced_indices(rule, want)
    print(f"grammar ({kv}): rule {rule}, {len(want)} outputs, forced at {sorted(forced)}")
    assert len(forced) >= 2  # the action pair and at least one comma pair ran as two-token passes
    assert got == want
    worst = 0.0
    for i, w in want_lg.items():
        a = got_lg[i]
        err = float(np.abs(a - w).max())
        assert err <= ATOL and cos_sim(a, w) >= COS, f"output {i}: max|d|={err}"
        worst = max(worst, err)
    print(f"grammar ({kv}): max|d| vs oracle {worst:.3e}")


def test_grammar_generate_vision_and_step_budget(tiny):
    """icua_generate applies the rule to the prefill's first token; a forced token can be the
    last output; ')' ends the output."""
    tensors, wq = tiny
    prompt = np.random.default_rng(5).integers(0, 1024, 40).astype(np.int32)
    rule = choose_rule(wq, "f16", prompt, 24)
    e = make(tensors)
    e.set_grammar_commit(True, actions=rule["actions"], comma=rule["comma"], space=rule["space"],
                         open_=rule["open"], close=rule["close"])
    for n in (1, 2, 3, 24):
        want, _ = oracle_run(wq, "f16", prompt, n, rule)
        got = e.generate_vision(prompt, max_new_tokens=n)
        assert got == want, n
    want, _ = oracle_run(wq, "f16", prompt, 24, rule)
    assert want[-1] == rule["close"] or len(want) == 24
    e.close()


def test_grammar_rejects_bad_rules(tiny):
    tensors, _ = tiny
    e = make(tensors)
    e.set_grammar_commit(True)  # the reference's ids ('(' and ' ' are inside the tiny vocabulary)
    with pytest.raises(L.IcuaError):
        e.set_grammar_commit(True, actions=[5000], comma=1, space=2, open_=3, close=4)
    with pytest.raises(ValueError):
        e.set_grammar_commit(True, actions=list(range(9)), comma=1, space=2, open_=3, close=4)
    e.set_grammar_commit(False)
    e.close()


def test_decode_step_ignores_the_rule(tiny):
    """Caller-driven steps carry one token and force none."""
    tensors, _ = tiny
    prompt = np.random.default_rng(2).integers(0, 1024, 20).astype(np.int32)
    e0 = make(tensors)
    first = e0.prefill(prompt)
    base = [e0.decode_step(first)]
    for _ in range(4):
        base.append(e0.decode_step(base[-1]))
    e0.close()
    e = make(tensors)
    e.set_grammar_commit(True, actions=[first], comma=base[0], space=220, open_=7, close=base[1])
    assert e.prefill(prompt) == first
    got = [e.decode_step(first)]
    for _ in range(4):
        got.append(e.decode_step(got[-1]))
    assert got == base
    e.close()
