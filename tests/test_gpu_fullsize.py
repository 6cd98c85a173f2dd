"""GPU parity at the BASELINE model size (28 layers, vocabulary 151936, seeded N(0,0.02) weights,
q4s decoder, q8 lm_head) against the numpy oracle on the same dequantized weights.

Config 0 shape (128-token prompt, greedy decode) and config 2's long-context decode (KV cache
pre-filled with N(0,1) values) at a context the CPU oracle finishes in seconds.  Bars (BASELINE):
per-step logits max-abs <= 2e-2 and cosine >= 0.999; greedy agreement >= 99%.
"""
import numpy as np
import pytest

from instantcua_b200 import Engine, model
from oracle import qwen3vl_oracle as O

pytestmark = pytest.mark.gpu

ATOL = 2e-2
COS = 0.999


@pytest.fixture(scope="module")
def full(require_gpu):
    tensors, raw = model.quantize_stream(model.synthetic_fp32(seed=0), keep_fp32=True)
    # oracle weights: the oracle's own quantizers on the same fp32 draws, then dequantized
    names = {}
    from _tiny import oracle_name_to_tid

    w = {}
    for name, arr in O.generate_fp32_weights(seed=0):
        tid = oracle_name_to_tid(name)
        key = tid[0] if isinstance(tid, tuple) else tid
        assert np.array_equal(arr, raw[key]), name  # same seeded stream in product and oracle
        if arr.ndim == 1:
            w[name] = arr
        elif name == "embed":
            w[name] = O.dequant_q8(*O.quantize_q8(arr))
        else:
            w[name] = O.dequant_q4s(*O.quantize_q4s(arr))
        names[name] = key
    del raw
    return tensors, w


def compare(got, want):
    errs = [float(np.abs(a - b).max()) for a, b in zip(got, want)]
    coss = [O.cos_sim(a, b) for a, b in zip(got, want)]
    return max(errs), min(coss)


def test_config0_prompt128_greedy(full):
    tensors, w = full
    steps = 32
    e = Engine(tensors=tensors, max_context=1024, max_pass=512, max_steps=128, kv_dtype="f16")
    e.stop_on_eos = False
    prompt = np.random.default_rng(1).integers(0, 151643, 128).astype(np.int32)
    cap = e.capture_step_logits(steps)
    first = e.prefill(prompt, write_logits=True)
    first_logits = cap[0].copy()
    rest = e.decode(steps - 1)
    toks = [first] + rest
    logits = np.concatenate([first_logits[None], cap[: steps - 1]])
    e.close()
    # teacher-forced oracle: feed the engine's tokens, compare each step's logits and argmax
    ref = O.TextModel(w, kv_dtype="f16")
    want_tok, want_logits = ref.generate(prompt, steps, teacher=toks)
    err, c = compare(logits, want_logits)
    agree = np.mean(np.array(want_tok) == np.array(toks))
    print(f"config0: max|d|={err:.3e} min cos={c:.6f} greedy agreement={agree:.4f}")
    assert err <= ATOL and c >= COS
    assert agree >= 0.99


@pytest.mark.parametrize("kv", ["bf16", "f16"])
def test_config2_long_context_decode(full, kv):
    tensors, w = full
    ctx, steps = 1536, 8
    rng = np.random.default_rng(2)
    k = rng.standard_normal((28, ctx, 8, 128), dtype=np.float32)
    v = rng.standard_normal((28, ctx, 8, 128), dtype=np.float32)
    e = Engine(tensors=tensors, max_context=ctx + 64, max_pass=16, max_steps=64, kv_dtype=kv)
    e.stop_on_eos = False
    e.inject_kv(k, v)
    cur = int(rng.integers(0, 151643))
    toks, logits = [], []
    t = cur
    for _ in range(steps):
        t = e.decode_step(t)
        toks.append(t)
        logits.append(e.logits())
    e.close()
    ref = O.TextModel(w, kv_dtype=kv)
    ref.inject_kv(list(k), list(v))
    want_tok, want_logits = [], []
    t = cur
    for i in range(steps):
        lg = ref.decode_step(t)
        want_logits.append(lg)
        want_tok.append(int(np.argmax(lg)))
        t = toks[i]  # teacher-forced
    err, c = compare(logits, want_logits)
    agree = np.mean(np.array(want_tok) == np.array(toks))
    print(f"config2 ({kv}, ctx {ctx}): max|d|={err:.3e} min cos={c:.6f} greedy agreement={agree:.3f}")
    assert err <= ATOL and c >= COS
    assert agree >= 0.99
