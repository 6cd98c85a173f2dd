"""GPU parity at the BASELINE configurations (28 layers, vocabulary 151936, seeded N(0,0.02) weights,
q4s decoder, q8 lm_head) against the numpy oracle on the same dequantized weights.  The oracle is
pinned to the reference's own qwen3vl_ref.py by tests/test_oracle_ref.py.

* Config 0 shape: 128-token prompt, then a 256-step free-running greedy decode through the CUDA
  graph path (icua_prefill + icua_decode).
* Config 2: KV cache pre-filled to 4096 N(0,1) positions in bf16 (the benchmarked workload), 16
  steps: the first through icua_decode_step, the rest through the graph path (icua_decode).
* Config 3: 1000 visual rows (25 x 40 grid, DeepStack at layers 0-2, 3-D M-RoPE) + 256 text
  tokens through the tensor-core prefill, then 4 decode steps, with the reference's fp16 KV cache.
* Config 4: 64 sessions with 2048 cached positions each, decoded together (icua_decode_batch);
  four of them carry host-known KV values and are checked against the oracle's per-session decode.

Each engine run is free-running; the oracle is then run teacher-forced on the engine's tokens (one
causal pass over prompt + generated tokens, whose row i is mathematically decode step i), so every
step's logits are compared given the same history.  Bars (BASELINE): per-step logits max-abs
<= 2e-2 and cosine >= 0.999; greedy (argmax) agreement >= 99%, with the oracle's top-1/top-2
margin printed at each disagreement.
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
    del raw
    return tensors, w


def teacher_logits(model_, prompt, gen, **vis):
    """Oracle logits of every generated step, teacher-forced on ``gen``: one causal pass over the
    prompt followed by gen[:-1]; the hidden row before each generated token gives its logits."""
    rows = np.concatenate([np.asarray(prompt, np.int64), np.asarray(gen[:-1], np.int64)])
    x = model_.prefill(rows, return_hidden=True, **vis)
    n0 = len(prompt) - 1
    return model_.logits(x[n0:n0 + len(gen)])


def check(tag, got_logits, want_logits, got_tok):
    """Per-step max-abs / cosine over all logits and argmax agreement; prints the oracle's margin at
    each disagreement."""
    errs = np.abs(got_logits - want_logits).max(axis=1)
    coss = np.array([O.cos_sim(a, b) for a, b in zip(got_logits, want_logits)])
    want_tok = want_logits.argmax(axis=1)
    agree = want_tok == np.asarray(got_tok)
    for s in np.nonzero(~agree)[0]:
        srt = np.sort(want_logits[s])
        print(f"{tag}: step {s} engine {got_tok[s]} oracle {want_tok[s]}, oracle top-1/top-2 margin "
              f"{srt[-1] - srt[-2]:.5f}, engine logit gap {got_logits[s, want_tok[s]] - got_logits[s, got_tok[s]]:.5f}")
    print(f"{tag}: {len(got_tok)} steps, max|d| {errs.max():.3e}, min cos {coss.min():.6f}, "
          f"greedy agreement {agree.mean():.4f}")
    assert errs.max() <= ATOL and coss.min() >= COS
    assert agree.mean() >= 0.99


def test_config0_prompt128_free_running_256(full):
    tensors, w = full
    steps = 256
    e = Engine(tensors=tensors, max_context=1024, max_pass=512, max_steps=steps + 8, kv_dtype="f16")
    e.stop_on_eos = False
    prompt = np.random.default_rng(1).integers(0, 151643, 128).astype(np.int32)
    cap = e.capture_step_logits(steps)
    first = e.prefill(prompt, write_logits=True)
    first_logits = cap[0].copy()
    rest = e.decode(steps - 1)
    e.close()
    toks = [first] + rest
    assert len(toks) == steps
    logits = np.concatenate([first_logits[None], cap[: steps - 1]])
    want = teacher_logits(O.TextModel(w, kv_dtype="f16"), prompt, toks)
    check("config0 256 steps", logits, want, toks)


@pytest.mark.parametrize("kv,ctx", [("bf16", 4096), ("f16", 1536)])
def test_config2_long_context_decode(full, kv, ctx):
    tensors, w = full
    steps = 16
    rng = np.random.default_rng(2)
    k = rng.standard_normal((28, ctx, 8, 128), dtype=np.float32)
    v = rng.standard_normal((28, ctx, 8, 128), dtype=np.float32)
    e = Engine(tensors=tensors, max_context=ctx + 64, max_pass=16, max_steps=64, kv_dtype=kv)
    e.stop_on_eos = False
    e.inject_kv(k, v)
    cur = int(rng.integers(0, 151643))
    t1 = e.decode_step(cur)
    lg1 = e.logits()
    cap = e.capture_step_logits(steps - 1)
    rest = e.decode(steps - 1)  # the CUDA-graph path of the benchmark
    e.close()
    toks = [t1] + rest
    logits = np.concatenate([lg1[None], cap])
    ref = O.TextModel(w, kv_dtype=kv)
    ref.inject_kv(list(k), list(v))
    del k, v
    want = teacher_logits(ref, [cur], toks)
    check(f"config2 ({kv}, ctx {ctx})", logits, want, toks)


@pytest.mark.parametrize("kv", ["f16"])  # the reference's KV type (Shaders.swift:776-783)
def test_config3_multimodal_prefill_full_size(full, kv):
    tensors, w = full
    import torch

    n_vis, llm_h, llm_w, n_text, steps = 1000, 25, 40, 256, 5
    rng = np.random.default_rng(3)

    def bf16(a):
        return torch.from_numpy(a).to(torch.bfloat16).float().numpy()

    pooler = bf16(rng.standard_normal((n_vis, 2048), dtype=np.float32))
    ds = [bf16(rng.standard_normal((n_vis, 2048), dtype=np.float32)) for _ in range(3)]
    prompt = np.concatenate([np.full(n_vis, O.IMAGE_PAD, np.int32), rng.integers(0, 151643, n_text).astype(np.int32)])
    e = Engine(tensors=tensors, max_context=len(prompt) + 64, max_pass=len(prompt), max_steps=16, kv_dtype=kv)
    e.stop_on_eos = False
    cap = e.capture_step_logits(steps)
    first = e.prefill(prompt, pooler=pooler, deepstack=ds, grid=(llm_h, llm_w), write_logits=True)
    first_logits = cap[0].copy()
    rest = e.decode(steps - 1)
    e.close()
    toks = [first] + rest
    logits = np.concatenate([first_logits[None], cap[: steps - 1]])
    want = teacher_logits(O.TextModel(w, kv_dtype=kv), prompt, toks, pooler=pooler, deepstack=ds,
                          llm_hw=(llm_h, llm_w))
    check(f"config3 1000 visual + 256 text ({kv} KV)", logits, want, toks)


def test_config4_batched_sessions_vs_oracle(full):
    tensors, w = full
    n_sess, ctx, steps, checked = 64, 2048, 4, (0, 21, 42, 63)
    rng = np.random.default_rng(4)
    e = Engine(tensors=tensors, max_context=ctx + 64, max_pass=n_sess, max_steps=64, kv_dtype="bf16",
               max_sessions=n_sess)
    e.stop_on_eos = False
    kv = {}
    for s in range(n_sess):
        if s in checked:
            k = rng.standard_normal((28, ctx, 8, 128), dtype=np.float32)
            v = rng.standard_normal((28, ctx, 8, 128), dtype=np.float32)
            e.inject_kv(k, v, session=s)
            kv[s] = (k, v)
        else:
            e.inject_kv_random(ctx, seed=100 + s, session=s)
    toks_in = rng.integers(0, 151643, n_sess).astype(np.int32)
    cap = e.capture_batch_logits(n_sess)
    sess = list(range(n_sess))
    out, logs = [], []
    for i in range(steps):  # one step per call, so every step's logits are captured
        o = e.decode_batch(sess, 1, in_tokens=toks_in if i == 0 else None)
        out.append(o[:, 0].copy())
        logs.append(cap.copy())
    e.close()
    out = np.stack(out, axis=1)      # [sessions, steps]
    logs = np.stack(logs, axis=1)    # [sessions, steps, vocab]
    for s in checked:
        ref = O.TextModel(w, kv_dtype="bf16")
        ref.inject_kv(list(kv[s][0]), list(kv[s][1]))
        want = teacher_logits(ref, [int(toks_in[s])], out[s].tolist())
        check(f"config4 session {s}", logs[s], want, out[s].tolist())
