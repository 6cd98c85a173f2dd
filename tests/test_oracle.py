"""CPU tests of the oracle against the committed golden fixtures (no GPU, no transformers)."""
import hashlib
import os

import numpy as np
import pytest

from oracle import qwen3vl_oracle as O


def test_round_half_away_edges():
    x = np.array([0.5, -0.5, 1.5, -1.5, 2.5, 0.49999997, -0.49999997, 126.5, -126.5, 0.0], np.float32)
    want = np.array([1, -1, 2, -2, 3, 0, 0, 127, -127, 0], np.float32)
    assert np.array_equal(O.round_half_away(x), want)


def test_bf16_rounding_matches_torch():
    torch = pytest.importorskip("torch")
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 3
    x[:4] = [1.0 + 2 ** -8, 1.0 + 3 * 2 ** -9, -1.0 - 2 ** -8, 65504.0]
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(O.to_bf16(x), ref)


def test_quantizer_known_answers(golden):
    kat = golden["kat_in"]
    c, s = O.quantize_q8(kat)
    assert np.array_equal(c, golden["kat_q8_codes"]) and np.array_equal(s.view(np.uint16), golden["kat_q8_scales"].view(np.uint16))
    p, s = O.quantize_q4s(kat)
    assert np.array_equal(p, golden["kat_q4s_packed"]) and np.array_equal(s.view(np.uint16), golden["kat_q4s_scales"].view(np.uint16))
    p, sb = O.quantize_q4_affine(kat)
    assert np.array_equal(p, golden["kat_q4_packed"]) and np.array_equal(sb.view(np.uint16), golden["kat_q4_sb"].view(np.uint16))


def test_quantizer_rules_by_hand():
    # q8: amax 1.0 -> sh = f16(1/127) is below amax/127 once rounded -> bumped one ulp
    w = np.zeros((1, 32), np.float32)
    w[0, 0] = 1.0
    c, s = O.quantize_q8(w)
    sh = np.float16(np.float32(1.0) / np.float32(127))
    if np.float32(sh) * 127 < 1.0:
        sh = np.array([sh]).view(np.uint16) + 1
        sh = sh.view(np.float16)[0]
    assert s[0, 0] == sh and c[0, 0] == 127 and np.all(c[0, 1:] == 0)
    # q4s: codes are symmetric in [-7, 7], stored as u = q + 8 (never 0)
    w = np.random.default_rng(1).standard_normal((8, 64)).astype(np.float32)
    p, s = O.quantize_q4s(w)
    u = O.unpack_q4(p)
    assert u.min() >= 1 and u.max() <= 15
    # every group reaches +-7 at its absolute maximum
    q = u.astype(np.int16) - 8
    assert np.all(np.abs(q.reshape(8, 2, 32)).max(axis=2) == 7)
    # dequant is exact: float(scale) * q has no rounding
    d = O.dequant_q4s(p, s)
    assert np.array_equal(d, (s.astype(np.float64)[:, :, None] * q.reshape(8, 2, 32)).reshape(8, 64).astype(np.float32))


def _digest(entry):
    h = hashlib.sha256()
    for a in entry[1:]:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


@pytest.fixture(scope="module")
def tiny_dequant():
    from _tiny import tiny_fp32

    qw = O.quantize_model(tiny_fp32().items(), layer_format="q4s", embed_format="q8")
    return qw, {k: O.dequant_tensor(v) for k, v in qw.items()}


def test_tiny_weights_pinned(golden, tiny_dequant):
    qw, _ = tiny_dequant
    names = [str(n) for n in golden["weight_names"]]
    assert names == sorted(qw)
    for n, h in zip(names, golden["weight_sha256"]):
        assert _digest(qw[n]) == str(h), n


@pytest.mark.parametrize("kv", [None, "f16", "bf16"])
def test_tiny_text_generation_reproduces(golden, tiny_dequant, kv):
    _, wd = tiny_dequant
    tag = "f32" if kv is None else kv
    toks, logits = O.TextModel(wd, kv_dtype=kv).generate(golden["text_tokens"], len(golden[f"text_{tag}_gen"]))
    assert toks == golden[f"text_{tag}_gen"].tolist()
    np.testing.assert_allclose(np.stack(logits), golden[f"text_{tag}_logits"], rtol=0, atol=1e-5)


def test_mrope_tables(golden):
    grid = tuple(golden["mm_grid"].tolist())
    n = len(golden["mm_tokens"])
    pos3, delta = O.mrope_positions(n, 3, *grid)
    assert np.array_equal(pos3.astype(np.int32), golden["mm_pos3"]) and delta == int(golden["mm_rope_delta"])
    cos, sin = O.mrope_cos_sin(pos3)
    np.testing.assert_array_equal(cos, golden["mm_cos"])
    np.testing.assert_array_equal(sin, golden["mm_sin"])
    # H at 1:60:3, W at 2:60:3, T elsewhere (interleaved sections [24, 20, 20])
    invf = O.inv_freq()
    v = 3 + 5  # a visual row: r = 1, c = 1 on a 3x4 grid
    assert cos[v, 1] == np.cos(np.float32(pos3[1, v]) * invf[1])
    assert cos[v, 2] == np.cos(np.float32(pos3[2, v]) * invf[2])
    assert cos[v, 60] == np.cos(np.float32(pos3[0, v]) * invf[60])


def test_multimodal_prefill_reproduces(golden, tiny_dequant):
    _, wd = tiny_dequant
    model = O.TextModel(dict(wd))
    model.w["embed"] = np.concatenate([wd["embed"], np.zeros((O.IMAGE_PAD + 1 - 1024, O.HIDDEN), np.float32)])
    lg = model.prefill(golden["mm_tokens"].astype(np.int64), pooler=golden["mm_pooler"],
                       deepstack=list(golden["mm_deepstack"]), llm_hw=tuple(golden["mm_grid"].tolist()))[:1024]
    np.testing.assert_allclose(lg, golden["mm_first_logits"], rtol=0, atol=1e-5)


def test_grammar_syntax_reference_ids():
    """k_commit's forced pairs (Shaders.swift:1548-1549): ',' -> ' ' at any step, an action word
    -> '(' only as the first output."""
    R = O.REFERENCE_GRAMMAR
    assert O.grammar_syntax(R, 11, 1) == 220 and O.grammar_syntax(R, 11, 7) == 220
    for a in R["actions"]:
        assert O.grammar_syntax(R, a, 1) == 7
        assert O.grammar_syntax(R, a, 2) is None
    assert O.grammar_syntax(R, 8, 1) is None and O.grammar_syntax(R, 100, 1) is None


def test_grammar_pair_steps_equal_a_two_row_pass(tiny_dequant):
    """The oracle feeds a forced pair as two single-token steps; that is the same causal
    computation as one two-row pass at the same positions (what the engine runs)."""
    _, wd = tiny_dequant
    prompt = np.random.default_rng(4).integers(0, 1024, 12)
    a = O.TextModel(wd, kv_dtype="f16")
    a.prefill(prompt)
    a.decode_step(17)
    la = a.decode_step(220)
    b = O.TextModel(wd, kv_dtype="f16")
    b.prefill(prompt)
    lb = b.prefill(np.array([17, 220]))
    assert a.cur_len == b.cur_len
    assert np.abs(la - lb).max() <= 1e-4 * np.abs(la).max()


def test_grammar_generation_rule(tiny_dequant):
    """Forced tokens follow their trigger, the closing token ends the output, the budget counts
    forced tokens, and a rule that never fires is plain greedy decoding."""
    _, wd = tiny_dequant
    prompt = np.random.default_rng(4).integers(0, 1024, 12)
    plain, _ = O.TextModel(wd).generate(prompt, 10)
    never = {"actions": (), "comma": -1, "space": 220, "open": 7, "close": -1}
    assert O.TextModel(wd).generate_grammar(prompt, 10, rule=never)[0] == plain
    rule = {"actions": (plain[0],), "comma": -1, "space": 220, "open": 7, "close": -1}
    out, lg = O.TextModel(wd).generate_grammar(prompt, 10, rule=rule)
    assert out[:2] == [plain[0], 7] and len(out) == 10 and 1 not in lg
    assert O.TextModel(wd).generate_grammar(prompt, 2, rule=rule)[0] == [plain[0], 7]
    rule["close"] = out[4]
    out2, _ = O.TextModel(wd).generate_grammar(prompt, 10, rule=rule)
    assert out2 == out[:out.index(out[4]) + 1]


def test_vision_oracle_reproduces_pinned_fixture():
    """The vision restatement on the narrow configuration that tests/golden/make_golden_vision.py
    pinned against Hugging Face Qwen3VLVisionModel (max |d| stored in the fixture)."""
    from golden.make_golden_vision import SEED, SMALL
    from oracle import qwen3vl_vision as V

    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_vision.npz"))
    assert float(g["hf_max_abs_diff"]) <= 1e-5
    w = V.generate_weights(int(g["seed"]), SMALL)
    patches, gh, gw = V.patchify(g["rgb"], SMALL)
    pooler, ds = V.encode_vision(w, patches, gh, gw, SMALL)
    assert np.allclose(pooler, g["pooler"], atol=1e-6, rtol=0)
    assert np.allclose(np.stack(ds), g["deepstack"], atol=1e-6, rtol=0)


def test_vision_patch_order_and_tables():
    """Merge-block patch order, the position resampling at the grid corners, and the 2-D RoPE
    angles (qwen3vl_ref.py:25-84) on hand-checkable inputs."""
    from oracle import qwen3vl_vision as V

    d = V.REFERENCE
    rgb = np.zeros((64, 64, 3), np.uint8)
    rgb[16:32, 0:16, 1] = 255  # patch (row 1, col 0), green channel
    p, gh, gw = V.patchify(rgb, d)
    assert (gh, gw) == (4, 4)
    hot = np.nonzero((p > 0).any(axis=1))[0]
    assert hot.tolist() == [2]  # block (0, 0) holds patches (0,0) (0,1) (1,0) (1,1)
    assert np.all(p[2, 256:512] == 1.0) and np.all(p[2, :256] == -1.0)
    table = np.random.default_rng(0).standard_normal((48 * 48, 8)).astype(np.float32)
    pos = V.pos_embed_interp(table, 4, 4, d)
    assert np.allclose(pos[0], table[0]) and np.allclose(pos[15], table[48 * 48 - 1])
    cos, sin = V.vision_rope(4, 4, d)
    # patch 3 of block 0 is (row 1, col 1): first-frequency angle 1 for both halves
    assert np.isclose(cos[3, 0], np.cos(1.0)) and np.isclose(cos[3, 16], np.cos(1.0)) and cos[0, 0] == 1.0
