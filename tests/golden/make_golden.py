"""Generates the committed golden fixtures under ``tests/golden/`` and pins the oracle.

Run in a container that has ``transformers`` (``python tests/golden/make_golden.py``).  It

1. builds a tiny Qwen3-VL text model (2 decoder layers, vocab 1024, every other dimension at
   full size) from seeded N(0, 0.02) weights, quantized with the oracle's quantizers;
2. runs the numpy oracle (``oracle/qwen3vl_oracle.py``) and, independently, Hugging Face
   ``Qwen3VLTextModel`` (transformers' own restatement of the same architecture: per-head QK
   RMSNorm, interleaved M-RoPE, GQA, SwiGLU, DeepStack) on the same dequantized weights, for a
   text prompt and for a multimodal prompt with DeepStack, and asserts that they agree;
3. writes the oracle's outputs as fixtures: quantizer known answers, first-token logits,
   greedy tokens and per-step logits, M-RoPE tables.

The fixtures let the CPU tests re-check the oracle and the GPU tests check the CUDA engine
without transformers, MLX or the reference sources on the GPU box.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import qwen3vl_oracle as O  # noqa: E402

sys.path.insert(0, os.path.dirname(HERE))
from _tiny import N_LAYERS, SEED, VOCAB, tiny_fp32  # noqa: E402
TEXT_PROMPT_LEN = 16
GEN_STEPS = 8
MM_PREFIX = 3
MM_GRID = (3, 4)  # llm_h, llm_w
MM_SUFFIX = 5
MM_STEPS = 4


def weight_digest(entry) -> str:
    import hashlib
    h = hashlib.sha256()
    for a in entry[1:]:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def quant_kat():
    """Known-answer inputs for the quantizers, including edge cases."""
    rng = np.random.default_rng(123)
    m = (rng.standard_normal((48, 256)) * 0.02).astype(np.float32)
    m[0, :64] = 0.0                                   # all-zero groups
    m[1, :32] = np.linspace(-1, 1, 32, dtype=np.float32)
    m[2, :32] = 0.5                                   # flat group
    m[3, 0] = 3.0                                     # single large outlier
    m[4, :32] = np.float32(0.07) * (np.arange(32) % 5 - 2)  # values on rounding ties
    m[5, :32] = -1e-8                                 # tiny negatives
    return m


def hf_logits(w, tokens, pos3, pooler=None, deepstack=None, vis_offset=-1):
    import torch
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextModel

    cfg = Qwen3VLTextConfig(
        vocab_size=VOCAB, hidden_size=O.HIDDEN, intermediate_size=O.FF, num_hidden_layers=N_LAYERS,
        num_attention_heads=O.N_HEADS, num_key_value_heads=O.N_KV, head_dim=O.HEAD_DIM,
        rms_norm_eps=O.EPS, attention_bias=False, hidden_act="silu", max_position_embeddings=4096,
        rope_parameters={"rope_type": "default", "rope_theta": O.ROPE_THETA,
                         "mrope_section": [24, 20, 20], "mrope_interleaved": True},
    )
    cfg._attn_implementation = "eager"
    m = Qwen3VLTextModel(cfg).eval()
    sd = {"embed_tokens.weight": w["embed"], "norm.weight": w["final_norm"]}
    for l in range(N_LAYERS):
        p = f"layers.{l}."
        qkv = w[f"l{l}.wqkv"]
        sd[p + "self_attn.q_proj.weight"] = qkv[:2048]
        sd[p + "self_attn.k_proj.weight"] = qkv[2048:3072]
        sd[p + "self_attn.v_proj.weight"] = qkv[3072:]
        sd[p + "self_attn.o_proj.weight"] = w[f"l{l}.wo"]
        sd[p + "self_attn.q_norm.weight"] = w[f"l{l}.q_norm"]
        sd[p + "self_attn.k_norm.weight"] = w[f"l{l}.k_norm"]
        sd[p + "input_layernorm.weight"] = w[f"l{l}.attn_norm"]
        sd[p + "post_attention_layernorm.weight"] = w[f"l{l}.mlp_norm"]
        sd[p + "mlp.gate_proj.weight"] = w[f"l{l}.wgu"][:O.FF]
        sd[p + "mlp.up_proj.weight"] = w[f"l{l}.wgu"][O.FF:]
        sd[p + "mlp.down_proj.weight"] = w[f"l{l}.wd"]
    m.load_state_dict({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in sd.items()}, strict=True)
    ids = torch.tensor([tokens], dtype=torch.long)
    emb = m.embed_tokens(ids)
    kw = {}
    if pooler is not None:
        emb[0, vis_offset:vis_offset + pooler.shape[0]] = torch.from_numpy(pooler)
        mask = torch.zeros((1, len(tokens)), dtype=torch.bool)
        mask[0, vis_offset:vis_offset + pooler.shape[0]] = True
        kw = {"visual_pos_masks": mask, "deepstack_visual_embeds": [torch.from_numpy(d) for d in deepstack]}
    pid = torch.from_numpy(pos3.astype(np.int64))[:, None, :]
    with torch.no_grad():
        h = m(inputs_embeds=emb, position_ids=pid, use_cache=False, **kw).last_hidden_state[0, -1]
        return (h @ m.embed_tokens.weight.T).numpy()


def main():
    out = {}
    # -- quantizer known answers ---------------------------------------------------------------
    kat = quant_kat()
    out["kat_in"] = kat
    out["kat_q8_codes"], out["kat_q8_scales"] = O.quantize_q8(kat)
    out["kat_q4s_packed"], out["kat_q4s_scales"] = O.quantize_q4s(kat)
    out["kat_q4_packed"], out["kat_q4_sb"] = O.quantize_q4_affine(kat)
    # hand-derived answers for rows 1..3 (see the docstrings of the quantizers)
    assert out["kat_q8_codes"][1, 31] == 127 and out["kat_q8_codes"][1, 0] == -127
    assert out["kat_q4s_packed"][2, 0] == (15 | (15 << 4))  # flat 0.5 -> q=7 -> u=15
    assert int(out["kat_q8_codes"][3, 0]) == 127

    # -- tiny model ----------------------------------------------------------------------------
    w32 = tiny_fp32()
    qw = O.quantize_model(w32.items(), layer_format="q4s", embed_format="q8")
    wd = {k: O.dequant_tensor(v) for k, v in qw.items()}
    # the weights are regenerated from the seed by the tests; their quantized bytes are pinned
    out["weight_names"] = np.array(sorted(qw))
    out["weight_sha256"] = np.array([weight_digest(qw[k]) for k in sorted(qw)])

    rng = np.random.default_rng(SEED + 2)
    text = rng.integers(0, VOCAB, TEXT_PROMPT_LEN).astype(np.int32)
    out["text_tokens"] = text

    for kv in (None, "f16", "bf16"):
        tag = "f32" if kv is None else kv
        model = O.TextModel(wd, kv_dtype=kv)
        toks, logits = model.generate(text, GEN_STEPS)
        out[f"text_{tag}_gen"] = np.array(toks, np.int32)
        out[f"text_{tag}_logits"] = np.stack(logits).astype(np.float32)

    # HF cross-check on the text prompt (fp32 KV semantics) and on the first decode step
    p = np.arange(TEXT_PROMPT_LEN)
    hf_first = hf_logits(wd, text.tolist(), np.stack([p, p, p]))
    ora_first = out["text_f32_logits"][0]
    err = float(np.abs(hf_first - ora_first).max())
    print(f"text prefill: oracle vs HF max|d|={err:.3e} cos={O.cos_sim(hf_first, ora_first):.8f}")
    assert err < 2e-4, err
    seq = list(text) + [int(out["text_f32_gen"][0])]
    p = np.arange(len(seq))
    hf_step = hf_logits(wd, seq, np.stack([p, p, p]))
    err = float(np.abs(hf_step - out["text_f32_logits"][1]).max())
    print(f"decode step 1: oracle vs HF max|d|={err:.3e}")
    assert err < 2e-4, err

    # -- multimodal prompt with DeepStack --------------------------------------------------------
    llm_h, llm_w = MM_GRID
    n_vis = llm_h * llm_w
    mm = np.concatenate([rng.integers(0, VOCAB, MM_PREFIX), np.full(n_vis, O.IMAGE_PAD),
                         rng.integers(0, VOCAB, MM_SUFFIX)]).astype(np.int64)
    pooler = rng.standard_normal((n_vis, O.HIDDEN)).astype(np.float32)
    deep = [rng.standard_normal((n_vis, O.HIDDEN)).astype(np.float32) for _ in range(3)]
    out["mm_tokens"], out["mm_pooler"] = mm.astype(np.int32), pooler
    out["mm_deepstack"] = np.stack(deep)
    out["mm_grid"] = np.array(MM_GRID, np.int32)
    # embed table only has VOCAB rows: IMAGE_PAD rows are replaced by the pooler, clamp the id
    mm_ids = np.where(mm == O.IMAGE_PAD, 0, mm)
    # the oracle gathers embed rows for every id before scattering the pooler over the pad rows,
    # so the 1024-row tiny table is padded up to the pad id for this prompt
    model = O.TextModel(dict(wd))
    model.w["embed"] = np.concatenate([wd["embed"], np.zeros((O.IMAGE_PAD + 1 - VOCAB, O.HIDDEN), np.float32)])
    lg = model.prefill(mm, pooler=pooler, deepstack=deep, llm_hw=MM_GRID)[:VOCAB]
    pos3, delta = O.mrope_positions(len(mm), MM_PREFIX, llm_h, llm_w)
    out["mm_pos3"], out["mm_rope_delta"] = pos3.astype(np.int32), np.array(delta, np.int32)
    cos, sin = O.mrope_cos_sin(pos3)
    out["mm_cos"], out["mm_sin"] = cos, sin
    out["mm_first_logits"] = lg
    hf = hf_logits(wd, mm_ids.tolist(), pos3, pooler=pooler, deepstack=deep, vis_offset=MM_PREFIX)
    err = float(np.abs(hf - lg).max())
    print(f"multimodal prefill: oracle vs HF max|d|={err:.3e} cos={O.cos_sim(hf, lg):.8f}")
    assert err < 2e-4, err
    # greedy continuation after the visual prompt (decode positions carry rope_delta)
    gen, logs = [int(np.argmax(lg))], [lg]
    for _ in range(MM_STEPS - 1):
        lgs = model.decode_step(gen[-1])[:VOCAB]
        logs.append(lgs)
        gen.append(int(np.argmax(lgs)))
    out["mm_gen"], out["mm_logits"] = np.array(gen, np.int32), np.stack(logs).astype(np.float32)
    seq_ids = mm_ids.tolist() + [gen[0]]
    nxt = pos3[:, -1].max() + 1
    pos_step = np.concatenate([pos3, np.full((3, 1), nxt)], axis=1)
    hf2 = hf_logits(wd, seq_ids, pos_step, pooler=pooler, deepstack=deep, vis_offset=MM_PREFIX)
    err = float(np.abs(hf2 - out["mm_logits"][1]).max())
    print(f"multimodal decode step 1: oracle vs HF max|d|={err:.3e}")
    assert err < 2e-4, err

    path = os.path.join(HERE, "golden_tiny.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
