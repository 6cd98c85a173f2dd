"""The model on which the reference's own oracle was run (``tests/golden/make_golden_ref.py``).

The reference oracle (``tools/reference/qwen3vl_ref.py:218-336``) has the decoder depth (28),
the head layout (16 x 128 query, 8 x 128 key/value) and the hidden size (2048) written into its
code, and it embeds every prompt id, IMAGE_PAD (151655) included, before the visual rows replace
them (qwen3vl_ref.py:242-245), so the vocabulary must be the full 151936 rows.  The pin model
keeps all of that and saves memory elsewhere: its 28 decoder layers cycle through ``DISTINCT``
seeded matrix sets (layer l uses set l % DISTINCT) while every layer has its own RMSNorm weights
(1 + 0.1 N(0, 1)), so a layer-indexing mistake still shows.  Matrices are N(0, 0.02) draws
quantized as the BASELINE configuration (decoder q4s, tied embedding q8) and dequantized, so the
CUDA engine can load the same model and be compared with the reference's outputs directly.
"""
from __future__ import annotations

import numpy as np

SEED = 11
N_LAYERS = 28
DISTINCT = 2
VOCAB = 151936


def pin_fp32_sets():
    """(embed fp32, [DISTINCT sets of {wqkv, wo, wgu, wd}], {norm name: fp32}) before quantization."""
    from oracle import qwen3vl_oracle as O

    rng = np.random.default_rng(SEED)
    sd = np.float32(0.02)

    def mat(r, c):
        return rng.standard_normal((r, c), dtype=np.float32) * sd

    embed = mat(VOCAB, O.HIDDEN)
    sets = [{"wqkv": mat(O.QKV_ROWS, O.HIDDEN), "wo": mat(O.HIDDEN, O.HIDDEN), "wgu": mat(O.GU_ROWS, O.HIDDEN),
             "wd": mat(O.HIDDEN, O.FF)} for _ in range(DISTINCT)]
    norms = {"final_norm": (1.0 + 0.1 * rng.standard_normal(O.HIDDEN)).astype(np.float32)}
    for l in range(N_LAYERS):
        for nm, n in (("attn_norm", O.HIDDEN), ("q_norm", O.HEAD_DIM), ("k_norm", O.HEAD_DIM), ("mlp_norm", O.HIDDEN)):
            norms[f"l{l}.{nm}"] = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    return embed, sets, norms


def pin_quantized():
    """Oracle-quantized tensors: ("q8", codes, scales) embed, ("q4s", packed, scales) per set."""
    from oracle import qwen3vl_oracle as O

    embed, sets, norms = pin_fp32_sets()
    qe = O.quantize_q8(embed)
    del embed
    qs = [{k: O.quantize_q4s(v) for k, v in s.items()} for s in sets]
    return qe, qs, norms


def pin_dequantized(q=None):
    """{oracle name: fp32} of the 28-layer model (matrices shared between layers l and l + DISTINCT)."""
    from oracle import qwen3vl_oracle as O

    qe, qs, norms = q if q is not None else pin_quantized()
    w = {"embed": O.dequant_q8(*qe)}
    deq = [{k: O.dequant_q4s(*v) for k, v in s.items()} for s in qs]
    w.update(norms)
    for l in range(N_LAYERS):
        for k, v in deq[l % DISTINCT].items():
            w[f"l{l}.{k}"] = v
    return w


def hf_names(w: dict) -> dict:
    """The same weights under the Hugging Face checkpoint names the reference oracle reads
    (qwen3vl_ref.py:241, 260-286, 308-330); q/k/v and gate/up are row slices (views)."""
    out = {"model.language_model.embed_tokens.weight": w["embed"],
           "model.language_model.norm.weight": w["final_norm"]}
    for l in range(N_LAYERS):
        p = f"model.language_model.layers.{l}."
        qkv, gu = w[f"l{l}.wqkv"], w[f"l{l}.wgu"]
        out[p + "input_layernorm.weight"] = w[f"l{l}.attn_norm"]
        out[p + "self_attn.q_proj.weight"] = qkv[:2048]
        out[p + "self_attn.k_proj.weight"] = qkv[2048:3072]
        out[p + "self_attn.v_proj.weight"] = qkv[3072:]
        out[p + "self_attn.q_norm.weight"] = w[f"l{l}.q_norm"]
        out[p + "self_attn.k_norm.weight"] = w[f"l{l}.k_norm"]
        out[p + "self_attn.o_proj.weight"] = w[f"l{l}.wo"]
        out[p + "post_attention_layernorm.weight"] = w[f"l{l}.mlp_norm"]
        out[p + "mlp.gate_proj.weight"] = gu[:6144]
        out[p + "mlp.up_proj.weight"] = gu[6144:]
        out[p + "mlp.down_proj.weight"] = w[f"l{l}.wd"]
    return out


# Prompt cases run through the reference's generate() (qwen3vl_ref.py:218-348).  The tokenizer is
# replaced by fixed id lists (prefix = the tokens before the visual block, suffix = after it);
# grid = (llm_h, llm_w) of the merged visual grid, (0, 0) for a prompt without visual rows.
CASES = {
    "text": {"prefix": 9, "suffix": 7, "grid": (0, 0), "new": 8, "seed": 101},
    "mm_wide": {"prefix": 6, "suffix": 5, "grid": (3, 4), "new": 8, "seed": 102},
    "mm_tall": {"prefix": 4, "suffix": 6, "grid": (5, 2), "new": 6, "seed": 103},
}
SAMPLE_IDS = 4096  # logits compared at this many fixed vocabulary ids (plus each step's top 32)


def case_inputs(name: str):
    """(prefix ids, suffix ids, pooler [n_vis, 2048], deepstack list of 3 [n_vis, 2048])."""
    c = CASES[name]
    rng = np.random.default_rng(c["seed"])
    prefix = rng.integers(0, 151643, c["prefix"]).astype(np.int64).tolist()
    suffix = rng.integers(0, 151643, c["suffix"]).astype(np.int64).tolist()
    n_vis = c["grid"][0] * c["grid"][1]
    pooler = rng.standard_normal((n_vis, 2048), dtype=np.float32)
    deepstack = [rng.standard_normal((n_vis, 2048), dtype=np.float32) for _ in range(3)] if n_vis else []
    return prefix, suffix, pooler, deepstack


def sample_ids() -> np.ndarray:
    return np.sort(np.random.default_rng(SEED + 1).choice(VOCAB, SAMPLE_IDS, replace=False)).astype(np.int64)


def engine_tensors(q=None) -> dict:
    """{tensor id: bytes} of the pin model in the .icua layout (q4s decoder, q8 embedding), from
    the oracle's quantizers, whose codes and scales are bit-exact with the product's."""
    from instantcua_b200 import _lib as L

    qe, qs, norms = q if q is not None else pin_quantized()
    out = {L.TID_EMBED: qe[0].tobytes(), L.TID_EMBED_SB: qe[1].view(np.uint16).tobytes(),
           L.TID_FINAL_NORM: norms["final_norm"].tobytes()}
    for l in range(N_LAYERS):
        base = L.TID_LAYER_BASE + l * L.TID_PER_LAYER
        for nm in ("attn_norm", "q_norm", "k_norm", "mlp_norm"):
            out[base + L.SLOT[nm]] = norms[f"l{l}.{nm}"].tobytes()
        for nm, (packed, scales) in qs[l % DISTINCT].items():
            out[base + L.SLOT[nm]] = packed.tobytes()
            out[base + L.SLOT[nm + "_sb"]] = scales.view(np.uint16).tobytes()
    return out
