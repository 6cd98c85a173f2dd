"""Runs the reference's own oracle and commits its outputs as fixtures (TEST INFRASTRUCTURE).

Usage: ``python tests/golden/make_golden_ref.py --ref-root <reference project checkout>``

1. ``mlx_numpy.install()`` registers a numpy stand-in for ``mlx.core`` (MLX is Apple-only).
2. The reference file ``tools/reference/qwen3vl_ref.py`` is imported from the checkout as it is
   (no edits, no bytecode written).  ``Qwen3VLRef`` is built with ``__new__`` and its weight dict
   is set to the pin model (``tests/_refpin.py``: 28 layers, full width and vocabulary, q4s / q8
   values dequantized) under the Hugging Face names it reads.  Its tokenizer is replaced by fixed
   id lists, ``load_image_patches`` by the grid size and ``encode_vision`` by seeded pooler and
   DeepStack rows: everything else -- embedding scatter, M-RoPE with rope_delta, the 28 layers with
   the causal mask, GQA repeat, DeepStack add, tied lm_head, greedy decode loop -- is the
   reference's code (qwen3vl_ref.py:218-336).
3. For every case of ``_refpin.CASES`` it records the reference's input ids, vis_offset,
   rope_delta, generated tokens, and for each step (first-token logits, then each decode step's
   logits as passed to ``mx.argmax``) the logits at ``_refpin.sample_ids()``, the top 32 ids and
   values, and float64 sum / sum of squares of the whole vector.
4. It runs ``oracle/qwen3vl_oracle.py`` on the same model and prompts and asserts that it
   reproduces the reference (same tokens, logits within 1e-4), then writes
   ``tests/golden/golden_ref.npz``.

``tests/test_oracle_ref.py`` repeats step 4 from the fixture (no reference needed), and
``tests/test_gpu_refpin.py`` compares the CUDA engine with the fixture.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

import _refpin as P  # noqa: E402
import mlx_numpy  # noqa: E402
from oracle import qwen3vl_oracle as O  # noqa: E402

TOPK = 32


def load_reference(ref_root: str):
    mlx_numpy.install()
    sys.dont_write_bytecode = True  # the checkout is read-only
    path = os.path.join(ref_root, "tools", "reference", "qwen3vl_ref.py")
    spec = importlib.util.spec_from_file_location("qwen3vl_ref", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class FixedTokenizer:
    """Stands in for the HF tokenizer: the prefix string (which starts with the system turn) maps
    to the prefix ids, the suffix string (which starts with <|vision_end|>) to the suffix ids."""

    class _Enc:
        def __init__(self, ids):
            self.ids = list(ids)

    def __init__(self, prefix, suffix):
        self.prefix, self.suffix = prefix, suffix

    def encode(self, s, add_special_tokens=False):
        return self._Enc(self.prefix if s.startswith("<|im_start|>system") else self.suffix)

    def decode(self, ids, skip_special_tokens=True):
        return ""


def step_record(logits: np.ndarray, ids: np.ndarray):
    lg = np.asarray(logits, np.float32)
    top = np.argsort(-lg, kind="stable")[:TOPK]
    l64 = lg.astype(np.float64)
    return lg[ids], top.astype(np.int64), lg[top], np.array([l64.sum(), (l64 * l64).sum()])


def run_reference(mod, w_hf, name):
    prefix, suffix, pooler, deepstack = P.case_inputs(name)
    c = P.CASES[name]
    gh, gw = c["grid"]
    ref = mod.Qwen3VLRef.__new__(mod.Qwen3VLRef)
    ref.w = w_hf
    ref.tok = FixedTokenizer(prefix, suffix)
    ref.encode_vision = lambda patches, grid_h, grid_w: (pooler, list(deepstack))
    mod.load_image_patches = lambda path, *a, **k: (None, 2 * gh, 2 * gw)
    mlx_numpy.ARGMAX_LOG.clear()
    out = ref.generate("system", "user", "image", max_new_tokens=c["new"])
    steps = [out["first_logits"]] + list(mlx_numpy.ARGMAX_LOG)
    return out, steps


def run_oracle(w, name):
    prefix, suffix, pooler, deepstack = P.case_inputs(name)
    c = P.CASES[name]
    gh, gw = c["grid"]
    n_vis = gh * gw
    tokens = prefix + [O.IMAGE_PAD] * n_vis + suffix
    m = O.TextModel(w)
    toks, logits = m.generate(tokens, c["new"], stop_on_eos=True, pooler=pooler if n_vis else None,
                              deepstack=deepstack if n_vis else None, llm_hw=(gh, gw))
    return tokens, toks, logits, m.rope_delta


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-root", required=True, help="checkout of the reference project")
    ap.add_argument("--out", default=os.path.join(HERE, "golden_ref.npz"))
    args = ap.parse_args()
    mod = load_reference(args.ref_root)
    t0 = time.time()
    w = P.pin_dequantized()
    w_hf = P.hf_names(w)
    print(f"pin model ready in {time.time() - t0:.1f}s")
    ids = P.sample_ids()
    fx = {"sample_ids": ids}
    for name in P.CASES:
        t0 = time.time()
        out, steps = run_reference(mod, w_hf, name)
        tokens, o_toks, o_logits, o_delta = run_oracle(w, name)
        gen = list(out["gen_tokens"])
        assert out["input_ids"] == tokens, name
        assert gen == o_toks, (name, gen, o_toks)
        assert out["rope_delta"] == o_delta, (name, out["rope_delta"], o_delta)
        assert len(steps) >= len(gen)
        worst = max(float(np.abs(np.asarray(a, np.float32) - b).max()) for a, b in zip(steps, o_logits))
        assert worst <= 1e-4, (name, worst)
        recs = [step_record(s, ids) for s in steps[: len(gen)]]
        fx[f"{name}.input_ids"] = np.asarray(out["input_ids"], np.int64)
        fx[f"{name}.vis_offset"] = np.int64(out["vis_offset"])
        fx[f"{name}.rope_delta"] = np.int64(out["rope_delta"])
        fx[f"{name}.gen_tokens"] = np.asarray(gen, np.int64)
        fx[f"{name}.sampled"] = np.stack([r[0] for r in recs])
        fx[f"{name}.top_ids"] = np.stack([r[1] for r in recs])
        fx[f"{name}.top_vals"] = np.stack([r[2] for r in recs])
        fx[f"{name}.sums"] = np.stack([r[3] for r in recs])
        margins = [float(r[2][0] - r[2][1]) for r in recs]
        print(f"{name}: {len(tokens)} prompt ids, tokens {gen}, rope_delta {out['rope_delta']}, "
              f"oracle max|d| {worst:.2e}, min top-1/top-2 margin {min(margins):.4f}, {time.time() - t0:.1f}s")
    np.savez_compressed(args.out, **fx)
    print("wrote", args.out, os.path.getsize(args.out), "bytes")


if __name__ == "__main__":
    main()
