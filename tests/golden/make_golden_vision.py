"""Pins the vision oracle (``oracle/qwen3vl_vision.py``) against Hugging Face ``Qwen3VLVisionModel``
and writes ``tests/golden/golden_vision.npz``.

Run in a container that has ``transformers`` (``python tests/golden/make_golden_vision.py``).  On a
narrow configuration (4 blocks of width 64, 4 heads of 16, DeepStack after blocks 0, 1, 2, a 4x4
position table) both implementations take the same seeded weights and a seeded 64x96 RGB image:
the oracle with the reference's folded 768-column patch matrix (Convert.swift:99-112), Hugging
Face with its Conv3d over two identical temporal frames holding half of that matrix each.  The
script asserts that pooler and DeepStack outputs agree, then stores the image and the oracle's
outputs for the CPU test, which re-derives them without transformers.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import qwen3vl_vision as V  # noqa: E402

SMALL = V.VisionDims(layers=4, hidden=64, ff=128, heads=4, head_dim=16, pos_side=4, deepstack=(0, 1, 2),
                     out_hidden=48)
SEED = 21
IMAGE_HW = (64, 96)  # grid 4 x 6 patches, 6 merged tokens


def small_image(seed: int = SEED):
    return np.random.default_rng(seed).integers(0, 256, (*IMAGE_HW, 3), dtype=np.uint8)


def hf_outputs(w, rgb, d):
    import torch
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLVisionConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLVisionModel

    cfg = Qwen3VLVisionConfig(depth=d.layers, hidden_size=d.hidden, hidden_act="gelu_pytorch_tanh",
                              intermediate_size=d.ff, num_heads=d.heads, in_channels=3, patch_size=d.patch,
                              spatial_merge_size=d.merge, temporal_patch_size=2, out_hidden_size=d.out_hidden,
                              num_position_embeddings=d.pos_side * d.pos_side,
                              deepstack_visual_indexes=list(d.deepstack))
    cfg._attn_implementation = "eager"
    model = Qwen3VLVisionModel(cfg).eval().float()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    sd = {}
    half = w["patch_w"].reshape(d.hidden, 3, 1, d.patch, d.patch) / 2.0
    sd["patch_embed.proj.weight"] = t(np.concatenate([half, half], axis=2))
    sd["patch_embed.proj.bias"] = t(w["patch_b"])
    sd["pos_embed.weight"] = t(w["pos"])
    for l in range(d.layers):
        p, q = f"blocks.{l}.", f"v{l}."
        for a, b in (("norm1.weight", "norm1_w"), ("norm1.bias", "norm1_b"), ("attn.qkv.weight", "qkv_w"),
                     ("attn.qkv.bias", "qkv_b"), ("attn.proj.weight", "proj_w"), ("attn.proj.bias", "proj_b"),
                     ("norm2.weight", "norm2_w"), ("norm2.bias", "norm2_b"), ("mlp.linear_fc1.weight", "fc1_w"),
                     ("mlp.linear_fc1.bias", "fc1_b"), ("mlp.linear_fc2.weight", "fc2_w"),
                     ("mlp.linear_fc2.bias", "fc2_b")):
            sd[p + a] = t(w[q + b])
    mergers = [f"deepstack_merger_list.{i}." for i in range(len(d.deepstack))] + ["merger."]
    for i, p in enumerate(mergers):
        q = f"m{i}."
        for a, b in (("norm.weight", "norm_w"), ("norm.bias", "norm_b"), ("linear_fc1.weight", "fc1_w"),
                     ("linear_fc1.bias", "fc1_b"), ("linear_fc2.weight", "fc2_w"), ("linear_fc2.bias", "fc2_b")):
            sd[p + a] = t(w[q + b])
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected and all("rotary" in k or "inv_freq" in k for k in missing), (missing, unexpected)
    patches, gh, gw = V.patchify(rgb, d)
    pix = np.repeat(patches.reshape(-1, 3, 1, d.patch * d.patch), 2, axis=2).reshape(len(patches), -1)
    with torch.no_grad():
        out = model(t(pix), grid_thw=torch.tensor([[1, gh, gw]]))
    return out.pooler_output.numpy(), [a.numpy() for a in out.deepstack_features]


def main():
    d = SMALL
    w = V.generate_weights(SEED, d)
    rgb = small_image()
    patches, gh, gw = V.patchify(rgb, d)
    pooler, ds = V.encode_vision(w, patches, gh, gw, d)
    hp, hds = hf_outputs(w, rgb, d)
    err = max(float(np.abs(pooler - hp).max()), *(float(np.abs(a - b).max()) for a, b in zip(ds, hds)))
    scale = max(float(np.abs(hp).max()), *(float(np.abs(b).max()) for b in hds))
    print(f"oracle vs Hugging Face Qwen3VLVisionModel: max |d| {err:.3e} (outputs up to {scale:.2f})")
    assert err <= 1e-4 * max(scale, 1.0)
    np.savez_compressed(os.path.join(HERE, "golden_vision.npz"), rgb=rgb, pooler=pooler, deepstack=np.stack(ds),
                        hf_max_abs_diff=np.float32(err), seed=np.int32(SEED))
    print("wrote golden_vision.npz")


if __name__ == "__main__":
    main()
