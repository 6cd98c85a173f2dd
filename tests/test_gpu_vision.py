"""GPU parity of the vision encoder + mergers (reference encodeVision, Engine.swift:317-473)
against the numpy oracle (oracle/qwen3vl_vision.py, pinned against Hugging Face
Qwen3VLVisionModel), at the reference's dimensions (24 blocks of 1024, 16 heads of 64, DeepStack
after blocks 5, 11, 17) with seeded synthetic weights.

The oracle takes the fp16-rounded patches the device computes from the image (the reference
rounds them too, Shaders.swift:82-110).  The device runs its GEMMs on fp16 operands with fp32
accumulation and keeps q / k / v, the attention probabilities, the LayerNorm outputs and the GELU
outputs in fp16, as the reference's Metal kernels do; the oracle is fp32 throughout.  Bar:
cosine >= 0.999 per output row and max |d| <= 2e-2 x max |oracle| for pooler and each DeepStack
output (the BASELINE logits bar, applied to the visual rows the language model consumes).
"""
import numpy as np
import pytest

from instantcua_b200 import Engine, model
from instantcua_b200 import _lib as L
from oracle import qwen3vl_vision as V
from oracle.qwen3vl_oracle import IMAGE_PAD, cos_sim

pytestmark = pytest.mark.gpu

COS = 0.999
REL = 2e-2


@pytest.fixture(scope="module")
def vision(require_gpu):
    from _tiny import engine_tensors

    w = V.generate_weights(31)
    tensors = dict(engine_tensors())
    tensors.update(model.vision_tensors(w))
    return w, tensors


def make(tensors, **kw):
    args = dict(n_layers=2, vocab=1024, max_context=512, max_pass=128, max_steps=16, kv_dtype="f16",
                steps_per_graph=4)
    args.update(kw)
    e = Engine(tensors=tensors, **args)
    e.stop_on_eos = False
    return e


def image(h, w, seed):
    return np.random.default_rng(seed).integers(0, 256, (h, w, 3), dtype=np.uint8)


def check(got, want, tag):
    scale = float(np.abs(want).max())
    err = float(np.abs(got - want).max())
    worst = min(cos_sim(a, b) for a, b in zip(got, want))
    print(f"{tag}: max|d| {err:.3e} of max {scale:.3f}, min row cosine {worst:.6f}")
    assert err <= REL * max(scale, 1.0) and worst >= COS, tag


@pytest.mark.parametrize("hw", [(64, 96), (224, 320)])
def test_encoder_matches_oracle(vision, hw):
    w, tensors = vision
    rgb = image(*hw, seed=hw[0])
    e = make(tensors)
    pooler, ds = e.encode_vision(rgb)
    e.close()
    patches, gh, gw = V.patchify(rgb)
    patches = patches.astype(np.float16).astype(np.float32)
    want_p, want_ds = V.encode_vision(w, patches, gh, gw)
    assert pooler.shape == want_p.shape == (gh * gw // 4, 2048)
    check(pooler, want_p, f"pooler {hw}")
    for d in range(3):
        check(ds[d], want_ds[d], f"deepstack {d} {hw}")


def test_generate_rgb_uses_the_encoder_rows(vision):
    """generateVision on an image == the token loop fed the encoder's rows from the host."""
    _, tensors = vision
    rgb = image(96, 128, seed=4)
    nv = (96 // 32) * (128 // 32)
    rng = np.random.default_rng(8)
    tokens = np.concatenate([rng.integers(0, 1024, 5), np.full(nv, IMAGE_PAD), rng.integers(0, 1024, 7)]).astype(np.int32)
    e = make(tensors)
    got = e.generate_rgb(rgb, tokens, max_new_tokens=6)
    t = e.last_timing
    assert t.vision_ms > 0
    pooler, ds = e.encode_vision(rgb)
    want = e.generate_vision(tokens, 6, pooler=pooler, deepstack=list(ds), grid=(3, 4))
    assert got == want
    e.close()


def test_vision_rejects_bad_inputs(vision):
    _, tensors = vision
    e = make(tensors, max_pass=16)
    with pytest.raises(L.IcuaError):
        e.encode_vision(image(48, 64, 0))    # height not a multiple of 32
    with pytest.raises(L.IcuaError):
        e.encode_vision(image(160, 160, 0))  # 25 visual tokens > max_pass 16
    e.close()
    from _tiny import engine_tensors

    e = make(engine_tensors())  # no vision tensors
    with pytest.raises(L.IcuaError, match="vision encoder tensors missing"):
        e.encode_vision(image(64, 64, 0))
    e.close()
