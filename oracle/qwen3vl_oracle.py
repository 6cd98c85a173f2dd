"""CPU oracle for the Qwen3VLTextModel token loop (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py`` (its ``cpu_baseline`` leg and its ``--impl reference`` arm) may import it.
The CUDA engine in ``instantcua_b200`` never routes through it.

What it restates, in numpy fp32, from the reference project (paths inside that project):

* ``tools/reference/qwen3vl_ref.py:148-150``  ``rmsnorm``      -> :func:`rmsnorm`
* ``tools/reference/qwen3vl_ref.py:153-155``  ``rotate_half``  -> :func:`rotate_half`
* ``tools/reference/qwen3vl_ref.py:87-118``   ``compute_mrope_cos_sin`` -> :func:`mrope_cos_sin`
* ``tools/reference/qwen3vl_ref.py:121-125``  ``compute_decode_rope_cos_sin`` -> :func:`decode_rope_cos_sin`
* ``tools/reference/qwen3vl_ref.py:233-288``  LLM prefill (embed scatter, 28 layers, DeepStack add,
  final norm, tied lm_head)                    -> :meth:`TextModel.prefill`
* ``tools/reference/qwen3vl_ref.py:290-336``  greedy decode loop -> :meth:`TextModel.decode_step`
* ``Sources/Engine/Convert.swift:215-241``    ``quantizeQ8``   -> :func:`quantize_q8`
* ``Sources/Engine/Convert.swift:246-320``    ``quantizeQ4Raw``/``quantGroup`` -> :func:`quantize_q4_affine`
* ``Sources/Engine/Shaders.swift:459-477``    ``embed_at`` (dequant per format) -> :func:`dequant_q8`,
  :func:`dequant_q4_affine`
* ``Sources/Engine/Shaders.swift:1497-1571``  ``k_commit`` grammar-forced pairs and ')' stop ->
  :func:`grammar_syntax`, :meth:`TextModel.generate_grammar`
* BASELINE q4 (symmetric int4, groups of 32, fp16 scale) has no reference counterpart; it is
  defined by analogy with ``quantizeQ8`` -> :func:`quantize_q4s` / :func:`dequant_q4s`.

Changes from the reference oracle, all explicit parameters:

1. ``stop_on_eos=False`` gives fixed-length greedy decoding (parity runs).
2. ``kv_dtype`` in {None, "f16", "bf16"} rounds K (after RoPE) and V to the storage type of the
   device cache before they are used; ``None`` is the reference's fp32 semantics.
3. Visual embeddings (pooler + 3 DeepStack tensors) are inputs instead of ``encode_vision``.
4. ``kv_inject`` pre-fills the cache with given K/V instead of a prefill.

The MLX arithmetic of the reference oracle (matmul, softmax, rsqrt) is restated with numpy fp32
operations; MLX is not pinned by any reference test, so parity against MLX itself is unpinned.
The restatement is cross-checked against Hugging Face ``Qwen3VLTextModel`` by
``tests/golden/make_golden.py``.
"""
from __future__ import annotations

import numpy as np

# Model constants (reference Sources/Engine/ModelFile.swift:47-59).
HIDDEN = 2048
FF = 6144
N_HEADS = 16
N_KV = 8
HEAD_DIM = 128
QKV_ROWS = 4096
GU_ROWS = 12288
VOCAB = 151936
N_LAYERS = 28
EPS = 1e-6
ROPE_THETA = 5_000_000.0
IMAGE_PAD = 151655
IM_END = 151645
ENDOFTEXT = 151643

F16 = np.float16
F32 = np.float32


# ----------------------------------------------------------------------------------------------
# Rounding helpers

def round_half_away(x: np.ndarray) -> np.ndarray:
    """Swift ``Float.rounded()`` (to nearest, ties away from zero), exact in fp32.

    ``floor(x + 0.5)`` is wrong for x = 0.5 - 2^-25, so the fraction is tested instead.
    """
    x = np.asarray(x, dtype=F32)
    t = np.trunc(x)
    frac = np.abs(x - t)  # exact for |x| < 2^23
    return (t + np.where(frac >= F32(0.5), np.sign(x), F32(0))).astype(F32)


def to_bf16(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bfloat16 (nearest even) and return the value as fp32."""
    u = np.ascontiguousarray(x, dtype=F32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    r = ((u + rounding) & np.uint32(0xFFFF0000)).astype(np.uint32)
    return r.view(F32)


def _f16_bump(sh: np.ndarray, amax: np.ndarray, qmax: int) -> np.ndarray:
    """``if Float(sh) * qmax < amax { sh = next fp16 }`` (Convert.swift:229), vectorised."""
    need = sh.astype(F32) * F32(qmax) < amax
    bits = sh.view(np.uint16).copy()
    bits[need] += np.uint16(1)
    return bits.view(F16)


# ----------------------------------------------------------------------------------------------
# Quantizers (offline) and dequantizers (the bit-exact definitions)

def quantize_q8(w: np.ndarray):
    """Symmetric int8, groups of 32 along K, fp16 scale (Convert.swift:215-241).

    Returns ``codes`` int8 [rows, K] and ``scales`` fp16 [rows, K/32].
    """
    rows, cols = w.shape
    g = w.astype(F32).reshape(rows, cols // 32, 32)
    amax = np.abs(g).max(axis=2)
    sh = (amax / F32(127)).astype(F16)
    sh = _f16_bump(sh, amax, 127)
    s = sh.astype(F32)
    inv = np.where(s > 0, F32(1) / np.where(s > 0, s, F32(1)), F32(0)).astype(F32)
    q = np.clip(round_half_away(g * inv[:, :, None]), -127, 127).astype(np.int8)
    return q.reshape(rows, cols), sh


def dequant_q8(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """fp32 value = float(scale) * q  (Shaders.swift:467-469)."""
    rows, cols = codes.shape
    q = codes.astype(F32).reshape(rows, cols // 32, 32)
    return (scales.astype(F32)[:, :, None] * q).reshape(rows, cols)


def quantize_q4s(w: np.ndarray):
    """BASELINE q4: symmetric int4, groups of 32 along K, fp16 scale.

    Defined by analogy with ``quantizeQ8`` (Convert.swift:215-241): ``sh = f16(amax/7)``, bumped
    one fp16 ulp when ``float(sh)*7 < amax``; ``q = clamp(round_half_away(w * (1/s)), -7, 7)``.
    Stored offset-binary ``u = q + 8`` in nibbles with the reference q4 packing
    (Convert.swift:262): byte j = u[2j] | u[2j+1] << 4.
    Returns ``packed`` uint8 [rows, K/2] and ``scales`` fp16 [rows, K/32].
    """
    rows, cols = w.shape
    g = w.astype(F32).reshape(rows, cols // 32, 32)
    amax = np.abs(g).max(axis=2)
    sh = (amax / F32(7)).astype(F16)
    sh = _f16_bump(sh, amax, 7)
    s = sh.astype(F32)
    inv = np.where(s > 0, F32(1) / np.where(s > 0, s, F32(1)), F32(0)).astype(F32)
    q = np.clip(round_half_away(g * inv[:, :, None]), -7, 7).astype(np.int16)
    u = (q + 8).astype(np.uint8).reshape(rows, cols)
    packed = (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)
    return packed, sh


def unpack_q4(packed: np.ndarray) -> np.ndarray:
    """Nibbles to uint8 [rows, K]; even index in the low nibble (Shaders.swift:473)."""
    rows, half = packed.shape
    out = np.empty((rows, half * 2), dtype=np.uint8)
    out[:, 0::2] = packed & 0xF
    out[:, 1::2] = packed >> 4
    return out


def dequant_q4s(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """fp32 value = float(scale) * (u - 8); exact in fp32."""
    u = unpack_q4(packed).astype(np.int16) - 8
    rows, cols = u.shape
    q = u.astype(F32).reshape(rows, cols // 32, 32)
    return (scales.astype(F32)[:, :, None] * q).reshape(rows, cols)


_CLIPS = np.array([0, 0.03, 0.06, 0.1, 0.15], dtype=F32)


def quantize_q4_affine(w: np.ndarray):
    """Reference q4: affine int4, groups of 64, fp16 (scale, bias) (Convert.swift:246-320).

    Per group: MSE search over the 25 (low clip, high clip) pairs of ``clips``, each with one
    least-squares refinement of (scale, bias), codes in 0..15, error measured with the
    fp16-rounded (scale, bias).  Vectorised over groups; the order of the search and the strict
    ``err < bestErr`` test are kept, so ties keep the earliest candidate as the reference does.
    Returns ``packed`` uint8 [rows, K/2] and ``sb`` fp16 [rows, K/64, 2] (scale, bias).
    """
    rows, cols = w.shape
    g = w.astype(F32).reshape(-1, 64)
    n = g.shape[0]
    mn = g.min(axis=1)
    mx = g.max(axis=1)
    rng = (mx - mn).astype(F32)
    best_err = np.full(n, np.inf, dtype=F32)
    best_s = np.zeros(n, dtype=F16)
    best_b = np.zeros(n, dtype=F16)
    best_q = np.zeros((n, 64), dtype=np.uint8)
    flat = rng < F32(1e-12)
    for a in _CLIPS:
        for c in _CLIPS:
            lo = (mn + a * rng).astype(F32)
            hi = (mx - c * rng).astype(F32)
            ok = (hi > lo) & ~flat
            s = np.where(ok, (hi - lo) / F32(15), F32(1)).astype(F32)
            b = lo.copy()
            active = ok.copy()
            for it in range(2):
                inv = (F32(1) / s).astype(F32)
                v = np.clip(round_half_away((g - b[:, None]) * inv[:, None]), 0, 15).astype(F32)
                if it == 1:
                    break
                sq = v.sum(axis=1, dtype=F32)
                sw = g.sum(axis=1, dtype=F32)
                sqq = (v * v).sum(axis=1, dtype=F32)
                sqw = (v * g).sum(axis=1, dtype=F32)
                den = (F32(64) * sqq - sq * sq).astype(F32)
                upd = active & (den > 0)
                s2 = np.where(upd, (F32(64) * sqw - sq * sw) / np.where(den > 0, den, F32(1)), F32(0)).astype(F32)
                upd &= s2 > 0
                s = np.where(upd, s2, s).astype(F32)
                b = np.where(upd, (sw - s2 * sq) / F32(64), b).astype(F32)
            sh = s.astype(F16)
            bh = b.astype(F16)
            sf = sh.astype(F32)
            bf = bh.astype(F32)
            valid = ok & (sf > 0)
            inv = (F32(1) / np.where(sf > 0, sf, F32(1))).astype(F32)
            q = np.clip(round_half_away((g - bf[:, None]) * inv[:, None]), 0, 15).astype(F32)
            d = sf[:, None] * q + bf[:, None] - g
            err = (d * d).sum(axis=1, dtype=F32)
            take = valid & (err < best_err)
            best_err = np.where(take, err, best_err)
            best_s = np.where(take, sh, best_s)
            best_b = np.where(take, bh, best_b)
            best_q[take] = q[take].astype(np.uint8)
    best_s = np.where(flat, F16(0), best_s)
    best_b = np.where(flat, mn.astype(F16), best_b)
    best_q[flat] = 0
    u = best_q.reshape(rows, cols)
    packed = (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)
    sb = np.stack([best_s, best_b], axis=1).reshape(rows, cols // 64, 2)
    return packed, sb


def dequant_q4_affine(packed: np.ndarray, sb: np.ndarray) -> np.ndarray:
    """fp32 value = scale * q + bias (Shaders.swift:471-476)."""
    u = unpack_q4(packed).astype(F32)
    rows, cols = u.shape
    s = sb[..., 0].astype(F32)[:, :, None]
    b = sb[..., 1].astype(F32)[:, :, None]
    return (s * u.reshape(rows, cols // 64, 64) + b).reshape(rows, cols)


# ----------------------------------------------------------------------------------------------
# Seeded synthetic weights: matrices N(0, 0.02), norms = 1.0

def generate_fp32_weights(seed: int = 0, n_layers: int = N_LAYERS, vocab: int = VOCAB, std: float = 0.02):
    """Yields (name, array) in reference TensorID order (ModelFile.swift:90-111).

    Draws come from one ``np.random.default_rng(seed)`` stream in this order: embed [V, H],
    then per layer wqkv [4096, H] (q|k|v rows), wo [H, H], wgu [12288, H] (gate|up rows),
    wd [H, FF].  Norm weights are 1.0 and take no draws.
    """
    rng = np.random.default_rng(seed)
    sd = F32(std)

    def mat(r, c):
        return rng.standard_normal((r, c), dtype=F32) * sd

    yield "embed", mat(vocab, HIDDEN)
    yield "final_norm", np.ones(HIDDEN, dtype=F32)
    for l in range(n_layers):
        yield f"l{l}.attn_norm", np.ones(HIDDEN, dtype=F32)
        yield f"l{l}.wqkv", mat(QKV_ROWS, HIDDEN)
        yield f"l{l}.q_norm", np.ones(HEAD_DIM, dtype=F32)
        yield f"l{l}.k_norm", np.ones(HEAD_DIM, dtype=F32)
        yield f"l{l}.wo", mat(HIDDEN, HIDDEN)
        yield f"l{l}.mlp_norm", np.ones(HIDDEN, dtype=F32)
        yield f"l{l}.wgu", mat(GU_ROWS, HIDDEN)
        yield f"l{l}.wd", mat(HIDDEN, FF)


def quantize_model(fp32_weights, layer_format: str = "q4s", embed_format: str = "q8"):
    """Quantizes a weight stream; returns {name: (kind, payload...)} with raw quantized tensors."""
    out = {}
    for name, w in fp32_weights:
        if w.ndim == 1:
            out[name] = ("f32", w.astype(F32))
            continue
        fmt = embed_format if name == "embed" else layer_format
        if fmt == "q8":
            out[name] = ("q8",) + quantize_q8(w)
        elif fmt == "q4s":
            out[name] = ("q4s",) + quantize_q4s(w)
        elif fmt == "q4":
            out[name] = ("q4",) + quantize_q4_affine(w)
        elif fmt == "f16":
            out[name] = ("f16", w.astype(F16))
        else:
            raise ValueError(fmt)
    return out


def dequant_tensor(entry) -> np.ndarray:
    kind = entry[0]
    if kind == "f32":
        return entry[1]
    if kind == "q8":
        return dequant_q8(entry[1], entry[2])
    if kind == "q4s":
        return dequant_q4s(entry[1], entry[2])
    if kind == "q4":
        return dequant_q4_affine(entry[1], entry[2])
    if kind == "f16":
        return entry[1].astype(F32)
    raise ValueError(kind)


# ----------------------------------------------------------------------------------------------
# Rotary tables

def inv_freq(head_dim: int = HEAD_DIM, theta: float = ROPE_THETA) -> np.ndarray:
    """``1 / theta ** (arange(0, d, 2) / d)`` in fp32 (qwen3vl_ref.py:112)."""
    return (F32(1.0) / (theta ** (np.arange(0, head_dim, 2, dtype=F32) / head_dim))).astype(F32)


def mrope_positions(seq_len: int, vis_offset: int, llm_h: int, llm_w: int):
    """3 x seq_len (t, h, w) positions and rope_delta (qwen3vl_ref.py:89-106)."""
    n_vis = llm_h * llm_w
    pos = np.zeros((3, seq_len), dtype=F32)
    if vis_offset < 0:
        pos[:] = np.arange(seq_len, dtype=F32)[None, :]
        return pos, 0
    for i in range(min(vis_offset, seq_len)):
        pos[:, i] = float(i)
    for r in range(llm_h):
        for c in range(llm_w):
            idx = vis_offset + r * llm_w + c
            if idx < seq_len:
                pos[0, idx] = float(vis_offset)
                pos[1, idx] = float(vis_offset + r)
                pos[2, idx] = float(vis_offset + c)
    after = vis_offset + max(llm_h, llm_w)
    for i in range(vis_offset + n_vis, seq_len):
        pos[:, i] = float(after + (i - (vis_offset + n_vis)))
    return pos, int(after - (vis_offset + n_vis))


def mrope_cos_sin(pos3: np.ndarray):
    """Interleaved M-RoPE (sections [24, 20, 20]) cos/sin [seq, 128] (qwen3vl_ref.py:108-118)."""
    invf = inv_freq()
    ft = pos3[0][:, None] * invf[None, :]
    fh = pos3[1][:, None] * invf[None, :]
    fw = pos3[2][:, None] * invf[None, :]
    freqs = ft.copy()
    freqs[:, 1:60:3] = fh[:, 1:60:3]
    freqs[:, 2:60:3] = fw[:, 2:60:3]
    ang = np.concatenate([freqs, freqs], axis=-1).astype(F32)
    return np.cos(ang).astype(F32), np.sin(ang).astype(F32)


def decode_rope_cos_sin(pos: int):
    """Uniform-position RoPE for one decode token (qwen3vl_ref.py:121-125)."""
    freqs = (F32(pos) * inv_freq()).astype(F32)
    ang = np.concatenate([freqs, freqs])
    return np.cos(ang).astype(F32), np.sin(ang).astype(F32)


# ----------------------------------------------------------------------------------------------
# Model

def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float = EPS) -> np.ndarray:
    """``x * rsqrt(mean(x^2) + eps) * w`` (qwen3vl_ref.py:148-150)."""
    var = np.mean(np.square(x, dtype=F32), axis=-1, keepdims=True, dtype=F32)
    return (x * (F32(1) / np.sqrt(var + F32(eps))) * w).astype(F32)


def rotate_half(x: np.ndarray) -> np.ndarray:
    """(qwen3vl_ref.py:153-155)"""
    d = x.shape[-1] // 2
    return np.concatenate([-x[..., d:], x[..., :d]], axis=-1)


def _store_kv(v: np.ndarray, kv_dtype):
    if kv_dtype is None:
        return v.astype(F32)
    if kv_dtype == "f16":
        return v.astype(F16).astype(F32)
    if kv_dtype == "bf16":
        return to_bf16(v)
    raise ValueError(kv_dtype)


def _silu(g: np.ndarray) -> np.ndarray:
    return (g * (F32(1) / (F32(1) + np.exp(-g)))).astype(F32)


class TextModel:
    """fp32 Qwen3VLTextModel with dequantized weights (the oracle's model state)."""

    def __init__(self, weights: dict, n_layers: int | None = None, kv_dtype=None):
        """``weights``: name -> fp32 array (dequantized), names from :func:`generate_fp32_weights`."""
        self.w = weights
        self.n_layers = n_layers if n_layers is not None else sum(1 for k in weights if k.endswith(".wqkv"))
        self.kv_dtype = kv_dtype
        self.k_cache = [np.zeros((0, N_KV, HEAD_DIM), F32) for _ in range(self.n_layers)]
        self.v_cache = [np.zeros((0, N_KV, HEAD_DIM), F32) for _ in range(self.n_layers)]
        self.rope_delta = 0
        self.cur_len = 0

    @classmethod
    def from_quantized(cls, qweights: dict, **kw):
        return cls({k: dequant_tensor(v) for k, v in qweights.items()}, **kw)

    # -- building blocks --------------------------------------------------------------------
    def _layer(self, l: int, x: np.ndarray, cos: np.ndarray, sin: np.ndarray, causal: bool):
        w = self.w
        n = x.shape[0]
        h = rmsnorm(x, w[f"l{l}.attn_norm"])
        qkv = (h @ w[f"l{l}.wqkv"].T).astype(F32)
        q = qkv[:, :2048].reshape(n, N_HEADS, HEAD_DIM)
        k = qkv[:, 2048:3072].reshape(n, N_KV, HEAD_DIM)
        v = qkv[:, 3072:].reshape(n, N_KV, HEAD_DIM)
        q = rmsnorm(q, w[f"l{l}.q_norm"])
        k = rmsnorm(k, w[f"l{l}.k_norm"])
        c = cos[:, None, :]
        s = sin[:, None, :]
        q = (q * c + rotate_half(q) * s).astype(F32)
        k = (k * c + rotate_half(k) * s).astype(F32)
        k = _store_kv(k, self.kv_dtype)
        v = _store_kv(v, self.kv_dtype)
        self.k_cache[l] = np.concatenate([self.k_cache[l], k], axis=0)
        self.v_cache[l] = np.concatenate([self.v_cache[l], v], axis=0)
        kc = self.k_cache[l]
        vc = self.v_cache[l]
        L = kc.shape[0]
        kr = np.repeat(kc, 2, axis=1).transpose(1, 0, 2)  # [16, L, 128]
        vr = np.repeat(vc, 2, axis=1).transpose(1, 0, 2)
        qt = q.transpose(1, 0, 2)  # [16, n, 128]
        scores = (qt @ kr.transpose(0, 2, 1)) * F32(128.0 ** -0.5)
        if causal and n > 1:
            past = L - n
            i = np.arange(n)[:, None]
            j = np.arange(L)[None, :]
            scores = scores + np.where(j > past + i, F32(-1e9), F32(0))[None]
        scores = scores.astype(F32)
        m = scores.max(axis=-1, keepdims=True)
        e = np.exp(scores - m)
        probs = (e / e.sum(axis=-1, keepdims=True)).astype(F32)
        attn = (probs @ vr).transpose(1, 0, 2).reshape(n, HIDDEN).astype(F32)
        x = (x + attn @ w[f"l{l}.wo"].T).astype(F32)
        h2 = rmsnorm(x, w[f"l{l}.mlp_norm"])
        gu = (h2 @ w[f"l{l}.wgu"].T).astype(F32)
        act = _silu(gu[:, :FF]) * gu[:, FF:]
        x = (x + act @ w[f"l{l}.wd"].T).astype(F32)
        return x

    def logits(self, x_last: np.ndarray) -> np.ndarray:
        h = rmsnorm(x_last, self.w["final_norm"])
        return (h @ self.w["embed"].T).astype(F32)

    # -- public API ---------------------------------------------------------------------------
    def inject_kv(self, k: list, v: list):
        """Pre-fill the cache: per layer [L, 8, 128] arrays."""
        self.k_cache = [_store_kv(np.asarray(a, F32), self.kv_dtype) for a in k]
        self.v_cache = [_store_kv(np.asarray(a, F32), self.kv_dtype) for a in v]
        self.cur_len = self.k_cache[0].shape[0]

    def prefill(self, tokens, pooler=None, deepstack=None, llm_hw=(0, 0), return_hidden=False):
        """Prompt pass (qwen3vl_ref.py:233-288).  Returns first-token logits [V].

        ``tokens`` may contain IMAGE_PAD runs; their rows come from ``pooler`` [n_vis, 2048] and
        ``deepstack`` (3 x [n_vis, 2048]) is added after layers 0..2 at those rows.  The prompt is
        appended after any tokens already in the cache (positions continue from ``cur_len``).
        """
        tokens = np.asarray(tokens, dtype=np.int64)
        n = tokens.shape[0]
        x = self.w["embed"][tokens].astype(F32)
        vis = np.nonzero(tokens == IMAGE_PAD)[0]
        vis_offset = int(vis[0]) if (pooler is not None and vis.size) else -1
        n_vis = 0
        if vis_offset >= 0:
            n_vis = int(pooler.shape[0])
            x[vis_offset:vis_offset + n_vis] = pooler
        start = self.cur_len
        if vis_offset >= 0:
            pos3, self.rope_delta = mrope_positions(start + n, start + vis_offset, llm_hw[0], llm_hw[1])
            pos3 = pos3[:, start:]
        else:
            p = np.arange(start, start + n, dtype=F32) + F32(self.rope_delta)
            pos3 = np.stack([p, p, p])
        cos, sin = mrope_cos_sin(pos3)
        for l in range(self.n_layers):
            x = self._layer(l, x, cos, sin, causal=True)
            if deepstack is not None and vis_offset >= 0 and l < len(deepstack):
                x[vis_offset:vis_offset + n_vis] += deepstack[l]
        self.cur_len = start + n
        if return_hidden:
            return x
        return self.logits(x[-1:])[0]

    def decode_step(self, token: int) -> np.ndarray:
        """One greedy step for ``token`` at position cur_len (qwen3vl_ref.py:295-333)."""
        x = self.w["embed"][np.array([token])].astype(F32)
        cos, sin = decode_rope_cos_sin(self.cur_len + self.rope_delta)
        for l in range(self.n_layers):
            x = self._layer(l, x, cos[None], sin[None], causal=False)
        self.cur_len += 1
        return self.logits(x)[0]

    def generate(self, tokens, max_new_tokens: int, stop_on_eos: bool = False, pooler=None,
                 deepstack=None, llm_hw=(0, 0), teacher=None):
        """Greedy loop.  Returns (generated tokens, per-step logits list).

        With ``teacher`` (a token list) the step inputs are the teacher's tokens instead of the
        oracle's own argmax (teacher-forced comparison), while the returned tokens are still the
        oracle's argmax at each step.
        """
        lg = self.prefill(tokens, pooler=pooler, deepstack=deepstack, llm_hw=llm_hw)
        out = [int(np.argmax(lg))]
        all_logits = [lg]
        while len(out) < max_new_tokens:
            if stop_on_eos and out[-1] in (IM_END, ENDOFTEXT):
                break
            inp = out[-1] if teacher is None else int(teacher[len(out) - 1])
            lg = self.decode_step(inp)
            all_logits.append(lg)
            out.append(int(np.argmax(lg)))
        return out, all_logits


# ----------------------------------------------------------------------------------------------
# Grammar-guided 2-token commit (Sources/Engine/Shaders.swift:1497-1571)

# The reference's ids (its Qwen tokenizer): '(' 7, ')' 8, ',' 11, ' ' 220 and eight action words.
REFERENCE_GRAMMAR = {"actions": (3678, 7241, 12476, 10855, 11862, 1339, 1472, 24769), "comma": 11, "space": 220,
                     "open": 7, "close": 8}


def grammar_syntax(rule: dict, tok: int, step: int):
    """Token forced after ``tok`` committed as output number ``step`` (1-based), or None
    (Shaders.swift:1548-1549: ',' -> ' ', a first-output action word -> '(')."""
    if tok == rule["comma"]:
        return rule["space"]
    if step == 1 and tok in rule["actions"]:
        return rule["open"]
    return None


def _generate_grammar(model, tokens, max_new_tokens: int, rule=None, stop_on_eos: bool = False, pooler=None,
                      deepstack=None, llm_hw=(0, 0)):
    """Greedy loop with the grammar-forced pairs.  Returns (tokens, {output index: logits}).

    A forced token gets no logits of its own; the step after a pair feeds both tokens at
    consecutive positions (two single-token steps here, which is the same causal computation) and
    its logits predict the token after the pair.  ')' ends the output; so does max_new_tokens,
    also right after a forced token (Shaders.swift:1539-1559).
    """
    rule = REFERENCE_GRAMMAR if rule is None else rule
    lg = model.prefill(tokens, pooler=pooler, deepstack=deepstack, llm_hw=llm_hw)
    out = [int(np.argmax(lg))]
    logits = {0: lg}
    while True:
        tok = out[-1]
        if (stop_on_eos and tok in (IM_END, ENDOFTEXT)) or tok == rule["close"] or len(out) >= max_new_tokens:
            break
        syn = grammar_syntax(rule, tok, len(out))
        if syn is not None:
            out.append(syn)
            if len(out) >= max_new_tokens:
                break
            model.decode_step(tok)
            lg = model.decode_step(syn)
        else:
            lg = model.decode_step(tok)
        logits[len(out)] = lg
        out.append(int(np.argmax(lg)))
    return out, logits


TextModel.generate_grammar = _generate_grammar


def cos_sim(a: np.ndarray, b: np.ndarray) -> float:
    """Cosine similarity in float64 with a 1e-12 guard (compare.py:16-19)."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.dot(a, b) / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-12))
