"""Python mirror of the reference ``Engine`` (Sources/Engine/Engine.swift) over the C ABI.

Same names and meaning as the Swift class where the path overlaps:
``Engine(model_path, max_context, max_pass, max_steps)``, ``generate_rgb`` (generateVision: vision
encoder on an RGB image, then the token loop), ``generate_vision`` (the same with the visual rows as
inputs), ``encode_vision`` (encodeVision), ``last_timing`` (Engine.Timing), ``eos``.  Errors
raise :class:`IcuaError` carrying the engine's message (the reference throws EngineError).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib as L
from ._lib import IcuaError  # noqa: F401  (re-export)

IMAGE_PAD = 151655

# The reference's grammar-commit token ids (its Qwen tokenizer, Shaders.swift:1541-1548).
REFERENCE_GRAMMAR = {"actions": (3678, 7241, 12476, 10855, 11862, 1339, 1472, 24769), "comma": 11, "space": 220,
                     "open": 7, "close": 8}


@dataclass
class Timing:
    vision_ms: float = 0.0
    prefill_ms: float = 0.0
    decode_ms: float = 0.0
    total_ms: float = 0.0
    prefill_tokens: int = 0
    generated_tokens: int = 0


class Engine:
    """One engine per CUDA device (replicas for multi-GPU)."""

    def __init__(self, model_path: str | None = None, tensors: dict | None = None, *, max_context: int = 2048,
                 max_pass: int = 512, max_steps: int = 256, n_layers: int = 28, vocab: int = 151936,
                 max_sessions: int = 1, kv_dtype: str = "f16", steps_per_graph: int = 8, device: int = 0,
                 prefill_gemm_min: int | None = None, weight_format: str = "q4s"):
        self._lib = L.lib()
        cfg = L.IcuaConfig()
        self._lib.icua_default_config(C.byref(cfg))
        cfg.device = device
        cfg.n_layers = n_layers
        cfg.vocab = vocab
        cfg.max_context = max_context
        cfg.max_pass = max_pass
        cfg.max_steps = max_steps
        cfg.max_sessions = max_sessions
        cfg.format = {"q4s": L.FMT_Q4S, "q8": L.FMT_Q8, "q4": L.FMT_Q4, "f16": L.FMT_F16}[weight_format]
        cfg.kv_dtype = {"f16": L.KV_F16, "bf16": L.KV_BF16}[kv_dtype]
        cfg.steps_per_graph = steps_per_graph
        if prefill_gemm_min is not None:
            cfg.prefill_gemm_min = prefill_gemm_min
        self.cfg = cfg
        h = C.c_void_p()
        L.check(self._lib.icua_engine_create(C.byref(cfg), C.byref(h)))
        self._h = h
        self._eos = (151645, 151643)
        self._stop_on_eos = True
        if model_path is not None:
            L.check(self._lib.icua_engine_load_file(self._h, model_path.encode()), self._h)
        if tensors is not None:
            self.set_tensors(tensors)

    # -- weights ---------------------------------------------------------------------------------
    def set_tensors(self, tensors: dict, ready: bool = True) -> None:
        """Uploads {tensor id: bytes}; ``ready`` then requires the language model to be complete
        (False for vision tensors alone)."""
        for tid in sorted(tensors):
            data = tensors[tid]
            buf = C.create_string_buffer(data, len(data)) if isinstance(data, (bytes, bytearray)) else data
            L.check(self._lib.icua_engine_set_tensor(self._h, tid, buf, len(data)), self._h)
        if ready:
            L.check(self._lib.icua_engine_ready(self._h), self._h)

    # -- reference properties ----------------------------------------------------------------------
    @property
    def eos(self):
        return self._eos

    @eos.setter
    def eos(self, pair):
        self._eos = (int(pair[0]), int(pair[1]))
        L.check(self._lib.icua_set_eos(self._h, self._eos[0], self._eos[1], int(self._stop_on_eos)), self._h)

    @property
    def stop_on_eos(self) -> bool:
        return self._stop_on_eos

    @stop_on_eos.setter
    def stop_on_eos(self, v: bool):
        self._stop_on_eos = bool(v)
        L.check(self._lib.icua_set_eos(self._h, self._eos[0], self._eos[1], int(self._stop_on_eos)), self._h)

    @property
    def last_timing(self) -> Timing:
        t = L.IcuaTiming()
        L.check(self._lib.icua_get_timing(self._h, C.byref(t)), self._h)
        return Timing(t.vision_ms, t.prefill_ms, t.decode_ms, t.total_ms, t.prefill_tokens, t.generated_tokens)

    # -- token loop --------------------------------------------------------------------------------
    @staticmethod
    def _visual(pooler, deepstack, grid):
        if pooler is None:
            return None, []
        keep = [np.ascontiguousarray(pooler, np.float32)]
        v = L.IcuaVisual()
        v.pooler = keep[0].ctypes.data_as(L._FP)
        for i in range(3):
            if deepstack is not None and i < len(deepstack) and deepstack[i] is not None:
                a = np.ascontiguousarray(deepstack[i], np.float32)
                keep.append(a)
                v.deepstack[i] = a.ctypes.data_as(L._FP)
            else:
                v.deepstack[i] = None
        v.n_vis = keep[0].shape[0]
        v.llm_h, v.llm_w = int(grid[0]), int(grid[1])
        return v, keep

    def generate_vision(self, tokens, max_new_tokens: int = 64, pooler=None, deepstack=None, grid=(0, 0),
                        write_first_logits: bool = False, session: int = 0) -> list:
        """Prefill + greedy decode (Engine.generateVision minus the ViT); returns generated tokens
        without the EOS token."""
        toks = np.ascontiguousarray(tokens, np.int32)
        vis, keep = self._visual(pooler, deepstack, grid)
        out = np.zeros(max(max_new_tokens, 1), np.int32)
        n = C.c_int32()
        L.check(self._lib.icua_generate(self._h, session, toks.ctypes.data_as(L._IP), len(toks),
                                        C.byref(vis) if vis is not None else None, max_new_tokens,
                                        int(write_first_logits), out.ctypes.data_as(L._IP), C.byref(n)), self._h)
        del keep
        return out[: n.value].tolist()

    def encode_vision(self, rgb) -> tuple:
        """Vision encoder + mergers on an RGB8 image [height, width, 3] (reference encodeVision,
        Engine.swift:317-473).  Returns (pooler [n_vis, 2048], deepstack [3, n_vis, 2048]) as host
        copies; the rows also stay on the device for the next prompt (``generate_rgb``)."""
        img = np.ascontiguousarray(rgb, np.uint8)
        h, w = img.shape[:2]
        nv = (h // 32) * (w // 32)
        pooler = np.zeros((max(nv, 1), 2048), np.float32)
        ds = np.zeros((3, max(nv, 1), 2048), np.float32)
        n = C.c_int32()
        L.check(self._lib.icua_encode_vision(self._h, img.ctypes.data, w, h, pooler.ctypes.data, ds.ctypes.data,
                                             C.byref(n)), self._h)
        return pooler[: n.value], ds[:, : n.value]

    def generate_rgb(self, rgb, tokens, max_new_tokens: int = 64, write_first_logits: bool = False,
                     session: int = 0) -> list:
        """Engine.generateVision(rgbBytes:width:height:tokens:...): vision encoder on the image, then
        prefill (the prompt's IMAGE_PAD block takes the encoder's rows) and greedy decode."""
        img = np.ascontiguousarray(rgb, np.uint8)
        h, w = img.shape[:2]
        toks = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(max(max_new_tokens, 1), np.int32)
        n = C.c_int32()
        L.check(self._lib.icua_generate_rgb(self._h, session, img.ctypes.data, w, h, toks.ctypes.data_as(L._IP),
                                            len(toks), max_new_tokens, int(write_first_logits),
                                            out.ctypes.data_as(L._IP), C.byref(n)), self._h)
        return out[: n.value].tolist()

    def reset(self, session: int = 0) -> None:
        L.check(self._lib.icua_reset_session(self._h, session), self._h)

    def prefill(self, tokens, pooler=None, deepstack=None, grid=(0, 0), write_logits: bool = False,
                session: int = 0) -> int:
        toks = np.ascontiguousarray(tokens, np.int32)
        vis, keep = self._visual(pooler, deepstack, grid)
        first = C.c_int32()
        L.check(self._lib.icua_prefill(self._h, session, toks.ctypes.data_as(L._IP), len(toks),
                                       C.byref(vis) if vis is not None else None, int(write_logits),
                                       C.byref(first)), self._h)
        del keep
        return first.value

    def decode(self, max_new: int, session: int = 0) -> list:
        out = np.zeros(max(max_new, 1), np.int32)
        n = C.c_int32()
        L.check(self._lib.icua_decode(self._h, session, max_new, out.ctypes.data_as(L._IP), C.byref(n)), self._h)
        return out[: n.value].tolist()

    @property
    def use_prefix_cache(self) -> bool:
        return getattr(self, "_prefix_cache", True)

    @use_prefix_cache.setter
    def use_prefix_cache(self, on: bool) -> None:
        """Engine.usePrefixCache: reuse the K/V of an unchanged system prompt before the image."""
        L.check(self._lib.icua_set_prefix_cache(self._h, int(bool(on))), self._h)
        self._prefix_cache = bool(on)

    def set_grammar_commit(self, enable: bool = True, actions=None, comma=None, space=None, open_=None,
                           close=None) -> None:
        """Grammar-guided 2-token commit (reference k_commit, Shaders.swift:1497-1571), opt-in.

        With no ids the reference's are used ('(' 7, ')' 8, ',' 11, ' ' 220 and its eight action
        words); passing any id replaces the whole rule, the others taking the reference's values.
        """
        rule = None
        if any(v is not None for v in (actions, comma, space, open_, close)):
            acts = list(actions) if actions is not None else list(REFERENCE_GRAMMAR["actions"])
            if len(acts) > 8:
                raise ValueError("at most 8 action ids")
            rule = L.IcuaGrammar()
            rule.n_action = len(acts)
            for i, a in enumerate(acts):
                rule.action[i] = int(a)
            ref = REFERENCE_GRAMMAR
            rule.comma = int(ref["comma"] if comma is None else comma)
            rule.space = int(ref["space"] if space is None else space)
            rule.open = int(ref["open"] if open_ is None else open_)
            rule.close = int(ref["close"] if close is None else close)
        L.check(self._lib.icua_set_grammar_commit(self._h, int(bool(enable)), C.byref(rule) if rule is not None else None),
                self._h)

    def decode_batch(self, sessions, steps: int, in_tokens=None) -> np.ndarray:
        """Batched greedy decode of several sessions at once; returns int32 [len(sessions), steps]
        (-1 after a session's EOS)."""
        ss = np.ascontiguousarray(sessions, np.int32)
        out = np.zeros((len(ss), max(steps, 1)), np.int32)
        it = None if in_tokens is None else np.ascontiguousarray(in_tokens, np.int32)
        L.check(self._lib.icua_decode_batch(self._h, ss.ctypes.data_as(L._IP), len(ss),
                                            it.ctypes.data_as(L._IP) if it is not None else None, steps,
                                            out.ctypes.data_as(L._IP)), self._h)
        return out[:, :steps]

    def capture_batch_logits(self, rows: int | None):
        """Returns a host array [rows, vocab] that the next decode_batch calls fill with the logits
        of their last step (or None to stop)."""
        if not rows:
            L.check(self._lib.icua_capture_batch_logits(self._h, None, 0), self._h)
            self._bcap = None
            return None
        self._bcap = np.zeros((rows, self.cfg.vocab), np.float32)
        L.check(self._lib.icua_capture_batch_logits(self._h, self._bcap.ctypes.data_as(L._FP), rows), self._h)
        return self._bcap

    def decode_step(self, in_token: int, session: int = 0) -> int:
        o = C.c_int32()
        L.check(self._lib.icua_decode_step(self._h, session, int(in_token), C.byref(o)), self._h)
        return o.value

    def logits(self) -> np.ndarray:
        out = np.empty(self.cfg.vocab, np.float32)
        L.check(self._lib.icua_get_logits(self._h, out.ctypes.data_as(L._FP)), self._h)
        return out

    def capture_step_logits(self, steps: int | None):
        """Returns a host array the next prefill / decode fills with per-step logits (or None)."""
        if steps is None:
            L.check(self._lib.icua_capture_step_logits(self._h, None, 0), self._h)
            self._cap = None
            return None
        self._cap = np.zeros((steps, self.cfg.vocab), np.float32)
        L.check(self._lib.icua_capture_step_logits(self._h, self._cap.ctypes.data_as(L._FP), steps), self._h)
        return self._cap

    def inject_kv(self, k: np.ndarray, v: np.ndarray, session: int = 0) -> None:
        """k, v: fp32 [n_layers, n_pos, 8, 128]."""
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        L.check(self._lib.icua_inject_kv(self._h, session, k.ctypes.data_as(L._FP), v.ctypes.data_as(L._FP),
                                         k.shape[1]), self._h)

    def inject_kv_random(self, n_pos: int, seed: int = 2, session: int = 0) -> None:
        L.check(self._lib.icua_inject_kv_random(self._h, session, n_pos, seed), self._h)

    @property
    def kernels_per_step(self) -> int:
        """Kernels one decode step launches (3 on the persistent layers kernel)."""
        return int(self._lib.icua_decode_kernels_per_step(self._h))

    @property
    def attn_o_cluster(self) -> int:
        """CTAs per cluster of the decode attention with the o-projection folded in (0: separate
        o-proj GEMV launch)."""
        return int(self._lib.icua_attn_o_cluster(self._h))

    @property
    def device_bytes(self) -> int:
        """Bytes of device memory the engine holds (its own allocations)."""
        return int(self._lib.icua_device_bytes(self._h))

    def profile_decode(self, steps: int, session: int = 0) -> tuple:
        """Decodes ``steps`` tokens with CUDA events around each step's layers and lm_head + commit;
        returns (layers ms, head ms) summed over the steps."""
        a, b = C.c_double(), C.c_double()
        L.check(self._lib.icua_profile_decode(self._h, session, steps, C.byref(a), C.byref(b)), self._h)
        return a.value, b.value

    def position(self, session: int = 0) -> int:
        p = C.c_int32()
        L.check(self._lib.icua_session_position(self._h, session, C.byref(p)), self._h)
        return p.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.icua_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
