"""ctypes binding of ``libicua_cuda.so`` (the C ABI declared in ``include/icua.h``).

The library is built in-tree (``instantcua_b200/libicua_cuda.so``).  Loading fails loudly when it
is missing: there is no CPU fallback for any operation of the engine.
"""
from __future__ import annotations

import ctypes as C
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libicua_cuda.so")

OK, ERR_INVALID, ERR_CUDA, ERR_OOM, ERR_IO, ERR_FORMAT, ERR_STATE, ERR_CAPACITY, ERR_UNSUPPORTED, ERR_TIMEOUT = range(10)
FMT_F16, FMT_Q8, FMT_Q4, FMT_Q4S = 0, 1, 2, 3
KV_F16, KV_BF16 = 0, 1
TID_EMBED, TID_EMBED_SB, TID_FINAL_NORM, TID_LAYER_BASE, TID_PER_LAYER = 315, 316, 317, 318, 14
SLOT = dict(attn_norm=0, wqkv=1, wqkv_sb=2, q_norm=3, k_norm=4, wo=5, wo_sb=6, mlp_norm=7, wgu=8, wgu_sb=9,
            wd=10, wd_sb=11)
TENSOR_COUNT = 710


class IcuaConfig(C.Structure):
    _fields_ = [("device", C.c_int32), ("n_layers", C.c_int32), ("vocab", C.c_int32), ("max_context", C.c_int32),
                ("max_pass", C.c_int32), ("max_steps", C.c_int32), ("max_sessions", C.c_int32),
                ("format", C.c_int32), ("kv_dtype", C.c_int32), ("steps_per_graph", C.c_int32),
                ("prefill_gemm_min", C.c_int32)]


class IcuaTiming(C.Structure):
    _fields_ = [("vision_ms", C.c_double), ("prefill_ms", C.c_double), ("decode_ms", C.c_double),
                ("total_ms", C.c_double), ("prefill_tokens", C.c_int32), ("generated_tokens", C.c_int32)]


class IcuaGrammar(C.Structure):
    _fields_ = [("n_action", C.c_int32), ("action", C.c_int32 * 8), ("comma", C.c_int32), ("space", C.c_int32),
                ("open", C.c_int32), ("close", C.c_int32)]


class IcuaVisual(C.Structure):
    _fields_ = [("pooler", C.POINTER(C.c_float)), ("deepstack", C.POINTER(C.c_float) * 3), ("n_vis", C.c_int32),
                ("llm_h", C.c_int32), ("llm_w", C.c_int32)]


class IcuaError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"icua status {status}: {msg}")
        self.status = status


_P = C.c_void_p
_I = C.c_int32
_FP = C.POINTER(C.c_float)
_IP = C.POINTER(C.c_int32)

# name -> (restype, argtypes); every function declared in include/icua.h
PROTOTYPES = {
    "icua_default_config": (None, [C.POINTER(IcuaConfig)]),
    "icua_engine_create": (_I, [C.POINTER(IcuaConfig), C.POINTER(_P)]),
    "icua_engine_destroy": (None, [_P]),
    "icua_last_error": (C.c_char_p, [_P]),
    "icua_global_error": (C.c_char_p, []),
    "icua_engine_load_file": (_I, [_P, C.c_char_p]),
    "icua_engine_set_tensor": (_I, [_P, _I, _P, C.c_uint64]),
    "icua_engine_ready": (_I, [_P]),
    "icua_set_eos": (_I, [_P, _I, _I, _I]),
    "icua_prefill": (_I, [_P, _I, _IP, _I, C.POINTER(IcuaVisual), _I, _IP]),
    "icua_decode": (_I, [_P, _I, _I, _IP, _IP]),
    "icua_decode_step": (_I, [_P, _I, _I, _IP]),
    "icua_generate": (_I, [_P, _I, _IP, _I, C.POINTER(IcuaVisual), _I, _I, _IP, _IP]),
    "icua_encode_vision": (_I, [_P, C.c_void_p, _I, _I, C.c_void_p, C.c_void_p, _IP]),
    "icua_generate_rgb": (_I, [_P, _I, C.c_void_p, _I, _I, _IP, _I, _I, _I, _IP, _IP]),
    "icua_reset_session": (_I, [_P, _I]),
    "icua_inject_kv": (_I, [_P, _I, _FP, _FP, _I]),
    "icua_inject_kv_random": (_I, [_P, _I, _I, C.c_uint64]),
    "icua_get_logits": (_I, [_P, _FP]),
    "icua_capture_step_logits": (_I, [_P, _FP, _I]),
    "icua_get_timing": (_I, [_P, C.POINTER(IcuaTiming)]),
    "icua_session_position": (_I, [_P, _I, _IP]),
    "icua_packed_bytes": (C.c_uint64, [_I, _I, _I]),
    "icua_pack_matrix": (_I, [_I, _I, _I, _P, _P, _P]),
    "icua_gemv": (_I, [_I, _I, _I, _P, _P, _I, _P, _P]),
    "icua_decode_batch": (_I, [_P, _IP, _I, _IP, _I, _IP]),
    "icua_set_prefix_cache": (_I, [_P, _I]),
    "icua_set_grammar_commit": (_I, [_P, _I, C.POINTER(IcuaGrammar)]),
    "icua_capture_batch_logits": (_I, [_P, _FP, _I]),
    "icua_gemm_q4s": (_I, [_I, _I, _I, _P, _P, _P, _P, _P]),
    "icua_dequant_q4s_f16": (_I, [_I, _I, _P, _P, _P]),
    "icua_gemm_f16": (_I, [_I, _I, _I, _P, _P, _P, _P, _P]),
    "icua_dequant": (_I, [_I, _I, _I, _P, _P, _P]),
    "icua_greedy_head_scratch_bytes": (C.c_uint64, [_I]),
    "icua_greedy_head": (_I, [_I, _P, _P, _P, _P, _P, _P, _P]),
    "icua_greedy_head_noalloc": (_I, [_I, _P, _P, _P, _P, _P, _P]),
    "icua_set_wait_limit": (_I, [C.c_uint32]),
    "icua_decode_kernels_per_step": (_I, [_P]),
    "icua_device_bytes": (C.c_uint64, [_P]),
    "icua_attn_o_cluster": (_I, [_P]),
    "icua_profile_decode": (_I, [_P, _I, _I, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "icua_quantize_q8": (_I, [_FP, _I, _I, _P, _P]),
    "icua_quantize_q4s": (_I, [_FP, _I, _I, _P, _P]),
}

_lib = None


def lib() -> C.CDLL:
    """Loads the library once; raises if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m instantcua_b200.build` (no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, eng=None) -> None:
    if status != OK:
        L = lib()
        msg = (L.icua_last_error(eng) if eng else L.icua_global_error()) or b""
        raise IcuaError(status, msg.decode(errors="replace"))
