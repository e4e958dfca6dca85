"""ctypes binding of libb2d.so (the C ABI in include/b2d.h).

The library is the product path: if it is missing or fails to load, every
entry point raises.  There is no CPU or PyTorch fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libb2d.so")

# b2d_status
B2D_OK = 0
B2D_ERR_INVALID_ARG = 1
B2D_ERR_UNSUPPORTED = 2
B2D_ERR_CUDA = 3
B2D_ERR_NO_MEMORY = 4
B2D_ERR_LAUNCH = 5
B2D_ERR_DEVICE_TIMEOUT = 6
B2D_ERR_DEVICE_INPUT = 7
B2D_ERR_DEVICE_HALTED = 8
B2D_ERR_SCRATCH_LIMIT = 9


class B2DError(RuntimeError):
    def __init__(self, status: int, where: str, detail: str = ""):
        self.status = status
        msg = f"{where}: {status_str(status)} (status {status})"
        if detail:
            msg += f": {detail}"
        super().__init__(msg)


class Config(ctypes.Structure):
    _fields_ = [("vocab_size", ctypes.c_int32), ("d_model", ctypes.c_int32),
                ("n_heads", ctypes.c_int32), ("n_kv_heads", ctypes.c_int32),
                ("n_layers", ctypes.c_int32), ("d_head", ctypes.c_int32),
                ("d_ff", ctypes.c_int32), ("context_len", ctypes.c_int32),
                ("rms_eps", ctypes.c_float), ("rope_base", ctypes.c_float)]


class WeightsLayout(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in
                ("layer_stride", "off_qkv", "off_o", "off_gu", "off_down", "off_emb",
                 "off_ln1", "off_ln2", "off_lnf", "off_cos", "off_sin", "total_bytes")]


class KVLayout(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in ("elems_per_seq", "layer_elems", "kv_half_elems")]


class Sampling(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_double), ("top_p", ctypes.c_double),
                ("rep_penalty", ctypes.c_double)]


#: every symbol include/b2d.h declares, with (restype, argtypes)
_P = ctypes.c_void_p
_SIGS = {
    "b2d_status_str": (ctypes.c_char_p, [ctypes.c_int]),
    "b2d_cuda_error": (ctypes.c_char_p, []),
    "b2d_config_supported": (ctypes.c_int, [ctypes.POINTER(Config)]),
    "b2d_weights_layout": (ctypes.c_int, [ctypes.POINTER(Config), ctypes.POINTER(WeightsLayout)]),
    "b2d_kv_layout": (ctypes.c_int, [ctypes.POINTER(Config), ctypes.POINTER(KVLayout)]),
    "b2d_model_create": (ctypes.c_int, [ctypes.POINTER(Config), _P, ctypes.c_uint64, ctypes.c_int,
                                        ctypes.POINTER(_P)]),
    "b2d_model_destroy": (ctypes.c_int, [_P]),
    "b2d_model_grid": (ctypes.c_int, [_P]),
    "b2d_workspace_create": (ctypes.c_int, [_P, ctypes.c_int, ctypes.POINTER(_P)]),
    "b2d_workspace_destroy": (ctypes.c_int, [_P]),
    "b2d_workspace_reset": (ctypes.c_int, [_P, _P]),
    "b2d_last_error": (ctypes.c_int, [_P, _P, ctypes.POINTER(ctypes.c_uint32)]),
    "b2d_decode_step": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_int, _P, _P, _P, _P]),
    "b2d_decode_token": (ctypes.c_int, [_P, _P, ctypes.c_int32, ctypes.c_int32, _P, _P, ctypes.POINTER(ctypes.c_int32),
                                        _P]),
    "b2d_decode_steps": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_int, _P, _P, _P, _P]),
    "b2d_decode_step_paged": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_int, _P, _P, ctypes.c_int, ctypes.c_int,
                                             _P, _P, _P]),
    "b2d_prefill": (ctypes.c_int, [_P, _P, _P, ctypes.c_int, ctypes.c_int, _P, _P, _P, _P]),
    "b2d_prefill_paged": (ctypes.c_int, [_P, _P, _P, ctypes.c_int, ctypes.c_int, _P, _P, ctypes.c_int,
                                         ctypes.c_int, _P, _P, _P]),
    "b2d_prefill_rows": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_int, _P, _P, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int, _P, _P, _P]),
    "b2d_prefill_rows_max": (ctypes.c_int, []),
    "b2d_batched_launches": (ctypes.c_int, [_P]),
    "b2d_sample": (ctypes.c_int, [_P, _P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, _P, _P,
                                  ctypes.POINTER(Sampling), _P, _P]),
    "b2d_decode_step_static": (ctypes.c_int, [ctypes.POINTER(Config), _P, ctypes.c_uint64, _P, _P, _P, _P,
                                              _P, _P]),
    "b2d_static_last_error": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_uint32)]),
    "b2d_debug_set": (ctypes.c_int, [_P, ctypes.c_uint64, ctypes.c_int]),
    "b2d_debug_trace": (ctypes.c_int, [_P, _P, ctypes.c_int]),
    "b2d_debug_tune": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_int64]),
    "b2d_test_gemm": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, ctypes.c_int, _P, _P, _P,
                                     ctypes.c_int, _P]),
}

_lib = None
_lock = threading.Lock()


def load(path: str = LIB_PATH):
    """Load libb2d.so (raises if absent: the GPU path has no fallback)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: build it with `python -m transformer_b200.build` "
                               "(there is no CPU fallback for the decode path)")
        lib = ctypes.CDLL(path)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def status_str(s: int) -> str:
    try:
        return load().b2d_status_str(int(s)).decode()
    except Exception:  # library missing: still produce a message
        return f"status {s}"


def check(status: int, where: str):
    if status != B2D_OK:
        detail = ""
        if status == B2D_ERR_CUDA or status == B2D_ERR_LAUNCH or status == B2D_ERR_NO_MEMORY:
            detail = load().b2d_cuda_error().decode()
        raise B2DError(status, where, detail)


def make_config(cfg) -> Config:
    return Config(cfg.vocab_size, cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.n_layers,
                  cfg.d_head, cfg.d_ff, cfg.context_len, cfg.rms_eps, cfg.rope_base)


def weights_layout(cfg) -> WeightsLayout:
    lay = WeightsLayout()
    c = make_config(cfg)
    check(load().b2d_weights_layout(ctypes.byref(c), ctypes.byref(lay)), "b2d_weights_layout")
    return lay


def kv_layout(cfg) -> KVLayout:
    lay = KVLayout()
    c = make_config(cfg)
    check(load().b2d_kv_layout(ctypes.byref(c), ctypes.byref(lay)), "b2d_kv_layout")
    return lay
