"""ctypes binding of libstealcode_cuda.so (the C ABI in include/stealcode_b200.h).

The shared library is built in-tree (``stealcode_b200/libstealcode_cuda.so``) by
``stealcode_b200.build``.  There is no fallback: if the library is missing or
fails to load, importing this module raises, so no caller can silently run a
CPU or PyTorch substitute.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libstealcode_cuda.so")

SC_OK = 0
SC_ERR_INVALID = -1
SC_ERR_ALLOC = -2
SC_ERR_CUDA = -3
SC_ERR_TIMEOUT = -4
SC_ERR_UNSUPPORTED = -5
SC_ERR_STATE = -6
SC_LAYOUT_FEATURE_MAJOR = 0
SC_LAYOUT_TIME_MAJOR = 1

_ERR_NAMES = {
    SC_ERR_INVALID: "SC_ERR_INVALID",
    SC_ERR_ALLOC: "SC_ERR_ALLOC",
    SC_ERR_CUDA: "SC_ERR_CUDA",
    SC_ERR_TIMEOUT: "SC_ERR_TIMEOUT",
    SC_ERR_UNSUPPORTED: "SC_ERR_UNSUPPORTED",
    SC_ERR_STATE: "SC_ERR_STATE",
}


class ScError(RuntimeError):
    """A negative return code from the C ABI, with sc_last_error()'s message."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"{_ERR_NAMES.get(code, code)}: {msg}")
        self.code = code


if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is missing: build it with `python -m stealcode_b200.build` "
        "(make -C stealcode_b200/csrc); there is no CPU fallback")

lib = ctypes.CDLL(LIB_PATH)

_P = c_void_p
_I = c_int64
# name: (restype, argtypes) -- must match include/stealcode_b200.h
SIGNATURES = {
    "sc_last_error": (c_char_p, []),
    "sc_abi_version": (c_int, []),
    "sc_device_status": (c_int, [POINTER(ctypes.c_uint32)]),
    "sc_launch_count": (ctypes.c_longlong, []),
    "sc_q8_repack": (c_int, [_P, _I, _I, _I, _I, POINTER(c_void_p)]),
    "sc_q8_repack_device": (c_int, [_P, _I, _I, _I, _I, _P, POINTER(c_void_p)]),
    "sc_q8w_free": (c_int, [_P]),
    "sc_q8w_shape": (c_int, [_P, POINTER(c_int64), POINTER(c_int64)]),
    "sc_q8w_device_layout": (c_int, [_P, POINTER(c_void_p), POINTER(c_void_p), POINTER(c_int64),
                                     POINTER(c_int64)]),
    "sc_q8_gemm_workspace_bytes": (c_int64, [_I, _I]),
    "sc_q8_gemm": (c_int, [_P, _P, _I, c_int32, _I, _P, _P, c_int32, _I, _P, _I, _P]),
    "sc_q8_gemm_noalloc": (c_int, [_P, _P, _I, c_int32, _I, _P, _P, c_int32, _I, _P]),
    "sc_q8_gemm_q": (c_int, [_P, _P, _P, _I, _I, _P, _P, c_int32, _I, _P]),
    "sc_q8_gemm_batch_workspace_bytes": (c_int64, [_P, c_int32]),
    "sc_q8_gemm_batch": (c_int, [_P, _P, _P, _P, c_int32, _I, c_int32, c_int32, _P, _I, _P]),
    "sc_q8mat_gemm_t": (c_int, [_P, _P, _I, _P]),
    "sc_q8_gemm_host": (c_int, [c_size_t, c_size_t, c_size_t, _P, c_size_t, c_size_t, c_size_t, _P, _P]),
    "sc_q8_quantize": (c_int, [_P, _I, _I, c_int32, _I, _P, _P, _P]),
    "sc_q8_block_dots": (c_int, [_P, _P, _I, c_int32, _I, _P, _P]),
    "sc_stream_encoder_create": (c_int, [_P, _P, c_int, _I, POINTER(c_void_p)]),
    "sc_stream_encoder_encode_new": (c_int, [_P, _P, _I, _I, c_int32, _P]),
    "sc_stream_encoder_total": (c_int64, [_P]),
    "sc_stream_encoder_frames": (c_int, [_P, _I, _I, _I, _P]),
    "sc_stream_encoder_output": (c_int, [_P, POINTER(c_void_p), POINTER(c_int64), POINTER(c_int64)]),
    "sc_stream_encoder_set_prompts": (c_int, [_P, _P]),
    "sc_stream_encoder_n_prompts": (c_int64, [_P]),
    "sc_stream_encoder_set_dump": (c_int, [_P, c_int32]),
    "sc_stream_encoder_set_concurrency": (c_int, [_P, c_int32]),
    "sc_stream_encoder_set_graphs": (c_int, [_P, c_int32]),
    "sc_stream_encoder_graph_stats": (c_int, [_P, POINTER(c_int64), POINTER(c_int64)]),
    "sc_stream_encoder_encode_new_host": (c_int, [_P, _P, c_int64, c_int64, c_int32, _P, _P, _P]),
    "sc_stream_encoder_dump": (c_int, [_P, c_int32, _P, POINTER(c_int64)]),
    "sc_stream_encoder_destroy": (c_int, [_P]),
    "sc_debug_set_device_alloc_cap": (c_int, [_I]),
    "sc_pre_encode_pointwise_relu": (c_int, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P]),
    "sc_rnnt_create": (c_int, [_P, _P, c_int, _I, POINTER(c_void_p)]),
    "sc_rnnt_decode_frames": (c_int, [_P, _P, _I, _P]),
    "sc_rnnt_tokens": (c_int, [_P, _I, _P, _P, c_int32, POINTER(c_int32)]),
    "sc_rnnt_tokens_device": (c_int, [_P, POINTER(c_void_p), POINTER(c_void_p), POINTER(c_void_p),
                                      POINTER(c_int32)]),
    "sc_rnnt_emitted": (c_int, [_P, _P]),
    "sc_rnnt_last_rounds": (c_int64, [_P]),
    "sc_rnnt_reset": (c_int, [_P, _I]),
    "sc_rnnt_state": (c_int, [_P, _I, _P, _P, POINTER(c_int32)]),
    "sc_rnnt_destroy": (c_int, [_P]),
    "sc_attn_stream": (c_int, [_P, _P, _P, _P, _I, _P, _P, _I, _I, _I, c_float,
                               _I, _I, _I, _I, _I, _I, _I, _P, _P]),
    "sc_attn_stream_host": (c_int, [_P, _P, _P, _P, _I, _P, _P, _I, _I, _I, c_float,
                                    _I, _I, _I, _I, _I, _I, _I, _P]),
    "sc_attn_stream_ring": (c_int, [_P, _I, _P, _P, _I, _P, _P, _I, _I, _P, _I,
                                    _P, _P, _I, _I, _I, c_float, _I, _I, _I,
                                    _I, _I, _I, _P, _I, _P]),
}

for _name, (_res, _args) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


def device_status() -> int:
    """Read and clear the kernels' status bits on the current device."""
    v = ctypes.c_uint32(0)
    check(lib.sc_device_status(ctypes.byref(v)))
    return v.value


def launch_count() -> int:
    """Kernel launches this library has issued in this process."""
    return int(lib.sc_launch_count())


def last_error() -> str:
    msg = lib.sc_last_error()
    return msg.decode() if msg else ""


def check(rc: int) -> None:
    """Raise ScError for a negative return code."""
    if rc != SC_OK:
        raise ScError(rc, last_error())
