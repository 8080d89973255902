"""ctypes binding of the in-tree C-ABI library ``libtsb_moe.so``.

The library is the product: there is no CPU or pure-PyTorch fallback.  If the
shared object is missing or cannot be loaded, :func:`lib` raises immediately.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from .formats import GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_Q8_0, TSB_MXFP4  # noqa: F401

LIB_PATH = Path(__file__).resolve().parent / "libtsb_moe.so"

TSB_OK = 0
TSB_ERR_INVALID = 1
TSB_ERR_UNSUPPORTED = 2
TSB_ERR_CUDA = 3
TSB_ERR_WORKSPACE = 4
TSB_ERR_DEVICE = 5

DT_F32, DT_BF16, DT_F16 = 0, 1, 2
GU_SEPARATE, GU_INTERLEAVED, GU_CHUNKED = 0, 1, 2
ACT_SILU, ACT_SWIGLU_OAI = 0, 1
T_GATE_UP, T_DOWN = 1, 2  # TsbMoeSpec.transposed bits (dense formats)

# Every symbol include/tsb_moe.h declares.
EXPORTS = (
    "tsb_version", "tsb_last_error", "tsb_format_info", "tsb_weight_bytes", "tsb_dequant",
    "tsb_quant_matvec", "tsb_moe_decode_workspace", "tsb_moe_decode", "tsb_read_device_error",
    "tsb_moe_decode_noalloc", "tsb_moe_prefill_workspace", "tsb_moe_prefill",
    "tsb_moe_packed_bytes", "tsb_moe_pack", "tsb_moe_decode_packed_workspace", "tsb_moe_decode_packed",
    "tsb_moe_route", "tsb_ep_decode_workspace", "tsb_ep_moe_decode", "tsb_ep_prefill_workspace",
    "tsb_ep_moe_prefill", "tsb_gqa_decode_workspace", "tsb_gqa_decode_attention", "tsb_add_rmsnorm",
    "tsb_gemv_bf16", "tsb_norm_gemv_bf16", "tsb_gemv_bf16_residual", "tsb_gqa_decode_batch_workspace",
    "tsb_gqa_decode_attention_batch", "tsb_norm_qkv_attention",
)


class TsbMoeSpec(ctypes.Structure):
    _fields_ = [
        ("fmt_gate_up", ctypes.c_int32), ("fmt_down", ctypes.c_int32),
        ("hidden", ctypes.c_int32), ("inter", ctypes.c_int32),
        ("n_experts", ctypes.c_int32), ("top_k", ctypes.c_int32),
        ("gate_up_layout", ctypes.c_int32), ("activation", ctypes.c_int32),
        ("limit", ctypes.c_float), ("alpha", ctypes.c_float),
        ("out_f32", ctypes.c_int32), ("transposed", ctypes.c_int32),
    ]


class TsbExpert(ctypes.Structure):
    _fields_ = [
        ("gate", ctypes.c_void_p), ("up", ctypes.c_void_p), ("down", ctypes.c_void_p),
        ("gate_scales", ctypes.c_void_p), ("up_scales", ctypes.c_void_p), ("down_scales", ctypes.c_void_p),
        ("gate_bias", ctypes.c_void_p), ("up_bias", ctypes.c_void_p), ("down_bias", ctypes.c_void_p),
    ]


_lib = None
_lock = threading.Lock()

_vp, _i32, _i64, _sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t


def _declare(L: ctypes.CDLL) -> None:
    L.tsb_version.restype = ctypes.c_int
    L.tsb_last_error.argtypes = [ctypes.c_char_p, _sz]
    L.tsb_format_info.argtypes = [ctypes.c_int, ctypes.POINTER(_i32), ctypes.POINTER(_i32)]
    L.tsb_weight_bytes.argtypes = [ctypes.c_int, _i64, _i64, ctypes.POINTER(_i64), ctypes.POINTER(_i64)]
    L.tsb_dequant.argtypes = [ctypes.c_int, _vp, _vp, _i64, _i64, _vp, ctypes.c_int, _vp]
    L.tsb_quant_matvec.argtypes = [ctypes.c_int, _vp, _vp, _i64, _i64, _vp, ctypes.c_int, _i64, _i64, _vp,
                                   ctypes.c_int, _i64, _vp, _vp]
    L.tsb_moe_decode_workspace.argtypes = [ctypes.POINTER(TsbMoeSpec), _i32]
    L.tsb_moe_decode_workspace.restype = _sz
    L.tsb_moe_decode.argtypes = [ctypes.POINTER(TsbMoeSpec), _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]
    L.tsb_read_device_error.argtypes = [_vp, ctypes.POINTER(_i32), _vp]
    L.tsb_moe_prefill_workspace.argtypes = [ctypes.POINTER(TsbMoeSpec), _i32]
    L.tsb_moe_prefill_workspace.restype = _sz
    L.tsb_moe_prefill.argtypes = [ctypes.POINTER(TsbMoeSpec), _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]
    L.tsb_moe_route.argtypes = [ctypes.POINTER(TsbMoeSpec), _vp, _i32, _vp, _vp, _vp, _vp, _vp]
    L.tsb_moe_decode_noalloc.argtypes = [ctypes.POINTER(TsbMoeSpec), _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp]
    L.tsb_moe_packed_bytes.argtypes = [ctypes.POINTER(TsbMoeSpec)]
    L.tsb_moe_packed_bytes.restype = _sz
    L.tsb_moe_pack.argtypes = [ctypes.POINTER(TsbMoeSpec), _vp, _vp, _sz, _vp]
    L.tsb_moe_decode_packed_workspace.argtypes = [ctypes.POINTER(TsbMoeSpec), _i32]
    L.tsb_moe_decode_packed_workspace.restype = _sz
    L.tsb_moe_decode_packed.argtypes = [ctypes.POINTER(TsbMoeSpec), _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp,
                                        _vp, _sz, _vp]
    L.tsb_ep_decode_workspace.argtypes = [ctypes.POINTER(TsbMoeSpec), _i32, _i32, _i32]
    L.tsb_ep_decode_workspace.restype = _sz
    L.tsb_ep_moe_decode.argtypes = [ctypes.POINTER(TsbMoeSpec), _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _i32, _i32,
                                    _vp, _sz, _vp]
    L.tsb_gqa_decode_workspace.argtypes = [_i32, _i32, _i32]
    L.tsb_gqa_decode_workspace.restype = _sz
    L.tsb_gqa_decode_attention.argtypes = [_vp, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp,
                                           ctypes.c_float, _vp, _vp, _sz, _vp]
    L.tsb_gqa_decode_batch_workspace.argtypes = [_i32, _i32, _i32, _i32]
    L.tsb_gqa_decode_batch_workspace.restype = _sz
    L.tsb_gqa_decode_attention_batch.argtypes = [_vp, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _i32, _i32,
                                                 _i32, _vp, ctypes.c_float, _vp, _i32, _vp, _sz, _vp]
    L.tsb_gemv_bf16.argtypes = [_vp, _vp, _i32, _i32, _vp, _vp, _vp]
    L.tsb_norm_qkv_attention.argtypes = [_vp, _vp, _vp, _vp, ctypes.c_float, _vp, _vp, _i32, _i32, _i32, _i32, _vp,
                                         _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp, ctypes.c_float, _vp, _vp]
    L.tsb_norm_gemv_bf16.argtypes = [_vp, _vp, _vp, _vp, ctypes.c_float, _vp, _vp, _i32, _i32, _vp, _vp]
    L.tsb_gemv_bf16_residual.argtypes = [_vp, _vp, _i32, _i32, _vp, _vp, _vp, ctypes.c_float, _vp, _vp, _vp]
    L.tsb_add_rmsnorm.argtypes = [_vp, _vp, _i32, _vp, ctypes.c_float, _i32, _i32, _vp, _vp]
    L.tsb_ep_prefill_workspace.argtypes = [ctypes.POINTER(TsbMoeSpec), _i32, _i32]
    L.tsb_ep_prefill_workspace.restype = _sz
    L.tsb_ep_moe_prefill.argtypes = [ctypes.POINTER(TsbMoeSpec), _vp, _vp, _i32, _vp, _vp, _vp, _vp, _i32, _i32, _vp,
                                     _sz, _vp]


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it is missing (build it with ``python -m tinyserve_b200.build``)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(f"{LIB_PATH.name} is not built; run `python -m tinyserve_b200.build`")
                L = ctypes.CDLL(str(LIB_PATH))
                _declare(L)
                _lib = L
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().tsb_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != TSB_OK:
        raise RuntimeError(last_error() or f"tsb error {rc}")
