"""Torch-facing wrappers over the C-ABI kernels.

These functions take CUDA tensors, call ``libtsb_moe.so`` on the current CUDA
stream and return CUDA tensors.  CPU tensors are rejected: there is no CPU
path in the product.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .formats import FORMATS, TSB_MXFP4, mxfp4_split

_DT = {torch.float32: _lib.DT_F32, torch.bfloat16: _lib.DT_BF16, torch.float16: _lib.DT_F16}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("tinyserve_b200 kernels need CUDA tensors")


def dequant(fmt: int, w: torch.Tensor, scales: torch.Tensor | None, rows: int, cols: int,
            dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Bit-exact dequantisation (same values as ``dequant_tensor`` /
    ``dequant_mxfp4_no_transpose``) of a [rows, cols] weight."""
    _require_cuda(w, scales)
    if dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("dequant dtype must be float32 or bfloat16")
    out = torch.empty(rows, cols, dtype=dtype, device=w.device)
    _lib.check(_lib.lib().tsb_dequant(fmt, _ptr(w), _ptr(scales), rows, cols, _ptr(out), _DT[dtype],
                                      _stream(w.device)))
    return out


def quant_matvec(fmt: int, w: torch.Tensor, scales: torch.Tensor | None, out_features: int, in_features: int,
                 x: torch.Tensor, out_dtype: torch.dtype | None = None,
                 dev_err: torch.Tensor | None = None) -> torch.Tensor:
    """y[M, N] = x[M, K] @ W[N, K]^T with W quantised; x is fp32/bf16/fp16 [M, K]."""
    _require_cuda(w, scales, x)
    if x.dim() == 1:
        x = x.view(1, -1)
    x = x.contiguous()
    M = x.shape[0]
    if x.shape[1] != in_features:
        raise ValueError(f"x has {x.shape[1]} features, expected {in_features}")
    y = torch.empty(M, out_features, dtype=out_dtype or x.dtype, device=x.device)
    _lib.check(_lib.lib().tsb_quant_matvec(
        fmt, _ptr(w), _ptr(scales), out_features, in_features, _ptr(x), _DT[x.dtype], M, in_features,
        _ptr(y), _DT[y.dtype], out_features, _ptr(dev_err), _stream(x.device)))
    return y


def weight_bytes(fmt: int, rows: int, cols: int) -> tuple[int, int]:
    d, s = ctypes.c_int64(), ctypes.c_int64()
    _lib.check(_lib.lib().tsb_weight_bytes(fmt, rows, cols, ctypes.byref(d), ctypes.byref(s)))
    return d.value, s.value


# ---------------------------------------------------------------------------
# Drop-in for torch.ops.tinyserve_ggml.ggml_mul_mat_vec
# (tinyserve/csrc/ggml_ops.cu:461-574): same schema, argument meaning, output
# dtype and error messages; callers ggml_forward.py:103-115 and
# ggml_linear.py:77-100 keep working unchanged.
# ---------------------------------------------------------------------------
def ggml_mul_mat_vec(activation: torch.Tensor, weight_data: torch.Tensor, ggml_type: int,
                     out_features: int, in_features: int) -> torch.Tensor:
    if not activation.is_cuda:
        raise RuntimeError("activation must be on CUDA")
    if not weight_data.is_cuda:
        raise RuntimeError("weight_data must be on CUDA")
    if weight_data.dtype != torch.uint8:
        raise RuntimeError("weight_data must be uint8")
    if ggml_type not in FORMATS or ggml_type == TSB_MXFP4:
        raise RuntimeError(f"Unsupported ggml_type: {ggml_type}. Supported: Q8_0(8), Q4_K(12), Q5_K(13), Q6_K(14)")
    _, bb, be = FORMATS[ggml_type]
    if in_features % 32 or (out_features * in_features) % be:
        raise RuntimeError(f"in_features ({in_features}) must be divisible by block_elements ({be})")
    expected = out_features * in_features // be * bb
    if weight_data.numel() < expected:
        raise RuntimeError(f"weight_data too small: got {weight_data.numel()} bytes, expected {expected}")
    act = activation.contiguous().view(-1)
    if act.numel() < in_features:
        raise RuntimeError(f"activation too small: got {act.numel()} elements, expected {in_features}")
    if act.dtype not in _DT:
        act = act.float()
    y = quant_matvec(ggml_type, weight_data, None, out_features, in_features, act[:in_features].view(1, -1),
                     out_dtype=activation.dtype if activation.dtype in _DT else torch.float32)
    return y.view(1, out_features).to(activation.dtype)


_registered = False


def register_torch_op() -> None:
    """Register ``torch.ops.tinyserve_ggml.ggml_mul_mat_vec`` (schema of ggml_ops.cu:571-574)."""
    global _registered
    if _registered or hasattr(torch.ops, "tinyserve_ggml") and hasattr(torch.ops.tinyserve_ggml, "ggml_mul_mat_vec"):
        _registered = True
        return
    lib = torch.library.Library("tinyserve_ggml", "DEF")
    lib.define("ggml_mul_mat_vec(Tensor activation, Tensor weight_data, int ggml_type, int out_features, "
               "int in_features) -> Tensor")
    lib.impl("ggml_mul_mat_vec", ggml_mul_mat_vec, "CUDA")
    register_torch_op._lib = lib  # keep the Library object alive
    _registered = True


def mxfp4_weight_views(blocks: torch.Tensor, scales: torch.Tensor, rows: int, cols: int):
    """Validate MXFP4 tensors of a [rows, cols] weight (blocks [rows, cols/32, 16], scales [rows, cols/32])."""
    nb, ns = mxfp4_split(rows, cols)
    if blocks.numel() != nb or scales.numel() != ns:
        raise ValueError(f"MXFP4 [{rows},{cols}] needs {nb} block bytes and {ns} scale bytes")
    return blocks, scales
