"""Shared test helpers: seeded quantised weights and oracle references."""
from __future__ import annotations

import numpy as np
import torch

from oracle import dequant as OD
from tinyserve_b200 import quantize as Q
from tinyserve_b200.formats import GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_Q8_0, TSB_MXFP4

ALL_FMTS = [GGML_Q8_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, TSB_MXFP4]
FMT_NAMES = {GGML_Q8_0: "Q8_0", GGML_Q4_K: "Q4_K", GGML_Q5_K: "Q5_K", GGML_Q6_K: "Q6_K", TSB_MXFP4: "MXFP4"}


def make_weight(fmt: int, rows: int, cols: int, seed: int, std: float = 0.02, device="cpu"):
    """(data uint8, scales uint8 | None) of a seeded N(0, std) [rows, cols] weight."""
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(rows, cols, generator=g) * std
    if device != "cpu":
        w = w.to(device)
    if fmt == TSB_MXFP4:
        b, s = Q.quantize_mxfp4(w, rows, cols)
        return b.reshape(-1), s.reshape(-1)
    return Q.quantize(fmt, w), None


def oracle_dequant(fmt: int, data, scales, rows: int, cols: int) -> np.ndarray:
    """fp32 [rows, cols] reference dequantisation (the oracle)."""
    d = np.asarray(data.cpu() if isinstance(data, torch.Tensor) else data, dtype=np.uint8)
    if fmt == TSB_MXFP4:
        s = np.asarray(scales.cpu() if isinstance(scales, torch.Tensor) else scales, dtype=np.uint8)
        return OD.dequant_mxfp4_no_transpose(d.reshape(rows, cols // 32, 16), s.reshape(rows, cols // 32), "f32")
    return OD.dequant_tensor(d, fmt, (rows, cols))


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def bits_equal_f32(a: np.ndarray, b: np.ndarray) -> bool:
    """Bitwise float32 equality, with any NaN equal to any NaN."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    same = a.view(np.uint32) == b.view(np.uint32)
    return bool((same | (np.isnan(a) & np.isnan(b))).all())


def layer_bound(out, ref, tol: float = 1e-3) -> float:
    """Relative-L2 bound for a layer output against float64 oracle math: the
    north-star 1e-3 for fp32 outputs; for bf16 outputs the rounding of the
    output itself (rel_l2(bf16(ref), ref), about 1.1e-3) plus 1e-3, so a kernel
    with more than 1e-3 of its own error fails either way."""
    if out.dtype == torch.bfloat16:
        from oracle.expert import bf16_round
        r = np.asarray(ref, dtype=np.float64)
        return rel_l2(bf16_round(r.astype(np.float32)), r) + tol
    return tol


def assert_layer(out, ref, tol: float = 1e-3) -> float:
    """Assert a layer output tensor (bf16 or fp32, any device) is within
    layer_bound of the oracle reference; returns the measured error."""
    got = out.float().cpu().numpy()
    err = rel_l2(got, ref)
    bound = layer_bound(out, ref, tol)
    assert err <= bound, f"relative L2 {err:.3e} > {bound:.3e} ({out.dtype})"
    return err
