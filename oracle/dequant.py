"""Bit-exact numpy restatement of the reference decoders (test infrastructure).

Follows, operation by operation and with the same float32 rounding steps:

- ``tinyserve/gguf_dequant_torch.py:35-78``  ``dequant_tensor`` (flat stream of
  blocks over the row-major buffer, then reshape)
- ``tinyserve/gguf_dequant_torch.py:118-122`` Q8_0
- ``tinyserve/gguf_dequant_torch.py:95-111``  K-quant 6-bit scale/min unpack
- ``tinyserve/gguf_dequant_torch.py:187-203`` Q4_K
- ``tinyserve/gguf_dequant_torch.py:206-227`` Q5_K
- ``tinyserve/gguf_dequant_torch.py:230-249`` Q6_K
- ``tinyserve/mxfp4.py:5-44``                 MXFP4 (``dequant_mxfp4_no_transpose``)

The reference computes ``(d * sc) * q - dmin * m`` as separately rounded
float32 operations (torch has no FMA contraction on CPU tensors); numpy
float32 arithmetic rounds the same way, so results are bit-identical.
"""
from __future__ import annotations

import numpy as np

GGML_Q8_0 = 8
GGML_Q4_K = 12
GGML_Q5_K = 13
GGML_Q6_K = 14
# MXFP4 has no ggml type id in the reference (gguf_reader.py:15-29); the
# product uses a private id outside ggml's table.
TSB_MXFP4 = 39

# (block_elements, block_bytes): gguf_dequant_torch.py:20-29
QUANT_SIZES = {
    GGML_Q8_0: (32, 34),
    GGML_Q4_K: (256, 144),
    GGML_Q5_K: (256, 176),
    GGML_Q6_K: (256, 210),
}

# mxfp4.py:5-8
FP4_LUT = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
    dtype=np.float32,
)


def _f16(b: np.ndarray) -> np.ndarray:
    """Little-endian fp16 from 2 bytes per row -> float32 (exact)."""
    return np.ascontiguousarray(b).view(np.float16).astype(np.float32)


def _scale_min(scales: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """6-bit scales / mins of K-quants (gguf_dequant_torch.py:95-111)."""
    s = scales.reshape(-1, 3, 4)
    d, m, md = s[:, 0], s[:, 1], s[:, 2]
    sc = np.concatenate([d & 0x3F, (md & 0x0F) | ((d >> 2) & 0x30)], axis=-1)
    mn = np.concatenate([m & 0x3F, (md >> 4) | ((m >> 2) & 0x30)], axis=-1)
    return sc.reshape(-1, 8), mn.reshape(-1, 8)


def _q8_0(b: np.ndarray) -> np.ndarray:
    d = _f16(b[:, 0:2])
    x = b[:, 2:34].view(np.int8).astype(np.float32)
    return d * x


def _q4_k(b: np.ndarray) -> np.ndarray:
    n = b.shape[0]
    d = _f16(b[:, 0:2])
    dmin = _f16(b[:, 2:4])
    sc, m = _scale_min(b[:, 4:16])
    dsc = (d * sc.astype(np.float32)).reshape(n, 8, 1)
    dm = (dmin * m.astype(np.float32)).reshape(n, 8, 1)
    qs = b[:, 16:144].reshape(n, 4, 1, 32)
    q = np.concatenate([qs & 0x0F, qs >> 4], axis=2).reshape(n, 8, 32).astype(np.float32)
    return (dsc * q - dm).reshape(n, 256)


def _q5_k(b: np.ndarray) -> np.ndarray:
    n = b.shape[0]
    d = _f16(b[:, 0:2])
    dmin = _f16(b[:, 2:4])
    sc, m = _scale_min(b[:, 4:16])
    dsc = (d * sc.astype(np.float32)).reshape(n, 8, 1)
    dm = (dmin * m.astype(np.float32)).reshape(n, 8, 1)
    qh = b[:, 16:48].reshape(n, 1, 32)
    qs = b[:, 48:176].reshape(n, 4, 1, 32)
    ql = np.concatenate([qs & 0x0F, qs >> 4], axis=2).reshape(n, 8, 32)
    hb = np.stack([(qh[:, 0] >> j) & 1 for j in range(8)], axis=1)  # [n, 8, 32]
    q = (ql | (hb << 4)).astype(np.float32)
    return (dsc * q - dm).reshape(n, 256)


def _q6_k(b: np.ndarray) -> np.ndarray:
    n = b.shape[0]
    ql = b[:, 0:128].reshape(n, 2, 1, 64)
    qh = b[:, 128:192].reshape(n, 2, 1, 32)
    scales = b[:, 192:208].view(np.int8).astype(np.float32)
    d = _f16(b[:, 208:210])
    dsc = (d * scales).reshape(n, 16, 1)
    lo = np.concatenate([ql & 0x0F, ql >> 4], axis=2).reshape(n, 8, 32)
    hi = np.concatenate([(qh >> s) & 0x03 for s in (0, 2, 4, 6)], axis=2).reshape(n, 8, 32)
    q = ((lo | (hi << 4)).astype(np.int16) - 32).astype(np.float32).reshape(n, 16, 16)
    return (dsc * q).reshape(n, 256)


_DEQ = {GGML_Q8_0: _q8_0, GGML_Q4_K: _q4_k, GGML_Q5_K: _q5_k, GGML_Q6_K: _q6_k}


def dequant_tensor(data: np.ndarray | bytes, ggml_type: int, shape) -> np.ndarray:
    """float32 dequant of a flat GGUF block stream (gguf_dequant_torch.py:35-78)."""
    if ggml_type not in _DEQ:
        raise ValueError(f"Unsupported GGML quantization type {ggml_type}")
    raw = np.frombuffer(bytes(data), dtype=np.uint8) if isinstance(data, (bytes, bytearray)) \
        else np.ascontiguousarray(data, dtype=np.uint8).reshape(-1)
    be, bb = QUANT_SIZES[ggml_type]
    nb = raw.size // bb
    blocks = raw[: nb * bb].reshape(nb, bb)
    return _DEQ[ggml_type](blocks).reshape(shape).astype(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit pattern, NaN -> 0x7FC0
    (the conversion torch applies when it writes a float32 into bfloat16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0x7FC0), r)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def dequant_mxfp4_no_transpose(blocks: np.ndarray, scales: np.ndarray, out_dtype: str = "bf16") -> np.ndarray:
    """MXFP4 -> [N, 32G] (mxfp4.py:20-44).

    Low nibble of byte b of group g is element 32g+2b, high nibble 32g+2b+1.
    ``torch.ldexp(out, si)`` is an exact power-of-two scaling (scale byte 255
    gives 0.5*2^128 = 2^127, and 0 * 2^128 = 0, not NaN); results too large
    for float32 become +-inf.  Every finite result has at most two
    significant bits, so the bfloat16 output is the same value.  Returns
    float32 values for ``out_dtype='f32'`` and bfloat16 *bit patterns*
    (uint16) for ``out_dtype='bf16'``.
    """
    blocks = np.asarray(blocks, dtype=np.uint8)
    scales = np.asarray(scales, dtype=np.uint8)
    n, g, b = blocks.shape
    lo = FP4_LUT[blocks & 0x0F]
    hi = FP4_LUT[blocks >> 4]
    v = np.empty((n, g, 2 * b), dtype=np.float32)
    v[..., 0::2] = lo
    v[..., 1::2] = hi
    with np.errstate(invalid="ignore", over="ignore"):
        out = np.ldexp(v, (scales.astype(np.int32) - 127)[..., None]).astype(np.float32).reshape(n, g * 2 * b)
    if out_dtype == "f32":
        return out
    return f32_to_bf16_bits(out)
