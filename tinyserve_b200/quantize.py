"""Round-to-nearest encoders for Q8_0, Q4_K, Q5_K, Q6_K and MXFP4.

The reference ships only a Q8_0 encoder (``tinyserve/mmap_store.py:280-306``,
``quantize_to_q8_0``); ``quantize_q8_0`` keeps its semantics (scale =
amax/127 clamped at 1e-10, ``round(x/scale)`` clamped to int8, scale stored
as fp16).  The K-quant and MXFP4 encoders are new: they write the byte
layouts that the reference decoders read (``gguf_dequant_torch.py:187-249``,
``mxfp4.py:20-44``) with plain per-block round-to-nearest choices.  Parity is
defined against the decoders, so encoder quality only affects how realistic
the synthetic weights are.

All encoders are vectorised torch code and run on whatever device the input
lives on (the GPU makes encoding a 448 MB expert set take well under a
second).  Input: a float tensor whose element count is a multiple of the
block size, read as one flat stream in row-major order (the flat-stream rule
of ``gguf_dequant_torch.py:72-78``).  Output: a flat uint8 tensor.
"""
from __future__ import annotations

import torch

from .formats import GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_Q8_0, TSB_MXFP4


def _f16_bytes(x: torch.Tensor) -> torch.Tensor:
    """[n] float -> [n, 2] little-endian fp16 bytes."""
    return x.to(torch.float16).contiguous().view(torch.uint8).reshape(-1, 2)


def quantize_q8_0(w: torch.Tensor) -> torch.Tensor:
    x = w.reshape(-1, 32).float()
    amax = x.abs().amax(dim=1)
    scale = (amax / 127.0).clamp(min=1e-10)
    q = torch.round(x / scale[:, None]).clamp(-128, 127).to(torch.int8)
    out = torch.empty(x.shape[0], 34, dtype=torch.uint8, device=x.device)
    out[:, 0:2] = _f16_bytes(scale)
    out[:, 2:34] = q.view(torch.uint8)
    return out.reshape(-1)


def _pack_kquant_scales(sc: torch.Tensor, mn: torch.Tensor) -> torch.Tensor:
    """Pack 8 six-bit scales and 8 six-bit mins into the 12-byte K-quant field
    (inverse of ``gguf_dequant_torch.py:95-111``)."""
    sc = sc.to(torch.int32)
    mn = mn.to(torch.int32)
    out = torch.empty(sc.shape[0], 12, dtype=torch.int32, device=sc.device)
    out[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    out[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    out[:, 8:12] = (sc[:, 4:8] & 15) | ((mn[:, 4:8] & 15) << 4)
    return out.to(torch.uint8)


def _kquant_affine(x: torch.Tensor, qmax: int):
    """Per-32 sub-block affine quantisation shared by Q4_K (qmax 15) and Q5_K (31).

    x: [nb, 8, 32] float32.  Returns (d, dmin, sc6, mn6, q) where the decoded
    value is (d*sc6)*q - dmin*mn6.
    """
    lo = x.amin(dim=2).clamp(max=0.0)
    hi = x.amax(dim=2)
    step = ((hi - lo) / qmax).clamp(min=0.0)
    off = -lo
    d = (step.amax(dim=1) / 63.0)
    dmin = (off.amax(dim=1) / 63.0)
    d16 = d.to(torch.float16).float()
    dmin16 = dmin.to(torch.float16).float()
    sc6 = torch.where(d16[:, None] > 0, torch.round(step / d16[:, None].clamp(min=1e-30)), torch.zeros_like(step)).clamp(0, 63)
    mn6 = torch.where(dmin16[:, None] > 0, torch.round(off / dmin16[:, None].clamp(min=1e-30)), torch.zeros_like(off)).clamp(0, 63)
    s = d16[:, None] * sc6
    m = dmin16[:, None] * mn6
    q = torch.where(s[..., None] > 0, torch.round((x + m[..., None]) / s[..., None].clamp(min=1e-30)), torch.zeros_like(x))
    q = q.clamp(0, qmax).to(torch.int32)
    return d, dmin, sc6, mn6, q


def quantize_q4_k(w: torch.Tensor) -> torch.Tensor:
    x = w.reshape(-1, 8, 32).float()
    nb = x.shape[0]
    d, dmin, sc6, mn6, q = _kquant_affine(x, 15)
    out = torch.empty(nb, 144, dtype=torch.uint8, device=x.device)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:4] = _f16_bytes(dmin)
    out[:, 4:16] = _pack_kquant_scales(sc6, mn6)
    # chunk c: byte c*32+l low nibble = element 64c+l, high nibble = 64c+32+l
    qq = q.reshape(nb, 4, 2, 32)
    out[:, 16:144] = (qq[:, :, 0] | (qq[:, :, 1] << 4)).reshape(nb, 128).to(torch.uint8)
    return out.reshape(-1)


def quantize_q5_k(w: torch.Tensor) -> torch.Tensor:
    x = w.reshape(-1, 8, 32).float()
    nb = x.shape[0]
    d, dmin, sc6, mn6, q = _kquant_affine(x, 31)
    out = torch.empty(nb, 176, dtype=torch.uint8, device=x.device)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:4] = _f16_bytes(dmin)
    out[:, 4:16] = _pack_kquant_scales(sc6, mn6)
    # qh[l] bit j = bit 4 of element 32j+l
    hb = (q >> 4) & 1  # [nb, 8, 32]
    qh = torch.zeros(nb, 32, dtype=torch.int32, device=x.device)
    for j in range(8):
        qh |= hb[:, j] << j
    out[:, 16:48] = qh.to(torch.uint8)
    ql = (q & 15).reshape(nb, 4, 2, 32)
    out[:, 48:176] = (ql[:, :, 0] | (ql[:, :, 1] << 4)).reshape(nb, 128).to(torch.uint8)
    return out.reshape(-1)


def quantize_q6_k(w: torch.Tensor) -> torch.Tensor:
    x = w.reshape(-1, 16, 16).float()
    nb = x.shape[0]
    amax_i = x.abs().argmax(dim=2, keepdim=True)
    vmax = torch.gather(x, 2, amax_i).squeeze(2)           # signed value of largest magnitude
    gscale = -vmax / 32.0                                    # maps vmax to -32 (full range)
    d = gscale.abs().amax(dim=1) / 127.0
    d16 = d.to(torch.float16).float()
    sc = torch.where(d16[:, None] > 0, torch.round(gscale / d16[:, None].clamp(min=1e-30)), torch.zeros_like(gscale)).clamp(-128, 127)
    s = d16[:, None] * sc
    q = torch.where(s[..., None] != 0, torch.round(x / torch.where(s == 0, torch.ones_like(s), s)[..., None]), torch.zeros_like(x))
    u = (q.clamp(-32, 31) + 32).to(torch.int32).reshape(nb, 256)
    out = torch.empty(nb, 210, dtype=torch.uint8, device=x.device)
    # half h (128 elements): groups 4h+0..3 are elements 128h + 32*gi + l
    uu = u.reshape(nb, 2, 4, 32)
    lo4 = uu & 15
    hi2 = uu >> 4
    ql = torch.empty(nb, 2, 64, dtype=torch.int32, device=x.device)
    ql[:, :, 0:32] = lo4[:, :, 0] | (lo4[:, :, 2] << 4)
    ql[:, :, 32:64] = lo4[:, :, 1] | (lo4[:, :, 3] << 4)
    qh = hi2[:, :, 0] | (hi2[:, :, 1] << 2) | (hi2[:, :, 2] << 4) | (hi2[:, :, 3] << 6)
    out[:, 0:128] = ql.reshape(nb, 128).to(torch.uint8)
    out[:, 128:192] = qh.reshape(nb, 64).to(torch.uint8)
    out[:, 192:208] = sc.to(torch.int8).view(torch.uint8)
    out[:, 208:210] = _f16_bytes(d)
    return out.reshape(-1)


_FP4_MAG = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def quantize_mxfp4(w: torch.Tensor, rows: int, cols: int) -> tuple[torch.Tensor, torch.Tensor]:
    """[rows, cols] -> (blocks [rows, cols/32, 16] uint8, scales [rows, cols/32] uint8).

    E8M0 scale = 2^ceil(log2(amax/6)) so every value fits in the e2m1 range;
    each value rounds to the nearest e2m1 magnitude (mxfp4.py:5-8 table)."""
    x = w.reshape(rows, cols // 32, 32).float()
    amax = x.abs().amax(dim=2)
    e = torch.ceil(torch.log2((amax / 6.0).clamp(min=2.0 ** -127)))
    e = e.clamp(-127, 127)
    scale_u8 = (e + 127).to(torch.uint8)
    y = x / torch.exp2(e)[..., None]
    mag = _FP4_MAG.to(x.device)
    idx = (y.abs()[..., None] - mag).abs().argmin(dim=-1)   # nearest magnitude code 0..7
    code = idx | ((y < 0).to(torch.int64) << 3)
    code = torch.where(idx == 0, torch.zeros_like(code), code)  # +0 for zeros
    blocks = (code[..., 0::2] | (code[..., 1::2] << 4)).to(torch.uint8)
    return blocks.contiguous(), scale_u8.contiguous()


def quantize(fmt: int, w: torch.Tensor) -> torch.Tensor:
    """Flat GGUF block stream of ``w`` (any shape) in ``fmt``."""
    if fmt == GGML_Q8_0:
        return quantize_q8_0(w)
    if fmt == GGML_Q4_K:
        return quantize_q4_k(w)
    if fmt == GGML_Q5_K:
        return quantize_q5_k(w)
    if fmt == GGML_Q6_K:
        return quantize_q6_k(w)
    raise ValueError(f"quantize(): use quantize_mxfp4 for MXFP4 (fmt {fmt})" if fmt == TSB_MXFP4
                     else f"Unsupported format {fmt}")
