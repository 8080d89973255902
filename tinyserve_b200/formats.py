"""Weight-format table shared by the host code and the C-ABI.

GGUF type ids and block sizes follow ``tinyserve/gguf_reader.py:15-29``
(``GGML_TYPES``) and ``tinyserve/gguf_dequant_torch.py:20-29``.  MXFP4 has no
ggml id in the reference (it arrives as HF ``*_blocks`` / ``*_scales``
tensors, ``tinyserve/mxfp4.py:20-44``); it gets the private id ``TSB_MXFP4``.
The numeric values are mirrored in ``include/tsb_moe.h``.
"""
from __future__ import annotations

GGML_Q8_0 = 8
GGML_Q4_K = 12
GGML_Q5_K = 13
GGML_Q6_K = 14
TSB_MXFP4 = 39
# dense expert formats (GGUF ids of the float types, gguf_reader.py:15-29)
GGML_F32 = 0
GGML_F16 = 1
GGML_BF16 = 30
DENSE = {GGML_F32: 4, GGML_F16: 2, GGML_BF16: 2}  # id -> bytes per element

# id -> (name, block_bytes, block_elements)
FORMATS: dict[int, tuple[str, int, int]] = {
    GGML_Q8_0: ("Q8_0", 34, 32),
    GGML_Q4_K: ("Q4_K", 144, 256),
    GGML_Q5_K: ("Q5_K", 176, 256),
    GGML_Q6_K: ("Q6_K", 210, 256),
    TSB_MXFP4: ("MXFP4", 17, 32),  # 16 B of nibbles + 1 E8M0 scale byte (separate tensors)
}

NAME_TO_ID = {v[0]: k for k, v in FORMATS.items()}


def weight_bytes(fmt: int, rows: int, cols: int) -> int:
    """Bytes of a [rows, cols] weight in ``fmt`` (flat block stream).

    For GGUF types this is ``rows*cols/block_elements * block_bytes`` exactly
    as ``ggml_forward.py:97-99`` computes it; for MXFP4 it is blocks + scales.
    """
    name, bb, be = FORMATS[fmt]
    n = rows * cols
    if n % be:
        raise ValueError(f"{name}: rows*cols={n} is not a multiple of {be}")
    return n // be * bb


def mxfp4_split(rows: int, cols: int) -> tuple[int, int]:
    """(bytes of the nibble blocks, bytes of the E8M0 scales) of an MXFP4 weight."""
    return rows * cols // 2, rows * cols // 32
