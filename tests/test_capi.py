"""The C-ABI library loads and exports every symbol include/tsb_moe.h declares;
argument checking and error reporting work without a GPU (no kernel runs)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from tinyserve_b200 import _lib
from tinyserve_b200.formats import FORMATS, GGML_Q4_K, TSB_MXFP4

HEADER = Path(__file__).resolve().parents[1] / "include" / "tsb_moe.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(tsb_\w+)\s*\(", text, re.M))


def test_header_declares_what_python_binds():
    assert declared_symbols() == set(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name


def test_version_and_format_table():
    L = _lib.lib()
    assert L.tsb_version() >= 100
    for fmt, (_, bb, be) in FORMATS.items():
        e, b = ctypes.c_int32(), ctypes.c_int32()
        _lib.check(L.tsb_format_info(fmt, ctypes.byref(e), ctypes.byref(b)))
        assert (e.value, b.value) == (be, bb)


def test_weight_bytes():
    L = _lib.lib()
    d, s = ctypes.c_int64(), ctypes.c_int64()
    _lib.check(L.tsb_weight_bytes(GGML_Q4_K, 2880, 2880, ctypes.byref(d), ctypes.byref(s)))
    assert (d.value, s.value) == (4665600, 0)
    _lib.check(L.tsb_weight_bytes(TSB_MXFP4, 5760, 2880, ctypes.byref(d), ctypes.byref(s)))
    assert (d.value, s.value) == (8294400, 518400)


def test_unsupported_type_message():
    """Same wording as the reference op (ggml_ops.cu:473-476; its test matches
    'Unsupported ggml_type')."""
    L = _lib.lib()
    rc = L.tsb_quant_matvec(99, None, None, 10, 32, None, 0, 1, 32, None, 0, 10, None, None)
    assert rc == _lib.TSB_ERR_UNSUPPORTED
    assert "Unsupported ggml_type" in _lib.last_error()
    with pytest.raises(RuntimeError, match="Unsupported ggml_type"):
        _lib.check(rc)


def test_bad_shapes_rejected_before_launch():
    L = _lib.lib()
    assert L.tsb_quant_matvec(GGML_Q4_K, None, None, 3, 40, None, 0, 1, 40, None, 0, 3, None, None) == _lib.TSB_ERR_INVALID
    assert L.tsb_quant_matvec(GGML_Q4_K, None, None, 3, 32, None, 0, 1, 32, None, 0, 3, None, None) == _lib.TSB_ERR_INVALID
    # misaligned weight pointer
    assert L.tsb_quant_matvec(GGML_Q4_K, 8, None, 16, 256, 64, 0, 1, 256, 128, 0, 16, None, None) == _lib.TSB_ERR_INVALID
    assert "aligned" in _lib.last_error()


def test_moe_decode_argument_checks():
    L = _lib.lib()
    spec = _lib.TsbMoeSpec(GGML_Q4_K, GGML_Q4_K, 2880, 2880, 32, 4, 0, 1, 7.0, 1.702)
    ws = L.tsb_moe_decode_workspace(ctypes.byref(spec), 1)
    assert ws >= 4 * 2880 * 4
    bad = _lib.TsbMoeSpec(GGML_Q4_K, GGML_Q4_K, 2880, 2880, 32, 9, 0, 1, 7.0, 1.702)
    rc = L.tsb_moe_decode(ctypes.byref(bad), 16, 16, 1, None, None, 16, 16, 16, 256, 1 << 20, None)
    assert rc == _lib.TSB_ERR_INVALID and "top_k" in _lib.last_error()
    rc = L.tsb_moe_decode(ctypes.byref(spec), 16, 16, 1, None, None, 16, 16, 16, 256, 16, None)
    assert rc == _lib.TSB_ERR_WORKSPACE


def test_packed_bytes_query():
    """tsb_moe_packed_bytes is host arithmetic: 768 bytes per (16 rows, 64
    columns) unit for gate/up (8 outputs x 2 rows per block) and down, padded
    to 256 bytes per expert; 0 for specs without a packed form."""
    import ctypes
    L = _lib.lib()
    H = I = 2880
    spec = _lib.TsbMoeSpec(12, 12, H, I, 32, 4, _lib.GU_SEPARATE, _lib.ACT_SWIGLU_OAI, 7.0, 1.702)
    per = (I // 8) * (H // 64) * 768 + (H // 16) * (I // 64) * 768
    per = (per + 255) // 256 * 256
    assert L.tsb_moe_packed_bytes(ctypes.byref(spec)) == 32 * per
    q4k = 3 * I * H // 256 * 144
    assert abs(per / q4k - 4 / 3) < 0.01
    mx = _lib.TsbMoeSpec(39, 39, H, I, 32, 4, _lib.GU_INTERLEAVED, _lib.ACT_SWIGLU_OAI, 7.0, 1.702)
    assert L.tsb_moe_packed_bytes(ctypes.byref(mx)) == 0
    odd = _lib.TsbMoeSpec(12, 12, 2880, 2880 + 32, 32, 4, _lib.GU_SEPARATE, _lib.ACT_SWIGLU_OAI, 7.0, 1.702)
    assert L.tsb_moe_packed_bytes(ctypes.byref(odd)) == 0


def test_packed_entry_points_validate_on_the_host():
    """tsb_moe_pack refuses specs without a packed form and short buffers
    before touching the device; the packed decode workspace holds the generic
    one plus the partial-sum scratch."""
    import ctypes
    L = _lib.lib()
    mx = _lib.TsbMoeSpec(39, 39, 2880, 2880, 32, 4, _lib.GU_INTERLEAVED, _lib.ACT_SWIGLU_OAI, 7.0, 1.702)
    buf = ctypes.create_string_buffer(512)
    rc = L.tsb_moe_pack(ctypes.byref(mx), 256, 256, 1 << 20, None)
    assert rc != 0
    L.tsb_last_error(buf, 512)
    assert b"no packed form" in buf.value
    q4 = _lib.TsbMoeSpec(12, 12, 2880, 2880, 32, 4, _lib.GU_SEPARATE, _lib.ACT_SWIGLU_OAI, 7.0, 1.702)
    need = L.tsb_moe_packed_bytes(ctypes.byref(q4))
    rc = L.tsb_moe_pack(ctypes.byref(q4), 256, 256, need - 1, None)
    assert rc != 0
    L.tsb_last_error(buf, 512)
    assert b"too small" in buf.value
    assert L.tsb_moe_decode_packed_workspace(ctypes.byref(q4), 1) > L.tsb_moe_decode_workspace(ctypes.byref(q4), 1)
    # T > 16 takes the grouped path: same workspace as tsb_moe_decode
    assert L.tsb_moe_decode_packed_workspace(ctypes.byref(q4), 64) == L.tsb_moe_decode_workspace(ctypes.byref(q4), 64)
