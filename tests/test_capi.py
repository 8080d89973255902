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


def _packed_bytes_expected(fmt, H, I, E, layout):
    """Host restatement of the decode-packed geometry: gate/up j-groups of 16
    outputs whose gate rows share a Q4_K superblock phase and whose up rows
    share one (MXFP4: phase 0), down groups of 32 rows of one phase; units of
    16 rows x 256 columns (Q4_K 2368 bytes, MXFP4 2176), C chunks per row
    block = ceil((K/32 + max phase) / 8); row maps first, 256-byte aligned."""
    al = lambda v: (v + 255) // 256 * 256  # noqa: E731
    q4 = fmt == 12
    phase = (lambda r, K: (r * K % 256) // 32) if q4 else (lambda r, K: 0)
    gate_row = (lambda j: 2 * j) if layout == _lib.GU_INTERLEAVED else (lambda j: j)
    up_row = {_lib.GU_INTERLEAVED: lambda j: 2 * j + 1, _lib.GU_CHUNKED: lambda j: I + j}.get(layout, lambda j: j)
    keys = {}
    for j in range(I):
        keys.setdefault((phase(gate_row(j), H), phase(up_row(j), H)), []).append(j)
    ngj = sum((len(v) + 15) // 16 for v in keys.values())
    pmax = max(max(k) for k in keys)
    c_gu = (H // 32 + pmax + 7) // 8
    dk = {}
    for h in range(H):
        dk.setdefault(phase(h, I), []).append(h)
    ndp = sum((len(v) + 31) // 32 for v in dk.values())
    c_dn = (I // 32 + max(dk) + 7) // 8
    unit = 2368 if q4 else 2176
    maps = al(al(al(al(4 * 16 * ngj) + 4 * 2 * ngj) + 4 * 32 * ndp) + 4 * ndp)
    expert = al((ngj * c_gu * 2 + ndp * c_dn * 2) * unit)
    return maps + E * expert, expert


def test_packed_bytes_query():
    """tsb_moe_packed_bytes is host arithmetic (see _packed_bytes_expected);
    0 for specs without a packed form."""
    import ctypes
    L = _lib.lib()
    H = I = 2880
    for fmt, layout in ((12, _lib.GU_SEPARATE), (12, _lib.GU_INTERLEAVED), (12, _lib.GU_CHUNKED),
                        (39, _lib.GU_INTERLEAVED)):
        spec = _lib.TsbMoeSpec(fmt, fmt, H, I, 32, 4, layout, _lib.ACT_SWIGLU_OAI, 7.0, 1.702)
        total, expert = _packed_bytes_expected(fmt, H, I, 32, layout)
        assert L.tsb_moe_packed_bytes(ctypes.byref(spec)) == total
        raw = 3 * I * H // 256 * 144 if fmt == 12 else 3 * I * H * 17 // 32
        assert 1.0 <= expert / raw < 1.11  # superblocks straddling rows, chunk and row padding
    # K % 256 == 0: one phase, whole chunks: only the header overhead is left
    spec = _lib.TsbMoeSpec(12, 12, 4096, 2048, 8, 2, _lib.GU_SEPARATE, _lib.ACT_SILU, 7.0, 1.702)
    total, expert = _packed_bytes_expected(12, 4096, 2048, 8, _lib.GU_SEPARATE)
    assert L.tsb_moe_packed_bytes(ctypes.byref(spec)) == total
    assert abs(expert / (3 * 4096 * 2048 // 256 * 144) - 2368 / 2304) < 1e-3
    mixed = _lib.TsbMoeSpec(12, 8, H, I, 32, 4, _lib.GU_SEPARATE, _lib.ACT_SWIGLU_OAI, 7.0, 1.702)
    assert L.tsb_moe_packed_bytes(ctypes.byref(mixed)) == 0
    q8 = _lib.TsbMoeSpec(8, 8, H, I, 32, 4, _lib.GU_SEPARATE, _lib.ACT_SWIGLU_OAI, 7.0, 1.702)
    assert L.tsb_moe_packed_bytes(ctypes.byref(q8)) == 0


def test_packed_entry_points_validate_on_the_host():
    """tsb_moe_pack refuses specs without a packed form and short buffers
    before touching the device; the packed decode workspace holds the generic
    one plus the partial-sum scratch."""
    import ctypes
    L = _lib.lib()
    q6 = _lib.TsbMoeSpec(14, 14, 2880, 2880, 32, 4, _lib.GU_SEPARATE, _lib.ACT_SWIGLU_OAI, 7.0, 1.702)
    buf = ctypes.create_string_buffer(512)
    rc = L.tsb_moe_pack(ctypes.byref(q6), 256, 256, 1 << 20, None)
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


def test_ep_decode_workspace_and_argument_checks():
    """tsb_ep_decode_workspace grows with world * T; tsb_ep_moe_decode rejects
    null pointers and a rank outside the communicator before any GPU work."""
    spec = _lib.TsbMoeSpec(39, 39, 2880, 2880, 16, 4, 0, 1, 7.0, 1.702)
    L = _lib.lib()
    w1 = L.tsb_ep_decode_workspace(ctypes.byref(spec), 1, 2, 0)
    w8 = L.tsb_ep_decode_workspace(ctypes.byref(spec), 1, 8, 0)
    assert 0 < w1 < w8
    assert L.tsb_ep_decode_workspace(ctypes.byref(spec), 0, 2, 0) == 0
    assert L.tsb_ep_decode_workspace(ctypes.byref(spec), 1, 0, 0) == 0
    rc = L.tsb_ep_moe_decode(ctypes.byref(spec), None, None, 16, 1, 16, 16, 16, 16, 0, 2, 256, w1, None)
    assert rc == _lib.TSB_ERR_INVALID
    rc = L.tsb_ep_moe_decode(ctypes.byref(spec), 16, None, 16, 1, 16, 16, 16, 16, 2, 2, 256, w1, None)
    assert rc == _lib.TSB_ERR_INVALID and "rank" in _lib.last_error()
