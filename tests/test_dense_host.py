"""Host-side checks of the dense expert formats in the C-ABI: format ids,
byte counts and spec validation (no kernel runs)."""
from __future__ import annotations

import ctypes

from tinyserve_b200 import _lib
from tinyserve_b200.formats import GGML_BF16, GGML_F16, GGML_F32, GGML_Q4_K


def _spec(fg, fd, transposed=0):
    return _lib.TsbMoeSpec(fg, fd, 256, 256, 4, 2, _lib.GU_SEPARATE, _lib.ACT_SILU, 7.0, 1.702, 0, transposed)


def test_dense_format_info_and_bytes():
    L = _lib.lib()
    for fmt, es in ((GGML_F32, 4), (GGML_F16, 2), (GGML_BF16, 2)):
        be, bb = ctypes.c_int32(), ctypes.c_int32()
        assert L.tsb_format_info(fmt, ctypes.byref(be), ctypes.byref(bb)) == 0
        assert (be.value, bb.value) == (1, es)
        d, s = ctypes.c_int64(), ctypes.c_int64()
        assert L.tsb_weight_bytes(fmt, 2880, 5760, ctypes.byref(d), ctypes.byref(s)) == 0
        assert (d.value, s.value) == (2880 * 5760 * es, 0)


def test_dense_spec_validation_before_any_launch():
    L = _lib.lib()
    dummy = ctypes.c_void_p(256)  # never dereferenced: validation fails first
    for spec, code, text in (
        (_spec(GGML_BF16, GGML_Q4_K), _lib.TSB_ERR_UNSUPPORTED, "both be dense"),
        (_spec(GGML_Q4_K, GGML_Q4_K, _lib.T_DOWN), _lib.TSB_ERR_INVALID, "dense formats only"),
        (_spec(GGML_BF16, GGML_BF16, 4), _lib.TSB_ERR_INVALID, "transposed bits"),
    ):
        rc = L.tsb_moe_decode(ctypes.byref(spec), dummy, dummy, 1, None, None, dummy, dummy, dummy, dummy, 1 << 30,
                              None)
        assert rc == code
        assert text in _lib.last_error()
    # the quantised matvec keeps the reference's format set and message
    rc = L.tsb_quant_matvec(GGML_BF16, dummy, None, 16, 32, dummy, 1, 1, 32, dummy, 1, 16, None, None)
    assert rc == _lib.TSB_ERR_UNSUPPORTED and "Unsupported ggml_type" in _lib.last_error()
