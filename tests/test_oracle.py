"""The CPU oracle against the reference's own outputs (golden fixtures made by
tests/golden/make_golden.py) and against the reference tests' known answers.
No GPU needed."""
from __future__ import annotations

import struct

import numpy as np
import pytest
import torch

from oracle import dequant as OD
from oracle import expert as OE
from tests.helpers import bits_equal_f32, oracle_dequant, rel_l2
from tinyserve_b200 import quantize as Q
from tinyserve_b200.formats import GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_Q8_0, TSB_MXFP4


@pytest.mark.parametrize("fmt", [GGML_Q8_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K])
@pytest.mark.parametrize("case", ["valid", "random", "enc_4x2880"])
def test_gguf_dequant_matches_reference(golden, fmt, case):
    g = golden["dequant_gguf"]
    raw, ref, shape = g[f"{fmt}_{case}_in"], g[f"{fmt}_{case}_out"], tuple(g[f"{fmt}_{case}_shape"])
    assert bits_equal_f32(OD.dequant_tensor(raw, fmt, shape), ref)


@pytest.mark.parametrize("case", ["kat_scales", "full_scales"])
def test_mxfp4_dequant_matches_reference(golden, case):
    m = golden["dequant_mxfp4"]
    b, s = m[f"{case}_blocks"], m[f"{case}_scales"]
    assert (OD.dequant_mxfp4_no_transpose(b, s, "bf16") == m[f"{case}_bf16"]).all()
    assert bits_equal_f32(OD.dequant_mxfp4_no_transpose(b, s, "f32"), m[f"{case}_f32"])


def test_mxfp4_known_answers():
    """tinyserve tests/test_mxfp4.py:8-61: 0x21 -> [0.5, 1.0], 0x43 -> [1.5, 2.0];
    scale 128 doubles; 0x0A -> -1.0."""
    blk = np.zeros((1, 1, 16), np.uint8)
    blk[0, 0, :2] = [0x21, 0x43]
    out = OD.dequant_mxfp4_no_transpose(blk, np.array([[127]], np.uint8), "f32")[0]
    assert list(out[:4]) == [0.5, 1.0, 1.5, 2.0]
    blk[0, 0, :2] = [0x02, 0]
    assert OD.dequant_mxfp4_no_transpose(blk, np.array([[128]], np.uint8), "f32")[0, 0] == 2.0
    blk[0, 0, 0] = 0x0A
    assert OD.dequant_mxfp4_no_transpose(blk, np.array([[127]], np.uint8), "f32")[0, 0] == -1.0


def test_q8_0_known_answers():
    """tinyserve tests/test_gguf_dequant_torch.py:126-170."""
    q = np.arange(1, 33, dtype=np.int8)
    blk = struct.pack("<e", np.float16(2.0)) + q.tobytes()
    np.testing.assert_array_equal(OD.dequant_tensor(blk, GGML_Q8_0, (32,)), q.astype(np.float32) * 2.0)
    q = np.array([-16, -8, 0, 8, 16] + [0] * 27, dtype=np.int8)
    blk = struct.pack("<e", np.float16(0.5)) + q.tobytes()
    np.testing.assert_array_equal(OD.dequant_tensor(blk, GGML_Q8_0, (32,)), q.astype(np.float32) * 0.5)


def test_unsupported_type_raises():
    with pytest.raises(ValueError, match="Unsupported"):
        OD.dequant_tensor(b"\0" * 32, 99, (32,))


@pytest.mark.parametrize("fmt,tol", [(GGML_Q8_0, 0.01), (GGML_Q4_K, 0.12), (GGML_Q5_K, 0.06),
                                     (GGML_Q6_K, 0.04), (TSB_MXFP4, 0.2)])
def test_encoder_round_trip(fmt, tol):
    """The repo's encoders write byte layouts the reference decoders read:
    encode -> oracle decode reproduces N(0, 0.02) weights within the format's
    round-to-nearest error."""
    rows, cols = 8, 2880
    w = torch.randn(rows, cols, generator=torch.Generator().manual_seed(3)) * 0.02
    if fmt == TSB_MXFP4:
        b, s = Q.quantize_mxfp4(w, rows, cols)
        deq = oracle_dequant(fmt, b.reshape(-1), s.reshape(-1), rows, cols)
    else:
        deq = oracle_dequant(fmt, Q.quantize(fmt, w), None, rows, cols)
    assert rel_l2(deq, w.numpy()) < tol


def test_q8_0_encoder_matches_reference_semantics():
    """quantize_q8_0 follows mmap_store.quantize_to_q8_0 (mmap_store.py:280-306)."""
    w = torch.randn(4, 64, generator=torch.Generator().manual_seed(9))
    b = Q.quantize_q8_0(w).numpy().reshape(-1, 34)
    x = w.reshape(-1, 32)
    scale = (x.abs().amax(1) / 127.0).clamp(min=1e-10)
    np.testing.assert_array_equal(b[:, 0:2].copy().view(np.float16)[:, 0], scale.to(torch.float16).numpy())
    np.testing.assert_array_equal(b[:, 2:].view(np.int8), torch.round(x / scale[:, None]).clamp(-128, 127).numpy())


def test_expert_math_matches_reference(golden):
    x = golden["expert"]
    o = OE.expert_forward(x["h"], x["w_gate"], x["w_up"], x["w_down"], "swiglu_oai")
    assert rel_l2(o, x["out_swiglu"]) < 1e-6
    o = OE.expert_forward(x["h"], x["w_gate2"], x["w_up2"], x["w_down2"], "silu")
    assert rel_l2(o, x["out_silu"]) < 1e-6


def test_gguf_expert_fallback_matches_reference(golden):
    """GGMLExpertForward._fallback_forward (ggml_forward.py:117-151, SiLU, fp32)."""
    x = golden["expert"]
    H, I = (int(v) for v in x["gguf_dims"])
    p = x["gguf_packed"]
    ng = I * H // 256 * 144
    nd = H * I // 32 * 34
    wg = OD.dequant_tensor(p[:ng], GGML_Q4_K, (I, H))
    wu = OD.dequant_tensor(p[ng:2 * ng], GGML_Q4_K, (I, H))
    wd = OD.dequant_tensor(p[2 * ng:2 * ng + nd], GGML_Q8_0, (H, I))
    o = OE.expert_forward(x["gguf_h"], wg, wu, wd, "silu")
    assert rel_l2(o, x["gguf_out"]) < 1e-6


def test_router_matches_reference(golden):
    """topk-then-softmax routing (_model_hooks.py:466-473).  The reference
    returns bf16 weights; ids agree except where bf16 logits tie."""
    x = golden["expert"]
    h = OD.bf16_bits_to_f32(x["router_h"])
    w = OD.bf16_bits_to_f32(x["router_w"])
    ids, wts, lg = OE.router_topk_softmax(h, w, 4)
    for t in range(ids.shape[0]):
        ref = x["router_ids"][t]
        if set(ids[t]) != set(ref):
            # only acceptable at an exact tie of the 4th and 5th logits
            srt = np.sort(lg[t])[::-1]
            assert srt[3] == srt[4]
        np.testing.assert_allclose(np.sort(wts[t]), np.sort(x["router_wts"][t]), rtol=8e-3, atol=2e-3)
