"""GPU parity of the C-ABI kernels against the oracle (and the reference's own
golden outputs).  Tolerances:
  dequant         bit-exact (NaN compared as NaN for fp32 output)
  matvec / layer  relative L2 <= 1e-3 against float64 math on the dequantised
                  weights for fp32 outputs; bf16
                  layer outputs may add their own rounding on top of the 1e-3
                  (tests.helpers.layer_bound)
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import dequant as OD
from oracle import expert as OE
from tests.helpers import assert_layer, ALL_FMTS, FMT_NAMES, bits_equal_f32, make_weight, oracle_dequant, rel_l2
from tinyserve_b200 import ops
from tinyserve_b200.formats import GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_Q8_0, TSB_MXFP4

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    return torch.device("cuda:0")


# ------------------------------------------------------------------ dequant
@pytest.mark.parametrize("fmt", [GGML_Q8_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K])
@pytest.mark.parametrize("case", ["valid", "random", "enc_4x2880"])
def test_dequant_gguf_bit_exact_golden(dev, golden, fmt, case):
    g = golden["dequant_gguf"]
    raw, ref, shape = g[f"{fmt}_{case}_in"], g[f"{fmt}_{case}_out"], tuple(g[f"{fmt}_{case}_shape"])
    rows, cols = (1, shape[0]) if len(shape) == 1 else shape
    w = torch.from_numpy(raw.copy()).to(dev)
    out = ops.dequant(fmt, w, None, rows, cols, torch.float32).cpu().numpy().reshape(ref.shape)
    assert bits_equal_f32(out, ref)


@pytest.mark.parametrize("case", ["kat_scales", "full_scales"])
def test_dequant_mxfp4_bit_exact_golden(dev, golden, case):
    m = golden["dequant_mxfp4"]
    b = torch.from_numpy(m[f"{case}_blocks"].copy()).to(dev)
    s = torch.from_numpy(m[f"{case}_scales"].copy()).to(dev)
    rows, cols = b.shape[0], b.shape[1] * 32
    o32 = ops.dequant(TSB_MXFP4, b, s, rows, cols, torch.float32).cpu().numpy()
    assert bits_equal_f32(o32, m[f"{case}_f32"])
    o16 = ops.dequant(TSB_MXFP4, b, s, rows, cols, torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16)
    assert (o16 == m[f"{case}_bf16"]).all()


@pytest.mark.parametrize("fmt", ALL_FMTS, ids=FMT_NAMES.get)
def test_dequant_bit_exact_encoded(dev, fmt):
    rows, cols = 12, 2880
    d, s = make_weight(fmt, rows, cols, seed=11)
    out = ops.dequant(fmt, d.to(dev), None if s is None else s.to(dev), rows, cols).cpu().numpy()
    assert bits_equal_f32(out, oracle_dequant(fmt, d, s, rows, cols))


# ------------------------------------------------------------------ matvec
def _matvec_case(dev, fmt, N, K, M, seed, xdtype=torch.bfloat16):
    d, s = make_weight(fmt, N, K, seed=seed)
    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(M, K, generator=g).to(xdtype)
    y = ops.quant_matvec(fmt, d.to(dev), None if s is None else s.to(dev), N, K, x.to(dev),
                         out_dtype=torch.float32)
    ref = x.double().numpy() @ oracle_dequant(fmt, d, s, N, K).astype(np.float64).T
    return y.cpu().numpy(), ref


@pytest.mark.parametrize("fmt", ALL_FMTS, ids=FMT_NAMES.get)
@pytest.mark.parametrize("N,K", [(2880, 2880), (5760, 2880), (64, 256), (37, 512), (300, 4096)])
def test_matvec_batch1(dev, fmt, N, K):
    y, ref = _matvec_case(dev, fmt, N, K, 1, seed=N + K)
    assert rel_l2(y, ref) <= TOL


@pytest.mark.parametrize("fmt", ALL_FMTS, ids=FMT_NAMES.get)
def test_matvec_long_rows_chunked(dev, fmt):
    """K = 14336 does not fit one stage: exercises the per-row k-chunk path."""
    y, ref = _matvec_case(dev, fmt, 96, 14336, 1, seed=5)
    assert rel_l2(y, ref) <= TOL


@pytest.mark.parametrize("fmt", ALL_FMTS, ids=FMT_NAMES.get)
@pytest.mark.parametrize("N,K", [(4096, 14336), (14336, 4096)])
def test_matvec_sweep_full_shapes(dev, fmt, N, K):
    """The two large BASELINE config-2 sweep shapes, whole matrices."""
    y, ref = _matvec_case(dev, fmt, N, K, 1, seed=N // 7 + K)
    assert rel_l2(y, ref) <= TOL


@pytest.mark.parametrize("fmt", ALL_FMTS, ids=FMT_NAMES.get)
@pytest.mark.parametrize("M", [2, 5, 8, 11])
def test_matvec_multi_vector(dev, fmt, M):
    y, ref = _matvec_case(dev, fmt, 200, 2880, M, seed=M)
    for i in range(M):
        assert rel_l2(y[i], ref[i]) <= TOL


@pytest.mark.parametrize("fmt", [GGML_Q8_0, GGML_Q4_K])
def test_matvec_fp32_activations(dev, fmt):
    y, ref = _matvec_case(dev, fmt, 128, 2880, 1, seed=7, xdtype=torch.float32)
    assert rel_l2(y, ref) <= TOL


def test_matvec_wide_dynamic_range(dev):
    """Per-block power-of-two scaling keeps activations far outside the f16
    range exact (values up to 1e30 and down to 1e-30)."""
    N, K = 64, 1024
    d, _ = make_weight(GGML_Q8_0, N, K, seed=2)
    x = torch.randn(1, K, generator=torch.Generator().manual_seed(3))
    x[0, :256] *= 1e30
    x[0, 256:512] *= 1e-30
    y = ops.quant_matvec(GGML_Q8_0, d.to(dev), None, N, K, x.to(dev), out_dtype=torch.float32).cpu().numpy()
    ref = x.double().numpy() @ oracle_dequant(GGML_Q8_0, d, None, N, K).astype(np.float64).T
    assert rel_l2(y, ref) <= TOL


def test_matvec_empty(dev):
    d, _ = make_weight(GGML_Q8_0, 16, 64, seed=1)
    y = ops.quant_matvec(GGML_Q8_0, d.to(dev), None, 0, 64, torch.zeros(1, 64, device=dev))
    assert y.shape == (1, 0)


# ------------------------------------------------------------------ ggml_mul_mat_vec drop-in
def test_ggml_op_registered_and_matches(dev):
    ops.register_torch_op()
    K, N = 512, 64
    d, _ = make_weight(GGML_Q4_K, N, K, seed=4)
    act = torch.randn(1, K, dtype=torch.bfloat16, device=dev)
    out = torch.ops.tinyserve_ggml.ggml_mul_mat_vec(act, d.to(dev), GGML_Q4_K, N, K)
    assert out.shape == (1, N) and out.dtype == torch.bfloat16
    ref = act.double().cpu().numpy() @ oracle_dequant(GGML_Q4_K, d, None, N, K).astype(np.float64).T
    assert rel_l2(out.float().cpu().numpy(), ref) <= 5e-3  # bf16 output rounding
    act32 = act.float()
    out32 = torch.ops.tinyserve_ggml.ggml_mul_mat_vec(act32, d.to(dev), GGML_Q4_K, N, K)
    assert out32.dtype == torch.float32 and rel_l2(out32.cpu().numpy(), ref) <= TOL


def test_ggml_op_errors(dev):
    act = torch.randn(1, 32, device=dev)
    with pytest.raises(RuntimeError, match="Unsupported ggml_type"):
        ops.ggml_mul_mat_vec(act, torch.zeros(100, dtype=torch.uint8, device=dev), 99, 10, 32)
    with pytest.raises(RuntimeError, match="weight_data too small"):
        ops.ggml_mul_mat_vec(act, torch.zeros(10, dtype=torch.uint8, device=dev), GGML_Q8_0, 10, 32)


# ------------------------------------------------------------------ fused MoE decode layer
def _build_layer(dev, fmt_gu, fmt_dn, H, I, E, k, layout, seed, bias=False, pack=None, activation="swiglu_oai"):
    from tinyserve_b200.moe import ExpertWeights, QuantMoE
    experts, dense = [], []
    for e in range(E):
        s0 = seed * 1000 + 10 * e
        if layout == "separate":
            g, gs = make_weight(fmt_gu, I, H, s0)
            u, us = make_weight(fmt_gu, I, H, s0 + 1)
            wg, wu = oracle_dequant(fmt_gu, g, gs, I, H), oracle_dequant(fmt_gu, u, us, I, H)
        else:
            g, gs = make_weight(fmt_gu, 2 * I, H, s0)
            u = us = None
            wgu = oracle_dequant(fmt_gu, g, gs, 2 * I, H)
            wg, wu = (wgu[0::2], wgu[1::2]) if layout == "interleaved" else (wgu[:I], wgu[I:])
        dn, ds = make_weight(fmt_dn, H, I, s0 + 2)
        wd = oracle_dequant(fmt_dn, dn, ds, H, I)
        to = lambda t: None if t is None else t.to(dev)  # noqa: E731
        bg = bu = bd = None
        if bias:
            gen = torch.Generator().manual_seed(s0 + 3)
            bg, bu, bd = (torch.randn(n, generator=gen) * 0.1 for n in (I, I, H))
        experts.append(ExpertWeights(gate=to(g), up=to(u), down=to(dn), gate_scales=to(gs), up_scales=to(us),
                                     down_scales=to(ds), gate_bias=to(bg), up_bias=to(bu), down_bias=to(bd)))
        dense.append((wg, wu, wd, bg, bu, bd))
    gen = torch.Generator().manual_seed(seed)
    router = (torch.randn(E, H, generator=gen) * 0.02).to(torch.bfloat16)
    layer = QuantMoE(experts, fmt_gate_up=fmt_gu, fmt_down=fmt_dn, hidden=H, inter=I, top_k=k,
                     router_w=router.to(dev), gate_up_layout=layout, activation=activation, pack=pack)
    return layer, dense, router


def _oracle_layer(x, ids, wts, dense, act="swiglu_oai"):
    out = np.zeros(x.shape[1])
    for e, w in zip(ids, wts):
        wg, wu, wd, bg, bu, bd = dense[e]
        out += w * OE.expert_forward(x, wg, wu, wd, act,
                                     None if bg is None else bg.numpy(), None if bu is None else bu.numpy(),
                                     None if bd is None else bd.numpy())[0]
    return out


@pytest.mark.parametrize("fmt_gu,fmt_dn,layout", [
    (GGML_Q4_K, GGML_Q4_K, "separate"),      # BASELINE config 1 (GGUF Q4_K, clamp-SwiGLU)
    (TSB_MXFP4, TSB_MXFP4, "interleaved"),   # GPT-OSS MXFP4 experts
    (GGML_Q8_0, GGML_Q6_K, "separate"),
    (GGML_Q5_K, GGML_Q8_0, "chunked"),
])
def test_moe_decode_layer(dev, fmt_gu, fmt_dn, layout):
    H = I = 2880
    E, k = 8, 4
    layer, dense, router = _build_layer(dev, fmt_gu, fmt_dn, H, I, E, k, layout, seed=fmt_gu + fmt_dn)
    for step in range(3):
        x = torch.randn(1, H, generator=torch.Generator().manual_seed(100 + step)).to(torch.bfloat16)
        out, ids, wts = layer.decode(x.to(dev))
        torch.cuda.synchronize()
        ids_o, wts_o, lg = OE.router_topk_softmax(x.float().numpy(), router.float().numpy(), k)
        ids_g = ids.cpu().numpy()[0]
        if set(ids_g) != set(ids_o[0]):
            srt = np.sort(lg[0])[::-1]
            assert abs(srt[k - 1] - srt[k]) <= 1e-2 * abs(srt[k - 1]) + 1e-6, "routing differs away from a tie"
        ref = _oracle_layer(x.float().numpy(), ids_g, wts.cpu().numpy()[0], dense)
        np.testing.assert_allclose(np.sort(wts.cpu().numpy()[0])[::-1], np.sort(wts_o[0])[::-1], rtol=1e-5, atol=1e-6)
        # bf16 output: its rounding on top of the 1e-3; fp32 output: 1e-3
        assert_layer(out[0], ref)
        out32, ids32, _ = layer.decode(x.to(dev), out_dtype=torch.float32)
        assert torch.equal(ids32, ids)
        assert_layer(out32[0], ref)
        assert layer.device_error() == 0


def test_moe_decode_given_ids_and_bias(dev):
    H, I, E, k = 1024, 512, 6, 2
    layer, dense, _ = _build_layer(dev, GGML_Q4_K, GGML_Q8_0, H, I, E, k, "separate", seed=77, bias=True)
    x = torch.randn(1, H, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    ids = torch.tensor([[5, 2]], dtype=torch.int32)
    wts = torch.tensor([[0.7, 0.3]])
    out, _, _ = layer.decode(x.to(dev), ids=ids.to(dev), weights=wts.to(dev))
    ref = _oracle_layer(x.float().numpy(), [5, 2], [0.7, 0.3], dense)
    assert_layer(out[0], ref)


def test_moe_decode_top8(dev):
    H, I, E, k = 512, 256, 16, 8
    layer, dense, router = _build_layer(dev, TSB_MXFP4, TSB_MXFP4, H, I, E, k, "interleaved", seed=3)
    x = torch.randn(1, H, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    out, ids, wts = layer.decode(x.to(dev))
    ref = _oracle_layer(x.float().numpy(), ids.cpu().numpy()[0], wts.cpu().numpy()[0], dense)
    assert_layer(out[0], ref)


def test_router_nan_input_gives_valid_ids(dev):
    """NaN logits sort lowest; the router still returns in-range ids."""
    H, I, E, k = 512, 256, 8, 4
    layer, _, _ = _build_layer(dev, GGML_Q8_0, GGML_Q8_0, H, I, E, k, "separate", seed=5)
    x = torch.full((1, H), float("nan"), dtype=torch.bfloat16, device=dev)
    _, ids, _ = layer.decode(x)
    torch.cuda.synchronize()
    got = ids.cpu().numpy()[0]
    assert ((got >= 0) & (got < E)).all() and len(set(got)) == k
    assert layer.device_error() == 0


def test_bad_expert_ids_are_reported_not_dereferenced(dev):
    """Caller-provided ids outside [0, E) set the device error word (2) and
    contribute nothing; valid ids still contribute."""
    H, I, E, k = 512, 256, 4, 2
    layer, dense, _ = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, E, k, "separate", seed=6)
    x = torch.randn(1, H, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    out, _, _ = layer.decode(x.to(dev), ids=torch.tensor([[1, 1000]], device=dev),
                             weights=torch.tensor([[0.5, 0.5]], device=dev))
    torch.cuda.synchronize()
    assert layer.device_error() == 2
    ref = _oracle_layer(x.float().numpy(), [1], [0.5], dense)
    assert_layer(out[0], ref)
    assert layer.device_error() == 0
