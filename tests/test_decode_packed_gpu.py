"""GPU parity of batch-1 decode on the decode-packed experts (tsb_moe_pack /
tsb_moe_decode_packed; Q4_K on the int8 tensor path, MXFP4 on the f16 path)
against the oracle layer (float64 math on the reference-dequantised weights)
and against the generic decode engine.

Tolerance (north star): relative L2 <= 1e-3 for fp32 outputs; bf16 outputs
may add their own rounding, rel_l2(bf16(ref), ref), on top of the 1e-3
(tests.helpers.layer_bound)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import expert as OE
from tests.helpers import assert_layer, layer_bound, rel_l2
from tests.test_kernels_gpu import _build_layer, _oracle_layer
from tinyserve_b200.formats import GGML_Q4_K, TSB_MXFP4

pytestmark = pytest.mark.gpu
FMTS = [(GGML_Q4_K, "separate"), (TSB_MXFP4, "interleaved")]
IDS = ["Q4_K", "MXFP4"]


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    return torch.device("cuda:0")


def _x(H, seed, scale=1.0):
    return (torch.randn(1, H, generator=torch.Generator().manual_seed(seed)) * scale).to(torch.bfloat16)


def _ref_w(x, router, k):
    return OE.router_topk_softmax(x.float().numpy(), router.float().numpy(), k)[1][0]


def _check_routing(x, router, k, ids, wts):
    """The in-kernel routing picks the oracle's experts (unless two logits tie
    after bf16 rounding) with the same softmax weights."""
    ids_o, _, lg = OE.router_topk_softmax(x.float().numpy(), router.float().numpy(), k)
    if set(ids.cpu().numpy()[0]) != set(ids_o[0]):
        srt = np.sort(lg[0])[::-1]
        assert abs(srt[k - 1] - srt[k]) <= 1e-2 * abs(srt[k - 1]) + 1e-6, "routing differs away from a tie"
    else:
        np.testing.assert_allclose(np.sort(wts.cpu().numpy()[0])[::-1], np.sort(_ref_w(x, router, k))[::-1],
                                   rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("fmt,layout", FMTS + [(GGML_Q4_K, "interleaved"), (GGML_Q4_K, "chunked")],
                         ids=IDS + ["Q4_K-interleaved", "Q4_K-chunked"])
def test_packed_layer_matches_oracle_and_engine(dev, fmt, layout):
    """GPT-OSS-20B shape (H = I = 2880: Q4_K rows start mid-superblock; for the
    interleaved layout gate and up rows of one output have different phases)."""
    H = I = 2880
    E, k = 8, 4
    packed, dense, router = _build_layer(dev, fmt, fmt, H, I, E, k, layout, seed=11)
    generic, _, _ = _build_layer(dev, fmt, fmt, H, I, E, k, layout, seed=11, pack=False)
    assert packed.packed and not generic.packed
    for step in range(3):
        x = _x(H, 200 + step)
        out, ids, wts = packed.decode(x.to(dev), out_dtype=torch.float32)
        out_g, ids_g, w_g = generic.decode(x.to(dev), out_dtype=torch.float32)
        torch.cuda.synchronize()
        _check_routing(x, router, k, ids, wts)
        ref = _oracle_layer(x.float().numpy(), ids.cpu().numpy()[0], wts.cpu().numpy()[0], dense)
        assert_layer(out[0], ref)
        ref_g = _oracle_layer(x.float().numpy(), ids_g.cpu().numpy()[0], w_g.cpu().numpy()[0], dense)
        assert_layer(out_g[0], ref_g)
        if torch.equal(ids, ids_g):
            assert rel_l2(out.cpu().numpy()[0], out_g.cpu().numpy()[0]) <= 2e-3
        assert packed.device_error() == 0


@pytest.mark.parametrize("fmt,layout", FMTS, ids=IDS)
def test_packed_bf16_output(dev, fmt, layout):
    """bf16 output: the layer's error on top of the output rounding stays <= 1e-3."""
    H = I = 2880
    layer, dense, _ = _build_layer(dev, fmt, fmt, H, I, 8, 4, layout, seed=12)
    x = _x(H, 300)
    out, ids, wts = layer.decode(x.to(dev))
    assert out.dtype == torch.bfloat16
    ref = _oracle_layer(x.float().numpy(), ids.cpu().numpy()[0], wts.cpu().numpy()[0], dense)
    assert_layer(out[0], ref)
    assert layer_bound(out, ref) < 3e-3


@pytest.mark.parametrize("fmt,layout", FMTS, ids=IDS)
def test_packed_given_ids_bias_and_silu(dev, fmt, layout):
    H, I, E, k = 1024, 576, 6, 2
    layer, dense, _ = _build_layer(dev, fmt, fmt, H, I, E, k, layout, seed=77, bias=True, activation="silu")
    assert layer.packed
    x = _x(H, 1)
    ids = torch.tensor([[5, 2]], dtype=torch.int32)
    wts = torch.tensor([[0.7, 0.3]])
    out, _, _ = layer.decode(x.to(dev), ids=ids.to(dev), weights=wts.to(dev), out_dtype=torch.float32)
    ref = _oracle_layer(x.float().numpy(), [5, 2], [0.7, 0.3], dense, act="silu")
    assert_layer(out[0], ref)


@pytest.mark.parametrize("fmt,layout", FMTS, ids=IDS)
def test_packed_top8_small_layer(dev, fmt, layout):
    H, I, E, k = 512, 256, 16, 8
    layer, dense, _ = _build_layer(dev, fmt, fmt, H, I, E, k, layout, seed=3)
    x = _x(H, 2)
    out, ids, wts = layer.decode(x.to(dev), out_dtype=torch.float32)
    ref = _oracle_layer(x.float().numpy(), ids.cpu().numpy()[0], wts.cpu().numpy()[0], dense)
    assert_layer(out[0], ref)


@pytest.mark.parametrize("scale", [1e-30, 1e30])
@pytest.mark.parametrize("fmt,layout", FMTS, ids=IDS)
def test_packed_wide_input_range(dev, fmt, layout, scale):
    """The activation vectors are staged with a power-of-two scale per
    32-element sub-block, so inputs far from 1 keep their precision."""
    H, I, E, k = 1024, 512, 4, 2
    layer, dense, _ = _build_layer(dev, fmt, fmt, H, I, E, k, layout, seed=9)
    x = _x(H, 3, scale)
    ids = torch.tensor([[0, 3]], dtype=torch.int32, device=dev)
    wts = torch.tensor([[0.6, 0.4]], device=dev)
    out, _, _ = layer.decode(x.to(dev), ids=ids, weights=wts, out_dtype=torch.float32)
    ref = _oracle_layer(x.double().numpy(), [0, 3], [0.6, 0.4], dense)
    assert np.isfinite(out.cpu().numpy()).all()
    assert_layer(out[0], ref)


@pytest.mark.parametrize("fmt,layout", FMTS, ids=IDS)
def test_packed_deterministic(dev, fmt, layout):
    H = I = 2880
    layer, _, _ = _build_layer(dev, fmt, fmt, H, I, 8, 4, layout, seed=21)
    x = _x(H, 5).to(dev)
    outs = [layer.decode(x)[0].clone() for _ in range(5)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def test_packed_bad_expert_ids(dev):
    H, I, E, k = 512, 256, 4, 2
    layer, dense, _ = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, E, k, "separate", seed=6)
    x = _x(H, 4)
    out, _, _ = layer.decode(x.to(dev), ids=torch.tensor([[1, 1000]], device=dev),
                             weights=torch.tensor([[0.5, 0.5]], device=dev), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert layer.device_error() == 2
    ref = _oracle_layer(x.float().numpy(), [1], [0.5], dense)
    assert_layer(out[0], ref)
    assert layer.device_error() == 0


@pytest.mark.parametrize("T", [3, 20])
def test_packed_several_tokens(dev, T):
    """T <= 16 runs the packed batch-1 path per token; larger T takes the
    grouped path on the raw streams."""
    H, I, E, k = 1024, 512, 8, 2
    layer, dense, router = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, E, k, "separate", seed=31)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16)
    out, ids, wts = layer.decode(x.to(dev), out_dtype=torch.float32)
    torch.cuda.synchronize()
    for t in range(T):
        ref = _oracle_layer(x[t:t + 1].float().numpy(), ids.cpu().numpy()[t], wts.cpu().numpy()[t], dense)
        assert_layer(out[t], ref)


def test_packed_decode_into_buffers(dev):
    """decode_ (prepared arguments, no allocation) on the packed layer."""
    H = I = 2880
    layer, dense, _ = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, 8, 4, "separate", seed=41)
    x = _x(H, 8).to(dev)
    out = torch.empty(1, H, dtype=torch.bfloat16, device=dev)
    ids = torch.empty(1, 4, dtype=torch.int32, device=dev)
    wts = torch.empty(1, 4, dtype=torch.float32, device=dev)
    for _ in range(2):
        layer.decode_(x, out, ids, wts)
    torch.cuda.synchronize()
    ref = _oracle_layer(x.float().cpu().numpy(), ids.cpu().numpy()[0], wts.cpu().numpy()[0], dense)
    assert_layer(out[0], ref)
    ids_o, _, _ = OE.router_topk_softmax(x.float().cpu().numpy(), layer.router_w.float().cpu().numpy(), 4)
    assert set(ids.cpu().numpy()[0]) == set(ids_o[0])


@pytest.mark.parametrize("fmt", [GGML_Q4_K, TSB_MXFP4], ids=IDS)
def test_config1_full_shape_token_stream(dev, fmt):
    """BASELINE config 1 as bench.py runs it: the GPT-OSS-20B-shaped layer
    (32 experts, top-4, H = I = 2880, clamp-SwiGLU) built by
    workloads.build_layer with the bench's seed, decoding 32 steps of the
    bench's seeded token stream; every step against the oracle (fp32 output,
    1e-3) using the experts the kernel routed to, whose routing is itself
    checked against the oracle router."""
    from tests.helpers import oracle_dequant
    from tinyserve_b200.workloads import build_layer, hidden_states
    layer = build_layer(fmt, seed=0, device=dev)
    assert layer.packed
    xs = hidden_states(32, device=dev)
    router = layer.router_w.cpu()
    dense_cache = {}

    def dense(e):
        if e not in dense_cache:
            ex = layer.experts[e]
            if fmt == TSB_MXFP4:
                gu = oracle_dequant(fmt, ex.gate.cpu(), ex.gate_scales.cpu(), 2 * 2880, 2880)
                wd = oracle_dequant(fmt, ex.down.cpu(), ex.down_scales.cpu(), 2880, 2880)
                dense_cache[e] = (gu[0::2], gu[1::2], wd, None, None, None)
            else:
                dense_cache[e] = (oracle_dequant(fmt, ex.gate.cpu(), None, 2880, 2880),
                                  oracle_dequant(fmt, ex.up.cpu(), None, 2880, 2880),
                                  oracle_dequant(fmt, ex.down.cpu(), None, 2880, 2880), None, None, None)
        return dense_cache[e]

    for t in range(32):
        x = xs[t:t + 1]
        out, ids, wts = layer.decode(x, out_dtype=torch.float32)
        torch.cuda.synchronize()
        xc = x.cpu()
        _check_routing(xc, router, 4, ids, wts)
        idl = [int(i) for i in ids.cpu().numpy()[0]]
        table = {e: dense(e) for e in idl}
        ref = _oracle_layer(xc.float().numpy(), idl, wts.cpu().numpy()[0], table)
        assert_layer(out[0], ref)
    assert layer.device_error() == 0
