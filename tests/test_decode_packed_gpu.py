"""GPU parity of batch-1 decode on the decode-packed Q4_K experts
(tsb_moe_pack / tsb_moe_decode_packed) against the oracle layer (float64 math
on the reference-dequantised weights) and against the generic decode engine.
Tolerance: relative L2 <= 1e-3 of the layer math plus bf16 output rounding
(4e-3), as for tsb_moe_decode."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import expert as OE
from tests.helpers import rel_l2
from tests.test_kernels_gpu import _build_layer, _oracle_layer
from tinyserve_b200.formats import GGML_Q4_K

pytestmark = pytest.mark.gpu
TOL = 1e-3 + 4e-3


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    return torch.device("cuda:0")


def _x(H, seed, scale=1.0):
    return (torch.randn(1, H, generator=torch.Generator().manual_seed(seed)) * scale).to(torch.bfloat16)


def _ref_w(x, router, k):
    return OE.router_topk_softmax(x.float().numpy(), router.float().numpy(), k)[1][0]


@pytest.mark.parametrize("layout", ["separate", "interleaved", "chunked"])
def test_packed_layer_matches_oracle_and_engine(dev, layout):
    """GPT-OSS-20B shape (H = I = 2880, K % 256 != 0: rows start mid-superblock)."""
    H = I = 2880
    E, k = 8, 4
    packed, dense, router = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, E, k, layout, seed=11)
    generic, _, _ = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, E, k, layout, seed=11, pack=False)
    assert packed.packed and not generic.packed
    for step in range(3):
        x = _x(H, 200 + step)
        out, ids, wts = packed.decode(x.to(dev))
        out_g, ids_g, _g_w = generic.decode(x.to(dev))
        torch.cuda.synchronize()
        # routing runs inside the packed gate/up launch (its own summation
        # order): the same experts unless two logits tie after bf16 rounding
        ids_o, _, lg = OE.router_topk_softmax(x.float().numpy(), router.float().numpy(), k)
        if set(ids.cpu().numpy()[0]) != set(ids_o[0]):
            srt = np.sort(lg[0])[::-1]
            assert abs(srt[k - 1] - srt[k]) <= 1e-2 * abs(srt[k - 1]) + 1e-6, "routing differs away from a tie"
        else:
            np.testing.assert_allclose(np.sort(wts.cpu().numpy()[0])[::-1], np.sort(_ref_w(x, router, k))[::-1],
                                       rtol=1e-5, atol=1e-6)
        ref = _oracle_layer(x.float().numpy(), ids.cpu().numpy()[0], wts.cpu().numpy()[0], dense)
        assert rel_l2(out.float().cpu().numpy()[0], ref) <= TOL
        # the generic engine on the raw streams (rows start mid-superblock:
        # covers its interleaved row order)
        if torch.equal(ids, ids_g):
            assert rel_l2(out.float().cpu().numpy()[0], out_g.float().cpu().numpy()[0]) <= TOL
        ref_g = _oracle_layer(x.float().numpy(), ids_g.cpu().numpy()[0], _g_w.cpu().numpy()[0], dense)
        assert rel_l2(out_g.float().cpu().numpy()[0], ref_g) <= TOL
        assert packed.device_error() == 0


def test_packed_given_ids_bias_and_silu(dev):
    H, I, E, k = 1024, 576, 6, 2
    layer, dense, _ = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, E, k, "separate", seed=77, bias=True,
                                   activation="silu")
    assert layer.packed
    x = _x(H, 1)
    ids = torch.tensor([[5, 2]], dtype=torch.int32)
    wts = torch.tensor([[0.7, 0.3]])
    out, _, _ = layer.decode(x.to(dev), ids=ids.to(dev), weights=wts.to(dev))
    ref = _oracle_layer(x.float().numpy(), [5, 2], [0.7, 0.3], dense, act="silu")
    assert rel_l2(out.float().cpu().numpy()[0], ref) <= TOL


def test_packed_top8_small_layer(dev):
    H, I, E, k = 512, 256, 16, 8
    layer, dense, _ = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, E, k, "interleaved", seed=3)
    x = _x(H, 2)
    out, ids, wts = layer.decode(x.to(dev))
    ref = _oracle_layer(x.float().numpy(), ids.cpu().numpy()[0], wts.cpu().numpy()[0], dense)
    assert rel_l2(out.float().cpu().numpy()[0], ref) <= TOL


@pytest.mark.parametrize("scale", [1e-30, 1e30])
def test_packed_wide_input_range(dev, scale):
    """The activation vector is staged with a power-of-two scale, so inputs far
    from 1 keep their precision in fp16."""
    H, I, E, k = 1024, 512, 4, 2
    layer, dense, _ = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, E, k, "separate", seed=9)
    x = _x(H, 3, scale)
    ids = torch.tensor([[0, 3]], dtype=torch.int32, device=dev)
    wts = torch.tensor([[0.6, 0.4]], device=dev)
    out, _, _ = layer.decode(x.to(dev), ids=ids, weights=wts)
    ref = _oracle_layer(x.double().numpy(), [0, 3], [0.6, 0.4], dense)
    got = out.float().cpu().numpy()[0]
    assert np.isfinite(got).all()
    assert rel_l2(got, ref) <= TOL


def test_packed_deterministic(dev):
    H = I = 2880
    layer, _, _ = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, 8, 4, "separate", seed=21)
    x = _x(H, 5).to(dev)
    outs = [layer.decode(x)[0].clone() for _ in range(5)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def test_packed_bad_expert_ids(dev):
    H, I, E, k = 512, 256, 4, 2
    layer, dense, _ = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, E, k, "separate", seed=6)
    x = _x(H, 4)
    out, _, _ = layer.decode(x.to(dev), ids=torch.tensor([[1, 1000]], device=dev),
                             weights=torch.tensor([[0.5, 0.5]], device=dev))
    torch.cuda.synchronize()
    assert layer.device_error() == 2
    ref = _oracle_layer(x.float().numpy(), [1], [0.5], dense)
    assert rel_l2(out.float().cpu().numpy()[0], ref) <= TOL
    assert layer.device_error() == 0


@pytest.mark.parametrize("T", [3, 20])
def test_packed_several_tokens(dev, T):
    """T <= 16 loops the packed batch-1 path per token; larger T takes the
    grouped path on the raw streams."""
    H, I, E, k = 1024, 512, 8, 2
    layer, dense, router = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, E, k, "separate", seed=31)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16)
    out, ids, wts = layer.decode(x.to(dev))
    torch.cuda.synchronize()
    for t in range(T):
        ref = _oracle_layer(x[t:t + 1].float().numpy(), ids.cpu().numpy()[t], wts.cpu().numpy()[t], dense)
        assert rel_l2(out[t].float().cpu().numpy(), ref) <= TOL


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
    assert rel_l2(out.float().cpu().numpy()[0], ref) <= TOL
    ids_o, _, _ = OE.router_topk_softmax(x.float().cpu().numpy(), layer.router_w.float().cpu().numpy(), 4)
    assert set(ids.cpu().numpy()[0]) == set(ids_o[0])
