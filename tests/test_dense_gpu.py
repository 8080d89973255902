"""Dense (fp32 / fp16 / bf16) expert layers through the C-ABI against float64
oracle math: the dense inline forward of the reference
(tinyserve/expert_forward.py:109-194, transposes :140-149, clamp-SwiGLU
:185-187) and its batched use in a layer (router, top-k, weighted combine)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import expert as OE
from tests.helpers import assert_layer, rel_l2
from tinyserve_b200 import _lib
from tinyserve_b200.formats import GGML_BF16, GGML_F16, GGML_F32

pytestmark = pytest.mark.gpu

DT = {GGML_F32: torch.float32, GGML_F16: torch.float16, GGML_BF16: torch.bfloat16}


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    return torch.device("cuda:0")


def _dense_layer(dev, fmt, H, I, E, k, layout, transposed, activation="swiglu_oai", bias=True, seed=0, router=True):
    """A QuantMoE over seeded dense experts and the float64 oracle's view of them."""
    from tinyserve_b200.moe import ExpertWeights, QuantMoE
    g = torch.Generator().manual_seed(seed)
    dt = DT[fmt]
    experts, dense = [], []
    for _ in range(E):
        wg = (torch.randn(I, H, generator=g) * 0.02).to(dt)
        wu = (torch.randn(I, H, generator=g) * 0.02).to(dt)
        wd = (torch.randn(H, I, generator=g) * 0.02).to(dt)
        bg = bu = bd = None
        if bias:
            bg, bu, bd = (torch.randn(n, generator=g) * 0.1 for n in (I, I, H))
        if layout == "separate":
            gate, up = wg, wu
        elif layout == "interleaved":
            gate, up = torch.stack([wg, wu], 1).reshape(2 * I, H), None
        else:
            gate, up = torch.cat([wg, wu]), None
        down = wd
        if transposed & _lib.T_GATE_UP:
            gate = gate.t().contiguous()
            up = up.t().contiguous() if up is not None else None
        if transposed & _lib.T_DOWN:
            down = down.t().contiguous()
        cu = lambda t: None if t is None else t.to(dev)  # noqa: E731
        experts.append(ExpertWeights(gate=cu(gate), up=cu(up), down=cu(down), gate_bias=cu(bg), up_bias=cu(bu),
                                     down_bias=cu(bd)))
        dense.append((wg.double().numpy(), wu.double().numpy(), wd.double().numpy(),
                      None if bg is None else (bg.double().numpy(), bu.double().numpy(), bd.double().numpy())))
    rw = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16) if router else None
    layer = QuantMoE(experts, fmt_gate_up=fmt, fmt_down=fmt, hidden=H, inter=I, top_k=k,
                     router_w=None if rw is None else rw.to(dev), gate_up_layout=layout, activation=activation,
                     transposed=transposed)
    return layer, dense, rw


def _oracle(x, ids, wts, dense, activation):
    x = x.float().numpy().astype(np.float64)
    out = np.zeros_like(x)
    for t in range(x.shape[0]):
        for j in range(ids.shape[1]):
            e = int(ids[t, j])
            if e < 0:
                continue
            wg, wu, wd, b = dense[e]
            bg, bu, bd = b if b is not None else (None, None, None)
            out[t] += float(wts[t, j]) * OE.expert_forward(x[t:t + 1], wg, wu, wd, activation, bg, bu, bd)[0]
    return out


@pytest.mark.parametrize("fmt", [GGML_BF16, GGML_F16, GGML_F32])
@pytest.mark.parametrize("layout", ["separate", "interleaved", "chunked"])
@pytest.mark.parametrize("transposed", [0, 3])
def test_dense_layer_formats_layouts(dev, fmt, layout, transposed):
    H, I, E, k, T = 512, 384, 8, 4, 3
    layer, dense, rw = _dense_layer(dev, fmt, H, I, E, k, layout, transposed, seed=fmt * 7 + transposed)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    out, ids, wts = layer.decode(x.to(dev), out_dtype=torch.float32)
    torch.cuda.synchronize()
    ids_c, wts_c = ids.cpu().numpy(), wts.cpu().numpy()
    r_ids, _, _ = OE.router_topk_softmax(x.float().numpy(), rw.float().numpy(), k)
    assert (np.sort(ids_c, 1) == np.sort(r_ids, 1)).all()
    ref = _oracle(x, ids_c, wts_c, dense, "swiglu_oai")
    err = assert_layer(out, ref)
    assert err < 1e-5, err  # fp32 accumulation of exact float weights: only summation-order error
    assert layer.device_error(T) == 0


@pytest.mark.parametrize("T", [1, 17, 64])
@pytest.mark.parametrize("transposed", [0, 1, 2])
def test_dense_layer_batches_and_bf16_out(dev, T, transposed):
    """Given ids (with skipped slots), bf16 output, SiLU, one launch set for any T."""
    H, I, E, k = 256, 512, 6, 2
    layer, dense, _ = _dense_layer(dev, GGML_BF16, H, I, E, k, "chunked", transposed, activation="silu",
                                   bias=False, seed=T, router=False)
    g = torch.Generator().manual_seed(100 + T)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    ids = torch.randint(0, E, (T, k), generator=g, dtype=torch.int32)
    ids[::3, 1] = -1  # slots owned elsewhere are skipped
    wts = torch.rand(T, k, generator=g)
    out, _, _ = layer.decode(x.to(dev), ids=ids, weights=wts)
    torch.cuda.synchronize()
    ref = _oracle(x, ids.numpy(), wts.numpy(), dense, "silu")
    assert out.dtype == torch.bfloat16
    assert_layer(out, ref)
    assert layer.device_error(T) == 0


def test_dense_bad_expert_id_reported(dev):
    layer, _, _ = _dense_layer(dev, GGML_BF16, 256, 256, 4, 2, "separate", 0, router=False)
    x = torch.randn(1, 256).to(torch.bfloat16).to(dev)
    ids = torch.tensor([[1, 9]], dtype=torch.int32)
    out, _, _ = layer.decode(x, ids=ids, weights=torch.ones(1, 2))
    torch.cuda.synchronize()
    assert layer.device_error() == 2
    assert torch.isfinite(out.float()).all()


def test_dense_misaligned_weight_reported_not_read(dev):
    """A weight pointer off the 16-byte grid is reported (code 3) and never read."""
    from tinyserve_b200.moe import ExpertWeights, QuantMoE
    H, I = 256, 256
    buf = torch.zeros(2 * I * H * 2 + 64, dtype=torch.uint8, device=dev)
    gate = buf[8:8 + 2 * I * H * 2]  # 8-byte offset
    down = torch.zeros(H * I * 2, dtype=torch.uint8, device=dev)
    layer = QuantMoE([ExpertWeights(gate=gate, down=down)], fmt_gate_up=GGML_BF16, fmt_down=GGML_BF16, hidden=H,
                     inter=I, top_k=1, gate_up_layout="interleaved")
    x = torch.randn(1, H).to(torch.bfloat16).to(dev)
    layer.decode(x, ids=torch.zeros(1, 1, dtype=torch.int32), weights=torch.ones(1, 1))
    torch.cuda.synchronize()
    assert layer.device_error() == 3


@pytest.mark.parametrize("act", [None, "silu"])
@pytest.mark.parametrize("H,I", [(512, 256), (384, 384)])
def test_dense_inline_forward_matches_reference_semantics(dev, act, H, I):
    """build_inline_forward on a packed [gate_up_proj, bias, down_proj, bias]
    buffer stored as GPT-OSS stores dense experts (gate_up [H, 2I], down [I, H]),
    checked against the reference's own arithmetic written in torch float64:
    transpose rule, F.linear, interleaved clamp-SwiGLU or chunked SiLU."""
    from tinyserve_b200.expert_forward import TensorLayout, build_inline_forward
    g = torch.Generator().manual_seed(H + I)
    gu = (torch.randn(H, 2 * I, generator=g) * 0.02).to(torch.bfloat16)
    gub = (torch.randn(2 * I, generator=g) * 0.1).to(torch.bfloat16)
    dn = (torch.randn(I, H, generator=g) * 0.02).to(torch.bfloat16)
    dnb = (torch.randn(H, generator=g) * 0.1).to(torch.bfloat16)
    tensors = {"gate_up_proj": gu, "gate_up_proj_bias": gub, "down_proj": dn, "down_proj_bias": dnb}
    layout = TensorLayout.from_tensors(tensors)
    packed = torch.cat([t.contiguous().view(-1).view(torch.uint8) for t in tensors.values()]).to(dev)
    fwd = build_inline_forward(layout, None if act is None else torch.nn.SiLU())
    h = torch.randn(5, H, generator=g).to(torch.bfloat16)
    out = fwd(packed, h.to(dev))
    # the reference's rule (expert_forward.py:140-149) in float64
    w_gu = gu.double()
    if gu.shape[0] == min(gu.shape):
        w_gu = w_gu.t()
    w_dn = dn.double()
    if dn.shape[0] == max(gu.shape) // 2:
        w_dn = w_dn.t()
    y = torch.nn.functional.linear(h.double(), w_gu, gub.double())
    if act is None:
        gate, up = y[..., ::2].clamp(max=7.0), y[..., 1::2].clamp(min=-7.0, max=7.0)
        a = (up + 1) * gate * torch.sigmoid(gate * 1.702)
    else:
        gate, up = y.chunk(2, dim=-1)
        a = torch.nn.functional.silu(gate) * up
    ref = torch.nn.functional.linear(a, w_dn, dnb.double()).numpy()
    assert out.dtype == torch.bfloat16 and out.shape == (5, H)
    assert_layer(out, ref)
    # a refilled cache slot (same address, new contents) is read afresh, biases included
    packed2 = packed.clone()
    packed.zero_()
    assert float(fwd(packed, h.to(dev)).float().abs().max()) == 0.0
    packed.copy_(packed2)
    assert rel_l2(fwd(packed, h.to(dev)).float().cpu().numpy(), out.float().cpu().numpy()) == 0.0


def test_dense_capi_workspace_any_T(dev):
    L = _lib.lib()
    spec = _lib.TsbMoeSpec(GGML_BF16, GGML_BF16, 2880, 2880, 32, 4, _lib.GU_INTERLEAVED, _lib.ACT_SWIGLU_OAI,
                           7.0, 1.702, 0, _lib.T_GATE_UP | _lib.T_DOWN)
    a = L.tsb_moe_decode_workspace(ctypes.byref(spec), 1)
    b = L.tsb_moe_decode_workspace(ctypes.byref(spec), 64)
    assert 0 < a <= b
    assert L.tsb_moe_prefill_workspace(ctypes.byref(spec), 64) == b
