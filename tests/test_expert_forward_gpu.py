"""The per-expert forward mirrors (tinyserve_b200.expert_forward) against
float64 math on oracle-dequantised weights: GGMLExpertForward on packed GGUF
bytes (tinyserve/ggml_forward.py:68-151), the GPT-OSS MXFP4 inline forward
(tinyserve/expert_forward.py:197-246) and GGMLLinear (ggml_linear.py:48-117)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import expert as OE
from tests.helpers import assert_layer, make_weight, oracle_dequant, rel_l2
from tinyserve_b200.formats import GGML_Q4_K, GGML_Q6_K, GGML_Q8_0, TSB_MXFP4

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    return torch.device("cuda:0")


@pytest.mark.parametrize("T", [1, 5, 40])
def test_ggml_expert_forward_packed(dev, T):
    from tinyserve_b200.expert_forward import GGMLExpertForward, TensorLayout
    H, I = 512, 256
    g, _ = make_weight(GGML_Q4_K, I, H, 1)
    u, _ = make_weight(GGML_Q4_K, I, H, 2)
    d, _ = make_weight(GGML_Q6_K, H, I, 3)
    layout = TensorLayout({"gate": ((g.numel(),), torch.uint8), "up": ((u.numel(),), torch.uint8),
                           "down": ((d.numel(),), torch.uint8)})
    packed = torch.cat([g, u, d]).to(dev)
    fwd = GGMLExpertForward(layout, {"gate": GGML_Q4_K, "up": GGML_Q4_K, "down": GGML_Q6_K}, torch.nn.SiLU(),
                            {"gate": (H, I), "up": (H, I), "down": (I, H)})
    h = torch.randn(T, H, generator=torch.Generator().manual_seed(T)).to(torch.bfloat16)
    out = fwd.forward(packed, h.to(dev))
    ref = OE.expert_forward(h.float().numpy(), oracle_dequant(GGML_Q4_K, g, None, I, H),
                            oracle_dequant(GGML_Q4_K, u, None, I, H), oracle_dequant(GGML_Q6_K, d, None, H, I), "silu")
    assert out.shape == (T, H) and out.dtype == torch.bfloat16
    assert_layer(out, ref)


@pytest.mark.parametrize("act", [None, "silu"])
def test_mxfp4_inline_forward(dev, act):
    from tinyserve_b200.expert_forward import TensorLayout, build_mxfp4_inline_forward
    H, I, T = 512, 256, 7
    gu, gus = make_weight(TSB_MXFP4, 2 * I, H, 11)
    dn, dns = make_weight(TSB_MXFP4, H, I, 12)
    g = torch.Generator().manual_seed(5)
    gub = (torch.randn(2 * I, generator=g) * 0.1).to(torch.bfloat16)
    dnb = (torch.randn(H, generator=g) * 0.1).to(torch.bfloat16)
    tensors = {"gate_up_proj": gu.view(2 * I, H // 32, 16), "gate_up_proj_scales": gus.view(2 * I, H // 32),
               "gate_up_proj_bias": gub, "down_proj": dn.view(H, I // 32, 16), "down_proj_scales": dns.view(H, I // 32),
               "down_proj_bias": dnb}
    layout = TensorLayout.from_tensors(tensors)
    packed = torch.cat([t.contiguous().view(-1).view(torch.uint8) for t in tensors.values()]).to(dev)
    fwd = build_mxfp4_inline_forward(layout, None if act is None else torch.nn.SiLU())
    h = torch.randn(T, H, generator=g).to(torch.bfloat16)
    out = fwd(packed, h.to(dev))
    wgu = oracle_dequant(TSB_MXFP4, gu, gus, 2 * I, H)
    wd = oracle_dequant(TSB_MXFP4, dn, dns, H, I)
    b = gub.float().numpy()
    if act is None:
        wg, wu, bg, bu = wgu[0::2], wgu[1::2], b[0::2], b[1::2]
    else:
        wg, wu, bg, bu = wgu[:I], wgu[I:], b[:I], b[I:]
    ref = OE.expert_forward(h.float().numpy(), wg, wu, wd, "swiglu_oai" if act is None else "silu", bg, bu,
                            dnb.float().numpy())
    assert_layer(out, ref)


@pytest.mark.parametrize("batch", [1, 3, 11])
def test_ggml_linear(dev, batch):
    from tinyserve_b200.expert_forward import GGMLLinear
    N, K = 384, 512
    w, _ = make_weight(GGML_Q8_0, N, K, 21)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(1)) * 0.1
    lin = GGMLLinear(w, GGML_Q8_0, N, K, bias=bias, device=dev)
    x = torch.randn(batch, K, generator=torch.Generator().manual_seed(batch)).to(torch.bfloat16)
    with torch.no_grad():
        y = lin(x.to(dev))
    mv = x.double().numpy() @ oracle_dequant(GGML_Q8_0, w, None, N, K).astype(np.float64).T
    ref = mv + bias.double().numpy()
    assert y.shape == (batch, N)
    # like the reference's GGMLLinear (ggml_linear.py:77-100) the matvec comes
    # back in the activation dtype (bf16) before the fp32 bias is added: the
    # bound is that rounding plus 1e-3
    from oracle.expert import bf16_round
    bound = rel_l2(bf16_round(mv.astype(np.float32)) + bias.double().numpy(), ref) + 1e-3
    assert rel_l2(y.float().cpu().numpy(), ref) <= bound
