"""The allocation-free MoE decode entry point.

tsb_moe_decode_noalloc exists for callers with no device scratch memory to
hand over: it runs the same layer as tsb_moe_decode with its scratch in a
static array inside the library.  Its output must match the workspace-taking
entry point call after call (the array keeps the previous call's contents, so
several calls in a row are checked), and the oracle layer within the
north-star tolerance.  This file is named to be collected last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from tests.helpers import assert_layer, make_weight, oracle_dequant
from tinyserve_b200 import _lib
from tinyserve_b200.formats import GGML_Q4_K

def _layer(dev, H=1024, I=512, E=8, k=4, seed=21, pack=None):
    from tinyserve_b200.moe import ExpertWeights, QuantMoE
    experts = []
    for e in range(E):
        g, _ = make_weight(GGML_Q4_K, I, H, seed * 100 + 3 * e)
        u, _ = make_weight(GGML_Q4_K, I, H, seed * 100 + 3 * e + 1)
        d, _ = make_weight(GGML_Q4_K, H, I, seed * 100 + 3 * e + 2)
        experts.append(ExpertWeights(gate=g.to(dev), up=u.to(dev), down=d.to(dev)))
    router = (torch.randn(E, H, generator=torch.Generator().manual_seed(seed)) * 0.02).to(torch.bfloat16)
    return QuantMoE(experts, fmt_gate_up=GGML_Q4_K, fmt_down=GGML_Q4_K, hidden=H, inter=I, top_k=k,
                    router_w=router.to(dev), pack=pack)


def _noalloc(layer, x):
    T = x.shape[0]
    ids = torch.empty(T, layer.top_k, dtype=torch.int32, device=x.device)
    wts = torch.empty(T, layer.top_k, dtype=torch.float32, device=x.device)
    out = torch.empty(T, layer.hidden, dtype=torch.bfloat16, device=x.device)
    rc = _lib.lib().tsb_moe_decode_noalloc(
        ctypes.byref(layer.spec), layer._table.data_ptr(), x.data_ptr(), T, layer.router_w.data_ptr(), None,
        ids.data_ptr(), wts.data_ptr(), out.data_ptr(), torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(rc)
    return out, ids, wts


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 3])
def test_noalloc_matches_workspace_entry_point_and_oracle(T):
    """Three calls in a row: the same routing, weights and output as
    tsb_moe_decode on the generic layer (the same kernels), and the oracle
    layer (float64 on the reference-dequantised weights) within 1e-3 on top
    of the bf16 output rounding."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    from tests.test_kernels_gpu import _oracle_layer
    dev = torch.device("cuda:0")
    layer = _layer(dev, pack=False)
    H, I = layer.hidden, layer.inter
    dense = {}
    for e, ex in enumerate(layer.experts):
        dense[e] = (oracle_dequant(GGML_Q4_K, ex.gate.cpu(), None, I, H), oracle_dequant(GGML_Q4_K, ex.up.cpu(), None, I, H),
                    oracle_dequant(GGML_Q4_K, ex.down.cpu(), None, H, I), None, None, None)
    for step in range(3):
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(500 + step)).to(torch.bfloat16).to(dev)
        ref, ref_ids, ref_w = layer.decode(x)
        got, ids, w = _noalloc(layer, x)
        torch.cuda.synchronize()
        assert torch.equal(ids.cpu(), ref_ids.cpu())
        np.testing.assert_allclose(w.cpu().numpy(), ref_w.cpu().numpy(), rtol=1e-6, atol=1e-7)
        assert torch.equal(got.cpu(), ref.cpu())
        for t in range(T):
            oref = _oracle_layer(x[t:t + 1].float().cpu().numpy(), ids.cpu().numpy()[t], w.cpu().numpy()[t], dense)
            assert_layer(got[t], oref)


def test_noalloc_rejects_layers_beyond_the_static_workspace():
    """A layer whose scratch exceeds the 1 MiB array is refused before any GPU work."""
    spec = _lib.TsbMoeSpec(GGML_Q4_K, GGML_Q4_K, 4096, 65536, 64, 8, 0, 1, 7.0, 1.702)
    rc = _lib.lib().tsb_moe_decode_noalloc(ctypes.byref(spec), 16, 16, 1, 16, None, 16, 16, 16, None)
    assert rc == _lib.TSB_ERR_WORKSPACE
    assert "static workspace" in _lib.last_error()
