"""The allocation-free MoE decode entry point.

tsb_moe_decode_noalloc exists for callers that cannot allocate device memory
(a stream under CUDA-graph capture, a host with a fixed memory plan): it runs
the same layer as tsb_moe_decode with its scratch in a static array inside the
library.  Its output must match the workspace-taking entry point, call after
call (the array keeps the previous call's contents, so two calls in a row are
checked).  This file is named to be collected last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from tests.helpers import make_weight, rel_l2
from tinyserve_b200 import _lib
from tinyserve_b200.formats import GGML_Q4_K

TOL = 1e-3 + 4e-3  # the layer tolerance of tests/test_kernels_gpu.py (bf16 output)


def _layer(dev, H=1024, I=512, E=8, k=4, seed=21):
    from tinyserve_b200.moe import ExpertWeights, QuantMoE
    experts = []
    for e in range(E):
        g, _ = make_weight(GGML_Q4_K, I, H, seed * 100 + 3 * e)
        u, _ = make_weight(GGML_Q4_K, I, H, seed * 100 + 3 * e + 1)
        d, _ = make_weight(GGML_Q4_K, H, I, seed * 100 + 3 * e + 2)
        experts.append(ExpertWeights(gate=g.to(dev), up=u.to(dev), down=d.to(dev)))
    router = (torch.randn(E, H, generator=torch.Generator().manual_seed(seed)) * 0.02).to(torch.bfloat16)
    return QuantMoE(experts, fmt_gate_up=GGML_Q4_K, fmt_down=GGML_Q4_K, hidden=H, inter=I, top_k=k,
                    router_w=router.to(dev))


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
def test_noalloc_matches_workspace_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    dev = torch.device("cuda:0")
    layer = _layer(dev)
    for step in range(2):
        x = torch.randn(1, layer.hidden, generator=torch.Generator().manual_seed(500 + step)).to(torch.bfloat16).to(dev)
        ref, ref_ids, ref_w = layer.decode(x)
        got, ids, w = _noalloc(layer, x)
        torch.cuda.synchronize()
        assert torch.equal(ids.cpu(), ref_ids.cpu())
        np.testing.assert_allclose(w.cpu().numpy(), ref_w.cpu().numpy(), rtol=1e-6, atol=1e-7)
        assert rel_l2(got.float().cpu().numpy(), ref.float().cpu().numpy()) <= TOL


def test_noalloc_rejects_layers_beyond_the_static_workspace():
    """A layer whose scratch exceeds the 1 MiB array is refused before any GPU work."""
    spec = _lib.TsbMoeSpec(GGML_Q4_K, GGML_Q4_K, 4096, 65536, 64, 8, 0, 1, 7.0, 1.702)
    rc = _lib.lib().tsb_moe_decode_noalloc(ctypes.byref(spec), 16, 16, 1, 16, None, 16, 16, 16, None)
    assert rc == _lib.TSB_ERR_WORKSPACE
    assert "static workspace" in _lib.last_error()
