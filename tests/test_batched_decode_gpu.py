"""Several tokens decoding together (the reference's ExpertBatcher,
tinyserve/expert_batcher.py:31-85, and execute_layer_experts for T > 1):
parity of tsb_moe_decode with T > 1 and of the Python mirrors of the
reference's layer API against float64 math on the dequantised weights."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import expert as OE
from tests.helpers import assert_layer, rel_l2
from tests.test_kernels_gpu import _build_layer
from tests.test_prefill_gpu import _oracle
from tinyserve_b200.formats import GGML_Q4_K, GGML_Q8_0, TSB_MXFP4


pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    return torch.device("cuda:0")


@pytest.mark.parametrize("fmt,layout,T", [(GGML_Q4_K, "separate", 5), (TSB_MXFP4, "interleaved", 64),
                                          (GGML_Q8_0, "chunked", 9)])
def test_decode_several_tokens_with_router(dev, fmt, layout, T):
    H, I, E, k = 1024, 512, 16, 4
    layer, dense, router = _build_layer(dev, fmt, fmt, H, I, E, k, layout, seed=100 + T)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(T)).to(torch.bfloat16)
    out, ids, wts = layer.decode(x.to(dev))
    torch.cuda.synchronize()
    ids_o, wts_o, lg = OE.router_topk_softmax(x.float().numpy(), router.float().numpy(), k)
    ids_g = ids.cpu().numpy()
    for t in range(T):
        if set(ids_g[t]) != set(ids_o[t]):
            srt = np.sort(lg[t])[::-1]
            assert abs(srt[k - 1] - srt[k]) <= 1e-2 * abs(srt[k - 1]) + 1e-6
    ref = _oracle(x.float().numpy(), ids_g, wts.cpu().numpy(), dense)
    assert_layer(out, ref)
    assert layer.device_error(T) == 0


def test_batcher_matches_per_request_decode(dev):
    from tinyserve_b200.pipeline import BatchItem, ExpertBatcher, ExpertPipeline
    H, I, E, k = 512, 256, 8, 2
    layer, dense, _ = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, E, k, "separate", seed=7)
    pipe = ExpertPipeline({3: layer})
    g = torch.Generator().manual_seed(1)
    items = []
    for r in range(6):
        ids = torch.randperm(E, generator=g)[:k]
        w = torch.softmax(torch.randn(k, generator=g), 0)
        items.append(BatchItem(torch.randn(1, H, generator=g).to(torch.bfloat16).to(dev), ids.to(dev), w.to(dev), r))
    outs = ExpertBatcher(pipe).batch_execute(items, 3)
    assert len(outs) == len(items)
    for it, o in zip(items, outs):
        assert o.shape == (1, H) and o.dtype == torch.bfloat16
        single = pipe.execute_layer_experts(it.hidden_states, 3, it.expert_indices.reshape(1, -1),
                                            it.routing_weights.reshape(1, -1))
        ref = _oracle(it.hidden_states.float().cpu().numpy(), it.expert_indices.cpu().numpy().reshape(1, -1),
                      it.routing_weights.float().cpu().numpy().reshape(1, -1), dense)
        assert_layer(o, ref)
        assert_layer(single, ref)
    assert pipe.execute_batched_experts([], 3) == []


def test_pipeline_batched_prefill_api(dev):
    from tinyserve_b200.pipeline import ExpertPipeline
    from tinyserve_b200.workloads import zipf_routing
    H, I, E, k, T = 512, 256, 8, 4, 200
    layer, dense, _ = _build_layer(dev, TSB_MXFP4, TSB_MXFP4, H, I, E, k, "interleaved", seed=9)
    pipe = ExpertPipeline([layer])
    ids, wts = zipf_routing(T, E, k, seed=3)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    out = pipe.execute_layer_experts_batched(x.to(dev), 0, ids.to(dev), wts.to(dev))
    ref = _oracle(x.float().numpy(), ids.numpy(), wts.numpy(), dense)
    assert_layer(out, ref)
    assert pipe.execute_layer_experts_batched(x[:0].to(dev), 0, ids[:0], wts[:0]).shape == (0, H)
    assert pipe.schedule_prefetch(0, [1, 2]) is None


def test_decode_inplace_matches_decode(dev):
    """QuantMoE.decode_ (caller-owned buffers, prepared arguments) gives the
    same routing and output as decode, with and without a router, T = 1 and 3."""
    H, I, E, k = 512, 256, 8, 2
    layer, _, _ = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, E, k, "separate", seed=13)
    for T in (1, 3):
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(T)).to(torch.bfloat16).to(dev)
        ref, ref_ids, ref_w = layer.decode(x)
        out = torch.empty_like(ref)
        ids = torch.empty_like(ref_ids)
        w = torch.empty_like(ref_w)
        layer.decode_(x, out, ids, w)
        torch.cuda.synchronize()
        assert torch.equal(ids, ref_ids) and torch.equal(w, ref_w) and torch.equal(out, ref)


def test_decode_session_graph_replays_match_decode(dev):
    """DecodeSession (one CUDA graph per token: host -> device -> layer ->
    host) returns what decode returns for each of a stream of tokens."""
    from tinyserve_b200.moe import DecodeSession
    H, I, E, k = 512, 256, 8, 2
    layer, _, _ = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, E, k, "separate", seed=17)
    sess = DecodeSession(layer, slots=3)
    xs = torch.randn(7, H, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    got = []
    pend = []
    for i in range(7):
        pend.append(sess.submit(xs[i]))
        if len(pend) == 3:
            got.append(sess.result(pend.pop(0)).clone())
    got += [sess.result(s).clone() for s in pend]
    for i in range(7):
        ref, _, _ = layer.decode(xs[i:i + 1].to(dev))
        assert torch.equal(got[i], ref.cpu()), i
