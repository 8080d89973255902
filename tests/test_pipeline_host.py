"""Host logic of the layer-API mirrors (tinyserve_b200.pipeline) on CPU, with a
stand-in layer: stacking of BatchItems, reshaping of routing tensors, per-item
split and dtype handling (tinyserve/expert_batcher.py:31-85 semantics)."""
from __future__ import annotations

import torch

from tinyserve_b200.pipeline import BatchItem, ExpertBatcher, ExpertPipeline


class _FakeLayer:
    """out[t] = sum_j w[t,j] * (ids[t,j] + 1) * x[t]  (a linear stand-in)."""

    def __init__(self):
        self.calls = []

    @staticmethod
    def _apply(x, ids, weights):
        scale = (weights.float() * (ids.float() + 1)).sum(1, keepdim=True)
        return (x.float() * scale).to(torch.bfloat16), ids, weights

    def decode(self, x, ids=None, weights=None, out=None):
        self.calls.append(("decode", tuple(x.shape), tuple(ids.shape)))
        return self._apply(x, ids, weights)

    def prefill(self, x, ids=None, weights=None, out=None):
        self.calls.append(("prefill", tuple(x.shape), tuple(ids.shape)))
        return self._apply(x, ids, weights)


def test_batcher_stacks_and_splits():
    layer = _FakeLayer()
    pipe = ExpertPipeline({5: layer})
    items = [BatchItem(torch.full((1, 4), float(r + 1)), torch.tensor([r % 3, 2]), torch.tensor([0.25, 0.75]), r)
             for r in range(3)]
    outs = ExpertBatcher(pipe).batch_execute(items, 5)
    assert layer.calls == [("decode", (3, 4), (3, 2))]
    for r, o in enumerate(outs):
        s = 0.25 * (r % 3 + 1) + 0.75 * 3
        assert o.shape == (1, 4)
        assert torch.allclose(o.float(), torch.full((1, 4), (r + 1) * s), rtol=1e-2)


def test_pipeline_routes_batched_to_prefill_and_keeps_dtype():
    layer = _FakeLayer()
    pipe = ExpertPipeline([layer])
    x = torch.ones(6, 4, dtype=torch.float32)
    ids = torch.zeros(6, 2, dtype=torch.int64)
    w = torch.full((6, 2), 0.5)
    out = pipe.execute_layer_experts_batched(x, 0, ids, w)
    assert layer.calls[-1][0] == "prefill" and out.dtype == torch.float32
    out = pipe.execute_layer_experts(x[:1], 0, ids[:1], w[:1])
    assert layer.calls[-1] == ("decode", (1, 4), (1, 2))
    assert ExpertBatcher(pipe).batch_execute([], 0) == []
    try:
        pipe.execute_layer_experts(x, 7, ids, w)
    except KeyError as e:
        assert "7" in str(e)
    else:
        raise AssertionError("missing layer must raise")
