"""Layer-level execution API of the reference, for HBM-resident experts.

Mirrors the calls tinyserve's model hooks make on its expert pipeline and
batcher, with the same argument meaning and return values:

- ``ExpertPipeline.execute_layer_experts(hidden_states [T,H], layer_idx,
  expert_indices [T,k], routing_weights [T,k]) -> [T,H]``
  (tinyserve/expert_pipeline.py:140-164): the per-token path; here one C-ABI
  call per layer (T = 1 fused decode kernels, T > 1 grouped).
- ``ExpertPipeline.execute_layer_experts_batched(...)`` (same signature,
  expert_pipeline.py:166-239): prefill, tokens grouped by expert; here the
  grouping, both GEMMs and the weighted scatter run on the GPU in one call.
- ``ExpertPipeline.execute_batched_experts(items, layer_idx)`` and
  ``ExpertBatcher(pipeline).batch_execute(items, layer_idx) -> list[[1,H]]``
  with ``BatchItem(hidden_states [1,H], expert_indices [k], routing_weights [k],
  request_idx)`` (tinyserve/expert_batcher.py:17-85): several requests decoding
  together; their tokens go through the layer as one batch so each routed
  expert is read once.
- ``schedule_prefetch`` is accepted and does nothing: every expert already
  lives in HBM (the reference's offload tiers, caches and transfer streams are
  not part of this path).

Outputs are in the hidden states' dtype (bf16).  Accumulation over a token's
experts is in fp32 in slot order (the reference adds in bf16 in first-seen
expert order), so results agree within rounding.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .moe import QuantMoE


@dataclass
class BatchItem:
    hidden_states: torch.Tensor    # [1, hidden_dim]
    expert_indices: torch.Tensor   # [top_k]
    routing_weights: torch.Tensor  # [top_k]
    request_idx: int


class ExpertPipeline:
    """Expert execution for the layers of a model whose experts are HBM-resident.

    ``layers`` maps a layer index to its :class:`QuantMoE` (a list is indexed
    by position)."""

    def __init__(self, layers: dict[int, QuantMoE] | list[QuantMoE]):
        self.layers = dict(enumerate(layers)) if isinstance(layers, list) else dict(layers)

    def _layer(self, layer_idx: int) -> QuantMoE:
        try:
            return self.layers[layer_idx]
        except KeyError:
            raise KeyError(f"no MoE layer {layer_idx}") from None

    def _run(self, hidden_states, layer_idx, expert_indices, routing_weights):
        layer = self._layer(layer_idx)
        T = hidden_states.shape[0]
        if T == 0:
            return hidden_states.clone()
        x = hidden_states.to(torch.bfloat16).contiguous()
        ids = expert_indices.reshape(T, -1)
        wts = routing_weights.reshape(T, -1)
        out, _, _ = layer.decode(x, ids=ids, weights=wts)
        return out.to(hidden_states.dtype)

    def execute_layer_experts(self, hidden_states: torch.Tensor, layer_idx: int, expert_indices: torch.Tensor,
                              routing_weights: torch.Tensor) -> torch.Tensor:
        return self._run(hidden_states, layer_idx, expert_indices, routing_weights)

    def execute_layer_experts_batched(self, hidden_states: torch.Tensor, layer_idx: int,
                                      expert_indices: torch.Tensor, routing_weights: torch.Tensor) -> torch.Tensor:
        layer = self._layer(layer_idx)
        T = hidden_states.shape[0]
        if T == 0:
            return hidden_states.clone()
        out, _, _ = layer.prefill(hidden_states.to(torch.bfloat16).contiguous(),
                                  ids=expert_indices.reshape(T, -1), weights=routing_weights.reshape(T, -1))
        return out.to(hidden_states.dtype)

    def execute_batched_experts(self, items: list[BatchItem], layer_idx: int) -> list[torch.Tensor]:
        return ExpertBatcher(self).batch_execute(items, layer_idx)

    def schedule_prefetch(self, layer_idx: int, expert_ids) -> None:
        """Experts are HBM-resident: nothing to prefetch."""
        return None


class ExpertBatcher:
    """Batches expert forwards across concurrent requests
    (tinyserve/expert_batcher.py:25-85)."""

    def __init__(self, pipeline: ExpertPipeline):
        self._pipeline = pipeline

    def batch_execute(self, items: list[BatchItem], layer_idx: int) -> list[torch.Tensor]:
        if not items:
            return []
        h = torch.cat([it.hidden_states.reshape(1, -1) for it in items], dim=0)
        ids = torch.stack([it.expert_indices.reshape(-1) for it in items])
        wts = torch.stack([it.routing_weights.reshape(-1) for it in items])
        out = self._pipeline._run(h, layer_idx, ids, wts)
        return [out[i:i + 1] for i in range(len(items))]
