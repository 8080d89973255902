"""TensorLayout offsets and sizes follow the reference's packing rule
(tinyserve/expert_store.py:57-77): insertion order, back to back, no padding."""
from __future__ import annotations

import torch

from tinyserve_b200.expert_forward import TensorLayout


def test_layout_offsets_in_insertion_order():
    L = TensorLayout({"gate_up_proj": ((5760, 90, 16), torch.uint8), "gate_up_proj_scales": ((5760, 90), torch.uint8),
                      "gate_up_proj_bias": ((5760,), torch.bfloat16), "down_proj": ((2880, 90, 16), torch.uint8)})
    assert L.offsets["gate_up_proj"] == 0
    assert L.offsets["gate_up_proj_scales"] == 8_294_400  # the reference's GPT-OSS-20B offset
    assert L.sizes["gate_up_proj_scales"] == 518_400
    assert L.offsets["gate_up_proj_bias"] == 8_812_800
    assert L.offsets["down_proj"] == 8_812_800 + 11_520
    assert L.total_bytes == L.offsets["down_proj"] + 4_147_200


def test_layout_from_tensors_and_view():
    t = {"a": torch.zeros(3, 4, dtype=torch.float32), "b": torch.zeros(5, dtype=torch.uint8)}
    L = TensorLayout.from_tensors(t)
    packed = torch.arange(L.total_bytes, dtype=torch.int64).to(torch.uint8)
    assert L.view(packed, "b").tolist() == list(range(48, 53))
