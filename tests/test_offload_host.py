"""load_and_offload keeps the reference's call shape
(tinyserve/offload.py:689-710) and resolves model ids without a network."""
from __future__ import annotations

import inspect

import pytest


def test_signature_matches_reference():
    from tinyserve_b200.offload import load_and_offload
    params = list(inspect.signature(load_and_offload).parameters.values())
    assert [p.name for p in params[:4]] == ["model_id", "device", "offload_config", "cache_capacity"]
    assert params[1].default == "cuda" and params[2].default is None and params[3].default == 0
    assert params[-1].kind is inspect.Parameter.VAR_KEYWORD


def test_presets_and_overrides():
    from tinyserve_b200.offload import _config
    c20 = _config("openai/gpt-oss-20b", {})
    assert (c20.num_hidden_layers, c20.num_local_experts, c20.hidden_size, c20.num_experts_per_tok) == (24, 32, 2880, 4)
    c120 = _config("gpt-oss-120b", {"num_hidden_layers": 2})
    assert (c120.num_hidden_layers, c120.num_local_experts) == (2, 128)
    with pytest.raises(ValueError, match="unknown model"):
        _config("some/other-model", {})


def test_cpu_device_refused():
    from tinyserve_b200.offload import load_and_offload
    with pytest.raises(ValueError, match="CUDA"):
        load_and_offload("gpt-oss-20b", device="cpu", num_hidden_layers=1)
