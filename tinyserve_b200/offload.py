"""One-call model entry point: ``load_and_offload`` with the reference's
signature (tinyserve/offload.py:689-710), for GPT-OSS models whose experts all
live in HBM.

The reference loads a checkpoint, moves the experts to a host/disk store and
installs a cache-and-fetch MoE forward on every layer.  On a B200 the experts
of GPT-OSS-20B (12 GB of MXFP4) and -120B (61 GB) fit in HBM, so this entry
point keeps the reference's call shape but builds every MoE block as a
:class:`tinyserve_b200.moe.QuantMoE` (MXFP4 experts, decode-packed, router
inside the decode launch).  There are no offload tiers: ``offload_config`` and
``cache_capacity`` are accepted and recorded but do not change anything.

Weights: this build has no checkpoint access, so the model is built from its
configuration with seeded random weights (``seed``), and the expert weights
are quantised to MXFP4 with the repository's encoder.  ``model_id`` is one of
the preset names in :data:`PRESETS`, a ``transformers.GptOssConfig``, or a
local directory holding a ``config.json``.
"""
from __future__ import annotations

import dataclasses
import os
from typing import Any

import torch

from .formats import TSB_MXFP4

# Shapes of the two published GPT-OSS models (hidden 2880, expert width 2880,
# top-4 routing, clamp-SwiGLU limit 7.0).
PRESETS: dict[str, dict[str, Any]] = {
    "openai/gpt-oss-20b": dict(num_hidden_layers=24, num_local_experts=32),
    "openai/gpt-oss-120b": dict(num_hidden_layers=36, num_local_experts=128),
}
PRESETS["gpt-oss-20b"] = PRESETS["openai/gpt-oss-20b"]
PRESETS["gpt-oss-120b"] = PRESETS["openai/gpt-oss-120b"]


@dataclasses.dataclass
class TinyserveConfig:
    """What the reference's TinyserveConfig (tinyserve/offload.py:44-68)
    controls that applies here: the expert format and whether decode uses the
    packed copy.  Offload-tier fields of a caller's config are kept in
    ``extra`` and otherwise ignored (every expert is HBM-resident)."""

    expert_format: int = TSB_MXFP4
    pack: bool | None = None
    extra: dict = dataclasses.field(default_factory=dict)


class OffloadedLM(torch.nn.Module):
    """The model with its MoE blocks replaced: ``forward`` / ``generate`` are
    the wrapped Hugging Face model's; ``moe_layers`` lists the QuantMoE of each
    decoder layer (tinyserve/offload.py:71-113 is the reference's wrapper)."""

    def __init__(self, model: torch.nn.Module, moe_layers: list, config: TinyserveConfig, cache_capacity: int):
        super().__init__()
        self.model = model
        self.moe_layers = moe_layers
        self.tinyserve_config = config
        self.cache_capacity = cache_capacity

    @property
    def config(self):
        return self.model.config

    @property
    def device(self):
        return next(self.model.parameters()).device

    def forward(self, *args, **kwargs):
        return self.model(*args, **kwargs)

    @torch.no_grad()
    def generate(self, *args, **kwargs):
        return self.model.generate(*args, **kwargs)


def _config(model_id, hf_kwargs: dict):
    from transformers import GptOssConfig
    if isinstance(model_id, GptOssConfig):
        cfg = model_id
        for k, v in hf_kwargs.items():
            setattr(cfg, k, v)
        return cfg
    if isinstance(model_id, str) and model_id in PRESETS:
        return GptOssConfig(**{**PRESETS[model_id], **hf_kwargs})
    if isinstance(model_id, (str, os.PathLike)) and os.path.isdir(model_id):
        return GptOssConfig.from_pretrained(model_id, local_files_only=True, **hf_kwargs)
    raise ValueError(f"unknown model {model_id!r}: pass one of {sorted(PRESETS)}, a GptOssConfig or a local "
                     "directory with config.json (no checkpoint download in this build)")


def quant_moe_from_mlp(mlp, fmt: int = TSB_MXFP4, pack: bool | None = None):
    """A QuantMoE equal to a Hugging Face ``GptOssMLP`` (router + experts):
    expert e's gate_up_proj[e] ([H, 2I], gate/up interleaved by column) and
    down_proj[e] ([I, H]) become MXFP4 [2I, H] (interleaved rows) and [H, I],
    their biases the gate / up / down biases, the router weight bf16 and its
    bias fp32 (routing as GptOssTopKRouter: top-k of the logits, softmax over
    the k)."""
    from . import quantize as Q
    from .moe import ExpertWeights, QuantMoE
    ex = mlp.experts
    E = ex.gate_up_proj.shape[0]
    H = ex.gate_up_proj.shape[1]
    I2 = ex.gate_up_proj.shape[2]
    experts = []
    for e in range(E):
        gu = ex.gate_up_proj[e].detach().t().float().contiguous()  # [2I, H], row 2j gate j, 2j+1 up j
        dn = ex.down_proj[e].detach().t().float().contiguous()  # [H, I]
        gb, gs = Q.quantize_mxfp4(gu, I2, H)
        db, ds = Q.quantize_mxfp4(dn, H, I2 // 2)
        b = ex.gate_up_proj_bias[e].detach().float()
        experts.append(ExpertWeights(gate=gb.reshape(-1), down=db.reshape(-1), gate_scales=gs.reshape(-1),
                                     down_scales=ds.reshape(-1), gate_bias=b[0::2].contiguous(),
                                     up_bias=b[1::2].contiguous(),
                                     down_bias=ex.down_proj_bias[e].detach().float().contiguous()))
    r = mlp.router
    return QuantMoE(experts, fmt_gate_up=fmt, fmt_down=fmt, hidden=H, inter=I2 // 2, top_k=r.top_k,
                    router_w=r.weight.detach().to(torch.bfloat16), router_b=r.bias.detach().float(),
                    gate_up_layout="interleaved", activation="swiglu_oai", limit=float(getattr(ex, "limit", 7.0)),
                    alpha=float(getattr(ex, "alpha", 1.702)), pack=pack)


def _install(mlp, layer) -> None:
    """Route the block's forward through the QuantMoE (same return shape as
    GptOssMLP.forward: (hidden_states, router_scores)); the dense expert
    tensors are released."""
    def forward(hidden_states):
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1])
        dt = x.dtype
        out, _, w = layer.decode(x.to(torch.bfloat16).contiguous())
        return out.to(dt).reshape(shape), w.to(dt)

    mlp.forward = forward
    mlp.experts = None
    mlp.tinyserve_moe = layer


def offload_model(model, config: TinyserveConfig | None = None) -> list:
    """Replace every GptOssMLP of ``model`` (already on its GPU) by a QuantMoE;
    returns them in layer order (tinyserve/offload.py:397-686 is the
    reference's counterpart)."""
    config = config or TinyserveConfig()
    layers = []
    for block in model.model.layers:
        q = quant_moe_from_mlp(block.mlp, config.expert_format, config.pack)
        _install(block.mlp, q)
        layers.append(q)
        torch.cuda.empty_cache()
    return layers


def load_and_offload(model_id, device: str = "cuda", offload_config: TinyserveConfig | dict | None = None,
                     cache_capacity: int = 0, *, seed: int = 0, dtype: torch.dtype = torch.bfloat16,
                     **hf_kwargs) -> OffloadedLM:
    """Build the GPT-OSS model ``model_id`` on ``device`` with seeded random
    weights (``dtype`` for the dense parts) and every MoE block on the B200
    expert path.  Same positional parameters as the reference's entry point
    (tinyserve/offload.py:689-710); ``hf_kwargs`` override configuration
    fields (e.g. ``num_hidden_layers``)."""
    from transformers import GptOssForCausalLM
    cfg = _config(model_id, hf_kwargs)
    if isinstance(offload_config, dict):
        known = {f.name for f in dataclasses.fields(TinyserveConfig)} - {"extra"}
        ts = TinyserveConfig(**{k: v for k, v in offload_config.items() if k in known},
                             extra={k: v for k, v in offload_config.items() if k not in known})
    else:
        ts = offload_config or TinyserveConfig()
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("the B200 expert path needs a CUDA device")
    torch.manual_seed(seed)
    with dev:
        model = GptOssForCausalLM(cfg).to(dtype)
    model.eval()
    layers = offload_model(model, ts)
    return OffloadedLM(model, layers, ts, cache_capacity)
