"""Seeded synthetic workloads of the BASELINE configurations.

Config 1 ("decode_q4k"): one GPT-OSS-20B-shaped MoE layer -- hidden 2880,
expert intermediate 2880, 32 experts, router top-4 with softmax over the
top-4 logits, clamp-SwiGLU (limit 7.0, alpha 1.702); expert gate/up/down
drawn from N(0, 0.02) with a seed and quantised to GGUF Q4_K with the repo's
encoder; router weight bf16 N(0, 0.02); hidden states bf16 N(0, 1), a fresh
seeded vector per decode step.  Real checkpoints are not used (random init).
"""
from __future__ import annotations

import torch

from . import quantize as Q
from .formats import GGML_Q4_K, TSB_MXFP4

H20, I20, E20, K20 = 2880, 2880, 32, 4


def gen_normal(shape, seed: int, std: float, device) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(*shape, generator=g, device=device) * std


def layer_weights(fmt: int = GGML_Q4_K, *, hidden: int = H20, inter: int = I20, n_experts: int = E20,
                  seed: int = 0, device="cuda", layout: str | None = None):
    """The seeded expert weights and router of one layer as plain tensors
    (no library call): a list of per-expert dicts of uint8 block streams
    (GGUF formats: gate, up, down; MXFP4: gate = interleaved gate_up [2I, H]
    blocks, gate_scales, down, down_scales) and the bf16 router [E, H]."""
    device = torch.device(device)
    layout = layout or ("interleaved" if fmt == TSB_MXFP4 else "separate")
    experts = []
    for e in range(n_experts):
        s = seed * 100003 + 7 * e
        if fmt == TSB_MXFP4:
            gu = gen_normal((2 * inter, hidden), s, 0.02, device)
            gb, gs = Q.quantize_mxfp4(gu, 2 * inter, hidden)
            dn = gen_normal((hidden, inter), s + 2, 0.02, device)
            db, ds = Q.quantize_mxfp4(dn, hidden, inter)
            experts.append(dict(gate=gb.reshape(-1), down=db.reshape(-1), gate_scales=gs.reshape(-1),
                                down_scales=ds.reshape(-1)))
            del gu, dn
        else:
            g = Q.quantize(fmt, gen_normal((inter, hidden), s, 0.02, device))
            u = Q.quantize(fmt, gen_normal((inter, hidden), s + 1, 0.02, device))
            d = Q.quantize(fmt, gen_normal((hidden, inter), s + 2, 0.02, device))
            experts.append(dict(gate=g, up=u, down=d))
    router = gen_normal((n_experts, hidden), seed * 100003 + 99991, 0.02, device).to(torch.bfloat16)
    return experts, router, layout


def build_layer(fmt: int = GGML_Q4_K, *, hidden: int = H20, inter: int = I20, n_experts: int = E20,
                top_k: int = K20, seed: int = 0, device="cuda", layout: str | None = None,
                activation: str = "swiglu_oai", pack: bool | None = None):
    """One MoE layer with every expert HBM-resident.  GGUF formats use separate
    gate/up matrices (GGUF stores, mmap_store.py:86-91); MXFP4 uses the
    interleaved gate_up [2I, H] of the HF GPT-OSS checkpoint."""
    from .moe import ExpertWeights, QuantMoE
    experts, router, layout = layer_weights(fmt, hidden=hidden, inter=inter, n_experts=n_experts, seed=seed,
                                            device=device, layout=layout)
    return QuantMoE([ExpertWeights(**e) for e in experts], fmt_gate_up=fmt, fmt_down=fmt, hidden=hidden,
                    inter=inter, top_k=top_k, router_w=router, gate_up_layout=layout, activation=activation,
                    pack=pack)


def hidden_states(steps: int, hidden: int = H20, seed: int = 0, device="cuda") -> torch.Tensor:
    """bf16 [steps, hidden] N(0, 1); row t is the fresh vector of decode step t."""
    return gen_normal((steps, hidden), 10_000_019 + seed, 1.0, device).to(torch.bfloat16)


def layer_bytes(layer) -> tuple[int, int]:
    """(bytes of one expert's weights, router bytes)."""
    e = layer.experts[0]
    n = sum(t.numel() for t in (e.gate, e.up, e.down, e.gate_scales, e.up_scales, e.down_scales) if t is not None)
    r = layer.router_w.numel() * 2 if layer.router_w is not None else 0
    return n, r


def zipf_routing(T: int, n_experts: int = E20, top_k: int = K20, s: float = 1.1, seed: int = 0):
    """Config 4 routing: top_k distinct experts per token drawn without
    replacement with p_e proportional to (e + 1)^-s, routing weights the
    softmax of top_k seeded N(0, 1) logits.  Returns (ids int32 [T, k],
    weights fp32 [T, k]) on the CPU."""
    g = torch.Generator().manual_seed(seed)
    p = torch.arange(1, n_experts + 1, dtype=torch.float64).pow(-s)
    ids = torch.multinomial(p.expand(T, n_experts), top_k, replacement=False, generator=g).to(torch.int32)
    w = torch.softmax(torch.randn(T, top_k, generator=g), dim=1).to(torch.float32)
    return ids, w
