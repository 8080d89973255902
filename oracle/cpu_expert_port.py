"""The reference's CPU expert path, restated for timing on the GPU box's host
cores (test / baseline infrastructure, never the product).

Restates ``tinyserve/cpu_expert.py`` ``CPUExpertForward`` (fused variant,
``cpu_expert.py:283-300``): ``F.linear`` (oneDNN) on dequantised fp32 weights,
gate_up interleaved rows with clamp-SwiGLU(7.0, 1.702), then ``F.linear`` for
down; plus the router of ``tinyserve/_model_hooks.py:466-473`` (bf16 Linear,
topk, softmax over the k logits) and the weighted combine of
``expert_pipeline.py:281``.  Weights are decoded once per expert with the
oracle's restatement of ``dequant_tensor`` and cached, as the baseline plan
prescribes (the reference caches its CPU-side conversions by data pointer,
``cpu_expert.py:158-160``).
"""
from __future__ import annotations

import time

import numpy as np
import torch
import torch.nn.functional as F

from . import dequant as OD

QUICK_GELU = 1.702


class CPUMoELayer:
    def __init__(self, fetch_expert, router_w_bf16: torch.Tensor, top_k: int, num_threads: int):
        """fetch_expert(e) -> (gate_up fp32 [2I, H] interleaved, down fp32 [H, I])."""
        self._fetch = fetch_expert
        self._cache: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        self.router_w = router_w_bf16
        self.top_k = top_k
        self.num_threads = num_threads

    def prefetch(self, experts) -> None:
        """Decode the given experts now, so timed tokens only run the math."""
        for e in experts:
            self._expert(int(e))

    def _expert(self, e: int):
        if e not in self._cache:
            self._cache[e] = self._fetch(e)
        return self._cache[e]

    def route(self, h: torch.Tensor):
        logits = F.linear(h, self.router_w)
        top_vals, top_idx = torch.topk(logits, self.top_k, dim=-1)
        return top_idx, F.softmax(top_vals.float(), dim=-1)

    def forward(self, h_bf16: torch.Tensor) -> torch.Tensor:
        ids, w = self.route(h_bf16)
        h = h_bf16.float()
        out = torch.zeros_like(h)
        for k in range(self.top_k):
            wgu, wdn = self._expert(int(ids[0, k]))
            gate_up = F.linear(h, wgu)
            gate = gate_up[..., ::2].clamp(max=7.0)
            up = gate_up[..., 1::2].clamp(min=-7.0, max=7.0)
            gated = (up + 1) * gate * torch.sigmoid(gate * QUICK_GELU)
            out += w[0, k] * F.linear(gated, wdn)
        return out


def gguf_expert_fetcher(host_bytes, fmt_gu: int, fmt_dn: int, H: int, I: int):
    """host_bytes(e) -> (gate bytes, up bytes, down bytes) numpy uint8 streams."""
    def fetch(e):
        g, u, d = host_bytes(e)
        wg = OD.dequant_tensor(g, fmt_gu, (I, H))
        wu = OD.dequant_tensor(u, fmt_gu, (I, H))
        wgu = np.empty((2 * I, H), np.float32)
        wgu[0::2], wgu[1::2] = wg, wu
        return torch.from_numpy(wgu), torch.from_numpy(OD.dequant_tensor(d, fmt_dn, (H, I)))
    return fetch


def time_tokens(layer: CPUMoELayer, xs: torch.Tensor, warmup: int = 2) -> float:
    """Median seconds per token over the rows of xs (bf16 [n, H]) after warm-up."""
    torch.set_num_threads(layer.num_threads)
    for i in range(min(warmup, xs.shape[0])):
        layer.forward(xs[i:i + 1])
    ts = []
    for i in range(xs.shape[0]):
        t0 = time.perf_counter()
        layer.forward(xs[i:i + 1])
        ts.append(time.perf_counter() - t0)
    return float(np.median(ts))
