"""fp32 restatement of the reference expert math, router and combine
(test infrastructure).

- clamp-SwiGLU: ``tinyserve/expert_forward.py:185-187`` (gate = even columns of
  gate_up, clamped above at 7; up = odd columns clamped to [-7, 7];
  ``(up + 1) * gate * sigmoid(1.702 * gate)``), constant ``_QUICK_GELU_COEFF``
  at ``expert_forward.py:30``.  For separate gate/up projections (GGUF stores,
  ``ggml_forward.py:103-112``) the same formula is applied to the two outputs.
- SiLU gate: ``ggml_forward.py:112`` ``act(gate) * up``.
- router "topk then softmax": ``tinyserve/_model_hooks.py:466-473``.
- weighted combine ``out[tok] += w * expert(h)``: ``expert_pipeline.py:281,496``.

Everything is float64 internally and returned as float32: the tolerance of
the GPU path is measured against exact math on the dequantised weights.
"""
from __future__ import annotations

import numpy as np

LIMIT = 7.0
ALPHA = 1.702


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 precision (RNE), returned as float32."""
    from .dequant import bf16_bits_to_f32, f32_to_bf16_bits
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, dtype=np.float32)))


def swiglu_oai(gate: np.ndarray, up: np.ndarray, limit: float = LIMIT, alpha: float = ALPHA) -> np.ndarray:
    g = np.minimum(gate, limit)
    u = np.clip(up, -limit, limit)
    return (u + 1.0) * g * (1.0 / (1.0 + np.exp(-alpha * g)))


def silu_mul(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    return gate / (1.0 + np.exp(-gate)) * up


def expert_forward(h: np.ndarray, w_gate: np.ndarray, w_up: np.ndarray, w_down: np.ndarray,
                   activation: str = "swiglu_oai", b_gate=None, b_up=None, b_down=None) -> np.ndarray:
    """h [T, H]; w_gate, w_up [I, H]; w_down [H, I]  ->  [T, H] (float64 math)."""
    h = np.asarray(h, dtype=np.float64)
    g = h @ np.asarray(w_gate, dtype=np.float64).T
    u = h @ np.asarray(w_up, dtype=np.float64).T
    if b_gate is not None:
        g = g + b_gate
        u = u + b_up
    a = swiglu_oai(g, u) if activation == "swiglu_oai" else silu_mul(g, u)
    o = a @ np.asarray(w_down, dtype=np.float64).T
    if b_down is not None:
        o = o + b_down
    return o


def split_interleaved(w_gate_up: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """[2I, H] gate_up (row 2j = gate j, 2j+1 = up j; expert_forward.py:239-240)."""
    return w_gate_up[0::2], w_gate_up[1::2]


def router_topk_softmax(h: np.ndarray, w_router: np.ndarray, top_k: int, bias=None,
                        logits_bf16: bool = True):
    """logits = h @ W_r^T (bf16 Linear: fp32 accumulate, result rounded to bf16),
    topk, softmax over the k selected logits.  Ties break toward the lower
    expert id.  Returns (ids [T, k] int64, weights [T, k] float32, logits)."""
    lg = np.asarray(h, dtype=np.float64) @ np.asarray(w_router, dtype=np.float64).T
    if bias is not None:
        lg = lg + bias
    lg = lg.astype(np.float32)
    if logits_bf16:
        lg = bf16_round(lg)
    order = np.argsort(-lg.astype(np.float64), axis=1, kind="stable")[:, :top_k]
    top = np.take_along_axis(lg, order, axis=1).astype(np.float64)
    e = np.exp(top - top.max(axis=1, keepdims=True))
    w = (e / e.sum(axis=1, keepdims=True)).astype(np.float32)
    return order.astype(np.int64), w, lg


def moe_layer(h: np.ndarray, ids: np.ndarray, weights: np.ndarray, experts) -> np.ndarray:
    """out[t] = sum_k weights[t,k] * expert_{ids[t,k]}(h[t]).

    ``experts(e)`` returns (w_gate [I,H], w_up [I,H], w_down [H,I]) float arrays.
    Grouping by expert is how the reference batches prefill
    (expert_pipeline.py:166-239); the result is the same as the per-token sum.
    """
    h = np.asarray(h, dtype=np.float64)
    out = np.zeros_like(h)
    for e in np.unique(ids):
        tok, kk = np.nonzero(ids == e)
        wg, wu, wd = experts(int(e))
        y = expert_forward(h[tok], wg, wu, wd)
        out[tok] += weights[tok, kk][:, None] * y
    return out


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))
