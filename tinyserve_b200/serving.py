"""Several requests served at once over the shared HBM-resident expert layers.

The reference serves concurrent requests by interleaving them one decode
step at a time under a GPU lock, each request running the whole model alone
(tinyserve/server.py:48-150).  Here the active requests decode in lockstep:
one step runs every active request's token through each layer together --
the attention projections and the LM head as one GEMM over the batch, the
decode-attention kernel over all rows (each with its own cache slot and
position), and the expert layer as one call with T = batch, which reads each
routed expert once for all the tokens routed to it (the grouped path above 16
tokens, ExpertBatcher's job in the reference, tinyserve/expert_batcher.py).

Requests wait in a queue until a cache slot frees (continuous batching); a
newly admitted request is prefilled into its slot and its first token comes
from the prefill.  Greedy decoding; a request ends after ``max_new_tokens``
or at ``eos_token_id``.
"""
from __future__ import annotations

import itertools
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import _lib
from .gptoss import GptOssDecoder


@dataclass
class Request:
    request_id: int
    prompt: torch.Tensor
    max_new_tokens: int
    generated: list[int] = field(default_factory=list)
    logits: list[torch.Tensor] = field(default_factory=list)  # per emitted token, when kept
    slot: int = -1
    pos: int = 0  # position of the next token to feed

    @property
    def done(self) -> bool:
        return len(self.generated) >= self.max_new_tokens


class ServingEngine:
    """Continuous-batching greedy decode of a GPT-OSS model whose MoE blocks
    are QuantMoE layers.  ``max_batch`` cache slots of ``max_seq`` tokens
    each; ``keep_logits`` stores every emitted token's logits (tests)."""

    def __init__(self, model, moe_layers, max_batch: int = 64, max_seq: int = 4096,
                 kv_dtype: torch.dtype = torch.float8_e4m3fn, prefill_chunk: int = 1024,
                 eos_token_id: int | None = None, keep_logits: bool = False):
        self.dec = GptOssDecoder(model, moe_layers, max_seq=1, kv_dtype=kv_dtype, prefill_chunk=prefill_chunk)
        d = self.dec
        # RoPE tables for the full context (the helper decoder was built with a 1-token cache)
        rot = model.model.rotary_emb
        p = torch.arange(max_seq, device=d.device, dtype=torch.float32)
        freqs = p[:, None] * rot.inv_freq.float().to(d.device)[None, :]
        d.cos = (freqs.cos() * rot.attention_scaling).to(torch.bfloat16)
        d.sin = (freqs.sin() * rot.attention_scaling).to(torch.bfloat16)
        d.max_seq = max_seq
        d._j = torch.arange(max_seq, device=d.device)
        self.max_batch, self.max_seq = max_batch, max_seq
        self.kv_dtype = kv_dtype
        self.k = torch.zeros(d.L, max_batch, d.nkv, max_seq, d.D, dtype=kv_dtype, device=d.device)
        self.v = torch.zeros_like(self.k)
        self.slot_stride = d.nkv * max_seq * d.D
        nws = _lib.lib().tsb_gqa_decode_batch_workspace(d.nq, d.nkv, max_seq, max_batch)
        self._aws = torch.zeros(nws, dtype=torch.uint8, device=d.device)
        self.eos = eos_token_id
        self.keep_logits = keep_logits
        self._ids = itertools.count()
        self.waiting: list[Request] = []
        self.running: list[Request] = []
        self.finished: dict[int, Request] = {}
        self._free = list(range(max_batch - 1, -1, -1))

    def submit(self, prompt: torch.Tensor, max_new_tokens: int) -> int:
        prompt = prompt.reshape(-1)
        if prompt.numel() + max_new_tokens > self.max_seq:
            raise ValueError("prompt + max_new_tokens exceeds the per-request cache")
        r = Request(next(self._ids), prompt, max_new_tokens)
        self.waiting.append(r)
        return r.request_id

    def _emit(self, r: Request, tok: int, logits: torch.Tensor | None) -> None:
        r.generated.append(tok)
        if self.keep_logits and logits is not None:
            r.logits.append(logits.float().cpu())
        if r.done or (self.eos is not None and tok == self.eos):
            r.max_new_tokens = len(r.generated)

    @torch.no_grad()
    def _admit(self) -> None:
        while self.waiting and self._free:
            r = self.waiting.pop(0)
            r.slot = self._free.pop()
            logits = self.dec.prefill(r.prompt.to(self.dec.device), self.k[:, r.slot], self.v[:, r.slot])
            r.pos = r.prompt.numel()
            self._emit(r, int(logits.argmax()), logits)
            self.running.append(r)

    def _retire(self) -> None:
        keep = []
        for r in self.running:
            if r.done:
                self._free.append(r.slot)
                self.finished[r.request_id] = r
            else:
                keep.append(r)
        self.running = keep

    @torch.no_grad()
    def _decode(self, batch: list[Request]) -> None:
        d = self.dec
        dev = d.device
        L = _lib.lib()
        stream = torch.cuda.current_stream(dev).cuda_stream
        B = len(batch)
        tok = torch.tensor([r.generated[-1] for r in batch], dtype=torch.long).to(dev)
        pos = torch.tensor([r.pos for r in batch], dtype=torch.int64).to(dev)
        slots = torch.tensor([r.slot for r in batch], dtype=torch.int32).to(dev)
        x = d.embed.index_select(0, tok).float()
        h = torch.empty(B, d.H, dtype=torch.bfloat16, device=dev)
        a = torch.empty(B, d.nq * d.D, dtype=torch.bfloat16, device=dev)
        y = torch.empty(B, d.H, dtype=torch.float32, device=dev)
        d._norm(x, None, d.layers[0]["ln1"], h)
        fp8 = 1 if self.kv_dtype == torch.float8_e4m3fn else 0
        for li, lay in enumerate(d.layers):
            qkv = F.linear(h, lay["wqkv"], lay["bqkv"])
            _lib.check(L.tsb_gqa_decode_attention_batch(
                qkv.data_ptr(), d.nq, d.nkv, d.D, d.cos.data_ptr(), d.sin.data_ptr(), pos.data_ptr(),
                slots.data_ptr(), self.slot_stride, self.k[li].data_ptr(), self.v[li].data_ptr(), fp8, self.max_seq,
                d.window if d.sliding[li] else 0, lay["sinks"].data_ptr(), d.scale, a.data_ptr(), B,
                self._aws.data_ptr(), self._aws.numel(), stream))
            d._norm(x, F.linear(a, lay["wo"], lay["bo"]), lay["ln2"], h)
            lay["moe"].decode(h, out=y)
            d._norm(x, y, d._next_norm(li), h)
        logits = F.linear(h, d.lm_head)
        nxt = logits.argmax(-1).tolist()
        for i, r in enumerate(batch):
            r.pos += 1
            self._emit(r, nxt[i], logits[i])

    def step(self) -> int:
        """Admit waiting requests into free slots (prefill), run one batched
        decode step for every running request, retire finished ones; returns
        the number of requests that decoded a token in this step."""
        self._admit()
        self._retire()
        batch = [r for r in self.running if not r.done]
        if batch:
            self._decode(batch)
        self._retire()
        return len(batch)

    def run(self) -> dict[int, list[int]]:
        """Serve until every submitted request has finished; returns
        {request id: generated token ids}."""
        while self.waiting or self.running:
            self.step()
        return {i: r.generated for i, r in sorted(self.finished.items())}
