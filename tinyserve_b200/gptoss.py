"""Whole-model GPT-OSS decode around the HBM-resident expert layers.

The caller side of the expert path for BASELINE config 3 (GPT-OSS-20B, batch
1, context 4096, FP8 KV cache): the reference decodes through Hugging Face's
model with its ``StaticKVCache`` (tinyserve/static_kv_cache.py:28-147, keys
and values stored as float8 e4m3 and read back as bf16) and its decode loop
(tinyserve/offload.py:219-287).  Here the same arithmetic runs as one
CUDA-graph replay per token:

  embedding -> per layer [RMSNorm -> fused q|k|v projection -> RoPE (the
  model's YaRN tables) -> K/V written to the FP8 cache at the position ->
  attention with the per-head sink logit over the cached positions (full, or
  the last ``sliding_window`` for sliding layers) -> o projection ->
  residual -> RMSNorm -> QuantMoE (one decode-packed launch) -> residual] ->
  RMSNorm -> LM head -> argmax.

The attention projections (bf16 GEMVs with the RMSNorm and residual steps
fused in), attention (RoPE, cache
store, sink softmax over the FP8 cache), the residual + RMSNorm steps and the
expert layers are the library's own kernels; the residual stream is kept in
fp32; the LM head is a cuBLAS GEMV.  Prompt prefill runs the same layers over chunks of
tokens (grouped expert GEMMs, causal attention over the cache).

Positions and the token id live in device buffers, so the captured graph is
replayed unchanged for every step.
"""
from __future__ import annotations

import os

import torch
import torch.nn.functional as F

from . import _lib


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [..., T, D] with the halves rotated (the GPT-OSS convention); cos/sin [T, D/2]."""
    a, b = x.chunk(2, dim=-1)
    return torch.cat((a * cos - b * sin, b * cos + a * sin), dim=-1)


class GptOssDecoder:
    """Batch-1 greedy decoder for a GPT-OSS model whose MoE blocks are
    QuantMoE layers (``load_and_offload``).

    model      the Hugging Face GptOssForCausalLM (dense weights are read from it
               once and re-laid out: q|k|v fused per layer)
    moe_layers one QuantMoE per decoder layer
    max_seq    KV-cache capacity in tokens
    kv_dtype   cache storage type: float8_e4m3fn (the reference's default) or bfloat16
    """

    def __init__(self, model, moe_layers, max_seq: int = 8192, kv_dtype: torch.dtype = torch.float8_e4m3fn,
                 prefill_chunk: int = 1024):
        cfg = model.config
        self.cfg = cfg
        m = model.model
        dev = m.embed_tokens.weight.device
        self.device = dev
        self.L = cfg.num_hidden_layers
        self.H = cfg.hidden_size
        self.nq, self.nkv = cfg.num_attention_heads, cfg.num_key_value_heads
        self.D = getattr(cfg, "head_dim", self.H // self.nq)
        self.eps = cfg.rms_norm_eps
        self.window = cfg.sliding_window
        self.sliding = [t == "sliding_attention" for t in cfg.layer_types[:self.L]]
        self.scale = self.D ** -0.5
        self.max_seq = max_seq
        self.chunk = prefill_chunk
        bf = torch.bfloat16
        with torch.no_grad():
            self.embed = m.embed_tokens.weight.detach().to(bf)
            self.lm_head = model.lm_head.weight.detach().to(bf)
            self.norm_w = m.norm.weight.detach().float()
            self.layers = []
            for i, blk in enumerate(m.layers):
                a = blk.self_attn
                wqkv = torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight]).detach().to(bf).contiguous()
                bqkv = None
                if a.q_proj.bias is not None:
                    bqkv = torch.cat([a.q_proj.bias, a.k_proj.bias, a.v_proj.bias]).detach().to(bf)
                self.layers.append(dict(
                    ln1=blk.input_layernorm.weight.detach().float(), ln2=blk.post_attention_layernorm.weight.detach().float(),
                    wqkv=wqkv, bqkv=bqkv, wo=a.o_proj.weight.detach().to(bf).contiguous(),
                    bo=None if a.o_proj.bias is None else a.o_proj.bias.detach().to(bf),
                    sinks=a.sinks.detach().float(), moe=moe_layers[i]))
            rot = m.rotary_emb
            pos = torch.arange(max_seq, device=dev, dtype=torch.float32)
            freqs = pos[:, None] * rot.inv_freq.float().to(dev)[None, :]
            self.cos = (freqs.cos() * rot.attention_scaling).to(bf)
            self.sin = (freqs.sin() * rot.attention_scaling).to(bf)
        self.kv_dtype = kv_dtype
        self.k_cache = torch.zeros(self.L, self.nkv, max_seq, self.D, dtype=kv_dtype, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.length = 0
        self._graph = None
        # RMSNorm + q|k|v + attention as one clustered launch (opt-in,
        # TSB_DECODE_FUSED=1; None: decided by the first step).  Measured on the
        # GPT-OSS-20B step it is slower than the two launches (30.6 us vs
        # 11.7 + 16.0 us per layer: its projection runs on one cluster of SMs
        # per KV head instead of the whole GPU), so two launches are the default.
        self._fused = None if os.environ.get("TSB_DECODE_FUSED", "0") == "1" else False
        self._tok = torch.zeros(1, dtype=torch.long, device=dev)
        self._pos = torch.zeros(1, dtype=torch.long, device=dev)
        self._next = torch.zeros(1, dtype=torch.long, device=dev)
        self._logits = None
        self._j = torch.arange(max_seq, device=dev)
        # decode-step buffers (fixed addresses for the captured graph)
        self._xe = torch.zeros(1, self.H, dtype=torch.float32, device=dev)     # embedding row
        self._xa = torch.zeros(1, self.H, dtype=torch.float32, device=dev)     # residual stream, two buffers
        self._xb = torch.zeros(1, self.H, dtype=torch.float32, device=dev)
        self._cnt = torch.zeros(1, dtype=torch.int32, device=dev)
        self._h = torch.zeros(1, self.H, dtype=torch.bfloat16, device=dev)     # normed sublayer input
        self._y = torch.zeros(1, self.H, dtype=torch.float32, device=dev)      # expert layer output
        self._a = torch.zeros(1, self.nq * self.D, dtype=torch.bfloat16, device=dev)
        self._qkv = torch.zeros(1, (self.nq + 2 * self.nkv) * self.D, dtype=torch.bfloat16, device=dev)
        nws = _lib.lib().tsb_gqa_decode_workspace(self.nq, self.nkv, max_seq)
        if nws == 0:
            raise ValueError("unsupported attention shape")
        self._aws = torch.zeros(nws, dtype=torch.uint8, device=dev)

    @staticmethod
    def _bytes(t: torch.Tensor) -> torch.Tensor:
        return t.view(torch.uint8) if t.element_size() == 1 else t

    @property
    def kv_bytes(self) -> int:
        return 2 * self.k_cache.numel() * self.k_cache.element_size()

    # ------------------------------------------------------------------ layers
    def _attn(self, li: int, q: torch.Tensor, pos0: int, T: int, ctx: int, kc: torch.Tensor, vc: torch.Tensor):
        """Prompt attention: q [nq, T, D] (roped) for positions pos0..pos0+T-1
        against the layer's cached keys kc / vc [nkv, S, D] at [0, ctx); returns
        [T, nq*D] bf16."""
        lay = self.layers[li]
        G = self.nq // self.nkv
        # cached values widened exactly (e4m3 and bf16 are subsets of fp32)
        K = kc[:, :ctx].float()  # [nkv, ctx, D]
        V = vc[:, :ctx].float()
        qg = q.reshape(self.nkv, G * T, self.D)
        s = torch.matmul(qg.float(), K.transpose(1, 2)).mul_(self.scale)  # [nkv, G*T, ctx]
        s = s.view(self.nkv, G, T, ctx)
        j = self._j[:ctx]
        qp = torch.arange(pos0, pos0 + T, device=q.device)
        valid = j[None, :] <= qp[:, None]                      # causal
        if self.sliding[li]:
            valid = valid & (j[None, :] > qp[:, None] - self.window)
        s = s.masked_fill(~valid.view(1, 1, T, ctx), float("-inf"))
        sink = lay["sinks"].view(self.nkv, G, 1, 1).expand(self.nkv, G, T, 1)
        comb = torch.cat([s, sink], dim=-1)
        p = torch.softmax(comb - comb.amax(-1, keepdim=True), dim=-1)[..., :ctx]
        o = torch.matmul(p.reshape(self.nkv, G * T, ctx), V)   # [nkv, G*T, D]
        o = o.view(self.nkv, G, T, self.D).permute(2, 0, 1, 3).reshape(T, self.nq * self.D)
        return o.to(torch.bfloat16)

    def _norm(self, x: torch.Tensor, delta, w: torch.Tensor, out: torch.Tensor) -> None:
        """x (fp32 residual [T, H]) += delta (bf16 / fp32 / None); out = bf16 RMSNorm(x) * w."""
        dt = 0 if delta is None or delta.dtype == torch.float32 else 1
        _lib.check(_lib.lib().tsb_add_rmsnorm(
            x.data_ptr(), None if delta is None else delta.data_ptr(), dt, w.data_ptr(), self.eps, x.shape[0],
            self.H, out.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream))

    def _prefill_layer(self, li: int, x: torch.Tensor, h: torch.Tensor, pos0: int, nxt_w: torch.Tensor,
                       kc: torch.Tensor, vc: torch.Tensor) -> None:
        """Prompt rows at positions pos0..: x fp32 residual [T, H] (in/out), h the
        bf16 RMSNorm of x on entry, replaced by the next sublayer's norm input."""
        lay = self.layers[li]
        T = x.shape[0]
        qkv = F.linear(h, lay["wqkv"], lay["bqkv"])
        nq, nkv, D = self.nq, self.nkv, self.D
        q = qkv[:, :nq * D].view(T, nq, D).transpose(0, 1)
        k = qkv[:, nq * D:(nq + nkv) * D].view(T, nkv, D).transpose(0, 1)
        v = qkv[:, (nq + nkv) * D:].view(T, nkv, D).transpose(0, 1)
        cos, sin = self.cos[pos0:pos0 + T], self.sin[pos0:pos0 + T]
        q, k = _rope(q, cos, sin), _rope(k, cos, sin)
        kc[:, pos0:pos0 + T] = k.to(self.kv_dtype)
        vc[:, pos0:pos0 + T] = v.to(self.kv_dtype)
        a = self._attn(li, q, pos0, T, pos0 + T, kc, vc)
        self._norm(x, F.linear(a, lay["wo"], lay["bo"]), lay["ln2"], h)
        y, _, _ = lay["moe"].decode(h, out_dtype=torch.float32)
        self._norm(x, y, nxt_w, h)

    def _next_norm(self, li: int) -> torch.Tensor:
        return self.layers[li + 1]["ln1"] if li + 1 < self.L else self.norm_w

    # ------------------------------------------------------------------ API
    @torch.no_grad()
    def prefill(self, ids: torch.Tensor, k_cache: torch.Tensor | None = None,
                v_cache: torch.Tensor | None = None) -> torch.Tensor:
        """Run prompt ids (1-D) from position 0, filling the cache (this
        decoder's, or the given [L, nkv, S, D] caches); returns the logits of
        the last prompt token (fp32 [V])."""
        kc_all = self.k_cache if k_cache is None else k_cache
        vc_all = self.v_cache if v_cache is None else v_cache
        ids = ids.reshape(-1).to(self.device)
        n = ids.numel()
        if n > self.max_seq:
            raise ValueError(f"prompt of {n} tokens exceeds the cache ({self.max_seq})")
        last = None
        for p0 in range(0, n, self.chunk):
            x = self.embed.index_select(0, ids[p0:p0 + self.chunk]).float()
            h = torch.empty(x.shape, dtype=torch.bfloat16, device=self.device)
            self._norm(x, None, self.layers[0]["ln1"], h)
            for li in range(self.L):
                self._prefill_layer(li, x, h, p0, self._next_norm(li), kc_all[li], vc_all[li])
            last = h[-1:]
        if k_cache is None:
            self.length = n
        return F.linear(last, self.lm_head)[0].float()

    def _step(self):
        """One decode token through every layer (the captured graph's body), four
        launches per layer: RMSNorm (folding the previous expert output into
        the residual) + q|k|v projection (tsb_norm_gemv_bf16), attention (RoPE,
        cache store, sink softmax; tsb_gqa_decode_attention) -- or both in one
        clustered kernel, tsb_norm_qkv_attention, when opted in -- the o GEMV adding into the residual and normalising it
        for the expert layer (tsb_gemv_bf16_residual), and the expert layer
        (fp32 output)."""
        L = _lib.lib()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        xin, xout = self._xe, self._xa
        xin.copy_(self.embed.index_select(0, self._tok))
        delta = None
        fp8 = 1 if self.kv_dtype == torch.float8_e4m3fn else 0
        for li, lay in enumerate(self.layers):
            dptr = None if delta is None else delta.data_ptr()
            bq = None if lay["bqkv"] is None else lay["bqkv"].data_ptr()
            win = self.window if self.sliding[li] else 0
            rc = 1
            if self._fused is not False:
                rc = L.tsb_norm_qkv_attention(
                    xin.data_ptr(), dptr, xout.data_ptr(), lay["ln1"].data_ptr(), self.eps, lay["wqkv"].data_ptr(), bq,
                    self.H, self.nq, self.nkv, self.D, self.cos.data_ptr(), self.sin.data_ptr(),
                    self._pos.data_ptr(), self.k_cache[li].data_ptr(), self.v_cache[li].data_ptr(), fp8,
                    self.max_seq, win, lay["sinks"].data_ptr(), self.scale, self._a.data_ptr(), stream)
                if self._fused is None and rc == _lib.TSB_ERR_UNSUPPORTED:
                    self._fused = False  # the shape does not fit the fused kernel: two launches
                else:
                    _lib.check(rc)
                    self._fused = True
            if not self._fused:
                _lib.check(L.tsb_norm_gemv_bf16(
                    xin.data_ptr(), dptr, xout.data_ptr(), lay["ln1"].data_ptr(), self.eps, lay["wqkv"].data_ptr(),
                    bq, lay["wqkv"].shape[0], self.H, self._qkv.data_ptr(), stream))
                _lib.check(L.tsb_gqa_decode_attention(
                    self._qkv.data_ptr(), self.nq, self.nkv, self.D, self.cos.data_ptr(), self.sin.data_ptr(),
                    self._pos.data_ptr(), self.k_cache[li].data_ptr(), self.v_cache[li].data_ptr(), fp8,
                    self.max_seq, win, lay["sinks"].data_ptr(), self.scale, self._a.data_ptr(),
                    self._aws.data_ptr(), self._aws.numel(), stream))
            _lib.check(L.tsb_gemv_bf16_residual(
                lay["wo"].data_ptr(), None if lay["bo"] is None else lay["bo"].data_ptr(), self.H, self.nq * self.D,
                self._a.data_ptr(), xout.data_ptr(), lay["ln2"].data_ptr(), self.eps, self._h.data_ptr(),
                self._cnt.data_ptr(), stream))
            lay["moe"].decode(self._h, out=self._y)
            delta = self._y
            xin, xout = xout, (self._xb if xout is self._xa else self._xa)
        self._norm(xin, delta, self.norm_w, self._h)
        self._logits = F.linear(self._h, self.lm_head)
        self._next.copy_(self._logits.argmax(-1))

    def _capture(self):
        st = torch.cuda.Stream(self.device)
        st.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(st):
            for _ in range(2):  # warm-up: workspaces, cuBLAS handles, library state
                self._step()
        torch.cuda.current_stream(self.device).wait_stream(st)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            self._step()
        self._graph = g

    @torch.no_grad()
    def step(self, token: int | torch.Tensor) -> torch.Tensor:
        """Append one token at the current position; returns the next greedy
        token as a device tensor (no host synchronisation)."""
        if self.length >= self.max_seq:
            raise ValueError("KV cache full")
        if isinstance(token, torch.Tensor):
            self._tok.copy_(token.reshape(1))
        else:
            self._tok.fill_(int(token))
        self._pos.fill_(self.length)
        if self._graph is None:
            self._capture()  # the warm-up steps write this position's K/V; the replay rewrites the same values
        self._graph.replay()
        self.length += 1
        return self._next

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, max_new_tokens: int) -> torch.Tensor:
        """Greedy decode: prefill the prompt, then max_new_tokens graph steps."""
        logits = self.prefill(prompt)
        tok = logits.argmax().reshape(1)
        out = [tok.clone()]
        for _ in range(max_new_tokens - 1):
            tok = self.step(tok)
            out.append(tok.clone())
        return torch.cat(out)

    def reset(self) -> None:
        self.length = 0
