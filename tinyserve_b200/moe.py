"""HBM-resident quantised MoE layer driven through the C-ABI.

``QuantMoE`` holds one layer's expert weights in device memory (raw GGUF
block streams or MXFP4 blocks + scales, exactly as the reference stores them,
``tinyserve/mmap_store.py:86-91`` and ``tinyserve/expert_store.py:365-387``),
builds the device table of expert pointers once, and runs a whole layer per
call: router -> top-k -> gate/up -> activation -> down -> weighted combine.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from .formats import TSB_MXFP4

ACTIVATIONS = {"silu": _lib.ACT_SILU, "swiglu_oai": _lib.ACT_SWIGLU_OAI}
LAYOUTS = {"separate": _lib.GU_SEPARATE, "interleaved": _lib.GU_INTERLEAVED, "chunked": _lib.GU_CHUNKED}


@dataclass
class ExpertWeights:
    """Device tensors of one expert (uint8 block streams; fp32 biases)."""
    gate: torch.Tensor                 # gate [I,H] stream, or gate_up [2I,H] for interleaved/chunked
    down: torch.Tensor                 # down [H,I] stream
    up: torch.Tensor | None = None     # up [I,H] stream for the separate layout
    gate_scales: torch.Tensor | None = None
    up_scales: torch.Tensor | None = None
    down_scales: torch.Tensor | None = None
    gate_bias: torch.Tensor | None = None
    up_bias: torch.Tensor | None = None
    down_bias: torch.Tensor | None = None


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


class QuantMoE:
    def __init__(self, experts: list[ExpertWeights], *, fmt_gate_up: int, fmt_down: int, hidden: int, inter: int,
                 top_k: int, router_w: torch.Tensor | None = None, router_b: torch.Tensor | None = None,
                 gate_up_layout: str = "separate", activation: str = "swiglu_oai", limit: float = 7.0,
                 alpha: float = 1.702, pack: bool | None = None, transposed: int = 0):
        if not experts:
            raise ValueError("no experts")
        self.device = experts[0].gate.device
        if self.device.type != "cuda":
            raise RuntimeError("QuantMoE needs the expert weights on a CUDA device")
        self.experts = experts
        # Dense experts (fmt GGML_F32 / F16 / BF16): weights are float tensors
        # [out, in], or [in, out] where `transposed` has _lib.T_GATE_UP /
        # _lib.T_DOWN set (read in place, tinyserve/expert_forward.py:140-149).
        self.spec = _lib.TsbMoeSpec(fmt_gate_up, fmt_down, hidden, inter, len(experts), top_k,
                                    LAYOUTS[gate_up_layout], ACTIVATIONS[activation], limit, alpha, 0, transposed)
        # the same layer with an fp32 output (the unrounded combine)
        self.spec_f32 = _lib.TsbMoeSpec(fmt_gate_up, fmt_down, hidden, inter, len(experts), top_k,
                                        LAYOUTS[gate_up_layout], ACTIVATIONS[activation], limit, alpha, 1, transposed)
        self.hidden, self.inter, self.top_k = hidden, inter, top_k
        self.router_w = router_w.contiguous() if router_w is not None else None
        self.router_b = router_b.float().contiguous() if router_b is not None else None
        table = (_lib.TsbExpert * len(experts))()
        for i, e in enumerate(experts):
            table[i] = _lib.TsbExpert(_p(e.gate), _p(e.up), _p(e.down), _p(e.gate_scales), _p(e.up_scales),
                                      _p(e.down_scales), _p(e.gate_bias), _p(e.up_bias), _p(e.down_bias))
        raw = bytes(ctypes.string_at(ctypes.addressof(table), ctypes.sizeof(table)))
        self._table = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(self.device)
        self._ws_cache: dict[int, torch.Tensor] = {}
        self._pws_cache: dict[int, torch.Tensor] = {}
        self._fast: dict[int, tuple] = {}
        # Batch-1 decode on a decode-packed copy of the experts (Q4_K and MXFP4
        # layers): built once here (~1.0-1.07x the quantised bytes); pack=None
        # packs when the spec has a packed form, pack=False keeps the generic
        # decode engine.
        self._packed = None
        nbytes = _lib.lib().tsb_moe_packed_bytes(ctypes.byref(self.spec))
        if pack and not nbytes:
            raise ValueError("this layer has no packed form (needs Q4_K or MXFP4 gate/up and down, H and I "
                             "multiples of 32)")
        if nbytes and pack is not False:
            self._packed = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
            _lib.check(_lib.lib().tsb_moe_pack(ctypes.byref(self.spec), self._table.data_ptr(),
                                               self._packed.data_ptr(), nbytes,
                                               torch.cuda.current_stream(self.device).cuda_stream))

    @property
    def packed(self) -> bool:
        """True when batch-1 decode runs on the decode-packed expert copy."""
        return self._packed is not None

    def _decode_call(self, f32: bool = False):
        """(C function, leading arguments) of this layer's decode entry point
        (fp32 output when `f32`)."""
        L = _lib.lib()
        spec = ctypes.byref(self.spec_f32 if f32 else self.spec)
        if self._packed is not None:
            return L.tsb_moe_decode_packed, (spec, self._packed.data_ptr(), self._table.data_ptr())
        return L.tsb_moe_decode, (spec, self._table.data_ptr())

    def workspace(self, T: int) -> torch.Tensor:
        if T not in self._ws_cache:
            L = _lib.lib()
            ws_fn = L.tsb_moe_decode_packed_workspace if self._packed is not None else L.tsb_moe_decode_workspace
            n = ws_fn(ctypes.byref(self.spec), T)
            self._ws_cache[T] = torch.zeros(n, dtype=torch.uint8, device=self.device)
        return self._ws_cache[T]

    def decode(self, x: torch.Tensor, ids: torch.Tensor | None = None, weights: torch.Tensor | None = None,
               out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16):
        """T tokens through the layer.  x: bf16 [T, H] ([1, H] for batch-1
        decode; up to 16 tokens run the batch-1 path per token, more the
        grouped path, each routed expert read once for all its tokens).  With a
        router, returns (out, ids, weights) where ids / weights are the routing
        it chose; without one, ``ids`` (int32 [T, k]) and ``weights`` (fp32
        [T, k]) are inputs.  ``out_dtype`` bf16 (default) or float32 (the
        unrounded combine; a given ``out`` decides by its own dtype)."""
        if x.dtype != torch.bfloat16:
            raise TypeError("x must be bfloat16")
        x = x.contiguous()
        T = x.shape[0] if x.dim() == 2 else 1
        given = ids is not None
        if not given:
            if self.router_w is None:
                raise ValueError("no router weights: pass ids and weights")
            ids = torch.empty(T, self.top_k, dtype=torch.int32, device=self.device)
            weights = torch.empty(T, self.top_k, dtype=torch.float32, device=self.device)
        else:
            ids = ids.to(device=self.device, dtype=torch.int32).contiguous()
            weights = weights.to(device=self.device, dtype=torch.float32).contiguous()
        if out is None:
            out = torch.empty(T, self.hidden, dtype=out_dtype, device=self.device)
        if out.dtype not in (torch.bfloat16, torch.float32):
            raise TypeError("out must be bfloat16 or float32")
        ws = self.workspace(T)
        fn, lead = self._decode_call(out.dtype == torch.float32)
        rc = fn(
            *lead, x.data_ptr(), T,
            None if given else _p(self.router_w), None if given else _p(self.router_b),
            ids.data_ptr(), weights.data_ptr(), out.data_ptr(), ws.data_ptr(), ws.numel(),
            torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(rc)
        return out, ids, weights

    def decode_(self, x: torch.Tensor, out: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                stream: int | None = None) -> None:
        """Allocation-free :meth:`decode` into caller-owned buffers (x bf16
        [T, H], out bf16 [T, H], ids int32 [T, k], weights fp32 [T, k], all
        contiguous on this device).  With a router the routing is written to
        ids / weights; without one they are read.  `stream` is a raw
        cudaStream_t (default: the current stream).  The C arguments that do not
        change between calls are prepared once per T, so a call is one ctypes
        call with no tensor allocation: the lean path for per-token serving."""
        T = x.shape[0]
        fast = self._fast.get(T)
        if fast is None:
            ws = self.workspace(T)
            fn, lead = self._decode_call()
            routed = self.router_w is not None
            fast = (fn, lead, _p(self.router_w) if routed else None, _p(self.router_b) if routed else None,
                    ws.data_ptr(), ws.numel())
            self._fast[T] = fast
        fn, lead, rw, rb, wsp, wsn = fast
        st = torch.cuda.current_stream(self.device).cuda_stream if stream is None else stream
        rc = fn(*lead, x.data_ptr(), T, rw, rb, ids.data_ptr(), weights.data_ptr(), out.data_ptr(), wsp, wsn, st)
        if rc:
            _lib.check(rc)

    def prefill_workspace(self, T: int) -> torch.Tensor:
        if T not in self._pws_cache:
            n = _lib.lib().tsb_moe_prefill_workspace(ctypes.byref(self.spec), T)
            self._pws_cache[T] = torch.zeros(n, dtype=torch.uint8, device=self.device)
        return self._pws_cache[T]

    def prefill(self, x: torch.Tensor, ids: torch.Tensor | None = None, weights: torch.Tensor | None = None,
                out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16):
        """T tokens through the layer as grouped GEMMs (the reference's batched
        path, ``ExpertPipeline.execute_layer_experts_batched``,
        tinyserve/expert_pipeline.py:166-239).  x: bf16 [T, H]; routing as in
        :meth:`decode`.  Returns (out, ids, weights)."""
        if x.dtype != torch.bfloat16:
            raise TypeError("x must be bfloat16")
        if x.dim() != 2 or x.shape[1] != self.hidden:
            raise ValueError(f"x must be [T, {self.hidden}]")
        x = x.contiguous()
        T = x.shape[0]
        given = ids is not None
        if not given:
            if self.router_w is None:
                raise ValueError("no router weights: pass ids and weights")
            ids = torch.empty(T, self.top_k, dtype=torch.int32, device=self.device)
            weights = torch.empty(T, self.top_k, dtype=torch.float32, device=self.device)
        else:
            ids = ids.to(device=self.device, dtype=torch.int32).contiguous()
            weights = weights.to(device=self.device, dtype=torch.float32).contiguous()
            if ids.shape != (T, self.top_k) or weights.shape != (T, self.top_k):
                raise ValueError(f"ids and weights must be [T, {self.top_k}]")
        if out is None:
            out = torch.empty(T, self.hidden, dtype=out_dtype, device=self.device)
        if out.dtype not in (torch.bfloat16, torch.float32):
            raise TypeError("out must be bfloat16 or float32")
        if T == 0:
            return out, ids, weights
        ws = self.prefill_workspace(T)
        rc = _lib.lib().tsb_moe_prefill(
            ctypes.byref(self.spec_f32 if out.dtype == torch.float32 else self.spec), self._table.data_ptr(), x.data_ptr(), T,
            None if given else _p(self.router_w), None if given else _p(self.router_b),
            ids.data_ptr(), weights.data_ptr(), out.data_ptr(), ws.data_ptr(), ws.numel(),
            torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(rc)
        return out, ids, weights

    def prefill_error(self, T: int) -> int:
        """Read and clear the device error word of the T-token prefill workspace."""
        code = ctypes.c_int32()
        ws = self.prefill_workspace(T)
        _lib.check(_lib.lib().tsb_read_device_error(ws.data_ptr(), ctypes.byref(code),
                                                    torch.cuda.current_stream(self.device).cuda_stream))
        return code.value

    def device_error(self, T: int = 1) -> int:
        code = ctypes.c_int32()
        ws = self.workspace(T)
        _lib.check(_lib.lib().tsb_read_device_error(ws.data_ptr(), ctypes.byref(code),
                                                    torch.cuda.current_stream(self.device).cuda_stream))
        return code.value

    @property
    def is_mxfp4(self) -> bool:
        return self.spec.fmt_gate_up == TSB_MXFP4


class Router:
    """The MoE router alone (tsb_moe_route): bf16 logits, top-k, softmax over
    the k selected logits (tinyserve/_model_hooks.py:466-473)."""

    def __init__(self, router_w: torch.Tensor, top_k: int, router_b: torch.Tensor | None = None):
        if router_w.dtype != torch.bfloat16 or router_w.dim() != 2:
            raise TypeError("router_w must be bf16 [E, H]")
        self.router_w = router_w.contiguous()
        self.router_b = router_b.float().contiguous() if router_b is not None else None
        E, H = router_w.shape
        self.spec = _lib.TsbMoeSpec(TSB_MXFP4, TSB_MXFP4, H, 32, E, top_k, 0, 1, 7.0, 1.702)
        self.top_k = top_k

    def __call__(self, x: torch.Tensor):
        if x.dtype != torch.bfloat16:
            raise TypeError("x must be bfloat16")
        x = x.contiguous()
        T = x.shape[0]
        ids = torch.empty(T, self.top_k, dtype=torch.int32, device=x.device)
        w = torch.empty(T, self.top_k, dtype=torch.float32, device=x.device)
        _lib.check(_lib.lib().tsb_moe_route(ctypes.byref(self.spec), x.data_ptr(), T, self.router_w.data_ptr(),
                                            _p(self.router_b), ids.data_ptr(), w.data_ptr(),
                                            torch.cuda.current_stream(x.device).cuda_stream))
        return ids, w


class DecodeSession:
    """Batch-1 decode of one layer per token as one CUDA-graph replay.

    For a serving loop that feeds one token at a time from the host: each
    slot's graph copies the token from a pinned host buffer to the device, runs
    the layer (two or three PDL-chained launches: packed or generic decode) and copies
    the result back to a pinned host buffer, so a token costs one host row copy
    and one graph launch instead of five separately issued operations.
    `slots` buffers rotate so the host can fill the next token while earlier
    ones run; a slot is reused only after its previous token finished.  Tokens
    run in submission order on the session's stream (pass one stream to
    several sessions to keep their tokens strictly sequential).

        sess = DecodeSession(layer)
        s = sess.submit(x_row)       # x_row: bf16 [1, H] or [H] on the host
        y = sess.result(s)           # pinned bf16 [1, H] (valid until slot s is reused)
    """

    def __init__(self, layer: QuantMoE, slots: int = 4, stream: torch.cuda.Stream | None = None):
        if layer.router_w is None:
            raise ValueError("DecodeSession needs a layer with router weights")
        dev = layer.device
        H, k = layer.hidden, layer.top_k
        self.layer, self.slots = layer, slots
        self.hin = torch.zeros(slots, 1, H, dtype=torch.bfloat16).pin_memory()
        self.hout = torch.zeros(slots, 1, H, dtype=torch.bfloat16).pin_memory()
        self.din = torch.zeros(1, H, dtype=torch.bfloat16, device=dev)
        self.dout = torch.empty(1, H, dtype=torch.bfloat16, device=dev)
        self.ids = torch.empty(1, k, dtype=torch.int32, device=dev)
        self.wts = torch.empty(1, k, dtype=torch.float32, device=dev)
        self.stream = stream if stream is not None else torch.cuda.Stream(dev)
        raw = self.stream.cuda_stream
        with torch.cuda.stream(self.stream):
            layer.decode_(self.din, self.dout, self.ids, self.wts, raw)  # workspace and arguments before capture
        torch.cuda.synchronize(dev)
        # The layer writes its output straight into the pinned host slot when
        # that memory is mapped at the same address on the device (unified
        # addressing): one device->host copy less per token.
        self._cu = ctypes.CDLL("libcuda.so.1")
        self.direct_out = all(self._mapped(self.hout[s].data_ptr()) for s in range(slots))
        self.graphs = []
        for s in range(slots):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                self.din.copy_(self.hin[s], non_blocking=True)
                if self.direct_out:
                    layer.decode_(self.din, self.hout[s], self.ids, self.wts, raw)
                else:
                    layer.decode_(self.din, self.dout, self.ids, self.wts, raw)
                    self.hout[s].copy_(self.dout, non_blocking=True)
            self.graphs.append(g)
        self.done = [torch.cuda.Event() for _ in range(slots)]
        for e in self.done:
            e.record(self.stream)  # creates the event handles
        torch.cuda.synchronize(dev)
        self.used = [False] * slots
        self.n = 0
        # The per-token path issues driver calls directly (graph launch, event
        # record / wait) and copies the row with one memmove: a token is
        # host-bound otherwise.  Runtime graph-exec, stream and event handles
        # are the driver's handles.
        self._exec = [ctypes.c_void_p(g.raw_cuda_graph_exec()) for g in self.graphs]
        self._ev = [ctypes.c_void_p(e.cuda_event) for e in self.done]
        self._st = ctypes.c_void_p(raw)
        self._hin = [self.hin[s].data_ptr() for s in range(slots)]
        self._row_bytes = H * 2

    def _mapped(self, host_ptr: int) -> bool:
        """Pinned host memory the device reaches at the same address."""
        dptr = ctypes.c_uint64()
        rc = self._cu.cuMemHostGetDevicePointer_v2(ctypes.byref(dptr), ctypes.c_void_p(host_ptr), 0)
        return rc == 0 and dptr.value == host_ptr

    def _drv(self, rc: int, what: str) -> None:
        if rc:
            raise RuntimeError(f"{what} failed (CUresult {rc})")

    def submit(self, x_row: torch.Tensor) -> int:
        s = self.n % self.slots
        self.n += 1
        if self.used[s]:
            self._drv(self._cu.cuEventSynchronize(self._ev[s]), "cuEventSynchronize")
        if x_row.dtype != torch.bfloat16 or x_row.device.type != "cpu" or x_row.numel() != self._row_bytes // 2:
            raise ValueError("x_row must be a bf16 host row of hidden elements")
        if not x_row.is_contiguous():
            x_row = x_row.contiguous()
        ctypes.memmove(self._hin[s], x_row.data_ptr(), self._row_bytes)
        self._drv(self._cu.cuGraphLaunch(self._exec[s], self._st), "cuGraphLaunch")
        self._drv(self._cu.cuEventRecord(self._ev[s], self._st), "cuEventRecord")
        self.used[s] = True
        return s

    def result(self, s: int) -> torch.Tensor:
        self.done[s].synchronize()
        return self.hout[s]
