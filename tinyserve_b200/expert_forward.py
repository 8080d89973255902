"""Per-expert forwards on packed expert bytes, mirroring the reference's
inline-forward contract ``(packed uint8 [expert_bytes] cuda, h [T, H] bf16)
-> [T, H]`` (tinyserve/expert_forward.py:164-246, ggml_forward.py:68-151)
and its GGUF linear layer (ggml_linear.py:48-117).

- ``TensorLayout``: named tensors packed back to back in insertion order
  (tinyserve/expert_store.py:57-77); offsets and sizes are the same numbers.
- ``GGMLExpertForward(layout, ggml_types, act_fn, proj_shapes)``: GGUF
  gate/up/down in one packed buffer.  ``proj_shapes`` use the GGML
  convention (in_features, out_features).  Every batch size runs through the
  C-ABI layer call with one expert (T = 1: the fused decode kernels; T > 1:
  token loop or grouped GEMMs), instead of three matvecs (batch 1) or CPU
  dequantisation + F.linear (batch > 1).
- ``build_mxfp4_inline_forward(layout, act_fn)``: GPT-OSS MXFP4 experts
  (gate_up_proj blocks/scales, down_proj blocks/scales).  ``act_fn=None``
  is the interleaved clamp-SwiGLU; an activation module (SiLU) means the
  chunked gate|up halves.  Biases in the layout (gate_up_proj_bias,
  down_proj_bias) are applied; the reference's inline MXFP4 forward ignores
  them.
- ``build_inline_forward(layout, act_fn)``: dense bf16 / fp16 / fp32 experts
  (tinyserve/expert_forward.py:109-194) through the C-ABI's dense layer, with
  the reference's transpose rule for weights stored [in, out] (read in
  place) and its activation rule (``act_fn`` SiLU over chunked halves, None
  for the interleaved clamp-SwiGLU).
- ``GGMLLinear``: one GGUF-quantised linear; every batch size is one
  multi-vector matvec call (the reference loops over tokens for batch > 1).
"""
from __future__ import annotations

import torch
from torch import nn

from . import ops
from . import _lib
from .formats import GGML_BF16, GGML_F16, GGML_F32, TSB_MXFP4
from .moe import ExpertWeights, QuantMoE

_DENSE_FMT = {torch.float32: GGML_F32, torch.float16: GGML_F16, torch.bfloat16: GGML_BF16}

_DTYPE_SIZE = {}


def _elem_size(dtype: torch.dtype) -> int:
    if dtype not in _DTYPE_SIZE:
        _DTYPE_SIZE[dtype] = torch.tensor([], dtype=dtype).element_size()
    return _DTYPE_SIZE[dtype]


class TensorLayout:
    """How named tensors are packed into one flat byte buffer (insertion order,
    no padding)."""

    def __init__(self, tensor_specs: dict[str, tuple[tuple[int, ...], torch.dtype]]):
        self.specs = tensor_specs
        self.offsets: dict[str, int] = {}
        self.sizes: dict[str, int] = {}
        off = 0
        for name, (shape, dtype) in tensor_specs.items():
            n = _elem_size(dtype)
            for d in shape:
                n *= int(d)
            self.offsets[name] = off
            self.sizes[name] = n
            off += n
        self.total_bytes = off

    @staticmethod
    def from_tensors(tensors: dict[str, torch.Tensor]) -> "TensorLayout":
        return TensorLayout({k: (tuple(v.shape), v.dtype) for k, v in tensors.items()})

    def view(self, packed: torch.Tensor, name: str) -> torch.Tensor:
        o, n = self.offsets[name], self.sizes[name]
        return packed[o:o + n]


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """The kernels read weights with 16-byte copies; copy an unaligned view."""
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _all_aligned(*ts: torch.Tensor) -> bool:
    return all(t.data_ptr() % 16 == 0 for t in ts)


def _act_kind(act_fn) -> str:
    if isinstance(act_fn, nn.SiLU) or act_fn is torch.nn.functional.silu:
        return "silu"
    raise ValueError(f"unsupported activation {act_fn!r}: SiLU (GGUF experts) or None (GPT-OSS clamp-SwiGLU)")


class _ExpertCache:
    """One single-expert QuantMoE per packed buffer address (cache slots keep
    their address while their contents change, and the device table only
    holds addresses)."""

    def __init__(self, make, cacheable):
        self._make = make
        self._cacheable = cacheable  # packed -> False when a projection had to be copied to align it
        self._by_ptr: dict[tuple[int, int], QuantMoE] = {}

    def get(self, packed: torch.Tensor) -> QuantMoE:
        key = (packed.data_ptr(), packed.device.index or 0)
        layer = self._by_ptr.get(key)
        if layer is None:
            layer = self._make(packed)
            if self._cacheable(packed):
                self._by_ptr[key] = layer
        return layer


def _run_one_expert(layer: QuantMoE, h: torch.Tensor) -> torch.Tensor:
    T = h.shape[0]
    ids = torch.zeros(T, 1, dtype=torch.int32, device=h.device)
    w = torch.ones(T, 1, dtype=torch.float32, device=h.device)
    out, _, _ = layer.decode(h.to(torch.bfloat16).contiguous(), ids=ids, weights=w)
    return out.to(h.dtype)


class GGMLExpertForward:
    """GGUF expert forward on packed bytes (tinyserve/ggml_forward.py:27-151)."""

    def __init__(self, layout: TensorLayout, ggml_types: dict[str, int], act_fn,
                 proj_shapes: dict[str, tuple[int, int]]):
        self._ggml_types = dict(ggml_types)
        self._act = _act_kind(act_fn)
        self._proj_shapes = dict(proj_shapes)
        self._layout = layout
        H, I = proj_shapes["gate"]
        if tuple(proj_shapes["up"]) != (H, I) or tuple(proj_shapes["down"]) != (I, H):
            raise ValueError("proj_shapes must be gate/up (H, I) and down (I, H) in GGML (in, out) order")
        if ggml_types["gate"] != ggml_types["up"]:
            raise ValueError("gate and up must share one format")
        self.hidden, self.inter = H, I
        self._cache = _ExpertCache(self._make, lambda p: _all_aligned(*(self._raw(p, n) for n in ("gate", "up", "down"))))

    def _raw(self, packed: torch.Tensor, name: str) -> torch.Tensor:
        fmt = self._ggml_types[name]
        n_in, n_out = self._proj_shapes[name]
        data, _ = ops.weight_bytes(fmt, n_out, n_in)
        o = self._layout.offsets[name]
        return packed[o:o + data]

    def _bytes(self, packed: torch.Tensor, name: str) -> torch.Tensor:
        return _aligned(self._raw(packed, name))

    def _make(self, packed: torch.Tensor) -> QuantMoE:
        ew = ExpertWeights(gate=self._bytes(packed, "gate"), up=self._bytes(packed, "up"),
                           down=self._bytes(packed, "down"))
        return QuantMoE([ew], fmt_gate_up=self._ggml_types["gate"], fmt_down=self._ggml_types["down"],
                        hidden=self.hidden, inter=self.inter, top_k=1, gate_up_layout="separate",
                        activation=self._act)

    def forward(self, packed: torch.Tensor, h: torch.Tensor, layer_idx: int = -1) -> torch.Tensor:
        return _run_one_expert(self._cache.get(packed), h)

    __call__ = forward


def build_mxfp4_inline_forward(layout: TensorLayout, act_fn):
    """(packed, h) -> out for GPT-OSS MXFP4 experts
    (tinyserve/expert_forward.py:197-246); None when the layout holds no
    MXFP4 scales."""
    specs = layout.specs
    if "gate_up_proj_scales" not in specs:
        return None
    gu_shape = specs["gate_up_proj"][0]   # [2I, H/32, 16]
    dn_shape = specs["down_proj"][0]      # [H, I/32, 16]
    I2, H = int(gu_shape[0]), int(gu_shape[1]) * 32
    I = I2 // 2
    if int(dn_shape[0]) != H or int(dn_shape[1]) * 32 != I:
        raise ValueError("down_proj shape does not match gate_up_proj")
    activation, gu_layout = ("swiglu_oai", "interleaved") if act_fn is None else (_act_kind(act_fn), "chunked")

    def make(packed: torch.Tensor) -> QuantMoE:
        v = lambda n: _aligned(layout.view(packed, n))  # noqa: E731
        biases = _Biases(layout, gu_layout, I, packed.device)
        ew = ExpertWeights(gate=v("gate_up_proj"), down=v("down_proj"), gate_scales=v("gate_up_proj_scales"),
                           down_scales=v("down_proj_scales"), gate_bias=biases.gate, up_bias=biases.up,
                           down_bias=biases.down)
        layer = QuantMoE([ew], fmt_gate_up=TSB_MXFP4, fmt_down=TSB_MXFP4, hidden=H, inter=I, top_k=1,
                         gate_up_layout=gu_layout, activation=activation)
        layer._biases = biases  # the table points at these buffers
        return layer

    names = ("gate_up_proj", "gate_up_proj_scales", "down_proj", "down_proj_scales")
    cache = _ExpertCache(make, lambda p: _all_aligned(*(layout.view(p, n) for n in names[::2])))

    def _forward(packed: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
        layer = cache.get(packed)
        layer._biases.refresh(packed)
        return _run_one_expert(layer, h)

    return _forward


class _Biases:
    """fp32 copies of an expert's biases for the device table.  The packed
    bytes behind a cached layer can change while its address stays (a cache
    slot refilled with another expert), so the copies are refreshed from the
    packed views on every call (three small device copies)."""

    def __init__(self, layout: TensorLayout, gu_layout: str, inter: int, device):
        specs = layout.specs
        self._layout = layout
        self._gu = "gate_up_proj_bias" in specs
        self._dn = "down_proj_bias" in specs
        self._interleaved = gu_layout == "interleaved"
        self.gate = self.up = self.down = None
        if self._gu:
            self.gate = torch.empty(inter, dtype=torch.float32, device=device)
            self.up = torch.empty(inter, dtype=torch.float32, device=device)
        if self._dn:
            self.down = torch.empty(int(specs["down_proj_bias"][0][-1]), dtype=torch.float32, device=device)

    def refresh(self, packed: torch.Tensor) -> None:
        specs = self._layout.specs
        if self._gu:
            b = self._layout.view(packed, "gate_up_proj_bias").view(specs["gate_up_proj_bias"][1])
            g, u = (b[0::2], b[1::2]) if self._interleaved else b.chunk(2)
            self.gate.copy_(g)
            self.up.copy_(u)
        if self._dn:
            self.down.copy_(self._layout.view(packed, "down_proj_bias").view(specs["down_proj_bias"][1]))


def build_inline_forward(layout: TensorLayout, act_fn):
    """(packed, h) -> out for dense experts (tinyserve/expert_forward.py:109-194);
    None when the layout has no dense gate_up_proj / down_proj (MXFP4 layouts
    go to build_mxfp4_inline_forward).

    Transpose rule of the reference (expert_forward.py:140-149): gate_up is
    stored [in, out] when its first dimension is the smaller one (hidden);
    down is stored [in, out] when its first dimension equals max(gate_up
    shape) // 2 -- for a square down projection (hidden == intermediate) that
    rule reads the weight transposed, and so does this forward.  Weights are
    read in place in either orientation.  ``h`` is rounded to bf16 (the
    layer kernels take bf16 hidden states); the output has ``h``'s dtype."""
    specs = layout.specs
    if "gate_up_proj" not in specs or "down_proj" not in specs or "gate_up_proj_scales" in specs:
        return None
    gu_shape, gu_dtype = specs["gate_up_proj"]
    dn_shape, dn_dtype = specs["down_proj"]
    if gu_dtype not in _DENSE_FMT or dn_dtype not in _DENSE_FMT:
        return None
    gu_shape, dn_shape = tuple(int(d) for d in gu_shape), tuple(int(d) for d in dn_shape)
    H = min(gu_shape)
    I = max(gu_shape) // 2
    gu_t = gu_shape[0] == H
    dn_t = dn_shape[0] == I
    if sorted(dn_shape) != sorted((H, I)):
        raise ValueError("down_proj shape does not match gate_up_proj")
    activation, gu_layout = ("swiglu_oai", "interleaved") if act_fn is None else (_act_kind(act_fn), "chunked")
    transposed = (_lib.T_GATE_UP if gu_t else 0) | (_lib.T_DOWN if dn_t else 0)

    def make(packed: torch.Tensor) -> QuantMoE:
        biases = _Biases(layout, gu_layout, I, packed.device)
        ew = ExpertWeights(gate=_aligned(layout.view(packed, "gate_up_proj")),
                           down=_aligned(layout.view(packed, "down_proj")),
                           gate_bias=biases.gate, up_bias=biases.up, down_bias=biases.down)
        layer = QuantMoE([ew], fmt_gate_up=_DENSE_FMT[gu_dtype], fmt_down=_DENSE_FMT[dn_dtype], hidden=H, inter=I,
                         top_k=1, gate_up_layout=gu_layout, activation=activation, transposed=transposed)
        layer._biases = biases
        return layer

    names = ("gate_up_proj", "down_proj")
    cache = _ExpertCache(make, lambda p: _all_aligned(*(layout.view(p, n) for n in names)))

    def _forward(packed: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
        layer = cache.get(packed)
        layer._biases.refresh(packed)
        return _run_one_expert(layer, h)

    return _forward


class GGMLLinear(nn.Module):
    """Linear layer on raw GGUF-quantised weights (tinyserve/ggml_linear.py:48-117)."""

    def __init__(self, raw_bytes, ggml_type: int, out_features: int, in_features: int,
                 bias: torch.Tensor | None = None, device="cuda"):
        super().__init__()
        if isinstance(raw_bytes, bytes):
            q = torch.frombuffer(bytearray(raw_bytes), dtype=torch.uint8)
        else:
            q = raw_bytes
        self._qweight = _aligned(q.to(device).contiguous())
        self._ggml_type = ggml_type
        self.out_features, self.in_features = out_features, in_features
        self.bias = nn.Parameter(bias.to(device)) if bias is not None else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1])
        out = ops.quant_matvec(self._ggml_type, self._qweight, None, self.out_features, self.in_features, x2)
        if self.bias is not None:
            out = out + self.bias
        return out.reshape(*x.shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"ggml_type={self._ggml_type}, qweight={self._qweight.shape[0]} bytes, bias={self.bias is not None}")
