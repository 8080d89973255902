"""On-disk expert weights straight into HBM expert tables.

Two checkpoint formats feed the layer path without any CPU-side decoding:

* GGUF (v2 / v3): the header, metadata and tensor table are parsed here; the
  data section is memory-mapped and each expert tensor's raw block stream is
  copied to the GPU as-is (one host-to-device copy per tensor).  Expert tensors
  come either fused per layer, ``blk.<L>.ffn_{gate,up,down}_exps.weight``
  (dims ``[in, out, n_experts]`` in GGUF's fastest-first order, so expert e is
  the e-th contiguous [out, in] block), or one per expert,
  ``blk.<L>.ffn_{gate,up,down}.<e>.weight``; the router is
  ``blk.<L>.ffn_gate_inp.weight`` (the naming tinyserve's reader matches,
  tinyserve/gguf_reader.py:173-214, and its store slices,
  tinyserve/mmap_store.py:166-274).
* Hugging Face safetensors with GPT-OSS MXFP4 experts:
  ``<prefix>.experts.{gate_up,down}_proj_{blocks,scales}``, their biases and
  ``<prefix>.router.{weight,bias}`` (tinyserve/expert_store.py:277-403 loads
  the same keys as raw uint8).  A directory with
  ``model.safetensors.index.json`` or a single file.

Both return a :class:`tinyserve_b200.moe.QuantMoE` whose experts live in HBM
(there is no host tier: the bytes are read from the page cache once).
"""
from __future__ import annotations

import json
import os
import re
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from .formats import DENSE, FORMATS, GGML_BF16, GGML_F16, GGML_F32, TSB_MXFP4

GGUF_MAGIC = 0x46554747  # "GGUF" little-endian

# metadata value types of the GGUF format
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)
_SCALAR = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f", _BOOL: "<?",
           _U64: "<Q", _I64: "<q", _F64: "<d"}


@dataclass
class GGUFTensor:
    name: str
    dims: tuple[int, ...]   # GGUF order: dims[0] is the fastest (the input features of a weight)
    ggml_type: int
    offset: int             # from the start of the data section
    nbytes: int

    @property
    def rows_cols(self) -> tuple[int, int]:
        """(rows, cols) of one 2-D slice: cols = dims[0], rows = dims[1]."""
        return (self.dims[1] if len(self.dims) > 1 else 1), self.dims[0]


def _tensor_nbytes(ggml_type: int, dims: tuple[int, ...]) -> int:
    n = int(np.prod(dims, dtype=np.int64)) if dims else 1
    if ggml_type in DENSE:
        return n * DENSE[ggml_type]
    if ggml_type in FORMATS and ggml_type != TSB_MXFP4:
        _, bb, be = FORMATS[ggml_type]
        if n % be:
            raise ValueError(f"tensor of {n} elements is not a whole number of {be}-element blocks")
        return n // be * bb
    return -1  # a type this library has no kernels for: listed, not loadable


class GGUFFile:
    """Header, metadata and tensor table of a GGUF file; tensor bytes are
    memory-mapped views (no copy until they are sent to the device)."""

    def __init__(self, path: str | os.PathLike):
        self.path = Path(path)
        with open(self.path, "rb") as f:
            buf = f.read(1 << 20)
            pos = 0

            def need(n):
                nonlocal buf
                while pos + n > len(buf):
                    more = f.read(1 << 20)
                    if not more:
                        raise ValueError("truncated GGUF header")
                    buf += more

            def take(fmt):
                nonlocal pos
                n = struct.calcsize(fmt)
                need(n)
                v = struct.unpack_from(fmt, buf, pos)[0]
                pos += n
                return v

            def string():
                nonlocal pos
                n = take("<Q")
                need(n)
                s = buf[pos:pos + n].decode("utf-8", errors="replace")
                pos += n
                return s

            def value(vt):
                if vt == _STR:
                    return string()
                if vt == _ARR:
                    et, count = take("<I"), take("<Q")
                    return [value(et) for _ in range(count)]
                if vt not in _SCALAR:
                    raise ValueError(f"unknown GGUF metadata type {vt}")
                return take(_SCALAR[vt])

            if take("<I") != GGUF_MAGIC:
                raise ValueError(f"{self.path}: not a GGUF file")
            self.version = take("<I")
            if self.version not in (2, 3):
                raise ValueError(f"GGUF version {self.version} is not supported (2 or 3)")
            n_tensors, n_kv = take("<Q"), take("<Q")
            self.metadata: dict = {}
            for _ in range(n_kv):
                key = string()
                self.metadata[key] = value(take("<I"))
            self.tensors: dict[str, GGUFTensor] = {}
            for _ in range(n_tensors):
                name = string()
                nd = take("<I")
                dims = tuple(take("<Q") for _ in range(nd))
                t = take("<I")
                off = take("<Q")
                self.tensors[name] = GGUFTensor(name, dims, t, off, _tensor_nbytes(t, dims))
            align = int(self.metadata.get("general.alignment", 32))
            self.data_offset = (pos + align - 1) // align * align
        self._mm = np.memmap(self.path, dtype=np.uint8, mode="r")

    def raw(self, t: GGUFTensor | str, start: int = 0, nbytes: int | None = None) -> np.ndarray:
        """Memory-mapped bytes of a tensor (or of [start, start + nbytes) within it)."""
        if isinstance(t, str):
            t = self.tensors[t]
        if t.nbytes < 0:
            raise ValueError(f"{t.name}: ggml type {t.ggml_type} has no kernels in this library")
        n = t.nbytes - start if nbytes is None else nbytes
        a = self.data_offset + t.offset + start
        if a + n > self._mm.size:
            raise ValueError(f"{t.name}: data past the end of the file")
        return self._mm[a:a + n]

    @property
    def arch(self) -> str:
        return str(self.metadata.get("general.architecture", ""))

    def expert_tensors(self, layer: int) -> dict[str, list[tuple[GGUFTensor, int]]]:
        """{proj: [(tensor, byte offset of expert e), ...]} for gate / up / down of
        a layer, from fused ``_exps`` tensors or per-expert tensors."""
        out: dict[str, list[tuple[GGUFTensor, int]]] = {}
        for proj in ("gate", "up", "down"):
            fused = self.tensors.get(f"blk.{layer}.ffn_{proj}_exps.weight")
            if fused is not None:
                if len(fused.dims) != 3:
                    raise ValueError(f"{fused.name}: expected 3 dims, got {fused.dims}")
                E = fused.dims[2]
                per = fused.nbytes // E
                out[proj] = [(fused, e * per) for e in range(E)]
                continue
            pat = re.compile(rf"blk\.{layer}\.ffn_{proj}\.(\d+)\.weight$")
            found = sorted((int(m.group(1)), t) for n, t in self.tensors.items() if (m := pat.match(n)))
            if found:
                if [e for e, _ in found] != list(range(len(found))):
                    raise ValueError(f"layer {layer} {proj}: expert ids are not 0..{len(found) - 1}")
                out[proj] = [(t, 0) for _, t in found]
        return out


def _to_device(a: np.ndarray, device) -> torch.Tensor:
    """One host-to-device copy of a byte range (16-byte aligned on the device;
    the mapped file pages are read once into a host buffer first)."""
    return torch.from_numpy(np.array(a, copy=True)).to(device)


def _al(t: torch.Tensor) -> torch.Tensor:
    """The kernels read weights with 16-byte copies: a per-expert view that
    does not start on the 16-byte grid gets its own (aligned) copy."""
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _float_tensor(a: np.ndarray, ggml_type: int, shape) -> torch.Tensor:
    dt = {GGML_F32: np.float32, GGML_F16: np.float16}.get(ggml_type)
    if dt is not None:
        return torch.from_numpy(np.array(a, copy=True).view(dt).reshape(shape).astype(np.float32))
    if ggml_type == GGML_BF16:
        u = np.array(a, copy=True).view(np.uint16).astype(np.uint32) << 16
        return torch.from_numpy(u.view(np.float32).reshape(shape))
    raise ValueError(f"router of ggml type {ggml_type} is not a float tensor")


def load_gguf_moe(gguf: str | os.PathLike | GGUFFile, layer: int, *, device="cuda", top_k: int | None = None,
                  activation: str = "silu", pack: bool | None = None):
    """The MoE layer ``layer`` of a GGUF file as a QuantMoE with every expert in
    HBM.  Experts keep their GGUF block streams byte for byte (Q8_0 / Q4_K /
    Q5_K / Q6_K, or dense F32 / F16 / BF16); gate and up stay separate (GGUF
    stores them so); the router is ``ffn_gate_inp`` rounded to bf16.  ``top_k``
    defaults to the file's ``<arch>.expert_used_count``."""
    from .moe import ExpertWeights, QuantMoE
    f = gguf if isinstance(gguf, GGUFFile) else GGUFFile(gguf)
    ex = f.expert_tensors(layer)
    if set(ex) != {"gate", "up", "down"}:
        raise ValueError(f"layer {layer}: no gate/up/down expert tensors in {f.path.name}")
    E = len(ex["gate"])
    if len(ex["up"]) != E or len(ex["down"]) != E:
        raise ValueError(f"layer {layer}: gate/up/down expert counts differ")
    g0, d0 = ex["gate"][0][0], ex["down"][0][0]
    I, H = g0.rows_cols
    if d0.rows_cols != (H, I):
        raise ValueError(f"layer {layer}: down is {d0.rows_cols}, expected {(H, I)}")
    fmt_gu, fmt_dn = g0.ggml_type, d0.ggml_type
    if ex["up"][0][0].ggml_type != fmt_gu:
        raise ValueError("gate and up must share one format")
    if top_k is None:
        top_k = int(f.metadata.get(f"{f.arch}.expert_used_count", 0)) or None
        if top_k is None:
            raise ValueError("top_k not given and the file has no <arch>.expert_used_count")
    device = torch.device(device)

    def per_expert(proj: str, rows: int, cols: int) -> list[torch.Tensor]:
        from .formats import weight_bytes
        fmt = ex[proj][0][0].ggml_type
        nb = rows * cols * DENSE[fmt] if fmt in DENSE else weight_bytes(fmt, rows, cols)
        tensors = {id(t): t for t, _ in ex[proj]}
        if len(tensors) == 1 and nb % 16 == 0:
            # fused: one copy of the whole [E, rows, cols] stream, per-expert views
            (t,) = tensors.values()
            dev = _to_device(f.raw(t), device)
            return [_al(dev[o:o + nb]) for _, o in ex[proj]]
        return [_to_device(f.raw(t, o, nb), device) for t, o in ex[proj]]

    gates, ups, downs = per_expert("gate", I, H), per_expert("up", I, H), per_expert("down", H, I)
    router = f.tensors.get(f"blk.{layer}.ffn_gate_inp.weight")
    rw = None
    if router is not None:
        rw = _float_tensor(f.raw(router), router.ggml_type, (E, H)).to(torch.bfloat16).to(device)
    experts = [ExpertWeights(gate=g, up=u, down=d) for g, u, d in zip(gates, ups, downs)]
    return QuantMoE(experts, fmt_gate_up=fmt_gu, fmt_down=fmt_dn, hidden=H, inter=I, top_k=top_k, router_w=rw,
                    gate_up_layout="separate", activation=activation, pack=pack)


# ---------------------------------------------------------------------------- safetensors

_ST_DTYPES = {"U8": np.uint8, "I8": np.int8, "F32": np.float32, "F16": np.float16, "BF16": np.uint16,
              "I32": np.int32, "I64": np.int64}


class SafetensorsFile:
    """Header of one .safetensors file; tensors are memory-mapped views."""

    def __init__(self, path: str | os.PathLike):
        self.path = Path(path)
        with open(self.path, "rb") as f:
            n = struct.unpack("<Q", f.read(8))[0]
            header = json.loads(f.read(n))
        self.metadata = header.pop("__metadata__", {})
        self.entries = header
        self._base = 8 + n
        self._mm = np.memmap(self.path, dtype=np.uint8, mode="r")

    def raw(self, name: str) -> tuple[np.ndarray, str, tuple[int, ...]]:
        e = self.entries[name]
        b, en = e["data_offsets"]
        return self._mm[self._base + b:self._base + en], e["dtype"], tuple(e["shape"])


class SafetensorsIndex:
    """Tensor name -> file for a checkpoint directory (``model.safetensors.index.json``)
    or a single file."""

    def __init__(self, path: str | os.PathLike):
        p = Path(path)
        self.files: dict[str, SafetensorsFile] = {}
        self.where: dict[str, str] = {}
        if p.is_dir():
            idx = p / "model.safetensors.index.json"
            if idx.exists():
                wm = json.loads(idx.read_text())["weight_map"]
                for name, fn in wm.items():
                    self.where[name] = str(p / fn)
            else:
                for fp in sorted(p.glob("*.safetensors")):
                    for name in SafetensorsFile(fp).entries:
                        self.where[name] = str(fp)
            self.config = json.loads((p / "config.json").read_text()) if (p / "config.json").exists() else {}
        else:
            for name in SafetensorsFile(p).entries:
                self.where[name] = str(p)
            self.config = {}

    def __contains__(self, name: str) -> bool:
        return name in self.where

    def raw(self, name: str):
        fn = self.where[name]
        if fn not in self.files:
            self.files[fn] = SafetensorsFile(fn)
        return self.files[fn].raw(name)


def _st_float(a: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype == "BF16":
        u = np.array(a, copy=True).view(np.uint16).astype(np.uint32) << 16
        return torch.from_numpy(u.view(np.float32))
    return torch.from_numpy(np.array(a, copy=True).view(_ST_DTYPES[dtype]).astype(np.float32))


def load_safetensors_mxfp4_moe(path: str | os.PathLike | SafetensorsIndex, layer: int, *, device="cuda",
                               top_k: int | None = None, prefix: str = "model.layers.{layer}.mlp",
                               limit: float = 7.0, alpha: float = 1.702, pack: bool | None = None):
    """The GPT-OSS MoE block of decoder layer ``layer`` from HF safetensors with
    MXFP4 experts, as a QuantMoE: ``gate_up_proj_blocks`` [E, 2I, H/32, 16]
    (rows 2j / 2j+1 = gate / up of output j), ``gate_up_proj_scales`` [E, 2I,
    H/32] (E8M0), ``down_proj_blocks`` [E, H, I/32, 16], ``down_proj_scales``,
    the biases and the router.  Blocks and scales go to the device unchanged
    (one copy per tensor); ``top_k`` defaults to the checkpoint config's
    ``num_experts_per_tok``."""
    from .moe import ExpertWeights, QuantMoE
    idx = path if isinstance(path, SafetensorsIndex) else SafetensorsIndex(path)
    pre = prefix.format(layer=layer)
    need = [f"{pre}.experts.{n}" for n in ("gate_up_proj_blocks", "gate_up_proj_scales", "down_proj_blocks",
                                          "down_proj_scales")]
    missing = [n for n in need if n not in idx]
    if missing:
        raise ValueError(f"layer {layer}: missing MXFP4 expert tensors {missing}")
    gub, gdt, gshape = idx.raw(need[0])
    gus, _, sshape = idx.raw(need[1])
    dnb, _, dshape = idx.raw(need[2])
    dns, _, _ = idx.raw(need[3])
    if gdt != "U8" or len(gshape) != 4 or gshape[3] != 16:
        raise ValueError(f"{need[0]}: expected U8 [E, 2I, H/32, 16], got {gdt} {gshape}")
    E, I2, G, _ = gshape
    H, I = G * 32, I2 // 2
    if tuple(dshape) != (E, H, I // 32, 16) or tuple(sshape) != (E, I2, G):
        raise ValueError(f"layer {layer}: down / scale shapes {dshape} {sshape} do not match gate_up {gshape}")
    if top_k is None:
        top_k = int(idx.config.get("num_experts_per_tok", idx.config.get("experts_per_token", 0))) or None
        if top_k is None:
            raise ValueError("top_k not given and the checkpoint config has no num_experts_per_tok")
    device = torch.device(device)
    dev = {n: _to_device(a, device) for n, a in (("gub", gub), ("gus", gus), ("dnb", dnb), ("dns", dns))}
    ngb, ngs, ndb, nds = I2 * H // 2, I2 * G, H * I // 2, H * (I // 32)
    gb = gu = db = None
    if f"{pre}.experts.gate_up_proj_bias" in idx:
        a, dt, _ = idx.raw(f"{pre}.experts.gate_up_proj_bias")
        b = _st_float(a, dt).reshape(E, I2).to(device)
        gb, gu = b[:, 0::2].contiguous(), b[:, 1::2].contiguous()
    if f"{pre}.experts.down_proj_bias" in idx:
        a, dt, _ = idx.raw(f"{pre}.experts.down_proj_bias")
        db = _st_float(a, dt).reshape(E, H).to(device)
    experts = []
    for e in range(E):
        experts.append(ExpertWeights(
            gate=_al(dev["gub"][e * ngb:(e + 1) * ngb]), gate_scales=_al(dev["gus"][e * ngs:(e + 1) * ngs]),
            down=_al(dev["dnb"][e * ndb:(e + 1) * ndb]), down_scales=_al(dev["dns"][e * nds:(e + 1) * nds]),
            gate_bias=None if gb is None else gb[e], up_bias=None if gu is None else gu[e],
            down_bias=None if db is None else db[e]))
    rw = rb = None
    if f"{pre}.router.weight" in idx:
        a, dt, _ = idx.raw(f"{pre}.router.weight")
        rw = _st_float(a, dt).reshape(E, H).to(torch.bfloat16).to(device)
        if f"{pre}.router.bias" in idx:
            a, dt, _ = idx.raw(f"{pre}.router.bias")
            rb = _st_float(a, dt).reshape(E).to(device)
    layer_ = QuantMoE(experts, fmt_gate_up=TSB_MXFP4, fmt_down=TSB_MXFP4, hidden=H, inter=I, top_k=top_k,
                      router_w=rw, router_b=rb, gate_up_layout="interleaved", activation="swiglu_oai", limit=limit,
                      alpha=alpha, pack=pack)
    layer_._storage = dev  # the per-expert views point into these buffers
    return layer_
