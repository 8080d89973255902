"""Generate the golden fixtures in this directory from the reference itself.

Run in a container that has the tinyserve reference source (read-only):

    python tests/golden/make_golden.py /path/to/tinyserve-reference

It copies the reference package to a temporary directory without its compiled
Cython module (so ``expert_pipeline.py:36-52`` falls back to pure Python),
imports the reference's own decoders and CPU expert code, runs them on seeded
inputs and writes ``*.npz`` fixtures next to this script.  The GPU box never
runs this script; tests read only the committed ``.npz`` files.

Reference functions exercised (tinyserve file:line):
- gguf_dequant_torch.dequant_tensor           gguf_dequant_torch.py:35-78
- mxfp4.dequant_mxfp4_no_transpose            mxfp4.py:20-44
- cpu_expert.CPUExpertForward (fused, clamp-SwiGLU; separate, SiLU)
                                              cpu_expert.py:187-331
- ggml_forward.GGMLExpertForward._fallback_forward (CPU, SiLU)
                                              ggml_forward.py:117-151
- _model_hooks._extract_routing_fn (topk then softmax)
                                              _model_hooks.py:466-473
- expert_store.TensorLayout / _pack_tensors   expert_store.py:57-90
"""
from __future__ import annotations

import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from tinyserve_b200 import quantize as Q  # noqa: E402
from tinyserve_b200.formats import GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_Q8_0  # noqa: E402

BLOCK = {GGML_Q8_0: (32, 34), GGML_Q4_K: (256, 144), GGML_Q5_K: (256, 176), GGML_Q6_K: (256, 210)}


def _import_reference(src: Path):
    tmp = Path(tempfile.mkdtemp(prefix="tsref_"))
    shutil.copytree(src / "tinyserve", tmp / "tinyserve",
                    ignore=shutil.ignore_patterns("*.so", "__pycache__"))
    sys.path.insert(0, str(tmp))
    import tinyserve.gguf_dequant_torch as gdt  # noqa: F401
    return tmp


def _valid_blocks(fmt: int, nblocks: int, rng: np.random.Generator) -> np.ndarray:
    """Structurally valid blocks with finite fp16 scales (the style of
    tests/test_ggml_ops.py:139-184 in the reference)."""
    be, bb = BLOCK[fmt]
    raw = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    f16 = lambda lo, hi: np.float16(rng.uniform(lo, hi, size=nblocks)).view(np.uint8).reshape(nblocks, 2)  # noqa: E731
    if fmt == GGML_Q8_0:
        raw[:, 0:2] = f16(0.001, 0.1)
    elif fmt in (GGML_Q4_K, GGML_Q5_K):
        raw[:, 0:2] = f16(0.001, 0.1)
        raw[:, 2:4] = f16(0.001, 0.1)
    elif fmt == GGML_Q6_K:
        raw[:, 208:210] = f16(0.001, 0.1)
    return raw.reshape(-1)


def main(ref_root: str) -> None:
    _import_reference(Path(ref_root))
    from tinyserve.gguf_dequant_torch import dequant_tensor
    from tinyserve.mxfp4 import dequant_mxfp4_no_transpose
    from tinyserve.cpu_expert import CPUExpertForward
    from tinyserve.expert_store import TensorLayout, _pack_tensors
    from tinyserve.ggml_forward import GGMLExpertForward
    from tinyserve._model_hooks import _extract_routing_fn

    rng = np.random.default_rng(1234)
    gen = torch.Generator().manual_seed(0)

    # ---- GGUF decoders -------------------------------------------------
    dq = {}
    for fmt in (GGML_Q8_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K):
        be, bb = BLOCK[fmt]
        cases = {
            # random but finite scales, two superblocks' worth
            "valid": (_valid_blocks(fmt, 8 if be == 256 else 64, rng), None),
            # fully random bytes: NaN / Inf / subnormal fp16 scales included
            "random": (rng.integers(0, 256, size=(8 if be == 256 else 64) * bb, dtype=np.uint8), None),
            # the repo's encoder on N(0, 0.02), 4 rows of K=2880: K-quant
            # superblocks straddle rows (flat-stream rule)
            "enc_4x2880": (Q.quantize(fmt, torch.randn(4, 2880, generator=gen) * 0.02).numpy(), (4, 2880)),
        }
        for name, (raw, shape) in cases.items():
            n = raw.size // bb * be
            shape = shape or (n,)
            out = dequant_tensor(torch.from_numpy(raw.copy()), fmt, shape).numpy()
            dq[f"{fmt}_{name}_in"] = raw
            dq[f"{fmt}_{name}_out"] = out.astype(np.float32)
            dq[f"{fmt}_{name}_shape"] = np.array(shape, dtype=np.int64)
    np.savez_compressed(HERE / "dequant_gguf.npz", **dq)

    # ---- MXFP4 decoder -------------------------------------------------
    mx = {}
    blocks = rng.integers(0, 256, size=(8, 90, 16), dtype=np.uint8)
    for name, scales in {
        "kat_scales": rng.integers(120, 135, size=(8, 90), dtype=np.uint8),   # HF KAT range
        "full_scales": rng.integers(0, 256, size=(8, 90), dtype=np.uint8),    # incl. 255 (inf/nan) and 0
    }.items():
        b_t, s_t = torch.from_numpy(blocks.copy()), torch.from_numpy(scales.copy())
        mx[f"{name}_blocks"] = blocks
        mx[f"{name}_scales"] = scales
        mx[f"{name}_bf16"] = dequant_mxfp4_no_transpose(b_t, s_t, torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        mx[f"{name}_f32"] = dequant_mxfp4_no_transpose(b_t, s_t, torch.float32).numpy()
    np.savez_compressed(HERE / "dequant_mxfp4.npz", **mx)

    # ---- expert math ---------------------------------------------------
    ex = {}
    H, I, T = 256, 192, 3  # 2I != H so the reference does not transpose (cpu_expert.py:233-236)
    torch.manual_seed(5)
    wg = torch.randn(I, H) * 0.05
    wu = torch.randn(I, H) * 0.05
    wd = torch.randn(H, I) * 0.05
    h = torch.randn(T, H)
    gu = torch.stack([wg, wu], dim=1).reshape(2 * I, H)            # interleaved rows
    lay = TensorLayout({"gate_up_proj": ((2 * I, H), torch.float32), "down_proj": ((H, I), torch.float32)})
    packed = torch.empty(lay.total_bytes, dtype=torch.uint8)
    _pack_tensors(packed, lay, {"gate_up_proj": gu, "down_proj": wd})
    out_swiglu = CPUExpertForward(lay, act_fn=None, num_threads=1).forward(h, packed)
    # separate layout: the reference takes min(gate.shape) as the hidden size
    # (cpu_expert.py:246-249), so this case uses I2 > H.
    I2 = 512
    wg2 = torch.randn(I2, H) * 0.05
    wu2 = torch.randn(I2, H) * 0.05
    wd2 = torch.randn(H, I2) * 0.05
    lay_s = TensorLayout({"gate_proj": ((I2, H), torch.float32), "up_proj": ((I2, H), torch.float32),
                          "down_proj": ((H, I2), torch.float32)})
    packed_s = torch.empty(lay_s.total_bytes, dtype=torch.uint8)
    _pack_tensors(packed_s, lay_s, {"gate_proj": wg2, "up_proj": wu2, "down_proj": wd2})
    out_silu = CPUExpertForward(lay_s, act_fn=torch.nn.SiLU(), num_threads=1).forward(h, packed_s)
    ex.update(h=h.numpy(), w_gate=wg.numpy(), w_up=wu.numpy(), w_down=wd.numpy(),
              w_gate2=wg2.numpy(), w_up2=wu2.numpy(), w_down2=wd2.numpy(),
              out_swiglu=out_swiglu.numpy(), out_silu=out_silu.numpy(),
              layout_offsets=np.array([lay.offsets["gate_up_proj"], lay.offsets["down_proj"], lay.total_bytes]))

    # GGUF expert through the reference's as-shipped CPU path (SiLU, dequant per call)
    Hq, Iq = 256, 256
    qg = Q.quantize(GGML_Q4_K, torch.randn(Iq, Hq, generator=gen) * 0.02)
    qu = Q.quantize(GGML_Q4_K, torch.randn(Iq, Hq, generator=gen) * 0.02)
    qd = Q.quantize(GGML_Q8_0, torch.randn(Hq, Iq, generator=gen) * 0.02)
    lay_q = TensorLayout({"gate": ((qg.numel(),), torch.uint8), "up": ((qu.numel(),), torch.uint8),
                          "down": ((qd.numel(),), torch.uint8)})
    packed_q = torch.cat([qg, qu, qd])
    fwd = GGMLExpertForward(lay_q, {"gate": GGML_Q4_K, "up": GGML_Q4_K, "down": GGML_Q8_0},
                            torch.nn.SiLU(), {"gate": (Hq, Iq), "up": (Hq, Iq), "down": (Iq, Hq)})
    hq = torch.randn(2, Hq, generator=gen)
    out_gguf = fwd._fallback_forward(packed_q, hq)
    ex.update(gguf_packed=packed_q.numpy(), gguf_h=hq.numpy(), gguf_out=out_gguf.numpy(),
              gguf_dims=np.array([Hq, Iq]))

    # router: topk-then-softmax branch of _extract_routing_fn
    class _Blk(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.router = torch.nn.Linear(2880, 32, bias=False, dtype=torch.bfloat16)

    blk = _Blk()
    with torch.no_grad():
        blk.router.weight.copy_((torch.randn(32, 2880, generator=gen) * 0.02).to(torch.bfloat16))
    route = _extract_routing_fn(blk, "router", 4, "topk_then_softmax")
    hr = torch.randn(16, 2880, generator=gen).to(torch.bfloat16)
    with torch.no_grad():
        ids, wts = route(hr)
    ex.update(router_w=blk.router.weight.detach().view(torch.int16).numpy().view(np.uint16),
              router_h=hr.view(torch.int16).numpy().view(np.uint16),
              router_ids=ids.numpy(), router_wts=wts.float().numpy())
    np.savez_compressed(HERE / "expert.npz", **ex)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the tinyserve reference checkout>")
    main(sys.argv[1])
