"""GGUF and safetensors parsing of tinyserve_b200.ingest on small files written
by tests/ingest_files.py (no GPU): metadata, tensor table, byte ranges of
fused and per-expert tensors, sharded safetensors indexes."""
from __future__ import annotations

import json

import numpy as np
import pytest

from tests.ingest_files import write_gguf, write_safetensors
from tinyserve_b200 import ingest
from tinyserve_b200.formats import GGML_F32, GGML_Q4_K, GGML_Q8_0, weight_bytes


def _rand_bytes(n, seed):
    return np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8).tobytes()


@pytest.mark.parametrize("alignment", [32, 64])
def test_gguf_fused_and_per_expert(tmp_path, alignment):
    H, I, E = 512, 256, 3
    ng, nd = weight_bytes(GGML_Q4_K, I, H), weight_bytes(GGML_Q8_0, H, I)
    gate, up, down = _rand_bytes(E * ng, 1), _rand_bytes(E * ng, 2), _rand_bytes(E * nd, 3)
    router = np.random.default_rng(4).standard_normal((E, H)).astype(np.float32)
    per = [(f"blk.1.ffn_gate.{e}.weight", (H, I), GGML_Q4_K, _rand_bytes(ng, 10 + e)) for e in range(E)]
    tensors = [("blk.0.ffn_gate_exps.weight", (H, I, E), GGML_Q4_K, gate),
               ("blk.0.ffn_up_exps.weight", (H, I, E), GGML_Q4_K, up),
               ("blk.0.ffn_down_exps.weight", (I, H, E), GGML_Q8_0, down),
               ("blk.0.ffn_gate_inp.weight", (H, E), GGML_F32, router.tobytes())] + per
    p = tmp_path / "m.gguf"
    write_gguf(p, tensors, {"general.architecture": ("str", "qwen3moe"), "qwen3moe.expert_used_count": ("u32", 2),
                            "tok.list": ("arr_u32", [1, 2, 3])}, alignment=alignment)
    f = ingest.GGUFFile(p)
    assert f.version == 3 and f.arch == "qwen3moe"
    assert f.metadata["qwen3moe.expert_used_count"] == 2 and f.metadata["tok.list"] == [1, 2, 3]
    assert f.data_offset % alignment == 0
    ex = f.expert_tensors(0)
    assert [o for _, o in ex["gate"]] == [0, ng, 2 * ng]
    for proj, blob, nb in (("gate", gate, ng), ("up", up, ng), ("down", down, nd)):
        for e, (t, o) in enumerate(ex[proj]):
            assert f.raw(t, o, nb).tobytes() == blob[e * nb:(e + 1) * nb]
    assert np.array_equal(f.raw("blk.0.ffn_gate_inp.weight").view(np.float32).reshape(E, H), router)
    ex1 = f.expert_tensors(1)
    assert list(ex1) == ["gate"] and [t.name for t, _ in ex1["gate"]] == [n for n, *_ in per]
    assert f.raw(ex1["gate"][2][0]).tobytes() == per[2][3]


def test_gguf_rejects_bad_files(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGUX" + b"\0" * 60)
    with pytest.raises(ValueError, match="not a GGUF"):
        ingest.GGUFFile(p)
    write_gguf(p, [("blk.0.ffn_gate_exps.weight", (32, 4, 2), 2, b"\0" * 72)])  # Q4_0: listed, not loadable
    f = ingest.GGUFFile(p)
    with pytest.raises(ValueError, match="no kernels"):
        f.raw("blk.0.ffn_gate_exps.weight")


def test_safetensors_single_and_sharded(tmp_path):
    a = np.arange(24, dtype=np.uint8).reshape(2, 3, 4)
    b = np.linspace(-1, 1, 6, dtype=np.float32).reshape(2, 3)
    write_safetensors(tmp_path / "one.safetensors", {"x.a": ("U8", a.shape, a.tobytes()),
                                                     "x.b": ("F32", b.shape, b.tobytes())})
    idx = ingest.SafetensorsIndex(tmp_path / "one.safetensors")
    raw, dt, shape = idx.raw("x.a")
    assert dt == "U8" and shape == (2, 3, 4) and raw.tobytes() == a.tobytes()
    d = tmp_path / "ckpt"
    d.mkdir()
    write_safetensors(d / "s1.safetensors", {"x.a": ("U8", a.shape, a.tobytes())})
    write_safetensors(d / "s2.safetensors", {"x.b": ("F32", b.shape, b.tobytes())})
    (d / "model.safetensors.index.json").write_text(json.dumps(
        {"weight_map": {"x.a": "s1.safetensors", "x.b": "s2.safetensors"}}))
    (d / "config.json").write_text(json.dumps({"num_experts_per_tok": 4}))
    idx = ingest.SafetensorsIndex(d)
    assert "x.b" in idx and idx.config["num_experts_per_tok"] == 4
    raw, dt, shape = idx.raw("x.b")
    assert np.array_equal(raw.view(np.float32).reshape(shape), b)
