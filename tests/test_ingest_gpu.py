"""Checkpoint files straight into HBM expert tables (tinyserve_b200.ingest):
a GGUF file with fused Q4_K / Q6_K expert tensors and a sharded GPT-OSS
MXFP4 safetensors checkpoint, loaded and run through the layer, against
float64 oracle math on the same bytes."""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from oracle import expert as OE
from tests.helpers import assert_layer, make_weight, oracle_dequant
from tests.ingest_files import bf16_bytes, write_gguf, write_safetensors
from tinyserve_b200 import ingest
from tinyserve_b200.formats import GGML_F32, GGML_Q4_K, GGML_Q6_K, TSB_MXFP4

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    return torch.device("cuda:0")


def test_gguf_fused_experts_layer(dev, tmp_path):
    H, I, E, k, T = 512, 256, 4, 2, 3
    g = [make_weight(GGML_Q4_K, I, H, 100 + e)[0] for e in range(E)]
    u = [make_weight(GGML_Q4_K, I, H, 200 + e)[0] for e in range(E)]
    d = [make_weight(GGML_Q6_K, H, I, 300 + e)[0] for e in range(E)]
    router = (np.random.default_rng(0).standard_normal((E, H)) * 0.02).astype(np.float32)
    cat = lambda ts: b"".join(t.numpy().tobytes() for t in ts)  # noqa: E731
    p = tmp_path / "moe.gguf"
    write_gguf(p, [("blk.0.ffn_gate_exps.weight", (H, I, E), GGML_Q4_K, cat(g)),
                   ("blk.0.ffn_up_exps.weight", (H, I, E), GGML_Q4_K, cat(u)),
                   ("blk.0.ffn_down_exps.weight", (I, H, E), GGML_Q6_K, cat(d)),
                   ("blk.0.ffn_gate_inp.weight", (H, E), GGML_F32, router.tobytes())],
               {"general.architecture": ("str", "mixtral"), "mixtral.expert_used_count": ("u32", k)})
    layer = ingest.load_gguf_moe(p, 0, device=dev)
    assert layer.top_k == k and (layer.hidden, layer.inter) == (H, I)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    out, ids, wts = layer.decode(x.to(dev), out_dtype=torch.float32)
    torch.cuda.synchronize()
    rb = torch.from_numpy(router).to(torch.bfloat16).float().numpy()
    r_ids, _, _ = OE.router_topk_softmax(x.float().numpy(), rb, k)
    ids_c, wts_c = ids.cpu().numpy(), wts.cpu().numpy()
    assert (np.sort(ids_c, 1) == np.sort(r_ids, 1)).all()
    deq = [(oracle_dequant(GGML_Q4_K, g[e], None, I, H), oracle_dequant(GGML_Q4_K, u[e], None, I, H),
            oracle_dequant(GGML_Q6_K, d[e], None, H, I)) for e in range(E)]
    ref = np.zeros((T, H))
    for t in range(T):
        for j in range(k):
            wg, wu, wd = deq[ids_c[t, j]]
            ref[t] += wts_c[t, j] * OE.expert_forward(x[t:t + 1].float().numpy(), wg, wu, wd, "silu")[0]
    assert_layer(out, ref)
    assert layer.device_error(T) == 0


def test_safetensors_mxfp4_sharded_layer(dev, tmp_path):
    H, I, E, k, T = 512, 256, 4, 2, 2
    gub, gus, dnb, dns = [], [], [], []
    for e in range(E):
        b, s = make_weight(TSB_MXFP4, 2 * I, H, 400 + e)
        gub.append(b.numpy()), gus.append(s.numpy())
        b, s = make_weight(TSB_MXFP4, H, I, 500 + e)
        dnb.append(b.numpy()), dns.append(s.numpy())
    rng = np.random.default_rng(7)
    gu_bias = (rng.standard_normal((E, 2 * I)) * 0.1).astype(np.float32)
    dn_bias = (rng.standard_normal((E, H)) * 0.1).astype(np.float32)
    rw = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    rbias = (rng.standard_normal(E) * 0.1).astype(np.float32)
    pre = "model.layers.3.mlp"
    d = tmp_path / "ckpt"
    d.mkdir()
    write_safetensors(d / "a.safetensors", {
        f"{pre}.experts.gate_up_proj_blocks": ("U8", (E, 2 * I, H // 32, 16), np.stack(gub).tobytes()),
        f"{pre}.experts.gate_up_proj_scales": ("U8", (E, 2 * I, H // 32), np.stack(gus).tobytes()),
        f"{pre}.experts.gate_up_proj_bias": ("BF16", (E, 2 * I), bf16_bytes(gu_bias))})
    write_safetensors(d / "b.safetensors", {
        f"{pre}.experts.down_proj_blocks": ("U8", (E, H, I // 32, 16), np.stack(dnb).tobytes()),
        f"{pre}.experts.down_proj_scales": ("U8", (E, H, I // 32), np.stack(dns).tobytes()),
        f"{pre}.experts.down_proj_bias": ("BF16", (E, H), bf16_bytes(dn_bias)),
        f"{pre}.router.weight": ("BF16", (E, H), bf16_bytes(rw)),
        f"{pre}.router.bias": ("BF16", (E,), bf16_bytes(rbias))})
    wm = {n: "a.safetensors" for n in (f"{pre}.experts.gate_up_proj_blocks", f"{pre}.experts.gate_up_proj_scales",
                                       f"{pre}.experts.gate_up_proj_bias")}
    wm.update({n: "b.safetensors" for n in (f"{pre}.experts.down_proj_blocks", f"{pre}.experts.down_proj_scales",
                                            f"{pre}.experts.down_proj_bias", f"{pre}.router.weight",
                                            f"{pre}.router.bias")})
    (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wm}))
    (d / "config.json").write_text(json.dumps({"num_experts_per_tok": k}))
    layer = ingest.load_safetensors_mxfp4_moe(d, 3, device=dev)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    out, ids, wts = layer.decode(x.to(dev), out_dtype=torch.float32)
    torch.cuda.synchronize()
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16).double().numpy()  # noqa: E731
    ids_c, wts_c = ids.cpu().numpy(), wts.cpu().numpy()
    r_ids, _, _ = OE.router_topk_softmax(x.float().numpy(), bf(rw), k, bias=bf(rbias))
    assert (np.sort(ids_c, 1) == np.sort(r_ids, 1)).all()
    ref = np.zeros((T, H))
    for t in range(T):
        for j in range(k):
            e = ids_c[t, j]
            wgu = oracle_dequant(TSB_MXFP4, gub[e], gus[e], 2 * I, H)
            wd = oracle_dequant(TSB_MXFP4, dnb[e], dns[e], H, I)
            b = bf(gu_bias[e])
            y = OE.expert_forward(x[t:t + 1].float().numpy(), wgu[0::2], wgu[1::2], wd, "swiglu_oai",
                                  b[0::2], b[1::2], bf(dn_bias[e]))
            ref[t] += wts_c[t, j] * y[0]
    assert_layer(out, ref)
    assert layer.device_error(T) == 0
