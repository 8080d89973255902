"""GPU parity of the grouped (prefill) MoE layer, tsb_moe_prefill, against
float64 math on the oracle-dequantised weights.

The reference's batched path groups tokens by expert and runs one expert
forward per group (tinyserve/expert_pipeline.py:166-239); its tests check the
grouped result against the per-token loop (tests/test_batched_prefill.py:52-119).
Here every case is checked against the exact per-token sum.  Products run in
fp16 with fp32 accumulation, so the layer math stays within 1e-3 relative L2
(fp32 outputs); bf16 outputs may add their own rounding on top of the 1e-3
(tests.helpers.layer_bound).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import expert as OE
from tests.helpers import assert_layer, rel_l2
from tests.test_kernels_gpu import _build_layer
from tinyserve_b200.formats import GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_Q8_0, TSB_MXFP4

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    return torch.device("cuda:0")


def _oracle(x, ids, wts, dense, act="swiglu_oai"):
    """Per-expert grouped float64 forward; out[t] = sum_j w[t,j] * expert(x[t])."""
    x = np.asarray(x, dtype=np.float64)
    out = np.zeros_like(x)
    for e in np.unique(ids):
        if e < 0 or e >= len(dense):
            continue
        tok, kk = np.nonzero(ids == e)
        wg, wu, wd, bg, bu, bd = dense[e]
        y = OE.expert_forward(x[tok], wg, wu, wd, act, None if bg is None else bg.numpy(),
                              None if bu is None else bu.numpy(), None if bd is None else bd.numpy())
        np.add.at(out, tok, wts[tok, kk][:, None] * y)
    return out


def _routing(T, E, k, seed):
    from tinyserve_b200.workloads import zipf_routing
    return zipf_routing(T, E, k, seed=seed)


@pytest.mark.parametrize("fmt_gu,fmt_dn,layout", [
    (GGML_Q4_K, GGML_Q4_K, "separate"),
    (TSB_MXFP4, TSB_MXFP4, "interleaved"),
    (GGML_Q8_0, GGML_Q6_K, "separate"),
    (GGML_Q5_K, GGML_Q8_0, "chunked"),
])
def test_prefill_layer_formats(dev, fmt_gu, fmt_dn, layout):
    H, I, E, k, T = 512, 256, 8, 2, 300
    layer, dense, _ = _build_layer(dev, fmt_gu, fmt_dn, H, I, E, k, layout, seed=fmt_gu * 7 + fmt_dn)
    ids, wts = _routing(T, E, k, seed=1)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    out, _, _ = layer.prefill(x.to(dev), ids=ids, weights=wts)
    torch.cuda.synchronize()
    ref = _oracle(x.float().numpy(), ids.numpy(), wts.numpy(), dense)
    assert_layer(out, ref)
    assert layer.prefill_error(T) == 0


def test_prefill_gpt_oss_shape_with_bias(dev):
    """H = I = 2880 (N tiles of 240 rows, 45 k-blocks), MXFP4 with biases,
    Zipf routing so that some experts get several 128-row blocks."""
    H = I = 2880
    E, k, T = 8, 4, 384
    layer, dense, _ = _build_layer(dev, TSB_MXFP4, TSB_MXFP4, H, I, E, k, "interleaved", seed=11, bias=True)
    ids, wts = _routing(T, E, k, seed=2)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    out, _, _ = layer.prefill(x.to(dev), ids=ids, weights=wts)
    torch.cuda.synchronize()
    ref = _oracle(x.float().numpy(), ids.numpy(), wts.numpy(), dense)
    assert_layer(out, ref)
    per_tok = np.linalg.norm(out.float().cpu().numpy() - ref, axis=1) / np.linalg.norm(ref, axis=1)
    assert per_tok.max() <= 3e-2


def test_prefill_router_matches_oracle_routing(dev):
    H, I, E, k, T = 1024, 512, 16, 4, 200
    layer, dense, router = _build_layer(dev, GGML_Q4_K, GGML_Q8_0, H, I, E, k, "separate", seed=21)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    out, ids, wts = layer.prefill(x.to(dev))
    torch.cuda.synchronize()
    ids_o, wts_o, lg = OE.router_topk_softmax(x.float().numpy(), router.float().numpy(), k)
    ids_g = ids.cpu().numpy()
    for t in range(T):
        if set(ids_g[t]) != set(ids_o[t]):
            srt = np.sort(lg[t])[::-1]
            assert abs(srt[k - 1] - srt[k]) <= 1e-2 * abs(srt[k - 1]) + 1e-6, "routing differs away from a tie"
    ref = _oracle(x.float().numpy(), ids_g, wts.cpu().numpy(), dense)
    assert_layer(out, ref)


def test_prefill_one_token_matches_decode(dev):
    H, I, E, k = 1024, 512, 8, 4
    layer, _, _ = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, E, k, "separate", seed=31)
    x = torch.randn(1, H, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16).to(dev)
    o1, ids1, w1 = layer.decode(x)
    o2, ids2, w2 = layer.prefill(x)
    torch.cuda.synchronize()
    assert torch.equal(ids1.cpu(), ids2.cpu())
    assert rel_l2(o2.float().cpu().numpy(), o1.float().cpu().numpy()) <= 4e-3


def test_prefill_unused_experts_and_all_to_one(dev):
    """Every token on expert 3 (several row blocks) and some experts unused."""
    H, I, E, k, T = 256, 128, 6, 1, 513
    layer, dense, _ = _build_layer(dev, GGML_Q8_0, GGML_Q8_0, H, I, E, k, "separate", seed=41)
    ids = torch.full((T, k), 3, dtype=torch.int32)
    wts = torch.ones(T, k)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16)
    out, _, _ = layer.prefill(x.to(dev), ids=ids, weights=wts)
    ref = _oracle(x.float().numpy(), ids.numpy(), wts.numpy(), dense)
    assert_layer(out, ref)


def test_prefill_row_scaling_wide_dynamic_range(dev):
    """Token rows of very different magnitudes (1e-6 .. 1e4) keep their own
    relative accuracy: each row is scaled by a power of two into fp16 range."""
    H, I, E, k, T = 512, 256, 4, 2, 64
    layer, dense, _ = _build_layer(dev, TSB_MXFP4, TSB_MXFP4, H, I, E, k, "interleaved", seed=51)
    ids, wts = _routing(T, E, k, seed=4)
    g = torch.Generator().manual_seed(8)
    mags = torch.tensor([1e-6, 1e-3, 1.0, 30.0, 1e4]).repeat(T // 5 + 1)[:T]
    x = (torch.randn(T, H, generator=g) * mags[:, None] * 0.05).to(torch.bfloat16)
    out, _, _ = layer.prefill(x.to(dev), ids=ids, weights=wts)
    ref = _oracle(x.float().numpy(), ids.numpy(), wts.numpy(), dense)
    got = out.float().cpu().numpy()
    for t in range(T):
        assert rel_l2(got[t], ref[t]) <= 2e-2, t


def test_prefill_deterministic(dev):
    H, I, E, k, T = 512, 256, 8, 4, 777
    layer, _, _ = _build_layer(dev, GGML_Q4_K, GGML_Q6_K, H, I, E, k, "separate", seed=61)
    ids, wts = _routing(T, E, k, seed=5)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16).to(dev)
    a, _, _ = layer.prefill(x, ids=ids, weights=wts)
    b, _, _ = layer.prefill(x, ids=ids, weights=wts)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_prefill_bad_ids_reported(dev):
    H, I, E, k, T = 256, 128, 4, 2, 40
    layer, dense, _ = _build_layer(dev, GGML_Q4_K, GGML_Q4_K, H, I, E, k, "separate", seed=71)
    ids, wts = _routing(T, E, k, seed=6)
    ids[5, 1] = 1000
    ids[7, 0] = -3
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(10)).to(torch.bfloat16)
    out, _, _ = layer.prefill(x.to(dev), ids=ids, weights=wts)
    torch.cuda.synchronize()
    assert layer.prefill_error(T) == 2
    ref = _oracle(x.float().numpy(), ids.numpy(), wts.numpy(), dense)
    assert_layer(out, ref)
    assert layer.prefill_error(T) == 0


@pytest.mark.parametrize("layout", ["separate", "chunked"])
def test_prefill_mxfp4_half_k_blocks(dev, layout):
    """MXFP4 decoded inside the GEMM with H and I odd multiples of 32 (the last
    64-wide k-block holds one 32-block) and non-interleaved gate/up."""
    H, I, E, k, T = 288, 160, 5, 2, 150
    layer, dense, _ = _build_layer(dev, TSB_MXFP4, TSB_MXFP4, H, I, E, k, layout, seed=81, bias=True)
    ids, wts = _routing(T, E, k, seed=8)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(11)).to(torch.bfloat16)
    out, _, _ = layer.prefill(x.to(dev), ids=ids, weights=wts)
    ref = _oracle(x.float().numpy(), ids.numpy(), wts.numpy(), dense)
    assert_layer(out, ref)


def test_prefill_mxfp4_extreme_scales(dev):
    """E8M0 scale bytes far from the usual range (2^-27 and 2^13) take the
    fp32 route of the in-kernel decode and still match."""
    from tinyserve_b200.moe import ExpertWeights, QuantMoE
    from tests.helpers import make_weight, oracle_dequant
    H, I, E, k, T = 256, 128, 3, 1, 64
    experts, dense = [], []
    for e in range(E):
        gu, gus = make_weight(TSB_MXFP4, 2 * I, H, 900 + e)
        dn, dns = make_weight(TSB_MXFP4, H, I, 950 + e)
        gus = gus.clone()
        gus.view(-1)[::7] = 100
        gus.view(-1)[3::11] = 140
        wgu = oracle_dequant(TSB_MXFP4, gu, gus, 2 * I, H)
        wd = oracle_dequant(TSB_MXFP4, dn, dns, H, I)
        experts.append(ExpertWeights(gate=gu.to(dev), down=dn.to(dev), gate_scales=gus.to(dev),
                                     down_scales=dns.to(dev)))
        dense.append((wgu[0::2], wgu[1::2], wd, None, None, None))
    layer = QuantMoE(experts, fmt_gate_up=TSB_MXFP4, fmt_down=TSB_MXFP4, hidden=H, inter=I, top_k=k,
                     gate_up_layout="interleaved")
    ids, wts = _routing(T, E, k, seed=9)
    x = (torch.randn(T, H, generator=torch.Generator().manual_seed(12)) * 1e-3).to(torch.bfloat16)
    out, _, _ = layer.prefill(x.to(dev), ids=ids, weights=wts)
    ref = _oracle(x.float().numpy(), ids.numpy(), wts.numpy(), dense)
    assert_layer(out, ref)


def test_prefill_mxfp4_tiled_decode_subprocess(dev):
    """The cases of this file are small enough that MXFP4 weights are decoded
    inside the GEMM by default; TSB_PREFILL_FUSED=0 (read once per process)
    forces the decode-once fp16 tiles that large batches use, and the MXFP4
    cases pass on that path too."""
    import os
    import subprocess
    import sys
    env = dict(os.environ, TSB_PREFILL_FUSED="0")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", __file__, "-k", "mxfp4 and not subprocess"],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


def test_prefill_cta_pair_subprocess(dev):
    """TSB_PREFILL_PAIR=1 runs the tiled GEMMs on CTA pairs (tcgen05
    cta_group::2, experts padded to 256 rows); with TSB_PREFILL_FUSED=0 every
    format takes the tiled path, so all cases of this file cover the pair
    kernel."""
    import os
    import subprocess
    import sys
    env = dict(os.environ, TSB_PREFILL_FUSED="0", TSB_PREFILL_PAIR="1")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", __file__, "-k", "not subprocess"],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


@pytest.mark.parametrize("fmt_gu,layout", [(GGML_Q4_K, "separate"), (TSB_MXFP4, "interleaved")])
def test_prefill_fp32_output(dev, fmt_gu, layout):
    """fp32 output: the grouped layer itself within the north-star 1e-3."""
    H, I, E, k, T = 1024, 512, 8, 4, 200
    layer, dense, _ = _build_layer(dev, fmt_gu, fmt_gu, H, I, E, k, layout, seed=61)
    ids, wts = _routing(T, E, k, seed=5)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(61)).to(torch.bfloat16)
    out, _, _ = layer.prefill(x.to(dev), ids=ids.to(dev), weights=wts.to(dev), out_dtype=torch.float32)
    assert out.dtype == torch.float32
    ref = _oracle(x.float().numpy(), ids.numpy(), wts.numpy(), dense)
    assert_layer(out, ref)


def test_prefill_config4_full_shape(dev):
    """BASELINE config 4 as bench.py runs it: the GPT-OSS-20B-shaped MXFP4
    layer (32 experts, H = I = 2880, interleaved gate/up) from
    workloads.build_layer, 4096 tokens with top-4 Zipf(1.1) routing, on the
    path the bench takes (tiled weights).  The whole output is computed on the
    GPU; the oracle checks a seeded sample of 256 tokens (fp32 output, 1e-3)."""
    from tests.helpers import oracle_dequant
    from tinyserve_b200.workloads import build_layer, hidden_states, zipf_routing
    T = 4096
    layer = build_layer(TSB_MXFP4, seed=4, device=dev)
    ids, wts = zipf_routing(T, 32, 4, seed=0)
    x = hidden_states(T, seed=4, device=dev)
    out, _, _ = layer.prefill(x, ids=ids.to(dev), weights=wts.to(dev), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert layer.prefill_error(T) == 0
    sample = np.sort(np.random.default_rng(0).choice(T, 256, replace=False))
    xs = x.cpu().float().numpy()[sample]
    idl, wl = ids.numpy()[sample], wts.numpy()[sample]
    dense = {}
    for e in np.unique(idl):
        ex = layer.experts[int(e)]
        gu = oracle_dequant(TSB_MXFP4, ex.gate.cpu(), ex.gate_scales.cpu(), 2 * 2880, 2880)
        wd = oracle_dequant(TSB_MXFP4, ex.down.cpu(), ex.down_scales.cpu(), 2880, 2880)
        dense[int(e)] = (gu[0::2], gu[1::2], wd, None, None, None)
    ref = np.zeros_like(xs, dtype=np.float64)
    for e, (wg, wu, wd, _, _, _) in dense.items():
        tok, kk = np.nonzero(idl == e)
        ref[tok] += wl[tok, kk][:, None] * OE.expert_forward(xs[tok], wg, wu, wd)
    assert_layer(out[torch.from_numpy(sample).to(dev)], ref)


@pytest.mark.parametrize("E,T", [(128, 1), (128, 3), (32, 64), (128, 257)])
def test_standalone_router_matches_oracle(dev, E, T):
    """tsb_moe_route (the router of the grouped path and of expert
    parallelism), including the GPT-OSS-120B expert count, against the
    oracle's routing; near-ties may order differently."""
    from tinyserve_b200.moe import Router
    H, k = 2880, 4
    g = torch.Generator().manual_seed(E + T)
    w = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    b = torch.randn(E, generator=g) * 0.01
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    ids, wts = Router(w.to(dev), k, b.to(dev))(x.to(dev))
    torch.cuda.synchronize()
    ids_o, wts_o, lg = OE.router_topk_softmax(x.float().numpy(), w.float().numpy(), k, bias=b.double().numpy())
    ids_g, wts_g = ids.cpu().numpy(), wts.cpu().numpy()
    for t in range(T):
        if list(ids_g[t]) != list(ids_o[t]):
            srt = np.sort(lg[t])[::-1]
            assert abs(srt[k - 1] - srt[k]) <= 1e-2 * abs(srt[k - 1]) + 1e-6, "routing differs away from a tie"
        else:
            np.testing.assert_allclose(wts_g[t], wts_o[t], rtol=2e-6, atol=1e-7)
