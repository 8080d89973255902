"""The decode-step kernels of the whole-model path through the C-ABI against
float64 torch math: tsb_gqa_decode_attention (RoPE, cache store, grouped
sink attention over an e4m3 or bf16 cache, full and sliding windows, the
semantics of GPT-OSS eager attention with tinyserve's StaticKVCache) and
tsb_add_rmsnorm."""
from __future__ import annotations

import pytest
import torch

from tinyserve_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    return torch.device("cuda:0")


def _rope(x, c, s):
    a, b = x.chunk(2, dim=-1)
    return torch.cat((a * c - b * s, b * c + a * s), dim=-1)


@pytest.mark.parametrize("fp8", [True, False])
@pytest.mark.parametrize("pos,window", [(0, 0), (37, 0), (1000, 0), (1000, 128), (5, 128), (4095, 0)])
def test_gqa_decode_attention(dev, fp8, pos, window):
    nq, nkv, D, S = 64, 8, 64, 4096
    g = torch.Generator(device=dev).manual_seed(pos * 3 + window + fp8)
    qkv = torch.randn(nq + 2 * nkv, D, generator=g, device=dev).to(torch.bfloat16)
    ang = torch.arange(S, device=dev, dtype=torch.float32)[:, None] * (10000 ** (-torch.arange(D // 2, device=dev) / (D // 2)))
    cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
    kdt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    kc = (torch.randn(nkv, S, D, generator=g, device=dev) * 2).to(kdt)
    vc = torch.randn(nkv, S, D, generator=g, device=dev).to(kdt)
    sinks = torch.randn(nq, generator=g, device=dev)
    scale = D ** -0.5
    k_before, v_before = kc.clone(), vc.clone()
    out = torch.empty(nq, D, dtype=torch.bfloat16, device=dev)
    ws = torch.zeros(_lib.lib().tsb_gqa_decode_workspace(nq, nkv, S), dtype=torch.uint8, device=dev)
    p = torch.tensor([pos], dtype=torch.int64, device=dev)
    for _ in range(2):  # the counters reset themselves between calls
        kc.copy_(k_before), vc.copy_(v_before)
        _lib.check(_lib.lib().tsb_gqa_decode_attention(
            qkv.data_ptr(), nq, nkv, D, cos.data_ptr(), sin.data_ptr(), p.data_ptr(), kc.data_ptr(), vc.data_ptr(),
            int(fp8), S, window, sinks.data_ptr(), scale, out.data_ptr(), ws.data_ptr(), ws.numel(),
            torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
    # reference: rope in fp64 from the bf16 tables, the new key rounded to bf16 then to the cache type
    q = qkv[:nq].double()
    c, s = cos[pos].double(), sin[pos].double()
    q = _rope(q, c, s)
    knew = _rope(qkv[nq:nq + nkv].double(), c, s).to(torch.bfloat16).to(kdt)
    vnew = qkv[nq + nkv:].to(kdt)
    assert torch.equal(kc[:, pos].view(torch.uint8 if fp8 else torch.int16),
                       knew.view(torch.uint8 if fp8 else torch.int16))
    assert torch.equal(vc[:, pos].float(), vnew.float())
    others = torch.ones(S, dtype=torch.bool, device=dev)
    others[pos] = False
    assert torch.equal(kc[:, others].float(), k_before[:, others].float())
    K, V = kc.double(), vc.double()
    lo = max(0, pos - window + 1) if window else 0
    G = nq // nkv
    ref = torch.empty(nq, D, dtype=torch.float64, device=dev)
    for h in range(nq):
        kv = h // G
        sc = (K[kv, lo:pos + 1] @ q[h]) * scale
        m = torch.maximum(sc.max(), sinks[h].double())
        e = torch.exp(sc - m)
        ref[h] = (e @ V[kv, lo:pos + 1]) / (e.sum() + torch.exp(sinks[h].double() - m))
    err = ((out.double() - ref).norm() / ref.norm()).item()
    assert err < 6e-3, err  # bf16 output rounding (~2e-3) plus fp32 accumulation


def test_add_rmsnorm(dev):
    g = torch.Generator(device=dev).manual_seed(0)
    T, H = 3, 2880
    x = torch.randn(T, H, generator=g, device=dev)
    d = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    w = torch.randn(H, generator=g, device=dev)
    x0 = x.clone()
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.lib().tsb_add_rmsnorm(x.data_ptr(), d.data_ptr(), _lib.DT_BF16, w.data_ptr(), 1e-5, T, H,
                                          out.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    xr = x0.double() + d.double()
    assert torch.allclose(x.double(), xr, rtol=0, atol=1e-6)
    ref = w.double() * xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5)
    assert ((out.double() - ref).norm() / ref.norm()).item() < 4e-3


@pytest.mark.parametrize("N,K", [(5120, 2880), (2880, 4096), (77, 64), (3, 16384)])
def test_gemv_bf16(dev, N, K):
    g = torch.Generator(device=dev).manual_seed(N + K)
    W = (torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    b = torch.randn(N, generator=g, device=dev).to(torch.bfloat16)
    x = torch.randn(K, generator=g, device=dev).to(torch.bfloat16)
    y = torch.empty(N, dtype=torch.bfloat16, device=dev)
    for bias in (b, None):
        _lib.check(_lib.lib().tsb_gemv_bf16(W.data_ptr(), None if bias is None else bias.data_ptr(), N, K,
                                            x.data_ptr(), y.data_ptr(), torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        ref = W.double() @ x.double() + (0 if bias is None else bias.double())
        assert ((y.double() - ref).norm() / ref.norm()).item() < 4e-3


def test_norm_gemv_and_residual_gemv(dev):
    """tsb_norm_gemv_bf16 (RMSNorm of x_in + delta in front of the GEMV, the sum
    stored to x_out) and tsb_gemv_bf16_residual (resid += bf16(W x + b), then
    the last CTA's RMSNorm of resid), twice in a row (the counter resets)."""
    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device=dev).manual_seed(9)
    H, N1, K2 = 2880, 5120, 4096
    x_in = torch.randn(H, generator=g, device=dev)
    delta = torch.randn(H, generator=g, device=dev)
    nw = torch.rand(H, generator=g, device=dev) + 0.5
    W1 = (torch.randn(N1, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    b1 = torch.randn(N1, generator=g, device=dev).to(torch.bfloat16)
    x_out = torch.empty(H, device=dev)
    y = torch.empty(N1, dtype=torch.bfloat16, device=dev)
    _lib.check(L.tsb_norm_gemv_bf16(x_in.data_ptr(), delta.data_ptr(), x_out.data_ptr(), nw.data_ptr(), 1e-5,
                                    W1.data_ptr(), b1.data_ptr(), N1, H, y.data_ptr(), st))
    torch.cuda.synchronize()
    v = x_in.double() + delta.double()
    assert torch.allclose(x_out.double(), v, rtol=0, atol=1e-6)
    hn = (nw.double() * v * torch.rsqrt(v.pow(2).mean() + 1e-5)).to(torch.bfloat16).double()
    ref = W1.double() @ hn + b1.double()
    assert ((y.double() - ref).norm() / ref.norm()).item() < 4e-3
    W2 = (torch.randn(H, K2, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    b2 = torch.randn(H, generator=g, device=dev).to(torch.bfloat16)
    a = torch.randn(K2, generator=g, device=dev).to(torch.bfloat16)
    cnt = torch.zeros(1, dtype=torch.int32, device=dev)
    h = torch.empty(H, dtype=torch.bfloat16, device=dev)
    resid = x_out.clone()
    for it in range(2):
        before = resid.double().clone()
        _lib.check(L.tsb_gemv_bf16_residual(W2.data_ptr(), b2.data_ptr(), H, K2, a.data_ptr(), resid.data_ptr(),
                                            nw.data_ptr(), 1e-5, h.data_ptr(), cnt.data_ptr(), st))
        torch.cuda.synchronize()
        o = (W2.double() @ a.double() + b2.double())
        want = before + o.to(torch.bfloat16).double()
        assert ((resid.double() - want).norm() / want.norm()).item() < 1e-3
        hr = nw.double() * resid.double() * torch.rsqrt(resid.double().pow(2).mean() + 1e-5)
        assert ((h.double() - hr).norm() / hr.norm()).item() < 4e-3
        assert int(cnt.item()) == 0


@pytest.mark.parametrize("fp8", [True, False])
@pytest.mark.parametrize("pos,window", [(3, 0), (2000, 0), (2000, 128)])
def test_fused_norm_qkv_attention_matches_two_launches(dev, fp8, pos, window):
    """tsb_norm_qkv_attention (clusters per KV head, projections exchanged in
    distributed shared memory) against tsb_norm_gemv_bf16 followed by
    tsb_gqa_decode_attention on the same inputs: the residual and the cached
    key/value bytes identical, the attention output within bf16 rounding."""
    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    nq, nkv, D, H, S = 64, 8, 64, 2880, 4096
    g = torch.Generator(device=dev).manual_seed(pos + window + fp8)
    x_in = torch.randn(H, generator=g, device=dev)
    delta = torch.randn(H, generator=g, device=dev)
    nw = torch.rand(H, generator=g, device=dev) + 0.5
    W = (torch.randn((nq + 2 * nkv) * D, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    b = (torch.randn((nq + 2 * nkv) * D, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    ang = torch.arange(S, device=dev, dtype=torch.float32)[:, None] * (10000 ** (-torch.arange(D // 2, device=dev) / (D // 2)))
    cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
    kdt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    k0 = (torch.randn(nkv, S, D, generator=g, device=dev) * 2).to(kdt)
    v0 = torch.randn(nkv, S, D, generator=g, device=dev).to(kdt)
    sinks = torch.randn(nq, generator=g, device=dev)
    p = torch.tensor([pos], dtype=torch.int64, device=dev)
    # two launches
    kc1, vc1 = k0.clone(), v0.clone()
    x1 = torch.empty(H, device=dev)
    qkv = torch.empty((nq + 2 * nkv) * D, dtype=torch.bfloat16, device=dev)
    out1 = torch.empty(nq * D, dtype=torch.bfloat16, device=dev)
    ws = torch.zeros(L.tsb_gqa_decode_workspace(nq, nkv, S), dtype=torch.uint8, device=dev)
    _lib.check(L.tsb_norm_gemv_bf16(x_in.data_ptr(), delta.data_ptr(), x1.data_ptr(), nw.data_ptr(), 1e-5,
                                    W.data_ptr(), b.data_ptr(), W.shape[0], H, qkv.data_ptr(), st))
    _lib.check(L.tsb_gqa_decode_attention(qkv.data_ptr(), nq, nkv, D, cos.data_ptr(), sin.data_ptr(), p.data_ptr(),
                                          kc1.data_ptr(), vc1.data_ptr(), int(fp8), S, window, sinks.data_ptr(),
                                          D ** -0.5, out1.data_ptr(), ws.data_ptr(), ws.numel(), st))
    # one launch, twice (nothing carries over between calls)
    for _ in range(2):
        kc2, vc2 = k0.clone(), v0.clone()
        x2 = torch.empty(H, device=dev)
        out2 = torch.empty(nq * D, dtype=torch.bfloat16, device=dev)
        _lib.check(L.tsb_norm_qkv_attention(x_in.data_ptr(), delta.data_ptr(), x2.data_ptr(), nw.data_ptr(), 1e-5,
                                            W.data_ptr(), b.data_ptr(), H, nq, nkv, D, cos.data_ptr(), sin.data_ptr(),
                                            p.data_ptr(), kc2.data_ptr(), vc2.data_ptr(), int(fp8), S, window,
                                            sinks.data_ptr(), D ** -0.5, out2.data_ptr(), st))
        torch.cuda.synchronize()
        assert torch.equal(x2, x1)
        bt = torch.uint8 if fp8 else torch.int16
        assert torch.equal(kc2.view(bt), kc1.view(bt)) and torch.equal(vc2.view(bt), vc1.view(bt))
        err = ((out2.double() - out1.double()).norm() / out1.double().norm()).item()
        assert err < 5e-3, err
