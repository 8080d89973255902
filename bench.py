"""Benchmark of the quantized MoE expert hot path on B200.

Default workload: one GPT-OSS-20B-shaped MoE layer,
batch-1 decode, Q4_K experts (32 experts, top-4, clamp-SwiGLU), one fresh
seeded hidden vector per decode step.  A "step" is one token through the whole
layer (router -> top-4 -> gate/up -> SwiGLU -> down -> weighted combine).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

The same JSON line carries secondary measurements as flat scalar keys of
objects the driver record keeps: roofline.mxfp4_* (the config-1 shape with
MXFP4 experts), prefill (4096-token MXFP4 layer as grouped
tcgen05 GEMMs, TFLOP/s against the measured tensor peak), prefill.matvec_*
(rank 0: fraction of HBM peak per format and shape) and
prefill.ep_* (the GPT-OSS-120B-shaped layer sharded
expert-parallel over the ranks; decode T=1, T=64 and 4096-token prefill
tok/s, with the collectives and the local layer timed alone beside each).

N > 1 runs under torchrun, one process per GPU; every rank decodes its own
token stream through its own HBM-resident copy of the layer (the batch-1
decode path has no exchange step, so it scales as independent replicas;
"scaling": "weak").  Rank 0 prints one JSON line.

L2 hygiene: the layer is replicated NL times in HBM with different seeds and
consecutive steps cycle through the replicas, so a step's 56 MB of expert
weights were last touched >= NL-1 steps (>= 168 MB of traffic) earlier,
more than the 126 MB L2 holds.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "moe_layer_decode_tok_s"
UNIT = "tok/s"
NL = 4  # layer replicas cycled per step


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _dist():
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl")
    return ws, rank, local


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.out = None

    def __enter__(self):
        if self.idx < 0:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *a):
        if self.proc is None:
            return
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.out, _ = self.proc.communicate()

    def summary(self):
        if not self.out:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def build(fmt, device, seed_base: int):
    from tinyserve_b200.workloads import build_layer
    return [build_layer(fmt, seed=seed_base + i, device=device) for i in range(NL)]


def time_decode(layers, xs, K: int, W: int, dev, ws: int, clocks: bool):
    """K decode steps (token i through layer replica i % NL, the layer's own
    decode entry point) captured as one CUDA graph after W warm-up steps;
    returns (ms for the K steps, max over ranks; clock summary)."""
    import torch
    from tinyserve_b200 import _lib
    H, k = layers[0].hidden, layers[0].top_k
    n = max(K, W)
    outs = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
    ids = torch.empty(n, k, dtype=torch.int32, device=dev)
    wts = torch.empty(n, k, dtype=torch.float32, device=dev)
    st = torch.cuda.Stream(dev)

    def step(i):
        L = layers[i % NL]
        fn, lead = L._decode_call()
        rc = fn(*lead, xs[i].data_ptr(), 1, L.router_w.data_ptr(), None, ids[i].data_ptr(), wts[i].data_ptr(),
                outs[i].data_ptr(), L.workspace(1).data_ptr(), L.workspace(1).numel(), st.cuda_stream)
        _lib.check(rc)

    with torch.cuda.stream(st):
        for i in range(W):
            step(i)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for i in range(K):
                step(i)
    torch.cuda.synchronize()
    g.replay()  # warm the graph itself
    torch.cuda.synchronize()
    for L in layers:
        assert L.device_error() == 0
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index if clocks else -1) as clk:
        with torch.cuda.stream(st):
            e0.record(st)
            g.replay()
            e1.record(st)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if ws > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    for L in layers:
        assert L.device_error() == 0
    return ms, clk.summary()


def decode_roofline(layers, ms_step: float):
    """Algorithmic bytes of one token-layer (the four routed experts' quantised
    gate/up/down bytes + router + bf16 x in / out + fp32 activations between
    gate/up and down, written and read) and the achieved HBM rate."""
    from tinyserve_b200.workloads import layer_bytes
    expert_b, router_b = layer_bytes(layers[0])
    H, I, k = layers[0].hidden, layers[0].inter, layers[0].top_k
    step_bytes = k * expert_b + router_b + 2 * H * 2 + k * I * 4 * 2
    peak, peak_kind = _peaks()
    achieved = step_bytes / (ms_step * 1e-3) / 1e9
    return step_bytes, achieved, peak, peak_kind, expert_b


CONFIG1 = {"workload": "BASELINE config 1: GPT-OSS-20B-shaped MoE layer, batch-1 decode, Q4_K experts",
           "hidden": 2880, "inter": 2880, "experts": 32, "top_k": 4, "activation": "clamp-swiglu(7.0,1.702)",
           "gate_up": "separate", "weights": "seeded N(0,0.02) quantised to Q4_K by tinyserve_b200.quantize",
           "tokens": "workloads.hidden_states (seeded N(0,1) bf16), one fresh vector per step"}


def config1(ws: int) -> dict:
    """The workload description both arms print (identical at equal N)."""
    cfg = dict(CONFIG1)
    cfg.update({"global_batch": ws, "parallelism": f"replicas x{ws} (batch-1 decode has no exchange step)",
                "l2": f"inputs larger than L2: {NL} layer replicas of 448 MB of Q4_K experts cycled",
                "timing": "K steps after W warm-up steps, max over ranks"})
    return cfg


def run_ours(args, ws, rank, local):
    import torch
    from tinyserve_b200 import _lib
    from tinyserve_b200.formats import GGML_Q4_K
    from tinyserve_b200.workloads import hidden_states

    _lib.lib()  # fail loudly if the library is missing
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    layers = build(GGML_Q4_K, dev, seed_base=1000 * rank)
    K, W = args.steps, args.warmup
    xs = hidden_states(max(K, W), seed=rank, device=dev)
    ms, clocks = time_decode(layers, xs, K, W, dev, ws, clocks=True)

    # ---- end to end through the public API: pinned host in, host out, per step
    # (DecodeSession: per token one host row copy into pinned memory and one
    # graph replay of host->device copy, layer, device->host copy)
    from tinyserve_b200.moe import DecodeSession
    E2E = min(K, 200)
    xh = xs[:E2E].cpu()
    sess_stream = torch.cuda.Stream(dev)
    sessions = [DecodeSession(L, slots=4, stream=sess_stream) for L in layers]
    for i in range(8):
        sessions[i % NL].submit(xh[i % E2E])
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(sess_stream)
    last = None
    for i in range(E2E):
        last = (sessions[i % NL], sessions[i % NL].submit(xh[i]))
    a1.record(sess_stream)
    torch.cuda.synchronize()
    _ = last[0].result(last[1])
    e2e_ms = a0.elapsed_time(a1)
    if ws > 1:
        import torch.distributed as dist
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    ms_step = ms / K
    step_bytes, achieved, peak, peak_kind, expert_b = decode_roofline(layers, ms_step)
    cfg = config1(ws)
    res = {
        "metric": METRIC, "value": ws * K / (ms * 1e-3), "unit": UNIT, "n_gpus": ws, "steps": K, "warmup": W,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q4_k weights x int8 tensor path (16-bit fixed-point activations), fp32 fold",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) hidden)",
        "config": cfg,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_kind, "traffic": DECODE_TRAFFIC,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of pk_layer_kernel, one "
                                       "launch = one token-layer of this workload",
                     "unit_of_work": f"one token through one layer = {step_bytes} algorithmic bytes (4 routed "
                                     "experts' Q4_K gate/up/down + router + activations); the decode-packed copy "
                                     "the kernel streams adds the superblocks that straddle two rows and unit "
                                     "headers (~1.10x the Q4_K bytes at H = I = 2880)",
                     "kernel": "pk_layer_kernel<Q4_K>: one cooperative launch per token-layer (routing, gate/up, "
                               "SwiGLU, down, combine)",
                     "packed": bool(layers[0].packed)},
        "e2e": {"value": ws * E2E / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": 2880 * 2,
                "d2h_bytes_per_step": 2880 * 2,
                "how": "tinyserve_b200.moe.DecodeSession.submit per token (public API: host row -> pinned "
                       "buffer, one CUDA-graph replay of pinned host x -> device and the layer, which writes its "
                       "output into mapped pinned host memory), "
                       "4 layer replicas cycled, CUDA events on the session stream"},
        "gpu_launches": (1 if layers[0].packed else 3) * K,
        "clocks": clocks,
    }
    return res, layers, xs


def run_decode_mxfp4(dev, K: int, W: int, ws: int, rank: int):
    """The config-1 layer shape with GPT-OSS's native MXFP4 experts
    (interleaved gate_up, E8M0 scales): same timing as the headline."""
    from tinyserve_b200.formats import TSB_MXFP4
    from tinyserve_b200.workloads import hidden_states
    layers = build(TSB_MXFP4, dev, seed_base=2000 + 1000 * rank)
    xs = hidden_states(max(K, W), seed=rank, device=dev)
    ms, _ = time_decode(layers, xs, K, W, dev, ws, clocks=False)
    ms_step = ms / K
    step_bytes, achieved, peak, _, _ = decode_roofline(layers, ms_step)
    return {"metric": "moe_layer_decode_tok_s", "workload": "config-1 shape, MXFP4 experts (GPT-OSS format)",
            "value": ws * K / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms_step, "achieved": achieved,
            "peak": peak, "frac": achieved / peak, "algorithmic_bytes": step_bytes,
            "kernel": "pk_layer_kernel<MXFP4>"}


# DRAM bytes per launch of pk_layer_kernel<Q4_K> on this workload (ncu
# dram__bytes_read.sum + dram__bytes_write.sum, mean of 3 launches on the
# config-1 layer, captured with -k regex:pk_layer -s 10 -c 3):
# 62.2 MB read (the packed copy of 4 experts, 1.10x their Q4_K bytes), 0.15 MB
# written.
DECODE_TRAFFIC = 62.28e6

PREFILL_T = 4096


C3_CTX = 4096  # decode at context 4096


def _config3_breakdown(dec) -> dict:
    """Microseconds per layer of each launch of GptOssDecoder's step (and of
    the LM head per token): 24 calls of one kind captured in a CUDA graph on
    the decoder's own buffers at its current position, CUDA events around 3
    replays."""
    import torch
    import torch.nn.functional as F
    from tinyserve_b200 import _lib
    L = _lib.lib()
    fp8 = 1 if dec.kv_dtype == torch.float8_e4m3fn else 0

    def sid():
        return torch.cuda.current_stream(dec.device).cuda_stream

    def qkv():
        for lay in dec.layers:
            L.tsb_norm_gemv_bf16(dec._xa.data_ptr(), dec._y.data_ptr(), dec._xb.data_ptr(), lay["ln1"].data_ptr(),
                                 dec.eps, lay["wqkv"].data_ptr(), lay["bqkv"].data_ptr(), lay["wqkv"].shape[0], dec.H,
                                 dec._qkv.data_ptr(), sid())

    def attn():
        for li, lay in enumerate(dec.layers):
            L.tsb_gqa_decode_attention(dec._qkv.data_ptr(), dec.nq, dec.nkv, dec.D, dec.cos.data_ptr(),
                                       dec.sin.data_ptr(), dec._pos.data_ptr(), dec.k_cache[li].data_ptr(),
                                       dec.v_cache[li].data_ptr(), fp8, dec.max_seq,
                                       dec.window if dec.sliding[li] else 0, lay["sinks"].data_ptr(), dec.scale,
                                       dec._a.data_ptr(), dec._aws.data_ptr(), dec._aws.numel(), sid())

    def fused():
        for li, lay in enumerate(dec.layers):
            L.tsb_norm_qkv_attention(dec._xa.data_ptr(), dec._y.data_ptr(), dec._xb.data_ptr(), lay["ln1"].data_ptr(),
                                     dec.eps, lay["wqkv"].data_ptr(), lay["bqkv"].data_ptr(), dec.H, dec.nq, dec.nkv,
                                     dec.D, dec.cos.data_ptr(), dec.sin.data_ptr(), dec._pos.data_ptr(),
                                     dec.k_cache[li].data_ptr(), dec.v_cache[li].data_ptr(), fp8, dec.max_seq,
                                     dec.window if dec.sliding[li] else 0, lay["sinks"].data_ptr(), dec.scale,
                                     dec._a.data_ptr(), sid())

    def oproj():
        for lay in dec.layers:
            L.tsb_gemv_bf16_residual(lay["wo"].data_ptr(), lay["bo"].data_ptr(), dec.H, dec.nq * dec.D,
                                     dec._a.data_ptr(), dec._xb.data_ptr(), lay["ln2"].data_ptr(), dec.eps,
                                     dec._h.data_ptr(), dec._cnt.data_ptr(), sid())

    def experts():
        for lay in dec.layers:
            lay["moe"].decode(dec._h, out=dec._y)

    def head():
        F.linear(dec._h, dec.lm_head)

    res = {}
    st = torch.cuda.Stream(dec.device)
    for name, fn, per in (("qkv_norm_gemv", qkv, 24), ("attention", attn, 24),
                          ("norm_qkv_attention_fused", fused, 24), ("o_residual_gemv", oproj, 24),
                          ("expert_layer", experts, 24), ("lm_head", head, 1)):
        with torch.cuda.stream(st):
            fn()
            torch.cuda.synchronize(dec.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                fn()
            g.replay()
            torch.cuda.synchronize(dec.device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(3):
                g.replay()
            e1.record(st)
        torch.cuda.synchronize(dec.device)
        res[name] = e0.elapsed_time(e1) * 1e3 / 3 / per
        del g
    return res


def run_config3(dev, steps: int = 64, warmup: int = 8, ctx: int = C3_CTX):
    """the whole GPT-OSS-20B architecture (24 layers, 32
    MXFP4 experts, top-4, 64/8 heads of 64, alternating 128-token sliding and
    full attention, FP8 KV cache, vocabulary 201088), random init, batch-1
    greedy decode after a `ctx`-token prompt of seeded uniform-random ids.
    Decode = GptOssDecoder's per-token CUDA-graph replay (dense projections
    on cuBLAS, the expert layers on the library's decode-packed kernel);
    tokens are fed back on the device.  CUDA events around `steps` replays
    after `warmup`."""
    import torch
    from tinyserve_b200.gptoss import GptOssDecoder
    from tinyserve_b200.offload import load_and_offload
    t0 = time.time()
    lm = load_and_offload("gpt-oss-20b", device=str(dev), seed=0)
    build_s = time.time() - t0
    dec = GptOssDecoder(lm.model, lm.moe_layers, max_seq=ctx + steps + warmup + 8)
    prompt = torch.randint(0, lm.config.vocab_size, (ctx,), generator=torch.Generator().manual_seed(0)).to(dev)
    torch.cuda.synchronize(dev)
    t0 = time.time()
    logits = dec.prefill(prompt)
    torch.cuda.synchronize(dev)
    prefill_s = time.time() - t0
    tok = logits.argmax().reshape(1)
    for _ in range(warmup):
        tok = dec.step(tok)
    torch.cuda.synchronize(dev)
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        tok = dec.step(tok)
    e1.record(st)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    # bytes one decode step must read: every layer's 4 routed experts + router,
    # attention projections, the KV cache up to the context, final norm + LM head
    cfg = lm.config
    L, H, D = cfg.num_hidden_layers, cfg.hidden_size, cfg.head_dim
    q = lm.moe_layers[0]
    e0b = sum(t.numel() for t in (q.experts[0].gate, q.experts[0].down, q.experts[0].gate_scales,
                                  q.experts[0].down_scales))
    moe_b = L * (cfg.num_experts_per_tok * e0b + cfg.num_local_experts * H * 2)
    attn_b = L * 2 * H * (cfg.num_attention_heads + 2 * cfg.num_key_value_heads) * D + L * 2 * cfg.num_attention_heads * D * H
    ctx_mean = ctx + warmup + steps / 2
    kv_b = sum(2 * cfg.num_key_value_heads * D * (min(ctx_mean, cfg.sliding_window) if sl else ctx_mean)
               for sl in dec.sliding)
    head_b = cfg.vocab_size * H * 2
    alg = moe_b + attn_b + kv_b + head_b
    peak, src = _peaks()
    achieved = alg / (ms * 1e-3) / 1e9
    out = {"c3_decode_tok_s": 1e3 / ms, "c3_ms_per_token": ms, "c3_context": ctx, "c3_steps": steps,
           "c3_alg_bytes_per_token": alg, "c3_achieved_gbs": achieved, "c3_frac": achieved / peak,
           "c3_moe_bytes": moe_b, "c3_kv": "float8_e4m3fn", "c3_prefill_s": prefill_s, "c3_build_s": build_s,
           "c3_launch": "one CUDA graph per token",
           "c3_fused_qkv_attention": bool(dec._fused),
           "c3_errors": int(sum(q.device_error() for q in lm.moe_layers))}
    out.update({f"c3_us_{k}": v for k, v in _config3_breakdown(dec).items()})
    del dec
    torch.cuda.empty_cache()
    # several requests at once: 64 requests with 128-token prompts decoding in
    # lockstep through ServingEngine (batched attention over per-request FP8
    # cache slots, one expert-layer call per step with T = 64)
    from tinyserve_b200.serving import ServingEngine
    B, P, NEW = 64, 128, 24
    eng = ServingEngine(lm.model, lm.moe_layers, max_batch=B, max_seq=P + NEW + 8)
    g = torch.Generator().manual_seed(1)
    for _ in range(B):
        eng.submit(torch.randint(0, cfg.vocab_size, (P,), generator=g), NEW)
    eng.step()  # admits (prefills) every request and runs the first batched step
    for _ in range(3):
        eng.step()
    torch.cuda.synchronize(dev)
    n_steps = 16
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(n_steps):
        assert eng.step() == B
    e1.record(st)
    torch.cuda.synchronize(dev)
    ms_b = e0.elapsed_time(e1) / n_steps
    out.update({"c3_batch64_tok_s": B * 1e3 / ms_b, "c3_batch64_ms_per_step": ms_b,
                "c3_batch64": f"{B} requests x {P}-token prompts, greedy, ServingEngine.step (eager, one host sync "
                              "per step for the sampled tokens)"})
    del eng, lm
    torch.cuda.empty_cache()
    return out


def run_prefill(dev, steps: int = 10, warmup: int = 3):
    """one GPT-OSS-20B-shaped MXFP4 MoE layer, 4096 tokens,
    top-4 Zipf(1.1) routing over 32 experts; grouped GEMMs on tcgen05 including
    the on-GPU permute, weight decode and unpermute/combine.  Inputs (423 MB
    of expert weights, GBs of workspace) are larger than L2."""
    import torch
    from tinyserve_b200.formats import TSB_MXFP4
    from tinyserve_b200.workloads import build_layer, hidden_states, zipf_routing
    L = build_layer(TSB_MXFP4, seed=4, device=dev)
    ids, wts = zipf_routing(PREFILL_T, 32, 4, seed=0)
    ids, wts = ids.to(dev), wts.to(dev)
    x = hidden_states(PREFILL_T, seed=4, device=dev)
    out = torch.empty_like(x)
    st = torch.cuda.Stream(dev)
    with torch.cuda.stream(st):
        for _ in range(warmup):
            L.prefill(x, ids=ids, weights=wts, out=out)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            L.prefill(x, ids=ids, weights=wts, out=out)
        e1.record(st)
    torch.cuda.synchronize()
    assert L.prefill_error(PREFILL_T) == 0
    ms = e0.elapsed_time(e1) / steps
    flops = 2.0 * PREFILL_T * 4 * (2880 * 5760 + 2880 * 2880)
    tf = flops / (ms * 1e-3) / 1e12
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(peaks.get("bf16_tflops", 1590.0))
    rows = int(torch.bincount(ids.flatten().long(), minlength=32).add(127).div(128, rounding_mode="floor").sum()) * 128
    return {"metric": "moe_layer_prefill_tflops", "value": tf, "unit": "TFLOP/s", "ms_per_layer": ms, "steps": steps,
            "warmup": warmup, "tokens": PREFILL_T,
            "config": {"workload": "BASELINE config 4: GPT-OSS-20B-shaped MXFP4 MoE layer, 4096 tokens, top-4 Zipf(1.1) "
                                   "routing over 32 experts (seeded ids, softmax of N(0,1) weights)",
                       "dtype": "fp16 x fp16 -> fp32 on tcgen05 (MXFP4 weights decoded bit-exactly, rounded to fp16)",
                       "l2": "inputs larger than L2 (423 MB of expert weights, multi-GB workspace)"},
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                         "peak_source": "measured cuBLAS bf16 burst" if peaks else "fallback",
                         "unit_of_work": f"2*T*k*(H*2I + I*H) = {flops:.4g} flop per layer; {rows} padded rows "
                                         "(experts padded to 128-row blocks) run on the tensor cores",
                         "kernel": "whole layer: route + gather + weight tiles + 2 grouped GEMMs + combine"},
            "gpu_launches_per_layer": 8}


SWEEP_SHAPES = [(2880, 2880), (5760, 2880), (4096, 14336), (14336, 4096)]


def _reference_kernels():
    """The reference's own GPU matvec kernels for the same-box A/B, from the
    unmodified install in baseline/_ref (None for each that is absent):
    dot_scaled_vecmat (tinyserve/triton_dot_scaled.py:68-122, the MXFP4 decode
    kernel) and torch.ops.tinyserve_ggml.ggml_mul_mat_vec
    (tinyserve/csrc/ggml_ops.cu:461-574, built for sm_100a by
    baseline/build_ggml_ref.py)."""
    import torch
    ref = Path(__file__).resolve().parent / "baseline" / "_ref"
    dot_scaled = ggml = None
    why = []
    if (ref / "tinyserve").is_dir():
        sys.path.insert(0, str(ref))
        try:
            from tinyserve.triton_dot_scaled import dot_scaled_vecmat as dot_scaled
        except Exception as e:  # noqa: BLE001
            why.append(f"dot_scaled_vecmat: {type(e).__name__}: {e}"[:160])
    else:
        why.append("baseline/_ref not installed")
    so = sorted((ref / "ggml").glob("tinyserve_ggml*.so")) if (ref / "ggml").is_dir() else []
    if so:
        try:
            torch.ops.load_library(str(so[0]))
            ggml = torch.ops.tinyserve_ggml.ggml_mul_mat_vec
        except Exception as e:  # noqa: BLE001
            why.append(f"ggml_mul_mat_vec: {type(e).__name__}: {e}"[:160])
    else:
        why.append("ggml_ops extension not built (baseline/build_ggml_ref.py)")
    return dot_scaled, ggml, "; ".join(why)


def _graph_us(fn, calls: int, st) -> float:
    """Microseconds per call of `calls` calls of fn(i) captured in one CUDA
    graph (after 3 eager warm-up calls), CUDA events on the replay stream."""
    import torch
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=st):
            for i in range(calls):
                fn(i)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        e0.record(st)
        graph.replay()
        e1.record(st)
    torch.cuda.synchronize()
    del graph
    return e0.elapsed_time(e1) * 1e3 / calls


def run_matvec_sweep(dev, reps: int = 6, calls: int = 24):
    """tsb_quant_matvec on each format x shape, batch 1,
    weights N(0, 0.02) quantised per format, bf16 N(0, 1) activations.  Each
    timing is a CUDA graph of `calls` matvecs cycling over `reps` distinct
    matrices (at least 26 MB apart in the cycle, so the timed reads come
    from HBM for the large shapes), CUDA events.  The reference's own GPU
    kernel for the cell, where it has one, is timed the same way on the same
    matrices: the Triton dot_scaled_vecmat for MXFP4, ggml_mul_mat_vec for
    Q8_0 and for K-quants with K % 256 == 0 (it rejects K = 2880,
    tinyserve/csrc/ggml_ops.cu:476-479)."""
    import torch
    from tinyserve_b200 import ops
    from tinyserve_b200 import quantize as Q
    from tinyserve_b200.formats import GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_Q8_0, TSB_MXFP4
    peak, _ = _peaks()
    names = {GGML_Q8_0: "Q8_0", GGML_Q4_K: "Q4_K", GGML_Q5_K: "Q5_K", GGML_Q6_K: "Q6_K", TSB_MXFP4: "MXFP4"}
    dot_scaled, ggml, why = _reference_kernels()
    out = []
    st = torch.cuda.Stream(dev)
    for fmt in (GGML_Q8_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, TSB_MXFP4):
        for (N, K) in SWEEP_SHAPES:
            g = torch.Generator(device=dev).manual_seed(N * 31 + K + fmt)
            ws = []
            for _ in range(reps):
                w = torch.randn(N, K, generator=g, device=dev) * 0.02
                if fmt == TSB_MXFP4:
                    b, sc = Q.quantize_mxfp4(w, N, K)
                    ws.append((b.reshape(-1), sc.reshape(-1)))
                else:
                    ws.append((Q.quantize(fmt, w), None))
                del w
            x = torch.randn(1, K, generator=g, device=dev).to(torch.bfloat16)
            nbytes = ws[0][0].numel() + (ws[0][1].numel() if ws[0][1] is not None else 0)
            us = _graph_us(lambda i: ops.quant_matvec(fmt, ws[i % reps][0], ws[i % reps][1], N, K, x), calls, st)
            alg = nbytes + 2 * K + 2 * N  # weights + bf16 x + bf16 y
            gbs = alg / us / 1e3
            row = {"format": names[fmt], "rows": N, "cols": K, "us": us, "GB/s": gbs, "frac": gbs / peak}
            ref_fn, ref_name = None, None
            if fmt == TSB_MXFP4 and dot_scaled is not None:
                mats = [(b.view(N, K // 32, 16), sc.view(N, K // 32)) for b, sc in ws]
                ref_fn, ref_name = (lambda i: dot_scaled(x, *mats[i % reps])), "triton dot_scaled_vecmat"
            elif fmt != TSB_MXFP4 and ggml is not None and (fmt == GGML_Q8_0 or K % 256 == 0):
                ref_fn, ref_name = (lambda i: ggml(x, ws[i % reps][0], fmt, N, K)), "ggml_mul_mat_vec"
            if ref_fn is not None:
                try:
                    # same inputs, outputs compared before timing
                    mine = ops.quant_matvec(fmt, ws[0][0], ws[0][1], N, K, x).float()
                    theirs = ref_fn(0).float().reshape(mine.shape)
                    rel = float((mine - theirs).norm() / theirs.norm().clamp_min(1e-30))
                    rus = _graph_us(ref_fn, calls, st)
                    row.update({"ref_kernel": ref_name, "ref_us": rus, "ref_GB/s": alg / rus / 1e3,
                                "speedup_vs_ref": rus / us, "rel_l2_vs_ref": rel})
                except Exception as e:  # noqa: BLE001
                    row.update({"ref_kernel": ref_name, "ref_error": f"{type(e).__name__}: {e}"[:200]})
            out.append(row)
            del ws
    torch.cuda.empty_cache()
    return {"metric": "quant_matvec_hbm_gbs", "unit": "GB/s", "peak": peak, "peak_source": "measured copy",
            "config": {"workload": "BASELINE config 2: batch-1 quantised matvec sweep (5 formats x 4 shapes)",
                       "timing": f"CUDA graph of {calls} calls over {reps} distinct matrices, CUDA events",
                       "reference_kernels": why or "dot_scaled_vecmat and ggml_mul_mat_vec loaded"},
            "results": out}


EP_T = 4096  # prefill tokens per rank per layer call (weak scaling)
EP_DECODE_T = (1, 64)  # decode tokens per rank per layer call


def _ep_time(call, steps: int, warmup: int, ws: int, dev) -> float:
    """ms per call: CUDA events on the current stream around `steps` calls
    after a barrier, max over ranks."""
    import torch
    for _ in range(warmup):
        call()
    torch.cuda.synchronize()
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        call()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if ws > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def _ep_graphed(call, dev):
    """`call` captured once into a CUDA graph (a decode-sized layer call is
    launch-bound when issued eagerly from Python); returns (replay, "graph"),
    or (call, "eager") when capture is refused."""
    import torch
    try:
        st = torch.cuda.Stream(dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(st):
            call()
        torch.cuda.current_stream(dev).wait_stream(st)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            call()
        torch.cuda.synchronize()
        return g.replay, "graph"
    except Exception as e:  # noqa: BLE001 - reported in the bench line
        torch.cuda.synchronize()
        return call, f"eager ({type(e).__name__})"


def run_ep(dev, ws: int, rank: int, steps: int = 5, warmup: int = 3):
    """GPT-OSS-120B-shaped MXFP4 layer (128 experts, top-4,
    H = I = 2880) sharded expert-parallel over the ranks (128/N experts each),
    every rank routing its own tokens (seeded N(0,1), router bf16 N(0,0.02)).

    Legs (each: tokens of all ranks / max-over-ranks time of one layer call):
    decode T=1 and T=64 per rank through ``forward_gather`` (all-gather of
    tokens and routing, local experts with other ranks' slots skipped, fp32
    reduce-scatter; no host synchronisation), and the 4096-token prefill
    through both schemes (``forward_gather`` and the all-to-all ``forward``).
    Beside each EP leg: the same collectives alone (``comm_ms``) and the local
    layer alone on the gathered rows (``local_ms``), which name the limiter.
    Every leg also runs through the C-ABI (``native_*``: tsb_ep_moe_decode /
    tsb_ep_moe_prefill on an NCCL communicator, router included), issued
    eagerly.  At N = 1 the whole layer runs on one GPU with no exchange (its
    decode legs captured in a CUDA graph)."""
    import torch
    from tinyserve_b200.formats import TSB_MXFP4
    from tinyserve_b200.moe import QuantMoE, Router
    from tinyserve_b200.workloads import build_layer, gen_normal, hidden_states
    E, k, H = 128, 4, 2880
    el = E // ws
    # only this rank's experts are built (seeded per rank)
    part = build_layer(TSB_MXFP4, n_experts=el, top_k=k, seed=5000 + rank, device=dev)
    router = Router(gen_normal((E, H), 77, 0.02, dev).to(torch.bfloat16), k)
    res = {"n_gpus": ws, "experts_per_gpu": el, "timing": "CUDA events around eager layer calls, max over ranks"}
    legs = [("decode_t1", 1, 50), ("decode_t64", 64, 30), ("prefill", EP_T, steps)]
    if ws == 1:
        whole = QuantMoE(part.experts, fmt_gate_up=TSB_MXFP4, fmt_down=TSB_MXFP4, hidden=H, inter=H, top_k=k,
                         router_w=router.router_w, gate_up_layout="interleaved")
        for name, T, n in legs:
            x = hidden_states(T, seed=100 + rank, device=dev)
            fn, how = (lambda: whole.decode(x)), "eager"
            if T <= 64:
                fn, how = _ep_graphed(fn, dev)
            ms = _ep_time(fn, n, warmup, ws, dev)
            res[f"{name}_tok_s"] = T / (ms * 1e-3)
            res[f"{name}_ms"] = ms
            res[f"{name}_launch"] = how
        res["exchange"] = "none (all 128 experts on one GPU)"
        return res
    import torch.distributed as dist
    from tinyserve_b200.ep import ExpertParallelMoE, NativeEPDecode, NcclComm, quant_layer_forward, quant_local_forward
    local1 = QuantMoE(part.experts, fmt_gate_up=TSB_MXFP4, fmt_down=TSB_MXFP4, hidden=H, inter=H, top_k=1,
                      gate_up_layout="interleaved", pack=False)
    lf = quant_layer_forward(part)
    gather = ExpertParallelMoE(E, k, H, router=router, layer_forward=lf)
    a2a = ExpertParallelMoE(E, k, H, quant_local_forward(local1), router=router)
    nccl = NcclComm()
    keep = []
    for name, T, n in legs:
        x = hidden_states(T, seed=100 + rank, device=dev)
        ms = _ep_time(lambda: gather.forward_gather(x), n, warmup, ws, dev)
        res[f"{name}_tok_s"] = ws * T / (ms * 1e-3)
        res[f"{name}_ms"] = ms
        # the collectives alone, same sizes
        xa = torch.empty(ws * T, H, dtype=torch.bfloat16, device=dev)
        ma = torch.empty(ws * T, 2 * k, dtype=torch.float32, device=dev)
        meta = torch.zeros(T, 2 * k, dtype=torch.float32, device=dev)
        pa = torch.zeros(ws * T, H, dtype=torch.float32, device=dev)
        o = torch.empty(T, H, dtype=torch.float32, device=dev)

        def coll():
            dist.all_gather_into_tensor(xa, x)
            dist.all_gather_into_tensor(ma, meta)
            dist.reduce_scatter_tensor(o, pa)
        res[f"{name}_comm_ms"] = _ep_time(coll, n, warmup, ws, dev)
        res[f"{name}_comm_mb"] = (xa.numel() * 2 + ma.numel() * 4 + pa.numel() * 4) * (ws - 1) / ws / 1e6
        # the local layer alone on gathered rows with this rank's share of slots
        ids, w = router(hidden_states(ws * T, seed=900 + rank, device=dev))
        lid = ids - rank * el
        lid = torch.where((lid >= 0) & (lid < el), lid, torch.full_like(lid, -1))
        xg = hidden_states(ws * T, seed=901, device=dev)
        res[f"{name}_local_ms"] = _ep_time(lambda: lf(xg, lid, w), n, warmup, 1, dev)
        if name != "prefill":
            nat = NativeEPDecode(part, nccl, T)
            fn, how = (lambda: nat(x, *router(x))), "eager"
            ms = _ep_time(fn, n, warmup, ws, dev)
            res[f"native_{name}_tok_s"] = ws * T / (ms * 1e-3)
            res[f"native_{name}_ms"] = ms
            res[f"native_{name}_launch"] = how
            keep.append((fn, nat))  # graphs released before the communicator
        if name == "prefill":
            nat = NativeEPDecode(part, nccl, T, prefill=True)
            ms = _ep_time(lambda: nat(x, *router(x)), n, warmup, ws, dev)
            res["native_prefill_tok_s"] = ws * T / (ms * 1e-3)
            res["native_prefill_ms"] = ms
            keep.append(nat)
            ms = _ep_time(lambda: a2a(x), n, warmup, ws, dev)
            res["prefill_a2a_tok_s"] = ws * T / (ms * 1e-3)
            res["prefill_a2a_ms"] = ms
        del xa, ma, pa
        torch.cuda.empty_cache()
    torch.cuda.synchronize()
    keep.clear()
    import gc
    gc.collect()
    nccl.close()
    res["exchange"] = ("forward_gather: NCCL all_gather_into_tensor (bf16 tokens + routing) and reduce_scatter_tensor "
                       "(fp32 partials); prefill_a2a: NCCL all_to_all_single with uneven splits")
    return res


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def cpu_decode(host_experts, router, xs, threads: int, warmup: int = 3):
    """The reference's CPU expert path (oracle port of CPUExpertForward, no
    product code) over the token rows of xs (bf16 [n, H] on the host).  The
    experts the sample routes to are decoded once before timing (the
    reference caches its CPU conversions); returns (tokens/s over the timed
    tokens, experts decoded)."""
    import time
    import torch
    from oracle.cpu_expert_port import CPUMoELayer, gguf_expert_fetcher
    from tinyserve_b200.formats import GGML_Q4_K

    def host_bytes(e):
        ex = host_experts[e]
        return ex["gate"], ex["up"], ex["down"]

    fetch = gguf_expert_fetcher(host_bytes, GGML_Q4_K, GGML_Q4_K, 2880, 2880)
    cpu = CPUMoELayer(fetch, router, 4, threads)
    torch.set_num_threads(threads)
    with torch.no_grad():
        cpu.prefetch(sorted({int(e) for i in range(xs.shape[0]) for e in cpu.route(xs[i:i + 1])[0][0]}))
        for i in range(min(warmup, xs.shape[0])):
            cpu.forward(xs[i:i + 1])
        t0 = time.perf_counter()
        for i in range(xs.shape[0]):
            cpu.forward(xs[i:i + 1])
        dt = time.perf_counter() - t0
    return xs.shape[0] / dt, len(cpu._cache)


def _reference_cpu():
    """The installed reference's CPU modules (baseline/_ref, unmodified), or
    None when it is not installed: cpu_expert (CPUExpertForward,
    tinyserve/cpu_expert.py:180-331), gguf_dequant_torch.dequant_tensor,
    expert_store.TensorLayout, _model_hooks._extract_routing_fn and
    ggml_forward.GGMLExpertForward."""
    ref = Path(__file__).resolve().parent / "baseline" / "_ref"
    if not (ref / "tinyserve").is_dir():
        return None
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    import tinyserve._model_hooks as mh
    import tinyserve.cpu_expert as ce
    import tinyserve.expert_store as es
    import tinyserve.ggml_forward as gf
    import tinyserve.gguf_dequant_torch as gd
    return {"ce": ce, "gd": gd, "es": es, "mh": mh, "gf": gf}


def _ref_route(R, router_bf16, top_k: int):
    """The reference's top-k-then-softmax routing function over a bf16 Linear."""
    import torch
    blk = torch.nn.Module()
    blk.router = torch.nn.Linear(router_bf16.shape[1], router_bf16.shape[0], bias=False, dtype=torch.bfloat16)
    with torch.no_grad():
        blk.router.weight.copy_(router_bf16)
    return R["mh"]._extract_routing_fn(blk, "router", top_k, "topk_then_softmax")


def ref_cpu_decode(R, host_experts, router, xs, threads: int, fmt: int, warmup: int = 3, H: int = 2880,
                   I: int = 2880):
    """One MoE layer per token through the reference's own CPU expert path
    (baseline/_ref): routing by _extract_routing_fn, each routed expert by
    CPUExpertForward (Q4_K: weights decoded once by dequant_tensor into the
    fused fp32 layout, gate_up [2I, H] interleaved and down stored [I, H] as
    the reference's transpose rule reads a square down projection; MXFP4: the
    MXFP4 layout, converted once to torch INT4 by its CPUINT4Forward), and
    out += w * y.  Expert conversion happens before timing (the reference
    caches it).  Returns (tokens/s, experts converted)."""
    import time
    import torch
    from tinyserve_b200.formats import GGML_Q4_K, TSB_MXFP4
    torch.set_num_threads(threads)
    route = _ref_route(R, router, 4)
    es, ce, gd = R["es"], R["ce"], R["gd"]
    fwds: dict[int, tuple] = {}

    def expert(e: int):
        if e in fwds:
            return fwds[e]
        ex = host_experts[e]
        if fmt == GGML_Q4_K:
            wg = gd.dequant_tensor(torch.from_numpy(ex["gate"]), GGML_Q4_K, (I, H))
            wu = gd.dequant_tensor(torch.from_numpy(ex["up"]), GGML_Q4_K, (I, H))
            wd = gd.dequant_tensor(torch.from_numpy(ex["down"]), GGML_Q4_K, (H, I))
            gu = torch.stack([wg, wu], 1).reshape(2 * I, H).float().contiguous()
            dn = wd.float().t().contiguous()
            lay = es.TensorLayout({"gate_up_proj": ((2 * I, H), torch.float32), "down_proj": ((I, H), torch.float32)})
            packed = torch.cat([gu.view(-1).view(torch.uint8), dn.view(-1).view(torch.uint8)])
        elif fmt == TSB_MXFP4:
            t = {"gate_up_proj": torch.from_numpy(ex["gate"]).view(2 * I, H // 32, 16),
                 "gate_up_proj_scales": torch.from_numpy(ex["gate_scales"]).view(2 * I, H // 32),
                 "down_proj": torch.from_numpy(ex["down"]).view(H, I // 32, 16),
                 "down_proj_scales": torch.from_numpy(ex["down_scales"]).view(H, I // 32)}
            lay = es.TensorLayout.from_tensors(t)
            packed = torch.cat([v.contiguous().view(-1) for v in t.values()])
        else:
            raise ValueError(fmt)
        f = ce.CPUExpertForward(lay, act_fn=None, num_threads=threads)
        fwds[e] = (f, packed)
        return fwds[e]

    def layer(h):
        ids, w = route(h)
        hf = h.float() if fmt == GGML_Q4_K else h
        out = torch.zeros(h.shape, dtype=torch.float32)
        for k in range(ids.shape[1]):
            f, packed = expert(int(ids[0, k]))
            out += float(w[0, k]) * f.forward(hf, packed).float()
        return out

    with torch.no_grad():
        for i in range(xs.shape[0]):
            for e in route(xs[i:i + 1])[0][0]:
                f, packed = expert(int(e))
                if fmt == TSB_MXFP4:
                    f.forward(xs[:1], packed)  # the INT4 conversion, cached by the reference
        for i in range(min(warmup, xs.shape[0])):
            layer(xs[i:i + 1])
        t0 = time.perf_counter()
        for i in range(xs.shape[0]):
            layer(xs[i:i + 1])
        dt = time.perf_counter() - t0
    return xs.shape[0] / dt, len(fwds)


def ref_cpu_gguf_fallback(R, host_experts, router, xs, threads: int, H: int = 2880, I: int = 2880):
    """The reference's as-shipped GGUF CPU path: GGMLExpertForward._fallback_forward
    (tinyserve/ggml_forward.py:117-151), which decodes the expert's bytes with
    dequant_tensor on every call and runs F.linear with SiLU; tokens/s of one
    layer (4 routed experts) over the rows of xs."""
    import time
    import torch
    from tinyserve_b200.formats import GGML_Q4_K
    torch.set_num_threads(threads)
    route = _ref_route(R, router, 4)
    n = host_experts[0]["gate"].size
    lay = R["es"].TensorLayout({"gate": ((n,), torch.uint8), "up": ((n,), torch.uint8), "down": ((n,), torch.uint8)})
    fwd = R["gf"].GGMLExpertForward(lay, {"gate": GGML_Q4_K, "up": GGML_Q4_K, "down": GGML_Q4_K}, torch.nn.SiLU(),
                                    {"gate": (H, I), "up": (H, I), "down": (I, H)})
    packs = {}
    with torch.no_grad():
        fwd._fallback_forward(torch.from_numpy(
            __import__("numpy").concatenate([host_experts[0][k] for k in ("gate", "up", "down")])), xs[:1].float())
        t0 = time.perf_counter()
        for i in range(xs.shape[0]):
            h = xs[i:i + 1]
            ids, w = route(h)
            out = torch.zeros(h.shape, dtype=torch.float32)
            for k in range(ids.shape[1]):
                e = int(ids[0, k])
                if e not in packs:
                    import numpy as np
                    packs[e] = torch.from_numpy(np.concatenate([host_experts[e][j] for j in ("gate", "up", "down")]))
                out += float(w[0, k]) * fwd._fallback_forward(packs[e], h.float())
        dt = time.perf_counter() - t0
    return xs.shape[0] / dt


def host_layer(seed: int, device):
    """Config-1 expert bytes and router on the host, generated with plain
    torch (the same seeded values as the GPU arm's replica `seed`); no
    product library involved."""
    from tinyserve_b200.formats import GGML_Q4_K
    from tinyserve_b200.workloads import layer_weights
    experts, router, _ = layer_weights(GGML_Q4_K, seed=seed, device=device)
    host = [{k: v.cpu().numpy() for k, v in e.items()} for e in experts]
    return host, router.cpu()


def cpu_baselines(host, router_cpu, xs, dev) -> dict:
    """The reference's CPU expert path timed on this box's host cores (rank 0,
    N = 1), on bounded samples of the bench's workloads: the headline Q4_K
    config-1 layer (40 tokens of the GPU arm's stream), GPT-OSS's MXFP4 experts
    through the reference's INT4 CPU path (4 tokens), and the as-shipped GGUF
    fallback that decodes every expert on every call (2 tokens).  The
    installed reference runs when present (kind "reference"), else the oracle
    port of CPUExpertForward (kind "port", Q4_K only)."""
    from tinyserve_b200.formats import GGML_Q4_K, TSB_MXFP4
    from tinyserve_b200.workloads import hidden_states, layer_weights
    threads = len(os.sched_getaffinity(0))
    n = 40
    R = _reference_cpu()
    xq = xs[:n].cpu()
    if R is None:
        tps, nexp = cpu_decode(host, router_cpu, xq, threads)
        return {"value": tps, "unit": UNIT, "cores": threads, "kind": "port", "cpu_model": cpu_model(),
                "sample": f"{n} tokens of the same stream through replica 0 ({nexp} experts decoded once before "
                          "timing; oracle port of CPUExpertForward)"}
    tps, nexp = ref_cpu_decode(R, host, router_cpu, xq, threads, GGML_Q4_K)
    out = {"value": tps, "unit": UNIT, "cores": threads, "kind": "reference", "cpu_model": cpu_model(),
           "sample": f"{n} tokens of the same stream through replica 0 ({nexp} experts decoded once by "
                     "dequant_tensor before timing; the installed reference's CPUExpertForward)"}
    mx, mrouter, _ = layer_weights(TSB_MXFP4, seed=2000, device=dev)
    mhost = [{k: v.cpu().numpy() for k, v in e.items()} for e in mx]
    del mx
    xm = hidden_states(4, seed=0, device=dev).cpu()
    mtps, mexp = ref_cpu_decode(R, mhost, mrouter.cpu(), xm, threads, TSB_MXFP4, warmup=1)
    out["mxfp4_int4_tok_s"] = mtps
    out["mxfp4_int4_sample"] = (f"4 tokens, MXFP4 config-1 shape ({mexp} experts converted to torch INT4 before "
                                "timing; the reference's CPUINT4Forward)")
    out["gguf_fallback_tok_s"] = ref_cpu_gguf_fallback(R, host, router_cpu, xs[:2].cpu(), threads)
    out["gguf_fallback_sample"] = ("2 tokens through GGMLExpertForward._fallback_forward (dequant_tensor of each "
                                   "routed expert on every call, SiLU)")
    return out


def run_reference(args, ws, rank, local):
    """--impl reference: the reference's CPU expert path on the host cores,
    same metric and config: the first K tokens of the GPU arm's token stream
    through its replica-0 layer.  Runs the unmodified reference installed in
    baseline/_ref (CPUExpertForward, dequant_tensor, its routing function:
    kind "reference"); without the install, the oracle port of the same code
    (kind "port").  Weights and tokens come from plain torch (CUDA RNG when a
    GPU is present, so the values match the GPU arm's); nothing of the
    product runs."""
    import torch
    if rank != 0:
        return None
    threads = len(os.sched_getaffinity(0))
    dev = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    from tinyserve_b200.formats import GGML_Q4_K
    from tinyserve_b200.workloads import hidden_states
    host, router = host_layer(0, dev)
    xs = hidden_states(args.steps, seed=0, device=dev).cpu()
    R = _reference_cpu()
    if R is not None:
        tps, nexp = ref_cpu_decode(R, host, router, xs, threads, GGML_Q4_K, warmup=args.warmup)
        kind, what = "reference", "the installed reference's CPUExpertForward (baseline/_ref)"
    else:
        tps, nexp = cpu_decode(host, router, xs, threads, warmup=args.warmup)
        kind, what = "port", "oracle port of CPUExpertForward (baseline/_ref not installed)"
    cfg = config1(ws)
    sample = (f"{args.steps} tokens of the GPU arm's stream through its replica-0 layer ({nexp} experts decoded "
              f"once before timing); {what}; {threads} threads on {cpu_model()}")
    return {"impl": "reference", "metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 / tps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32 (weights decoded once by dequant_tensor)",
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) hidden)", "config": cfg,
            "cpu_baseline": {"value": tps, "unit": UNIT, "cores": threads, "kind": kind, "sample": sample,
                             "cpu_model": cpu_model()},
            "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-4 prefill measurement")
    ap.add_argument("--prefill-only", action="store_true",
                    help="run only the config-4 prefill leg (--steps layers after --warmup) and print its object")
    ap.add_argument("--config3-only", action="store_true",
                    help="run only the config-3 whole-model decode (GPT-OSS-20B, context 4096) and print its object")
    ap.add_argument("--sweep-only", action="store_true",
                    help="run only the config-2 matvec sweep (with the reference-kernel A/B) and print its object")
    ap.add_argument("--ep-only", action="store_true",
                    help="run only the config-5 expert-parallel legs and print their object")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    ws, rank, local = _dist()
    if args.impl == "reference":
        res = run_reference(args, ws, rank, local)
        if rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
        return
    if args.ep_only:
        import torch
        ep = run_ep(torch.device("cuda", local), ws, rank)
        if rank == 0:
            print(json.dumps(ep), flush=True)
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.config3_only:
        import torch
        c3 = run_config3(torch.device("cuda", local))
        if rank == 0:
            print(json.dumps(c3), flush=True)
        return
    if args.sweep_only:
        import torch
        sw = run_matvec_sweep(torch.device("cuda", local))
        if rank == 0:
            print(json.dumps(sw), flush=True)
        return
    if args.prefill_only:
        import torch
        from tinyserve_b200 import _lib
        _lib.lib()
        pf = run_prefill(torch.device("cuda", local), steps=args.steps, warmup=args.warmup)
        if rank == 0:
            print(json.dumps(pf), flush=True)
        return
    res, layers, xs = run_ours(args, ws, rank, local)
    import torch
    dev = torch.device("cuda", local)
    host = None
    if rank == 0 and not args.no_cpu_baseline and ws == 1:
        host = [{k: getattr(layers[0].experts[e], k).cpu().numpy() for k in ("gate", "up", "down")}
                for e in range(32)]
        router_cpu = layers[0].router_w.cpu()
    del layers
    torch.cuda.empty_cache()
    if not args.no_prefill:
        # secondary measurements ride as flat scalar keys of objects the
        # driver record keeps (nested objects are dropped from it)
        mx = run_decode_mxfp4(dev, min(args.steps, 200), args.warmup, ws, rank)
        res["roofline"].update({"mxfp4_tok_s": mx["value"], "mxfp4_us_per_step": mx["ms_per_step"] * 1e3,
                                "mxfp4_achieved": mx["achieved"], "mxfp4_frac": mx["frac"]})
        torch.cuda.empty_cache()
        pf = run_prefill(dev)
        torch.cuda.empty_cache()
        if rank == 0:
            for r in run_matvec_sweep(dev)["results"]:
                pf[f"matvec_{r['format']}_{r['rows']}x{r['cols']}_frac"] = round(r["frac"], 4)
                if "speedup_vs_ref" in r:
                    pf[f"matvec_{r['format']}_{r['rows']}x{r['cols']}_vs_ref"] = round(r["speedup_vs_ref"], 3)
        torch.cuda.empty_cache()
        ep = run_ep(dev, ws, rank)
        torch.cuda.empty_cache()
        pf.update({f"ep_{k}": (round(v, 4) if isinstance(v, float) else v) for k, v in ep.items()})
        if rank == 0 and ws == 1:
            # BASELINE config 3 (whole GPT-OSS-20B decode at context 4096) and a
            # 64-request serving step, on the single-GPU run
            pf.update(run_config3(dev))
            torch.cuda.empty_cache()
        res["prefill"] = pf
    if host is not None:
        res["cpu_baseline"] = cpu_baselines(host, router_cpu, xs, dev)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
