"""Worker of tests/test_ep_gpu.py, run under torchrun (one process per GPU,
NCCL): the layer's experts are split over the ranks, every rank routes its own
tokens, and the sharded result is compared with the whole layer on one GPU and
with the oracle layer (float64 on the reference-dequantised weights).

Both exchange schemes run: the all-to-all dispatch (``forward``, any T per
rank, bf16 expert outputs on the wire) and the all-gather / reduce-scatter
decode scheme (``forward_gather``, fp32 partial sums, fp32 output)."""
from __future__ import annotations

import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from tests.helpers import assert_layer, make_weight, oracle_dequant, rel_l2  # noqa: E402
from tests.test_kernels_gpu import _oracle_layer  # noqa: E402
from tinyserve_b200.ep import (ExpertParallelMoE, NativeEPDecode, NcclComm, quant_layer_forward,  # noqa: E402
                               quant_local_forward)
from tinyserve_b200.formats import TSB_MXFP4  # noqa: E402
from tinyserve_b200.moe import ExpertWeights, QuantMoE, Router  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl")
    H, I, E, k = 512, 256, 8, 2
    experts = []
    for e in range(E):
        gu, gus = make_weight(TSB_MXFP4, 2 * I, H, 500 + e)
        dn, dns = make_weight(TSB_MXFP4, H, I, 600 + e)
        experts.append(ExpertWeights(gate=gu.to(dev), down=dn.to(dev), gate_scales=gus.to(dev), down_scales=dns.to(dev)))
    router_w = (torch.randn(E, H, generator=torch.Generator().manual_seed(7)) * 0.02).to(torch.bfloat16).to(dev)
    full = QuantMoE(experts, fmt_gate_up=TSB_MXFP4, fmt_down=TSB_MXFP4, hidden=H, inter=I, top_k=k,
                    gate_up_layout="interleaved")
    el = E // world
    mine = QuantMoE(experts[rank * el:(rank + 1) * el], fmt_gate_up=TSB_MXFP4, fmt_down=TSB_MXFP4, hidden=H, inter=I,
                    top_k=1, gate_up_layout="interleaved")
    ep = ExpertParallelMoE(E, k, H, quant_local_forward(mine), router=Router(router_w, k))
    worst = 0.0
    for T in (3 + 5 * rank, 300 + 40 * rank, 0 if rank == 0 else 20):
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(1000 * rank + T)).to(torch.bfloat16).to(dev)
        out = ep(x)
        if T:
            ids, w = Router(router_w, k)(x)
            ref, _, _ = full.decode(x, ids=ids, weights=w)
            torch.cuda.synchronize()
            err = rel_l2(out.float().cpu().numpy(), ref.float().cpu().numpy())
            worst = max(worst, err)
            assert err <= 1e-2, (rank, T, err)
    # decode scheme: same T on every rank, fp32 output
    mine_k = QuantMoE(experts[rank * el:(rank + 1) * el], fmt_gate_up=TSB_MXFP4, fmt_down=TSB_MXFP4, hidden=H,
                      inter=I, top_k=k, gate_up_layout="interleaved")
    epg = ExpertParallelMoE(E, k, H, router=Router(router_w, k), layer_forward=quant_layer_forward(mine_k))
    dense = {}
    for e in range(E):
        ex = experts[e]
        gu = oracle_dequant(TSB_MXFP4, ex.gate.cpu(), ex.gate_scales.cpu(), 2 * I, H)
        wd = oracle_dequant(TSB_MXFP4, ex.down.cpu(), ex.down_scales.cpu(), H, I)
        dense[e] = (gu[0::2], gu[1::2], wd, None, None, None)
    for T in (1, 4, 24):
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(5000 + 100 * rank + T)).to(torch.bfloat16).to(dev)
        out = epg.forward_gather(x, out_dtype=torch.float32)
        ids, w = Router(router_w, k)(x)
        ref, _, _ = full.decode(x, ids=ids, weights=w, out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert out.dtype == torch.float32 and out.shape == (T, H)
        err = rel_l2(out.cpu().numpy(), ref.cpu().numpy())
        worst = max(worst, err)
        assert err <= 1e-4, (rank, T, err)  # the same kernels, summed in another order
        idn, wn = ids.cpu().numpy(), w.cpu().numpy()
        for t in range(min(T, 4)):
            assert_layer(out[t], _oracle_layer(x[t:t + 1].float().cpu().numpy(), list(idn[t]), list(wn[t]), dense))
    assert mine_k.device_error(1) == 0
    # the same scheme through the C-ABI (tsb_ep_moe_decode on an NCCL communicator)
    comm = NcclComm()
    for T in (1, 4, 24):
        nat = NativeEPDecode(mine_k, comm, T)
        for step in range(2):
            x = torch.randn(T, H, generator=torch.Generator().manual_seed(7000 + 100 * rank + 10 * T + step))
            x = x.to(torch.bfloat16).to(dev)
            ids, w = Router(router_w, k)(x)
            out = nat(x, ids, w, out_dtype=torch.float32)
            out_b = nat(x, ids, w)
            ref, _, _ = full.decode(x, ids=ids, weights=w, out_dtype=torch.float32)
            torch.cuda.synchronize()
            err = rel_l2(out.cpu().numpy(), ref.cpu().numpy())
            worst = max(worst, err)
            assert err <= 1e-4, ("native", rank, T, err)
            assert torch.equal(out_b, out.to(torch.bfloat16))
            idn, wn = ids.cpu().numpy(), w.cpu().numpy()
            assert_layer(out[0], _oracle_layer(x[0:1].float().cpu().numpy(), list(idn[0]), list(wn[0]), dense))
        assert nat.device_error() == 0
    # the grouped-GEMM form (tsb_ep_moe_prefill), a prefill-sized batch
    T = 300
    nat = NativeEPDecode(mine_k, comm, T, prefill=True)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(9000 + rank)).to(torch.bfloat16).to(dev)
    ids, w = Router(router_w, k)(x)
    out = nat(x, ids, w, out_dtype=torch.float32)
    ref, _, _ = full.prefill(x, ids=ids, weights=w, out_dtype=torch.float32)
    torch.cuda.synchronize()
    err = rel_l2(out.cpu().numpy(), ref.cpu().numpy())
    worst = max(worst, err)
    assert err <= 1e-4, ("native prefill", rank, err)
    idn, wn = ids.cpu().numpy(), w.cpu().numpy()
    for t in (0, T - 1):
        assert_layer(out[t], _oracle_layer(x[t:t + 1].float().cpu().numpy(), list(idn[t]), list(wn[t]), dense))
    assert nat.device_error() == 0
    comm.close()
    dist.barrier()
    print(f"EP_OK rank={rank} world={world} worst_rel_l2={worst:.2e}", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
