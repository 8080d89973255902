"""Expert-parallel dispatch / combine (tinyserve_b200.ep) on CPU: two gloo
ranks, each with its own tokens and half of the experts; dense float64
experts stand in for the GPU kernels.  The sharded result must equal the
single-process grouped forward (tinyserve/expert_pipeline.py:166-239
semantics: out[t] = sum_j w[t,j] * expert_{ids[t,j]}(x[t]))."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H, E, K = 16, 8, 2


def _experts():
    g = torch.Generator().manual_seed(0)
    return [torch.randn(H, H, generator=g, dtype=torch.float64) * 0.3 for _ in range(E)]


def _tokens(rank, T, mode):
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(T, H, generator=g, dtype=torch.float64)
    if mode == "one_owner":
        ids = torch.stack([torch.zeros(T, dtype=torch.int64), torch.ones(T, dtype=torch.int64)], 1)
    else:
        ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]) if T else torch.zeros(0, K, dtype=torch.int64)
    w = torch.softmax(torch.randn(T, K, generator=g, dtype=torch.float64), 1)
    return x, ids.to(torch.int32), w


def _reference(x, ids, w, experts):
    out = torch.zeros_like(x)
    for t in range(x.shape[0]):
        for j in range(K):
            out[t] += w[t, j] * torch.tanh(x[t] @ experts[int(ids[t, j])].T)
    return out


def _worker(rank, world, port, sizes, mode, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from tinyserve_b200.ep import ExpertParallelMoE
    experts = _experts()
    el = E // world
    mine = experts[rank * el:(rank + 1) * el]
    calls = []

    def local_forward(rows, lid):
        calls.append(int(rows.shape[0]))
        assert int(lid.min()) >= 0 and int(lid.max()) < el
        return torch.stack([torch.tanh(rows[i] @ mine[int(lid[i])].T) for i in range(rows.shape[0])])

    ep = ExpertParallelMoE(E, K, H, local_forward)
    x, ids, w = _tokens(rank, sizes[rank], mode)
    out = ep(x, ids, w)
    ref = _reference(x, ids, w, experts)
    torch.save({"err": float((out - ref).abs().max()) if out.numel() else 0.0, "calls": calls,
                "shape": tuple(out.shape)}, os.path.join(outdir, f"r{rank}.pt"))
    dist.destroy_process_group()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("sizes,mode", [((5, 7), "random"), ((0, 6), "random"), ((4, 3), "one_owner")])
def test_ep_two_ranks_matches_single_process(tmp_path, sizes, mode):
    mp.spawn(_worker, args=(2, _port(), sizes, mode, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        res = torch.load(tmp_path / f"r{r}.pt")
        assert res["shape"] == (sizes[r], H)
        assert res["err"] < 1e-6  # combine accumulates in fp32
    if mode == "one_owner":  # experts 0 and 1 live on rank 0: rank 1 computes nothing
        assert torch.load(tmp_path / "r1.pt")["calls"] == []


def test_ep_rejects_uneven_split(tmp_path):
    mp.spawn(_bad_worker, args=(2, _port()), nprocs=2, join=True)


def _bad_worker(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from tinyserve_b200.ep import ExpertParallelMoE
    try:
        ExpertParallelMoE(5, 2, H, lambda r, l: r)
    except ValueError:
        pass
    else:
        raise AssertionError("5 experts over 2 ranks must be rejected")
    dist.destroy_process_group()


def _gather_worker(rank, world, port, T, mode, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from tinyserve_b200.ep import ExpertParallelMoE
    experts = _experts()
    el = E // world
    mine = experts[rank * el:(rank + 1) * el]
    seen = []

    def layer_forward(xa, lid, wa):
        # the weighted local layer: rows routed elsewhere carry -1 and add nothing
        seen.append((int(xa.shape[0]), int((lid >= 0).sum())))
        assert lid.dtype == torch.int32 and int(lid.max()) < el
        out = torch.zeros(xa.shape[0], H, dtype=torch.float64)
        for t in range(xa.shape[0]):
            for j in range(lid.shape[1]):
                if int(lid[t, j]) >= 0:
                    out[t] += float(wa[t, j]) * torch.tanh(xa[t] @ mine[int(lid[t, j])].T)
        return out

    ep = ExpertParallelMoE(E, K, H, layer_forward=layer_forward)
    x, ids, w = _tokens(rank, T, mode)
    out = ep.forward_gather(x, ids, w)
    ref = _reference(x, ids, w, experts)
    torch.save({"err": float((out - ref).abs().max()) if out.numel() else 0.0, "seen": seen,
                "shape": tuple(out.shape), "dtype": str(out.dtype)}, os.path.join(outdir, f"g{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("T,mode", [(1, "random"), (5, "random"), (3, "one_owner")])
def test_ep_gather_two_ranks_matches_single_process(tmp_path, T, mode):
    """The decode scheme: all-gathered tokens and routing, local layer with
    skipped rows, fp32 reduce-scatter back to each rank's own T rows."""
    mp.spawn(_gather_worker, args=(2, _port(), T, mode, str(tmp_path)), nprocs=2, join=True)
    total = 0
    for r in range(2):
        res = torch.load(tmp_path / f"g{r}.pt")
        assert res["shape"] == (T, H) and res["dtype"] == "torch.float64"
        assert res["err"] < 1e-5  # partial outputs travel in fp32
        rows, active = res["seen"][0]
        assert rows == 2 * T
        total += active
    assert total == 2 * T * K  # every (token, slot) pair computed exactly once
    if mode == "one_owner":
        assert torch.load(tmp_path / "g1.pt")["seen"][0][1] == 0
