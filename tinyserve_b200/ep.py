"""Expert parallelism: the experts of a layer sharded over the ranks of a
process group (one process per GPU), token dispatch and combine over NCCL.

Rank r owns experts [r*E/G, (r+1)*E/G) (contiguous ranges) and brings its own
tokens.  Two exchange schemes:

* ``forward_gather`` (decode-sized batches, the same T on every rank): the
  tokens and their routing are all-gathered (G*T rows), every rank runs its
  local experts on the (token, slot) pairs routed to them (the other ranks'
  pairs carry a negative id, which the kernels skip), and the fp32 partial
  outputs are summed across ranks by one reduce-scatter that hands each rank
  its own T rows.  Shapes are static and no count ever goes to the host, so a
  step can be captured in a CUDA graph; the combine is the reduce-scatter.
* ``forward`` (prefill-sized batches, any T per rank): all-to-all dispatch of
  only the routed rows, as below.  The row counts per rank pair are exchanged
  first and read on the host to size the uneven splits (one synchronisation
  per layer call, small next to a prefill layer).

``forward`` on every rank:

1. route its tokens (router weights are replicated; ``Router``);
2. order its (token, slot) rows by owning rank (stable, so the order is
   deterministic) and exchange the per-rank row counts (all_to_all);
3. send the rows and their local expert ids to their owners
   (all_to_all_single with uneven splits: NCCL send/recv over NVLink);
4. run the received rows through the local experts as one grouped call, one
   expert per row (``local_forward``);
5. send the expert outputs back along the reverse splits;
6. combine on the source rank: out[t] = sum_j w[t,j] * y[t,j] in slot order,
   accumulated in fp32.

The reference runs every expert of a layer on one device
(tinyserve/expert_pipeline.py:166-239); sharding is what lets the 120B-shaped
layer (128 experts) spread over 1/2/4/8 GPUs.  Remote rows land in local
memory through NCCL before any kernel reads them.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

LocalForward = Callable[[torch.Tensor, torch.Tensor], torch.Tensor]
LayerForward = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


class ExpertParallelMoE:
    """One MoE layer sharded expert-parallel over ``group``.

    ``local_forward(x_rows [R, H], local_ids [R] int32) -> [R, H]`` runs each
    row through local expert ``local_ids[i]`` (unweighted; the ``forward``
    scheme); ``layer_forward`` is the weighted local layer of the
    ``forward_gather`` scheme.  ``router(x) -> (ids [T,k] int32 global,
    weights [T,k] fp32)`` is used when the caller does not pass routing."""

    def __init__(self, n_experts: int, top_k: int, hidden: int, local_forward: LocalForward | None = None, *,
                 router: Callable | None = None, group=None, layer_forward: LayerForward | None = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_experts % self.world:
            raise ValueError(f"{n_experts} experts do not split evenly over {self.world} ranks")
        self.n_experts, self.top_k, self.hidden = n_experts, top_k, hidden
        self.e_local = n_experts // self.world
        self.base = self.rank * self.e_local
        self.local_forward = local_forward
        self.layer_forward = layer_forward
        self.router = router

    def owner(self, ids: torch.Tensor) -> torch.Tensor:
        return torch.div(ids, self.e_local, rounding_mode="floor")

    def forward(self, x: torch.Tensor, ids: torch.Tensor | None = None,
                weights: torch.Tensor | None = None) -> torch.Tensor:
        if ids is None:
            if self.router is None:
                raise ValueError("no router: pass ids and weights")
            ids, weights = self.router(x)
        T, H = x.shape
        k = ids.shape[1]
        dev = x.device
        flat = ids.reshape(-1).to(torch.int64)
        if flat.numel() and (int(flat.min()) < 0 or int(flat.max()) >= self.n_experts):
            raise ValueError("expert id out of range")
        dest = self.owner(flat)
        order = torch.argsort(dest, stable=True)
        send_counts = torch.bincount(dest, minlength=self.world).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        n_send, n_recv = sum(sc), sum(rc)

        send_rows = x.index_select(0, torch.div(order, k, rounding_mode="floor")).contiguous()
        send_lid = (flat.index_select(0, order) - dest.index_select(0, order) * self.e_local).to(torch.int32)
        recv_rows = torch.empty(n_recv, H, dtype=x.dtype, device=dev)
        recv_lid = torch.empty(n_recv, dtype=torch.int32, device=dev)
        dist.all_to_all_single(recv_rows, send_rows, rc, sc, group=self.group)
        dist.all_to_all_single(recv_lid, send_lid, rc, sc, group=self.group)

        y_recv = self.local_forward(recv_rows, recv_lid) if n_recv else torch.empty(0, H, dtype=x.dtype, device=dev)
        y_recv = y_recv.to(x.dtype).contiguous()
        y_send = torch.empty(n_send, H, dtype=x.dtype, device=dev)
        dist.all_to_all_single(y_send, y_recv, sc, rc, group=self.group)

        y = torch.empty(T * k, H, dtype=torch.float32, device=dev)
        y[order] = y_send.float()
        # weighted combine in one batched product: out[t] = sum_j w[t,j] y[t,j]
        w = weights.to(torch.float32).reshape(T, 1, k)
        out = torch.bmm(w, y.view(T, k, H)).view(T, H)
        return out.to(x.dtype)

    __call__ = forward

    def forward_gather(self, x: torch.Tensor, ids: torch.Tensor | None = None,
                       weights: torch.Tensor | None = None, layer_forward: LayerForward | None = None,
                       out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """Decode step of T tokens per rank (T equal on every rank): all-gather
        tokens and routing, local experts on the rows routed here (other
        ranks' rows skipped), reduce-scatter of the fp32 partial outputs.
        ``layer_forward(x_all [G*T, H], local_ids [G*T, k] int32 (negative =
        skip), weights [G*T, k] fp32) -> fp32 [G*T, H]`` runs this rank's
        experts (default: the one given at construction as ``layer_forward``)."""
        fwd = layer_forward or self.layer_forward
        if fwd is None:
            raise ValueError("no layer_forward for the gather scheme")
        if ids is None:
            if self.router is None:
                raise ValueError("no router: pass ids and weights")
            ids, weights = self.router(x)
        T, H = x.shape
        k = ids.shape[1]
        G = self.world
        x_all = torch.empty(G * T, H, dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(x_all, x.contiguous(), group=self.group)
        meta = torch.cat([ids.to(torch.int32).view(torch.float32).reshape(T, k),
                          weights.to(torch.float32).reshape(T, k)], dim=1).contiguous()
        meta_all = torch.empty(G * T, 2 * k, dtype=torch.float32, device=x.device)
        dist.all_gather_into_tensor(meta_all, meta, group=self.group)
        ids_all = meta_all[:, :k].contiguous().view(torch.int32)
        w_all = meta_all[:, k:].contiguous()
        lid = ids_all - self.base
        lid = torch.where((lid >= 0) & (lid < self.e_local), lid, torch.full_like(lid, -1))
        part = fwd(x_all, lid, w_all).to(torch.float32).contiguous()
        out = torch.empty(T, H, dtype=torch.float32, device=x.device)
        dist.reduce_scatter_tensor(out, part, group=self.group)
        return out.to(out_dtype or x.dtype)


def quant_local_forward(layer) -> LocalForward:
    """``local_forward`` backed by a :class:`tinyserve_b200.moe.QuantMoE` that
    holds this rank's experts with top_k = 1: each received row is one
    (token, expert) pair with weight 1."""
    if layer.top_k != 1:
        raise ValueError("the local layer must be built with top_k=1")

    def f(rows: torch.Tensor, lid: torch.Tensor) -> torch.Tensor:
        ones = torch.ones(rows.shape[0], 1, dtype=torch.float32, device=rows.device)
        out, _, _ = layer.decode(rows.contiguous(), ids=lid.reshape(-1, 1), weights=ones)
        return out

    return f


def quant_layer_forward(layer) -> LayerForward:
    """``layer_forward`` backed by a :class:`tinyserve_b200.moe.QuantMoE`
    holding this rank's experts with the model's top_k: one decode call over
    the gathered tokens (per-token packed path up to 16 tokens, grouped path
    above), the (token, slot) pairs of other ranks' experts skipped through
    their negative ids, fp32 output."""
    def f(x: torch.Tensor, lid: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        out, _, _ = layer.decode(x.contiguous(), ids=lid, weights=w, out_dtype=torch.float32)
        return out

    return f


class NcclComm:
    """An NCCL communicator for the C-ABI's expert-parallel entry point
    (tsb_ep_moe_decode takes a raw ``ncclComm_t``).  Built with NCCL's public
    API through the process's libnccl.so.2 (the one PyTorch loaded): rank 0
    makes the unique id and the ranks of ``group`` (a torch.distributed
    process group, any backend) share it; this GPU must be current."""

    def __init__(self, group=None):
        import ctypes
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self._nccl = ctypes.CDLL("libnccl.so.2", mode=ctypes.RTLD_GLOBAL)
        uid = ctypes.create_string_buffer(128)  # ncclUniqueId: 128 opaque bytes
        if self.rank == 0:
            rc = self._nccl.ncclGetUniqueId(uid)
            if rc:
                raise RuntimeError(f"ncclGetUniqueId failed ({rc})")
        box = [bytes(uid.raw)]
        dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        uid = ctypes.create_string_buffer(box[0], 128)

        class _Uid(ctypes.Structure):
            _fields_ = [("internal", ctypes.c_char * 128)]

        u = _Uid()
        ctypes.memmove(ctypes.addressof(u), uid, 128)
        self.comm = ctypes.c_void_p()
        self._nccl.ncclCommInitRank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, _Uid, ctypes.c_int]
        rc = self._nccl.ncclCommInitRank(ctypes.byref(self.comm), self.world, u, self.rank)
        if rc:
            raise RuntimeError(f"ncclCommInitRank failed ({rc})")

    def close(self) -> None:
        import ctypes
        if self.comm:
            self._nccl.ncclCommDestroy.argtypes = [ctypes.c_void_p]
            self._nccl.ncclCommDestroy(self.comm)
            self.comm = ctypes.c_void_p()


class NativeEPDecode:
    """The gather scheme of :meth:`ExpertParallelMoE.forward_gather` as one
    C-ABI call: all-gather, local experts, reduce-scatter, all on the current
    stream inside the library (tsb_ep_moe_decode; with ``prefill`` the local
    experts run as grouped tensor-core GEMMs, tsb_ep_moe_prefill).  ``local``
    is a :class:`tinyserve_b200.moe.QuantMoE` holding this rank's experts
    (top_k = the model's); T is fixed per instance (the workspace is sized
    for it)."""

    def __init__(self, local, comm: NcclComm, T: int, prefill: bool = False):
        import ctypes
        from . import _lib
        self.local, self.comm, self.T, self.prefill = local, comm, T, prefill
        self._spec = {False: local.spec, True: local.spec_f32}
        L = _lib.lib()
        n = (L.tsb_ep_prefill_workspace(ctypes.byref(local.spec), T, comm.world) if prefill else
             L.tsb_ep_decode_workspace(ctypes.byref(local.spec), T, comm.world, int(local.packed)))
        self.ws = torch.zeros(n, dtype=torch.uint8, device=local.device)

    def __call__(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                 out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        import ctypes
        from . import _lib
        if x.shape != (self.T, self.local.hidden) or x.dtype != torch.bfloat16:
            raise ValueError(f"x must be bf16 [{self.T}, {self.local.hidden}]")
        ids = ids.to(torch.int32).contiguous()
        weights = weights.to(torch.float32).contiguous()
        out = torch.empty(self.T, self.local.hidden, dtype=out_dtype, device=x.device)
        L = self.local
        spec = ctypes.byref(self._spec[out_dtype == torch.float32])
        stream = torch.cuda.current_stream(x.device).cuda_stream
        if self.prefill:
            rc = _lib.lib().tsb_ep_moe_prefill(
                spec, L._table.data_ptr(), x.contiguous().data_ptr(), self.T, ids.data_ptr(), weights.data_ptr(),
                out.data_ptr(), self.comm.comm, self.comm.rank, self.comm.world, self.ws.data_ptr(), self.ws.numel(),
                stream)
        else:
            rc = _lib.lib().tsb_ep_moe_decode(
                spec, L._table.data_ptr(), L._packed.data_ptr() if L.packed else None, x.contiguous().data_ptr(),
                self.T, ids.data_ptr(), weights.data_ptr(), out.data_ptr(), self.comm.comm, self.comm.rank,
                self.comm.world, self.ws.data_ptr(), self.ws.numel(), stream)
        _lib.check(rc)
        return out

    def device_error(self) -> int:
        import ctypes
        from . import _lib
        code = ctypes.c_int32()
        _lib.check(_lib.lib().tsb_read_device_error(self.ws.data_ptr(), ctypes.byref(code),
                                                    torch.cuda.current_stream(self.local.device).cuda_stream))
        return code.value
