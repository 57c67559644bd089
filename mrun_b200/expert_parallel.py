"""Expert parallelism for the routed-MoE layer: experts sharded over the GPUs of one box,
tokens exchanged with NCCL all-to-all over NVLink.

The reference runs every expert on one device (engine/qwen3_moe_cuda.py:2698-2788); this
module spreads the same computation. Expert ``e`` lives on rank ``e // (E / world)``; each
rank routes its own tokens (data-parallel attention), then per layer:

1. assignments are ordered by destination rank (stable, so the order is the same on every
   run) and the per-destination counts are exchanged (``all_to_all_single`` of counts);
2. each assignment's activation row and its destination-local expert id are sent
   (``all_to_all_single`` with split sizes);
3. the owner runs the grouped int8 expert MLP on what it received;
4. the outputs travel back by the reverse all-to-all;
5. the source combines every token's k outputs in route-rank order.

Each expert output row depends only on its own activation row and the combine order is
fixed, so the layer's result is bit-identical for every world size. The collectives and
the planners are injected, so the host-side logic is testable on CPU with the gloo
backend; on GPUs the planner is the native route compiler and compute is the grouped
int8 MLP.
"""
from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass

import torch
import torch.distributed as dist

# planner(keys int64 [n], num_groups) -> (order int64 [n], counts int64 [num_groups], inverse int64 [n])
# with order = stable argsort of keys and inverse[order] = arange(n).
Planner = Callable[[torch.Tensor, int], tuple[torch.Tensor, torch.Tensor, torch.Tensor]]


def torch_stable_planner(keys: torch.Tensor, groups: int):
    """Reference planner (any device): stable argsort, bincount, inverse bijection."""
    order = torch.argsort(keys, stable=True)
    counts = torch.bincount(keys, minlength=groups).to(torch.int64)
    inverse = torch.empty_like(order)
    inverse[order] = torch.arange(order.numel(), device=order.device)
    return order, counts, inverse


def native_planner(keys: torch.Tensor, groups: int):
    """The native deterministic route compiler with k = 1 (same order as the reference)."""
    from .moe import grouped_route_tensors_with_inverse

    token_ids, _, _, counts, inverse, _ = grouped_route_tensors_with_inverse(
        keys.reshape(-1, 1), torch.zeros((keys.numel(), 1), device=keys.device), num_experts=groups)
    return token_ids, counts.to(torch.int64), inverse


@dataclass
class ExpertShard:
    """Rank ``rank`` of ``world`` owns experts [first, first + count)."""

    world: int
    rank: int
    num_experts: int

    @property
    def per_rank(self) -> int:
        if self.num_experts % self.world:
            raise ValueError("expert count must divide evenly over the ranks")
        return self.num_experts // self.world

    @property
    def first(self) -> int:
        return self.rank * self.per_rank


class ExpertParallelMoE:
    """Dispatch / local compute / return / combine for one MoE layer on one rank.

    ``local_mlp(rows bf16 [n, H], local_expert int64 [n]) -> bf16 [n, H]`` computes the
    owned experts' outputs for received rows (any row order)."""

    def __init__(self, shard: ExpertShard, local_mlp, *, group=None, planner: Planner = torch_stable_planner,
                 combine=None) -> None:
        self.shard = shard
        self.local_mlp = local_mlp
        self.group = group
        self.planner = planner
        self.combine = combine or torch_combine
        self.last_stats: dict[str, int] = {}

    def _all_to_all(self, out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits) -> None:
        dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits, group=self.group)

    def forward(self, source: torch.Tensor, top_indices: torch.Tensor, top_weights: torch.Tensor) -> torch.Tensor:
        """source [T, H] bf16, top_indices [T, k], top_weights [T, k] -> bf16 [T, H]."""
        sh = self.shard
        t, k = (int(v) for v in top_indices.shape)
        hidden = int(source.shape[1])
        device = source.device
        flat_e = top_indices.reshape(-1).to(torch.int64)
        dest = torch.div(flat_e, sh.per_rank, rounding_mode="floor")
        order, send_counts, inverse = self.planner(dest, sh.world)
        # 1. counts
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        send_split = [int(v) for v in send_counts.tolist()]
        recv_split = [int(v) for v in recv_counts.tolist()]
        n_recv = sum(recv_split)
        # 2. rows and destination-local expert ids, in destination order
        token_of = torch.div(order, k, rounding_mode="floor")
        send_rows = source.index_select(0, token_of)
        send_expert = (flat_e.index_select(0, order) - dest.index_select(0, order) * sh.per_rank).contiguous()
        recv_rows = torch.empty((n_recv, hidden), dtype=source.dtype, device=device)
        recv_expert = torch.empty((n_recv,), dtype=torch.int64, device=device)
        self._all_to_all(recv_rows, send_rows.contiguous(), recv_split, send_split)
        self._all_to_all(recv_expert, send_expert, recv_split, send_split)
        # 3. owned experts
        recv_out = self.local_mlp(recv_rows, recv_expert) if n_recv else recv_rows
        # 4. return
        back = torch.empty((t * k, hidden), dtype=source.dtype, device=device)
        self._all_to_all(back, recv_out.contiguous(), send_split, recv_split)
        # 5. combine in route-rank order: assignment a's output sits at back[inverse[a]]
        coef = top_weights.reshape(-1).float().index_select(0, order).contiguous()
        self.last_stats = {"sent_rows": t * k, "received_rows": n_recv}
        return self.combine(back, coef, inverse, t, k)


class FixedCapacityExpertParallelMoE:
    """The same exchange with sizes fixed on the host, so a decode step can be captured in a
    CUDA graph (no device-to-host synchronisation): every (source, destination) block holds
    T*k rows (the worst case, so nothing overflows). ``mrb_ep_pack`` plans the slots on the
    device (padding slots carry a dummy local expert), rows and destination-local expert ids
    travel by equal-split ``all_to_all_single``, the owner runs the grouped int8 MLP over the
    real experts only, outputs come back the same way, and the fixed-rank combine reads each
    assignment's slot. Results are bit-identical to one GPU (row-independent experts, combine
    in route-rank order). Exchange cost: world * T*k rows each way per layer."""

    def __init__(self, shard: ExpertShard, pages: torch.Tensor, layout, *, group=None) -> None:
        self.shard = shard
        self.pages = pages
        self.layout = layout
        self.group = group

    def forward(self, source: torch.Tensor, top_indices: torch.Tensor, top_weights: torch.Tensor) -> torch.Tensor:
        from . import _lib
        from .moe import grouped_expert_mlp, grouped_route_tensors_with_inverse

        sh = self.shard
        t, k = (int(v) for v in top_indices.shape)
        hidden = int(source.shape[1])
        device = source.device
        world, per = sh.world, sh.per_rank
        cap = t * k
        slots = world * cap
        stream = _lib.stream_handle(device)
        idx = top_indices.to(torch.int64).contiguous()
        w32 = top_weights.float().contiguous()
        send_expert = torch.empty(slots, dtype=torch.int32, device=device)
        coef_slot = torch.empty(slots, dtype=torch.float32, device=device)
        slot_of_assign = torch.empty(cap, dtype=torch.int64, device=device)
        slot_src = torch.empty(slots, dtype=torch.int32, device=device)
        _lib.call("mrb_ep_pack", idx.data_ptr(), w32.data_ptr(), t, k, per, world, cap, send_expert.data_ptr(),
                  coef_slot.data_ptr(), slot_of_assign.data_ptr(), slot_src.data_ptr(), None, stream)
        send_rows = torch.empty((slots, hidden), dtype=torch.bfloat16, device=device)
        src = source.contiguous()
        _lib.call("mrb_ep_gather_rows", src.data_ptr(), hidden, slot_src.data_ptr(), slots, send_rows.data_ptr(),
                  stream)
        recv_rows = torch.empty_like(send_rows)
        recv_expert = torch.empty_like(send_expert)
        dist.all_to_all_single(recv_rows, send_rows, group=self.group)
        dist.all_to_all_single(recv_expert, send_expert, group=self.group)
        # padding slots route to the dummy expert `per`, which the grouped MLP never runs
        token_ids, _, starts, counts, inverse, _ = grouped_route_tensors_with_inverse(
            recv_expert.view(-1, 1).to(torch.int64), torch.zeros((slots, 1), device=device), num_experts=per + 1)
        eo = grouped_expert_mlp(recv_rows, token_ids, starts[:per], counts[:per], self.pages, self.layout)
        back_local = eo.index_select(0, inverse)  # received-slot order
        back = torch.empty_like(back_local)
        dist.all_to_all_single(back, back_local, group=self.group)
        out = torch.empty((t, hidden), dtype=torch.bfloat16, device=device)
        _lib.call("mrb_stable_route_reduce", back.data_ptr(), coef_slot.data_ptr(), slot_of_assign.data_ptr(), t, k,
                  hidden, None, out.data_ptr(), stream)
        return out


class P2PExpertParallelMoE:
    """The fixed-capacity plan exchanged over NVLink peer memory instead of NCCL: each rank owns
    a mailbox (CUDA IPC-mapped into every peer); the dispatch kernel stores only the real rows
    straight into their owners' mailboxes and release-publishes a per-exchange epoch flag, the
    owner acquires every source's flag (bounded wait), runs the grouped int8 MLP on the rows
    in place and stores the outputs straight back into the sources' mailboxes, and the source
    combines in route-rank order once every owner's flag has arrived. Results are
    bit-identical to one GPU and to the NCCL exchange. One instance per call site (each MoE
    layer) and per process group; every rank must call forward in the same order. ``close()``
    unmaps the peers' mailboxes and frees this rank's (after the last use, before the process
    group goes away).

    Without resident ``pages`` (None, with ``device`` given) the pages come from
    ``page_cache``, a ``streaming.ExpertPageCache`` over a host tier holding this rank's
    experts only: each call acquires every local expert page of ``layer`` before the expert
    MLP -- a static plan, so no routes are read on the host (at large batch every local expert
    receives rows) -- and releases the slots after it; such calls run eagerly, not in a CUDA
    graph. The owner sets ``page_cache`` (it may swap the cache between calls)."""

    def __init__(self, shard: ExpertShard, pages: torch.Tensor | None, layout, *, tokens: int, k: int, hidden: int,
                 group=None, page_cache=None, layer: int = 0, device: torch.device | None = None) -> None:
        import ctypes

        from . import _lib

        if pages is None and device is None:
            raise ValueError("give the resident expert pages, or the device of a streamed layer")
        self.shard = shard
        self.pages = pages
        self.page_cache = page_cache
        self.layer = int(layer)
        self._local_ids = torch.arange(shard.per_rank, dtype=torch.int64)  # on the host: no sync to plan
        self.layout = layout
        self.group = group
        self.tokens, self.k, self.hidden = int(tokens), int(k), int(hidden)
        device = pages.device if pages is not None else torch.device(device)
        self.device = device
        world, rank = shard.world, shard.rank
        self.cap = self.tokens * self.k
        slots = world * self.cap
        lib = _lib.load()
        nbytes = int(lib.mrb_ep_mailbox_bytes(world, self.cap, self.hidden))
        offsets = (ctypes.c_int64 * 6)()
        _lib.call("mrb_ep_mailbox_offsets", world, self.cap, self.hidden, offsets)
        self.offsets = list(offsets)
        own = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        _lib.call("mrb_ep_mailbox_create", nbytes, ctypes.byref(own), handle)
        self._own = own.value
        self._peers: list[int] = []
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
        everyone = torch.empty(world * 64, dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(everyone, mine, group=group)
        handles = everyone.cpu().numpy().reshape(world, 64)
        ptrs = []
        for r in range(world):
            if r == rank:
                ptrs.append(self._own)
                continue
            peer = ctypes.c_void_p()
            h = (ctypes.c_ubyte * 64).from_buffer_copy(handles[r].tobytes())
            _lib.call("mrb_ep_mailbox_open", h, ctypes.byref(peer))
            self._peers.append(peer.value)
            ptrs.append(peer.value)
        self.mailboxes = torch.tensor(ptrs, dtype=torch.int64, device=device)
        self.state = torch.zeros(4, dtype=torch.int32, device=device)
        # the plan and receive-side buffers live as long as the instance (graph friendly)
        self.send_expert = torch.empty(slots, dtype=torch.int32, device=device)
        self.coef_slot = torch.empty(slots, dtype=torch.float32, device=device)
        self.slot_of_assign = torch.empty(self.cap, dtype=torch.int64, device=device)
        self.slot_src = torch.empty(slots, dtype=torch.int32, device=device)
        self.ids64 = torch.empty((slots, 1), dtype=torch.int64, device=device)
        self.zeros = torch.zeros((slots, 1), dtype=torch.float32, device=device)
        self.mlp_sync = torch.zeros(2 * shard.per_rank + 1, dtype=torch.int32, device=device)
        # routes of the received rows, compiled by the receive kernel (real rows only)
        per = shard.per_rank
        self.rt_counts = torch.empty(per, dtype=torch.int32, device=device)
        self.rt_starts = torch.empty(per, dtype=torch.int32, device=device)
        self.rt_token_ids = torch.empty(slots, dtype=torch.int64, device=device)
        self.rt_coef = torch.empty(slots, dtype=torch.float32, device=device)
        self.rt_inverse = torch.empty(slots, dtype=torch.int64, device=device)
        dist.barrier(group=group)  # every mailbox exists and is zeroed before any dispatch

    def forward(self, source: torch.Tensor, top_indices: torch.Tensor, top_weights: torch.Tensor) -> torch.Tensor:
        from . import _lib
        from .moe import grouped_route_tensors_with_inverse

        sh = self.shard
        t, k = (int(v) for v in top_indices.shape)
        if t > self.tokens or k != self.k or int(source.shape[1]) != self.hidden:
            raise ValueError("P2P expert exchange was sized for a smaller batch")
        device = source.device
        world, per, cap, hidden = sh.world, sh.per_rank, self.cap, self.hidden
        slots = world * cap
        stream = _lib.stream_handle(device)
        idx = top_indices.to(torch.int64).contiguous()
        w32 = top_weights.float().contiguous()
        _lib.call("mrb_ep_pack", idx.data_ptr(), w32.data_ptr(), t, k, per, world, cap, self.send_expert.data_ptr(),
                  self.coef_slot.data_ptr(), self.slot_of_assign.data_ptr(), self.slot_src.data_ptr(), None, stream)
        src = source.contiguous()
        _lib.call("mrb_ep_p2p_dispatch", src.data_ptr(), hidden, self.slot_src.data_ptr(), self.send_expert.data_ptr(),
                  world, sh.rank, cap, self.mailboxes.data_ptr(), self.state.data_ptr(), stream)
        # receive + route compile of the rows that arrived, in one launch
        _lib.call("mrb_ep_p2p_wait_route", self._own, world, cap, hidden, per, self.ids64.data_ptr(),
                  self.zeros.data_ptr(), self.rt_counts.data_ptr(), self.rt_starts.data_ptr(),
                  self.rt_token_ids.data_ptr(), self.rt_coef.data_ptr(), self.rt_inverse.data_ptr(),
                  self.state.data_ptr(), stream)
        if self.pages is None:
            if self.page_cache is None or self.page_cache.host.experts != per:
                raise ValueError("a streamed layer needs a page cache over this rank's experts")
            pages, slot_of = self.page_cache.layer_pages(self.layer, self._local_ids)
        else:
            pages, slot_of = self.pages, None
        if self.pages is None:
            # a streamed layer runs eagerly: experts that received many rows (a large batch
            # over few experts per rank) go to the tensor-core GEMMs
            from .moe import expert_mlp_large_counts

            received = _device_rows(self._own + self.offsets[4], slots, hidden, device)
            eo = expert_mlp_large_counts(received, self.rt_token_ids, self.rt_starts, self.rt_counts, pages,
                                         self.layout, slot_of=slot_of, sync=self.mlp_sync)
        else:
            eo = _grouped_mlp_from_pointer(self._own + self.offsets[4], self.rt_token_ids, self.rt_starts,
                                           self.rt_counts, pages, self.layout, hidden, device, self.mlp_sync,
                                           rows=slots, slot_of=slot_of)
        if self.pages is None:
            self.page_cache.release_layer()  # its slots may be refilled once these kernels are done
        _lib.call("mrb_ep_p2p_return", eo.data_ptr(), self.rt_inverse.data_ptr(), hidden, world, sh.rank, cap,
                  self.mailboxes.data_ptr(), self.state.data_ptr(), stream)
        # wait for every owner's return + the fixed-rank combine, in one launch
        out = torch.empty((t, hidden), dtype=torch.bfloat16, device=device)
        _lib.call("mrb_ep_p2p_combine", self._own, world, cap, hidden, self.coef_slot.data_ptr(),
                  self.slot_of_assign.data_ptr(), t, k, out.data_ptr(), self.state.data_ptr(), stream)
        return out

    def check(self) -> None:
        """Raise if a bounded wait of the exchange or of the expert MLP timed out (synchronises)."""
        if int(self.state[3].item()):
            raise RuntimeError("expert-parallel peer exchange timed out waiting for a rank")
        if int(self.mlp_sync[-1].item()):
            raise RuntimeError("expert MLP: the down projection timed out waiting for the gate/up projection")

    def close(self) -> None:
        from . import _lib

        for p in self._peers:
            _lib.call("mrb_ep_mailbox_close", p, 0)
        self._peers = []
        if self._own:
            _lib.call("mrb_ep_mailbox_close", self._own, 1)
            self._own = 0


class _RowsInterface:
    """``__cuda_array_interface__`` of bf16 rows at a raw device address (read as int16)."""

    def __init__(self, ptr: int, rows: int, hidden: int) -> None:
        self.__cuda_array_interface__ = {"shape": (int(rows), int(hidden)), "typestr": "<i2",
                                         "data": (int(ptr), False), "version": 3, "strides": None}


def _device_rows(ptr: int, rows: int, hidden: int, device) -> torch.Tensor:
    """A bf16 [rows, hidden] tensor viewing this rank's memory at ``ptr`` (no copy)."""
    return torch.as_tensor(_RowsInterface(ptr, rows, hidden), device=device).view(torch.bfloat16)


def _grouped_mlp_from_pointer(rows_ptr: int, token_ids, starts, counts, pages, layout, hidden: int, device,
                              sync: torch.Tensor | None = None, rows: int | None = None,
                              slot_of: torch.Tensor | None = None):
    """grouped_expert_mlp over activation rows given by a raw device pointer (a mailbox).
    ``rows``: the assignment slots the outputs are indexed by (default token_ids' length);
    ``slot_of``: int32 [experts] page slot of each expert in ``pages`` (None: identity)."""
    from . import _lib
    from .moe import expert_mlp_sync

    ly = layout
    f = ly.intermediate_size
    a = int(token_ids.numel()) if rows is None else int(rows)
    e = int(counts.numel())
    act = torch.empty((a, f), dtype=torch.bfloat16, device=device)
    y = torch.empty((a, hidden), dtype=torch.bfloat16, device=device)
    if sync is None:
        sync = expert_mlp_sync(e, device)
    _lib.call("mrb_grouped_expert_mlp", rows_ptr, token_ids.data_ptr(), starts.data_ptr(), counts.data_ptr(), e,
              pages.data_ptr(), ly.page_stride, ly.gate_up_codes_offset, ly.gate_up_scales_offset,
              ly.down_codes_offset, ly.down_scales_offset, _lib.ptr(slot_of), hidden, f, a, act.data_ptr(),
              y.data_ptr(), sync.data_ptr(), _lib.stream_handle(device))
    return y


def torch_combine(rows: torch.Tensor, coef: torch.Tensor, inverse: torch.Tensor, t: int, k: int) -> torch.Tensor:
    """out[t] = sum_r coef[p] * rows[p], p = inverse[t*k + r]: fp32 products added in rank order."""
    per = rows.index_select(0, inverse).reshape(t, k, -1).float()
    c = coef.index_select(0, inverse).reshape(t, k, 1)
    out = per[:, 0] * c[:, 0]
    for r in range(1, k):
        out = out + per[:, r] * c[:, r]
    return out.to(rows.dtype)


def native_combine(rows: torch.Tensor, coef: torch.Tensor, inverse: torch.Tensor, t: int, k: int) -> torch.Tensor:
    """The same combine on the native fixed-rank kernel (bf16 output)."""
    from . import _lib

    out = torch.empty((t, rows.shape[1]), dtype=torch.bfloat16, device=rows.device)
    _lib.call("mrb_stable_route_reduce", rows.contiguous().data_ptr(), coef.data_ptr(), inverse.contiguous().data_ptr(),
              t, k, int(rows.shape[1]), None, out.data_ptr(), _lib.stream_handle(rows.device))
    return out


def local_expert_mlp_fn(pages: torch.Tensor, layout, experts_per_rank: int):
    """local_mlp for ExpertParallelMoE over this rank's resident expert pages."""
    from .moe import grouped_expert_mlp, grouped_route_tensors_with_inverse

    def run(rows: torch.Tensor, local_expert: torch.Tensor) -> torch.Tensor:
        token_ids, _, starts, counts, inverse, _ = grouped_route_tensors_with_inverse(
            local_expert.reshape(-1, 1), torch.zeros((local_expert.numel(), 1), device=rows.device),
            num_experts=experts_per_rank)
        eo = grouped_expert_mlp(rows, token_ids, starts, counts, pages, layout)
        return eo.index_select(0, inverse)  # back to received-row order

    return run


__all__ = [
    "ExpertParallelMoE",
    "FixedCapacityExpertParallelMoE",
    "P2PExpertParallelMoE",
    "ExpertShard",
    "local_expert_mlp_fn",
    "native_combine",
    "native_planner",
    "torch_combine",
    "torch_stable_planner",
]
