"""Expert-parallel dispatch/combine host logic on CPU ranks (gloo, world size 2), and
failure detection without a GPU fault: a rank that leaves before a collective makes the
survivor's collective fail within a short process-group timeout instead of hanging."""
from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mrun_b200.expert_parallel import ExpertParallelMoE, ExpertShard, torch_combine

E, K, H, T = 8, 2, 16, 12


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _expert_fn(global_first: int):
    # a deterministic per-expert map standing in for the expert MLP
    def run(rows: torch.Tensor, local_expert: torch.Tensor) -> torch.Tensor:
        scale = (global_first + local_expert + 1).to(torch.float32)[:, None]
        return (rows.float() * scale - 0.5 * scale).to(rows.dtype)

    return run


def _inputs(rank: int):
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)])
    w = torch.rand(T, K, generator=g).to(torch.bfloat16)
    return x, idx, w


def _single_process_reference(x, idx, w):
    flat = idx.reshape(-1)
    rows = x.index_select(0, torch.arange(T).repeat_interleave(K))
    outs = _expert_fn(0)(rows, flat)
    inv = torch.arange(T * K)
    return torch_combine(outs, w.reshape(-1).float(), inv, T, K)


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    shard = ExpertShard(world, rank, E)
    moe = ExpertParallelMoE(shard, _expert_fn(shard.first))
    x, idx, w = _inputs(rank)
    out = moe.forward(x, idx, w)
    ref = _single_process_reference(x, idx, w)
    result_q.put((rank, bool(torch.equal(out, ref)), moe.last_stats))
    dist.barrier()
    dist.destroy_process_group()


def test_expert_parallel_matches_single_process_bitwise():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in results)
    assert sum(stats["received_rows"] for _, _, stats in results) == 2 * T * K


def _dropout_worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    dist.barrier()
    if rank == 1:
        os._exit(0)  # leaves between steps, with no collective in flight
    shard = ExpertShard(world, rank, E)
    moe = ExpertParallelMoE(shard, _expert_fn(shard.first))
    x, idx, w = _inputs(rank)
    try:
        moe.forward(x, idx, w)
        result_q.put("completed")
    except Exception as exc:  # the survivor's collective must fail, not hang
        result_q.put(type(exc).__name__)


def test_rank_leaving_is_detected_by_collective_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    outcome = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert outcome != "completed"


@pytest.mark.parametrize("world", [1, 2, 4])
def test_shard_ownership(world):
    owners = [e // ExpertShard(world, 0, 128).per_rank for e in range(128)]
    assert owners == sorted(owners) and len(set(owners)) == world


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_p2p_mailbox_layout(world):
    """The peer-memory mailbox (host-side layout, no GPU): every region 256-byte aligned and
    disjoint, sized for world x capacity rows each way, flags for up to 64 ranks."""
    import ctypes

    from mrun_b200 import _lib

    cap, hidden = 256, 2048
    lib = _lib.load()
    total = int(lib.mrb_ep_mailbox_bytes(world, cap, hidden))
    offsets = (ctypes.c_int64 * 6)()
    _lib.call("mrb_ep_mailbox_offsets", world, cap, hidden, offsets)
    flags_d, flags_r, counts, ids, rows, back = list(offsets)
    assert all(v % 256 == 0 for v in offsets)
    assert flags_d == 0 and flags_r >= 64 * 4 and counts >= flags_r + 64 * 4 and ids >= counts + world * 4
    assert rows >= ids + world * cap * 4
    assert back >= rows + world * cap * hidden * 2
    assert total >= back + world * cap * hidden * 2 and total % 256 == 0
    assert int(lib.mrb_ep_mailbox_bytes(65, cap, hidden)) == 0  # above the 64-rank flag area
    with pytest.raises(ValueError, match="bad shape"):
        _lib.call("mrb_ep_mailbox_offsets", 0, cap, hidden, offsets)
