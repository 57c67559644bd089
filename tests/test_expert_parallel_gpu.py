"""Expert parallelism on 2+ GPUs: each rank's MoE output must be bit-identical to the
single-GPU backend over all experts, for the host-sized NCCL exchange, the fixed-capacity NCCL
exchange (eager and replayed from a CUDA graph) and the fixed-capacity exchange over NVLink
peer memory (eager and graph-replayed, no wait timed out), also with each rank's expert pages
streamed from a pinned host tier through a slot cache. Skipped with fewer than 2 GPUs."""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

E, K, H, F, T = 16, 4, 512, 256, 24


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from mrun_b200.expert_parallel import (
        ExpertParallelMoE, ExpertShard, FixedCapacityExpertParallelMoE, P2PExpertParallelMoE, local_expert_mlp_fn,
        native_combine, native_planner,
    )
    from mrun_b200.moe import ExpertPageLayout, PagedInt8ExpertBackend, ResidentInt8ExpertPages, pack_expert_page, router_topk
    from oracle import qrow as oq

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        rng = np.random.default_rng(7)  # same experts on every rank
        ly = ExpertPageLayout.create(H, F)
        pages = torch.zeros((E, ly.page_stride), dtype=torch.uint8, device=dev)
        for e in range(E):
            gu = oq.quant_row_int8((rng.standard_normal((2 * F, H)) * 0.02).astype(np.float32))
            dn = oq.quant_row_int8((rng.standard_normal((H, F)) * 0.02).astype(np.float32))
            pack_expert_page(ly, torch.from_numpy(gu[0]), torch.from_numpy(gu[1]), torch.from_numpy(dn[0]),
                             torch.from_numpy(dn[1]), pages[e])
        trng = np.random.default_rng(100 + rank)  # this rank's own tokens
        x = torch.from_numpy(trng.standard_normal((T, H)).astype(np.float32)).to(dev).to(torch.bfloat16)
        idx, w, _ = router_topk(torch.from_numpy(trng.standard_normal((T, E)).astype(np.float32)).to(dev), K)
        single = PagedInt8ExpertBackend(ResidentInt8ExpertPages(ly, [pages]), num_experts=E).moe(0, x, idx, w)
        shard = ExpertShard(world, rank, E)
        mine = pages[shard.first : shard.first + shard.per_rank].contiguous()
        ep = ExpertParallelMoE(shard, local_expert_mlp_fn(mine, ly, shard.per_rank), planner=native_planner,
                               combine=native_combine)
        out = ep.forward(x, idx, w)
        # the fixed-capacity exchange, eager and captured in a CUDA graph with its NCCL calls
        fixed = FixedCapacityExpertParallelMoE(shard, mine, ly)
        out_fixed = fixed.forward(x, idx, w)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            fixed.forward(x, idx, w)  # warm-up outside the graph
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            out_graph = fixed.forward(x, idx, w)
        graph.replay()
        torch.cuda.synchronize()
        ok = bool(torch.equal(out, single) and torch.equal(out_fixed, single) and torch.equal(out_graph, single))
        del graph  # before the process group goes away
        # the same plan over NVLink peer memory (mailboxes), eager twice and graph-replayed twice
        p2p = P2PExpertParallelMoE(shard, mine, ly, tokens=T, k=K, hidden=H)
        outs = [p2p.forward(x, idx, w) for _ in range(2)]
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            p2p.forward(x, idx, w)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            out_p2p_graph = p2p.forward(x, idx, w)
        for _ in range(2):
            graph.replay()
            torch.cuda.synchronize()
            outs.append(out_p2p_graph.clone())
        p2p.check()
        ok = ok and all(bool(torch.equal(o, single)) for o in outs)
        del graph
        dist.barrier()
        p2p.close()
        # the same exchange with this rank's pages streamed from a pinned host tier: two layers
        # holding the same pages share a slot cache of one layer's pages, so every call evicts
        from mrun_b200.streaming import ExpertPageCache, HostPageTier

        tier = HostPageTier(ly, 2, shard.per_rank)
        tier.pages[0].copy_(mine)
        tier.pages[1].copy_(mine)
        cache = ExpertPageCache(tier, budget_bytes=shard.per_rank * ly.page_stride, device=dev,
                                cache_policy="global-lru-v1", route_prefetch=False)
        layers = [P2PExpertParallelMoE(shard, None, ly, tokens=T, k=K, hidden=H, layer=i, device=dev)
                  for i in range(2)]
        for layer in layers:
            layer.page_cache = cache
        streamed = [layers[i % 2].forward(x, idx, w) for i in range(3)]
        torch.cuda.synchronize()
        for layer in layers:
            layer.check()
        ok = ok and all(bool(torch.equal(o, single)) for o in streamed) and cache.stats.evictions > 0
        dist.barrier()
        for layer in layers:
            layer.close()
        q.put((rank, ok, ep.last_stats))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_expert_parallel_bit_identical_to_single_gpu():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in results), results
