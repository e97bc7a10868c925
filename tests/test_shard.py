"""Head sharding and the output all-gather, with world_size-2 gloo ranks on CPU.

The per-rank compute here is the oracle (CPU); on the B200 the same ``sharded_heads`` call runs
the CUDA kernel on each GPU's slice and the all-gather goes over NCCL."""

from __future__ import annotations

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from shapeforge_b200 import shard


def test_head_ranges_and_lpt():
    assert shard.head_ranges(128, 8) == [(16 * i, 16 * i + 16) for i in range(8)]
    r = shard.head_ranges(10, 4)
    assert r == [(0, 3), (3, 6), (6, 8), (8, 10)]
    parts = shard.lpt_assign([864, 1220, 1400, 2231, 3155, 3845, 1932, 1905], 2)
    loads = [sum([864, 1220, 1400, 2231, 3155, 3845, 1932, 1905][i] for i in p) for p in parts]
    assert sorted(i for p in parts for i in p) == list(range(8))
    assert max(loads) - min(loads) <= 3845


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import ops as oref

        g = torch.Generator().manual_seed(0)
        b, h, s, d = 2, 3, 16, 8
        q, k, v = (torch.randn((b, h, s, d), generator=g, dtype=torch.float64) for _ in range(3))

        def attn(qs, ks, vs):
            return torch.from_numpy(oref.attention(qs[None].numpy(), ks[None].numpy(), vs[None].numpy(), 0.3, causal=True)[0])

        flat = [t.reshape(b * h, s, d) for t in (q, k, v)]
        out = shard.sharded_heads(attn, flat, b * h, head_dim=0)
        full = attn(*flat)
        results[rank] = float((out - full).abs().max())
    finally:
        dist.destroy_process_group()


def test_sharded_attention_gathers_the_full_output_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(results) == {0: 0.0, 1: 0.0}
