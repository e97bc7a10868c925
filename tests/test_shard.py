"""Head and chain sharding and the output all-gathers, with world_size-2 gloo ranks on CPU.

The per-rank compute here is the oracle (CPU); on the B200 the same ``sharded_heads`` /
``sharded_chains`` calls run the CUDA kernels on each GPU's share and the all-gathers go over NCCL."""

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


def test_chain_assign_balances_tokens_and_covers_every_chain():
    lengths = [864, 1220, 1400, 2231, 3155, 3845, 1932, 1905]
    for world in (1, 2, 3, 5, 8):
        parts = shard.chain_assign(lengths, 16, world)
        flat = sorted(c for p in parts for c in p)
        assert flat == [(s, h) for s in range(8) for h in range(16)]
        loads = [sum(lengths[s] for s, _ in p) for p in parts]
        assert max(loads) - min(loads) <= max(lengths)
    # Three ranks over 16 heads: contiguous head ranges would put 6/5/5 heads (all sequences) on
    # the ranks; the token balance is within one chain.
    parts = shard.chain_assign(lengths, 16, 3)
    loads = [sum(lengths[s] for s, _ in p) for p in parts]
    assert max(loads) - min(loads) <= 864


def test_pack_and_unpack_chains_round_trip():
    g = torch.Generator().manual_seed(3)
    cu = [0, 5, 5, 12, 20]
    x = torch.randn((20, 3, 4), generator=g)
    st = torch.randn((4, 3, 4, 4), generator=g)
    chains = [(2, 1), (0, 2), (1, 0), (3, 0)]
    px = shard.pack_chains(x, cu, chains)
    assert px.shape == (7 + 5 + 0 + 8, 1, 4)
    assert shard.chain_offsets(cu, chains) == [0, 7, 12, 12, 20]
    back = torch.zeros_like(x)
    shard.unpack_chains(px, cu, chains, back)
    for s_, h in chains:
        assert torch.equal(back[cu[s_]:cu[s_ + 1], h], x[cu[s_]:cu[s_ + 1], h])
    ps = shard.pack_states(st, chains)
    sback = torch.zeros_like(st)
    shard.unpack_states(ps, chains, sback)
    for s_, h in chains:
        assert torch.equal(sback[s_, h], st[s_, h])


def _kda_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import ops as oref

        g = torch.Generator().manual_seed(1)
        lengths, heads, d = [5, 40, 0, 17, 33], 3, 8
        cu = [0]
        for n in lengths:
            cu.append(cu[-1] + n)
        t = cu[-1]
        q = torch.nn.functional.normalize(torch.randn((t, heads, d), generator=g, dtype=torch.float64), dim=-1)
        k = torch.nn.functional.normalize(torch.randn((t, heads, d), generator=g, dtype=torch.float64), dim=-1)
        v = torch.randn((t, heads, d), generator=g, dtype=torch.float64)
        gl = torch.nn.functional.logsigmoid(torch.randn((t, heads, d), generator=g, dtype=torch.float64))
        beta = torch.sigmoid(torch.randn((t, heads), generator=g, dtype=torch.float64))
        s0 = 0.1 * torch.randn((len(lengths), heads, d, d), generator=g, dtype=torch.float64)

        def run(q_, k_, v_, g_, b_, cu_, s0_):
            o, f = oref.varlen_kda_gated(q_.numpy(), k_.numpy(), v_.numpy(), g_.numpy(), b_.numpy(), cu_.numpy(), 0.3,
                                         state0=None if s0_ is None else s0_.numpy())
            return torch.from_numpy(o), torch.from_numpy(f)

        out, fin = shard.sharded_chains(run, [q, k, v, gl, beta], cu, heads, state0=s0)
        ro, rf = run(q, k, v, gl, beta, torch.tensor(cu), s0)
        results[rank] = (float((out - ro).abs().max()), float((fin - rf).abs().max()))
    finally:
        dist.destroy_process_group()


def test_sharded_kda_chains_gather_output_and_final_state_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_kda_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(2):
        assert results[r][0] < 1e-12 and results[r][1] < 1e-12, results[r]
