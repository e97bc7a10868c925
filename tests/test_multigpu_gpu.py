"""Sharded attention and varlen KDA over 2+ GPUs with NCCL all-gathers (needs >= 2 GPUs).

Attention: each rank runs the tcgen05 kernel on its contiguous (b*h) head range.  KDA: each rank
runs the chunked kernel on the (sequence, head) chains the token balance deals it, repacked as a
single-head batch.  The shards (KDA: outputs and final states) are all-gathered over NCCL; the
result must be bitwise identical to one GPU running everything (the kernels compute every head /
chain independently).  Skipped on single-GPU machines."""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, out):
    import datetime

    import torch.distributed as dist

    from shapeforge_b200 import cases, ops, shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        shape = (2, 8, 512, 128)
        inp = cases.attention_bench_inputs(shape, "bf16")
        q, k, v = (inp[n].cuda().reshape(16, 512, 128) for n in ("q", "k", "v"))

        def attn(qs, ks, vs):
            return ops.flash_attention(qs[None], ks[None], vs[None], 128 ** -0.5, causal=True)[0]

        full_sharded = shard.sharded_heads(attn, [q, k, v], 16, head_dim=0)
        full_local = attn(q, k, v)
        torch.cuda.synchronize()
        out[rank] = bool(torch.equal(full_sharded, full_local))
    finally:
        dist.destroy_process_group()


def test_sharded_attention_over_nccl(cuda_device):
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs at least 2 GPUs")
    world = min(world, 8)
    ctx = torch.multiprocessing.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert all(out[r] for r in range(world))


def _kda_rank(rank, world, port, out):
    import datetime
    import math

    import torch.distributed as dist

    from shapeforge_b200 import cases, ops, shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        lengths = cases.kda_gated_lengths()
        heads, dim = 16, 128
        inp = {k: v.cuda() for k, v in cases.kda_gated_inputs(lengths, heads, dim, "bf16").items()}
        cu = [int(c) for c in inp["cu_seqlens"].tolist()]
        scale = 1.0 / math.sqrt(dim)

        def run(q, k, v, g, beta, cu_r, s0):
            return ops.varlen_kda_gated(q, k, v, g, beta, cu_r, scale, initial_state=s0)

        o_sh, f_sh = shard.sharded_chains(run, [inp[n] for n in ("q", "k", "v", "g", "beta")], cu, heads)
        o_1, f_1 = ops.varlen_kda_gated(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], inp["cu_seqlens"], scale)
        torch.cuda.synchronize()
        code, _ = ops.kernel_status()
        out[rank] = bool(torch.equal(o_sh, o_1)) and bool(torch.equal(f_sh, f_1)) and code == 0
    finally:
        dist.destroy_process_group()


def test_sharded_kda_chains_over_nccl(cuda_device):
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs at least 2 GPUs")
    world = min(world, 8)
    ctx = torch.multiprocessing.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _port()
    procs = [ctx.Process(target=_kda_rank, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert all(out[r] for r in range(world))
