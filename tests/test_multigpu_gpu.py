"""Head-sharded attention over 2+ GPUs with the NCCL output all-gather (needs >= 2 GPUs).

Each rank runs the tcgen05 attention kernel on its contiguous (b*h) head range and the shards are
all-gathered over NCCL; the result must be bitwise identical to one GPU running all heads (the
kernel computes every head independently).  Skipped on single-GPU machines."""

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
