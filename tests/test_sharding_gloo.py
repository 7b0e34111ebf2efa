"""Multi-rank reassembly of a sharded layer, run as gloo ranks on CPU.

Each rank takes its shard's slice of a known full [B, T, Hq, D] output
(KV-group split for world <= Hkv, half-group split beyond) and the gather
must rebuild the full tensor on every rank.  Also checks that a rank that
fails before the collective surfaces as an error on the host, not a hang.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from spruce_research_b200.sharding import ShardedSparsePrefill, plan


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, kv_heads, tokens, failures):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        rep, D, B = 3, 8, 1
        gen = torch.Generator().manual_seed(0)
        full = torch.randn((B, tokens, kv_heads * rep, D), generator=gen)
        shard = plan(world, rank, kv_heads, tokens // 64)
        g0, g1 = shard.groups
        i0, i1 = shard.q_blocks
        chunk = full[:, i0 * 64:i1 * 64, g0 * rep:g1 * rep].contiguous()
        got = ShardedSparsePrefill(shard, layer=None).gather(chunk, kv_heads, tokens)
        if not torch.equal(got, full):
            failures.put(f"rank {rank}: gathered layout differs")
    except Exception as e:  # surface to the parent test
        failures.put(f"rank {rank}: {type(e).__name__}: {e}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,kv_heads", [(2, 2), (4, 2)])
def test_gather_rebuilds_token_major_output(world, kv_heads):
    ctx = mp.get_context("spawn")
    failures = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, kv_heads, 256, failures)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    errs = []
    while not failures.empty():
        errs.append(failures.get())
    assert not errs, errs


def _dropout_worker(rank, world, port, failures):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, before the collective
    try:
        t = torch.zeros(4)
        out = torch.zeros(8)
        dist.all_gather_into_tensor(out, t)
        failures.put("rank 0: collective completed without its peer")
    except Exception:
        pass  # expected: the short process-group timeout ends the collective with an error


def test_missing_rank_ends_collective_with_error_not_hang():
    ctx = mp.get_context("spawn")
    failures = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, failures)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode is not None for p in procs)
    assert failures.empty()
