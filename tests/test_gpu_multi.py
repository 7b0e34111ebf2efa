"""Sharded layer on 2+ GPUs: the fused output all-gather (NVLink peer stores in the
attention epilogue) must reproduce the single-GPU output bit for bit.

Runs as NCCL ranks in child processes; skipped with fewer than 2 GPUs.  NVLS
is off (NCCL_NVLS_ENABLE=0) and the kernels use plain peer stores only.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q_blocks_tokens, errors):
    import datetime

    import torch.distributed as dist

    from spruce_research_b200 import native
    from spruce_research_b200.pipeline import SparsePrefillLayer
    from spruce_research_b200.sharding import PeerOutput, plan
    from spruce_research_b200.synthetic import LayerShape, k_for_density, make_gate_weights, make_layer_inputs

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    peer = None
    try:
        shape = LayerShape(1, 28, 4, q_blocks_tokens, 128)
        K = k_for_density(shape.query_blocks, 0.10)
        q, k, v = make_layer_inputs(shape, torch.bfloat16, 3, device=dev)
        wq, wk = make_gate_weights(1, 128, 128, 4, device=dev)
        layer = SparsePrefillLayer(wq[0], wk[0], K)
        ref, sel_full = layer(q, k, v)                      # single-GPU result on this device
        s = plan(world, rank, 4, shape.query_blocks)
        g0, g1 = s.groups
        rep = 7
        peer = PeerOutput(ref.shape, ref.dtype, dev)
        peer.local.zero_()
        torch.cuda.synchronize()
        dist.barrier(device_ids=[rank])
        view = peer.local[:, :, g0 * rep:g1 * rep]
        ptrs = [p + view.storage_offset() * view.element_size() for p in peer.peer_ptrs]
        i0, i1 = s.q_blocks
        sel = layer.select(q[:, g0 * rep:g1 * rep], k[:, g0:g1], q_blocks=(i0, i1))
        native.sparse_attention(q[:, g0 * rep:g1 * rep], k[:, g0:g1], v[:, g0:g1], sel, out=view,
                                q_blocks=s.q_blocks, peer_outs=ptrs)
        peer.fence()
        torch.cuda.synchronize()
        if not torch.equal(peer.local, ref):
            own = slice(g0 * rep, g1 * rep)
            i0, i1 = s.q_blocks
            mine = peer.local[:, i0 * 64:i1 * 64, own]
            diff = (peer.local != ref)
            errors.put(f"rank {rank}: fused all-gather output differs from the single-GPU output: "
                       f"{diff.float().mean().item():.4f} of elements; own rows equal="
                       f"{torch.equal(mine, ref[:, i0 * 64:i1 * 64, own])}; zeros left="
                       f"{(peer.local == 0).float().mean().item():.4f}; "
                       f"max abs diff {(peer.local.float() - ref.float()).abs().max().item():.3e}")
        if not torch.equal(sel[:, :, i0:i1], sel_full[:, g0:g1, i0:i1]):
            errors.put(f"rank {rank}: sharded selection differs")
    except Exception as e:
        errors.put(f"rank {rank}: {type(e).__name__}: {e}")
    finally:
        torch.cuda.synchronize()
        dist.barrier(device_ids=[rank])
        if peer is not None:
            peer.close()
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_output_all_gather_matches_single_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, 8192, errors)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert codes == [0] * world and not msgs, (codes, msgs)
