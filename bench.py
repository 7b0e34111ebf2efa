#!/usr/bin/env python
"""Benchmark of the SPRUCE sparse-prefill layer on B200.

One step = the whole hot path of one 28Q/4KV-head, d=128, bf16 attention
layer at 131072 tokens and 10% block density (K=106): block-mean pooling of
Q and K, FlatGate scores, masked top-k packed into selected_blocks, and causal
GQA block-sparse attention over the selected tiles.  With N GPUs (torchrun)
the layer is sharded by KV group (N=2, 4) or half group (N=8) and the outputs
are all-gathered over NCCL; total work is fixed, so scaling is strong.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    python bench.py --sweep          # config 4: variable-length batch, densities 2..100%
    python bench.py --model          # config 3: whole-model prefill TTFT, dense vs SPRUCE flows
    python bench.py --tree-selector  # deployed selector (P=8 prototypes, key tree, beam 16) ms/layer
    python bench.py --residual       # residual-summary attention (summary table + attention) ms/layer

`value` is effective TFLOP/s of the selected tiles (algorithmic FLOPs of the
step / device time of the step, max over ranks); `e2e` is the same metric
with the inputs copied from pinned host memory and the output copied back
inside the timed region; `--impl reference` times the CPU restatement of the
reference path (the oracle port) on a bounded sample of the same workload.
Inputs are synthetic (seeded N(0,1) with RoPE and planted affinity) and
larger than L2 (Q alone is 0.94 GB), so no L2 flush is needed.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sparse-prefill ms/layer & effective TFLOP/s at 128K, 10% density, 1/2/4/8 B200"
PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
# The attention kernel the library runs (SPRUCE_ATTN_KERNEL=single selects the one-block-per-step kernel)
# and the ncu summary that holds its DRAM bytes per full-size launch.
ATTN_KERNEL = ("attn_fwd_sm100_kernel<bf16,128,4>" if os.environ.get("SPRUCE_ATTN_KERNEL") == "single"
               else "attn_pair_sm100_kernel<bf16,128,2>")
TRAFFIC_FILE = os.path.join(ROOT, "profiles", "attn_fwd_sm100_c2.md" if os.environ.get("SPRUCE_ATTN_KERNEL") == "single"
                            else "attn_pair_sm100_c2.md")
FALLBACK_PEAK_TFLOPS = 1590.0


# The one JSON line goes to the process's real stdout; everything else -- including what
# native libraries (NCCL's version banner, for one) write to file descriptor 1 -- goes to
# stderr, so rank 0's stdout carries exactly one line.
_JSON_OUT = None


def _claim_stdout():
    global _JSON_OUT
    if _JSON_OUT is None:
        sys.stdout.flush()
        _JSON_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)


def emit(result: dict) -> None:
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(result) + "\n")
    out.flush()


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--tokens", type=int, default=131072)
    ap.add_argument("--density", type=float, default=0.10)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end measurement")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-chunks", type=int, default=16, help="query-block chunks of the streamed e2e step")
    ap.add_argument("--e2e-schedule", choices=("balanced", "equal"), default="balanced",
                    help="chunk bounds of the streamed e2e step: equal attention work or equal query blocks")
    ap.add_argument("--no-numa-bind", action="store_true",
                    help="pin the e2e host buffers wherever the process runs, not on the GPU's NUMA node")
    ap.add_argument("--cpu-seconds", type=float, default=24.0, help="target length of one CPU sample")
    ap.add_argument("--gather", choices=("fused", "nccl"), default="fused",
                    help="N>1 output all-gather: NVLink peer stores in the attention epilogue, or NCCL")
    ap.add_argument("--sweep", action="store_true",
                    help="config 4 instead: 8 variable-length sequences, densities 2..100%%, one GPU")
    ap.add_argument("--model", action="store_true",
                    help="config 3 instead: whole Qwen2-7B-shaped model prefill TTFT, dense vs SPRUCE flows")
    ap.add_argument("--model-tokens", type=int, default=65536)
    ap.add_argument("--residual", action="store_true",
                    help="residual-summary attention at config 2 (summary table + attention, P = 1 and 4)")
    ap.add_argument("--tree-selector", action="store_true",
                    help="time the deployed tree selector (P=8, beam 16) beside the flat one at config 2's shape")
    return ap.parse_args()


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader",
                 "-lms", "200", "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            with open(self.path) as f:
                for r in csv.reader(io.StringIO(f.read())):
                    if len(r) >= 9:
                        rows.append([c.strip() for c in r])
            os.unlink(self.path)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def mhz(s):
            try:
                return float(s.split()[0])
            except (ValueError, IndexError):
                return None

        sm = [mhz(r[1]) for r in rows if mhz(r[1]) is not None]
        loaded = [x for x in sm if x > 500] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k].lower().startswith("active")})
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": mhz(rows[0][2]), "reasons": reasons, "samples": len(rows)}


# ----------------------------------------------------------------- helpers
def measured_peak(sustained: bool = False):
    """Dense bf16 peak for the roofline: the burst cuBLAS figure for kernels timed over a short
    region at full clock (the default: a timed region of ~0.1-0.2 s), the sustained one for
    seconds-long loops under the power cap."""
    key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    try:
        with open(PEAKS_FILE) as f:
            peaks = json.load(f)
        return float(peaks[key]), f"measured {key} (MEASURED_PEAKS.json)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_PEAK_TFLOPS, "fallback 1.59 PFLOP/s (no MEASURED_PEAKS.json)"


def profiled_traffic(tokens: int):
    """DRAM bytes per attention launch from the committed ncu summary, scaled to `tokens`."""
    try:
        with open(TRAFFIC_FILE) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_c2_launch:"):
                    b = float(line.split(":", 1)[1].split()[0])
                    return b if tokens == 131072 else None
    except (OSError, ValueError):
        pass
    return None


def workload(args):
    from spruce_research_b200.synthetic import LayerShape, causal_block_entries, k_for_density, sparse_attention_flops

    shape = LayerShape(1, 28, 4, args.tokens, 128)
    K = k_for_density(shape.query_blocks, args.density)
    entries = causal_block_entries(shape.query_blocks, K)
    flops = sparse_attention_flops(shape, entries)
    return shape, K, entries, flops


def config_dict(args, shape, K, entries, world):
    par = {1: "single GPU", 2: "kv-group x2", 4: "kv-group x4", 8: "half kv-group x8"}.get(world, f"x{world}")
    if world > 1:
        par += (", output all-gather fused into the attention epilogue (NVLink peer stores)"
                if args.gather == "fused" else ", NCCL all_gather")
    return {
        "workload": (f"config 2: one Qwen2.5-7B-shaped attention layer, {shape.tokens} tokens, "
                     f"{shape.q_heads}Q/{shape.kv_heads}KV heads, d={shape.head_dim}, bf16, "
                     f"{args.density:.0%} block density (K={K}), selector + block-sparse attention"),
        "tokens": shape.tokens, "q_heads": shape.q_heads, "kv_heads": shape.kv_heads, "head_dim": shape.head_dim,
        "block": 64, "k_selected": K, "entries_per_kv_group": entries, "parallelism": par,
        "l2": "inputs larger than L2 (Q 0.94 GB, K/V 0.13 GB each); no flush",
    }


def shard_flops(shape, K, shard) -> float:
    """Algorithmic FLOPs of this rank's attention launch (its groups and query blocks)."""
    g0, g1 = shard.groups
    i0, i1 = shard.q_blocks
    rep = shape.q_heads // shape.kv_heads
    entries = sum(min(i + 1, K) for i in range(i0, i1))
    rows = i1 - i0
    pairs = (entries - rows) * 64 * 64 + rows * 64 * 65 / 2
    return 4.0 * shape.head_dim * rep * (g1 - g0) * pairs * shape.batch


# ----------------------------------------------------------------- CPU baseline (oracle port)
def cpu_sample(shape, K, q, k, v, wq, wk, target_s: float, rows: int | None = None):
    """Time the CPU restatement of the reference path on a bounded sample.

    Sample: KV group 0 (7 query heads) -- its whole selector (pooling, gate,
    top-k, packing) plus attention of the last M query blocks (each with K
    selected blocks); M is calibrated so one sample takes ~target_s seconds.
    Returned TFLOP/s = attention FLOPs of the M rows / (attention time + the
    selector time prorated to M/qb of the rows).  The third value holds the
    oracle's group-0 selection and the fp32 output rows of the sample, which
    the GPU arm compares with its own step.
    """
    import torch

    from oracle import oracle as O

    rep = shape.q_heads // shape.kv_heads
    qb = shape.query_blocks
    q0 = q[:, 0:rep].transpose(1, 2).contiguous().cpu().transpose(1, 2)
    k0 = k[:, 0:1].transpose(1, 2).contiguous().cpu().transpose(1, 2)
    v0 = v[:, 0:1].transpose(1, 2).contiguous().cpu().transpose(1, 2)
    wq, wk = wq.cpu(), wk.cpu()

    t0 = time.perf_counter()
    sel = O.select_blocks(q0, k0, wq, wk, K, 0, 1)["selected"]
    t_sel = time.perf_counter() - t0
    last = {}

    def attn_rows(m):
        t = time.perf_counter()
        last["out"] = O.sparse_attention(q0, k0, v0, sel, out_dtype=torch.float32, q_blocks=(qb - m, qb))
        return time.perf_counter() - t

    m = rows
    if m is None:
        t4 = attn_rows(4)
        m = int(max(1, min(qb, round(4 * max(target_s, 0.5) / max(t4, 1e-3)))))
    best = attn_rows(m) + t_sel * m / qb
    rows_flops = 4.0 * shape.head_dim * rep * m * ((K - 1) * 4096 + 64 * 65 / 2)
    checked = {"selected_g0": sel[:, 0], "out_rows": last["out"][:, (qb - m) * 64:], "blocks": (qb - m, qb)}
    return {
        "value": rows_flops / best / 1e12, "unit": "TFLOP/s", "cores": O.num_threads(), "kind": "port",
        "seconds": best,
        "sample": (f"oracle C port (OpenMP, {O.num_threads()} threads): KV group 0 selector "
                   f"({t_sel:.2f} s, prorated {m}/{qb}) + attention of the last {m} query blocks x {rep} heads, "
                   f"K={K}; fp32 math on bf16 inputs"),
    }, m, checked


def headline_fixture(args, shape, K):
    """The reference's outputs for this exact workload (tests/golden/c2.npz), or None.

    They exist for BASELINE config 2 with the default inputs: 131072 tokens, 10%
    density, seed 0 (gate seed 1).
    """
    path = os.path.join(ROOT, "tests", "golden", "c2.npz")
    if not os.path.exists(path):
        return None
    import numpy as np

    z = np.load(path)
    shp = [int(x) for x in z["shape"]]
    if (shp != [shape.batch, shape.q_heads, shape.kv_heads, shape.tokens, shape.head_dim]
            or int(z["policy"][0]) != K or int(z["seed"][0]) != args.seed or int(z["wseed"][0]) != args.seed + 1):
        return None
    return z


def reference_cpu_record(fixture, flops: float):
    """The reference's own CPU torch path at this workload, as timed where the fixture was made.

    tests/golden/make_golden.py runs the reference's functions (pooling, FlatGate, mask and
    top-k, selected_ids_to_blocks, sparse_prefill_attention_forward) on these inputs and
    stores their wall time; the reference checkout itself does not travel to the GPU box.
    """
    if fixture is None or "ref_cpu" not in fixture.files:
        return None
    t_sel, t_attn, threads, cpus = (float(x) for x in fixture["ref_cpu"])
    return {"value": flops / (t_sel + t_attn) / 1e12, "unit": "TFLOP/s", "seconds_per_layer": t_sel + t_attn,
            "selector_s": t_sel, "attention_s": t_attn, "torch_threads": int(threads), "cpu_count": int(cpus),
            "kind": "reference",
            "where": ("the reference's own torch functions, whole layer (all 4 KV groups, every query block), timed "
                      "by tests/golden/make_golden.py on the host that generated the fixtures, not on this box")}


def attention_error(got, want) -> dict:
    err = (got.float().cpu() - want.float().cpu()).abs()
    return {"max_abs": err.max().item(), "mean_abs": err.mean().item()}


# ----------------------------------------------------------------- GPU arm
def run_b200(args):
    import datetime

    import torch
    import torch.distributed as dist

    from spruce_research_b200 import hostmem, native
    from spruce_research_b200.pipeline import HostStreamedLayer, SparsePrefillLayer
    from spruce_research_b200.sharding import PeerOutput, ShardedSparsePrefill, plan
    from spruce_research_b200.synthetic import make_gate_weights, make_layer_inputs

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # rank 0's stdout must carry exactly one JSON line: keep NCCL's version banner off it
    if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
        os.environ["NCCL_DEBUG"] = "WARN"
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))

    shape, K, entries, flops = workload(args)
    qb = shape.query_blocks
    # Made on the CPU (seeded torch.Generator), as the golden fixtures' inputs are, then moved to
    # HBM in the [B, T, H, D] storage the reference's callers hand over.
    q_host, k_host, v_host = make_layer_inputs(shape, torch.bfloat16, args.seed)
    q, k, v = (t.transpose(1, 2).to(dev).transpose(1, 2) for t in (q_host, k_host, v_host))
    wq, wk = (w.to(dev) for w in make_gate_weights(1, shape.head_dim, shape.head_dim, args.seed + 1))
    layer = SparsePrefillLayer(wq[0], wk[0], K, local_window=0, sink_blocks=1)
    # the fused gather takes unequal chunks, so its half-group split balances selected tiles
    shard = plan(world, rank, shape.kv_heads, qb, k_selected=K if args.gather == "fused" else None)
    runner = ShardedSparsePrefill(shard, layer)
    g0, g1 = shard.groups
    rep = shape.q_heads // shape.kv_heads
    i0, i1 = shard.q_blocks
    B, T, D = shape.batch, shape.tokens, shape.head_dim
    sel_buf = torch.empty((B, g1 - g0, qb, K), device=dev, dtype=torch.int32)
    fused = world > 1 and args.gather == "fused"
    peer = None
    if fused:
        # every rank's full output is mapped into every other rank; this rank's heads are a view
        peer = PeerOutput((B, T, shape.q_heads, D), torch.bfloat16, dev)
        local_out = peer.local[:, :, g0 * rep:g1 * rep]
        view_bytes = local_out.storage_offset() * local_out.element_size()
        peer_ptrs = [ptr + view_bytes for ptr in peer.peer_ptrs]
    else:
        local_out = torch.empty((B, T, (g1 - g0) * rep, D), device=dev, dtype=torch.bfloat16)
        peer_ptrs = None

    def step(qs, ks, vs, marks=None):
        """This rank's selector + attention (+ all-gather); q/k/v are its shard's views."""
        if marks is not None:
            marks[0].record()
        sel = layer.select(qs, ks, out=sel_buf, q_blocks=(i0, i1))
        if marks is not None:
            marks[1].record()
        native.sparse_attention(qs, ks, vs, sel, out=local_out, q_blocks=(i0, i1), peer_outs=peer_ptrs)
        if marks is not None:
            marks[2].record()
        full = local_out
        if fused:
            peer.fence()
            full = peer.local
        elif world > 1:
            full = runner.gather(local_out[:, i0 * 64:i1 * 64], shape.kv_heads, T)
        if marks is not None:
            marks[3].record()
        return full

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    q_shard, k_shard, v_shard = q[:, g0 * rep:g1 * rep], k[:, g0:g1], v[:, g0:g1]
    for _ in range(args.warmup):
        step(q_shard, k_shard, v_shard)
    barrier()
    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        for s in range(args.steps):
            step(q_shard, k_shard, v_shard, marks[s])
        stop.record()
        barrier()
    elapsed_ms = max_over_ranks(start.elapsed_time(stop))
    ms = elapsed_ms / args.steps
    sel_ms = statistics.mean(m[0].elapsed_time(m[1]) for m in marks)
    attn_ms = statistics.mean(m[1].elapsed_time(m[2]) for m in marks)
    gather_ms = statistics.mean(m[2].elapsed_time(m[3]) for m in marks)
    attn_ms_max = max_over_ranks(attn_ms)
    sel_ms_max = max_over_ranks(sel_ms)
    gather_ms_max = max_over_ranks(gather_ms)

    # ---- end to end through the public API with pinned host buffers
    e2e = None
    if not args.no_e2e:
        # pinned on this GPU's NUMA node (hostmem.near), unless --no-numa-bind
        pin = (lambda t: t.contiguous().cpu().pin_memory()) if args.no_numa_bind else \
            (lambda t: hostmem.pinned_copy(t, dev))
        hq = pin(q[:, g0 * rep:g1 * rep].transpose(1, 2))   # [B, T, Hr, D]
        hk = pin(k[:, g0:g1].transpose(1, 2))
        hv = pin(v[:, g0:g1].transpose(1, 2))
        dq, dk, dv = (torch.empty_like(t, device=dev) for t in (hq, hk, hv))
        # each rank reads back the rows and heads it computed: over all ranks, the whole output
        hout = (torch.empty((B, T, (g1 - g0) * rep, D), dtype=torch.bfloat16).pin_memory() if args.no_numa_bind
                else hostmem.pinned_empty((B, T, (g1 - g0) * rep, D), torch.bfloat16, dev))
        streamer = HostStreamedLayer(layer, dev, chunks=args.e2e_chunks, schedule=args.e2e_schedule)

        def e2e_step():
            # H2D of chunk c+1, selector + attention of chunk c and D2H of chunk c-1 overlap
            streamer(hq, hk, hv, dq, dk, dv, local_out, hout=hout, q_blocks=(i0, i1), peer_outs=peer_ptrs)
            if world > 1:  # the on-device all-gather completes as part of the step
                if fused:
                    peer.fence()
                else:
                    runner.gather(local_out[:, i0 * 64:i1 * 64], shape.kv_heads, T)

        for _ in range(max(1, args.warmup)):
            e2e_step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            e2e_step()
        e1.record()
        barrier()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
        moved = torch.tensor([streamer.h2d_bytes, streamer.d2h_bytes], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(moved)
        e2e = {"value": flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": int(moved[0].item()), "d2h_bytes_per_step": int(moved[1].item()),
               "path": ("pinned host Q/K/V -> HostStreamedLayer (copies of chunk c+1, selector + attention of "
                        f"chunk c and copy-back of chunk c-1 overlap; {args.e2e_chunks} query-block chunks, "
                        f"{args.e2e_schedule} schedule) -> "
                        "pinned host output" + ("" if world == 1 else
                                                "; each rank copies its own query rows, the K/V rows they "
                                                "attend and its output shard (bytes summed over ranks)")),
               "host_numa": "process default" if args.no_numa_bind else
               f"pinned on the GPU's NUMA node ({len(hostmem.gpu_local_cpus(dev)) or 'unknown'} local CPUs)"}
        del dq, dk, dv

    # ---- parity of this very workload (untimed): the reference's outputs, then the oracle's
    full = step(q_shard, k_shard, v_shard)
    torch.cuda.synchronize()
    parity = {}
    fixture = headline_fixture(args, shape, K)
    if fixture is not None:
        import numpy as np

        cs = np.array([t.double().sum().item() for t in (q_host, k_host, v_host)])
        if np.allclose(cs, fixture["checksum"], rtol=1e-12, atol=1e-6):
            want = torch.from_numpy(fixture["selected"].astype(np.int32))[:, g0:g1, i0:i1].to(dev)
            counts = torch.tensor([(sel_buf[:, :, i0:i1] == want).all(-1).sum().item(), want[..., 0].numel()],
                                  dtype=torch.float64, device=dev)
            if world > 1:
                dist.all_reduce(counts)
            blocks = [int(b) for b in fixture["out_blocks"]]
            rows = torch.cat([torch.arange(b * 64, min((b + 1) * 64, T)) for b in blocks]).to(dev)
            ref_out = torch.from_numpy(fixture["out"]).view(torch.bfloat16)
            parity["reference"] = {"rows_equal": int(counts[0].item()), "rows_total": int(counts[1].item()),
                                   "sampled_query_blocks": blocks,
                                   "attn": attention_error(full[:, rows], ref_out),
                                   "source": "tests/golden/c2.npz: the reference's own selector and "
                                             "sparse_prefill_attention_forward on these inputs"}
        else:
            parity["reference"] = {"skipped": "this host regenerated other inputs than the fixture's"}

    # ---- CPU baseline (rank 0, single GPU only)
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu, _, checked = cpu_sample(shape, K, q_host, k_host, v_host, wq[0], wk[0], args.cpu_seconds)
        ref_rec = reference_cpu_record(fixture, flops)
        if ref_rec is not None:
            cpu["reference_torch_path"] = ref_rec
        c0, c1 = checked["blocks"]
        parity["oracle"] = {"rows_equal": int((sel_buf[:, 0].cpu() == checked["selected_g0"]).all(-1).sum()),
                            "rows_total": qb, "kv_group": 0, "query_blocks": [c0, c1],
                            "attn": attention_error(full[:, c0 * 64:c1 * 64, 0:rep], checked["out_rows"])}

    peak, peak_src = measured_peak()
    r_flops = shard_flops(shape, K, shard)
    achieved = r_flops / (attn_ms * 1e-3) / 1e12
    result = {
        "metric": METRIC,
        "value": flops / (ms * 1e-3) / 1e12,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "ms_per_layer": ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) Q/K/V, RoPE base 1e6, planted affinity (3 blocks/query block)",
        "config": config_dict(args, shape, K, entries, world),
        "breakdown_ms": {"selector": sel_ms_max, "attention": attn_ms_max,
                         ("fence" if fused else "gather"): gather_ms_max},
        "roofline": {"bound": "tensor", "kernel": ATTN_KERNEL,
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                     "peak_source": peak_src + ", of measured",
                     "frac_of_sustained": achieved / measured_peak(sustained=True)[0],
                     "flops_per_launch": r_flops, "traffic": profiled_traffic(shape.tokens)},
        "gpu_launches": layer.launches_per_call(B, g1 - g0, (i0, i1)) * args.steps,
        "clocks": clocks.summary(),
        "parity": parity,
    }
    if e2e is not None:
        result["e2e"] = e2e
    if cpu is not None:
        result["cpu_baseline"] = cpu
    if rank == 0:
        emit(result)
    if world > 1:
        dist.barrier(device_ids=[local])
        if peer is not None:
            torch.cuda.synchronize()
            peer.close()
            dist.barrier(device_ids=[local])
        dist.destroy_process_group()


# ----------------------------------------------------------------- reference arm
def run_reference(args):
    """CPU restatement of the reference path (oracle port) on the host cores, rank 0 only."""
    import torch

    from spruce_research_b200.synthetic import make_gate_weights, make_layer_inputs

    if int(os.environ.get("RANK", "0")) != 0:
        return
    shape, K, entries, flops = workload(args)
    # the GPU arm's inputs: made on the CPU from the same seeds
    q, k, v = make_layer_inputs(shape, torch.bfloat16, args.seed)
    wq, wk = make_gate_weights(1, shape.head_dim, shape.head_dim, args.seed + 1)
    # Size the sample once (about cpu_seconds of CPU work), then time it per step.
    info, m, _ = cpu_sample(shape, K, q, k, v, wq[0], wk[0], target_s=min(args.cpu_seconds, 8.0))
    steps = []
    for s in range(args.warmup + args.steps):
        r, _, _ = cpu_sample(shape, K, q, k, v, wq[0], wk[0], 0.0, rows=m)
        if s >= args.warmup:
            steps.append(r["value"])
            info = r
    value = statistics.median(steps)
    ms = flops / (value * 1e12) * 1e3
    result = {
        "metric": METRIC, "impl": "reference", "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "ms_per_layer": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) Q/K/V, RoPE base 1e6, planted affinity (3 blocks/query block)",
        "config": config_dict(args, shape, K, entries, args.gpus),
        "cpu_baseline": {**info, "value": value},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("ms_per_step extrapolates the sample's rate to the whole layer; the reference's Python checkout "
                 "cannot run on this box, so this arm times the C restatement of its path (kind 'port'); "
                 "cpu_baseline.reference_torch_path is the reference's own torch path timed where the fixtures "
                 "were made"),
    }
    ref_rec = reference_cpu_record(headline_fixture(args, shape, K), flops)
    if ref_rec is not None:
        result["cpu_baseline"]["reference_torch_path"] = ref_rec
    emit(result)


def run_sweep(args):
    """a packed batch of 8 sequences, lengths U[8192, 131072] rounded to 64,
    28Q/4KV heads, d=128, bf16, at densities 2/5/10/25/50/100%; the 100% case is checked
    against dense causal attention (torch's SDPA in bf16, a checker only)."""
    import torch
    import torch.nn.functional as F

    from spruce_research_b200.synthetic import (LayerShape, causal_block_entries, k_for_density,
                                                make_gate_weights, make_layer_inputs, sparse_attention_flops)
    from spruce_research_b200.varlen import VarlenSparsePrefill

    dev = torch.device("cuda", 0)
    gen = torch.Generator().manual_seed(args.seed + 4)
    lengths = [int(x) // 64 * 64 for x in torch.randint(8192, 131072 + 1, (8,), generator=gen)]
    Hq, Hkv, D = 28, 4, 128
    qs, ks, vs = [], [], []
    for n, T in enumerate(lengths):
        q, k, v = make_layer_inputs(LayerShape(1, Hq, Hkv, T, D), torch.bfloat16, args.seed + 100 + n)
        qs.append(q[0].transpose(0, 1))
        ks.append(k[0].transpose(0, 1))
        vs.append(v[0].transpose(0, 1))
    q = torch.cat(qs).contiguous().to(dev)
    k = torch.cat(ks).contiguous().to(dev)
    v = torch.cat(vs).contiguous().to(dev)
    del qs, ks, vs
    cu = [0]
    for T in lengths:
        cu.append(cu[-1] + T)
    wq, wk = make_gate_weights(1, D, D, args.seed + 1000, device=dev)
    runner = VarlenSparsePrefill(wq[0], wk[0])
    out = torch.empty_like(q)
    peak, peak_src = measured_peak(sustained=True)  # the sweep runs for seconds under the power cap
    rows = []
    for density in (0.02, 0.05, 0.10, 0.25, 0.50, 1.0):
        flops = 0.0
        for T in lengths:
            qb = (T + 63) // 64
            K = runner.k_for(T, density, None)
            flops += sparse_attention_flops(LayerShape(1, Hq, Hkv, T, D), causal_block_entries(qb, K))
        for _ in range(max(1, args.warmup)):
            runner(q, k, v, cu, density=density, out=out)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            runner(q, k, v, cu, density=density, out=out)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        rows.append({"density": density, "ms_per_batch": ms, "tflops": flops / (ms * 1e-3) / 1e12,
                     "frac_of_peak": flops / (ms * 1e-3) / 1e12 / peak,
                     "k_selected": [runner.k_for(T, density, None) for T in lengths]})
    # 100%: every causal block, which must equal dense causal attention
    runner(q, k, v, cu, density=1.0, out=out)
    worst_max, err_sum, n_el = 0.0, 0.0, 0
    for a, b in zip(cu, cu[1:]):
        dense = F.scaled_dot_product_attention(q[a:b].transpose(0, 1)[None], k[a:b].transpose(0, 1)[None],
                                               v[a:b].transpose(0, 1)[None], is_causal=True,
                                               enable_gqa=True)[0].transpose(0, 1)
        err = (out[a:b].float() - dense.float()).abs()
        worst_max = max(worst_max, err.max().item())
        err_sum += err.sum().item()
        n_el += err.numel()
    ten = next(r for r in rows if r["density"] == 0.10)
    result = {
        "metric": "sparse-prefill density/length sweep (config 4), effective TFLOP/s",
        "value": ten["tflops"], "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ten["ms_per_batch"], "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) Q/K/V, RoPE base 1e6, planted affinity",
        "config": {"workload": "config 4: packed batch of 8 sequences, 28Q/4KV heads, d=128, bf16",
                   "lengths": lengths, "tokens": cu[-1]},
        "peak": peak, "peak_source": peak_src,
        "sweep": rows,
        "dense_check": {"max_abs": worst_max, "mean_abs": err_sum / n_el,
                        "pass": worst_max < 2e-2 and err_sum / n_el < 2e-3,
                        "reference": "torch scaled_dot_product_attention (bf16, causal, GQA) per sequence"},
    }
    emit(result)


def run_model(args):
    """prefill of a random-init bf16 Qwen2-7B-shaped model (hidden 3584, FFN 18944,
    28 layers, 28/4 heads, vocab 152064, RoPE base 1e6 with YaRN factor 4) on seeded random token ids.

    Each flow's TTFT is timed with CUDA events from the pinned host token ids to the first generated
    token id back in pinned host memory: the dense SDPA model, and SPRUCE's one-pass (route inside each
    layer's attention call) and two-pass (dense feature capture, routing, sparse forward) flows with the
    flat gate at ``--density`` and the deployed tree gate (P=8, beam 16).  The random-init model's last
    logits at 10% density need not resemble the dense model's; the all-blocks flow (every causal block
    selected) must."""
    import math

    import torch
    from transformers import Qwen2Config, Qwen2ForCausalLM

    from spruce_research_b200.kernels.sparse_prefill import SPRUCE_TRITON_SPARSE_PREFILL
    from spruce_research_b200.live import LiveSelector, capture_selector_features, sparse_prefill
    from spruce_research_b200.selector.gate import FlatGate
    from spruce_research_b200.synthetic import causal_block_entries

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    T = args.model_tokens
    cfg = Qwen2Config(vocab_size=152064, hidden_size=3584, intermediate_size=18944, num_hidden_layers=28,
                      num_attention_heads=28, num_key_value_heads=4, max_position_embeddings=131072,
                      rope_parameters={"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 32768,
                                       "rope_theta": 1e6})
    torch.manual_seed(args.seed)
    default = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(dev):
            model = Qwen2ForCausalLM(cfg).eval()
            gate = FlatGate(28, 128, 128).float().eval()
    finally:
        torch.set_default_dtype(default)
    model.set_attn_implementation("sdpa")
    ids_host = torch.randint(0, cfg.vocab_size, (1, T), generator=torch.Generator().manual_seed(args.seed + 3))
    ids_host = ids_host.pin_memory()
    tok_host = torch.empty((), dtype=torch.int64).pin_memory()
    qb = math.ceil(T / 64)
    flat = LiveSelector(gate, mode="flat", density=args.density, local_window=0, sink_blocks=1)
    tree = LiveSelector(gate, mode="tree", beam=16, radix=2, prototypes=8, local_window=1, sink_blocks=0)
    # every causal block: the sparse path must then reproduce the dense model
    full = LiveSelector(gate, mode="flat", k_selected=qb, local_window=0, sink_blocks=1)

    def two_pass(selector, marks):
        def run(ids):
            marks.append(torch.cuda.Event(enable_timing=True))
            marks[-1].record()
            feats = capture_selector_features(model, ids, selector.feature_prototypes)
            marks.append(torch.cuda.Event(enable_timing=True))
            marks[-1].record()
            selected = selector.route(feats)
            del feats
            marks.append(torch.cuda.Event(enable_timing=True))
            marks[-1].record()
            model.set_attn_implementation(SPRUCE_TRITON_SPARSE_PREFILL)
            try:
                return model(ids, use_cache=True, logits_to_keep=1, selected_blocks=selected, block_size=64)
            finally:
                model.set_attn_implementation("sdpa")
        return run

    phase_marks = {"spruce_two_pass_flat": [], "spruce_two_pass_tree": []}
    flows = {
        "dense_sdpa": lambda ids: model(ids, use_cache=True, logits_to_keep=1),
        "spruce_one_pass_flat": lambda ids: sparse_prefill(model, ids, flat, flow="one_pass")[0],
        "spruce_two_pass_flat": two_pass(flat, phase_marks["spruce_two_pass_flat"]),
        "spruce_one_pass_tree": lambda ids: sparse_prefill(model, ids, tree, flow="one_pass")[0],
        "spruce_two_pass_tree": two_pass(tree, phase_marks["spruce_two_pass_tree"]),
        "spruce_one_pass_all_blocks": lambda ids: sparse_prefill(model, ids, full, flow="one_pass")[0],
    }
    results, dense_logits = {}, None
    with torch.no_grad():
        for name, fn in flows.items():
            times, logits = [], None
            for it in range(max(1, args.warmup) + args.steps):
                marks = phase_marks.get(name)
                if marks is not None:
                    marks.clear()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                e0.record()
                ids = ids_host.to(dev, non_blocking=True)
                out = fn(ids)
                tok_host.copy_(out.logits[0, -1].argmax(), non_blocking=True)
                e1.record()
                e1.synchronize()
                if it >= max(1, args.warmup):
                    times.append(e0.elapsed_time(e1))
                logits = out.logits[0, -1].float()
                del out
            row = {"ttft_ms": statistics.median(times), "ttft_ms_all": times, "first_token": int(tok_host)}
            if name in phase_marks:
                m = phase_marks[name]
                row["phases_ms_last_step"] = {"capture": m[0].elapsed_time(m[1]), "route": m[1].elapsed_time(m[2]),
                                              "sparse_forward_and_first_token": m[2].elapsed_time(e1)}
            if dense_logits is None:
                dense_logits = logits
            else:
                row["last_logits_vs_dense"] = {
                    "cosine": torch.nn.functional.cosine_similarity(logits, dense_logits, dim=0).item(),
                    "max_abs": (logits - dense_logits).abs().max().item(),
                    "same_first_token": row["first_token"] == results["dense_sdpa"]["first_token"]}
            results[name] = row
            torch.cuda.empty_cache()
    K_flat = flat.width(qb)
    flat_density = causal_block_entries(qb, K_flat) / (qb * (qb + 1) // 2)
    one = results["spruce_one_pass_flat"]["ttft_ms"]
    emit({
        "metric": "config 3 prefill TTFT, Qwen2-7B-shaped random-init bf16 model",
        "value": one, "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": one, "higher_is_better": False, "dtype": "bf16",
        "data": "synthetic: random-init weights (seeded), random token ids",
        "config": {"workload": f"config 3: Qwen2-7B shape, {T} tokens, YaRN factor 4",
                   "tokens": T, "query_blocks": qb, "flat_k_selected": K_flat, "flat_charged_density": flat_density,
                   "tree": {"beam": 16, "prototypes": 8, "k_selected": tree.width(qb)}},
        "flows": results,
        "speedup_vs_dense": {k: results["dense_sdpa"]["ttft_ms"] / v["ttft_ms"] for k, v in results.items()},
    })


def run_tree_selector(args):
    """The deployed selector at config 2's layer shape: P=8 outlier
    prototypes, the key tree and a beam-16 traversal (K = 18), beside the flat P=1 selector (K at
    ``--density``).  Device time per layer with CUDA events; selection only, no attention."""
    import torch

    from spruce_research_b200.pipeline import SparsePrefillLayer
    from spruce_research_b200.selector.gate import FlatGate
    from spruce_research_b200.selector.tree import tree_select_blocks
    from spruce_research_b200.synthetic import LayerShape, k_for_density, make_gate_weights, make_layer_inputs

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    shape = LayerShape(1, 28, 4, args.tokens, 128)
    q, k, _ = make_layer_inputs(shape, torch.bfloat16, args.seed, device=dev)
    wq, wk = make_gate_weights(1, 128, 128, args.seed + 1, device=dev)
    gate = FlatGate(1, 128, 128).to(dev).eval()
    with torch.no_grad():
        gate.Wq.copy_(wq)
        gate.Wk.copy_(wk)
    qb = (args.tokens + 63) // 64
    flat = SparsePrefillLayer(wq[0], wk[0], k_for_density(qb, args.density), 0, 1)

    def timed(fn):
        for _ in range(max(1, args.warmup)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    tree_ms = timed(lambda: tree_select_blocks(q, k, gate, beam=16, radix=2, prototypes=8))
    flat_ms = timed(lambda: flat.select(q, k))
    sel = tree_select_blocks(q, k, gate, beam=16, radix=2, prototypes=8)
    emit({
        "metric": "deployed tree selector ms/layer (P=8, beam 16) beside the flat selector",
        "value": tree_ms, "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": tree_ms, "higher_is_better": False, "dtype": "bf16 features, fp32 scores",
        "data": "synthetic: seeded N(0,1) Q/K, RoPE base 1e6, planted affinity; kaiming-uniform gate",
        "config": {"workload": f"config 2 layer shape, {args.tokens} tokens, 28Q/4KV, d=p=128",
                   "tree": {"prototypes": 8, "beam": 16, "radix": 2, "k_selected": int(sel.shape[-1]),
                            "entries_per_group": int((sel[0, 0] >= 0).sum())},
                   "flat": {"k_selected": flat.k_selected}},
        "flat_selector_ms": flat_ms,
    })


def run_residual(args):
    """Residual-summary attention at config 2 (sparse/attention.py:83-274 with residual_summaries=True):
    the flat selector's routes at ``--density``, their maximal residual frontiers, and per step the
    K/V summary table (built inside the reference's attention call) plus the attention over selected
    blocks and summary keys.  Summary prototypes P = 1 and 4; plain block-sparse attention beside."""
    import torch

    from spruce_research_b200 import native
    from spruce_research_b200.interfaces.residual_summaries import (build_residual_summary_nodes,
                                                                    build_residual_tree_layout)
    from spruce_research_b200.pipeline import SparsePrefillLayer
    from spruce_research_b200.sparse.summaries import build_kv_summary_table
    from spruce_research_b200.synthetic import make_gate_weights, make_layer_inputs

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    shape, K, entries, flops = workload(args)
    qb, D, rep = shape.query_blocks, shape.head_dim, shape.q_heads // shape.kv_heads
    q, k, v = make_layer_inputs(shape, torch.bfloat16, args.seed, device=dev)
    wq, wk = make_gate_weights(1, D, D, args.seed + 1, device=dev)
    sel = SparsePrefillLayer(wq[0], wk[0], K, local_window=0, sink_blocks=1).select(q, k)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    nodes = build_residual_summary_nodes(sel[:, None], validate_selected=False)[:, 0]
    e1.record()
    torch.cuda.synchronize()
    frontier_ms = e0.elapsed_time(e1)
    layout = build_residual_tree_layout(qb)
    out = torch.empty((1, shape.tokens, shape.q_heads, D), device=dev, dtype=torch.bfloat16)

    def timed(fn):
        for _ in range(max(1, args.warmup)):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / args.steps

    plain_ms = timed(lambda: native.sparse_attention(q, k, v, sel, out=out))
    rows = []
    for P in (1, 4):
        ws = {}

        def step():
            table = build_kv_summary_table(k, v, layout, block_size=64, prototypes=P)
            native.residual_sparse_attention(q, k, v, sel, nodes, table, out=out, workspace=ws.get("w"))

        table = build_kv_summary_table(k, v, layout, block_size=64, prototypes=P)
        need = native._lib.load().spruce_residual_workspace_bytes(1, shape.kv_heads, shape.tokens, D,
                                                                   nodes.shape[-1], P, 1)
        ws["w"] = torch.empty(need, device=dev, dtype=torch.uint8)
        step_ms = timed(step)
        table_ms = timed(lambda: build_kv_summary_table(k, v, layout, block_size=64, prototypes=P))
        attn_ms = timed(lambda: native.residual_sparse_attention(q, k, v, sel, nodes, table, out=out,
                                                                 workspace=ws["w"]))
        valid = table.counts[0][nodes.clamp(min=0).long()] > 0          # [G, qb, S, P]
        summary_keys = int((valid & (nodes >= 0)[..., None]).sum())
        sflops = 4.0 * D * rep * 64 * summary_keys  # every query token of the row's block scores every summary key
        rows.append({"prototypes": P, "step_ms": step_ms, "table_ms": table_ms, "attention_ms": attn_ms,
                     "summary_keys": summary_keys, "summary_tflop": sflops / 1e12,
                     "effective_tflops": (flops + sflops) / (attn_ms * 1e-3) / 1e12,
                     "workspace_gb": need / 1e9})
        del ws
    emit({
        "metric": "residual-summary sparse prefill ms/layer at config 2 (summary table + attention)",
        "value": rows[0]["step_ms"], "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": rows[0]["step_ms"], "higher_is_better": False, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) Q/K/V, RoPE base 1e6, planted affinity",
        "config": {**config_dict(args, shape, K, entries, 1), "residual_width": int(nodes.shape[-1]),
                   "frontier_ms": frontier_ms},
        "plain_attention_ms": plain_ms, "residual": rows,
    })


def main():
    args = parse_args()
    _claim_stdout()
    if args.impl == "reference":
        run_reference(args)
    elif args.sweep:
        run_sweep(args)
    elif args.model:
        run_model(args)
    elif args.tree_selector:
        run_tree_selector(args)
    elif args.residual:
        run_residual(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
