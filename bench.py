#!/usr/bin/env python3
"""Benchmark: GCN inference (2 layers, 128 -> 128 -> 128, ReLU between layers)
on a seeded R-MAT graph shaped like ogbn-products (2,449,029 nodes,
61,859,140 directed entries + self-loops, symmetric normalisation), fp32.

One step = one full forward over the whole graph: per layer the GCN
aggregation (libgnnb200 SpMM), then X·W with bias and ReLU fused into the
GEMM epilogue; with N GPUs the rows are split into N equal-nnz ranges (one
process per GPU; rows are dealt to ranks so that each gets the same number of
rows and about the same cost) and the layer-1 output rows are exchanged between
the GPUs over NVLink.

Metric: algorithmic SpMM bytes of the step (CSR + gathered neighbour rows +
output, per layer) divided by the step time, in GB/s, whole job. The JSON line
adds ms/layer, the SpMM kernel's roofline fraction against the measured HBM
copy bandwidth, an end-to-end figure through the public API with host buffers
(H2D of the inputs and D2H of the output inside the timed region), and the
CPU oracle timed on a bounded sample on this host.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...   (N > 1)
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from gnn_cuda_b200 import _native as N  # noqa: E402
from gnn_cuda_b200 import partition, synth  # noqa: E402
from gnn_cuda_b200.GNN_cuda_common import agg_ops, gcn_ops, native_ops  # noqa: E402

METRIC = "SpMM GB/s & GNN fwd ms/layer at 1/2/4/8 B200; % of HBM roofline"
WORKLOAD = "gcn_products_like"
FEAT = 128
LAYERS = 2
HBM_FALLBACK_GBS = 6650.0


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="target CPU-baseline sample time (0: skip)")
    ap.add_argument("--scale", type=float, default=1.0, help="scale the graph down (smoke runs only)")
    ap.add_argument("--gin-path", choices=["chunks", "fused"], default="fused",
                    help="gin_papers_like at full size: one fused kernel per layer, or the separate calls over row "
                         "ranges (same bits; measured on one B200: 288 vs 370 ms per layer)")
    ap.add_argument("--no-check", dest="check", action="store_false",
                    help="skip the check of sampled output rows against the oracle after the timed region")
    ap.add_argument("--no-other-configs", dest="other_configs", action="store_false",
                    help="skip the Pubmed- and Reddit-shaped configurations measured after the headline")
    ap.add_argument("--no-reference-gpu", dest="reference_gpu", action="store_false",
                    help="skip timing the reference's own CUDA kernels on the same tensors")
    ap.add_argument("--chunks", type=int, default=0,
                    help="row pieces per rank, exchanged as they finish (N > 1; 0: 1)")
    ap.add_argument("--exchange", choices=["push", "halo", "allgather"], default="halo",
                    help="N > 1: pushes of whole row pieces into the peers' IPC-mapped buffers, pushes of only "
                         "the rows each peer reads (halo), or NCCL all_gather")
    ap.add_argument("--transport", choices=["sm", "ce"], default="sm",
                    help="push transport: one SM kernel storing to every peer, or copy engines")
    ap.add_argument("--push-ctas", type=int, default=0, help="grid of the halo push kernel (0: the library default, 1 per SM)")
    ap.add_argument("--layout", choices=["balanced", "contiguous"], default="balanced",
                    help="N > 1: rows dealt to ranks by cost, or contiguous cost-balanced ranges")
    ap.add_argument("--push-from", choices=["kernel", "transform"], default="transform",
                    help="N > 1 halo exchange: the transform's epilogue storing the halo rows to the peers itself "
                         "(gnn_linear_push_forward; per-step median 1.770 vs 1.81 ms at N = 8, 4.19 vs 4.33 ms at "
                         "N = 2), or a push kernel after the transform")
    ap.add_argument("--no-graphs", dest="graphs", action="store_false",
                    help="N > 1: issue every step from Python instead of replaying it as a captured CUDA graph")
    ap.add_argument("--long-rows", choices=["shard", "graph"], default="shard",
                    help="N > 1: long-row threshold of a 1/N share of the graph (every shard call), or the whole "
                         "graph's (the one-GPU forward's bits; slower shards)")
    ap.add_argument("--padded-order", choices=["rank", "chunk"], default="rank",
                    help="N > 1 with pushes: every rank's rows one block of the exchange matrix (the last layer "
                         "then runs as one call), or piece-major blocks (the all_gather exchange always uses these)")
    ap.add_argument("--workload", choices=["gcn_products_like", "gcn_pubmed_like", "sage_reddit_like",
                                           "gin_papers_like", "locality_products_like"],
                    default="gcn_products_like",
                    help="the GCN forward (default); the GraphSAGE-mean forward on the Reddit-shaped graph (1 GPU); "
                         "or the UVM locality preprocessing of the products-shaped graph (1 GPU)")
    return ap.parse_args()


def measured_hbm_gbs() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        v = float(json.loads(p.read_text())["hbm_gbs"])
        return v, "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


def spmm_layer_bytes(n: int, nnz: int, f: int, rp_bytes: int = 4) -> int:
    """Algorithmic bytes of one GCN aggregation: row_ptr + col_ind + deg_inv_sqrt
    + one gathered feature row per CSR entry + the output matrix."""
    return (n + 1) * rp_bytes + nnz * 4 + n * 4 + nnz * f * 4 + n * f * 4


# DRAM bytes of one full-size aggregation launch of the default workload, from an
# ncu capture of the kernels this build launches (dram__bytes_read.sum +
# dram__bytes_write.sum of every aggregation kernel of one layer, a one-pass
# launch list of `bench.py --steps 3 --warmup 3 --cpu-seconds 0 --e2e-steps 1
# --no-check --no-reference-gpu`), with the L2 sector hit rate of the per-row
# kernel from a --set full capture of the quarter-scale graph. Re-measured
# whenever the aggregation kernels change; the capture summary is kept with the
# other profiles.
DRAM_PROFILE = {
    "gcn_products_like": {"traffic": 12.541e9, "l2_hit_rate": 0.672,
                          "kernels": "spmm_vec_kernel 8.635 + 1.443 GB, spmm_long_kernel 2.443 + 0.020 GB "
                                     "(read + write per launch)",
                          "profile": "profiles/spmm_gcn_products_like.md"},
}


def profiled_traffic(workload: str) -> dict | None:
    """The measured DRAM traffic of one aggregation of `workload`, if captured."""
    return DRAM_PROFILE.get(workload)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, enabled: bool = True):
        self.gpu = gpu_index
        self.enabled = enabled
        self.proc = None
        self.file = None

    def __enter__(self):
        if not self.enabled:
            return self
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", str(self.gpu)], stdout=self.file,
                                         stderr=subprocess.DEVNULL)
            # the timed region starts only once sampling has (nvidia-smi takes a moment to start)
            t0 = time.time()
            while time.time() - t0 < 5.0 and os.path.getsize(self.file.name) == 0 and self.proc.poll() is None:
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        try:
            for line in Path(self.file.name).read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].isdigit():
                    rows.append(parts)
            os.unlink(self.file.name)
        except Exception:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [int(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        power = []
        for r in rows:
            try:
                power.append(float(r[3]))
            except ValueError:
                pass
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": int(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(power) if power else None}


# ---------------------------------------------------------------------------
# problem construction (setup; not timed)
# ---------------------------------------------------------------------------

def build_problem(seed: int, device: torch.device, scale: float):
    t0 = time.time()
    src, dst, n = synth.make_graph(WORKLOAD, seed=seed, device=device, scale_nodes=scale)
    rp, ci, dis = synth.csr_on_device(src, dst, n, add_self_loops=True)
    del src, dst
    x = synth.features(n, FEAT, seed=seed + 1, device=device)
    ws = [synth.glorot(FEAT, FEAT, seed=seed + 10 + li, device=device) for li in range(LAYERS)]
    bs = [torch.zeros(FEAT, device=device) for _ in range(LAYERS)]
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    log(f"[bench] graph n={n} nnz={ci.numel()} built on {device.type} in {time.time() - t0:.1f}s")
    return dict(n=n, nnz=int(ci.numel()), rp=rp, ci=ci, dis=dis, x=x, ws=ws, bs=bs)


def row_order() -> str:
    """The per-row aggregation kernel's row order (spmm.schedule knob)."""
    mode = N.config_get("spmm.schedule")
    return {0: "row id", 1: f"degree-descending within windows of {N.config_get('spmm.schedule_window')} rows",
            2: "degree-descending (global)",
            3: "degree-descending: global below 64 entries per row on average, else within windows of "
               f"{N.config_get('spmm.schedule_window')} rows"}[mode]


def default_chunks(chunks: int, world: int) -> int:
    """Row pieces per rank: as given, else 1. Measured on 8 B200s with the step replayed as
    a CUDA graph: 1.82 ms per step with one piece, 1.95 ms with two (two pieces hide most of
    the halo exchange but each is an aggregation call of its own, and the push slows the
    second piece's aggregation beside it)."""
    del world
    return chunks if chunks > 0 else 1


def describe(prob, world: int, gemm: str | None = None, chunks: int = 1, exchange: str = "halo",
             transport: str = "sm", layout: str = "balanced", order: str | None = None,
             padded_order: str = "rank", push_from: str = "transform") -> dict:
    if gemm is None:
        gemm = "tcgen05-tf32" if N.lib().gnn_gemm_uses_tensor_cores(prob["n"], FEAT, FEAT) else "ffma-fp32"
    if order is None:
        order = row_order()
    return {"workload": f"{WORKLOAD}: GCN {LAYERS} layers {FEAT}->{FEAT}->{FEAT}, ReLU between layers",
            "nodes": prob["n"], "csr_entries": int(prob["nnz"]), "feat_dim": FEAT, "layers": LAYERS,
            "self_loops": True, "graph": "R-MAT(0.57,0.19,0.19,0.05), symmetrised, de-duplicated",
            "parallelism": f"rows{world}" + ("" if world == 1 else
                                             f"+{layout}_{transport}_push_pieces{chunks}_{padded_order}_major"
                                             if exchange == "push" else
                                             f"+{layout}_halo_push_pieces{chunks}_{padded_order}_major"
                                             + ("_from_transform" if push_from == "transform" else "")
                                             if exchange == "halo" else
                                             f"+{layout}_nccl_allgather_pieces{chunks}"),
            "l2": "inputs larger than L2 (X is %.2f GB), no flush" % (prob["n"] * FEAT * 4 / 1e9),
            "gemm": gemm, "row_order": order}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_ours(args, rank: int, world: int, device: torch.device):
    prob = build_problem(args.seed, device, args.scale)
    n = prob["n"]
    nnz = int(prob["ci"].numel())
    rp_cpu = prob["rp"].to(torch.int64).cpu().numpy()
    exchange = None
    halo = None
    push_masks = None
    args.chunks = default_chunks(args.chunks, world)
    if world == 1:
        shard = partition.make_shard(prob["rp"], prob["ci"], 0, n)
        bufs = {"agg": torch.empty(n, FEAT, device=device), "out0": torch.empty(n, FEAT, device=device),
                "out1": torch.empty(n, FEAT, device=device)}
    else:
        # rows dealt to ranks by cost (or contiguous ranges), renumbered into the padded
        # exchange layout (rank-major for the pushes); sums are unchanged, only column ids
        # are rewritten
        rank_major = args.exchange in ("push", "halo") and args.padded_order == "rank"
        layout = partition.make_padded_layout(rp_cpu, world, args.chunks, balanced=args.layout == "balanced",
                                              row_cost=partition.ROW_COST_IN_ENTRIES, rank_major=rank_major)
        shard = partition.make_padded_shard(prob["rp"], prob["ci"], layout, rank)
        if args.exchange == "halo":
            halo = partition.make_halo_plan(prob["rp"], prob["ci"], layout, rank)
            if args.push_from == "transform":
                push_masks = halo.piece_masks(shard)
        # one long-row threshold for every call on every rank: the automatic value of a
        # 1/N share of the graph (or the whole graph's); a row's sum depends only on it,
        # so the output equals the one-GPU forward run at the same threshold, bit for bit
        share = (-(-n // world), -(-nnz // world)) if args.long_rows == "shard" else (n, nnz)
        N.config_set("spmm.long_row_threshold", int(N.lib().gnn_spmm_long_row_threshold(*share)))
        if args.check:
            whole_graph = {k: prob[k] for k in ("rp", "ci", "dis", "x")}
        prob["dis"] = layout.pad_rows(prob["dis"])
        prob["x"] = layout.pad_rows(prob["x"])
        del prob["rp"], prob["ci"]
        torch.cuda.empty_cache()
        if args.exchange in ("push", "halo"):
            exchange = partition.PeerRowExchange(layout.padded_rows, FEAT, rank, world, device,
                                                 transport="sm" if args.exchange == "halo" else args.transport,
                                                 ctas=args.push_ctas)
            # with rank-major rows the last layer aggregates all of them in one call
            bufs = {"agg": torch.empty(layout.local_rows if rank_major else layout.chunk_rows, FEAT, device=device),
                    "out": torch.empty(layout.local_rows, FEAT, device=device)}
        else:
            bufs = partition.allgather_buffers(layout, FEAT, device)
    rows = shard.num_rows
    torch.backends.cuda.matmul.allow_tf32 = True  # the reference driver's --tf32 default

    def step(timers=None, final_out=None, inputs=None):
        if world == 1:
            # the reference-facing op surface, exactly what gcn_inference calls
            p = prob if inputs is None else inputs
            x = p["x"]
            for li in range(LAYERS):
                ev = partition._mark(timers, "spmm_begin")
                gcn_ops.spmm_gcn_forward_(p["rp"], p["ci"], p["dis"], x, bufs["agg"])
                partition._mark(timers, "spmm_end", ev)
                out = bufs["out0" if li % 2 == 0 else "out1"]
                if final_out is not None and li == LAYERS - 1:
                    out = final_out
                agg_ops.linear_forward_(bufs["agg"], p["ws"][li], p["bs"][li], out, li != LAYERS - 1)
                x = out
            return x
        if args.exchange in ("push", "halo"):
            return partition.gcn_forward_push(shard, prob["dis"], prob["x"], prob["ws"], prob["bs"], layout, exchange,
                                              bufs["agg"], bufs["out"] if final_out is None else final_out,
                                              timers=timers, halo=halo, push_masks=push_masks)
        return partition.gcn_forward_allgather(shard, prob["dis"], prob["x"], prob["ws"], prob["bs"], layout, bufs,
                                               timers=timers)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)

    # N > 1: the step captured as CUDA graphs (one launch per step), when every rank captured it
    graphs, graph_note = None, None
    launches_per_step = None
    if world > 1 and exchange is not None and args.graphs:
        l0 = N.lib().gnn_kernel_launches()
        try:
            graphs = partition.PushForwardGraphs(step, exchange)
        except Exception as e:  # noqa: BLE001 - reported, and every rank then runs eagerly
            graphs, graph_note = None, f"capture failed: {type(e).__name__}: {str(e)[:200]}"
        launches_per_step = (N.lib().gnn_kernel_launches() - l0) / 2
        ok = torch.tensor([1 if graphs is not None else 0], device=device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if int(ok.item()) == 0 and graphs is not None:
            graphs.close()
            graphs, graph_note = None, "another rank's capture failed"
        for _ in range(2 * max(1, args.warmup // 2) if graphs is not None else 0):
            graphs.replay()
        torch.cuda.synchronize(device)

    timers: dict = {}
    launches0 = N.lib().gnn_kernel_launches()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    step_ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    # only rank 0's samples reach the JSON line; the other ranks run no sampler
    with ClockSampler(device.index, enabled=rank == 0) as clocks:
        t_start.record()
        h0 = time.perf_counter()
        for i in range(args.steps):
            step_ev[i].record()
            if graphs is not None:
                graphs.replay()
            else:
                step(timers)
        step_ev[-1].record()
        host_ms = (time.perf_counter() - h0) * 1e3  # the host's time to issue the steps
        t_end.record()
        torch.cuda.synchronize(device)
    step_ms = [a.elapsed_time(b) for a, b in zip(step_ev[:-1], step_ev[1:])]
    if world > 1:
        dist.barrier()
    launches = N.lib().gnn_kernel_launches() - launches0
    if graphs is not None:
        # replays launch without the host counting them: the kernels each captured step holds
        launches = int(round(launches_per_step * args.steps))
    ms_total = t_start.elapsed_time(t_end)
    eager_ms = None
    if graphs is not None:
        # the per-phase figures (aggregation per rank, exchange wait) from eager steps,
        # which carry the timing events that graph replays do not record
        phase_steps = min(args.steps, 10)
        torch.cuda.synchronize(device)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(phase_steps):
            step(timers)
        e1.record()
        torch.cuda.synchronize(device)
        eager_ms = e0.elapsed_time(e1) / phase_steps
    timed_steps = min(args.steps, 10) if graphs is not None else args.steps  # the steps the timers saw
    trace = None
    if world > 1 and args.exchange in ("push", "halo"):
        # one more step with a timeline of its phases on every rank (not part of the timed steps)
        ev_list: list = []
        partition.gcn_forward_push(shard, prob["dis"], prob["x"], prob["ws"], prob["bs"], layout, exchange,
                                   bufs["agg"], bufs["out"], halo=halo, trace=ev_list, push_masks=push_masks)
        torch.cuda.synchronize(device)
        trace = partition.trace_offsets(ev_list)
        everyone: list = [None] * world
        dist.all_gather_object(everyone, trace)
        trace = everyone
    parity = None
    if world == 1 and args.check:
        # the last timed step left h1 in out0, the layer-2 aggregate in agg, the output in out1
        parity = check_forward_sample(prob, bufs["out0"], bufs["agg"], bufs["out1"], device)
    elif args.check:
        rows_out = graphs.replay() if graphs is not None else step()  # what the timed steps ran
        parity = check_partitioned_forward(whole_graph, prob["ws"], prob["bs"], layout, rank, rows_out, device)
        del whole_graph
        torch.cuda.empty_cache()
    # SpMM time per layer on this rank (summed over its row pieces when N > 1)
    spmm_ms = [b.elapsed_time(e) for b, e in timers.get("spmm", [])]
    agg_calls = len(spmm_ms) // max(1, timed_steps)
    host_calls = {k: round(v * 1e3 / max(1, timed_steps), 4) for k, v in timers.get("host", {}).items()}
    if world > 1:
        everyone_host: list = [None] * world
        dist.all_gather_object(everyone_host, host_calls)
        host_calls = everyone_host
    spmm_ms_avg = sum(spmm_ms) / max(1, timed_steps * LAYERS)
    # exposed exchange: how long the compute stream waits at each layer boundary
    xchg_ms = sum(b.elapsed_time(e) for b, e in timers.get("xchg", [])) / max(1, timed_steps)

    # ---- e2e through the public API with host buffers ----
    # every step copies this rank's inputs (its CSR rows, the normalisation vector,
    # the full feature matrix, the weights) from pinned host memory, runs the
    # forward and reads its output rows back into pinned host memory. The copies
    # overlap across steps, as a serving loop would run them: step i+1's inputs
    # go up on one copy stream while step i's output comes down on another (the
    # PCIe link carries both directions at once); the forward of step i+1 waits
    # for its inputs, and two output buffers alternate so that it never
    # overwrites rows still being read back. On one GPU two input sets alternate
    # as well, so the upload of step i+1 also overlaps the forward of step i.
    x_rows = None
    if world == 1:
        dev_in = [prob["rp"], prob["ci"], prob["dis"], prob["x"]]
    else:
        # a rank's first layer reads only the feature rows its column ids name (its own
        # rows and the rows of its halo): those go up every step, into a staging matrix
        # that is scattered into the padded feature matrix on the device
        cols = shard.whole.col_ind if shard.whole is not None else torch.cat([p.col_ind for p in shard.pieces])
        x_rows = torch.unique(cols.to(torch.int64))
        x_stage = prob["x"][x_rows]
        dev_in = shard.device_tensors() + [prob["dis"], x_stage]
    dev_in += prob["ws"] + prob["bs"]
    host_in = [t.cpu().pin_memory() for t in dev_in]
    in_sets = [dev_in]
    if world == 1:
        in_sets.append([torch.empty_like(t) for t in dev_in])

    def as_inputs(ts):
        return {"rp": ts[0], "ci": ts[1], "dis": ts[2], "x": ts[3], "ws": ts[4:4 + LAYERS],
                "bs": ts[4 + LAYERS:4 + 2 * LAYERS]}
    out_host = [torch.empty(rows, FEAT, pin_memory=True) for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = out_host[0].numel() * 4
    pipelined = world == 1 or args.exchange in ("push", "halo")
    if pipelined:
        first = bufs["out1"] if world == 1 else bufs["out"]
        out_dev = [first, torch.empty_like(first)]
    else:
        out_dev = [None, None]
    comp = torch.cuda.current_stream(device)
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_out: list = [None, None]
    ev_used: list = [None, None]  # the forward that last read input set j is done
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record(comp)
    for i in range(args.e2e_steps):
        k = i % 2 if pipelined else 0
        j = i % len(in_sets)
        if len(in_sets) == 1:
            s_in.wait_stream(comp)  # the previous forward no longer reads the inputs
        elif ev_used[j] is not None:
            s_in.wait_event(ev_used[j])  # the forward two steps back is done with this input set
        with torch.cuda.stream(s_in):
            for dst_t, src_t in zip(in_sets[j], host_in):
                dst_t.copy_(src_t, non_blocking=True)
            if x_rows is not None:
                prob["x"].index_copy_(0, x_rows, x_stage)
        comp.wait_stream(s_in)
        if ev_out[k] is not None:
            comp.wait_event(ev_out[k])  # the read-back that used this output buffer is done
        out = step(final_out=out_dev[k], inputs=as_inputs(in_sets[j]) if world == 1 else None)
        ev_used[j] = torch.cuda.Event()
        ev_used[j].record(comp)
        s_out.wait_stream(comp)
        with torch.cuda.stream(s_out):
            out_host[k].copy_(out, non_blocking=True)
            ev_out[k] = torch.cuda.Event()
            ev_out[k].record(s_out)
    comp.wait_stream(s_out)
    e_end.record(comp)
    torch.cuda.synchronize(device)
    e2e_ms = e_start.elapsed_time(e_end)
    # the same copies alone (no forward): the host link's share of the end-to-end step
    copy_ms = None
    if world == 1:
        torch.cuda.synchronize(device)
        c0 = torch.cuda.Event(enable_timing=True)
        c1 = torch.cuda.Event(enable_timing=True)
        c0.record(comp)
        for i in range(args.e2e_steps):
            s_in.wait_stream(comp)
            with torch.cuda.stream(s_in):
                for dst_t, src_t in zip(in_sets[i % len(in_sets)], host_in):
                    dst_t.copy_(src_t, non_blocking=True)
            with torch.cuda.stream(s_out):
                out_host[i % 2].copy_(out_dev[i % 2], non_blocking=True)
            comp.wait_stream(s_in)
            comp.wait_stream(s_out)
        c1.record(comp)
        torch.cuda.synchronize(device)
        copy_ms = c0.elapsed_time(c1) / args.e2e_steps

    # ---- reduce over ranks ----
    # per-layer algorithmic bytes of this rank's aggregation (its rows, its CSR entries)
    shard_bytes = spmm_layer_bytes(rows, shard.num_edges, FEAT)
    vals = torch.tensor([ms_total, e2e_ms, spmm_ms_avg, float(launches), float(shard_bytes), xchg_ms,
                         host_ms / args.steps, statistics.median(step_ms), max(step_ms), min(step_ms),
                         eager_ms if eager_ms is not None else 0.0, float(step_ms.index(max(step_ms)))],
                        dtype=torch.float64, device=device)
    per_rank = [vals.clone() for _ in range(world)]
    if world > 1:
        dist.all_gather(per_rank, vals)
    table = torch.stack(per_rank).cpu()
    ms_total, e2e_ms = float(table[:, 0].max()), float(table[:, 1].max())
    launches = int(table[:, 3].sum())
    slow = int(table[:, 2].argmax())  # the rank whose aggregation took longest
    spmm_ms_avg, shard_bytes = float(table[slow, 2]), int(table[slow, 4])
    bytes_layer = spmm_layer_bytes(n, nnz, FEAT)
    bytes_step = bytes_layer * LAYERS
    ms_step = ms_total / args.steps
    value = bytes_step / (ms_step * 1e-3) / 1e9
    e2e_value = bytes_step / ((e2e_ms / args.e2e_steps) * 1e-3) / 1e9
    if graphs is not None:
        graphs.close()  # graphs holding the barrier collective go before the exchange and the process group
    if exchange is not None:
        exchange.close()

    if rank != 0:
        return None
    peak, peak_kind = measured_hbm_gbs()
    achieved = shard_bytes / (spmm_ms_avg * 1e-3) / 1e9 if spmm_ms_avg > 0 else None
    prof = profiled_traffic(WORKLOAD) if world == 1 and args.scale == 1.0 else None
    traffic = prof["traffic"] if prof else None
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "ms_per_layer": round(ms_step / LAYERS, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": f"synthetic: seeded R-MAT graph (seed {args.seed}) with ogbn-products shape, N(0,1) features, "
                "Glorot weights, zero bias",
        "config": describe(prob, world, chunks=args.chunks, exchange=args.exchange, transport=args.transport,
                           layout=args.layout, padded_order=args.padded_order, push_from=args.push_from),
        "roofline": {"bound": "hbm", "kernel": "spmm_vec_kernel + spmm_long_kernel (GCN aggregation)",
                     "achieved": round(achieved, 1) if achieved else None, "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4) if achieved else None, "peak_source": peak_kind,
                     "spmm_ms_per_layer": round(spmm_ms_avg, 4), "algorithmic_bytes_per_layer": shard_bytes,
                     "aggregation_calls_per_step": agg_calls,
                     "traffic": traffic, "rank": slow,
                     "frac_dram": round(traffic / (spmm_ms_avg * 1e-3) / 1e9 / peak, 4) if traffic and spmm_ms_avg else None,
                     "l2_hit_rate": prof["l2_hit_rate"] if prof else None,
                     "traffic_source": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum, full-size launch list: "
                                        f"{prof['kernels']} ({prof['profile']})") if prof else None,
                     "frac_note": "frac = algorithmic bytes / aggregation time / peak (gathered rows served from L2 "
                                  "count too, so it can exceed 1); frac_dram = measured DRAM bytes / the same time / "
                                  "peak",
                     "spmm_ms_per_rank": [round(float(v), 4) for v in table[:, 2]],
                     "exchange_wait_ms_per_step_per_rank": [round(float(v), 4) for v in table[:, 5]],
                     "step_timeline_ms_per_rank": trace},
        "steps_per_rank": {"host_issue_ms_per_step": [round(float(v), 4) for v in table[:, 6]],
                           "gpu_ms_median": [round(float(v), 4) for v in table[:, 7]],
                           "gpu_ms_max": [round(float(v), 4) for v in table[:, 8]],
                           "gpu_ms_min": [round(float(v), 4) for v in table[:, 9]],
                           "gpu_ms_max_step_index": [int(v) for v in table[:, 11]],
                           "host_issue_ms_by_call": host_calls or None,
                           "note": "per timed step on each rank: the host's time to issue it, and the device time "
                                   "between events at step boundaries on the compute stream"},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "ms_per_step": round(e2e_ms / args.e2e_steps, 3),
                "copies": ("overlapped across steps (two input sets and two output buffers; inputs up / output "
                           "down on two copy streams beside the forward)" if world == 1 else
                           "overlapped across steps (inputs up / output down on two copy streams); each rank "
                           "uploads its CSR rows, the normalisation vector, the weights and the feature rows its "
                           "column ids name (scattered into the padded matrix on the device), and reads back its "
                           "output rows") if pipelined
                else "in step order",
                "api": "gnn_cuda_b200.GNN_cuda_common.gcn_ops/agg_ops over libgnnb200.so",
                "copies_only_ms_per_step": round(copy_ms, 3) if copy_ms is not None else None},
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
    }
    if world > 1 and exchange is not None:
        result["cuda_graphs"] = {
            "used": graphs is not None, "note": graph_note,
            "kernels_per_step": launches_per_step,
            "eager_ms_per_step": round(float(table[:, 10].max()), 4) if graphs is not None else None,
            "how": "each step is one replay of a captured graph (two graphs, one per exchange copy, replayed in "
                   "turn); gpu_launches = the kernels a captured step holds x steps; the per-phase figures come "
                   "from min(steps, 10) eager steps after the timed ones, whose time is eager_ms_per_step"}
    if parity is not None:
        result["parity"] = parity
    if world == 1 and args.reference_gpu:
        result["reference_gpu"] = reference_gpu_baseline(prob, device, args.seed, args.scale)
    if world == 1 and args.cpu_seconds > 0:
        result["cpu_baseline"] = cpu_baseline(prob, args.cpu_seconds)
    if world == 1 and args.other_configs and args.scale == 1.0:
        del prob, bufs
        torch.cuda.empty_cache()
        result["other_configs"] = other_configs(args, device)
    return result


def other_configs(args, device) -> dict:
    """The Pubmed-shaped one-layer GCN and the Reddit-shaped GraphSAGE forward, measured
    in the same run (10 timed steps after 3 warm-up steps each), so that every
    configuration that fits one GPU quickly has a number from the default bench."""
    import copy
    sub = copy.copy(args)
    sub.steps, sub.warmup, sub.cpu_seconds, sub.e2e_steps = 10, 3, 0.0, 2
    keep = ("metric", "value", "unit", "ms_per_step", "ms_per_layer", "roofline", "parity", "config", "e2e",
            "gpu_launches")
    out = {}
    for name, fn in (("gcn_pubmed_like", run_pubmed), ("sage_reddit_like", run_sage)):
        try:
            r = fn(sub, device)
            out[name] = {k: r[k] for k in keep if k in r}
        except Exception as e:  # reported, never fatal for the headline line
            out[name] = {"error": str(e)[:300]}
        torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# output check of the timed forward (after the timed region; the oracle is the checker)
# ---------------------------------------------------------------------------

def auto_long_threshold(nnz: int, device) -> int:
    """The engine's automatic long-row threshold, clamp(nnz / (SMs * 32 * 8), 256, 8192)."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    return max(32, min(8192, max(256, nnz // (sms * 32 * 8))))


def check_forward_sample(prob, h1: torch.Tensor, agg2: torch.Tensor, out: torch.Tensor, device,
                         n_short: int = 4000, seed: int = 7) -> dict:
    """Sampled rows of the forward just timed, against the oracle.

    Every row above the long-row threshold plus `n_short` others. The layer-2
    aggregation (agg2 = aggregate(h1), the GPU's own layer-1 output) is compared
    bit for bit with the oracle's restatement of this engine's schedule and held
    to 1e-5 of float64; the layer-1 output h1 and the final output are held to
    the TF32 tolerance (2e-3 of sum |a w|) against float64 transforms of the
    oracle's aggregates of the same rows."""
    from oracle import oracle as O
    rp, ci, dis, x = prob["rp"], prob["ci"], prob["dis"], prob["x"]
    thr = auto_long_threshold(int(ci.numel()), device)
    deg = (rp[1:] - rp[:-1]).to(torch.int64)
    long_rows = torch.nonzero(deg > thr).flatten()
    short = torch.nonzero(deg <= thr).flatten()
    g = torch.Generator(device=device).manual_seed(seed)
    short = short[torch.randperm(short.numel(), generator=g, device=device)[:n_short]]
    rows = torch.cat([long_rows, short]).cpu().numpy()
    k = rows.size
    idx = torch.as_tensor(rows, device=device)
    w = [t.cpu().numpy().astype(np.float64) for t in prob["ws"]]
    b = [t.cpu().numpy().astype(np.float64) for t in prob["bs"]]

    def tf32_err(got, a32, li, relu):
        a = a32.astype(np.float64)
        exp = a @ w[li] + b[li]
        if relu:
            exp = np.maximum(exp, 0.0)
        scale = np.abs(a) @ np.abs(w[li]) + np.abs(b[li]) + 1e-30
        return float(np.max(np.abs(got.astype(np.float64) - exp) / scale))

    # layer 1: the oracle's aggregate of x on these rows, then the transform
    srp, sci, sx, sdis = O.compact_rows_problem(rp, ci, x, rows, dis)
    agg1 = O.spmm(srp, sci, sx, mode=O.W_GCN, dis=sdis, split_warps=16, long_thr=thr, rows=(0, k))
    err_h1 = tf32_err(h1[idx].cpu().numpy(), agg1, 0, True)
    # layer 2: aggregate of the GPU's h1, bit for bit
    srp, sci, sh, sdis = O.compact_rows_problem(rp, ci, h1, rows, dis)
    exp2 = O.spmm(srp, sci, sh, mode=O.W_GCN, dis=sdis, split_warps=16, long_thr=thr, rows=(0, k))
    got2 = agg2[idx].cpu().numpy()
    same = np.all(got2.view(np.uint32) == exp2.view(np.uint32), axis=1)
    f64, ab = O.spmm_f64_rows(srp, sci, sh, np.arange(k), mode=O.W_GCN, dis=sdis)
    err_agg = O.check_close_to_f64(got2, f64, ab, rel=1e-5)
    err_out = tf32_err(out[idx].cpu().numpy(), got2, 1, False)
    nl = int(long_rows.numel())
    return {"rows_checked": int(k), "long_rows_checked": nl, "long_row_threshold": thr,
            "agg_bit_exact_rows": int(same.sum()), "bit_exact_short_rows": bool(same[nl:].all()),
            "bit_exact_long_rows": bool(same[:nl].all()),
            "agg_err_vs_f64": round(err_agg, 4), "agg_tolerance": "|ours - f64| <= 1e-5 (sum|w x| + |f64|); "
            "the figure is the worst ratio to that bound (<= 1 passes)",
            "max_rel_err": round(max(err_h1, err_out), 6), "tf32_tolerance": 2e-3,
            "ok": bool(same.all() and err_agg <= 1.0 and max(err_h1, err_out) <= 2e-3),
            "checked": "layer-1 output (TF32) and layer-2 aggregation (bits) and output (TF32) of the last timed "
                       "step, sampled rows (every long row + random others), against the C oracle"}


def check_partitioned_forward(graph: dict, ws, bs, layout, rank: int, rows_out: torch.Tensor, device) -> dict:
    """This rank's output rows of the partitioned forward against the same rows
    of the one-GPU forward (the reference-facing calls over the whole graph, on
    this rank's GPU, at the long-row threshold the shards use), bit for bit; the
    count of differing rows is summed over ranks. The one-GPU forward is itself
    checked against the oracle by the N = 1 line."""
    agg = torch.empty(graph["x"].shape, device=device)
    h = graph["x"]
    for li in range(LAYERS):
        gcn_ops.spmm_gcn_forward_(graph["rp"], graph["ci"], graph["dis"], h, agg)
        o = torch.empty(h.shape[0], FEAT, device=device)
        agg_ops.linear_forward_(agg, ws[li], bs[li], o, li != LAYERS - 1)
        h = o
    mine = h[layout.order[rank].to(device)]
    differ = (mine.view(torch.int32) != rows_out.view(torch.int32)).any(dim=1).sum().to(torch.int64)
    counts = torch.stack([differ, torch.tensor(rows_out.shape[0], dtype=torch.int64, device=device)])
    dist.all_reduce(counts)
    differ, total = (int(v) for v in counts.cpu())
    return {"rows_checked": total, "rows_differing": differ, "ok": differ == 0,
            "long_row_threshold": int(N.config_get("spmm.long_row_threshold")),
            "checked": "every output row of the partitioned forward (one extra step after the timed region, "
                       "a graph replay when the timed steps were replays) "
                       "against the one-GPU forward of the whole graph at the same long-row threshold, bit for bit"}


# ---------------------------------------------------------------------------
# the reference's own GPU kernels, timed on the same box and tensors
# ---------------------------------------------------------------------------

REF_SO = ROOT / "oracle" / "_ref"


def _load_ref(name: str):
    import importlib.machinery
    import importlib.util
    path = REF_SO / f"{name}.so"
    if not path.exists():
        return None
    loader = importlib.machinery.ExtensionFileLoader(name, str(path))
    spec = importlib.util.spec_from_loader(name, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def _median_ms(fn, device, reps: int = 10, warm: int = 3) -> float:
    for _ in range(warm):
        fn()
    torch.cuda.synchronize(device)
    times = []
    for _ in range(reps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    return float(statistics.median(times))


def reference_gpu_baseline(prob, device, seed: int, scale: float = 1.0) -> dict:
    """The reference's own CUDA kernels (compiled from its sources, unmodified) and
    this library's kernel for the same call, each timed alone with CUDA events on
    the same device tensors: median of 10 calls after 3 warm-up calls."""
    ref = {n: _load_ref(n) for n in ("ref_gcn_ops", "ref_pyg_gcn_ops", "ref_agg_ops")}
    if any(m is None for m in ref.values()):
        return {"unavailable": "the reference kernels are not built into oracle/_ref (python oracle/build_ref.py)"}
    from gnn_cuda_b200.GNN_cuda_common import pyg_gcn_ops
    rp, ci, dis, x = prob["rp"], prob["ci"], prob["dis"], prob["x"]
    n = prob["n"]
    out = torch.empty(n, FEAT, device=device)
    res: dict = {}

    def pair(name, theirs, ours, what):
        t_ref = _median_ms(theirs, device)
        t_ours = _median_ms(ours, device)
        res[name] = {"call": what, "reference_ms": round(t_ref, 4), "ours_ms": round(t_ours, 4),
                     "speedup": round(t_ref / t_ours, 3)}

    pair("gcn_aggregation", lambda: ref["ref_gcn_ops"].spmm_gcn_hmm_forward_(rp, ci, dis, x, out),
         lambda: gcn_ops.spmm_gcn_forward_(rp, ci, dis, x, out),
         "spmm_gcn_hmm_forward_ (gcn_spmm_hmm_kernel, gcn_ops.cu:34-109), products-shaped graph, F = 128")
    rows_of = torch.repeat_interleave(torch.arange(n, device=device), (rp[1:] - rp[:-1]).to(torch.int64))
    ew = dis[rows_of] * dis[ci.to(torch.int64)]
    del rows_of
    pair("pyg_gcn_aggregation", lambda: ref["ref_pyg_gcn_ops"].spmm_pyg_gcn_plain_forward_(rp, ci, ew, x, out),
         lambda: pyg_gcn_ops.spmm_pyg_gcn_forward_(rp, ci, ew, x, out, spmm_mode="plain"),
         "spmm_pyg_gcn_plain_forward_ (pyg_gcn_ops.cu:33-108), products-shaped graph, F = 128")
    del ew
    pair("sum_aggregation", lambda: ref["ref_agg_ops"].spmm_sum_forward_(rp, ci, x, out),
         lambda: agg_ops.spmm_sum_forward_(rp, ci, x, out),
         "spmm_sum_forward_ (csr_agg_kernel<false>, agg_ops.cu:23-47), products-shaped graph, F = 128")
    agg = torch.empty(n, FEAT, device=device)
    gcn_ops.spmm_gcn_forward_(rp, ci, dis, x, agg)
    w = prob["ws"][0]
    pair("gemm", lambda: ref["ref_agg_ops"].gemm_forward_(agg, w, out), lambda: agg_ops.gemm_forward_(agg, w, out),
         f"gemm_forward_ (cublasSgemm FP32 with a handle created per call, agg_ops.cu:369-391) vs this library's "
         f"tcgen05 TF32 GEMM, {n} x {FEAT} x {FEAT}")
    del agg, out
    torch.cuda.empty_cache()
    # the Reddit-shaped mean aggregation (the GraphSAGE configuration), F = 256
    src, dst, nr = synth.make_graph("sage_reddit_like", seed=seed, device=device, scale_nodes=scale)
    rrp, rci, _ = synth.csr_on_device(src, dst, nr, add_self_loops=False)
    del src, dst
    rx = synth.features(nr, SAGE_FEAT, seed=seed + 1, device=device)
    rout = torch.empty(nr, SAGE_FEAT, device=device)
    torch.cuda.empty_cache()
    pair("mean_aggregation", lambda: ref["ref_agg_ops"].spmm_mean_forward_(rrp, rci, rx, rout),
         lambda: agg_ops.spmm_mean_forward_(rrp, rci, rx, rout),
         f"spmm_mean_forward_ (csr_agg_kernel<true>, agg_ops.cu:23-47), Reddit-shaped graph ({nr} nodes, "
         f"{rci.numel()} entries), F = {SAGE_FEAT}")
    del rrp, rci, rx, rout
    torch.cuda.empty_cache()
    res["note"] = ("each kernel timed alone on the same seeded device tensors (inputs larger than L2); reference "
                   "kernels compiled unmodified from the reference's sources by oracle/build_ref.py")
    return res


# ---------------------------------------------------------------------------
# CPU oracle (baseline leg of our arm, and the whole --impl reference arm)
# ---------------------------------------------------------------------------

def _host_problem(prob):
    return dict(n=prob["n"], rp=prob["rp"].cpu().numpy(), ci=prob["ci"].cpu().numpy(),
                dis=prob["dis"].cpu().numpy(), x=prob["x"].cpu().numpy(),
                ws=[w.cpu().numpy() for w in prob["ws"]], bs=[b.cpu().numpy() for b in prob["bs"]])


def _cpu_rows_layer(O, hp, r0: int, r1: int, threads: int):
    """One GCN layer (aggregation + X·W + bias + ReLU) on rows [r0, r1) with the oracle."""
    agg = O.spmm(hp["rp"], hp["ci"], hp["x"], mode=O.W_GCN, dis=hp["dis"], rows=(r0, r1), nthreads=threads)
    return O.gemm_fp32(agg, hp["ws"][0], hp["bs"][0], True, nthreads=threads)


def _cpu_sample_rows(O, hp, seconds: float, threads: int) -> tuple[int, float]:
    """Rows [0, rows) whose one-layer oracle pass takes about `seconds`: grow a
    probe until it runs for at least 1/8 of the target, then extrapolate."""
    n = hp["n"]
    probe = max(1, n // 512)
    while True:
        t0 = time.perf_counter()
        _cpu_rows_layer(O, hp, 0, probe, threads)
        dt = max(time.perf_counter() - t0, 1e-4)
        if dt >= seconds / 8 or probe >= n:
            break
        probe = min(n, probe * 4)
    rows = int(min(n, max(probe, probe * seconds / dt)))
    return rows, dt


def _sample_bytes(hp, rows: int) -> int:
    nnz = int(hp["rp"][rows]) - int(hp["rp"][0])
    return spmm_layer_bytes(rows, nnz, FEAT)


def cpu_baseline(prob, seconds: float) -> dict:
    from oracle import oracle as O
    hp = _host_problem(prob)
    threads = O.max_threads()
    _cpu_rows_layer(O, hp, 0, 1, threads)  # warm the oracle library and page in the inputs
    rows, _ = _cpu_sample_rows(O, hp, seconds, threads)
    t0 = time.perf_counter()
    _cpu_rows_layer(O, hp, 0, rows, threads)
    dt = time.perf_counter() - t0
    return {"value": round(_sample_bytes(hp, rows) / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"one GCN layer (aggregation + X·W + bias + ReLU) on rows [0, {rows}) of {hp['n']} "
                      f"({_sample_bytes(hp, rows) / 1e9:.2f} algorithmic GB) in {dt:.2f} s; C oracle, OpenMP"}


def run_reference(args):
    """The reference arm: its CPU arithmetic (the C restatement) on the host's
    cores. Inputs are built on the host with torch CPU ops (same generator and
    shape as the GPU arm, the host's random stream); no GPU and nothing of this
    library is used."""
    from oracle import oracle as O
    prob = build_problem(args.seed, torch.device("cpu"), args.scale)
    hp = _host_problem(prob)
    cfg = describe(prob, args.gpus, gemm="cpu-fp32", order="CSR row order (C restatement, OpenMP over rows)",
                   chunks=default_chunks(args.chunks, args.gpus), exchange=args.exchange, transport=args.transport,
                   layout=args.layout, padded_order=args.padded_order, push_from=args.push_from)
    del prob
    threads = O.max_threads()
    total = args.steps + args.warmup
    per_step = max(0.5, min(4.0, 150.0 / max(1, total)))  # whole run within a few minutes
    rows, _ = _cpu_sample_rows(O, hp, per_step, threads)
    for _ in range(args.warmup):
        _cpu_rows_layer(O, hp, 0, rows, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _cpu_rows_layer(O, hp, 0, rows, threads)
    dt = time.perf_counter() - t0
    value = _sample_bytes(hp, rows) * args.steps / dt / 1e9
    sample = (f"each step: one GCN layer (aggregation + X·W + bias + ReLU) on rows [0, {rows}) of {hp['n']} "
              f"({_sample_bytes(hp, rows) / 1e9:.2f} algorithmic GB); C restatement of the reference arithmetic, "
              f"OpenMP over rows")
    return {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "impl": "reference",
            "data": f"synthetic: seeded R-MAT graph (seed {args.seed}) with ogbn-products shape, built on the host",
            "config": cfg,
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# Pubmed-shaped workload (1 GCN layer, the configuration the reference runs on its CPU path)
# ---------------------------------------------------------------------------

def _l2_flush_buffer(device) -> torch.Tensor:
    """A buffer twice the size of L2 whose rewrite evicts every cached line."""
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    return torch.empty(max(2 * l2, 256 << 20) // 4, dtype=torch.float32, device=device)


def run_pubmed(args, device: torch.device) -> dict:
    """gcn_inference.py's layer on the Pubmed-shaped Chung-Lu graph (19,717 nodes,
    88,648 directed entries + self-loops, F = 128, one layer, no ReLU). Its inputs
    (10 MB of features) fit in L2, so L2 is flushed before every step and each
    step is timed alone with CUDA events. The whole output is checked against the
    oracle afterwards (aggregate bit for bit, layer within the TF32 tolerance)."""
    from oracle import oracle as O
    torch.backends.cuda.matmul.allow_tf32 = True
    src, dst, n = synth.make_graph("gcn_pubmed_like", seed=args.seed, device="cpu")
    rp_h, ci_h, dis_h = O.gcn_normalized_csr(src.numpy(), dst.numpy(), n)  # the reference's builder, restated
    x_h = synth.features(n, FEAT, seed=args.seed + 1).numpy()
    w_h = synth.glorot(FEAT, FEAT, seed=args.seed + 10).numpy()
    rp, ci, dis, x, w = (torch.from_numpy(a).to(device) for a in (rp_h, ci_h, dis_h, x_h, w_h))
    b = torch.zeros(FEAT, device=device)
    nnz = int(ci.numel())
    agg = torch.empty(n, FEAT, device=device)
    out = torch.empty(n, FEAT, device=device)
    flush = _l2_flush_buffer(device)

    def step():
        gcn_ops.spmm_gcn_forward_(rp, ci, dis, x, agg)
        agg_ops.linear_forward_(agg, w, b, out, False)

    def timed(fn, k):
        ms, spmm = [], []
        for _ in range(k):
            flush.fill_(0.0)
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record()
            gcn_ops.spmm_gcn_forward_(rp, ci, dis, x, agg)
            e1.record()
            agg_ops.linear_forward_(agg, w, b, out, False)
            e2.record()
            e2.synchronize()
            ms.append(e0.elapsed_time(e2))
            spmm.append(e0.elapsed_time(e1))
        return ms, spmm

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    launches0 = N.lib().gnn_kernel_launches()
    with ClockSampler(device.index) as clocks:
        ms, spmm = timed(step, args.steps)
    launches = N.lib().gnn_kernel_launches() - launches0
    ms_step, spmm_ms = sum(ms) / len(ms), sum(spmm) / len(spmm)
    bytes_layer = spmm_layer_bytes(n, nnz, FEAT)
    # the whole output against the oracle
    got_agg = agg.cpu().numpy()
    exp_agg = O.spmm(rp_h, ci_h, x_h, mode=O.W_GCN, dis=dis_h)
    f64, ab = O.spmm_f64(rp_h, ci_h, x_h, mode=O.W_GCN, dis=dis_h)
    a64 = got_agg.astype(np.float64)
    scale = np.abs(a64) @ np.abs(w_h.astype(np.float64)) + 1e-30
    err_out = float(np.max(np.abs(out.cpu().numpy().astype(np.float64) - a64 @ w_h.astype(np.float64)) / scale))
    parity = {"rows_checked": n, "agg_bit_exact": bool(np.array_equal(got_agg.view(np.uint32), exp_agg.view(np.uint32))),
              "agg_err_vs_f64": round(O.check_close_to_f64(got_agg, f64, ab, rel=1e-5), 4),
              "max_rel_err": round(err_out, 6), "tf32_tolerance": 2e-3, "checked": "the whole graph, against the C oracle"}
    peak, peak_kind = measured_hbm_gbs()
    res = {
        "metric": METRIC, "value": round(bytes_layer / (ms_step * 1e-3) / 1e9, 2), "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "ms_per_layer": round(ms_step, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": f"synthetic: seeded Chung-Lu graph (seed {args.seed}, exponent 2.1, max expected degree 170) with the "
                "Pubmed shape, N(0,1) features, Glorot weights, zero bias",
        "config": {"workload": "gcn_pubmed_like: GCN 1 layer 128->128", "nodes": n, "csr_entries": nnz,
                   "feat_dim": FEAT, "layers": 1, "self_loops": True,
                   "l2": "L2 flushed before every step (features 10 MB), each step timed alone"},
        "roofline": {"bound": "hbm", "kernel": "spmm_vec_kernel (GCN aggregation)", "spmm_ms_per_layer": round(spmm_ms, 5),
                     "achieved": round(bytes_layer / (spmm_ms * 1e-3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(bytes_layer / (spmm_ms * 1e-3) / 1e9 / peak, 4), "peak_source": peak_kind,
                     "algorithmic_bytes_per_layer": bytes_layer, "traffic": None,
                     "frac_note": "a 66 MB layer: launch latency, not bandwidth, bounds it"},
        "parity": parity, "gpu_launches": int(launches), "clocks": clocks.summary(),
    }
    if args.cpu_seconds > 0:
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < min(args.cpu_seconds, 5.0):
            agg_c = O.spmm(rp_h, ci_h, x_h, mode=O.W_GCN, dis=dis_h)
            O.gemm_fp32(agg_c, w_h, None, False)
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        res["cpu_baseline"] = {"value": round(bytes_layer / dt / 1e9, 3), "unit": "GB/s", "cores": O.max_threads(),
                               "kind": "port", "sample": f"the whole layer (aggregation + X·W), {reps} times, "
                                                         f"{dt * 1e3:.2f} ms each; C oracle, OpenMP"}
    return res


# ---------------------------------------------------------------------------
# GraphSAGE-mean workload (Reddit-shaped graph, 2 layers 256 -> 256 -> 256)
# ---------------------------------------------------------------------------

SAGE_FEAT = 256


def mean_layer_bytes(n: int, nnz: int, f: int) -> int:
    """Algorithmic bytes of one mean aggregation: row_ptr + col_ind + one gathered
    feature row per CSR entry + the output matrix."""
    return (n + 1) * 4 + nnz * 4 + nnz * f * 4 + n * f * 4


def run_sage(args, device: torch.device) -> dict:
    """graphsage_inference.py's layer, per layer: mean aggregation, agg·W_n + b_n,
    x·W_r, add, ReLU between layers — the reference's composition
    (graphsage_inference.py:310-354) on this library's kernels."""
    t0 = time.time()
    src, dst, n = synth.make_graph("sage_reddit_like", seed=args.seed, device=device, scale_nodes=args.scale)
    rp, ci, _ = synth.csr_on_device(src, dst, n, add_self_loops=False)
    del src, dst
    nnz = int(ci.numel())
    x = synth.features(n, SAGE_FEAT, seed=args.seed + 1, device=device)
    wn = [synth.glorot(SAGE_FEAT, SAGE_FEAT, seed=args.seed + 10 + i, device=device) for i in range(LAYERS)]
    wr = [synth.glorot(SAGE_FEAT, SAGE_FEAT, seed=args.seed + 20 + i, device=device) for i in range(LAYERS)]
    bn = [torch.zeros(SAGE_FEAT, device=device) for _ in range(LAYERS)]
    agg = torch.empty(n, SAGE_FEAT, device=device)
    root = torch.empty(n, SAGE_FEAT, device=device)
    outs = [torch.empty(n, SAGE_FEAT, device=device) for _ in range(2)]
    torch.cuda.empty_cache()
    torch.cuda.synchronize(device)
    log(f"[bench] sage graph n={n} nnz={nnz} built in {time.time() - t0:.1f}s")
    torch.backends.cuda.matmul.allow_tf32 = True
    timers: dict = {}

    def step(tm=None):
        h = x
        for li in range(LAYERS):
            ev = partition._mark(tm, "spmm_begin")
            agg_ops.spmm_mean_forward_(rp, ci, h, agg)
            partition._mark(tm, "spmm_end", ev)
            o = outs[li % 2]
            agg_ops.linear_forward_(agg, wn[li], bn[li], o, False)
            agg_ops.gemm_forward_(h, wr[li], root)
            agg_ops.tensor_add_inplace_(o, root, 1.0)
            if li != LAYERS - 1:
                agg_ops.relu_inplace_(o)
            h = o
        return h

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    launches0 = N.lib().gnn_kernel_launches()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clocks:
        e0.record()
        for _ in range(args.steps):
            step(timers)
        e1.record()
        torch.cuda.synchronize(device)
    launches = N.lib().gnn_kernel_launches() - launches0
    ms_step = e0.elapsed_time(e1) / args.steps
    spmm_ms = sum(b.elapsed_time(e) for b, e in timers["spmm"]) / (args.steps * LAYERS)
    bytes_layer = mean_layer_bytes(n, nnz, SAGE_FEAT)
    # e2e through the public ops with host buffers
    dev_in = [rp, ci, x] + wn + wr + bn
    host_in = [t.cpu().pin_memory() for t in dev_in]
    out_host = torch.empty(n, SAGE_FEAT, pin_memory=True)
    torch.cuda.synchronize(device)
    q0 = torch.cuda.Event(enable_timing=True)
    q1 = torch.cuda.Event(enable_timing=True)
    q0.record()
    for _ in range(args.e2e_steps):
        for d_t, h_t in zip(dev_in, host_in):
            d_t.copy_(h_t, non_blocking=True)
        out_host.copy_(step(), non_blocking=True)
    q1.record()
    torch.cuda.synchronize(device)
    e2e_ms = q0.elapsed_time(q1) / args.e2e_steps
    peak, peak_kind = measured_hbm_gbs()
    achieved = bytes_layer / (spmm_ms * 1e-3) / 1e9
    res = {
        "metric": METRIC, "value": round(bytes_layer * LAYERS / (ms_step * 1e-3) / 1e9, 2), "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "ms_per_layer": round(ms_step / LAYERS, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp32",
        "data": f"synthetic: seeded log-normal community graph (seed {args.seed}) with Reddit shape, N(0,1) "
                "features, Glorot weights, zero bias",
        "config": {"workload": "sage_reddit_like: GraphSAGE-mean 2 layers 256->256->256 (self || mean-neighbour "
                               "linear, ReLU between layers)", "nodes": n, "csr_entries": nnz, "feat_dim": SAGE_FEAT,
                   "layers": LAYERS, "self_loops": False,
                   "gemm": "tcgen05-tf32" if N.lib().gnn_gemm_uses_tensor_cores(n, SAGE_FEAT, SAGE_FEAT)
                   else "ffma-fp32", "row_order": row_order(),
                   "l2": "X is %.2f GB (reused ~%d times per layer), no flush" % (n * SAGE_FEAT * 4 / 1e9,
                                                                                 nnz // max(1, n))},
        "roofline": {"bound": "hbm", "kernel": "spmm_vec_kernel + spmm_long_kernel (mean aggregation)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "peak_source": peak_kind, "spmm_ms_per_layer": round(spmm_ms, 4),
                     "algorithmic_bytes_per_layer": bytes_layer, "traffic": None},
        "e2e": {"value": round(bytes_layer * LAYERS / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": int(sum(t.numel() * t.element_size() for t in host_in)),
                "d2h_bytes_per_step": int(out_host.numel() * 4), "ms_per_step": round(e2e_ms, 3),
                "api": "gnn_cuda_b200.GNN_cuda_common.agg_ops over libgnnb200.so"},
        "gpu_launches": int(launches), "clocks": clocks.summary(),
    }
    return res


# ---------------------------------------------------------------------------
# GIN workload (papers100M-shaped R-MAT graph, 3 layers, MLP 128-128-128)
# ---------------------------------------------------------------------------

GIN_FEAT, GIN_LAYERS = 128, 3
GIN_ROW_CHUNKS = 32


def run_gin(args, device: torch.device) -> dict:
    """gin_inference.py's layer, per layer: sum aggregation, + (1 + eps)·x (eps = 0),
    Linear(128,128)+ReLU, Linear(128,128) (+ReLU between layers) — the reference's
    composition (gin_inference.py:317-359) on this library's kernels. The whole
    111M-node, 1.6B-entry graph (int64 row_ptr) needs X and two output matrices
    (3 x 57 GB) plus the CSR; the separate calls would add the aggregate and the
    hidden matrices (2 x 57 GB more), which one GPU does not hold, so at full
    size every layer runs as one fused kernel (gnn_fused_aggregate_linear: the
    same results as the separate calls, no [N, F] intermediate). --scale picks
    a fraction of the nodes and entries; below 1/2 the separate calls run."""
    from gnn_cuda_b200.GNN_cuda_common import fused_ops
    scale = args.scale
    torch.backends.cuda.matmul.allow_tf32 = True
    t0 = time.time()
    src, dst, n = synth.make_graph("gin_papers_like", seed=args.seed, device=device, scale_nodes=scale)
    full = scale >= 1.0
    nnz_est = int(src.numel())
    rp, ci, _ = synth.csr_on_device(src, dst, n, add_self_loops=False,
                                    index_dtype=torch.int64 if (full or nnz_est > 2**31 - 1) else torch.int32)
    del src, dst
    torch.cuda.empty_cache()
    nnz = int(ci.numel())
    x = synth.features(n, GIN_FEAT, seed=args.seed + 1, device=device)
    w1 = [synth.glorot(GIN_FEAT, GIN_FEAT, seed=args.seed + 10 + i, device=device) for i in range(GIN_LAYERS)]
    w2 = [synth.glorot(GIN_FEAT, GIN_FEAT, seed=args.seed + 20 + i, device=device) for i in range(GIN_LAYERS)]
    b = [torch.zeros(GIN_FEAT, device=device) for _ in range(GIN_LAYERS)]
    # full size: one fused kernel per layer, or the separate calls over 32 row ranges (two
    # [N/32, F] buffers; --gin-path chunks); both give the separate calls' bits
    path = "whole" if scale < 0.5 else args.gin_path
    if path == "fused" and not fused_ops.fused_supported(GIN_FEAT, GIN_FEAT, GIN_FEAT):
        path = "chunks"
    fused = path == "fused"
    torch.cuda.empty_cache()
    outs = [torch.empty(n, GIN_FEAT, device=device) for _ in range(2)]
    if path == "whole":
        agg = torch.empty(n, GIN_FEAT, device=device)
        hid = torch.empty(n, GIN_FEAT, device=device)
    torch.cuda.synchronize(device)
    log(f"[bench] gin graph n={n} nnz={nnz} built in {time.time() - t0:.1f}s; "
        f"{ {'fused': 'fused layers', 'chunks': f'separate calls over {GIN_ROW_CHUNKS} row ranges', 'whole': 'separate calls'}[path]}; "
        f"{torch.cuda.memory_allocated(device) / 1e9:.1f} GB allocated")
    timers: dict = {}

    def step(tm=None):
        h = x
        for li in range(GIN_LAYERS):
            o = outs[li % 2]
            ev = partition._mark(tm, "spmm_begin")
            if fused:
                fused_ops.gin_layer_forward_(rp, ci, h, 0.0, w1[li], b[li], w2[li], b[li], o, li != GIN_LAYERS - 1)
                partition._mark(tm, "spmm_end", ev)
            elif path == "chunks":
                fused_ops.gin_layer_row_chunks_(rp, ci, h, 0.0, w1[li], b[li], w2[li], b[li], o, li != GIN_LAYERS - 1,
                                                chunks=GIN_ROW_CHUNKS)
                partition._mark(tm, "spmm_end", ev)
            else:
                agg_ops.spmm_sum_forward_(rp, ci, h, agg)
                partition._mark(tm, "spmm_end", ev)
                agg_ops.tensor_add_inplace_(agg, h, 1.0)  # (1 + eps) * x with eps = 0
                agg_ops.linear_forward_(agg, w1[li], b[li], hid, True)
                agg_ops.linear_forward_(hid, w2[li], b[li], o, li != GIN_LAYERS - 1)
            h = o
        return h

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    launches0 = N.lib().gnn_kernel_launches()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clocks:
        e0.record()
        for _ in range(args.steps):
            step(timers)
        e1.record()
        torch.cuda.synchronize(device)
    launches = N.lib().gnn_kernel_launches() - launches0
    ms_step = e0.elapsed_time(e1) / args.steps
    spmm_ms = sum(bb.elapsed_time(ee) for bb, ee in timers["spmm"]) / (args.steps * GIN_LAYERS)
    bytes_layer = mean_layer_bytes(n, nnz, GIN_FEAT) + (rp.element_size() - 4) * (n + 1)
    peak, peak_kind = measured_hbm_gbs()
    achieved = bytes_layer / (spmm_ms * 1e-3) / 1e9
    return {
        "metric": METRIC, "value": round(bytes_layer * GIN_LAYERS / (ms_step * 1e-3) / 1e9, 2), "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "ms_per_layer": round(ms_step / GIN_LAYERS, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp32",
        "data": f"synthetic: seeded R-MAT graph (seed {args.seed}) with the ogbn-papers100M shape at {scale:g} of its "
                "nodes and entries, N(0,1) features, Glorot weights, zero bias",
        "config": {"workload": f"gin_papers_like x{scale:g}: GIN 3 layers, eps = 0, MLP Linear(128,128)-ReLU-"
                               "Linear(128,128), ReLU between layers", "nodes": n, "csr_entries": nnz,
                   "layer": {"fused": "fused aggregation + MLP (one kernel per layer)",
                             "chunks": f"separate calls over {GIN_ROW_CHUNKS} row ranges (two [N/{GIN_ROW_CHUNKS}, F] "
                                       "buffers)", "whole": "separate calls"}[path],
                   "feat_dim": GIN_FEAT, "layers": GIN_LAYERS, "self_loops": False,
                   "row_ptr": "int64" if rp.dtype == torch.int64 else "int32", "row_order": row_order(),
                   "l2": "inputs larger than L2 (X is %.1f GB), no flush" % (n * GIN_FEAT * 4 / 1e9)},
        "roofline": {"bound": "hbm", "kernel": {"fused": "fused_layer_kernel + spmm_long_kernel (sum aggregation and "
                                                         "MLP; the time includes the two transforms)",
                                                "chunks": "spmm_vec_kernel + spmm_long_kernel + the MLP, per row range "
                                                          "(the time includes the add and the two transforms)",
                                                "whole": "spmm_vec_kernel + spmm_long_kernel (sum aggregation)"}[path],
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "peak_source": peak_kind, "spmm_ms_per_layer": round(spmm_ms, 4),
                     "algorithmic_bytes_per_layer": bytes_layer, "traffic": None},
        "gpu_launches": int(launches), "clocks": clocks.summary(),
    }


# ---------------------------------------------------------------------------
# locality preprocessing workload (the input of spmm_mode=optimized)
# ---------------------------------------------------------------------------

LOCALITY_METRIC = "GCN locality preprocessing throughput (CSR entries/s), 1 B200"
LOCALITY_CPU_SCALE = 1.0 / 16


def _locality_graph(seed: int, device, scale: float):
    src, dst, n = synth.make_graph(WORKLOAD, seed=seed, device=device, scale_nodes=scale)
    return src, dst, n


def run_locality(args, device: torch.device) -> dict:
    from gnn_cuda_b200.GNN_cuda_common.locality import preprocess_gcn_graph
    src, dst, n = _locality_graph(args.seed, device, args.scale)
    entries = int(src.numel()) + n  # CSR entries incl. self-loops (the graph is duplicate-free)
    for _ in range(max(1, args.warmup)):
        preprocess_gcn_graph(src, dst, num_nodes=n)
    torch.cuda.synchronize(device)
    launches0 = N.lib().gnn_kernel_launches()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clocks:
        t0.record()
        for _ in range(args.steps):
            pay = preprocess_gcn_graph(src, dst, num_nodes=n)
        t1.record()
        torch.cuda.synchronize(device)
    ms = t0.elapsed_time(t1) / args.steps
    launches = N.lib().gnn_kernel_launches() - launches0
    value = entries / (ms * 1e-3) / 1e6
    # e2e: host edge lists in, the payload back on the host
    h_src, h_dst = src.cpu().pin_memory(), dst.cpu().pin_memory()
    e0 = time.perf_counter()
    pay_h = preprocess_gcn_graph(h_src, h_dst, num_nodes=n)
    e2e_s = time.perf_counter() - e0
    d2h = sum(v.numel() * v.element_size() for v in pay_h.values() if isinstance(v, torch.Tensor))
    res = {
        "metric": LOCALITY_METRIC, "value": round(value, 2), "unit": "M entries/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int64",
        "data": f"synthetic: seeded R-MAT graph (seed {args.seed}) with ogbn-products shape",
        "config": {"workload": "locality_products_like: page schedule -> co-access order -> hot partition -> "
                               "renumbered page schedule (run/preprocess_gcn_graph.py defaults)",
                   "nodes": n, "csr_entries": entries, "feat_dim": 128, "page_bytes": 4096,
                   "hot_cutoff": int(pay["hot_node_cutoff"]), "num_pages": int(pay["num_pages"])},
        "e2e": {"value": round(entries / e2e_s / 1e6, 2), "unit": "M entries/s",
                "h2d_bytes_per_step": int(2 * src.numel() * 8), "d2h_bytes_per_step": int(d2h),
                "api": "gnn_cuda_b200.GNN_cuda_common.locality.preprocess_gcn_graph on host tensors"},
        "gpu_launches": int(launches), "clocks": clocks.summary(),
    }
    if args.cpu_seconds > 0:
        res["cpu_baseline"] = locality_cpu_baseline(args.seed)
    return res


def locality_cpu_baseline(seed: int) -> dict:
    """The numpy restatement of the reference's preprocessing (oracle/locality.py,
    one core) on the same generator at 1/16 of the nodes and entries. The
    reference's own functions need a dense [row blocks x pages] int64 array
    (94 GB at the full products shape), so the port stands in for them."""
    from oracle import locality as OL
    src, dst, n = _locality_graph(seed, "cpu", LOCALITY_CPU_SCALE)
    s, d = src.numpy(), dst.numpy()
    t0 = time.perf_counter()
    OL.preprocess(s, d, num_nodes=n)
    dt = time.perf_counter() - t0
    entries = int(s.size) + n
    return {"value": round(entries / dt / 1e6, 3), "unit": "M entries/s", "cores": 1, "kind": "port",
            "sample": f"the whole preprocessing chain on a 1/16-scale graph ({n} nodes, {entries} entries) "
                      f"in {dt:.2f} s; vectorised numpy restatement of graph_utils.py:174-446"}


def main() -> int:
    args = parse_args()
    if args.workload == "gin_papers_like":
        # three 57 GB matrices next to the graph: let the allocator grow segments
        # instead of failing on fragments left by the graph construction
        os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        log(f"[bench] WORLD_SIZE={world} but --gpus={args.gpus}; using WORLD_SIZE")
    device = torch.device("cuda", local_rank)
    if args.impl != "reference":
        torch.cuda.set_device(device)
    if args.workload == "gin_papers_like":
        if rank != 0:
            return 0
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the CPU reference arm is measured on the "
                              "default workload (gcn_products_like)"}), flush=True)
        else:
            print(json.dumps(run_gin(args, device)), flush=True)
        return 0
    if args.workload == "gcn_pubmed_like":
        if rank != 0:
            return 0
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the CPU reference arm is measured on the "
                              "default workload (gcn_products_like)"}), flush=True)
        else:
            print(json.dumps(run_pubmed(args, device)), flush=True)
        return 0
    if args.workload == "sage_reddit_like":
        if rank != 0:
            return 0
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the CPU reference arm is measured on the "
                              "default workload (gcn_products_like)"}), flush=True)
        else:
            print(json.dumps(run_sage(args, device)), flush=True)
        return 0
    if args.workload == "locality_products_like":
        if rank != 0:
            return 0
        if args.impl == "reference":
            cpu = locality_cpu_baseline(args.seed)
            print(json.dumps({"metric": LOCALITY_METRIC, "value": cpu["value"], "unit": cpu["unit"], "n_gpus": 1,
                              "impl": "reference", "higher_is_better": True, "cpu_baseline": cpu,
                              "e2e": {"value": cpu["value"], "unit": cpu["unit"], "h2d_bytes_per_step": 0,
                                      "d2h_bytes_per_step": 0}}), flush=True)
        else:
            print(json.dumps(run_locality(args, device)), flush=True)
        return 0
    if args.impl == "reference":
        if rank != 0:
            return 0
        print(json.dumps(run_reference(args)), flush=True)
        return 0
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    try:
        res = run_ours(args, rank, world, device)
        if res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
