#!/usr/bin/env python3
"""SpMM time and unified-memory migration per inference iteration, without nsys
(reference: run/profile_spmm_migration.py).

The reference wraps the model's inference script in ``nsys profile``, exports
SQLite, finds the feature matrix's address range in the script's stdout and
sums the unified-memory migrations and GPU page faults over it
(:146-461). Here the same inference runs in this process with CUPTI's
unified-memory counters switched on before CUDA starts
(``um_profiler.UMProfiler``, libgnnb200_umprof.so), and the driver hands back
the feature range, its SpMM phase time and the measured-loop window. Same
flags (conda-related ones are accepted and ignored: there is no environment
dispatch), same summary file name and the same four report lines:

    Summary Report:
    spmm_ns, ...      average aggregation time per measured iteration
    HtoD_bytes, ...   feature-range host-to-device migration bytes
    DtoH_bytes, ...   feature-range device-to-host migration bytes
    GPU_faults, ...   feature-range GPU page faults

Counting follows the reference: for ``--ft_matrix uvm`` every feature-range
record of the run counts (prefetch and first-touch migrations happen before the
measured loop), otherwise the records inside the measured loop, averaged per
iteration.
"""
from __future__ import annotations

import argparse
import contextlib
import io
import os
import sys
from pathlib import Path

REPO_ROOT = Path(__file__).resolve().parents[2]
DEFAULT_DATA_ROOT = os.environ.get("GNN_DATASET_ROOT", "/root/workspace/mnt/dataset_npz")
MODELS = {"gcn": "gcn", "gin": "gin", "sag": "graphsage", "graphsage": "graphsage"}


def _prefetch_to_location(prefetch: int) -> str:
    if int(prefetch) == 0:
        return "none"
    if int(prefetch) == 1:
        return "cuda"
    raise ValueError("--prefetch expects 0 or 1")


def _artifact_base(output_dir: Path, a) -> Path:
    host_token = f"host{a.ft_host_alloc:g}".replace(".", "p")
    return output_dir / (f"{a.framework}_{MODELS[a.model] if a.model != 'sag' else 'sag'}_"
                         f"{a.dataset.replace('/', '_')}_dim{int(a.dim)}_{a.ft_matrix}_{host_token}_"
                         f"prefetch{a.resolved_prefetch_location}_spmm_um")


def _inference_argv(a) -> list[str]:
    argv = ["--dataset", a.dataset, "--data_root", a.data_root, "--dim", str(a.dim), "--num_layers",
            str(a.num_layers), "--adj_matrix", a.adj_matrix, "--ft_matrix", a.ft_matrix, "--weight", a.weight,
            "--warmup", str(a.warmup), "--iters", str(a.iters), "--device", a.device,
            "--preferred_location", a.resolved_prefetch_location, "--prefetch_to", a.resolved_prefetch_location,
            "--ft_host_alloc", str(a.ft_host_alloc)]
    extra = list(a.extra_args or [])
    if extra and extra[0] == "--":
        extra = extra[1:]
    return argv + extra


def _runner(framework: str, model: str):
    from gnn_cuda_b200.GNN_cuda_common import npz_utils
    key = MODELS[model]
    load = npz_utils.load_pyg_graph_features_from_npz if framework == "pyg" else \
        npz_utils.load_dgl_graph_features_from_npz
    if key == "gcn":
        from gnn_cuda_b200.GNN_cuda_common.gcn_inference import run_gcn_inference as run
    elif key == "gin":
        from gnn_cuda_b200.GNN_cuda_common.gin_inference import run_gin_inference as run
    else:
        from gnn_cuda_b200.GNN_cuda_common.graphsage_inference import run_graphsage_inference as run
    return run, load


def _synthetic_loader(spec: str, framework: str, device: str):
    """Loader for ``--synthetic rmat:NODES:PAIRS[:SEED]``: a seeded R-MAT graph
    (a=0.57, b=c=0.19) of PAIRS distinct undirected pairs, symmetrised, built
    on the GPU, with N(0, 1) host features of the requested width — the same
    tuple an npz loader returns, without writing the graph to disk."""
    parts = spec.split(":")
    if len(parts) not in (3, 4) or parts[0] != "rmat":
        raise ValueError("--synthetic expects rmat:NODES:PAIRS[:SEED]")
    n, pairs = int(parts[1]), int(parts[2])
    seed = int(parts[3]) if len(parts) == 4 else 1

    def load(_path: str, feat_dim: int, use_npz_features: bool):
        import torch
        from gnn_cuda_b200 import synth
        u, v = synth.rmat_undirected(n, pairs, seed=seed, device=device)
        src, dst = synth.symmetrize(u, v)
        del u, v
        feats = synth.features(n, feat_dim if feat_dim > 0 else 128, seed=seed + 1)
        torch.cuda.empty_cache()
        if framework == "pyg":
            return torch.stack([src, dst]), feats, n
        return src, dst, feats, n
    return load


def profile(a) -> dict:
    """Runs the inference in-process under the UM counters; returns the summary."""
    from gnn_cuda_b200.GNN_cuda_common.um_profiler import UMProfiler
    prof = UMProfiler()
    try:
        prof.start()  # before the first CUDA call of the run
        counters = ""
    except RuntimeError as e:  # no unified-memory counters here: SpMM time only
        prof, counters = None, str(e)
        print(f"warning: {counters}; HtoD_bytes, DtoH_bytes and GPU_faults are reported as nan", file=sys.stderr)
    import torch
    from gnn_cuda_b200.GNN_cuda_common import npz_utils
    run, load = _runner(a.framework, a.model)
    if a.synthetic:
        load = _synthetic_loader(a.synthetic, a.framework, a.device)
    window = {}
    pcie = None
    if prof is None:
        # no unified-memory counters: the host-link bytes of the measured loop from NVML instead
        try:
            from gnn_cuda_b200.GNN_cuda_common.um_profiler import PcieSampler
            pcie = PcieSampler(torch.device(a.device).index or 0)
            pcie._read = pcie._nvml_reader()
        except Exception as e:  # no NVML either: SpMM time only
            pcie = None
            print(f"warning: no NVML PCIe counters either ({e})", file=sys.stderr)
    cap = {"on_measure_begin": lambda: (window.__setitem__("t0", UMProfiler.timestamp()) if prof is not None
                                        else pcie.start() if pcie is not None else None),
           "on_measure_end": lambda: (window.__setitem__("t1", UMProfiler.timestamp()) if prof is not None
                                      else pcie.stop() if pcie is not None else None)}
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        rc = run(framework_label=a.framework, select_device=npz_utils.select_device, load_graph_features=load,
                 load_kind=a.framework, argv=_inference_argv(a), capture=cap)
    if rc != 0:
        raise RuntimeError(f"inference returned {rc}")
    torch.cuda.synchronize()
    nan = float("nan")
    um = {"htod_bytes": nan, "dtoh_bytes": nan, "gpu_page_faults": nan, "records": 0, "dropped_records": 0}
    if prof is not None:
        prof.flush()
        lo, hi = cap["feature_range"]
        iters = max(1, int(cap["iters"]))
        if a.ft_matrix == "uvm":
            um = prof.totals((lo, hi))
        else:
            um = prof.totals((lo, hi), (window["t0"], window["t1"]))
            um = {k: (v / iters if isinstance(v, float) else v) for k, v in um.items()}
        prof.stop()
    if pcie is not None and pcie.samples:
        iters = max(1, int(cap["iters"]))
        um = dict(um, htod_bytes=pcie.rx_bytes / iters, dtoh_bytes=pcie.tx_bytes / iters)
        counters = "nvml-pcie: whole-device host-link bytes per iteration of the measured loop (no fault count)"
    return {"spmm_ns": float(cap["spmm_avg_ns"]), "htod_bytes": um["htod_bytes"], "dtoh_bytes": um["dtoh_bytes"],
            "gpu_faults": um["gpu_page_faults"], "records": um["records"], "dropped_records": um["dropped_records"],
            "counters": counters or "cupti", "stdout": out.getvalue()}


def _report(s: dict) -> str:
    return ("Summary Report:\n"
            f"spmm_ns, {s['spmm_ns']:.3f}\n"
            f"HtoD_bytes, {s['htod_bytes']:.3f}\n"
            f"DtoH_bytes, {s['dtoh_bytes']:.3f}\n"
            f"GPU_faults, {s['gpu_faults']:.3f}\n")


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(description="Profile GNN inference in-process (CUPTI unified-memory counters) and "
                                            "print average SpMM time plus UM migration metrics.")
    p.add_argument("--framework", type=str, default="pyg", choices=("pyg", "dgl"))
    p.add_argument("--model", type=str, default="gcn", choices=("gcn", "gin", "sag", "graphsage"))
    p.add_argument("--dataset", type=str, required=True)
    p.add_argument("--data_root", type=str, default=DEFAULT_DATA_ROOT)
    p.add_argument("--dim", type=int, default=128)
    p.add_argument("--num_layers", type=int, default=1)
    p.add_argument("--adj_matrix", type=str, default="device", choices=("device", "uvm", "hmm"))
    p.add_argument("--ft_matrix", type=str, required=True, choices=("device", "uvm", "hmm"))
    p.add_argument("--ft_host_alloc", type=float, default=0.0,
                   help="target percent of the feature matrix that should not fit in remaining effective GPU memory")
    p.add_argument("--weight", type=str, default="device", choices=("device", "uvm"))
    p.add_argument("--prefetch", type=int, default=0, choices=(0, 1))
    p.add_argument("--warmup", type=int, default=1)
    p.add_argument("--iters", type=int, default=5)
    p.add_argument("--device", type=str, default="cuda:0")
    p.add_argument("--conda_env", type=str, default="", help="accepted for compatibility; unused")
    p.add_argument("--output_dir", type=str, default=str(REPO_ROOT / "report" / "um_spmm"))
    p.add_argument("--synthetic", type=str, default="",
                   help="rmat:NODES:PAIRS[:SEED]: generate the graph on the GPU instead of reading <dataset>.npz")
    p.add_argument("extra_args", nargs=argparse.REMAINDER)
    a = p.parse_args(argv)
    if a.ft_host_alloc < 0.0 or a.ft_host_alloc >= 100.0:
        raise ValueError("--ft_host_alloc expects a value in [0, 100)")
    if a.ft_host_alloc > 0.0 and a.model != "gcn":
        raise ValueError("--ft_host_alloc is currently implemented for --model gcn")
    a.resolved_prefetch_location = _prefetch_to_location(a.prefetch)
    out_dir = Path(a.output_dir).resolve()
    out_dir.mkdir(parents=True, exist_ok=True)
    base = _artifact_base(out_dir, a)
    s = profile(a)
    base.with_name(base.name + "_target.stdout").write_text(s["stdout"])
    base.with_name(base.name + "_summary.txt").write_text(_report(s))
    sys.stdout.write(_report(s))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
