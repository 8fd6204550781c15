"""Seeded synthetic graphs and inputs with the shapes of the benchmark workloads.

The public datasets the workloads mirror (Pubmed, ogbn-products, Reddit,
ogbn-papers100M) are not available offline; these generators reproduce their
node count, exact directed-entry count and degree character:

  chung_lu_undirected     power-law expected degrees with a capped maximum
                          (Pubmed-like: 19,717 nodes, 44,324 undirected pairs)
  rmat_undirected         R-MAT(a, b, c, d) recursive quadrant sampling at
                          scale ceil(log2 N), ids >= N rejected
                          (ogbn-products-like: 2,449,029 nodes, 61,859,140 entries)
  community_lognormal     log-normal degrees (sigma 1.0) with 80% of each node's
                          edges inside its contiguous community block
                          (Reddit-like: 232,965 nodes, 114,615,892 entries)

Every generator returns *unique undirected pairs without self-pairs*; callers
symmetrise them (``symmetrize``) into the reference's npz edge-list format
(``src_li``, ``dst_li``, ``num_nodes``; npz_utils.py:72-87). Randomness comes from
one seeded torch.Generator per call, so a (seed, device) pair always gives the
same graph. Large graphs are generated on the GPU with PyTorch ops (setup, not
the measured path) and CSR-built there too (``csr_on_device``), with the GCN
normalisation taken from an exact float32 table so it matches the host builder
bit for bit.
"""
from __future__ import annotations

import math

import numpy as np
import torch


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=torch.device(device))
    g.manual_seed(int(seed))
    return g


def _take_exact_unique(keys: torch.Tensor, target: int, g: torch.Generator) -> torch.Tensor:
    """Unique keys, then a seeded random subset of exactly `target` of them (sorted)."""
    u = torch.unique(keys)
    if u.numel() < target:
        raise RuntimeError(f"generator produced {u.numel()} unique pairs < target {target}")
    idx = torch.randperm(u.numel(), generator=g, device=u.device)[:target]
    return torch.sort(u[idx]).values


def _pairs_from_keys(keys: torch.Tensor, n: int) -> tuple[torch.Tensor, torch.Tensor]:
    a = keys // n
    return a, keys - a * n


def _canonical_keys(u: torch.Tensor, v: torch.Tensor, n: int) -> torch.Tensor:
    keep = u != v
    u, v = u[keep], v[keep]
    lo, hi = torch.minimum(u, v), torch.maximum(u, v)
    return lo * n + hi


def chung_lu_undirected(n: int, num_pairs: int, *, exponent: float = 2.1, max_degree: float = 170.0,
                        seed: int = 0, device="cpu") -> tuple[torch.Tensor, torch.Tensor]:
    """Unique undirected pairs with expected degrees d_i = d_max * (1 + i / i0)^(-1/(exponent-1))."""
    alpha = 1.0 / (exponent - 1.0)
    mean_target = 2.0 * num_pairs / n

    def mean_deg(i0: float) -> float:
        i = np.arange(n, dtype=np.float64)
        return float(np.mean(max_degree * (1.0 + i / i0) ** (-alpha)))

    lo, hi = 1e-6, float(n) * 1e3
    for _ in range(200):  # bisection on the offset i0 so the mean degree hits the target
        mid = math.sqrt(lo * hi)
        if mean_deg(mid) < mean_target:
            lo = mid
        else:
            hi = mid
    i0 = math.sqrt(lo * hi)
    w = max_degree * (1.0 + np.arange(n, dtype=np.float64) / i0) ** (-alpha)
    g = _gen(seed, device)
    p = torch.as_tensor(w / w.sum(), dtype=torch.float64, device=device)
    cdf = torch.cumsum(p, 0)
    cdf[-1] = 1.0
    keys = torch.zeros(0, dtype=torch.int64, device=device)
    batch = int(num_pairs * 1.3) + 1024
    while True:
        u = torch.searchsorted(cdf, torch.rand(batch, generator=g, dtype=torch.float64, device=device))
        v = torch.searchsorted(cdf, torch.rand(batch, generator=g, dtype=torch.float64, device=device))
        keys = torch.unique(torch.cat([keys, _canonical_keys(u.clamp_max(n - 1), v.clamp_max(n - 1), n)]))
        if keys.numel() >= num_pairs:
            break
    return _pairs_from_keys(_take_exact_unique(keys, num_pairs, g), n)


def rmat_undirected(n: int, num_pairs: int, *, a: float = 0.57, b: float = 0.19, c: float = 0.19,
                    seed: int = 0, device="cpu", batch: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Unique undirected R-MAT pairs: each of ceil(log2 n) levels picks a quadrant
    with probabilities (a, b, c, 1-a-b-c); pairs with an id >= n or u == v are rejected."""
    scale = max(1, int(math.ceil(math.log2(max(2, n)))))
    g = _gen(seed, device)
    keys = torch.zeros(0, dtype=torch.int64, device=device)
    batch = int(batch or min(max(num_pairs // 2, 1 << 16), 1 << 27))
    ab, abc = a + b, a + b + c
    while True:
        src = torch.zeros(batch, dtype=torch.int64, device=device)
        dst = torch.zeros(batch, dtype=torch.int64, device=device)
        for level in range(scale):
            r = torch.rand(batch, generator=g, device=device)
            src |= (r >= ab).to(torch.int64) << level
            dst |= (((r >= a) & (r < ab)) | (r >= abc)).to(torch.int64) << level
        ok = (src < n) & (dst < n)
        keys = torch.unique(torch.cat([keys, _canonical_keys(src[ok], dst[ok], n)]))
        if keys.numel() >= num_pairs:
            break
    return _pairs_from_keys(_take_exact_unique(keys, num_pairs, g), n)


def community_lognormal(n: int, num_pairs: int, *, sigma: float = 1.0, communities: int = 50, p_in: float = 0.8,
                        seed: int = 0, device="cpu") -> tuple[torch.Tensor, torch.Tensor]:
    """Unique undirected pairs: node weights ~ LogNormal(0, sigma); one endpoint is
    drawn by weight, the other by weight inside its community block (prob. p_in)
    or over all nodes."""
    g = _gen(seed, device)
    w = torch.exp(torch.randn(n, generator=g, dtype=torch.float64, device=device) * sigma)
    cdf = torch.cumsum(w / w.sum(), 0)
    cdf[-1] = 1.0
    zero = torch.zeros(1, dtype=torch.float64, device=device)
    cdf0 = torch.cat([zero, cdf])  # cdf0[i] = mass of nodes < i
    bounds = torch.linspace(0, n, communities + 1, device=device).round().to(torch.int64)
    comm_of = torch.bucketize(torch.arange(n, device=device), bounds[1:], right=True)
    keys = torch.zeros(0, dtype=torch.int64, device=device)
    batch = min(max(num_pairs // 2, 1 << 16), 1 << 26)
    while True:
        u = torch.searchsorted(cdf, torch.rand(batch, generator=g, dtype=torch.float64, device=device)).clamp_max(n - 1)
        inside = torch.rand(batch, generator=g, device=device) < p_in
        cu = comm_of[u]
        lo_m, hi_m = cdf0[bounds[cu]], cdf0[bounds[cu + 1]]
        r = torch.rand(batch, generator=g, dtype=torch.float64, device=device)
        t = torch.where(inside, lo_m + r * (hi_m - lo_m), r)
        v = torch.searchsorted(cdf, t).clamp_max(n - 1)
        keys = torch.unique(torch.cat([keys, _canonical_keys(u, v, n)]))
        if keys.numel() >= num_pairs:
            break
    return _pairs_from_keys(_take_exact_unique(keys, num_pairs, g), n)


def symmetrize(u: torch.Tensor, v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Directed edge list (src, dst) holding both directions of every pair."""
    return torch.cat([u, v]), torch.cat([v, u])


def features(n: int, f: int, *, seed: int, device="cpu") -> torch.Tensor:
    """i.i.d. N(0, 1) float32 node features."""
    return torch.randn(n, f, generator=_gen(seed, device), dtype=torch.float32, device=device)


def glorot(fan_in: int, fan_out: int, *, seed: int, device="cpu") -> torch.Tensor:
    """Glorot-uniform weight stored [in, out] (nn.Linear.weight transposed)."""
    bound = math.sqrt(6.0 / (fan_in + fan_out))
    u = torch.rand(fan_in, fan_out, generator=_gen(seed, device), dtype=torch.float32, device=device)
    return (u * 2.0 - 1.0) * bound


def deg_inv_sqrt_table(max_degree: int) -> np.ndarray:
    """table[d] = float32 clip(d, 1)^-0.5 via numpy's float32 power, d in [0, max_degree]."""
    d = np.arange(max_degree + 1, dtype=np.float32)
    return np.power(np.clip(d, np.float32(1.0), None), np.float32(-0.5)).astype(np.float32)


def csr_on_device(src: torch.Tensor, dst: torch.Tensor, n: int, *, add_self_loops: bool,
                  index_dtype: torch.dtype = torch.int32):
    """dst-major CSR of a duplicate-free edge list, built with device sorts.

    Returns (row_ptr, col_ind int32, deg_inv_sqrt f32) on src's device; equal to
    the host builder's output for duplicate-free input without self-pairs.
    """
    if add_self_loops:
        loop = torch.arange(n, dtype=torch.int64, device=src.device)
        src, dst = torch.cat([src, loop]), torch.cat([dst, loop])
    keys = torch.sort(dst.to(torch.int64) * n + src.to(torch.int64)).values
    rows = keys // n
    col = (keys - rows * n).to(torch.int32)
    counts = torch.bincount(rows, minlength=n)
    row_ptr = torch.zeros(n + 1, dtype=torch.int64, device=src.device)
    torch.cumsum(counts, 0, out=row_ptr[1:])
    table = torch.as_tensor(deg_inv_sqrt_table(int(counts.max().item()) if n else 0), device=src.device)
    dis = table[counts]
    return row_ptr.to(index_dtype), col, dis


# ---- the workloads -----------------------------------------------------------------

WORKLOADS = {
    # name: (nodes, undirected pairs, generator, feat_dim, layers, model)
    "gcn_pubmed_like": dict(n=19_717, pairs=44_324, gen="chung_lu", f=128, layers=1, model="gcn", loops=True),
    "gcn_products_like": dict(n=2_449_029, pairs=30_929_570, gen="rmat", f=128, layers=2, model="gcn", loops=True),
    "sage_reddit_like": dict(n=232_965, pairs=57_307_946, gen="community", f=256, layers=2, model="sage", loops=False),
    "gin_papers_like": dict(n=111_059_956, pairs=807_842_936, gen="rmat", f=128, layers=3, model="gin", loops=False),
}


def make_graph(name: str, *, seed: int = 1, device="cpu", scale_nodes: float = 1.0):
    """(src, dst, n) directed edge list of a named workload (optionally scaled down)."""
    w = WORKLOADS[name]
    n = max(8, int(w["n"] * scale_nodes))
    pairs = max(1, int(w["pairs"] * scale_nodes))
    if w["gen"] == "chung_lu":
        u, v = chung_lu_undirected(n, pairs, seed=seed, device=device)
    elif w["gen"] == "rmat":
        u, v = rmat_undirected(n, pairs, seed=seed, device=device)
    else:
        u, v = community_lognormal(n, pairs, seed=seed, device=device)
    s, d = symmetrize(u, v)
    return s, d, n
