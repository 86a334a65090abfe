"""Seeded synthetic inputs with the shapes and distributions of the benchmark
configurations (no public dataset is involved).

Gaussian mixtures: pick a centre uniformly per row, add per-coordinate
Gaussian noise.  Queries come from the same mixture on an independent stream.
"""
from __future__ import annotations

import numpy as np

# The five benchmark configurations (index shape and search parameters).
CONFIGS = {
    0: dict(name="c0_ivfpq_n1e5_d96", n=100_000, d=96, nlist=256, M=16, ks=256, nprobe=16, k=10, nq=1_000,
            centres=100, centre="normal", sigma=0.15, integer=False),
    1: dict(name="c1_ivfpq_n1e6_d128", n=1_000_000, d=128, nlist=4096, M=32, ks=256, nprobe=32, k=10, nq=10_000,
            centres=1_000, centre="uniform120", sigma=12.0, integer=True),
    2: dict(name="c2_flat_ip_n1e6_d100", n=1_000_000, d=100, k=100, nq=10_000, centre="flat"),
    3: dict(name="c3_ivfpq4_n1e7_d96", n=10_000_000, d=96, nlist=16_384, M=48, ks=16, nprobe=64, k=10, nq=10_000,
            centres=10_000, centre="normal", sigma=0.15, integer=False),
    4: dict(name="c4_ivfpq_n1e8_d96", n=100_000_000, d=96, nlist=65_536, M=16, ks=256, nprobe=128, k=10,
            nq=100_000, centres=100_000, centre="normal", sigma=0.15, integer=False, generated="device",
            train_sample=2_097_152),
}


def mixture(n: int, d: int, centres: int, sigma: float, seed: int, centre: str = "normal",
            integer: bool = False, nq: int = 0, chunk: int = 1 << 20):
    """Return (database [n, d], queries [nq, d]) float32 from one mixture."""
    crng = np.random.default_rng([seed, 0])
    if centre == "normal":
        cen = crng.standard_normal((centres, d), dtype=np.float32)
    elif centre == "uniform120":
        cen = crng.uniform(0.0, 120.0, size=(centres, d)).astype(np.float32)
    else:
        raise ValueError(centre)

    def draw(count: int, stream: int) -> np.ndarray:
        out = np.empty((count, d), dtype=np.float32)
        rng = np.random.default_rng([seed, stream])
        for s in range(0, count, chunk):
            m = min(chunk, count - s)
            lab = rng.integers(0, centres, size=m)
            blk = rng.standard_normal((m, d), dtype=np.float32)
            blk *= np.float32(sigma)
            blk += cen[lab]
            if integer:
                np.rint(blk, out=blk)
                np.clip(blk, 0.0, 255.0, out=blk)
            out[s:s + m] = blk
        return out

    return draw(n, 1), draw(nq, 2)


def unit_gaussian(n: int, d: int, seed: int, nq: int = 0):
    """N(0,1) rows, L2-normalised (the flat inner-product configuration)."""
    def draw(count: int, stream: int) -> np.ndarray:
        x = np.random.default_rng([seed, stream]).standard_normal((count, d), dtype=np.float32)
        x /= np.linalg.norm(x, axis=1, keepdims=True)
        return x

    return draw(n, 1), draw(nq, 2)


def config_data(cfg: int, seed: int = 0, n: int | None = None, nq: int | None = None):
    c = CONFIGS[cfg]
    n = c["n"] if n is None else n
    nq = c["nq"] if nq is None else nq
    if c["centre"] == "flat":
        return unit_gaussian(n, c["d"], seed, nq)
    return mixture(n, c["d"], c["centres"], c["sigma"], seed, c["centre"], c["integer"], nq)


def exact_topk_cosine(db_n: np.ndarray, q_n: np.ndarray, k: int) -> np.ndarray:
    """Exact top-k by dot product on normalised rows (host ground truth for
    recall@k on small sets; float64 accumulation)."""
    out = np.empty((q_n.shape[0], k), dtype=np.int64)
    block = max(1, (1 << 26) // max(1, db_n.shape[0]))
    dbt = db_n.T.astype(np.float64)
    for s in range(0, q_n.shape[0], block):
        sims = q_n[s:s + block].astype(np.float64) @ dbt
        part = np.argpartition(-sims, k - 1, axis=1)[:, :k]
        order = np.take_along_axis(sims, part, axis=1)
        idx = np.argsort(-order, axis=1, kind="stable")
        out[s:s + block] = np.take_along_axis(part, idx, axis=1)
    return out


def recall_at_k(found: np.ndarray, truth: np.ndarray) -> float:
    k = truth.shape[1]
    hits = 0
    for f, t in zip(found, truth):
        hits += len(set(f[:k].tolist()) & set(t.tolist()))
    return hits / float(truth.size)


def device_mixture(cfg: int, seed: int, device: int, n: int | None = None, nq: int | None = None,
                   chunk: int = 1 << 22):
    """The configuration's Gaussian mixture drawn on the GPU (configuration 4:
    1e8 rows are generated on the device and never held on the host).

    ``device`` is a CUDA ordinal (or a torch device string).  Returns
    (centres, chunks, queries): ``chunks`` yields [rows, d] float32 tensors of
    the database in order, on that device; ``queries`` is a host array from
    an independent stream of the same mixture.  Every chunk is a pure function
    of (seed, chunk index), so each rank of a multi-GPU job regenerates the
    identical database.
    """
    import torch

    c = CONFIGS[cfg]
    d, centres, sigma = c["d"], c["centres"], c["sigma"]
    n = c["n"] if n is None else n
    nq = c["nq"] if nq is None else nq
    dev = torch.device(device) if isinstance(device, str) else torch.device("cuda", device)

    def gen(stream: int) -> "torch.Generator":
        g = torch.Generator(device=dev)
        g.manual_seed((seed * 1_000_003 + stream) & 0x7FFF_FFFF_FFFF_FFFF)
        return g

    cen = torch.randn((centres, d), generator=gen(0), device=dev, dtype=torch.float32)

    def draw(count: int, g: "torch.Generator") -> "torch.Tensor":
        lab = torch.randint(0, centres, (count,), generator=g, device=dev)
        out = torch.randn((count, d), generator=g, device=dev, dtype=torch.float32)
        out.mul_(sigma).add_(cen.index_select(0, lab))
        return out

    def chunks():
        for i, s in enumerate(range(0, n, chunk)):
            yield draw(min(chunk, n - s), gen(1000 + i))

    queries = draw(nq, gen(1)).cpu().numpy()
    return cen, chunks(), queries
