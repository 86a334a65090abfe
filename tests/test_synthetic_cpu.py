"""The device-side generator of the 1e8-vector configuration, run on the CPU
at a reduced size: chunks are a pure function of (seed, chunk index), the
queries of the seed, and rows follow the configuration's mixture."""
from __future__ import annotations

import numpy as np
import torch

from vicinity_b200.synthetic import CONFIGS, device_mixture


def _draw(seed=0, n=10_000, nq=64, chunk=4096):
    cen, chunks, q = device_mixture(4, seed=seed, device="cpu", n=n, nq=nq, chunk=chunk)
    return cen, [c.clone() for c in chunks], q


def test_chunks_cover_n_rows_in_order():
    cen, chunks, q = _draw()
    cfg = CONFIGS[4]
    assert cen.shape == (cfg["centres"], cfg["d"])
    assert [c.shape[0] for c in chunks] == [4096, 4096, 1808]
    assert all(c.dtype == torch.float32 and c.shape[1] == cfg["d"] for c in chunks)
    assert q.shape == (64, cfg["d"]) and q.dtype == np.float32


def test_same_seed_same_data_other_seed_other_data():
    _, a, qa = _draw(seed=0)
    _, b, qb = _draw(seed=0)
    _, c, qc = _draw(seed=1)
    assert all(torch.equal(x, y) for x, y in zip(a, b)) and np.array_equal(qa, qb)
    assert not torch.equal(a[0], c[0]) and not np.array_equal(qa, qc)


def test_each_chunk_depends_only_on_its_index():
    # a rank that regenerates the database draws the same rows whatever the
    # total size, so chunk i is identical for n = 10,000 and n = 20,000
    _, a, _ = _draw(n=10_000)
    _, b, _ = _draw(n=20_000)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_rows_are_a_centre_plus_sigma_noise():
    cen, chunks, _ = _draw(n=4096, chunk=4096)
    x = chunks[0]
    # every row's nearest centre is within the noise radius: sigma * sqrt(d) ~ 1.47
    dist = torch.cdist(x[:256], cen).min(dim=1).values
    sigma, d = CONFIGS[4]["sigma"], CONFIGS[4]["d"]
    assert float(dist.max()) < 2.0 * sigma * d ** 0.5
    assert abs(float(dist.mean()) - sigma * d ** 0.5) < 0.1
