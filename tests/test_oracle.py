"""The CPU oracle pinned against the reference's own known-answer tests and
properties (CPU only).  These run on every host; they are what makes the
oracle trustworthy as the checker for the GPU parity tests."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as orc


def f32(x):
    return np.asarray(x, dtype=np.float32)


# ---- known answers ----------------------------------------------------------

@pytest.mark.parametrize("name", ["adc_table_dsub1", "adc_table_dsub3"])
def test_adc_table_known_answers(kats, name):
    kat = kats[name]
    table = orc.adc_table(kat["query"], kat["num_codebooks"], kat["codebook_size"], kat["codebooks"])
    assert table.tolist() == kat["expected_table"]


def test_finish_top_k_keeps_sorted_prefix(kats):
    kat = kats["finish_top_k_sorted_prefix"]
    ids, dists = orc.finish_top_k(kat["ids"], kat["dists"], kat["k"])
    assert ids.tolist() == kat["expected_ids"]
    assert dists.tolist() == kat["expected_dists"]


def test_finish_top_k_short_inputs(kats):
    for case in kats["finish_top_k_short_inputs"]["cases"]:
        ids, dists = orc.finish_top_k(case["ids"], case["dists"], case["k"])
        assert ids.tolist() == case["expected_ids"]
        assert dists.tolist() == case["expected_dists"]


def test_fastscan_u16_accumulator_exact_at_limit(kats):
    kat = kats["fastscan_u16_limit"]
    m, n = kat["num_codebooks"], kat["num_vectors"]
    packed = orc.pack_4bit(np.zeros(n * m, np.uint8), n, m)
    lut_q = np.full(m * 16, kat["lut_value"], np.uint8)
    acc = orc.fastscan_block(packed[: m * 16], lut_q, m)
    assert (acc == kat["expected_sum"]).all()


def test_fastscan_refuses_past_the_limit(kats):
    kat = kats["fastscan_over_limit"]
    m, n = kat["num_codebooks"], kat["num_vectors"]
    packed = orc.pack_4bit(np.zeros(n * m, np.uint8), n, m)
    with pytest.raises(OverflowError, match="overflow"):
        orc.fastscan_batch_flat(packed, n, m, np.full(m * 16, kat["lut_value"], np.float32))


def test_adc_distance_basic(kats):
    kat = kats["adc_distance_basic"]
    m, ks = kat["num_codebooks"], kat["codebook_size"]
    lut = (np.arange(m * ks, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    got = orc.distance_with_table(lut, m, ks, kat["codes"])
    assert abs(got - kat["expected"]) < kat["tolerance"]


def _lut_4bit(m):
    return (np.arange(m * 16, dtype=np.float32) * np.float32(0.5)).astype(np.float32)


def test_quantize_lut_range(kats):
    kat = kats["quantize_lut_range"]
    lut = _lut_4bit(kat["num_codebooks"])
    q, scale, offset = orc.quantize_lut_flat(lut, kat["num_codebooks"])
    assert q[0] == kat["expected_first"] and q[-1] == kat["expected_last"]
    recon = q.astype(np.float32) * np.float32(scale) + np.float32(offset)
    assert (np.abs(recon - lut) <= scale / 2 + 1e-5).all()


def test_packed_4bit_roundtrip(kats):
    kat = kats["packed_4bit_roundtrip"]
    n, m = kat["num_vectors"], kat["num_codebooks"]
    codes = np.array([[(i + j) % 16 for j in range(m)] for i in range(n)], np.uint8)
    packed = orc.pack_4bit(codes, n, m)
    assert packed.size == kat["expected_blocks"] * m * 16
    for i in range(n):
        for j in range(m):
            byte = packed[j * 16 + (i % 16)]
            code = byte & 0x0F if i < 16 else byte >> 4
            assert code == codes[i, j]


def _odd_lut(m, ks):
    i = np.arange(m * ks)
    return (np.float32(0.25) + ((i * 7919) % 1009).astype(np.float32) * np.float32(0.003)).astype(np.float32)


def test_adc_batch_matches_sequential_sum_at_odd_sizes(kats):
    kat = kats["adc_odd_sizes"]
    for ks in kat["codebook_sizes"]:
        for m in kat["num_codebooks"]:
            lut = _odd_lut(m, ks)
            for n in kat["n_candidates"]:
                codes = ((np.arange(n * m) * 131 + 17) % ks).astype(np.uint8)
                got = orc.adc_batch(codes, m, lut, ks)
                want = []
                for row in codes.reshape(n, m):
                    s = np.float32(0.0)
                    for j, c in enumerate(row.tolist()):
                        s = np.float32(s + lut[j * ks + c])
                    want.append(s)
                assert got.tolist() == [float(w) for w in want]


def test_fastscan_within_quantisation_error():
    # pq_simd.rs:1206-1318: |fastscan - scalar| <= M * scale / 2 + 1e-3
    for m, n, gen in [(8, 100, lambda i: (i * 7 + 3) % 16), (4, 100, lambda i: (i * 11 + 5) % 16),
                      (5, 40, lambda i: i % 16)]:
        lut = _lut_4bit(m)
        codes = np.array([gen(i) for i in range(n * m)], np.uint8).reshape(n, m)
        packed = orc.pack_4bit(codes, n, m)
        got = orc.fastscan_batch_flat(packed, n, m, lut)
        _, scale, _ = orc.quantize_lut_flat(lut, m)
        scalar = np.array([sum(float(lut[j * 16 + c]) for j, c in enumerate(r)) for r in codes])
        assert (np.abs(got - scalar) <= m * scale * 0.5 + 1e-3).all()


# ---- properties of pq.rs (ported proptests) -----------------------------------

def _lcg_values(count, seed):
    """pq.rs:372-382 next_value: LCG uniform values in [-1, 1)."""
    state = (seed | 1) & 0xFFFFFFFFFFFFFFFF
    out = np.empty(count, np.float32)
    for i in range(count):
        state = (state * 6364136223846793005 + 1) & 0xFFFFFFFFFFFFFFFF
        out[i] = np.float32(np.float32(state >> 33) / np.float32(1 << 31)) - np.float32(1.0)
    return out


@pytest.mark.parametrize("seed", range(12))
def test_adc_table_sum_equals_squared_l2_to_reconstruction(seed):
    rng = np.random.default_rng(seed)
    m = int(rng.integers(1, 5))
    dsub = int(rng.integers(1, 11))
    ks = int(rng.integers(4, 17))
    d = m * dsub
    cb = _lcg_values(m * ks * dsub, 1000 + seed)
    q = _lcg_values(d, 2000 + seed)
    codes = rng.integers(0, ks, size=m).astype(np.uint8)
    table = orc.adc_table(q, m, ks, cb)
    acc = orc.distance_with_table(table, m, ks, codes)
    recon = orc.pq_reconstruct(codes, d, m, ks, cb)
    exact = float(np.sum((q.astype(np.float64) - recon.astype(np.float64)) ** 2))
    assert abs(acc - exact) <= 1e-4 * max(abs(exact), 1.0)


@pytest.mark.parametrize("seed", range(12))
def test_encode_is_the_argmin_and_decode_is_a_fixed_point(seed):
    rng = np.random.default_rng(100 + seed)
    m = int(rng.integers(1, 5))
    dsub = int(rng.integers(1, 11))
    ks = int(rng.integers(4, 17))
    d = m * dsub
    cb = _lcg_values(m * ks * dsub, 3000 + seed)
    x = _lcg_values(d, 4000 + seed)
    codes = orc.pq_quantize(x.reshape(1, -1), m, ks, cb)[0]
    recon = orc.pq_reconstruct(codes, d, m, ks, cb)
    for j in range(m):
        sub = x[j * dsub:(j + 1) * dsub].astype(np.float64)
        observed = np.sum((sub - recon[j * dsub:(j + 1) * dsub]) ** 2)
        for c in range(ks):
            cw = cb[(j * ks + c) * dsub:(j * ks + c + 1) * dsub].astype(np.float64)
            assert observed <= np.sum((sub - cw) ** 2) * (1 + 1e-5) + 1e-6
    again = orc.pq_reconstruct(orc.pq_quantize(recon.reshape(1, -1), m, ks, cb)[0], d, m, ks, cb)
    assert np.array_equal(again, recon)


def test_total_order_key_matches_total_cmp():
    vals = [float("-inf"), -1.0, -0.0, 0.0, 1e-30, 1.0, float("inf")]
    keys = [orc.total_order_key(v) for v in vals]
    assert keys == sorted(keys) and len(set(keys)) == len(keys)


def _seq_dot(a, b):
    # simd.rs:90-92 (fallback `dot`): products rounded to f32, summed in index order
    s = np.float32(0.0)
    for x, y in zip(a, b):
        s = np.float32(s + np.float32(x * y))
    return s


@pytest.mark.parametrize("k", [1, 10, 57, 300])
def test_flat_search_ip_is_the_sequential_exhaustive_scan(k):
    # distance.rs:125-130 (-dot) over every row, ranked by total_cmp as the
    # ground truth of evaluation.rs:250-268 does, ties to the lower row, rows
    # past n padded with 0xffffffff / +inf
    rng = np.random.default_rng(k)
    n, d = 200, 13
    db = rng.standard_normal((n, d)).astype(np.float32)
    db[50:60] = db[7]          # ties
    db[120] = 0.0              # a zero row: distance -0.0
    q = rng.standard_normal((4, d)).astype(np.float32)
    q[3] = db[7] * np.float32(2.0)
    ids, dist, cnt = orc.flat_search_ip(db, q, k)
    for i in range(q.shape[0]):
        ds = [np.float32(-_seq_dot(q[i], db[r])) for r in range(n)]
        order = sorted(range(n), key=lambda r: (orc.total_order_key(float(ds[r])), r))
        want = order[:k]
        assert cnt[i] == min(k, n)
        assert list(ids[i, : min(k, n)]) == want
        assert np.array_equal(dist[i, : min(k, n)].view(np.uint32),
                              np.array([ds[r] for r in want], np.float32).view(np.uint32))
        assert (ids[i, n:] == 0xFFFFFFFF).all() and np.isinf(dist[i, n:]).all()


# ---- index-level properties of search.rs ----------------------------------------

def _small_index(n=256, d=16, L=32, M=4, ks=16, nprobe=32, seed=7):
    rng = np.random.default_rng(seed)
    x = rng.random((n, d), dtype=np.float32)
    xn = orc.normalize(x)
    cent = xn[rng.choice(n, L, replace=False)]
    cb = rng.standard_normal((M, ks, d // M)).astype(np.float32) * np.float32(0.1)
    ix = orc.OracleIndex(d, L, M, ks, nprobe)
    ix.set_trained(cent, cb)
    ix.add(np.arange(60_000, 60_000 + n, dtype=np.uint32), x)
    ix.finalize()
    return ix, x, xn, rng


def test_full_probe_equals_exhaustive_scan_over_reconstructions():
    # search.rs:2589-2645
    ix, x, xn, rng = _small_index()
    q = orc.normalize(rng.random((1, 16), dtype=np.float32))[0]
    ids, dists, cnt = ix.search_batch(q.reshape(1, -1), 10, nprobe=32)
    exact = []
    for i in range(len(ix)):
        v = ix.reconstruct(i)
        dd = np.float32(0.0)
        for a, b in zip(q, v):
            dd = np.float32(dd + np.float32(np.float32(a - b) * np.float32(a - b)))
        exact.append((orc.total_order_key(float(dd)), i))
    exact.sort()
    assert ids[0].tolist() == [60_000 + i for _, i in exact[:10]]


def test_adc_distance_matches_exact_l2_to_reconstruction():
    # search.rs:3294-3333: worst relative error <= 1e-3
    ix, x, xn, rng = _small_index(n=512, L=8, ks=256)  # 8-bit: exact table sums
    q = xn[5]
    ids, dists, cnt = ix.search_batch(q.reshape(1, -1), 50, nprobe=3)
    for doc, dist in zip(ids[0][: cnt[0]], dists[0][: cnt[0]]):
        v = ix.reconstruct(int(doc) - 60_000)
        exact = float(np.sum((q.astype(np.float64) - v) ** 2))
        assert abs(dist - exact) <= 1e-3 * max(exact, 1e-6) + 1e-6


def test_query_scale_invariance_and_padding():
    # correctness_regression tests_feature_gated.rs:39-...; test_python.py:555
    ix, x, xn, rng = _small_index()
    q = rng.random((3, 16), dtype=np.float32)
    a = ix.search_batch(q, 10, nprobe=8)
    b = ix.search_batch(q * np.float32(4.0), 10, nprobe=8)
    assert np.array_equal(a[0], b[0])
    ids, dists, cnt = ix.search_batch(q, 300, nprobe=32)
    assert (cnt == 256).all()
    assert (ids[:, 256:] == 0xFFFFFFFF).all() and np.isinf(dists[:, 256:]).all()


# ---- OPQ rotation (opq.rs) ---------------------------------------------------

def test_opq_matrix_vector_multiply(kats):
    for case in kats["opq_matrix_vector_multiply"]["cases"]:
        got = orc.rotate(case["matrix"], case["vector"])
        np.testing.assert_allclose(got, case["expected"], atol=case["tolerance"], rtol=0)


def test_opq_identity_rotation_is_a_no_op(kats):
    kat = kats["opq_identity_rotation"]
    v = np.asarray(kat["vector"], np.float32)
    assert np.array_equal(orc.rotate(np.eye(kat["dimension"]), v), v)


def test_opq_encode_rotates_and_decode_applies_the_transpose(kats):
    kat = kats["opq_decode_applies_transpose"]
    d, m, ks = kat["dimension"], kat["num_codebooks"], kat["codebook_size"]
    rot = np.asarray(kat["rotation"], np.float32).reshape(d, d)
    g = np.random.default_rng(11)
    cb = g.uniform(-1, 1, (m, ks, d // m)).astype(np.float32)
    x = g.uniform(-1, 0.9, (5, d)).astype(np.float32)
    ix = orc.OracleIndex(d, 1, m, ks, 1)
    ix.set_trained(np.zeros((1, d), np.float32), cb)
    ix.set_rotation(rot)
    ix.add(np.arange(5, dtype=np.uint32), x)
    ix.finalize()
    xn = ix.vectors()
    for i in range(5):
        codes = ix.codes()[i]
        # encoding quantises the rotated residual (opq.rs:107-113)
        assert np.array_equal(codes, orc.pq_quantize(orc.rotate(rot, xn[i]), m, ks, cb)[0])
        rotated_space = orc.pq_reconstruct(codes, d, m, ks, cb)
        decoded = ix.reconstruct(i)
        expected = orc.rotate(rot, rotated_space, transpose=True)
        np.testing.assert_allclose(decoded, expected, atol=kat["tolerance"], rtol=0)
        err = np.linalg.norm(xn[i] - decoded)
        forgot = np.linalg.norm(xn[i] - rotated_space)
        assert err <= forgot + 1e-6
