"""The cluster package's host side, no GPU: the oracle (oracle/cluster.py)
against the properties the reference's own tests assert
(cluster/cluster_test.go), the Go PCG restatement's arithmetic, and the
host-only Cosine of ai_b200.cluster."""
import math

import numpy as np
import pytest

from oracle import cluster as OC


def planted(n, d, seed, noise=0.05):
    """Rows around three unit vectors (the shape of cluster_test.go:14-27's
    planted data, drawn with numpy)."""
    rng = np.random.default_rng(seed)
    centres = OC.normalize(rng.standard_normal((3, d)).astype(np.float32))
    truth = np.arange(n) % 3
    data = centres[truth] + (rng.standard_normal((n, d)) * noise).astype(np.float32)
    return OC.normalize(data.astype(np.float32)), truth


def test_go_rand_stream_shape():
    r = OC.GoRand(1, 2)
    a = [r.uint64() for _ in range(4)]
    r2 = OC.GoRand(1, 2)
    assert a == [r2.uint64() for _ in range(4)]
    assert len(set(a)) == 4 and all(0 <= v < 2**64 for v in a)
    r = OC.GoRand(7, 7 ^ 0x9E3779B97F4A7C15)
    for n in (1, 2, 3, 600, 1 << 20, (1 << 40) + 3):
        for _ in range(20):
            assert 0 <= r.intn(n) < n
    fs = [r.float64() for _ in range(2000)]
    assert all(0.0 <= f < 1.0 for f in fs)
    assert 0.45 < sum(fs) / len(fs) < 0.55
    with pytest.raises(ValueError):
        r.intn(0)


def test_go_rand_state_is_the_128_bit_lcg():
    # one step by hand: state' = state * mul + inc (mod 2^128), DXSM on state'
    r = OC.GoRand(3, 5)
    st = ((3 << 64 | 5) * OC.PCG_MUL + OC.PCG_INC) % (1 << 128)
    hi, lo = st >> 64, st & OC.M64
    h = hi ^ (hi >> 32)
    h = (h * OC.DXSM_MUL) % (1 << 64)
    h ^= h >> 48
    h = (h * (lo | 1)) % (1 << 64)
    assert r.uint64() == h
    assert (r.hi, r.lo) == (hi, lo)


def test_kmeans_recovers_planted_clusters():
    """cluster_test.go:29-63 on the oracle."""
    x, truth = planted(600, 64, seed=1)
    res = OC.kmeans(x, 3, 20, 7)
    mapping = {}
    for i, a in enumerate(res.assignment):
        assert mapping.setdefault(int(truth[i]), int(a)) == a, "group split"
    assert len(set(mapping.values())) == 3, "groups merged"
    assert res.similarity.min() >= 0.85
    idx, sim = OC.nearest(x[:3], res.centres)
    assert list(idx) == list(res.assignment[:3]) and sim.min() >= 0.85
    rnd = OC.normalize(np.random.default_rng(5).standard_normal((1, 64)).astype(np.float32))
    assert OC.nearest(rnd, res.centres)[1][0] <= 0.6
    assert res.inertia() <= 0.1
    assert res.sizes.sum() == 600 and 1 <= res.iterations <= 20


def test_kmeans_rejects_bad_k():
    x, _ = planted(10, 8, seed=2)
    for k in (0, -1, 11):
        with pytest.raises(ValueError, match="k must be between 1"):
            OC.kmeans(x, k, 5, 1)


def test_kmeans_restarts_empty_centres():
    # one-hot rows: every similarity is exactly 0 or 1, so the seeding runs
    # out of distance after 4 centres and repeats row 0; the repeats are
    # empty after the argmax (first maximum) and restart on row 0
    x = np.zeros((40, 8), np.float32)
    x[np.arange(40), np.arange(40) % 4] = 1
    res = OC.kmeans(x, 6, 5, 3)
    assert res.sizes.sum() == 40
    assert sorted(res.sizes.tolist())[:2] == [0, 0]
    assert res.iterations == 2


def test_argmax_first_maximum_and_nan():
    s = np.array([[1, 3, 3, 2], [np.nan, 5, 6, 1], [1, np.nan, 0, 1], [-np.inf, -np.inf, -np.inf, -np.inf]],
                 np.float32)
    assert OC.argmax_rows(s).tolist() == [1, 0, 0, 0]


def test_cosine_known_answers():
    """cluster_test.go:81-110 on the host function and the oracle."""
    from ai_b200 import cluster as CL

    for cos in (CL.Cosine, OC.cosine):
        a = [1, 2, 3, 4]
        assert abs(cos(a, a) - 1) <= 1e-6
        assert abs(cos(a, [-1, -2, -3, -4]) + 1) <= 1e-6
        assert cos([1, 0], [0, 1]) == 0
        assert cos(a, [0, 0, 0, 0]) == 0
        assert cos([], []) == 0
        rng = np.random.default_rng(9)
        for n in (1, 7, 8, 9, 768, 1001):
            x = rng.standard_normal(n).astype(np.float32)
            y = rng.standard_normal(n).astype(np.float32)
            xd, yd = x.astype(np.float64), y.astype(np.float64)
            want = (xd @ yd) / math.sqrt((xd @ xd) * (yd @ yd))
            assert abs(cos(x, y) - want) <= 1e-5
        with pytest.raises(ValueError):
            cos([1, 2], [1, 2, 3])
