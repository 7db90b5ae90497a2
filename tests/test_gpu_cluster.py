"""The cluster package on the device (ai_b200/csrc/fg_cluster.cu through
ai_b200.cluster) against the oracle (oracle/cluster.py) on the same inputs.

Bar: discrete results identical (assignments, sizes, iteration counts,
nearest indices wherever the best two similarities are more than 1e-5
apart); similarities and centres within 1e-5 (split-TF32 products against
float64 ones)."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _planted(n, d, groups, seed, noise=0.05):
    from oracle import cluster as OC

    rng = np.random.default_rng(seed)
    centres = OC.normalize(rng.standard_normal((groups, d)).astype(np.float32))
    truth = np.arange(n) % groups
    data = centres[truth] + (rng.standard_normal((n, d)) * noise).astype(np.float32)
    return OC.normalize(data.astype(np.float32)), truth


def _dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda)


def test_normalize_rows(cuda):
    from ai_b200 import cluster as CL
    from oracle import cluster as OC

    x = np.random.default_rng(1).standard_normal((37, 100)).astype(np.float32) * 3
    x[5] = 0
    got = CL.Normalize(_dev(x, cuda)).cpu().numpy()
    assert np.all(got[5] == 0)
    np.testing.assert_allclose(got, OC.normalize(x), atol=1e-6, rtol=0)
    np.testing.assert_allclose(np.linalg.norm(np.delete(got, 5, 0).astype(np.float64), axis=1), 1, atol=1e-6)


@pytest.mark.parametrize("q,n,d", [(5, 7, 64), (33, 1001, 768), (1, 1, 4)])
def test_similarities_vs_float64(cuda, q, n, d):
    """cluster_test.go:112-129: shape [q, n], each entry the cosine."""
    from ai_b200 import cluster as CL
    from oracle import cluster as OC

    rng = np.random.default_rng(q * 1000 + n)
    qs = OC.normalize(rng.standard_normal((q, d)).astype(np.float32))
    ds = OC.normalize(rng.standard_normal((n, d)).astype(np.float32))
    s = CL.Similarities(_dev(qs, cuda), _dev(ds, cuda))
    assert tuple(s.shape) == (q, n)
    want = qs.astype(np.float64) @ ds.astype(np.float64).T
    assert np.abs(s.cpu().numpy() - want).max() <= TOL


def _check_nearest(idx, sim, x, c):
    from oracle import cluster as OC

    want_i, want_s = OC.nearest(x, c)
    full = x.astype(np.float64) @ c.astype(np.float64).T
    top2 = np.sort(full, axis=1)[:, -2:] if c.shape[0] > 1 else np.hstack([full - 1, full])
    clear = (top2[:, 1] - top2[:, 0]) > TOL
    idx = np.asarray(idx)
    assert np.array_equal(idx[clear], want_i[clear])
    # where the best two are within the tolerance either is a correct answer
    assert np.all(full[np.arange(len(idx)), idx] >= top2[:, 1] - TOL)
    assert np.abs(np.asarray(sim, np.float64) - full[np.arange(len(idx)), idx]).max() <= TOL


def test_nearest_vs_oracle(cuda):
    from ai_b200 import cluster as CL
    from oracle import cluster as OC

    rng = np.random.default_rng(4)
    x = OC.normalize(rng.standard_normal((3000, 96)).astype(np.float32))
    c = OC.normalize(rng.standard_normal((13, 96)).astype(np.float32))
    idx, sim = CL.Nearest(_dev(x, cuda), _dev(c, cuda))
    _check_nearest(idx, sim, x, c)
    # ties keep the first centre
    c2 = np.vstack([c[:3], c[:3]])
    idx, _ = CL.Nearest(_dev(x[:50], cuda), _dev(c2, cuda))
    assert max(idx) < 3


def test_nearest_50000_rows_40_centres(cuda):
    """The size of the reference's TestNearestSpeed (cluster_test.go:65-79,
    bound 200 ms on a CPU), with parity on a sample of rows."""
    import torch

    from ai_b200 import cluster as CL
    from oracle import cluster as OC

    g = torch.Generator(device=cuda).manual_seed(5)
    x = CL.Normalize(torch.randn(50000, 768, generator=g, device=cuda))
    c = CL.Normalize(torch.randn(40, 768, generator=g, device=cuda))
    CL.Nearest(x, c)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    idx, sim = CL.Nearest(x, c)
    el = time.perf_counter() - t0
    print(f"Nearest 50000 x 768 against 40 centres: {el * 1e3:.2f} ms (host call, results on the host)")
    assert el < 0.2
    rows = np.arange(0, 50000, 97)
    xs = x[rows].cpu().numpy()
    _check_nearest(np.asarray(idx)[rows], np.asarray(sim)[rows], xs, c.cpu().numpy())


@pytest.mark.parametrize("n,d,groups,k,iters,seed", [(600, 64, 3, 3, 20, 7), (3000, 96, 12, 12, 30, 11),
                                                     (2000, 768, 8, 5, 10, 3), (500, 32, 4, 9, 15, 1)])
def test_kmeans_matches_oracle(cuda, n, d, groups, k, iters, seed):
    from ai_b200 import cluster as CL
    from oracle import cluster as OC

    x, truth = _planted(n, d, groups, seed=seed + 100)
    want = OC.kmeans(x, k, iters, seed)
    got = CL.KMeans(_dev(x, cuda), k, iters, seed)
    assert got.Iterations == want.iterations
    assert np.array_equal(np.asarray(got.Assignment), want.assignment)
    assert np.array_equal(np.asarray(got.Sizes), want.sizes)
    assert np.abs(np.asarray(got.Similarity) - want.similarity).max() <= TOL
    assert np.abs(got.Centres.cpu().numpy() - want.centres).max() <= TOL
    assert abs(got.Inertia() - want.inertia()) <= TOL
    again = CL.KMeans(_dev(x, cuda), k, iters, seed)
    assert again.Assignment == got.Assignment and np.array_equal(again.Centres.cpu().numpy(),
                                                                   got.Centres.cpu().numpy())


def test_kmeans_recovers_planted_clusters(cuda):
    """cluster_test.go:29-63 on the device."""
    from ai_b200 import cluster as CL
    from oracle import cluster as OC

    x, truth = _planted(600, 64, 3, seed=1)
    res = CL.KMeans(_dev(x, cuda), 3, 20, 7)
    mapping = {}
    for i, a in enumerate(res.Assignment):
        assert mapping.setdefault(int(truth[i]), a) == a
    assert len(set(mapping.values())) == 3
    assert min(res.Similarity) >= 0.85
    idx, sim = CL.Nearest(_dev(x[:3], cuda), res.Centres)
    assert idx == res.Assignment[:3] and min(sim) >= 0.85
    rnd = OC.normalize(np.random.default_rng(5).standard_normal((1, 64)).astype(np.float32))
    assert CL.Nearest(_dev(rnd, cuda), res.Centres)[1][0] <= 0.6
    assert res.Inertia() <= 0.1


def test_kmeans_empty_centres_and_zero_iterations(cuda):
    from ai_b200 import cluster as CL
    from oracle import cluster as OC

    x = np.zeros((40, 8), np.float32)
    x[np.arange(40), np.arange(40) % 4] = 1
    for iters in (0, 1, 5):
        want = OC.kmeans(x, 6, iters, 3)
        got = CL.KMeans(_dev(x, cuda), 6, iters, 3)
        assert got.Iterations == want.iterations
        assert np.array_equal(np.asarray(got.Assignment), want.assignment)
        assert np.array_equal(np.asarray(got.Sizes), want.sizes)
        assert np.array_equal(np.asarray(got.Similarity, np.float32), want.similarity)
        assert np.array_equal(got.Centres.cpu().numpy(), want.centres)


def test_kmeans_bad_k(cuda):
    from ai_b200 import cluster as CL

    x = _dev(np.eye(4, dtype=np.float32), cuda)
    for k in (0, 5):
        with pytest.raises(CL.ClusterError):
            CL.KMeans(x, k, 3, 1)
