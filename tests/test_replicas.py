"""Host logic of the multi-GPU path (ai_b200/replicas.py) on CPU: the
length-sorted, cost-balanced split of a batch over ranks, and the gather
of the embeddings onto rank 0 in the caller's order, run as world-size-2
`gloo` process groups with a stand-in model (no GPU needed). A rank that
fails before the gather makes rank 0's gather end with an error, not hang.
"""
import datetime
import os
import socket

import numpy as np
import pytest

from ai_b200 import replicas as R


class FakeModel:
    """Deterministic embeddings from the token ids (what Model.embed_ids
    returns in shape and order)."""

    def __init__(self, dim=16):
        self.dim = dim

    def Dim(self):
        return self.dim

    def embed_ids(self, seqs, dim=None):
        dim = dim or self.dim
        out = []
        for s in seqs:
            v = np.zeros(dim, np.float32)
            for j, t in enumerate(s):
                v[(t + j) % dim] += 1.0 + (t % 7)
            v[0] += len(s)
            out.append(v / max(1.0, float(np.linalg.norm(v))))
        return out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _seqs(n, seed):
    rng = np.random.default_rng(seed)
    lens = rng.integers(0, 300, n)
    return [list(rng.integers(3, 1000, int(L))) for L in lens]


def test_plan_slices_cover_each_sequence_once_in_sorted_runs():
    rng = np.random.default_rng(1)
    for world in (1, 2, 3, 4, 8):
        for n in (0, 1, 3, 7, 64, 257):
            lengths = rng.integers(0, 2048, n)
            sl = R.plan_slices(lengths, world)
            assert len(sl) == world
            allidx = np.concatenate(sl) if n else np.zeros(0, np.int64)
            assert sorted(allidx.tolist()) == list(range(n))
            order = np.argsort(lengths, kind="stable")
            assert np.array_equal(allidx, order)  # contiguous runs of the sorted batch


def test_plan_slices_balance_cost():
    rng = np.random.default_rng(2)
    lengths = rng.integers(1, 2048, 1000)
    cost = R.sequence_cost(lengths)
    for world in (2, 4, 8):
        sl = R.plan_slices(lengths, world)
        per = np.array([cost[s].sum() for s in sl])
        assert per.max() <= cost.sum() / world + cost.max() + 1e-9


def test_plan_slices_small_batch_leaves_ranks_idle():
    sl = R.plan_slices([5, 9], 4)
    assert sum(len(s) for s in sl) == 2
    assert [len(s) for s in sl].count(0) == 2


def _worker(rank, world, port, seqs, result_path, fail_rank):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=4))
    try:
        if rank == fail_rank:
            raise RuntimeError("rank failed before the gather")
        out = R.embed_replicated(FakeModel(), seqs)
        if rank == 0:
            np.save(result_path, out)
    except Exception as e:  # noqa: BLE001 - report to the parent
        with open(result_path + f".err{rank}", "w") as f:
            f.write(type(e).__name__ + ": " + str(e))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, seqs, tmp_path, fail_rank=-1):
    import torch.multiprocessing as mp

    path = str(tmp_path / "emb.npy")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, seqs, path, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    hung = [p for p in procs if p.exitcode is None]
    for p in hung:
        p.terminate()  # this test's own child process
        p.join(10)
    assert not hung, "a rank did not finish"
    return path


@pytest.mark.parametrize("n", [1, 5, 33])
def test_world2_gather_restores_caller_order(tmp_path, n):
    seqs = _seqs(n, seed=n)
    path = _run(2, seqs, tmp_path)
    assert not any(f.name.startswith("emb.npy.err") for f in tmp_path.iterdir()), \
        [f.read_text() for f in tmp_path.iterdir() if ".err" in f.name]
    got = np.load(path)
    want = np.stack(FakeModel().embed_ids(seqs))
    assert np.array_equal(got, want)


def test_world2_failed_rank_ends_gather_with_error(tmp_path):
    seqs = _seqs(8, seed=3)
    _run(2, seqs, tmp_path, fail_rank=1)
    err1 = (tmp_path / "emb.npy.err1").read_text()
    assert "rank failed" in err1
    # rank 0 saw the peer gone (connection closed or the collective timed out)
    assert (tmp_path / "emb.npy.err0").exists()
    assert not (tmp_path / "emb.npy").exists()
