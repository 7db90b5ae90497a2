"""Bounded device waits that run out: with a short pipeline-wait limit
(fg_set_wait_limit), a GEMM on SM pairs and the tensor-core attention give
up their waits, drain their own copies and MMAs, free their tensor memory
and return; fg_synchronize reports FG_ETIMEOUT once and clears the record;
and the next call with the default limit gives the same result, bit for
bit, as before. No fault is injected: the limit (1 µs) is shorter than
waits the kernels have anyway, so those run out on their own and the
context stays usable. A wait checks its limit between tries of the
barrier, and a try holds the thread about 4 µs on B200, so the cases are
chosen for waits longer than that: a K = 8192 main loop under the GEMM
epilogue; for attention, a first wave of 148 CTAs whose Q and K come from
HBM together (operands larger than L2) before the first score tile.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LIMIT_NS = 1000


def _expect_timeout(run):
    from ai_b200 import _lib

    lib = _lib.lib()
    _lib.check(lib.fg_synchronize(0))
    try:
        _lib.check(lib.fg_set_wait_limit(0, LIMIT_NS))
        run()
        rc = lib.fg_synchronize(0)
        msg = lib.fg_last_error().decode()
    finally:
        _lib.check(lib.fg_set_wait_limit(0, 0))
    assert rc == _lib.FG_ETIMEOUT, rc
    assert "wait gave up" in msg
    assert lib.fg_synchronize(0) == _lib.FG_OK


@pytest.mark.parametrize("precision", [0, 1])
def test_gemm_wait_limit_reports_timeout_and_recovers(cuda, precision):
    import torch

    from ai_b200 import tensor as T

    g = torch.Generator(device=cuda).manual_seed(5)
    a = torch.randn(512, 8192, generator=g, device=cuda)
    w = torch.randn(768, 8192, generator=g, device=cuda).t()
    ref = T.MatMul(a, w, precision=precision)
    torch.cuda.synchronize()
    _expect_timeout(lambda: T.MatMul(a, w, precision=precision))
    again = T.MatMul(a, w, precision=precision)
    torch.cuda.synchronize()
    assert torch.equal(again, ref)


def test_attention_wait_limit_reports_timeout_and_recovers(cuda):
    import torch

    from ai_b200 import tensor as T

    g = torch.Generator(device=cuda).manual_seed(6)
    B = 128  # 1536 CTAs; split q, k and vᵀ are 168 MB, more than L2 holds
    q = torch.randn(B, 3, 512, 256, generator=g, device=cuda)
    k = torch.randn(B, 1, 512, 256, generator=g, device=cuda)
    v = torch.randn(B, 1, 512, 256, generator=g, device=cuda)
    lens = torch.full((B,), 512, dtype=torch.int32)
    lens[1] = 300
    ref = T.AttentionScaled(q, k, v, lens, 0, 1 / 16)
    torch.cuda.synchronize()
    _expect_timeout(lambda: T.AttentionScaled(q, k, v, lens, 0, 1 / 16))
    again = T.AttentionScaled(q, k, v, lens, 0, 1 / 16)
    torch.cuda.synchronize()
    assert torch.equal(again, ref)


def test_model_wait_limit_reports_timeout_and_recovers(cuda):
    """The whole encoder forward under the short limit: fg_model_check
    reports the timeout; the next forward is bitwise the first."""
    from ai_b200 import _lib, gemma
    from ai_b200 import synthetic as S

    cfg = S.small_config(layers=2, vocab=2048)
    w = S.make_weights(cfg, seed=0)
    ids = S.make_ids(4, 512, 1, cfg["vocab_size"])
    lengths = np.full(4, 512, np.int32)
    model = gemma.from_synthetic(cfg, w, device=0, max_batch_tokens=2048)
    try:
        ref = model.embed_padded(ids, lengths)
        lib = _lib.lib()
        try:
            _lib.check(lib.fg_set_wait_limit(0, LIMIT_NS))
            with pytest.raises(_lib.FGError) as e:
                model.embed_padded(ids, lengths)
                model.check()
        finally:
            _lib.check(lib.fg_set_wait_limit(0, 0))
        assert e.value.code == _lib.FG_ETIMEOUT
        assert lib.fg_synchronize(0) == _lib.FG_OK
        again = model.embed_padded(ids, lengths)
        assert np.array_equal(again, ref)
    finally:
        model.close()
