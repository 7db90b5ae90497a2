"""fg_embed_many_multi: (*Model).Embed (models/gemma/embed.go:15-80) over
several GPUs of one process, one model per GPU, one host thread per model.
The cost-balanced contiguous slices of the length-sorted batch
(fg_plan_split) are each embedded by fg_embed_many, so every embedding is
bitwise what fg_embed_many gives for that slice alone, and lands in the
caller's order. Run with two models on one GPU (two threads driving one
device) everywhere, and with one model per GPU where the box has more.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _models(devices, cfg, w, budget):
    from ai_b200 import gemma

    return [gemma.from_synthetic(cfg, w, device=d, max_batch_tokens=budget,
                                 options=[gemma.BatchTokens(budget)]) for d in devices]


def _check(models, seqs):
    from ai_b200 import gemma

    got = gemma.embed_ids_multi(models, seqs)
    assert got.shape == (len(seqs), models[0].Dim())
    slices = gemma.plan_split([len(s) for s in seqs], len(models))
    assert sorted(np.concatenate(slices).tolist()) == list(range(len(seqs)))
    for m, idx in zip(models, slices):
        if len(idx) == 0:
            continue
        alone = np.stack(m.embed_ids([seqs[i] for i in idx]))
        assert np.array_equal(got[idx], alone)
    return got


def test_two_models_on_one_gpu_equal_their_slices_alone(cuda):
    from ai_b200 import synthetic as S
    from oracle import oracle as O

    cfg = S.small_config(layers=3, vocab=4096)
    w = S.make_weights(cfg, seed=21, norm_std=0.05)
    seqs, lengths = S.make_ragged(40, 1, 700, 9, vocab=cfg["vocab_size"])
    seqs[3] = []  # a length-0 sequence pools the pad token alone
    lengths[3] = 0
    models = _models([0, 0], cfg, w, 4096)
    try:
        got = _check(models, seqs)
        orc = O.from_bf16(cfg, w)
        for i in (3, int(np.argmax(lengths)), 17):
            s = np.asarray(seqs[i], np.int32)
            want = orc.embed_padded(np.zeros((1, max(len(s), 1)), np.int32) if len(s) == 0 else s[None],
                                    np.array([len(s)], np.int32), mode=O.F64)[0]
            assert np.abs(got[i] - want).max() <= 1e-4
    finally:
        for m in models:
            m.close()


def test_one_model_equals_embed_ids(cuda):
    from ai_b200 import gemma
    from ai_b200 import synthetic as S

    cfg = S.small_config(layers=2, vocab=4096)
    w = S.make_weights(cfg, seed=22)
    seqs, _ = S.make_ragged(25, 1, 400, 10, vocab=cfg["vocab_size"])
    (m,) = _models([0], cfg, w, 2048)
    try:
        assert np.array_equal(gemma.embed_ids_multi([m], seqs), np.stack(m.embed_ids(seqs)))
    finally:
        m.close()


def test_one_model_per_gpu(cuda):
    import torch

    from ai_b200 import synthetic as S

    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("one GPU on this box: the per-GPU case needs two or more")
    cfg = S.small_config(layers=3, vocab=4096)
    w = S.make_weights(cfg, seed=23)
    seqs, _ = S.make_ragged(64, 1, 1024, 11, vocab=cfg["vocab_size"])
    models = _models(list(range(n)), cfg, w, 8192)
    try:
        _check(models, seqs)
    finally:
        for m in models:
            m.close()


def test_failure_in_one_slice_is_reported(cuda):
    """A token id outside the vocabulary in one slice fails that slice's
    fg_embed_many; the call returns its error naming the model."""
    from ai_b200 import _lib, gemma
    from ai_b200 import synthetic as S

    cfg = S.small_config(layers=1, vocab=1024)
    w = S.make_weights(cfg, seed=24)
    seqs = [[5, 6, 7], [8] * 300, [9, 10]]
    seqs[1][10] = 5000
    models = _models([0, 0], cfg, w, 1024)
    try:
        with pytest.raises(_lib.FGError) as e:
            gemma.embed_ids_multi(models, seqs)
        assert e.value.code == _lib.FG_EINVAL and "model" in str(e.value)
    finally:
        for m in models:
            m.close()
