"""EmbeddingGemma 2's text tower on the device (forward_v2) against the
float64 restatement (oracle/gemma2.py) on the same random-init weights:
per-sentence cosine ≥ 0.99999 and max-abs ≤ 1e-4 in split-TF32, as for
EmbeddingGemma-300m. Covers sliding layers with 256-wide heads (tensor-core
attention) and global layers with 512-wide heads (SIMT attention), ragged
lengths with the window active, lengths 0 and 1, and the 12-layer
EmbeddingGemma 2 shape."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

COS_MIN = 0.99999
MAXABS = 1e-4


def _cmp(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    cos = (got * want).sum(1) / np.linalg.norm(got, axis=1) / np.linalg.norm(want, axis=1)
    return float(cos.min()), float(np.abs(got - want).max())


@pytest.fixture(scope="module")
def small():
    from ai_b200 import gemma
    from ai_b200 import synthetic as S
    from oracle import gemma2 as G

    cfg = S.eg2_small_config(layers=4, full=(1, 3), window=48)
    w = S.make_weights_eg2(cfg, seed=3)
    model = gemma.from_synthetic(cfg, w, device=0, max_batch_tokens=8192)
    yield cfg, w, model, G.from_bf16(cfg, w)
    model.close()


def test_small_ragged_vs_oracle(small):
    from ai_b200 import synthetic as S

    cfg, w, model, orc = small
    ids = S.make_ids(5, 150, 7, 4096)
    lengths = np.array([150, 97, 1, 0, 60], np.int32)
    got = model.embed_padded(ids, lengths)
    assert got.shape == (5, 192)
    want = orc.embed_padded(ids, lengths)
    c, m = _cmp(got, want)
    print(f"EmbeddingGemma 2 small: cos {c:.9f} maxabs {m:.2e}")
    assert c >= COS_MIN and m <= MAXABS


def test_small_plain_tf32_and_determinism(small):
    from ai_b200 import gemma
    from ai_b200 import synthetic as S

    cfg, w, model, orc = small
    ids = S.make_ids(2, 120, 8, 4096)
    lengths = np.array([120, 64], np.int32)
    a = model.embed_padded(ids, lengths)
    assert np.array_equal(a, model.embed_padded(ids, lengths))
    p = model.embed_padded(ids, lengths, precision=gemma.PREC_TF32)
    c, m = _cmp(p, orc.embed_padded(ids, lengths))
    print(f"EmbeddingGemma 2 small plain TF32: cos {c:.9f} maxabs {m:.2e}")
    assert c >= 0.999


def test_small_embed_ids_and_dim(small):
    from ai_b200 import synthetic as S

    cfg, w, model, orc = small
    seqs, _ = S.make_ragged(9, 1, 200, 11, cfg["text_config"]["vocab_size"])
    got = np.stack(model.embed_ids(seqs, Dim=64))
    lengths = np.array([len(s) for s in seqs], np.int32)
    ids = np.zeros((9, int(lengths.max())), np.int32)
    for b, s in enumerate(seqs):
        ids[b, :len(s)] = s
    want = orc.embed_padded(ids, lengths, dim=64)
    c, m = _cmp(got, want)
    assert c >= COS_MIN and m <= MAXABS


def test_eg2_shape_vs_oracle():
    """The 12-layer EmbeddingGemma 2 shape (the reference's TestConfig2),
    window 513 active at 600 tokens."""
    from ai_b200 import gemma
    from ai_b200 import synthetic as S
    from oracle import gemma2 as G

    text = dict(S.EMBEDDINGGEMMA2_TEXT)
    text["vocab_size"] = 8192
    cfg = S.eg2_config(text)
    w = S.make_weights_eg2(cfg, seed=5)
    model = gemma.from_synthetic(cfg, w, device=0, max_batch_tokens=4096)
    try:
        ids = S.make_ids(2, 600, 9, 8192)
        lengths = np.array([600, 333], np.int32)
        got = model.embed_padded(ids, lengths)
    finally:
        model.close()
    c, m = _cmp(got, G.from_bf16(cfg, w).embed_padded(ids, lengths))
    print(f"EmbeddingGemma 2 shape: cos {c:.9f} maxabs {m:.2e}")
    assert c >= COS_MIN and m <= MAXABS
