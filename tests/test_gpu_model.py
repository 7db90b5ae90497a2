"""GPU parity of the whole encoder path (fg_embed_ids) against the CPU
oracle and the committed Hugging Face goldens.

Bar (split-TF32, the default): per-sentence cosine ≥ 0.99999 and max-abs
elementwise error ≤ 1e-4 against the float64 oracle and the goldens.
Plain TF32 is measured and reported, with a looser sanity bound.
"""
import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"
COS_MIN = 0.99999
MAXABS = 1e-4


def _cmp(got, want):
    got = got.astype(np.float64)
    want = want.astype(np.float64)
    cos = (got * want).sum(1) / np.linalg.norm(got, axis=1) / np.linalg.norm(want, axis=1)
    return float(cos.min()), float(np.abs(got - want).max())


def _case(name):
    from ai_b200 import synthetic as S

    m = json.loads((GOLD / "manifest.json").read_text())[name]
    cfg = dict(S.EMBEDDINGGEMMA_300M)
    cfg.update(m["config"])
    w = S.make_weights(cfg, seed=m["seed"], norm_std=m["norm_std"])
    z = np.load(GOLD / f"{name}.npz")
    return cfg, w, z


@pytest.fixture(scope="module")
def c1():
    from ai_b200 import gemma
    from oracle import oracle as O

    cfg, w, z = _case("c1")
    model = gemma.from_synthetic(cfg, w, device=0, max_batch_tokens=4096)
    orc = O.from_bf16(cfg, w)
    yield cfg, w, z, model, orc
    model.close()


def test_c1_split_tf32_matches_goldens_and_oracle(c1):
    from oracle import oracle as O

    cfg, w, z, model, orc = c1
    got = model.embed_padded(z["ids"], z["lengths"])
    ref64 = orc.embed_padded(z["ids"], z["lengths"], mode=O.F64)
    ref32 = orc.embed_padded(z["ids"], z["lengths"], mode=O.F32)
    c_hf, m_hf = _cmp(got, z["hf"])
    c_or, m_or = _cmp(got, ref64)
    c_rr, m_rr = _cmp(ref32, ref64)
    print(f"\nC1 split-TF32 vs HF: cos {c_hf:.9f} maxabs {m_hf:.3e}; vs oracle f64: cos {c_or:.9f} "
          f"maxabs {m_or:.3e}; reference-f32 arithmetic vs f64: cos {c_rr:.9f} maxabs {m_rr:.3e}")
    assert c_hf >= COS_MIN and m_hf <= MAXABS
    assert c_or >= COS_MIN and m_or <= MAXABS


def test_c1_plain_tf32_deviation(c1):
    from ai_b200 import gemma

    cfg, w, z, model, orc = c1
    got = model.embed_padded(z["ids"], z["lengths"], precision=gemma.PREC_TF32)
    c, m = _cmp(got, z["hf"])
    print(f"\nC1 plain TF32 vs HF: cos {c:.9f} maxabs {m:.3e}")
    assert c >= 0.999


def test_c1_deterministic(c1):
    cfg, w, z, model, orc = c1
    a = model.embed_padded(z["ids"], z["lengths"])
    b = model.embed_padded(z["ids"], z["lengths"])
    assert np.array_equal(a, b)


@pytest.mark.parametrize("name", ["window", "ragged"])
def test_padded_window_and_ragged_goldens(name):
    from ai_b200 import gemma
    from oracle import oracle as O

    cfg, w, z = _case(name)
    model = gemma.from_synthetic(cfg, w, device=0, max_batch_tokens=4096)
    try:
        got = model.embed_padded(z["ids"], z["lengths"])
        ref = O.from_bf16(cfg, w).embed_padded(z["ids"], z["lengths"], mode=O.F64)
    finally:
        model.close()
    c_hf, m_hf = _cmp(got, z["hf"])
    c_or, m_or = _cmp(got, ref)
    print(f"\n{name}: vs HF cos {c_hf:.9f} maxabs {m_hf:.3e}; vs oracle cos {c_or:.9f} maxabs {m_or:.3e}")
    assert c_hf >= COS_MIN and m_hf <= MAXABS
    assert c_or >= COS_MIN and m_or <= MAXABS


@pytest.fixture(scope="module")
def small():
    from ai_b200 import gemma
    from ai_b200 import synthetic as S
    from oracle import oracle as O

    cfg = S.small_config(layers=6, vocab=4096)
    w = S.make_weights(cfg, seed=21, norm_std=0.1)
    model = gemma.from_synthetic(cfg, w, device=0, max_batch_tokens=8192)
    yield cfg, w, model, O.from_bf16(cfg, w)
    model.close()


def test_length_zero_and_one(small):
    """A length-0 sequence embeds as the reference's all-padding row 0
    (embed.go:131-137, 386-389); checked against the oracle, which runs the
    reference's literal masks."""
    from ai_b200 import synthetic as S
    from oracle import oracle as O

    cfg, w, model, orc = small
    ids = S.make_ids(4, 40, 3, cfg["vocab_size"])
    lengths = np.array([0, 1, 40, 0], np.int32)
    got = model.embed_padded(ids, lengths)
    ref = orc.embed_padded(ids, lengths, mode=O.F64)
    c, m = _cmp(got, ref)
    assert c >= COS_MIN and m <= MAXABS, (c, m)


def test_embedding_table_bf16_residency(small, monkeypatch):
    """A bf16-exact table is kept as bf16 on the device and widened in the
    gather: the result is bitwise the fp32-resident table's
    (FG_EMBED_BF16=0). A table that is not bf16-exact stays fp32 and
    matches the oracle on the same weights."""
    from ai_b200 import _lib, gemma
    from ai_b200 import synthetic as S
    from oracle import oracle as O

    cfg, w, model, orc = small
    ids = S.make_ids(3, 64, 5, cfg["vocab_size"])
    lengths = np.array([64, 17, 40], np.int32)
    base = model.embed_padded(ids, lengths)
    monkeypatch.setenv("FG_EMBED_BF16", "0")
    m32 = gemma.from_synthetic(cfg, w, device=0, max_batch_tokens=8192)
    try:
        assert np.array_equal(m32.embed_padded(ids, lengths), base)
    finally:
        m32.close()
    monkeypatch.delenv("FG_EMBED_BF16")

    wf = {k: S.bf16_to_f32(v) for k, v in w.items()}
    t = wf["embed_tokens.weight"]
    noise = np.random.default_rng(9).standard_normal(t.shape).astype(np.float32)
    wf["embed_tokens.weight"] = (t * (1 + 1e-3 * noise)).astype(np.float32)
    assert np.any(wf["embed_tokens.weight"].view(np.uint32) & 0xFFFF)
    body = {k: (_lib.DT_BF16, v) for k, v in w.items() if not k.startswith("dense.")}
    body["embed_tokens.weight"] = (_lib.DT_F32, wf["embed_tokens.weight"])
    dense = [gemma.DenseSpec(w[f"dense.{j}.linear.weight"], _lib.DT_BF16)
             for j in range(len([k for k in w if k.startswith("dense.")]))]
    mf = gemma.Model(gemma.config_from_dict(cfg), body, dense, True, device=0, max_batch_tokens=8192)
    try:
        got = mf.embed_padded(ids, lengths)
    finally:
        mf.close()
    ref = O.OracleModel(cfg, wf).embed_padded(ids, lengths, mode=O.F64)
    c, m = _cmp(got, ref)
    assert c >= COS_MIN and m <= MAXABS, (c, m)
    assert not np.array_equal(got, base)


@pytest.mark.parametrize("norm_std", [0.0, 0.1])
def test_bf16_resident_projections_are_bitwise_identical(norm_std):
    """gemma.WeightsBF16(): projections resident in 2 bytes per value,
    widened, gain-folded and split per layer on the device where a product
    needs fp32, give the same embeddings bit for bit as the fp32-resident
    weights, in all three precisions, with zero norm weights (folded weights
    bf16-exact, no low parts) and non-zero ones (folded weights with low
    parts); the weights take fewer device bytes. Projections with an exact
    fp16 form stay resident in it: the split-fp16 products (PREC_SPLIT) read
    it as it is, split-TF32 and plain TF32 widen it."""
    from ai_b200 import _lib, gemma
    from ai_b200 import synthetic as S

    cfg = S.small_config(layers=3, vocab=2048)
    w = S.make_weights(cfg, seed=31, norm_std=norm_std)
    ids = S.make_ids(4, 96, 6, cfg["vocab_size"])
    lengths = np.array([96, 50, 1, 77], np.int32)
    m32 = gemma.from_synthetic(cfg, w, device=0, max_batch_tokens=4096)
    m16 = gemma.from_synthetic(cfg, w, device=0, max_batch_tokens=4096, options=[gemma.WeightsBF16()])
    try:
        for prec in (_lib.PREC_SPLIT, _lib.PREC_SPLIT_TF32, _lib.PREC_TF32):
            a = m32.embed_padded(ids, lengths, precision=prec)
            b = m16.embed_padded(ids, lengths, precision=prec)
            assert np.array_equal(a, b), prec
        b32, b16 = m32.weight_bytes(), m16.weight_bytes()
        print(f"norm_std {norm_std}: weight bytes fp32 {b32}, bf16 {b16}")
        assert b16 < b32
    finally:
        m32.close()
        m16.close()


@pytest.mark.parametrize("norm_std,T,lengths", [
    (0.0, 128, [128, 100, 1, 77, 128, 64]),
    (0.1, 128, [128, 100, 1, 77, 128, 64]),
    # query tiles past a sequence's length (the attention's empty-tile path)
    (0.0, 512, [512, 1, 200, 129, 300, 512]),
    (0.1, 512, [3, 512, 255, 130, 384, 90]),
])
def test_split_fp16_matches_split_tf32(norm_std, T, lengths):
    """The split-fp16 encoder GEMMs (bf16-exact weights as exact fp16, A as
    two fp16 parts under a power-of-two row scale, made by A's producer for
    O, gate/up and down) agree with split-TF32 to the size of split-TF32's
    own error, are in use (not bitwise equal) and repeatable. With non-zero
    norm gains the folded Q/K/V and gate/up weights have no exact fp16 form:
    those GEMMs take the unfolded weights and apply the gains to A."""
    from ai_b200 import gemma
    from ai_b200 import synthetic as S

    cfg = S.small_config(layers=3, vocab=2048)
    w = S.make_weights(cfg, seed=43, norm_std=norm_std)
    ids = S.make_ids(len(lengths), T, 14, cfg["vocab_size"])
    lengths = np.array(lengths, np.int32)
    m1 = gemma.from_synthetic(cfg, w, device=0, max_batch_tokens=len(lengths) * T)
    try:
        a = m1.embed_padded(ids, lengths)
        b = m1.embed_padded(ids, lengths, precision=gemma.PREC_SPLIT_TF32)
        d = np.abs(a.astype(np.float64) - b).max()
        print(f"norm_std {norm_std}: split-fp16 vs split-TF32 max |diff| {d:.3e}")
        assert d <= 5e-6
        assert not np.array_equal(a, b)
        assert np.array_equal(a, m1.embed_padded(ids, lengths))  # repeatable
    finally:
        m1.close()


def test_batch_invariance(small):
    """A sequence embeds the same alone and inside a padded batch
    (models/gemma/gemma_test.go:117-135 asks ≥ 0.9999)."""
    from ai_b200 import synthetic as S

    cfg, w, model, orc = small
    seqs, _ = S.make_ragged(6, 5, 400, 9, cfg["vocab_size"])
    together = model.embed_batch(seqs)
    for i, s in enumerate(seqs):
        alone = model.embed_batch([s])
        c, m = _cmp(alone, together[i:i + 1])
        assert c >= COS_MIN and m <= MAXABS, (i, c, m)


def test_matryoshka_dim(small):
    """Dim(d) narrows the head output and renormalises (embed.go:421-427)."""
    from ai_b200 import synthetic as S

    cfg, w, model, orc = small
    ids = S.make_ids(3, 50, 4, cfg["vocab_size"])
    lengths = np.array([50, 30, 10], np.int32)
    full = model.embed_padded(ids, lengths)
    part = model.embed_padded(ids, lengths, dim=256)
    want = full[:, :256] / np.linalg.norm(full[:, :256].astype(np.float64), axis=1, keepdims=True)
    assert np.abs(part - want).max() <= 1e-6


def test_embed_ids_batches_and_restores_order(small):
    from ai_b200 import gemma
    from ai_b200 import synthetic as S

    cfg, w, model, orc = small
    seqs, _ = S.make_ragged(10, 1, 300, 13, cfg["vocab_size"])
    model.batch_tokens = 600  # forces several greedy batches (embed.go:61-74)
    try:
        got = np.stack(model.embed_ids(seqs))
    finally:
        model.batch_tokens = 8192
    want = np.stack([model.embed_batch([s])[0] for s in seqs])
    c, m = _cmp(got, want)
    assert c >= COS_MIN and m <= MAXABS


def test_embed_ids_pipeline_equals_batch_by_batch(small):
    """fg_embed_many (batches packed and copied in while the previous one
    runs) gives, bit for bit, what running each planned batch alone gives;
    truncation to MaxTokens (embed.go:38-40) and empty sequences included."""
    from ai_b200 import gemma
    from ai_b200 import synthetic as S

    cfg, w, model, orc = small
    seqs, _ = S.make_ragged(37, 1, 400, 17, cfg["vocab_size"])
    seqs[3] = []
    seqs[20] = list(seqs[20]) * 3  # longer than the budget: runs alone
    model.batch_tokens = 1000
    model.max_tokens = 700
    try:
        got = np.stack(model.embed_ids(seqs))
        cut = [list(s)[:700] for s in seqs]
        _, batches = gemma.plan_batches([len(s) for s in cut], 1000)
        want = np.zeros_like(got)
        for b in batches:
            want[b] = model.embed_batch([cut[i] for i in b])
    finally:
        model.batch_tokens = 8192
        model.max_tokens = 2048
    assert len(batches) > 5
    assert np.array_equal(got, want)


def test_errors_are_reported_not_fatal(small):
    from ai_b200 import _lib, gemma

    cfg, w, model, orc = small
    with pytest.raises(_lib.FGError) as e:
        model.embed_padded(np.full((1, 4), cfg["vocab_size"], np.int32), np.array([4], np.int32))
    assert e.value.code == _lib.FG_EINVAL
    with pytest.raises(gemma.GemmaError):
        model.embed_ids([[2, 5, 6]], Dim=769)
    with pytest.raises(_lib.FGError):
        model.embed_padded(np.zeros((1, 3000), np.int32), np.array([3000], np.int32))
    # the model still works afterwards
    out = model.embed_padded(np.array([[2, 7, 9]], np.int32), np.array([3], np.int32))
    assert np.isfinite(out).all()
    model.check()


def test_device_api(small):
    import torch

    from ai_b200 import synthetic as S

    cfg, w, model, orc = small
    ids = S.make_ids(4, 64, 17, cfg["vocab_size"])
    lengths = np.array([64, 10, 33, 1], np.int32)
    d_ids = torch.from_numpy(ids).cuda()
    d_len = torch.from_numpy(lengths).cuda()
    out = torch.empty((4, 768), dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream()
    model.embed_device(d_ids, d_len, 4, 64, 768, out, s)
    s.synchronize()
    model.check()
    want = model.embed_padded(ids, lengths)
    assert np.array_equal(out.cpu().numpy(), want)


def test_device_api_graph_replay(small):
    """Repeated device-API calls with one shape and one set of buffers: the
    first runs eagerly, the second is captured into a CUDA graph and
    launched, the third launches the graph. Every result is bitwise the
    eager forward's, the per-phase launch counts still count every call,
    and ids written into the same buffer afterwards are the ones embedded."""
    import torch

    from ai_b200 import synthetic as S

    cfg, w, model, orc = small
    B, T = 4, 64
    ids = S.make_ids(B, T, 31, cfg["vocab_size"])
    lengths = np.array([64, 17, 40, 2], np.int32)
    d_ids = torch.from_numpy(ids).cuda()
    d_len = torch.from_numpy(lengths).cuda()
    out = torch.empty((B, 768), dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream()

    def run():
        model.embed_device(d_ids, d_len, B, T, 768, out, s)
        s.synchronize()
        model.check()
        return out.cpu().numpy().copy()

    def launches():
        return sum(v["launches"] for v in model.read_profile().values())

    launches()
    first = run()
    per_call = launches()
    second = run()
    third = run()
    assert per_call > 0 and launches() == 2 * per_call
    assert np.array_equal(first, second) and np.array_equal(first, third)
    ids2 = S.make_ids(B, T, 32, cfg["vocab_size"])
    d_ids.copy_(torch.from_numpy(ids2))
    got = run()
    assert np.array_equal(got, model.embed_padded(ids2, lengths))
    assert not np.array_equal(got, first)
