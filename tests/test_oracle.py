"""Pins the CPU oracle (test infrastructure) before it is trusted as the
checker of the CUDA path.

1. Model level: against the committed Hugging Face Gemma3TextModel goldens
   (tests/golden/make_golden.py) — float64 mode within 1e-6, the
   reference's float32 arithmetic within 2e-6.
2. Op level: the reference's own known-answer tests, restated:
   - RoPE: angle 1 rad at position 1, identity at position 0, norm kept
     (tensor/rope_test.go:9-38);
   - WindowMask exact pattern (rope_test.go:66-81), PaddingMask (attention.go:33-42);
   - attention against a naive float64 softmax at 1e-4, with and without a
     padding mask (tensor/attention_test.go:57-92);
   - masked attention weights exactly 0; causal row 0 reproduces v[0]
     (attention_test.go:266-285);
   - RMSNorm fused vs composed, rtol 1e-5 atol 1e-6 (rope_test.go:83-102);
   - GEMM vs float64 at 1e-4·(1+|w|) (internal/blas/gemm_test.go:22-124) and
     the fused epilogue order (internal/blas/epilogue_test.go);
   - exp and tanh within 2e-6 relative, exp flushes to exactly 0 below −87
     (internal/kernel/kernel.go:307-333, exp_flush_test.go);
   - bf16 widening is exact (safetensors/convert.go:31-38).
"""
import json
import math
from pathlib import Path

import numpy as np
import pytest

from ai_b200 import synthetic as S
from oracle import oracle as O

GOLD = Path(__file__).resolve().parent / "golden"


def _case(name):
    m = json.loads((GOLD / "manifest.json").read_text())[name]
    cfg = dict(S.EMBEDDINGGEMMA_300M)
    cfg.update(m["config"])
    w = S.make_weights(cfg, seed=m["seed"], norm_std=m["norm_std"])
    return cfg, w, np.load(GOLD / f"{name}.npz"), m


@pytest.mark.parametrize("name", ["window", "ragged", "c1"])
def test_oracle_matches_hf_goldens(name):
    cfg, w, z, m = _case(name)
    assert S.make_weights.__doc__  # generator present
    om = O.from_bf16(cfg, w)
    e64 = om.embed_padded(z["ids"], z["lengths"], mode=O.F64)
    assert np.abs(e64 - z["hf"]).max() <= 1e-6
    e32 = om.embed_padded(z["ids"], z["lengths"], mode=O.F32)
    assert np.abs(e32 - z["hf"]).max() <= 2e-6


def test_synthetic_weights_are_reproducible():
    import hashlib

    man = json.loads((GOLD / "manifest.json").read_text())
    m = man["window"]
    cfg = dict(S.EMBEDDINGGEMMA_300M)
    cfg.update(m["config"])
    w = S.make_weights(cfg, seed=m["seed"], norm_std=m["norm_std"])
    h = hashlib.sha256()
    for k in sorted(w):
        h.update(k.encode())
        h.update(np.ascontiguousarray(w[k]).tobytes())
    assert h.hexdigest() == m["weights_sha256"]


def test_length_zero_is_the_pad_token_alone():
    """embedBatch pads a length-0 sequence with id 0 and pools row 0
    (embed.go:131-137, 386-389); every padded row is the same token with
    equal attention weights, so the result is the single pad token's
    embedding."""
    cfg = S.small_config(layers=6, vocab=512)
    w = S.make_weights(cfg, seed=3, norm_std=0.1)
    om = O.from_bf16(cfg, w)
    ids = S.make_ids(2, 300, 1, 512)
    a = om.embed_padded(ids, np.array([0, 300], np.int32))
    b = om.embed_padded(np.zeros((1, 1), np.int32), np.array([1], np.int32))
    assert np.abs(a[0] - b[0]).max() <= 1e-6


def test_rope_known_answers():
    got = O.rope(np.array([[1, 0]], np.float32), 10000, [1])
    assert abs(got[0, 0] - math.cos(1)) <= 1e-6 and abs(got[0, 1] - math.sin(1)) <= 1e-6
    x = np.array([[3, -4, 5, 6]], np.float32)
    assert np.abs(O.rope(x, 10000, [0]) - x).max() <= 1e-6
    rng = np.random.default_rng(1)
    y = rng.standard_normal((2 * 3 * 8, 16), dtype=np.float32)
    r = O.rope(y.reshape(2, 3, 8, 16), 1e6, [0, 5, 9, 100, 500, 1000, 3, 7]).reshape(-1, 16)
    xn, yn = (y.astype(np.float64) ** 2).sum(-1), (r.astype(np.float64) ** 2).sum(-1)
    assert np.all(np.abs(xn - yn) <= 1e-3 * (xn + 1))


def test_window_and_padding_masks():
    m = O.window_mask(5, 2)
    for i in range(5):
        for j in range(5):
            assert m[i, j] == (-1e9 if (j - i >= 2 or i - j >= 2) else 0)
    p = O.padding_mask([5, 3], 5)
    assert (p[0] == 0).all() and (p[1, :3] == 0).all() and (p[1, 3:] == np.float32(-1e9)).all()


def _naive(q, k, v, mask):
    s = q.astype(np.float64) @ k.astype(np.float64).T / math.sqrt(q.shape[1])
    if mask is not None:
        s = s + mask
    s = np.exp(s - s.max(1, keepdims=True))
    return (s / s.sum(1, keepdims=True)) @ v.astype(np.float64)


@pytest.mark.parametrize("mode", [O.F64, O.F32])
def test_attention_vs_naive(mode):
    rng = np.random.default_rng(41)
    T, S_, D = 5, 7, 4
    for masked in (False, True):
        q = rng.standard_normal((T, D), dtype=np.float32)
        k = rng.standard_normal((S_, D), dtype=np.float32)
        v = rng.standard_normal((S_, D), dtype=np.float32)
        mask = np.broadcast_to(O.padding_mask([3], S_)[0], (T, S_)).copy() if masked else None
        got = O.attention_head(q, k, v, mask, 1 / math.sqrt(D), mode)
        assert np.abs(got - _naive(q, k, v, mask)).max() <= 1e-4


def test_masked_weights_exact_zero():
    rng = np.random.default_rng(11)
    n, d = 64, 16
    q, k, v = (rng.standard_normal((n, d), dtype=np.float32) for _ in range(3))
    causal = np.triu(np.full((n, n), -1e9, np.float32), 1)
    for mode in (O.F64, O.F32):
        out = O.attention_head(q, k, v, causal, 0.25, mode)
        assert np.array_equal(out[0], v[0])


def test_rmsnorm_fused_vs_composed():
    rng = np.random.default_rng(7)
    x = rng.standard_normal((4, 5, 64), dtype=np.float32)
    g = rng.standard_normal(64, dtype=np.float32)
    x64 = x.astype(np.float64)
    comp = x64 / np.sqrt((x64 ** 2).mean(-1, keepdims=True) + 1e-6) * g
    for mode in (O.F64, O.F32):
        assert np.allclose(O.rmsnorm(x, g, 1e-6, mode), comp, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (7, 13, 5), (64, 300, 129), (200, 96, 300)])
def test_gemm_vs_float64(m, k, n):
    rng = np.random.default_rng(3)
    a = rng.standard_normal((m, k), dtype=np.float32)
    w = rng.standard_normal((k, n), dtype=np.float32)
    want = a.astype(np.float64) @ w.astype(np.float64)
    for mode in (O.F64, O.F32):
        got = O.matmul_fused(a, w, mode=mode)
        assert np.all(np.abs(got - want) <= 1e-4 * (1 + np.abs(want)))


def test_epilogue_order():
    rng = np.random.default_rng(5)
    m, k, n = 20, 30, 40
    a, w = rng.standard_normal((m, k)), rng.standard_normal((k, n))
    bias, rs = rng.standard_normal(n), rng.uniform(0.5, 2, m)
    mul, res = rng.standard_normal((m, n)), rng.standard_normal((m, n))
    y = (a @ w + bias) * rs[:, None]
    gelu = 0.5 * y * (1 + np.tanh(0.7978845608028654 * (y + 0.044715 * y ** 3)))
    want = gelu * mul + res
    for mode in (O.F64, O.F32):
        got = O.matmul_fused(a, w, bias, rs, 2, mul, res, mode)
        assert np.allclose(got, want, rtol=1e-4, atol=1e-4)


def test_exp_and_tanh_accuracy():
    x = np.linspace(-87, 88, 200001).astype(np.float32)
    e = O.exp_ref(x).astype(np.float64)
    want = np.exp(x.astype(np.float64))
    assert np.all(np.abs(e - want) <= 2e-6 * want)
    assert np.all(O.exp_ref(np.array([-87.01, -100, -1e9], np.float32)) == 0)
    t = np.linspace(-12, 12, 200001).astype(np.float32)
    tt = O.tanh_ref(t).astype(np.float64)
    assert np.all(np.abs(tt - np.tanh(t.astype(np.float64))) <= 2e-6 * np.maximum(1e-3, np.abs(np.tanh(t.astype(np.float64)))) + 1e-9)
    g = O.gelu_ref(t).astype(np.float64)
    t64 = t.astype(np.float64)
    gw = 0.5 * t64 * (1 + np.tanh(0.7978845608028654 * (t64 + 0.044715 * t64 ** 3)))
    assert np.all(np.abs(g - gw) <= 1e-5 * (1 + np.abs(gw)))


def test_bf16_widening_exact():
    bits = np.arange(0, 1 << 16, dtype=np.uint32).astype(np.uint16)
    f = S.bf16_to_f32(bits)
    back = (f.view(np.uint32) >> 16).astype(np.uint16)
    assert np.array_equal(back, bits)
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32)
    r = S.bf16_to_f32(S.bf16_round(x))
    assert np.all(np.abs(r - x) <= np.abs(x) * 2.0 ** -8)


@pytest.mark.parametrize("m,k,n", [(1, 7, 5), (13, 768, 33), (14, 64, 32), (29, 1152, 768),
                                   (130, 768, 3072), (300, 96, 97)])
def test_fast_f32_gemm_is_bitwise_the_simple_loops(m, k, n):
    """The packed AVX-512 float32 GEMM (14×32 register tiles over packed
    panels) computes every element as the same sequential chain of fused
    multiply-adds over k as the simple loops: bit for bit equal, ragged
    edges included."""
    rng = np.random.default_rng(m * 1000 + n)
    a = rng.standard_normal((m, k), dtype=np.float32)
    w = rng.standard_normal((k, n), dtype=np.float32)
    try:
        O.set_fast_kernels(False)
        slow = O.matmul_fused(a, w, mode=O.F32)
        O.set_fast_kernels(True)
        fast = O.matmul_fused(a, w, mode=O.F32)
    finally:
        O.set_fast_kernels(True)
    assert np.array_equal(fast, slow)


def test_fast_f32_encoder_is_bitwise_the_simple_loops():
    """The whole float32-mode encoder (packed GEMMs, attention scores 16 keys
    at a time over a transposed K) equals the simple loops bit for bit, with
    padding and the sliding window active."""
    cfg = S.small_config(layers=2, vocab=512, sliding_window=64)
    w = S.make_weights(cfg, seed=5, norm_std=0.1)
    ids = S.make_ids(3, 150, 2, cfg["vocab_size"])
    lengths = np.array([150, 77, 1], np.int32)
    om = O.from_bf16(cfg, w)
    try:
        O.set_fast_kernels(False)
        slow = om.embed_padded(ids, lengths, mode=O.F32)
        O.set_fast_kernels(True)
        fast = om.embed_padded(ids, lengths, mode=O.F32)
    finally:
        O.set_fast_kernels(True)
    assert np.array_equal(fast, slow)
