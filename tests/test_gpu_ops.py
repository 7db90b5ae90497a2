"""GPU parity of the op-level C ABI (fg_matmul, fg_attention, fg_rmsnorm,
fg_rope, fg_row_sum_squares) against float64 restatements of the
reference's operations, with the reference's own tolerances:
GEMM 1e-4·(1+|w|) (internal/blas/gemm_test.go:22-124), attention 1e-4
(tensor/attention_test.go:12-92), RMSNorm rtol 1e-5 / atol 1e-6
(tensor/rope_test.go:83-102), RoPE 1e-6 (rope_test.go:9-25).
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)


def _gemm_tol(got, want, a=None, w=None, rel=1e-5):
    """The reference's bound 1e-4·(1+|w|), or, for long inner dimensions,
    rel·‖a_i‖·‖w_j‖ — the scale of an fp32 GEMM's rounding error: the tensor
    core's FP32 accumulator truncates on each of the K/8 updates, so its error
    grows with ‖a_i‖‖w_j‖ rather than with |C_ij|."""
    ok = np.abs(got - want) <= 1e-4 * (1 + np.abs(want))
    if a is not None:
        scale = np.linalg.norm(a.astype(np.float64), axis=1)[:, None] * \
            np.linalg.norm(w.astype(np.float64), axis=0)[None, :]
        ok |= np.abs(got - want) <= rel * scale
    return ok


@pytest.mark.parametrize("m,k,n", [(128, 768, 768), (1024, 768, 1152), (128, 768, 2304),
                                   (128, 768, 3072), (1024, 1152, 768), (1, 3, 1), (7, 17, 5),
                                   (130, 33, 200), (257, 768, 129), (300, 1152, 2304), (300, 100, 300),
                                   (1000, 45, 513)])
@pytest.mark.parametrize("transposed", [False, True])
def test_matmul_split_tf32_vs_float64(cuda, m, k, n, transposed):
    from ai_b200 import tensor as T

    rng = np.random.default_rng(3)
    a = rng.standard_normal((m, k), dtype=np.float32)
    w = rng.standard_normal((k, n), dtype=np.float32)
    want = a.astype(np.float64) @ w.astype(np.float64)
    x = _t(a, cuda)
    if transposed:
        wt = _t(w.T.copy(), cuda).t()  # [k, n] view of an [n, k] matrix, no copy
    else:
        wt = _t(w, cuda)
    got = T.MatMul(x, wt).cpu().numpy()
    ok = _gemm_tol(got, want, a, w, rel=3e-6)  # split: measured <= 1.95e-6
    scale = np.linalg.norm(a.astype(np.float64), axis=1)[:, None] * \
        np.linalg.norm(w.astype(np.float64), axis=0)[None, :]
    print(f"gemm m={m} k={k} n={n} T={transposed}: max|err| {np.abs(got - want).max():.3e} "
          f"max err/(|a||w|) {(np.abs(got - want) / scale).max():.3e}")
    assert ok.all(), f"max err {np.abs(got - want).max()} at {np.argwhere(~ok)[:3]}"


def test_matmul_split_rows_of_any_scale(cuda):
    """The split-fp16 product scales each row of A by its own power of two
    (from the row's norm) and B by one: rows of norm 0, 1e-15 and 1e15 and a
    B of tiny entries keep fp32-level accuracy relative to their own size."""
    from ai_b200 import tensor as T

    rng = np.random.default_rng(17)
    m, k, n = 512, 768, 384
    a = rng.standard_normal((m, k), dtype=np.float32)
    a[3] = 0.0
    a[5] *= np.float32(1e-15)
    a[7] *= np.float32(1e15)
    a[9, :100] *= np.float32(1e-6)  # small entries beside large ones in one row
    for bscale in (1.0, 1e-12):
        w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(bscale))
        want = a.astype(np.float64) @ w.T.astype(np.float64)
        got = T.MatMul(_t(a, cuda), _t(w, cuda).t()).cpu().numpy().astype(np.float64)
        scale = np.linalg.norm(a.astype(np.float64), axis=1)[:, None] * \
            np.linalg.norm(w.astype(np.float64), axis=1)[None, :]
        err = np.abs(got - want)
        assert np.all(err[3] == 0), err[3].max()
        ok = err <= 3e-6 * scale
        assert ok.all(), (bscale, (err / np.maximum(scale, 1e-300)).max(), np.argwhere(~ok)[:3])


def test_matmul_plain_tf32_error_is_tf32_sized(cuda):
    from ai_b200 import tensor as T

    rng = np.random.default_rng(5)
    a = rng.standard_normal((512, 768), dtype=np.float32)
    w = rng.standard_normal((768, 768), dtype=np.float32)
    want = a.astype(np.float64) @ w.astype(np.float64)
    got = T.MatMul(_t(a, cuda), _t(w, cuda), precision=T.PREC_TF32).cpu().numpy()
    rel = np.abs(got - want).max() / np.abs(want).max()
    split = T.MatMul(_t(a, cuda), _t(w, cuda)).cpu().numpy()
    rel_split = np.abs(split - want).max() / np.abs(want).max()
    assert rel < 1e-2
    assert rel_split < rel / 50, (rel_split, rel)


def test_tf32_operands_are_truncated_by_the_tensor_core(cuda):
    """A plain-TF32 product of raw fp32 operands equals the product of the
    operands with their low 13 mantissa bits cleared: the tensor core reads
    the top 19 bits. The split-TF32 path relies on this to pass raw fp32
    activations as the high part."""
    from ai_b200 import tensor as T

    rng = np.random.default_rng(6)
    a = rng.standard_normal((256, 512), dtype=np.float32)
    w = rng.standard_normal((512, 256), dtype=np.float32)
    trunc = lambda v: (v.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
    r1 = T.MatMul(_t(a, cuda), _t(w, cuda), precision=T.PREC_TF32).cpu().numpy()
    r2 = T.MatMul(_t(trunc(a), cuda), _t(trunc(w), cuda), precision=T.PREC_TF32).cpu().numpy()
    assert np.array_equal(r1, r2), np.abs(r1 - r2).max()


@pytest.mark.parametrize("m,k,n", [(256, 64, 256), (1000, 768, 768), (600, 256, 1280),
                                   (513, 32, 2304), (300, 1152, 300)])
def test_matmul_plain_tf32_equals_truncated_product(cuda, m, k, n):
    """Plain TF32 with M >= 256 and N > 128 runs on SM pairs (256-row
    tiles, ragged M and N edges included); the result is the float64
    product of the TF32-truncated operands up to fp32 accumulation."""
    from ai_b200 import tensor as T

    rng = np.random.default_rng(11)
    a = rng.standard_normal((m, k), dtype=np.float32)
    w = rng.standard_normal((k, n), dtype=np.float32)
    trunc = lambda v: (v.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
    want = trunc(a).astype(np.float64) @ trunc(w).astype(np.float64)
    wt = _t(w.T.copy(), cuda).t()  # K-major weights: no copy on the way in
    got = T.MatMul(_t(a, cuda), wt, precision=T.PREC_TF32).cpu().numpy()
    ok = _gemm_tol(got, want, a, w, rel=1e-6)  # vs the truncated product: <= 5.9e-7
    assert ok.all(), f"max err {np.abs(got - want).max()} at {np.argwhere(~ok)[:3]}"


def _gelu64(x):
    return 0.5 * x * (1 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


@pytest.mark.parametrize("act", [0, 1, 2])
def test_matmul_fused_epilogue_order(cuda, act):
    """bias → RowScale → Act → Mul → Residual (internal/blas/gemm.go:276-288)."""
    from ai_b200 import tensor as T

    rng = np.random.default_rng(7)
    m, k, n = 200, 96, 300
    a = rng.standard_normal((m, k), dtype=np.float32)
    w = rng.standard_normal((k, n), dtype=np.float32)
    bias = rng.standard_normal(n, dtype=np.float32)
    rs = rng.uniform(0.5, 2, m).astype(np.float32)
    mul = rng.standard_normal((m, n), dtype=np.float32)
    res = rng.standard_normal((m, n), dtype=np.float32)
    y = a.astype(np.float64) @ w.astype(np.float64) + bias
    y = y * rs[:, None]
    y = [y, np.maximum(y, 0), _gelu64(y)][act]
    want = y * mul + res
    f = T.Fused(Bias=_t(bias, cuda), Act=act, Mul=_t(mul, cuda), RowScale=_t(rs, cuda),
                Residual=_t(res, cuda))
    got = T.MatMulFused(_t(a, cuda), _t(w, cuda), f).cpu().numpy()
    assert np.allclose(got, want, rtol=1e-4, atol=1e-4), np.abs(got - want).max()


@pytest.mark.parametrize("act", [0, 1, 2])
def test_matmul_fused_epilogue_on_sm_pairs(cuda, act):
    """The same epilogue on the SM-pair kernel (plain TF32, M >= 256): each
    CTA of a pair applies it to its own 128 rows of the 256-row tile."""
    from ai_b200 import tensor as T

    rng = np.random.default_rng(8)
    m, k, n = 700, 96, 520
    trunc = lambda v: (v.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
    a = rng.standard_normal((m, k), dtype=np.float32)
    w = rng.standard_normal((k, n), dtype=np.float32)
    bias = rng.standard_normal(n, dtype=np.float32)
    rs = rng.uniform(0.5, 2, m).astype(np.float32)
    mul = rng.standard_normal((m, n), dtype=np.float32)
    res = rng.standard_normal((m, n), dtype=np.float32)
    y = trunc(a).astype(np.float64) @ trunc(w).astype(np.float64) + bias
    y = y * rs[:, None]
    y = [y, np.maximum(y, 0), _gelu64(y)][act]
    want = y * mul + res
    f = T.Fused(Bias=_t(bias, cuda), Act=act, Mul=_t(mul, cuda), RowScale=_t(rs, cuda),
                Residual=_t(res, cuda))
    wt = _t(w.T.copy(), cuda).t()
    got = T.MatMulFused(_t(a, cuda), wt, f, precision=T.PREC_TF32).cpu().numpy()
    assert np.allclose(got, want, rtol=1e-4, atol=1e-4), np.abs(got - want).max()


def _naive_attention(q, k, v, lens, window, scale):
    B, Hq, Tq, D = q.shape
    Hkv, S = k.shape[1], k.shape[2]
    out = np.zeros((B, Hq, Tq, D))
    for b in range(B):
        for h in range(Hq):
            hk = h // (Hq // Hkv)
            s = q[b, h].astype(np.float64) @ k[b, hk].astype(np.float64).T * scale
            i = np.arange(Tq)[:, None]
            j = np.arange(S)[None, :]
            # −1e9 per mask (padding, window); in float32 it swamps the score
            cnt = (j >= (lens[b] if lens is not None else S)).astype(int) + 0 * i
            if window:
                cnt = cnt + (np.abs(i - j) >= window)
            minc = cnt.min(axis=1, keepdims=True)
            keep = cnt == minc
            s = np.where(keep, np.where(minc == 0, s, 0.0), -np.inf)
            mx = s.max(axis=1, keepdims=True)
            p = np.exp(s - mx)
            p = p / p.sum(axis=1, keepdims=True)
            out[b, h] = p @ v[b, hk].astype(np.float64)
    return out


@pytest.mark.parametrize("B,Hq,Hkv,T,S,D,window,padded", [
    (2, 3, 3, 5, 7, 4, 0, True),
    (2, 3, 1, 65, 65, 40, 0, True),
    (2, 3, 1, 300, 300, 256, 257, True),
    (1, 3, 1, 600, 600, 256, 257, False),
    (2, 2, 2, 33, 7, 3, 0, False),
    (1, 2, 1, 65, 1753, 256, 0, True),
    (2, 3, 1, 512, 512, 64, 128, True),
    (2, 4, 1, 300, 300, 512, 0, True),     # head_dim 512: tensor cores, Q streamed
    (1, 4, 2, 700, 700, 512, 257, False),
])
def test_attention_vs_naive_float64(cuda, B, Hq, Hkv, T, S, D, window, padded):
    from ai_b200 import tensor as TT
    import torch

    rng = np.random.default_rng(41)
    q = rng.standard_normal((B, Hq, T, D), dtype=np.float32)
    k = rng.standard_normal((B, Hkv, S, D), dtype=np.float32)
    v = rng.standard_normal((B, Hkv, S, D), dtype=np.float32)
    lens = np.array([S] + [max(1, S // 2)] * (B - 1), dtype=np.int32) if padded else None
    scale = 1 / math.sqrt(D)
    want = _naive_attention(q, k, v, lens, window, scale)
    got = TT.AttentionScaled(_t(q, cuda), _t(k, cuda), _t(v, cuda),
                             None if lens is None else torch.from_numpy(lens), window,
                             scale).cpu().numpy()
    assert np.abs(got - want).max() <= 1e-4, np.abs(got - want).max()


def test_attention_masked_weights_are_exact_zeros(cuda):
    """A query that sees one key reproduces that key's value exactly
    (tensor/attention_test.go:266-285, with a padding mask of length 1)."""
    from ai_b200 import tensor as TT
    import torch

    rng = np.random.default_rng(11)
    q = rng.standard_normal((1, 1, 64, 16), dtype=np.float32)
    k = rng.standard_normal((1, 1, 64, 16), dtype=np.float32)
    v = rng.standard_normal((1, 1, 64, 16), dtype=np.float32)
    got = TT.AttentionScaled(_t(q, cuda), _t(k, cuda), _t(v, cuda),
                             torch.tensor([1], dtype=torch.int32), 0, 0.25).cpu().numpy()
    assert np.array_equal(got[0, 0], np.broadcast_to(v[0, 0, 0], (64, 16)))


def test_rmsnorm_and_row_sum_squares(cuda):
    from ai_b200 import tensor as T

    rng = np.random.default_rng(7)
    x = rng.standard_normal((4, 5, 64), dtype=np.float32)
    g = rng.standard_normal(64, dtype=np.float32)
    x64 = x.astype(np.float64)
    want = x64 / np.sqrt((x64 ** 2).mean(-1, keepdims=True) + 1e-6) * g
    got = T.RMSNorm(_t(x, cuda), _t(g, cuda), 1e-6).cpu().numpy()
    assert np.allclose(got, want, rtol=1e-5, atol=1e-6)
    ss = T.RowSumSquares(_t(x.reshape(20, 64), cuda)).cpu().numpy()
    assert np.allclose(ss, (x64.reshape(20, 64) ** 2).sum(-1), rtol=1e-5)


def test_rope_known_answers(cuda):
    """Angle 1 rad at position 1; position 0 is the identity (rope_test.go:9-25)."""
    from ai_b200 import tensor as T

    got = T.RoPE(_t(np.array([[1, 0]], np.float32), cuda), 10000, [1]).cpu().numpy()
    assert abs(got[0, 0] - math.cos(1)) <= 1e-6 and abs(got[0, 1] - math.sin(1)) <= 1e-6
    x = np.array([[3, -4, 5, 6]], np.float32)
    ident = T.RoPE(_t(x, cuda), 10000, [0]).cpu().numpy()
    assert np.abs(ident - x).max() <= 1e-6
    rng = np.random.default_rng(1)
    y = rng.standard_normal((2, 3, 8, 16), dtype=np.float32)
    r = T.RoPE(_t(y, cuda), 1e6, [0, 5, 9, 100, 500, 1000, 3, 7]).cpu().numpy()
    xn, yn = (y.astype(np.float64) ** 2).sum(-1), (r.astype(np.float64) ** 2).sum(-1)
    assert np.all(np.abs(xn - yn) <= 1e-3 * (xn + 1))


@pytest.mark.parametrize("T,window,lens", [(2048, 0, [2048]), (2048, 257, [2048]),
                                           (1000, 257, [1000, 700]), (129, 0, [129, 1])])
def test_attention_tensor_core_long(cuda, T, window, lens):
    """head_dim 256 runs on the tcgen05 kernel: long global and windowed rows."""
    from ai_b200 import tensor as TT
    import torch

    rng = np.random.default_rng(T + window)
    B = len(lens)
    q = rng.standard_normal((B, 3, T, 256), dtype=np.float32)
    k = rng.standard_normal((B, 1, T, 256), dtype=np.float32)
    v = rng.standard_normal((B, 1, T, 256), dtype=np.float32)
    lens = np.array(lens, np.int32)
    want = _naive_attention(q, k, v, lens, window, 1 / 16)
    got = TT.AttentionScaled(_t(q, cuda), _t(k, cuda), _t(v, cuda), torch.from_numpy(lens),
                             window, 1 / 16).cpu().numpy()
    err = np.abs(got - want).max()
    print(f"\ntc attention T={T} window={window}: max err {err:.3e}")
    assert err <= 1e-4


def test_attention_running_max_rescale(cuda):
    """Scores that grow by far more than 2^8 from one key tile to the next
    exercise the O rescaling in tensor memory."""
    from ai_b200 import tensor as TT

    T = 640
    rng = np.random.default_rng(2)
    q = (np.ones((1, 1, T, 256)) * 0.5 + 0.01 * rng.standard_normal((1, 1, T, 256))).astype(np.float32)
    ramp = np.linspace(0.0, 3.0, T)[None, None, :, None]
    k = (ramp * (1 + 0.01 * rng.standard_normal((1, 1, T, 256)))).astype(np.float32)
    v = rng.standard_normal((1, 1, T, 256), dtype=np.float32)
    want = _naive_attention(q, k, v, None, 0, 1 / 16)
    got = TT.AttentionScaled(_t(q, cuda), _t(k, cuda), _t(v, cuda), None, 0, 1 / 16).cpu().numpy()
    assert np.abs(got - want).max() <= 1e-4, np.abs(got - want).max()
