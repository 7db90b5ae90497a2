"""Host-side checks of the split-fp16 product the encoder GEMMs use
(ai_b200/csrc/fg_gemm.cu, gemm_pair_kernel<..., H16>), restated in numpy:

- the row exponent from the RMS row scale keeps every scaled element below
  2^14, so both fp16 parts are finite;
- A = hi + lo with hi = a's top 11 significant bits (exact in fp16) and lo =
  fp16(a − hi) keeps 22 significant bits of a, down to 2^-17 of the bound;
- a bf16 weight times a power of two is exactly an fp16 value;
- A_hi·B + A_lo·B, unscaled, matches the float64 product to split-TF32's
  accuracy;
- the GeGLU epilogue's x·σ(2u) is the tanh-GELU 0.5·x·(1 + tanh(u)).

No GPU: these pin the arithmetic the kernels implement, not the kernels.
"""
import numpy as np


def _tf32_hi(x: np.ndarray) -> np.ndarray:
    u = np.asarray(x, np.float32).view(np.uint32) & np.uint32(0xFFFFE000)
    return u.view(np.float32)


def _row_exp_from_rs(rs: np.ndarray, k: int) -> np.ndarray:
    # e_r = 13 - ilogb(sqrt(K) / rs): the kernel's a_row_exp
    b = np.float32(np.sqrt(np.float32(k))) / rs.astype(np.float32)
    return 13 - np.floor(np.log2(b.astype(np.float64))).astype(np.int64)


def _split(a: np.ndarray):
    hi = _tf32_hi(a)
    lo = (a - hi).astype(np.float16)
    return hi.astype(np.float16), lo


def test_row_exponent_bounds_scaled_rows():
    rng = np.random.default_rng(3)
    k, eps = 768, 1e-6
    for scale in (1e-3, 1.0, 40.0, 3e3):
        x = (rng.standard_normal((64, k)) * scale).astype(np.float32)
        x[0, :] = 0
        x[1, :] = 0
        x[1, 5] = scale * 50  # one dominant element: max|x| = ‖x‖
        ms = (x.astype(np.float64) ** 2).mean(1)
        rs = (1.0 / np.sqrt(ms + eps)).astype(np.float32)
        e = _row_exp_from_rs(rs, k)
        scaled = np.abs(x.astype(np.float64)) * np.exp2(e)[:, None]
        assert scaled.max() < 2.0 ** 14
        hi, lo = _split((x * np.exp2(e)[:, None].astype(np.float32)).astype(np.float32))
        assert np.isfinite(hi).all() and np.isfinite(lo).all()


def test_hi_is_exact_and_parts_keep_22_bits():
    rng = np.random.default_rng(4)
    a = (rng.standard_normal(200_000) * np.exp2(rng.uniform(-16, 13.9, 200_000))).astype(np.float32)
    a = a[np.abs(a) < 2.0 ** 14]
    hi, lo = _split(a)
    h32 = _tf32_hi(a)
    normal = np.abs(h32) >= 2.0 ** -14
    assert np.array_equal(hi.astype(np.float32)[normal], h32[normal])
    err = np.abs(a.astype(np.float64) - hi.astype(np.float64) - lo.astype(np.float64))
    big = np.abs(a) >= 2.0 ** -3  # 2^-17 of the 2^14 bound
    assert (err[big] <= 2.0 ** -22 * np.abs(a[big].astype(np.float64))).all()
    # below 2^-14 both parts round on fp16's subnormal grid: 2^-25 each
    assert (err <= 2.0 ** -22 * np.abs(a.astype(np.float64)) + 2.0 ** -24).all()


def test_bf16_weights_are_fp16_exact_under_one_power_of_two():
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((256, 768)) * 0.02).astype(np.float32)
    w = (w.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)  # bf16 values
    t = 13 - int(np.floor(np.log2(np.abs(w).max())))
    s = w * np.float32(2.0 ** t)
    assert np.abs(s).max() < 2.0 ** 14
    assert np.array_equal(s.astype(np.float16).astype(np.float32), s)


def test_split_product_matches_float64():
    rng = np.random.default_rng(6)
    m, k, n, eps = 48, 768, 64, 1e-6
    a = (rng.standard_normal((m, k)) * np.exp2(rng.uniform(-4, 6, (m, 1)))).astype(np.float32)
    w = (rng.standard_normal((n, k)) * 0.03).astype(np.float32)
    w = (w.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)
    rs = (1.0 / np.sqrt((a.astype(np.float64) ** 2).mean(1) + eps)).astype(np.float32)
    e = _row_exp_from_rs(rs, k)
    t = 13 - int(np.floor(np.log2(np.abs(w).max())))
    b16 = (w * np.float32(2.0 ** t)).astype(np.float16).astype(np.float64)
    hi, lo = _split((a * np.exp2(e)[:, None].astype(np.float32)).astype(np.float32))
    prod = (hi.astype(np.float64) @ b16.T + lo.astype(np.float64) @ b16.T) * np.exp2(-(e + t))[:, None]
    ref = a.astype(np.float64) @ w.astype(np.float64).T
    bound = 2.0 ** -21 * np.linalg.norm(a, axis=1)[:, None] * np.linalg.norm(w, axis=1)[None, :]
    assert (np.abs(prod - ref) <= bound).all()


def test_gelu_sigmoid_form_equals_tanh_form():
    x = np.linspace(-12, 12, 200_001)
    c = np.sqrt(2.0 / np.pi)
    u = c * (x + 0.044715 * x ** 3)
    tanh_form = 0.5 * x * (1.0 + np.tanh(u))
    with np.errstate(over="ignore"):
        sig_form = x / (1.0 + np.exp2(-2.0 * u / np.log(2.0)))
    # the tanh form flushes the far negative tail to -0 (1 + tanh = 0 in
    # float64); the sigmoid form keeps it, below 1e-15 there
    assert np.allclose(sig_form, tanh_form, rtol=1e-12, atol=1e-15)


def test_static_bounds_of_attention_output_and_gated_activations():
    """The model's split-fp16 exponents for the O and down inputs come from
    bounds on the weights alone (fg_model.cu, finalize): with rs =
    1/sqrt(mean(x²) + eps), ‖rs·x‖ < sqrt(H), so |v| < sqrt(H)·max‖W'_v row‖
    and any convex combination of v rows (the attention output) too; and
    |GELU(g)·u| < max(sqrt(H)‖W'_g row‖, 0.2)·sqrt(H)‖W'_u row‖."""
    rng = np.random.default_rng(7)
    h, f, d, eps = 768, 1152, 256, 1e-6
    gain = (1.0 + 0.3 * rng.standard_normal(h)).astype(np.float32)
    wv = (rng.standard_normal((d, h)) * 0.05).astype(np.float32) * gain
    wg = (rng.standard_normal((f, h)) * 0.05).astype(np.float32) * gain
    wu = (rng.standard_normal((f, h)) * 0.05).astype(np.float32) * gain
    x = (rng.standard_normal((512, h)) * np.exp2(rng.uniform(-6, 8, (512, 1)))).astype(np.float64)
    x[:8] = wv[:8] / np.linalg.norm(wv[:8], axis=1, keepdims=True) * 1e3  # aligned with W'_v rows
    rs = 1.0 / np.sqrt((x ** 2).mean(1) + eps)
    xs = x * rs[:, None]
    sh = np.sqrt(h)
    bv = sh * np.linalg.norm(wv.astype(np.float64), axis=1).max()
    v = xs @ wv.T.astype(np.float64)
    assert np.abs(v).max() < bv
    p = rng.dirichlet(np.ones(512), size=64)  # softmax rows: convex weights
    assert np.abs(p @ v).max() < bv
    g = xs @ wg.T.astype(np.float64)
    u = xs @ wu.T.astype(np.float64)
    c = np.sqrt(2.0 / np.pi)
    gelu = g / (1.0 + np.exp(-2.0 * c * (g + 0.044715 * g ** 3)))
    bg = sh * np.linalg.norm(wg.astype(np.float64), axis=1)
    bu = sh * np.linalg.norm(wu.astype(np.float64), axis=1)
    assert np.abs(gelu * u).max() < (np.maximum(bg, 0.2) * bu).max()
