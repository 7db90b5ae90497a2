"""The standalone tensor.MatMul sweep (tensor/matmul.go:19-72 on
internal/blas, whose own test is internal/blas/gemm_test.go:91-145), at
every shape of the sweep: M ∈ {128, 1024, 8192, 65536} × (K, N) ∈
{768} × {768, 1152, 2304, 3072} plus (1152, 768); each as A·B (B [K, N]
row-major) and as A·Wᵀ (the transposed view of an [N, K] matrix, no copy,
the `w.T()` case); in split precision (fp32-level) and in plain TF32.
Entries are i.i.d. N(0, 1) from seed 3.

Bounds:
- split: |C − C64| ≤ 1e-4·(1 + |C64|) (the reference's bound) or
  REL_SPLIT·‖a_i‖·‖w_j‖. The second term is the size of the tensor core's
  fp32 accumulation error, which grows with the operands' norms, not with
  |C|: measured ≤ 1.1e-6 of ‖a_i‖‖w_j‖ for the split-fp16 products (M ≥
  256: A and B in two fp16 parts each, three passes) and ≤ 1.4e-6 for the
  split-TF32 ones (M = 128).
- plain TF32: the same against the float64 product of the operands with
  their low 13 mantissa bits cleared (the bits the tensor core reads).
- split, first 128 rows: against the reference's own float32 arithmetic
  (the oracle's ORC_F32 GEMM: sequential fused multiply-adds, as
  internal/blas accumulates) within the split bound plus that arithmetic's
  own error.

Set FG_MATMUL_RECORD=<file> to write every case's measured maxima as JSON.
"""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MS = [128, 1024, 8192, 65536]
KN = [(768, 768), (768, 1152), (768, 2304), (768, 3072), (1152, 768)]
REL_SPLIT = 2e-6
REL_TF32 = 3e-6
REL_REF32 = 3e-7  # the float32 reference arithmetic's own error, ≤ 2.1e-7 of ‖a‖‖w‖ here
CHUNK = 8192

_RECORD = []


@pytest.fixture(scope="module", autouse=True)
def _write_record():
    yield
    path = os.environ.get("FG_MATMUL_RECORD")
    if path and _RECORD:
        with open(path, "w") as f:
            json.dump(_RECORD, f, indent=1)


def _trunc(t):
    import torch

    return (t.view(torch.int32) & 0xFFFFE000).view(torch.float32)


@pytest.mark.parametrize("m", MS)
@pytest.mark.parametrize("k,n", KN)
@pytest.mark.parametrize("transposed", [False, True])
@pytest.mark.parametrize("prec", ["split", "tf32"])
def test_matmul_sweep(cuda, m, k, n, transposed, prec):
    import torch

    from ai_b200 import tensor as T

    g = torch.Generator(device=cuda).manual_seed(3)
    a = torch.randn(m, k, generator=g, device=cuda, dtype=torch.float32)
    if transposed:
        w = torch.randn(n, k, generator=g, device=cuda, dtype=torch.float32).t()  # [k, n] view
    else:
        w = torch.randn(k, n, generator=g, device=cuda, dtype=torch.float32)
    precision = T.PREC_SPLIT if prec == "split" else T.PREC_TF32
    got = T.MatMul(a, w, precision=precision)
    torch.cuda.synchronize()
    a_ref = a if prec == "split" else _trunc(a)
    w_ref = (w if prec == "split" else _trunc(w.contiguous())).double()
    wn = w.double().norm(dim=0)[None, :]
    rel = REL_SPLIT if prec == "split" else REL_TF32
    worst_abs = worst_scaled = worst_refbound = 0.0
    bad = 0
    for r0 in range(0, m, CHUNK):
        ar = a_ref[r0:r0 + CHUNK].double()
        want = ar @ w_ref
        err = (got[r0:r0 + CHUNK].double() - want).abs()
        scale = a[r0:r0 + CHUNK].double().norm(dim=1)[:, None] * wn
        ref_bound = 1e-4 * (1 + want.abs())
        ok = (err <= ref_bound) | (err <= rel * scale)
        bad += int((~ok).sum())
        worst_abs = max(worst_abs, err.max().item())
        worst_scaled = max(worst_scaled, (err / scale).max().item())
        worst_refbound = max(worst_refbound, (err / ref_bound).max().item())
        del want, err, scale, ref_bound, ok
    rec = {"m": m, "k": k, "n": n, "transposed": transposed, "precision": prec,
           "max_abs": worst_abs, "max_err_over_norms": worst_scaled,
           "max_err_over_ref_bound": worst_refbound}
    if prec == "split" and m <= 1024:
        from oracle import oracle as O

        a32 = a[:128].cpu().numpy()
        w32 = w.contiguous().cpu().numpy()
        ref32 = O.matmul_fused(a32, w32, mode=O.F32)
        d = np.abs(got[:128].cpu().numpy().astype(np.float64) - ref32)
        sc = np.linalg.norm(a32.astype(np.float64), axis=1)[:, None] * \
            np.linalg.norm(w32.astype(np.float64), axis=0)[None, :]
        ok32 = (d <= 1e-4 * (1 + np.abs(ref32))) | (d <= (REL_SPLIT + REL_REF32) * sc)
        rec["vs_reference_f32_max_abs"] = float(d.max())
        bad += int((~ok32).sum())
    _RECORD.append(rec)
    print(rec)
    assert bad == 0, rec
