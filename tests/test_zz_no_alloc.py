"""fg_matmul_noalloc: the same product as fg_matmul for callers that cannot
allocate device memory during a call (a host allocator that has reserved
the GPU's memory, a latency-critical path). Its scratch is a fixed 32 MiB
device array in the library. Checked through the C ABI against fg_matmul on
two calls in a row (the second reuses the array the first left behind), and
refused beyond its limit.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _call(fn, x, w, out, epi, transposed, precision):
    import torch

    from ai_b200 import _lib

    m, k = x.shape
    n = out.shape[1]
    ldw = w.stride(1) if transposed else w.stride(0)
    rc = fn(m, n, k, x.data_ptr(), x.stride(0), w.data_ptr(), ldw, int(transposed),
            out.data_ptr(), out.stride(0), C.byref(epi) if epi is not None else None, precision,
            C.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc)


@pytest.mark.parametrize("precision", [0, 1])
def test_noalloc_matches_fg_matmul_twice(cuda, precision):
    import torch

    from ai_b200 import _lib

    lib = _lib.lib()
    rng = np.random.default_rng(123)
    for call, (m, k, n, transposed) in enumerate([(300, 768, 256, False), (257, 1152, 384, True)]):
        a = torch.from_numpy(rng.standard_normal((m, k), dtype=np.float32)).to(cuda)
        wm = rng.standard_normal((n, k) if transposed else (k, n), dtype=np.float32)
        w = torch.from_numpy(wm).to(cuda)
        w = w.t() if transposed else w
        rs = torch.from_numpy(rng.uniform(0.5, 2, m).astype(np.float32)).to(cuda)
        epi = _lib.Epilogue(None, rs.data_ptr(), _lib.ACT_GELU, None, 0, None, 0)
        ref = torch.empty((m, n), dtype=torch.float32, device=cuda)
        got = torch.full((m, n), float("nan"), dtype=torch.float32, device=cuda)
        _call(lib.fg_matmul, a, w, ref, epi, transposed, precision)
        _call(lib.fg_matmul_noalloc, a, w, got, epi, transposed, precision)
        torch.cuda.synchronize()
        r, g = ref.cpu().numpy(), got.cpu().numpy()
        assert np.isfinite(g).all(), f"call {call}"
        assert np.allclose(g, r, rtol=1e-5, atol=1e-5), (call, np.abs(g - r).max())


def test_noalloc_refuses_more_than_its_scratch(cuda):
    import torch

    from ai_b200 import _lib

    m, k, n = 4096, 1024, 1024  # needs 4·(2·m·k + 3·n·k) ≈ 46 MB > 32 MiB
    x = torch.zeros((m, k), device=cuda)
    w = torch.zeros((k, n), device=cuda)
    out = torch.zeros((m, n), device=cuda)
    with pytest.raises(_lib.FGError) as e:
        _call(_lib.lib().fg_matmul_noalloc, x, w, out, None, False, 0)
    assert e.value.code == _lib.FG_EINVAL and "scratch" in str(e.value)
