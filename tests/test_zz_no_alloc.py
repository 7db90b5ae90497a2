"""fg_matmul_noalloc: the same product as fg_matmul for callers that cannot
allocate device memory during a call — a host whose own allocator has
reserved the GPU's memory up front (a cudaMalloc inside the library would
fail or fragment that pool), or a latency-critical path that cannot take
cudaMalloc's implicit synchronisation. Its scratch is a fixed 32 MiB device
array in the library.

Checked through the C ABI: bitwise equal to fg_matmul on two calls in a row
(the second reuses the array the first left behind), on shapes that take
the transpose and split paths; the device's free memory unchanged across
repeated calls after the first; refused beyond its limit; and a bounded
wait that gives up inside its kernels reported by fg_synchronize.

This file is collected last on purpose, so that a run that stops at the
first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# (m, k, n, w given as the transposed view of an [n, k] matrix)
SHAPES = [(300, 768, 256, False), (257, 1152, 384, True), (512, 768, 768, True)]


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


def _operands(cuda, rng, m, k, n, transposed):
    import torch

    from ai_b200 import _lib

    a = torch.from_numpy(rng.standard_normal((m, k), dtype=np.float32)).to(cuda)
    wm = rng.standard_normal((n, k) if transposed else (k, n), dtype=np.float32)
    w = torch.from_numpy(wm).to(cuda)
    w = w.t() if transposed else w
    rs = torch.from_numpy(rng.uniform(0.5, 2, m).astype(np.float32)).to(cuda)
    epi = _lib.Epilogue(None, rs.data_ptr(), _lib.ACT_GELU, None, 0, None, 0)
    return a, w, rs, epi


@pytest.mark.parametrize("precision", [0, 1])
def test_noalloc_matches_fg_matmul_twice(cuda, precision):
    import torch

    from ai_b200 import _lib

    lib = _lib.lib()
    rng = np.random.default_rng(123)
    for call, (m, k, n, transposed) in enumerate(SHAPES[:2]):
        a, w, rs, epi = _operands(cuda, rng, m, k, n, transposed)
        ref = torch.empty((m, n), dtype=torch.float32, device=cuda)
        got = torch.full((m, n), float("nan"), dtype=torch.float32, device=cuda)
        _call(lib.fg_matmul, a, w, ref, epi, transposed, precision)
        _call(lib.fg_matmul_noalloc, a, w, got, epi, transposed, precision)
        _lib.check(lib.fg_synchronize(0))
        # same split / transpose kernels and the same GEMM on the same layout
        assert torch.equal(got, ref), (call, float((got - ref).abs().max()))


def test_noalloc_takes_no_device_memory(cuda):
    """After a first call (which loads the module holding the array), further
    calls on every path leave the device's free memory exactly unchanged."""
    import torch

    from ai_b200 import _lib

    lib = _lib.lib()
    rng = np.random.default_rng(7)
    cases = []
    for m, k, n, transposed in SHAPES:
        a, w, rs, epi = _operands(cuda, rng, m, k, n, transposed)
        out = torch.empty((m, n), dtype=torch.float32, device=cuda)
        cases.append((a, w, rs, epi, out, transposed))
    # first calls: the module holding the array and every kernel these
    # calls launch are loaded (lazy loading may take device memory for them)
    for precision in (0, 1):
        for a, w, rs, epi, out, transposed in cases:
            _call(lib.fg_matmul_noalloc, a, w, out, epi, transposed, precision)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        for precision in (0, 1):
            for a, w, rs, epi, out, transposed in cases:
                _call(lib.fg_matmul_noalloc, a, w, out, epi, transposed, precision)
    _lib.check(lib.fg_synchronize(0))
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)


def test_noalloc_refuses_more_than_its_scratch(cuda):
    import torch

    from ai_b200 import _lib

    m, k, n = 256, 1024, 8192  # w as [k, n]: transposed copy + low part = 4·2·n·k = 64 MiB > 32 MiB
    x = torch.zeros((m, k), device=cuda)
    w = torch.zeros((k, n), device=cuda)
    out = torch.zeros((m, n), device=cuda)
    with pytest.raises(_lib.FGError) as e:
        _call(_lib.lib().fg_matmul_noalloc, x, w, out, None, False, 0)
    assert e.value.code == _lib.FG_EINVAL and "scratch" in str(e.value)


def test_noalloc_wait_timeout_is_reported(cuda):
    """A pipeline wait that runs out inside the entry point's own kernels
    (a 1 µs limit against a K = 8192 main loop) is reported by the next
    fg_synchronize as FG_ETIMEOUT, and the next call with the default limit
    gives fg_matmul's result again."""
    import torch

    from ai_b200 import _lib

    lib = _lib.lib()
    rng = np.random.default_rng(11)
    m, k, n = 512, 8192, 512
    a, w, rs, epi = _operands(cuda, rng, m, k, n, True)
    ref = torch.empty((m, n), dtype=torch.float32, device=cuda)
    got = torch.empty((m, n), dtype=torch.float32, device=cuda)
    _call(lib.fg_matmul, a, w, ref, epi, True, 1)
    _lib.check(lib.fg_synchronize(0))
    _call(lib.fg_matmul_noalloc, a, w, got, epi, True, 1)  # set-up before the limit changes
    _lib.check(lib.fg_synchronize(0))
    try:
        _lib.check(lib.fg_set_wait_limit(0, 1000))
        _call(lib.fg_matmul_noalloc, a, w, got, epi, True, 1)
        rc = lib.fg_synchronize(0)
    finally:
        _lib.check(lib.fg_set_wait_limit(0, 0))
    assert rc == _lib.FG_ETIMEOUT, rc
    assert lib.fg_synchronize(0) == _lib.FG_OK  # the record was cleared
    got.fill_(float("nan"))
    _call(lib.fg_matmul_noalloc, a, w, got, epi, True, 1)
    _lib.check(lib.fg_synchronize(0))
    assert torch.equal(got, ref)
