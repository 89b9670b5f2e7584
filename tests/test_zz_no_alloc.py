"""f16_norm_update_static (library-owned scratch, no allocation) vs f16_norm_update -- needs a B200.

Both entry points are called through the C ABI on the same inputs, twice in a row, so the second
call merges into the running statistics the first produced.  The running mean / var / count
must agree within 1e-6 relative after each call (the two run the same kernels, so in practice
they are identical).  A size whose partial sums do not fit the static array is refused with
F16_ERR_TOO_LARGE before any launch.  This file is named to be collected last, so it also runs
after every other GPU test in the same process.
"""
import ctypes as C

import pytest
import torch

from conftest import pkg_module

pytestmark = pytest.mark.gpu

F16_ERR_TOO_LARGE = 6
STATIC_PAIRS = 131072          # F16_NORM_STATIC_SCRATCH_PAIRS in include/f16env.h
ROWS_PER_BLOCK = 512


def _call_both(lib, _lib, xs, D):
    dev = xs[0].device
    stream = _lib.stream_of(xs[0])
    st_a = [torch.zeros(D, device=dev), torch.ones(D, device=dev), torch.full((1,), 1e-4, device=dev)]
    st_b = [t.clone() for t in st_a]
    for x in xs:
        B = x.shape[0]
        n = int(lib.f16_norm_scratch_doubles(B, D))
        scratch = torch.empty(n, dtype=torch.float64, device=dev)
        _lib.check(lib.f16_norm_update(_lib.ptr(x), B, D, x.stride(0), *[_lib.ptr(t) for t in st_a],
                                       _lib.ptr(scratch), n, stream), "f16_norm_update")
        _lib.check(lib.f16_norm_update_static(_lib.ptr(x), B, D, x.stride(0), *[_lib.ptr(t) for t in st_b],
                                              stream), "f16_norm_update_static")
        torch.cuda.synchronize()
        for name, a, b in zip(("mean", "var", "count"), st_a, st_b):
            torch.testing.assert_close(b, a, rtol=1e-6, atol=0.0, msg=f"{name} after a call of {B} rows")
    return st_a, st_b


def test_static_scratch_matches_caller_scratch_two_calls(cuda):
    _lib = pkg_module("_lib")
    lib = _lib.load()
    g = torch.Generator(device=cuda).manual_seed(17)
    D = 184
    # 262,144 rows (the largest batch the static array takes at D = 184 is 364,544), then a ragged one
    x1 = torch.randn(262144, D, device=cuda, generator=g) * 3.0 + 1.0
    x2 = torch.randn(1000, 200, device=cuda, generator=g)[:, :D] * 0.5 - 2.0    # ldx 200 > D
    a, b = _call_both(lib, _lib, [x1, x2], D)
    assert float(b[2].item()) == pytest.approx(1e-4 + 262144 + 1000, rel=1e-6)


def test_static_scratch_rejects_oversize_without_launch(cuda):
    _lib = pkg_module("_lib")
    lib = _lib.load()
    D = 184
    x = torch.zeros(4, D, device=cuda)
    st = [torch.zeros(D, device=cuda), torch.ones(D, device=cuda), torch.zeros(1, device=cuda)]
    too_many_rows = (STATIC_PAIRS // D + 1) * ROWS_PER_BLOCK      # checked before anything reads x
    rc = lib.f16_norm_update_static(_lib.ptr(x), too_many_rows, D, D, *[_lib.ptr(t) for t in st],
                                    _lib.stream_of(x))
    assert rc == F16_ERR_TOO_LARGE
    assert lib.f16_status_string(rc) == b"size above the documented maximum"
    torch.cuda.synchronize()
    assert float(st[2].item()) == 0.0 and bool((st[0] == 0).all())
