"""The allocation-free attention backward, called through its exported C symbol.

`mia_attention_bwd_noalloc` exists for callers that may not allocate device memory themselves (a
host runtime or plugin that owns the GPU memory budget and hands out only buffers it manages). It
keeps its scratch in a fixed device array inside the library. This test calls it twice in a row on
different inputs -- so the second call runs on scratch the first one left behind -- and compares
each result with the allocating `attention_bwd` binding, within the tolerance the kernel tests use.
It also checks that a problem larger than the fixed scratch is refused before anything launches.

Kept in its own file, in a directory that sorts after every other test directory, so pytest
collects it last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs CUDA", allow_module_level=True)

DEV = torch.device("cuda", 0)
MAX_SCRATCH_FLOATS = 1 << 21
ERR_TOO_LARGE = -2


def _library() -> ctypes.CDLL:
    import mia_train_b200._C as ext

    lib = ctypes.CDLL(ext.__file__)
    fn = lib.mia_attention_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_void_p] + [ctypes.c_void_p] * 3 + [ctypes.c_int] * 5 + [
        ctypes.c_float,
        ctypes.c_void_p,
    ]
    return lib


def _problem(seed: int, b: int, h: int, n: int, d: int):
    import mia_train_b200._C as ext

    g = torch.Generator(device=DEV).manual_seed(seed)
    q, k, v = (torch.randn(b, h, n, d, device=DEV, generator=g).bfloat16() for _ in range(3))
    o = torch.empty(b, n, h, d, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(b, h, n, device=DEV, dtype=torch.float32)
    scale = d**-0.5
    ext.attention_fwd(q, k, v, o, lse, scale)
    dout = torch.randn(b, n, h, d, device=DEV, generator=g).bfloat16()
    return q, k, v, o, dout, lse, scale


def _call(lib, q, k, v, o, dout, lse, scale):
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    b, h, n, d = q.shape
    stream = torch.cuda.current_stream(DEV).cuda_stream
    rc = lib.mia_attention_bwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dout.data_ptr(), lse.data_ptr(),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), b, h, n, n, d, scale, stream,
    )
    return rc, dq, dk, dv


def _reference(q, k, v, o, dout, lse, scale):
    import mia_train_b200._C as ext

    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ext.attention_bwd(q, k, v, o, dout, lse, dq, dk, dv, scale)
    return dq, dk, dv


def _close(actual, expected, rel=2e-2, atol=2e-2):
    a, e = actual.float(), expected.float()
    err = (a - e).abs().max().item()
    assert err <= atol + rel * (e.abs().max().item() + 1e-6), f"max error {err:.4g}"


def test_noalloc_matches_allocating_entry_point_twice():
    torch.cuda.set_device(DEV)
    lib = _library()
    for seed, shape in ((11, (2, 4, 128, 64)), (12, (1, 3, 200, 32))):
        prob = _problem(seed, *shape)
        rc, dq, dk, dv = _call(lib, *prob)
        assert rc == 0
        torch.cuda.synchronize()
        rq, rk, rv = _reference(*prob)
        torch.cuda.synchronize()
        _close(dq, rq)
        _close(dk, rk)
        _close(dv, rv)


def test_noalloc_rejects_oversized_problem():
    lib = _library()
    b, h, n, d = 4, 16, 1024, 64  # needs b*h*n*(d+1) > the fixed scratch
    assert b * h * n * (d + 1) > MAX_SCRATCH_FLOATS
    rc = lib.mia_attention_bwd_noalloc(*([None] * 9), b, h, n, n, d, 0.125, None)
    assert rc == ERR_TOO_LARGE
