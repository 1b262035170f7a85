"""The allocation-free attention backward, called through its exported C symbol.

`mia_attention_bwd_noalloc` exists for callers that may not allocate device memory themselves (a
host runtime or plugin that owns the GPU memory budget and hands out only buffers it manages). It
keeps its scratch in a fixed device array inside the library. This test calls it three times in a
row on different inputs -- so every later call runs on scratch the one before left behind -- and
compares each result with the allocating `attention_bwd` binding and with an fp32 PyTorch autograd
gradient, within the tolerance the kernel tests use. The third call uses head dim 128 and more keys
than queries, so the fallback kernel and the cross-attention strides are covered too. It also checks
that a problem larger than the fixed scratch, or a misaligned pointer, is refused before anything
launches.

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
ERR_ARGS = -1
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


def _problem(seed: int, b: int, h: int, nq: int, d: int, nk: int | None = None):
    import mia_train_b200._C as ext

    nk = nq if nk is None else nk
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.randn(b, h, nq, d, device=DEV, generator=g).bfloat16()
    k, v = (torch.randn(b, h, nk, d, device=DEV, generator=g).bfloat16() for _ in range(2))
    o = torch.empty(b, nq, h, d, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(b, h, nq, device=DEV, dtype=torch.float32)
    scale = d**-0.5
    ext.attention_fwd(q, k, v, o, lse, scale)
    dout = torch.randn(b, nq, h, d, device=DEV, generator=g).bfloat16()
    return q, k, v, o, dout, lse, scale


def _call(lib, q, k, v, o, dout, lse, scale):
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    b, h, nq, d = q.shape
    nk = k.shape[2]
    stream = torch.cuda.current_stream(DEV).cuda_stream
    rc = lib.mia_attention_bwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dout.data_ptr(), lse.data_ptr(),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), b, h, nq, nk, d, scale, stream,
    )
    return rc, dq, dk, dv


def _reference(q, k, v, o, dout, lse, scale):
    import mia_train_b200._C as ext

    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ext.attention_bwd(q, k, v, o, dout, lse, dq, dk, dv, scale)
    return dq, dk, dv


def _oracle(q, k, v, o, dout, lse, scale):
    """fp32 PyTorch autograd gradients of sum(softmax(q k^T scale) v * dout)."""
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    p = torch.softmax(qf @ kf.transpose(-1, -2) * scale, dim=-1)
    out = (p @ vf).permute(0, 2, 1, 3)  # (B, Nq, H, D), the layout of dout
    (out * dout.float()).sum().backward()
    return qf.grad, kf.grad, vf.grad


def _close(actual, expected, rel=2e-2, atol=2e-2):
    a, e = actual.float(), expected.float()
    err = (a - e).abs().max().item()
    assert err <= atol + rel * (e.abs().max().item() + 1e-6), f"max error {err:.4g}"


def test_noalloc_matches_allocating_entry_point_and_fp32_oracle():
    torch.cuda.set_device(DEV)
    lib = _library()
    for seed, shape in ((11, (2, 4, 128, 64)), (12, (1, 3, 200, 32)), (13, (1, 2, 96, 128, 160))):
        prob = _problem(seed, *shape)
        rc, dq, dk, dv = _call(lib, *prob)
        assert rc == 0
        torch.cuda.synchronize()
        rq, rk, rv = _reference(*prob)
        fq, fk, fv = _oracle(*prob)
        torch.cuda.synchronize()
        for got, alloc, exact in ((dq, rq, fq), (dk, rk, fk), (dv, rv, fv)):
            _close(got, alloc)
            _close(got, exact)


def test_noalloc_rejects_oversized_problem():
    lib = _library()
    b, h, n, d = 4, 16, 1024, 64  # needs b*h*n*(d+1) > the fixed scratch
    assert b * h * n * (d + 1) > MAX_SCRATCH_FLOATS
    rc = lib.mia_attention_bwd_noalloc(*([None] * 9), b, h, n, n, d, 0.125, None)
    assert rc == ERR_TOO_LARGE


def test_noalloc_rejects_misaligned_pointer():
    torch.cuda.set_device(DEV)
    lib = _library()
    q, k, v, o, dout, lse, scale = _problem(14, 1, 2, 64, 64)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    rc = lib.mia_attention_bwd_noalloc(
        q.data_ptr() + 2, k.data_ptr(), v.data_ptr(), o.data_ptr(), dout.data_ptr(), lse.data_ptr(),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), 1, 2, 63, 64, 64, scale, stream,
    )
    assert rc == ERR_ARGS
