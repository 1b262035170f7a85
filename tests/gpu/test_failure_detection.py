"""Device-side failure detection on one GPU: a bounded wait that runs out reports, and returns.

The peer-memory collectives wait on flag words that other ranks write. Here the "peer" of a
2-rank exchange is a second local buffer that nothing ever writes, and the wait limit is 5 ms: the
kernel must give up, record its code in the device error word, leave the context usable and (for
the gradient-norm exchange) zero the clip coefficient so AdamW applies nothing. No GPU is faulted
or hung: the wait is bounded and nothing traps.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _native():
    from mia_train_b200.ops._native import native

    return native()


def _flags(dev):
    n = _native()
    words = n.comm_flag_bytes() // 4
    mine = torch.zeros(words, dtype=torch.int32, device=dev)
    silent_peer = torch.zeros(words, dtype=torch.int32, device=dev)  # nobody ever signals here
    return mine, silent_peer


def test_norm_exchange_wait_runs_out(cuda_device):
    from mia_train_b200.ops._native import DeviceWaitError, raise_on_device_errors

    n = _native()
    n.check_errors(cuda_device.index)  # start from a clean error word
    mine, silent = _flags(cuda_device)
    partial = torch.ones(4, device=cuda_device)
    epoch = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    scale = torch.full((), 7.0, device=cuda_device)
    norm = torch.zeros((), device=cuda_device)
    n.zero_norm_exchange([mine.data_ptr(), silent.data_ptr()], partial, epoch, 0, 1.0, scale, norm, 5.0)
    torch.cuda.synchronize(cuda_device)  # the kernel returned
    assert float(scale) == 0.0  # a missing peer: no partial gradient is applied
    with pytest.raises(DeviceWaitError) as info:
        raise_on_device_errors(cuda_device)
    assert info.value.code == 402
    assert n.check_errors(cuda_device.index) == 0  # read-and-clear
    # the context is still usable
    x = torch.randn(64, 64, device=cuda_device)
    assert torch.isfinite(x @ x).all()


def test_reduce_scatter_wait_runs_out(cuda_device):
    n = _native()
    n.check_errors(cuda_device.index)
    mine, silent = _flags(cuda_device)
    grads = [torch.ones(1024, device=cuda_device), torch.ones(1024, device=cuda_device)]
    partial = torch.zeros(8, device=cuda_device)
    epoch = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    n.zero_reduce_scatter([g.data_ptr() for g in grads], [mine.data_ptr(), silent.data_ptr()], 0, 512, partial, epoch,
                          0, 5.0, 0, 128)
    torch.cuda.synchronize(cuda_device)
    assert n.check_errors(cuda_device.index) == 401
    assert torch.all(partial == 0)  # no block summed anything after giving up


def _tp_buffers(dev, gather_bytes, recv_bytes):
    """(flags, gather area, receive area) of one rank of the fused TP kernels, zeroed."""
    n = _native()
    flags = torch.zeros(n.tp_flag_bytes() // 4, dtype=torch.int32, device=dev)
    gather = torch.zeros(2 * gather_bytes, dtype=torch.uint8, device=dev)
    recv = torch.zeros(2 * recv_bytes, dtype=torch.uint8, device=dev)
    return flags, gather, recv


def test_tp_all_gather_gemm_wait_runs_out(cuda_device):
    """Rank 0 of a 2-rank all-gather -> GEMM whose peer never pushes its rows: the GEMM CTAs give up
    on the peer's block flags, the kernel records kErrTpChunkWait (502) and returns."""
    n = _native()
    n.check_errors(cuda_device.index)
    s, k, cols = 256, 128, 256
    gather_bytes = 2 * s * k * 2
    mine = _tp_buffers(cuda_device, gather_bytes, 256)
    silent = _tp_buffers(cuda_device, gather_bytes, 256)  # rank 1: nothing ever runs there
    x = torch.randn(s, k, device=cuda_device).bfloat16()
    w = torch.randn(cols, k, device=cuda_device).bfloat16()
    out = torch.zeros(2 * s, cols, device=cuda_device, dtype=torch.bfloat16)
    full = torch.zeros(2 * s, k, device=cuda_device, dtype=torch.bfloat16)
    n.tp_ag_gemm(x, w, out, full, None, None, None, True, 0, [mine[0].data_ptr(), silent[0].data_ptr()],
                 [mine[1].data_ptr(), silent[1].data_ptr()], gather_bytes, 0, 5.0)
    torch.cuda.synchronize(cuda_device)  # the kernel returned
    assert n.check_errors(cuda_device.index) == 502
    # this rank's own rows were still gathered and computed
    assert torch.equal(full[:s], x)
    ref = x.float() @ w.float().t()
    assert float((out[:s].float() - ref).norm() / ref.norm()) < 1e-2
    # and they were pushed into the peer's gather area (slot 0, parity 1: the first launch) and published
    pushed = silent[1][gather_bytes:].view(torch.bfloat16).view(2, s, k)[0]
    assert torch.equal(pushed, x)
    assert int(silent[0][:4096].max()) == 1


def test_tp_gemm_reduce_scatter_wait_runs_out(cuda_device):
    """Rank 0 of a 2-rank GEMM -> reduce-scatter whose peer never sends its partial rows: the
    producer gives up before adding them, the kernel records kErrTpSlotWait (503) and returns without
    writing the output."""
    n = _native()
    n.check_errors(cuda_device.index)
    s, k, cols = 256, 128, 256
    recv_bytes = 2 * s * cols * 2
    mine = _tp_buffers(cuda_device, 256, recv_bytes)
    silent = _tp_buffers(cuda_device, 256, recv_bytes)
    a = torch.randn(2 * s, k, device=cuda_device).bfloat16()
    w = torch.randn(cols, k, device=cuda_device).bfloat16()
    out = torch.zeros(s, cols, device=cuda_device, dtype=torch.bfloat16)
    n.tp_gemm_rs(a, w, out, None, None, None, None, True, [mine[0].data_ptr(), silent[0].data_ptr()],
                 [mine[2].data_ptr(), silent[2].data_ptr()], recv_bytes, 0, 5.0,
                 torch.eye(128, dtype=torch.bfloat16, device=cuda_device))
    torch.cuda.synchronize(cuda_device)
    assert n.check_errors(cuda_device.index) == 503
    assert int(out.view(torch.int16).abs().max()) == 0
    # the partial rows owned by rank 1 went to its receive slot 0 (parity 1: the first launch)
    slot = silent[2].view(torch.bfloat16)[recv_bytes // 2:].view(2, s, cols)[0]
    ref = a[s:].float() @ w.float().t()
    assert float((slot.float() - ref).norm() / ref.norm()) < 1e-2
