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
