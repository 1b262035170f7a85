"""The fused TP collective GEMMs on one GPU (a TP group of one) against fp32 PyTorch.

With one rank the all-gather is a local copy and the reduce-scatter a sum over one slot, so these
tests check the GEMM, the epilogues (bias, GELU with the pre-activation kept, GELU', LayerScale,
residual), both operand layouts, ragged row counts and the alternation of the double-buffered
workspace over consecutive launches. The multi-rank transfer is checked by test_tp_multi.py.
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.distributed as dist

pytestmark = pytest.mark.gpu

needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs CUDA")


@pytest.fixture(scope="module")
def group(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    created = False
    if not dist.is_initialized():
        init = tmp_path_factory.mktemp("pg") / "init"
        dist.init_process_group("gloo", init_method=f"file://{init}", rank=0, world_size=1)
        created = True
    yield dist.group.WORLD
    if created:
        dist.destroy_process_group()


def _gelu_grad(h):
    h = h.float()
    return 0.5 * (1 + torch.erf(h / math.sqrt(2))) + h * torch.exp(-0.5 * h * h) / math.sqrt(2 * math.pi)


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-6))


@needs_cuda
@pytest.mark.parametrize("m,k,n,b_kmajor", [(1000, 256, 768, True), (512, 1024, 256, False), (384, 192, 1024, True)])
def test_ag_gemm_one_rank(group, m, k, n, b_kmajor):
    from mia_train_b200.ops import _native
    from mia_train_b200.ops.linear import ACT_DGELU, ACT_GELU, ACT_NONE
    from mia_train_b200.ops.tp import TpComm, ag_gemm

    dev = torch.device("cuda", 0)
    comm = TpComm(group, "fused")
    g = torch.Generator(device=dev).manual_seed(m + k + n)
    x = torch.randn(m, k, device=dev, generator=g).bfloat16()
    w = (torch.randn(n, k, device=dev, generator=g) / math.sqrt(k)).bfloat16()
    wb = w if b_kmajor else w.t().contiguous()
    bias = torch.randn(n, device=dev, generator=g)
    ref = x.float() @ w.float().t()
    # three launches in a row (workspace parities 1, 0, 1)
    out, full, _ = ag_gemm(comm, x, wb, b_kmajor=b_kmajor, bias=bias, act=ACT_NONE)
    assert torch.equal(full, x)
    assert _rel(out, ref + bias) < 1e-2
    out, full, pre = ag_gemm(comm, x, wb, b_kmajor=b_kmajor, bias=bias, act=ACT_GELU, want_pre=True)
    assert _rel(pre, ref + bias) < 1e-2
    assert _rel(out, torch.nn.functional.gelu(ref + bias)) < 1e-2
    aux = torch.randn(m, n, device=dev, generator=g).bfloat16()
    out, _, _ = ag_gemm(comm, x, wb, b_kmajor=b_kmajor, act=ACT_DGELU, aux=aux)
    assert _rel(out, ref * _gelu_grad(aux)) < 1e-2
    torch.cuda.synchronize()
    assert _native.native().check_errors(0) == 0
    comm.release()


@needs_cuda
@pytest.mark.parametrize("m,k,n,b_kmajor", [(1000, 256, 1024, True), (640, 768, 1024, False), (256, 128, 256, True)])
def test_gemm_rs_one_rank(group, m, k, n, b_kmajor):
    from mia_train_b200.ops import _native
    from mia_train_b200.ops.tp import TpComm, gemm_rs

    dev = torch.device("cuda", 0)
    comm = TpComm(group, "fused")
    g = torch.Generator(device=dev).manual_seed(m * 3 + k + n)
    a = torch.randn(m, k, device=dev, generator=g).bfloat16()
    w = (torch.randn(n, k, device=dev, generator=g) / math.sqrt(k)).bfloat16()
    wb = w if b_kmajor else w.t().contiguous()
    bias = torch.randn(n, device=dev, generator=g)
    gamma = torch.rand(n, device=dev, generator=g) + 0.5
    res = torch.randn(m, n, device=dev, generator=g).bfloat16()
    prod = a.float() @ w.float().t()
    for _ in range(3):
        out, pre = gemm_rs(comm, a, wb, b_kmajor=b_kmajor, bias=bias, gamma=gamma, residual=res, want_pre=True)
        assert _rel(pre, prod + bias) < 1e-2
        assert _rel(out, res.float() + gamma * (prod + bias)) < 1e-2
    out, pre = gemm_rs(comm, a, wb, b_kmajor=b_kmajor)
    assert pre is None
    assert _rel(out, prod) < 1e-2
    torch.cuda.synchronize()
    assert _native.native().check_errors(0) == 0
    comm.release()


@needs_cuda
def test_sequence_parallel_block_one_rank(group):
    """A DINOv3 block through the sequence-parallel path (one rank, fused kernels) vs the plain block."""
    import copy

    from mia_train_b200.models.dinov3_vit3d import DinoVisionTransformer3D
    from mia_train_b200.ops import _native
    from mia_train_b200.ops.tp import TpComm
    from mia_train_b200.parallel.sequence_parallel import SequenceParallel, sync_partial_grads
    from mia_train_b200.parallel.tensor_parallel import apply_tensor_parallel

    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    dense = DinoVisionTransformer3D(img_size=32, patch_size=4, embed_dim=256, depth=2, num_heads=4,
                                    n_storage_tokens=4, layerscale_init=0.5, window_size=4, global_every=2).to(dev)
    sp = copy.deepcopy(dense)
    apply_tensor_parallel(sp.tensor_parallel_plan(), group)
    sp.enable_sequence_parallel(SequenceParallel(TpComm(group, "fused")))
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(2, 1, 32, 32, 32, device=dev, generator=g)
    w = torch.randn(2, 512, 256, device=dev, generator=g)

    def loss_of(model):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = model.forward_features(x)
        return (out["x_norm_patchtokens"].float() * w).sum()

    ref = loss_of(dense)
    ref.backward()
    loss = loss_of(sp)
    loss.backward()
    sync_partial_grads(sp)
    assert abs(float(loss) - float(ref)) < 2e-2 * max(1.0, abs(float(ref)))
    dense_p = dict(dense.named_parameters())
    for name, p in sp.named_parameters():
        if p.grad is None:
            continue
        assert _rel(p.grad, dense_p[name].grad) < 0.05, name
    torch.cuda.synchronize()
    assert _native.native().check_errors(0) == 0
    sp._sequence_parallel.comm.release()
