"""Sequence-parallel tensor parallelism on CPU (Gloo, 2 and 4 ranks) against the dense model.

The same fp32 DINOv3 3-D backbone (global and windowed blocks, LayerScale, register tokens) runs
dense and sharded with its tensor-parallel plan plus sequence parallelism (`tp_comm = "fused"`
takes the collective path on CPU). Loss, every replicated parameter's gradient (after the
sequence-parallel partial sums are synchronised) and every gathered sharded gradient must match.
"""

from __future__ import annotations

import copy

import pytest
import torch

pytestmark = pytest.mark.cpu_dist


def _loss(model, x, w, wc):
    out = model.forward_features(x)
    return (out["x_norm_patchtokens"] * w).sum() + (out["x_norm_clstoken"] * wc).sum()


def _sp_vs_dense(rank, world, window):
    import torch.distributed as dist

    from mia_train_b200.models.dinov3_vit3d import DinoVisionTransformer3D
    from mia_train_b200.ops.tp import TpComm
    from mia_train_b200.parallel.sequence_parallel import SequenceParallel, partial_params, sync_partial_grads
    from mia_train_b200.parallel.tensor_parallel import apply_tensor_parallel, is_tensor_parallel

    torch.manual_seed(0)
    dense = DinoVisionTransformer3D(img_size=16, patch_size=4, embed_dim=32, depth=2, num_heads=4,
                                    n_storage_tokens=2, layerscale_init=0.5, window_size=window,
                                    global_every=2 if window else 0)
    tp = copy.deepcopy(dense)
    group = dist.group.WORLD
    apply_tensor_parallel(tp.tensor_parallel_plan(), group)
    tp.enable_sequence_parallel(SequenceParallel(TpComm(group, "fused")))
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 1, 16, 16, 16, generator=g)
    w = torch.randn(2, 64, 32, generator=g)
    wc = torch.randn(2, 32, generator=g)
    ref = _loss(dense, x, w, wc)
    ref.backward()
    loss = _loss(tp, x, w, wc)
    loss.backward()
    n_partial = sync_partial_grads(tp)
    dense_params = dict(dense.named_parameters())
    worst = 0.0
    for name, p in tp.named_parameters():
        rg = dense_params[name].grad
        if p.grad is None:
            assert rg is None or float(rg.abs().max()) == 0.0, name
            continue
        mod = tp.get_submodule(name.rsplit(".", 1)[0]) if "." in name else tp
        gp = p.grad
        if is_tensor_parallel(mod) and p.shape != rg.shape:
            parts = [torch.empty_like(gp) for _ in range(world)]
            dist.all_gather(parts, gp.contiguous())
            if mod._tp_mode == "qkv":
                per = gp.shape[0] // 3
                gp = torch.cat([parts[r][q * per:(q + 1) * per] for q in range(3) for r in range(world)])
            elif mod._tp_mode == "column" or gp.dim() == 1:
                gp = torch.cat(parts, dim=0)
            else:
                gp = torch.cat(parts, dim=1)
        err = float((gp - rg).norm() / (rg.norm() + 1e-12))
        worst = max(worst, err)
        assert err < 1e-4, (name, err)
    return float(loss), float(ref), worst, n_partial, len(partial_params(tp))


@pytest.mark.parametrize("world,window", [(2, 0), (2, 2), (4, 2)])
def test_sequence_parallel_matches_dense(run_distributed, world, window):
    res = run_distributed(_sp_vs_dense, world, window)
    for loss, ref, worst, n_partial, n_marked in res.values():
        assert abs(loss - ref) < 1e-4 * max(1.0, abs(ref)), (loss, ref)
        assert n_partial == n_marked == 2 * 6  # norm1 / norm2 weight + bias, ls1 / ls2 gamma per block
        assert worst < 1e-4


def _gathered_grad(p, mod, world, dense_shape):
    import torch.distributed as dist

    from mia_train_b200.parallel.tensor_parallel import is_tensor_parallel

    gp = p.grad
    if not is_tensor_parallel(mod) or p.shape == dense_shape:
        return gp
    parts = [torch.empty_like(gp) for _ in range(world)]
    dist.all_gather(parts, gp.contiguous())
    if mod._tp_mode == "qkv":
        per = gp.shape[0] // 3
        return torch.cat([parts[r][q * per:(q + 1) * per] for q in range(3) for r in range(world)])
    if mod._tp_mode == "column" or gp.dim() == 1:
        return torch.cat(parts, dim=0)
    return torch.cat(parts, dim=1)


def _affinity_split_vs_dense(rank, world, batch):
    import torch.distributed as dist

    from mia_train_b200.algorithms.affinity_seg import AffinitySegmentation
    from mia_train_b200.data.synthetic import voronoi_volume
    from mia_train_b200.models.dinov3_vit3d import DinoVisionTransformer3D
    from mia_train_b200.ops.tp import TpComm
    from mia_train_b200.parallel.sequence_parallel import SequenceParallel, partial_params, sync_partial_grads
    from mia_train_b200.parallel.tensor_parallel import apply_tensor_parallel

    torch.manual_seed(0)
    enc = DinoVisionTransformer3D(img_size=16, patch_size=4, embed_dim=32, depth=2, num_heads=4)
    dense = AffinitySegmentation(enc, input_axes="lcxyz", offsets="nisb12", decoder="subpixel",
                                 decoder_hidden_dim=16, decoder_readout_dim=8, decoder_zero_init_output=False,
                                 split_disconnected=False)
    tp = copy.deepcopy(dense)
    group = dist.group.WORLD
    apply_tensor_parallel(tp.encoder.tensor_parallel_plan(), group)
    tp.encoder.enable_sequence_parallel(SequenceParallel(TpComm(group, "fused")))
    imgs, labs = [], []
    for i in range(batch):
        img, lab = voronoi_volume((16,) * 3, 12, 0.08, 1.0, torch.Generator().manual_seed(i))
        imgs.append(img)
        labs.append(lab)
    batch = {"img": torch.stack(imgs)[:, None, None].float(), "label": torch.stack(labs)[:, None].long()}
    ref = dense(batch)
    ref["loss"].backward()
    out = tp(batch)
    out["loss"].backward()
    n_partial = sync_partial_grads(tp)
    dense_params = dict(dense.named_parameters())
    worst = 0.0
    for name, p in tp.named_parameters():
        rg = dense_params[name].grad
        if p.grad is None:
            assert rg is None or float(rg.abs().max()) == 0.0, name
            continue
        mod = tp.get_submodule(name.rsplit(".", 1)[0]) if "." in name else tp
        gp = _gathered_grad(p, mod, world, rg.shape)
        err = float((gp - rg).norm() / (rg.norm() + 1e-12))
        worst = max(worst, err)
        assert err < 1e-4, (name, err)
    acc = abs(float(out["affinity_accuracy"]) - float(ref["affinity_accuracy"]))
    return float(out["loss"]), float(ref["loss"]), worst, n_partial, len(partial_params(tp)), acc


@pytest.mark.parametrize("world,batch", [(2, 4), (2, 3)])
def test_affinity_decoder_split_over_tp_matches_dense(run_distributed, world, batch):
    """Each TP rank decodes its own samples (an uneven share when the batch does not divide); loss,
    metrics and every gradient match the dense model."""
    res = run_distributed(_affinity_split_vs_dense, world, batch)
    for loss, ref, worst, n_partial, n_marked, acc in res.values():
        assert abs(loss - ref) < 1e-5 * max(1.0, abs(ref)), (loss, ref)
        assert worst < 1e-4
        assert n_partial == n_marked > 2 * 6  # block norms / LayerScale plus the final norm and decoder
        assert acc < 1e-6
