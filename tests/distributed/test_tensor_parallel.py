"""Tensor parallelism over Gloo: sharded blocks reproduce the unsharded model and its gradients."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.cpu_dist


def _build(kind: str):
    from mia_train_b200.models.dinov3_vit3d import DinoVisionTransformer3D
    from mia_train_b200.models.vit import ViT3D

    torch.manual_seed(0)
    if kind == "vit3d":
        return ViT3D(img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=2, num_heads=4)
    if kind == "dinov3_swiglu":
        return DinoVisionTransformer3D(img_size=16, patch_size=4, embed_dim=32, depth=2, num_heads=4, n_storage_tokens=2,
                                       ffn_layer="swiglu", layerscale_init=0.1, mask_k_bias=True)
    return DinoVisionTransformer3D(img_size=16, patch_size=4, embed_dim=32, depth=2, num_heads=4, n_storage_tokens=1,
                                   window_size=2, global_every=2)


def _loss(model, x):
    if hasattr(model, "forward_features"):
        out = model.forward_features(x)
        return (out["x_norm_patchtokens"].square().mean() + out["x_norm_clstoken"].sum() * 0.1)
    return model(x).square().mean()


def _tp_matches_dense(rank, world, kind):
    import torch.distributed as dist

    from mia_train_b200.parallel.tensor_parallel import apply_tensor_parallel

    dense = _build(kind)
    tp = _build(kind)
    torch.manual_seed(1)
    x = torch.randn(2, 1, 16, 16, 16)
    ref = _loss(dense, x)
    ref.backward()
    n = apply_tensor_parallel(tp.tensor_parallel_plan(), dist.group.WORLD)
    out = _loss(tp, x)
    out.backward()
    loss_diff = float((out - ref).abs())
    # replicated parameters get the full gradient on every rank
    worst = 0.0
    for (name, p), (_, q) in zip(tp.named_parameters(), dense.named_parameters(), strict=True):
        if p.shape == q.shape and p.grad is not None:
            worst = max(worst, float((p.grad - q.grad).abs().max()))
    # the state dict is the unsharded one
    sd = tp.state_dict()
    sd_diff = max(float((sd[k] - v).abs().max()) for k, v in dense.state_dict().items())
    # and it loads back into a fresh sharded model
    fresh = _build(kind)
    apply_tensor_parallel(fresh.tensor_parallel_plan(), dist.group.WORLD)
    fresh.load_state_dict(dense.state_dict())
    again = float((_loss(fresh, x) - ref).abs())
    return n, loss_diff, worst, sd_diff, again


@pytest.mark.parametrize("kind", ["vit3d", "dinov3_swiglu", "dinov3_windowed"])
def test_tp_matches_dense(run_distributed, kind):
    out = run_distributed(_tp_matches_dense, 2, kind)
    for n, loss_diff, worst, sd_diff, again in out.values():
        assert n > 0
        assert loss_diff < 1e-5 and again < 1e-5
        assert worst < 1e-5
        assert sd_diff == 0.0


def _tp_fsdp_step(rank, world):
    from mia_train_b200.algorithms.mae import MAE
    from mia_train_b200.models.vit import ViT3D
    from mia_train_b200.parallel.parallel_dims import ParallelDims
    from mia_train_b200.parallel.parallelize import parallelize_algorithm

    dims = ParallelDims(dp_shard=2, tp=2)
    mesh = dims.build_mesh("cpu")
    torch.manual_seed(0)
    model = ViT3D(img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=2, num_heads=4)
    alg = MAE(model, input_axes="lcxyz", decoder_embed_dim=16, decoder_depth=1, decoder_num_heads=2)
    alg = parallelize_algorithm(alg, mesh, dims)
    torch.manual_seed(10 + dims.dp_rank(mesh))
    out = alg({"img": torch.randn(2, 1, 1, 16, 16, 16)})
    out["loss"].backward()
    return float(out["loss"])


def test_tp_with_fsdp_steps(run_distributed):
    out = run_distributed(_tp_fsdp_step, 4)
    assert all(v == v for v in out.values())
    # TP peers saw the same batch and computed the same loss
    assert abs(out[0] - out[1]) < 1e-5 and abs(out[2] - out[3]) < 1e-5
