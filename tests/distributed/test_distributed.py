"""Multi-process CPU tests over Gloo: parallel wrappers, the training loop, run orchestration."""

from __future__ import annotations

from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.cpu_dist

CONFIG = """
experiment_name = "dist"

[model]
name = "vit3d"
img_size = [16, 16, 16]
patch_size = [8, 8, 8]
embed_dim = 32
depth = 2
num_heads = 2

[algorithm]
name = "mae"
mask_ratio = 0.5
decoder_embed_dim = 16
decoder_depth = 1
decoder_num_heads = 2

[data]
name = "synthetic_volumes"
shape = [16, 16, 16]
samples_per_epoch = 16

[trainer]
max_steps = {steps}
batch_size = 2
lr = 1e-3
warmup_steps = 1
precision = "fp32"
log_every = 2
checkpoint_every = 3
seed = 0

[parallelism]
{parallelism}
"""


def _all_reduce(rank, world):
    import torch.distributed as dist

    t = torch.tensor([float(rank + 1)])
    dist.all_reduce(t)
    return float(t)


def test_harness(run_distributed):
    out = run_distributed(_all_reduce, 2)
    assert out == {0: 3.0, 1: 3.0}


def _wrapped_step(rank, world, layout):
    import torch.distributed as dist

    from mia_train_b200.algorithms.mae import MAE
    from mia_train_b200.models.vit import ViT3D
    from mia_train_b200.parallel.parallel_dims import ParallelDims
    from mia_train_b200.parallel.parallelize import parallelize_algorithm

    dims = ParallelDims(**layout)
    mesh = dims.build_mesh("cpu")
    torch.manual_seed(0)
    model = ViT3D(img_size=(16, 16, 16), patch_size=(8, 8, 8), embed_dim=32, depth=2, num_heads=2)
    alg = MAE(model, input_axes="lcxyz", decoder_embed_dim=16, decoder_depth=1, decoder_num_heads=2)
    alg = parallelize_algorithm(alg, mesh, dims)
    torch.manual_seed(100 + rank)
    out = alg({"img": torch.randn(2, 1, 1, 16, 16, 16)})
    out["loss"].backward()
    # the gradient of one shared parameter, reassembled, must agree across ranks
    g = alg.model.blocks[0].attn.qkv.weight.grad
    full = g.full_tensor() if hasattr(g, "full_tensor") else g
    gathered = [torch.zeros_like(full) for _ in range(world)]
    dist.all_gather(gathered, full.contiguous())
    return float(max((x - gathered[0]).abs().max() for x in gathered)), float(out["loss"])


@pytest.mark.parametrize("layout,world", [
    ({"dp_replicate": 2}, 2),
    ({"dp_shard": 2}, 2),
    ({"dp_shard": 2, "fsdp_unit": "model", "param_dtype": "fp32"}, 2),
    ({"dp_replicate": 2, "dp_shard": 2}, 4),
])
def test_data_parallel_layouts_agree(run_distributed, layout, world):
    out = run_distributed(_wrapped_step, world, layout)
    for diff, loss in out.values():
        assert diff < 1e-6 and loss == loss


def _run_training(rank, world, root, config_path, resume):
    from mia_train_b200.engine.run import run

    return str(run(Path(config_path), output_root=Path(root), resume=resume))


def test_run_then_resume(run_distributed, tmp_path):
    cfg = tmp_path / "dist.toml"
    cfg.write_text(CONFIG.format(steps=4, parallelism="dp_shard = 2"))
    root = tmp_path / "runs"
    out = run_distributed(_run_training, 2, str(root), str(cfg), None)
    assert len(set(out.values())) == 1  # every rank agreed on one run directory
    run_dir = Path(out[0])
    assert (run_dir / "checkpoints" / "step_4").is_dir() or any((run_dir / "checkpoints").glob("step_*"))
    assert (run_dir / "resolved_config.json").is_file()
    cfg.write_text(CONFIG.format(steps=6, parallelism="dp_shard = 2"))
    out2 = run_distributed(_run_training, 2, str(root), str(cfg), "latest")
    assert out2[0] == out[0]
    steps = sorted(int(p.name.split("_")[1]) for p in (run_dir / "checkpoints").glob("step_*") if "tmp" not in p.name)
    assert steps[-1] == 6


def _prep_failure(rank, world, root):
    from mia_train_b200.engine.run import prepare_run_dir

    try:
        prepare_run_dir(Path(root) / "x", Path(root) / "does_not_exist.toml", {}, rank)
    except RuntimeError as error:
        return str(error)
    return "no error"


def test_prep_failure_reaches_every_rank(run_distributed, tmp_path):
    out = run_distributed(_prep_failure, 2, str(tmp_path), timeout=120)
    assert all("could not prepare" in v for v in out.values())


def _device_wait_timeout(rank, world, root, config_path):
    """Every rank's kernels report an abandoned wait at the first logging step (what the surviving
    ranks see when a peer is lost): the Trainer must stop with DeviceWaitError, not keep stepping."""
    import mia_train_b200.engine.trainer as trainer_module
    from mia_train_b200.engine.run import run
    from mia_train_b200.ops._native import DeviceWaitError

    calls = []

    def fake_check(device):
        calls.append(device)
        raise DeviceWaitError(402, 0)

    trainer_module.raise_on_device_errors = fake_check
    try:
        run(Path(config_path), output_root=Path(root), resume=None)
    except DeviceWaitError as error:
        return f"raised after {len(calls)} check(s): {error}"
    return "no error"


def test_device_wait_timeout_stops_training(run_distributed, tmp_path):
    cfg = tmp_path / "dist.toml"
    cfg.write_text(CONFIG.format(steps=6, parallelism="dp_shard = 2"))
    out = run_distributed(_device_wait_timeout, 2, str(tmp_path / "runs"), str(cfg), timeout=180)
    for msg in out.values():
        assert msg.startswith("raised after 1 check"), msg
        assert "code 402" in msg


SP_CONFIG = """
experiment_name = "sp"

[model]
name = "dinov3_vit3d"
img_size = 16
patch_size = 4
embed_dim = 32
depth = 2
num_heads = 2

[algorithm]
name = "simmim"
mask_ratio = 0.5

[data]
name = "synthetic_volumes"
shape = [16, 16, 16]
samples_per_epoch = 8

[trainer]
max_steps = 2
batch_size = 1
lr = 1e-3
warmup_steps = 1
precision = "fp32"
log_every = 1
checkpoint_every = 100
seed = 0

[parallelism]
tp = 2
tp_comm = "collective"
"""


def _sp_trainer_syncs(rank, world, root, config_path):
    """The Trainer's eager step must sum the sequence-parallel partial gradients over the TP group."""
    import mia_train_b200.engine.trainer as trainer_module
    from mia_train_b200.engine.run import run

    counts = []
    real = trainer_module.sync_partial_grads

    def counting(module):
        n = real(module)
        counts.append(n)
        return n

    trainer_module.sync_partial_grads = counting
    run(Path(config_path), output_root=Path(root), resume=None)
    return counts


def test_trainer_syncs_sequence_parallel_partial_grads(run_distributed, tmp_path):
    cfg = tmp_path / "sp.toml"
    cfg.write_text(SP_CONFIG)
    out = run_distributed(_sp_trainer_syncs, 2, str(tmp_path / "runs"), str(cfg))
    for counts in out.values():
        assert len(counts) == 2 and all(n == 2 * 4 for n in counts), counts  # norm1 / norm2 weight + bias x 2 blocks


def test_trainer_syncs_partial_grads_under_tp_and_fsdp(run_distributed, tmp_path):
    """TP 2 x FSDP dp_shard 2: the partial marks survive FSDP's parameter replacement and the sharded
    gradients are summed over the TP group."""
    cfg = tmp_path / "sp_fsdp.toml"
    cfg.write_text(SP_CONFIG.replace("tp = 2\n", "tp = 2\ndp_shard = 2\n"))
    out = run_distributed(_sp_trainer_syncs, 4, str(tmp_path / "runs"), str(cfg), timeout=300)
    for counts in out.values():
        assert len(counts) == 2 and all(n == 2 * 4 for n in counts), counts


def test_run_then_resume_under_tensor_parallelism(run_distributed, tmp_path):
    """Checkpoints written under TP 2 (sequence-parallel) hold unsharded tensors and resume onto the
    same layout."""
    cfg = tmp_path / "sp.toml"
    cfg.write_text(SP_CONFIG.replace("max_steps = 2", "max_steps = 3").replace("checkpoint_every = 100",
                                                                               "checkpoint_every = 2"))
    root = tmp_path / "runs"
    out = run_distributed(_run_training, 2, str(root), str(cfg), None)
    run_dir = Path(out[0])
    assert any((run_dir / "checkpoints").glob("step_*"))
    cfg.write_text(SP_CONFIG.replace("max_steps = 2", "max_steps = 4").replace("checkpoint_every = 100",
                                                                               "checkpoint_every = 2"))
    out2 = run_distributed(_run_training, 2, str(root), str(cfg), "latest")
    assert out2[0] == out[0]
    steps = sorted(int(p.name.split("_")[1]) for p in (run_dir / "checkpoints").glob("step_*") if "tmp" not in p.name)
    assert steps[-1] == 4


def test_trainer_affinity_decoder_split_under_tensor_parallelism(run_distributed, tmp_path):
    """affinity_seg under TP 2 through the Trainer: each rank decodes its own sample, so the decoder
    and final-norm gradients join the TP sum next to the blocks' norms."""
    cfg = tmp_path / "aff.toml"
    text = SP_CONFIG.replace('name = "simmim"\nmask_ratio = 0.5',
                             'name = "affinity_seg"\ndecoder = "subpixel"\noffsets = "nisb12"\n'
                             'decoder_hidden_dim = 16\ndecoder_readout_dim = 8\nsplit_disconnected = false')
    text = text.replace('shape = [16, 16, 16]', 'shape = [16, 16, 16]\ngenerator = "voronoi"\nn_seeds = 12')
    text = text.replace("batch_size = 1", "batch_size = 2")
    cfg.write_text(text)
    out = run_distributed(_sp_trainer_syncs, 2, str(tmp_path / "runs"), str(cfg))
    for counts in out.values():
        assert len(counts) == 2 and all(n > 2 * 4 for n in counts), counts


def test_affinity_batch_smaller_than_tp_group_decodes_replicated(run_distributed, tmp_path):
    """A per-replica batch of 1 under TP 2 cannot be split by samples: every TP rank decodes it, and
    the decoder's gradients are not summed over the group (only the blocks' norms are)."""
    cfg = tmp_path / "aff1.toml"
    text = SP_CONFIG.replace('name = "simmim"\nmask_ratio = 0.5',
                             'name = "affinity_seg"\ndecoder = "subpixel"\noffsets = "nisb12"\n'
                             'decoder_hidden_dim = 16\ndecoder_readout_dim = 8\nsplit_disconnected = false')
    text = text.replace('shape = [16, 16, 16]', 'shape = [16, 16, 16]\ngenerator = "voronoi"\nn_seeds = 12')
    assert "batch_size = 1" in text
    cfg.write_text(text)
    out = run_distributed(_sp_trainer_syncs, 2, str(tmp_path / "runs"), str(cfg))
    for counts in out.values():
        assert len(counts) == 2 and all(n == 2 * 4 for n in counts), counts


def _run_or_error(rank, world, root, config_path):
    from mia_train_b200.engine.run import run

    try:
        run(Path(config_path), output_root=Path(root), resume=None)
    except ValueError as error:
        return str(error)
    return "trained"


def test_drop_path_under_tensor_parallelism(run_distributed, tmp_path):
    """Stochastic depth is refused at setup under sequence-parallel TP (its blocks have no
    sample-subset path) and trains with replicated activations (tp_comm = "allreduce")."""
    text = SP_CONFIG.replace('name = "dinov3_vit3d"\n', 'name = "dinov3_vit3d"\ndrop_path_rate = 0.5\n', 1)
    assert "drop_path_rate" in text
    cfg = tmp_path / "drop_sp.toml"
    cfg.write_text(text)
    out = run_distributed(_run_or_error, 2, str(tmp_path / "runs"), str(cfg))
    assert all("drop_path" in v and "allreduce" in v for v in out.values()), out
    cfg = tmp_path / "drop_allreduce.toml"
    cfg.write_text(text.replace('tp_comm = "collective"', 'tp_comm = "allreduce"'))
    out = run_distributed(_run_or_error, 2, str(tmp_path / "runs2"), str(cfg))
    assert set(out.values()) == {"trained"}, out


DINO_CONFIG = """
experiment_name = "dino"

[model]
name = "dinov3_vit3d"
img_size = 16
patch_size = 4
embed_dim = 32
depth = 2
num_heads = 2

[algorithm]
name = "dinov3"
global_crop_size = 16
local_crop_size = 8
n_local_crops = 2
head_n_prototypes = 64
head_hidden_dim = 32
head_bottleneck_dim = 16
total_steps = 10
warmup_teacher_temp_steps = 4

[data]
name = "synthetic_volumes"
shape = [24, 24, 24]
samples_per_epoch = 16

[trainer]
max_steps = {steps}
batch_size = 2
lr = 1e-3
warmup_steps = 1
precision = "fp32"
log_every = 1
checkpoint_every = 2
seed = 0

[parallelism]
dp_shard = 2
"""


def _dino_steps_seen(rank, world, root, config_path, resume):
    """Run training and record the algorithm's step counter at the start of every training step."""
    from mia_train_b200.algorithms.dinov3_ssl import DINOv3
    from mia_train_b200.engine.run import run

    seen = []
    real = DINOv3._step_impl

    def recording(self, batch, train):
        if train:
            seen.append(self.step)
        return real(self, batch, train)

    DINOv3._step_impl = recording
    run(Path(config_path), output_root=Path(root), resume=resume)
    return seen


def test_dinov3_step_counter_survives_resume_under_fsdp(run_distributed, tmp_path):
    """DINOv3 trains under FSDP (its teacher, a container, is sharded child by child) and its step
    counter - hence the teacher temperature and momentum schedules - resumes where it stopped."""
    cfg = tmp_path / "dino.toml"
    cfg.write_text(DINO_CONFIG.format(steps=2))
    root = tmp_path / "runs"
    first = run_distributed(_dino_steps_seen, 2, str(root), str(cfg), None)
    # the first call of each run is the FLOP measurement, which restores the counter afterwards
    assert all(v[-2:] == [0, 1] for v in first.values()), first
    cfg.write_text(DINO_CONFIG.format(steps=4))
    second = run_distributed(_dino_steps_seen, 2, str(root), str(cfg), "latest")
    assert all(v[-2:] == [2, 3] for v in second.values()), second


def test_dinov3_trains_under_tensor_parallelism(run_distributed, tmp_path):
    """The teacher backbone takes the student's TP layout, so the EMA pairs matching shards."""
    cfg = tmp_path / "dino_tp.toml"
    cfg.write_text(DINO_CONFIG.format(steps=2).replace("dp_shard = 2", 'tp = 2\ntp_comm = "collective"'))
    out = run_distributed(_dino_steps_seen, 2, str(tmp_path / "runs"), str(cfg), None)
    assert all(v[-2:] == [0, 1] for v in out.values()), out


def test_affinity_interpolate_decoder_under_fsdp(run_distributed, tmp_path):
    """The voxel head's fp32 upsampling output meets FSDP's low-precision compute parameters."""
    cfg = tmp_path / "aff_fsdp.toml"
    text = CONFIG.format(steps=2, parallelism="dp_shard = 2")
    text = text.replace('name = "mae"\nmask_ratio = 0.5\ndecoder_embed_dim = 16\ndecoder_depth = 1\ndecoder_num_heads = 2',
                        'name = "affinity_seg"\nsplit_disconnected = false')
    text = text.replace('shape = [16, 16, 16]', 'shape = [16, 16, 16]\ngenerator = "voronoi"\nn_seeds = 12')
    assert 'name = "affinity_seg"' in text
    cfg.write_text(text)
    out = run_distributed(_run_training, 2, str(tmp_path / "runs"), str(cfg), None)
    assert len(set(out.values())) == 1


def test_backbone_unfreezes_under_fsdp_mixed_precision(run_distributed, tmp_path):
    """A backbone frozen for the first steps trains once unfrozen under FSDP with bf16 parameters:
    the units' gradient dtypes are re-derived when requires_grad flips (FSDP fixes them from the
    parameters that require grad at its first forward, and a frozen unit then has none)."""
    cfg = tmp_path / "freeze.toml"
    text = CONFIG.format(steps=4, parallelism='dp_shard = 2\nparam_dtype = "bf16"')
    text = text.replace("seed = 0\n", "seed = 0\nfreeze_backbone_steps = 2\nunfreeze_warmup_steps = 1\n", 1)
    assert "freeze_backbone_steps" in text
    cfg.write_text(text)
    out = run_distributed(_run_training, 2, str(tmp_path / "runs"), str(cfg), None)
    assert len(set(out.values())) == 1


def _lora_under_tp(rank, world, root, config_path):
    from mia_train_b200.engine.run import run

    try:
        run(Path(config_path), output_root=Path(root), resume=None)
    except ValueError as error:
        return str(error)
    return "no error"


def test_lora_with_tensor_parallelism_is_refused(run_distributed, tmp_path):
    """The sequence-parallel blocks read the base weights: LoRA under TP must fail loudly rather
    than train without its adapters."""
    cfg = tmp_path / "lora_tp.toml"
    cfg.write_text(SP_CONFIG + '\n[lora]\nrank = 4\nalpha = 8.0\ntargets = ["attn_qkv"]\n')
    out = run_distributed(_lora_under_tp, 2, str(tmp_path / "runs"), str(cfg))
    assert all("cannot be combined with tensor parallelism" in v for v in out.values()), out
