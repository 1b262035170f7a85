import subprocess
from pathlib import Path

import pytest
import torch
import torch.nn as nn

from mia_train_b200.utils.device import move_to_device, pin_batch, tensor_bytes
from mia_train_b200.utils.hardware_flops import known_devices, lookup_device, peak_flops
from mia_train_b200.utils.module_ops import named_apply, named_replace
from mia_train_b200.utils.provenance import write_run_artifacts


def test_b200_peak_table():
    peak, why = peak_flops("NVIDIA B200", "bf16")
    assert peak == pytest.approx(2250e12) and why == ""
    assert peak_flops("NVIDIA B200", "fp32", allow_tf32=True)[0] == pytest.approx(1100e12)
    assert peak_flops("NVIDIA B200", "fp32", allow_tf32=False)[0] == pytest.approx(80e12)
    assert lookup_device("NVIDIA H100 80GB HBM3").label.startswith("NVIDIA H100")
    assert peak_flops("Tesla T4", "bf16")[0] is None
    assert peak_flops("Mystery GPU", "bf16")[0] is None
    assert "NVIDIA B200" in known_devices()


def test_move_and_pin_recursive():
    batch = {"a": torch.zeros(3), "b": [torch.ones(2), (torch.ones(1), "s")], "c": 5}
    moved = move_to_device(batch, torch.device("cpu"))
    assert moved["c"] == 5 and moved["b"][1][1] == "s"
    assert tensor_bytes(batch) == 4 * (3 + 2 + 1)
    assert pin_batch({"x": 1})["x"] == 1


def test_named_apply_and_replace():
    m = nn.Sequential(nn.Linear(2, 2), nn.Sequential(nn.ReLU(), nn.Linear(2, 2)))
    seen = []
    named_apply(lambda module, name: seen.append(name), m)
    assert "1.1" in seen or any(s.endswith("1.1") for s in seen)
    named_replace(lambda module, name: nn.Identity() if isinstance(module, nn.ReLU) else module, m)
    assert isinstance(m[1][0], nn.Identity)


def git(repo: Path, *args: str) -> None:
    subprocess.run(["git", "-C", str(repo), *args], check=True, capture_output=True)


def test_provenance_records_dirty_tree(tmp_path):
    repo = tmp_path / "repo"
    repo.mkdir()
    git(repo, "init", "-q")
    git(repo, "-c", "user.email=a@b", "-c", "user.name=n", "commit", "--allow-empty", "-qm", "init")
    (repo / "f.txt").write_text("x")
    git(repo, "add", "f.txt")
    cfg = tmp_path / "run.toml"
    cfg.write_text("experiment_name='t'\n")
    extra = tmp_path / "data.yaml"
    extra.write_text("a: 1\n")
    out = tmp_path / "out"
    write_run_artifacts(out, cfg, {"k": 1}, repo, [extra])
    write_run_artifacts(out, cfg, {"k": 1}, repo, [extra])
    assert (out / "config.toml").read_text() == "experiment_name='t'\n"
    assert "(dirty)" in (out / "git_commit.txt").read_text()
    assert (out / "dirty.patch").exists() and (out / "data.yaml").exists()
    assert len((out / "attempts.log").read_text().splitlines()) == 2


def test_provenance_without_git(tmp_path):
    cfg = tmp_path / "run.toml"
    cfg.write_text("x=1\n")
    write_run_artifacts(tmp_path / "o", cfg, {}, tmp_path / "nogit")
    assert "unavailable" in (tmp_path / "o" / "git_commit.txt").read_text()
