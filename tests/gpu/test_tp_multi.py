"""Tensor parallelism on 2 and 4 GPUs with the native kernels against the dense model: replicated
activations with NCCL all-reduces, and sequence parallelism on NCCL collectives or on the fused
all-gather -> GEMM / GEMM -> reduce-scatter kernels over NVLink peer memory."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

WORKER = Path(__file__).with_name("tp_worker.py")


def _gpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("world,mode,port", [(2, "allreduce", 29533), (2, "collective", 29534), (2, "fused", 29535),
                                             (4, "collective", 29536), (4, "fused", 29537)])
def test_tp_dinov3_matches_dense(world, mode, port):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(port), str(WORKER), mode]
    out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert out.returncode == 0, out.stderr[-4000:]
    res = json.loads([x for x in out.stdout.splitlines() if x.startswith("{")][-1])
    assert res["errors"] == 0
    assert res["mode"] == mode
    # qkv, proj and SwiGLU w1 / w2 / w3, or the GELU MLP's fc1 / fc2, per block
    assert res["sharded_layers"] == 2 * (5 if mode == "allreduce" else 4)
    assert abs(res["loss"] - res["ref"]) < 2e-2 * max(1.0, abs(res["ref"]))
    assert res["grad_rel"] < 0.05, res  # relative L2 error of every replicated parameter's gradient
    assert res["shard_rel"] < 0.05, res
    assert res["sd_diff"] == 0.0
