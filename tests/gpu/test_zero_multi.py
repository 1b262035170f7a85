"""Sharded data-parallel step (peer-memory kernels and NCCL) against the all-reduce path, 2 GPUs."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

WORKER = Path(__file__).with_name("zero_worker.py")


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_paths_match_allreduce():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MIA_PG_TIMEOUT_S="120")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29531", str(WORKER)]
    out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert out.returncode == 0, out.stderr[-4000:]
    line = [x for x in out.stdout.splitlines() if x.startswith("{")][-1]
    res = json.loads(line)
    assert res["errors"] == 0
    assert res["replica_diff"] == 0.0
    for impl, d in res["rel_diff"].items():
        assert d < 2e-2, (impl, res)
