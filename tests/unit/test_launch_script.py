"""The launch script parses and reports its usage (no processes are started)."""

from __future__ import annotations

import subprocess
from pathlib import Path

SCRIPT = Path(__file__).resolve().parents[2] / "deploy" / "launch.sh"


def test_launch_script_syntax():
    assert subprocess.run(["bash", "-n", str(SCRIPT)]).returncode == 0


def test_launch_script_usage_without_arguments():
    out = subprocess.run(["bash", str(SCRIPT)], capture_output=True, text=True)
    assert out.returncode != 0
    assert "usage: launch.sh" in out.stderr


def test_launch_script_needs_node_rank_for_several_nodes(tmp_path):
    env = {"PATH": "/usr/bin:/bin", "NODES": "a b", "PYTHON": "false"}
    out = subprocess.run(["bash", str(SCRIPT), "8", "cfg.toml"], capture_output=True, text=True, env=env)
    assert out.returncode != 0
    assert "NODE_RANK" in out.stderr
