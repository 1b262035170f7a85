"""Single entrypoint for every job (reference `src/train.py:14-51`). Launch with torchrun:

    torchrun --standalone --nproc_per_node=<gpus> -m mia_train_b200.train --config configs/<run>.toml
"""

from __future__ import annotations

import argparse
from pathlib import Path


def parse_args(argv: list[str] | None = None) -> argparse.Namespace:
    parser = argparse.ArgumentParser(description="Train a model described by a .toml config.")
    parser.add_argument("--config", type=Path, required=True, help="path to the run's .toml configuration")
    parser.add_argument(
        "--output-root",
        type=Path,
        default=None,
        help="directory under which the run directory is created; defaults to "
        "[environment].checkpoint_dir from configs/cluster/active.toml",
    )
    parser.add_argument(
        "--resume",
        nargs="?",
        const="latest",
        default=None,
        metavar="RUN_DIR",
        help="continue the newest run of this experiment (or start fresh if none), or the given run directory",
    )
    return parser.parse_args(argv)


def main(argv: list[str] | None = None) -> None:
    args = parse_args(argv)
    from . import components  # noqa: F401  (populates the registries)
    from .engine.run import run

    output_dir = run(args.config, args.output_root, args.resume)
    print(f"run artifacts: {output_dir}", flush=True)


if __name__ == "__main__":
    main()
