"""`torchrun src/train.py --config X.toml [--resume] [--output-root DIR]` -- the same command line as
the reference; forwards to `mia_train_b200.train`."""

from __future__ import annotations

import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from mia_train_b200.train import main  # noqa: E402

if __name__ == "__main__":
    main()
