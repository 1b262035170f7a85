"""Package structure: native sources present, nothing imports scratch space, no compat layers."""

from pathlib import Path

import mia_train_b200

PKG = Path(mia_train_b200.__file__).resolve().parent
REPO = PKG.parent


def test_layout():
    for sub in ("models", "ops", "parallel", "utils", "engine", "layers", "algorithms", "data", "evals", "csrc"):
        assert (PKG / sub).is_dir(), sub
    assert (REPO / "bench.py").is_file() and (REPO / "__graft_entry__.py").is_file()
    assert list((PKG / "csrc").glob("*.cu"))


def test_no_scratch_imports_and_no_compat_layers():
    import re

    banned = ("import triton", "from triton", "tilelang", "torch.compile(")
    scratch = re.compile(r"[\"'/]_work[/\"']|import _work|from _work")
    for path in list(PKG.rglob("*.py")) + [REPO / "bench.py", REPO / "__graft_entry__.py"]:
        text = path.read_text()
        for word in banned:
            assert word not in text, f"{path} mentions {word!r}"
        assert not scratch.search(text), f"{path} refers to the scratch folder"
