"""Package layering, checked statically (AST) so nothing has to run.

* `ls mia_train_b200/models/` is the list of trainable models: every module there registers one
  with `ModelRegistry` (besides `base.py` and `registry.py`, the contract itself).
* `ls mia_train_b200/algorithms/*.py` is the list of training strategies: every top-level module
  registers one with `AlgorithmRegistry`; a strategy's supporting code lives in a subpackage and
  registers nothing there.
* Dependencies point downwards: `ops` (the native kernels' Python side) imports none of the
  framework layers above it; `layers` imports neither models, algorithms nor the engine; `models`
  imports neither algorithms nor the engine.

The reference enforces the same boundaries for its `src/` tree (`tests/unit/test_package_layout.py`).
"""

from __future__ import annotations

import ast
from pathlib import Path

import mia_train_b200

PKG = Path(mia_train_b200.__file__).resolve().parent
CONTRACT = {"base.py", "registry.py", "__init__.py"}


def _modules(sub: str, recursive: bool = True) -> list[Path]:
    root = PKG / sub
    files = root.rglob("*.py") if recursive else root.glob("*.py")
    return sorted(p for p in files if p.name != "__init__.py")


def _package_of(path: Path) -> list[str]:
    return list(path.relative_to(PKG).parent.parts)


def _imported_layers(path: Path) -> set[str]:
    """First-level subpackages of mia_train_b200 that `path` imports (absolute or relative)."""
    tree = ast.parse(path.read_text())
    out: set[str] = set()
    here = _package_of(path)
    for node in ast.walk(tree):
        if isinstance(node, ast.ImportFrom):
            if node.level:
                base = here[: len(here) - (node.level - 1)] if node.level > 1 else here
                parts = base + (node.module.split(".") if node.module else [])
                if not parts:  # `from .. import x`: x is a subpackage
                    out.update(alias.name for alias in node.names)
                else:
                    out.add(parts[0])
            elif node.module and node.module.startswith("mia_train_b200."):
                out.add(node.module.split(".")[1])
        elif isinstance(node, ast.Import):
            for alias in node.names:
                if alias.name.startswith("mia_train_b200."):
                    out.add(alias.name.split(".")[1])
    return out


def _registers(path: Path, registry: str) -> bool:
    tree = ast.parse(path.read_text())
    for node in ast.walk(tree):
        if isinstance(node, ast.ClassDef):
            for dec in node.decorator_list:
                target = dec.func if isinstance(dec, ast.Call) else dec
                if isinstance(target, ast.Attribute) and target.attr == "register":
                    if isinstance(target.value, ast.Name) and target.value.id == registry:
                        return True
    return False


def test_every_model_module_registers_a_model():
    for path in _modules("models", recursive=False):
        if path.name in CONTRACT:
            continue
        assert _registers(path, "ModelRegistry"), f"models/{path.name} registers no model; move it to layers/"


def test_every_top_level_algorithm_registers_a_strategy():
    for path in _modules("algorithms", recursive=False):
        if path.name in CONTRACT:
            continue
        assert _registers(path, "AlgorithmRegistry"), (
            f"algorithms/{path.name} registers no strategy; put supporting code in a subpackage"
        )


def test_algorithm_subpackages_register_nothing():
    for path in _modules("algorithms"):
        if len(path.relative_to(PKG / "algorithms").parts) > 1:
            assert not _registers(path, "AlgorithmRegistry"), f"{path.relative_to(PKG)} registers a strategy"


def test_layers_import_no_models_algorithms_or_engine():
    for path in _modules("layers"):
        leaked = _imported_layers(path) & {"models", "algorithms", "engine"}
        assert not leaked, f"{path.relative_to(PKG)} imports {sorted(leaked)}"


def test_models_import_no_algorithms_or_engine():
    for path in _modules("models"):
        leaked = _imported_layers(path) & {"algorithms", "engine"}
        assert not leaked, f"{path.relative_to(PKG)} imports {sorted(leaked)}"


def test_ops_sit_below_the_framework():
    for path in _modules("ops"):
        leaked = _imported_layers(path) & {"models", "algorithms", "engine", "layers", "data", "evals"}
        if path.name == "microbench.py":  # a command-line tool that times whole steps
            leaked -= {"algorithms", "engine", "models"}
        assert not leaked, f"{path.relative_to(PKG)} imports {sorted(leaked)}"


def test_layer_scan_sees_relative_imports():
    imports = _imported_layers(PKG / "models" / "dinov3_vit3d.py")
    assert {"layers", "utils"} <= imports, imports
