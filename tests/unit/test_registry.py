import pytest
import torch.nn as nn

from mia_train_b200 import components  # noqa: F401
from mia_train_b200.algorithms.registry import AlgorithmRegistry
from mia_train_b200.data.registry import DataRegistry
from mia_train_b200.evals.registry import EvalRegistry
from mia_train_b200.models.registry import ModelRegistry
from mia_train_b200.utils.registry import Registry


class Base(nn.Module):
    pass


def test_register_build_and_errors():
    reg: Registry[Base] = Registry(Base, kind="thing")

    @reg.register("a")
    class A(Base):
        def __init__(self, x=1):
            super().__init__()
            self.x = x

    assert reg.build("a", x=3).x == 3
    assert "a" in reg and reg.available() == ["a"]
    with pytest.raises(ValueError, match="already registered"):
        reg.register("a")(A)
    with pytest.raises(TypeError):
        reg.register("b")(int)
    with pytest.raises(KeyError, match="available"):
        reg.get("missing")


def test_public_component_names():
    assert set(ModelRegistry.available()) >= {"vit3d", "dinov3_vit3d", "dinov3_vit", "muvit3d"}
    assert set(AlgorithmRegistry.available()) >= {"mae", "muvit_mae", "simmim", "dinov3", "affinity_seg", "semantic_seg"}
    assert set(DataRegistry.available()) >= {"synthetic_volumes", "miao_volumes", "hf_semantic_seg"}
    assert "semantic_seg" in EvalRegistry.available()
