import importlib.util
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

PKG_DIR = ROOT / "low-precision-transformer-accelerator-for-edge-llms_b200"


def load_package():
    """Import the product package (its directory name is not a Python
    identifier) under the module name ``lpta_b200``."""
    if "lpta_b200" in sys.modules:
        return sys.modules["lpta_b200"]
    spec = importlib.util.spec_from_file_location(
        "lpta_b200", PKG_DIR / "__init__.py", submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["lpta_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def reference_root():
    """The reference checkout named by TL_REFERENCE_ROOT, or None (tests that
    need it skip; the committed fixtures carry its outputs)."""
    v = os.environ.get("TL_REFERENCE_ROOT")
    if not v:
        return None
    p = Path(v)
    return p if (p / "model" / "tinyllama_gemm_int8.py").exists() else None


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built CUDA library")
    config.addinivalue_line("markers", "slow: long-running CPU case")


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return {p.stem: np.load(p) for p in GOLDEN.glob("*.npz")}


@pytest.fixture(scope="session")
def tinyllama22():
    """The full 22-layer TinyLlama with seeded random per-channel INT8
    weights, and an exact INT8 matmul that caches its float32 weight copies,
    shared by the full-size GPU tests (drawing the model takes ~30 s)."""
    from oracle import golden as G
    from oracle import weights as W
    return W.random_qmodel(2025, 22), G.ExactMatmul()
