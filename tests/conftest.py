"""Shared pytest setup: the `gpu` marker, package/oracle loading and model fixtures."""
from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG_DIR = REPO / "plamo3-0.8b-runtime_b200"
GOLDEN = REPO / "tests" / "golden"

# The seeded test checkpoints' .p12 archives are bound to the safetensors file beside them, which
# the loader accepts only when asked to (by default it accepts the reference checkpoint's digest).
os.environ.setdefault("PLAMO_P12_LOCAL_SOURCE", "1")


def load_package():
    if "plamo_b200" in sys.modules:
        return sys.modules["plamo_b200"]
    spec = importlib.util.spec_from_file_location("plamo_b200", PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["plamo_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def load_oracle():
    if "plamo_oracle" in sys.modules:
        return sys.modules["plamo_oracle"]
    spec = importlib.util.spec_from_file_location("plamo_oracle", REPO / "oracle" / "oracle.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["plamo_oracle"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def oracle():
    return load_oracle()


def _model_dir(tmp_root: Path, name: str, cfg, packed: bool):
    p = load_package()
    d = tmp_root / name
    if not (d / "model.safetensors").exists():
        p.synthetic.write_model(d, cfg, seed=0)
    if packed and not (d / "model.p12").exists():
        p.packing.write_p12(d)
    return d


@pytest.fixture(scope="session")
def models_root(tmp_path_factory):
    root = os.environ.get("PLAMO_TEST_MODELS")
    if root:
        r = Path(root)
        r.mkdir(parents=True, exist_ok=True)
        return r
    return tmp_path_factory.mktemp("models")


@pytest.fixture(scope="session")
def tiny_dir(models_root):
    return _model_dir(models_root, "tiny", load_package().synthetic.TINY, packed=True)


@pytest.fixture(scope="session")
def micro_dir():
    return GOLDEN / "micro"


@pytest.fixture(scope="session")
def reference_dir(models_root):
    """Full reference-dims synthetic model (1.78 GB on disk, plus the .p12 archive)."""
    return _model_dir(models_root, "reference", load_package().synthetic.REFERENCE, packed=True)


@pytest.fixture(scope="session")
def example_dir(models_root):
    """BASELINE.json's example dims per layer (d 2048, 16 q-heads over 4 KV heads, FFN 5632, vocab
    80000) in 2 layers with a 32-key window, so grouped-query attention runs with rings that wrap."""
    s = load_package().synthetic
    cfg = s.ModelConfig(hidden_size=2048, num_hidden_layers=2, num_attention_heads=16, num_key_value_heads=4,
                        intermediate_size=5632, vocab_size=80000, window_size=32, sliding_window_pattern=2)
    return _model_dir(models_root, "example_gqa", cfg, packed=True)
