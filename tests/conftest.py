"""Shared pytest setup: import paths, the `gpu` marker, fixture loaders."""
import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "nvfp4-qsa_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _cases(path):
    data = np.load(path)
    names = sorted({k.split("__")[0] for k in data.files})
    return data, names


@pytest.fixture(scope="session")
def golden_kat():
    return json.loads((GOLDEN / "kat.json").read_text())


@pytest.fixture(scope="session")
def golden_hashes():
    return json.loads((GOLDEN / "config_hashes.json").read_text())


@pytest.fixture(scope="session")
def codec_cases():
    return _cases(GOLDEN / "codec_cases.npz")


@pytest.fixture(scope="session")
def attention_cases():
    return _cases(GOLDEN / "attention_cases.npz")


@pytest.fixture(scope="session")
def bf16_attention_cases():
    return _cases(GOLDEN / "bf16_attention_cases.npz")


@pytest.fixture(scope="session")
def decode_golden():
    return np.load(GOLDEN / "decode_config.npz")
