import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


def load_golden(name: str) -> dict:
    return torch.load(GOLDEN / name, weights_only=False)


def oracle_config(d: dict):
    from oracle import OracleConfig

    return OracleConfig(**d)
