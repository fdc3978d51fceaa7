"""Shared pytest configuration: the ``gpu`` marker and fixture loading."""
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")
GOLDEN_CASES = ["hofa_r16", "hofa_r16_alpha", "hofa_r16_fixedmix", "hofa_dh128_r32", "gla_r0"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name):
    return torch.load(os.path.join(GOLDEN_DIR, f"{name}.pt"), weights_only=False)


@pytest.fixture(scope="session")
def golden():
    return {n: load_golden(n) for n in GOLDEN_CASES}
