"""Shared fixtures. GPU tests carry @pytest.mark.gpu; the CPU suite runs with -m "not gpu"."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and libqtt.so")


@pytest.fixture(scope="session")
def full_weights():
    """Spec weights: Qwen3-TTS-0.6B shapes, bf16 N(0, 0.02), norms = 1, seeds 0 (backbone) / 1 (CP)."""
    from qwentts_turbo_b200.weights import synthetic_weights
    return synthetic_weights()


@pytest.fixture(scope="session")
def small_weights():
    """2 backbone + 2 code-predictor layers with random norm weights (1 + N(0, 0.1)), so a
    mixed-up norm vector or layer order changes the result."""
    from qwentts_turbo_b200.weights import synthetic_weights
    return synthetic_weights(backbone_layers=2, cp_layers=2, seed_backbone=10, seed_cp=11, norm_std=0.1)
