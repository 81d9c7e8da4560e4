from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden" / "q6_reference_golden.npz"


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def golden() -> dict[str, np.ndarray]:
    with np.load(GOLDEN) as data:
        return {key: data[key] for key in data.files}


def golden_case(golden: dict[str, np.ndarray], prefix: str):
    """(x, Q6Weights, y, gelu) for one golden linear case."""

    import oracle

    bias = golden.get(f"{prefix}.bias")
    w = oracle.Q6Weights(
        golden[f"{prefix}.weight"],
        golden[f"{prefix}.scales"],
        golden[f"{prefix}.biases"],
        bias,
        int(golden[f"{prefix}.group_size"]),
    )
    return golden[f"{prefix}.x"], w, golden[f"{prefix}.y"], bool(golden[f"{prefix}.gelu"])
