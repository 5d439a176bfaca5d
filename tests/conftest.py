"""Shared pytest configuration: the ``gpu`` marker and fixture loading."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the CUDA library")


def load_golden(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{name}.npz") as data:
        return {k: data[k] for k in data.files}


def golden_manifest() -> dict:
    return json.loads((GOLDEN / "manifest.json").read_text())


def bf16_from_bits(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << np.uint32(16)).view(np.float32)


def seeded_bf16_normal(seed: int, *shapes):
    """Regenerate ``mx.array(rng.normal(size=s).astype(f32)).astype(bf16)`` draws."""

    from oracle.convrot_oracle import round_bf16

    rng = np.random.default_rng(seed)
    return [round_bf16(rng.normal(size=s).astype(np.float32)) for s in shapes]


@pytest.fixture
def golden():
    return load_golden
