"""Shared test configuration: the ``gpu`` marker, the golden fixtures and seeded input draws."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built library")


@pytest.fixture(scope="session")
def golden():
    """Dict case -> dict of arrays from tests/golden/kata_attn_golden.npz."""
    z = np.load(GOLDEN / "kata_attn_golden.npz")
    out: dict[str, dict[str, np.ndarray]] = {}
    for key in z.files:
        case, name = key.split("/")
        out.setdefault(case, {})[name] = z[key]
    return out


@pytest.fixture(scope="session")
def golden_delta():
    """Dict case -> dict of arrays from tests/golden/delta_golden.npz (reference U solve)."""
    z = np.load(GOLDEN / "delta_golden.npz")
    out: dict[str, dict[str, np.ndarray]] = {}
    for key in z.files:
        case, name = key.split("/")
        out.setdefault(case, {})[name] = z[key]
    return out


@pytest.fixture(scope="session")
def golden_delta_gpu():
    """Dict case -> dict of arrays from tests/golden/delta_golden_gpu.npz: the reference's own Triton
    flash_delta (U, readout, den, o and all gradients) run on a B200 by make_golden_delta_gpu.py."""
    return load_delta_gpu_golden()


def load_delta_gpu_golden():
    z = np.load(GOLDEN / "delta_golden_gpu.npz")
    out: dict[str, dict[str, np.ndarray]] = {}
    for key in z.files:
        if "/" not in key:
            continue
        case, name = key.split("/")
        out.setdefault(case, {})[name] = z[key]
    return out


def attn_case_meta(rec):
    B, T, HQ, H, D, Dv, M, is_sum, decay = (int(x) for x in rec["meta"])
    return dict(B=B, T=T, HQ=HQ, H=H, D=D, Dv=Dv, M=M, score="sum" if is_sum else "concat", decay=bool(decay))
