"""Shared test setup: import paths, the `gpu` marker, golden-vector loading."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT / "blackhole-harness_b200", ROOT / "oracle", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


def golden(name: str) -> dict:
    with np.load(GOLDEN / name) as z:
        return {k: z[k] for k in z.files}


def golden_tiers(z: dict) -> list[dict]:
    """Tier dicts (numpy) from a golden file written by make_golden.flat_tiers."""
    tiers = []
    for ti in range(int(z["ntiers"])):
        t = {"bits": int(z[f"t{ti}_bits"]), "experts": z[f"t{ti}_experts"]}
        for proj in ("gate_proj", "up_proj", "down_proj"):
            t[proj] = {q: z[f"t{ti}_{proj}_{q}"] for q in ("idx", "block_scale", "expert_scale", "levels")}
        tiers.append(t)
    return tiers


@pytest.fixture(scope="session")
def oracle():
    import hexoracle
    hexoracle.build()
    return hexoracle
