"""The quantizer golden cases (tests/golden/quant.npz): seeds, shapes, table
sizes, scale blocks, and the seeded inputs regenerated with numpy."""

from __future__ import annotations

import numpy as np

# name: (seed, out, in, levels, block, weighted, zero block (row, first input) or None)
CASES = {
    "b3_blk32": (101, 40, 96, 8, 32, False, (3, 32)),
    "b4_blk32_energy": (102, 64, 160, 16, 32, True, None),
    "b3_blk128": (103, 32, 256, 8, 128, False, (5, 128)),
    "b3_blk32_sampled": (104, 384, 384, 8, 32, False, None),     # 147456 values > the 131072-value fit sample
}


def case_inputs(seed: int, out: int, n: int, block: int, weighted: bool, zero):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((out, n)) * 0.02).astype(np.float32)
    W[:, : n // 8] *= 4.0                                          # a few wide input columns
    if zero is not None:
        W[zero[0], zero[1]: zero[1] + block] = 0.0
    energy = (rng.random(n).astype(np.float32) + 0.05) if weighted else None
    return W, energy


# GPTQ onto the table (quantize(W, L, block, H=H), hex.py:207-227 -> gptq_table,
# hex.py:256-298): name: (seed, out, in, levels, block, calibration rows)
GPTQ_CASES = {
    "gptq_b3_blk32": (201, 64, 256, 8, 32, 512),
    "gptq_b4_blk32": (202, 48, 384, 16, 32, 768),
}


def gptq_inputs(seed: int, out: int, n: int, rows: int):
    """W [out, n] f32 and H = X^T X (float64) of seeded calibration rows X
    [rows, n], one input column never active (a dead column)."""
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((out, n)) * 0.02).astype(np.float32)
    X = rng.standard_normal((rows, n)).astype(np.float32) * np.linspace(0.2, 2.0, n, dtype=np.float32)
    X[:, 7] = 0.0
    H = X.T.astype(np.float64) @ X.astype(np.float64)
    return W, H
