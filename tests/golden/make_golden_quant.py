"""Write tests/golden/quant.npz by running the reference HEX quantizer.

Run in a container that has the reference tree (OliverVillson/BlackHole-Harness):

    REF=/path/to/BlackHole-Harness python tests/golden/make_golden_quant.py

Each case quantizes a seeded matrix with blackhole.anatomy.hex.quantize
(blackhole/anatomy/hex.py:207-227: block scales, the k-means level table, nearest
rounding, or with a Hessian GPTQ onto the table, gptq_table hex.py:256-298) and
records the saved parts (Hex.packed()).
The inputs are not stored: they are regenerated from the recorded seed with
numpy's default_rng (checked by sha256), and so are the per-input energies of
the weighted case.
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

if "REF" not in os.environ:
    sys.exit("make_golden_quant.py: set REF to the root of a BlackHole-Harness checkout (the reference implementation)")
sys.path.insert(0, str(Path(os.environ["REF"])))

import numpy as np  # noqa: E402
from blackhole.anatomy.hex import quantize  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from quant_cases import CASES, GPTQ_CASES, case_inputs, gptq_inputs  # noqa: E402


def main() -> None:
    out = {}
    for name, (seed, o, n, L, block, weighted, zero) in CASES.items():
        W, energy = case_inputs(seed, o, n, block, weighted, zero)
        h = quantize(W, L=L, block=block, energy=energy)
        p = h.packed()
        out[f"{name}/sha256"] = np.frombuffer(hashlib.sha256(W.tobytes()).digest(), np.uint8)
        out[f"{name}/idx"] = p["idx"].view(np.int32)
        out[f"{name}/block_scale"] = p["block_scale"]
        out[f"{name}/expert_scale"] = p["expert_scale"]
        out[f"{name}/levels"] = p["levels"]
        out[f"{name}/codes"] = h.idx
        print(name, W.shape, "levels", p["levels"][:3], "es", p["expert_scale"], "words", p["idx"].shape)
    for name, (seed, o, n, L, block, rows) in GPTQ_CASES.items():
        W, H = gptq_inputs(seed, o, n, rows)
        h = quantize(W, L=L, block=block, H=H)
        p = h.packed()
        out[f"{name}/sha256"] = np.frombuffer(hashlib.sha256(W.tobytes() + H.tobytes()).digest(), np.uint8)
        out[f"{name}/idx"] = p["idx"].view(np.int32)
        out[f"{name}/block_scale"] = p["block_scale"]
        out[f"{name}/expert_scale"] = p["expert_scale"]
        out[f"{name}/levels"] = p["levels"]
        out[f"{name}/codes"] = h.idx
        print(name, W.shape, "levels", p["levels"][:3])
    np.savez_compressed(HERE / "quant.npz", **out)


if __name__ == "__main__":
    main()
