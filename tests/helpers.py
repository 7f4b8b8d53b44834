"""Shared helpers for the parity tests: synthetic layers on the device and their
numpy copies for the CPU oracle."""

from __future__ import annotations

import numpy as np
import torch

PROJ = ("gate_proj", "up_proj", "down_proj")
PARTS = ("idx", "block_scale", "expert_scale", "levels")


def np_tiers(tiers: list[dict]) -> list[dict]:
    """Tier dicts of torch tensors (any device) -> numpy copies for the oracle."""
    out = []
    for t in tiers:
        d = {"bits": int(t["bits"]), "experts": np.asarray(t["experts"].cpu().numpy() if torch.is_tensor(t["experts"])
                                                          else t["experts"]).astype(np.int64)}
        for p in PROJ:
            d[p] = {}
            for q in PARTS:
                v = t[p][q]
                if torch.is_tensor(v):
                    v = v.cpu()
                    if v.dtype == torch.uint32:
                        v = v.view(torch.int32)
                    v = v.numpy()
                d[p][q] = v
        out.append(d)
    return out


def torch_tiers(tiers: list[dict], device) -> list[dict]:
    """numpy / torch tier dicts -> torch tensors on `device` (fresh copies)."""
    out = []
    for t in tiers:
        d = {"bits": int(t["bits"]), "experts": torch.as_tensor(np.asarray(t["experts"])).to(device)}
        for p in PROJ:
            d[p] = {q: torch.as_tensor(np.asarray(t[p][q])).clone().to(device) if not torch.is_tensor(t[p][q])
                    else t[p][q].clone().to(device) for q in PARTS}
        out.append(d)
    return out


def hex_tiers(tiers: list[dict], E: int, device):
    from blackhole_b200.hex_moe import HexTier
    return [HexTier(t["bits"], t["experts"], *(dict(t[p]) for p in PROJ)).prepare(E)
            for t in torch_tiers(tiers, device)]


def rel_err(got: np.ndarray, want: np.ndarray) -> float:
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


def within(got: np.ndarray, want: np.ndarray, rtol: float = 2e-2, atol: float = 1e-2) -> bool:
    """The layer tolerance of the benchmark spec: |got - want| <= atol + rtol * |want|."""
    return bool(np.all(np.abs(got - want) <= atol + rtol * np.abs(want)))
