"""Bit-exact probes of the small-batch kernels' own operands at the short tile
heights (32 and 64 weight rows) that few slots select.

As tests/test_gpu_probe.py, with one-hot activations so that each output is one
weight times an exact factor, but in many small calls of 8 tokens per expert
(one align block each), so that the layer picks its shortest tiles: with H=1024
and I=512, gate/up runs 32-row tiles (eight step groups over eight 128-input
steps) and down 64-row tiles (four step groups over four steps).  Every
(expert, row, input) of the up and down projections is compared with the
oracle's fp32 dequantization rounded to bf16 (blackhole/anatomy/hex.py:180-204).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from helpers import np_tiers

from blackhole_b200 import hex_data as hd

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
E, H, I = 4, 1024, 512
NB = 8                       # tokens per expert per call: one 8-slot block each


@pytest.fixture(scope="module", autouse=True)
def _clean_error_word():
    from blackhole_b200.hex_moe import device_status
    device_status(0, clear=True)
    yield
    assert device_status(0, clear=True) == 0, "a kernel set the device error word"


def _layer(block: int, seed: int, gate_const: float | None = None):
    from blackhole_b200.hex_moe import HexTier, layer_for
    L = hd.synth_layer(E, H, I, "mixed", block, seed=seed)
    tiers = []
    for t in L.tiers:
        if gate_const is not None:
            p = t["gate_proj"]
            p["levels"] = torch.full_like(p["levels"], gate_const)
            p["block_scale"] = torch.full_like(p["block_scale"], 0x38)
            p["expert_scale"] = torch.ones_like(p["expert_scale"])
        parts = [{q: v.clone().to(DEV) for q, v in t[p].items()} for p in ("gate_proj", "up_proj", "down_proj")]
        tiers.append(HexTier(t["bits"], t["experts"].to(DEV), *parts).prepare(E))
    return L, layer_for(tiers)


def _weights(L, proj: str, oracle) -> np.ndarray:
    rows, cols = (H, I) if proj == "down_proj" else (I, H)
    W = np.zeros((E, rows, cols), np.float32)
    for t in np_tiers(L.tiers):
        d = oracle.dequant(t[proj], t["bits"], L.block)
        for local, e in enumerate(t["experts"].tolist()):
            W[e] = d[local]
    return W


def _rne_bf16(a: np.ndarray) -> np.ndarray:
    return torch.as_tensor(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def _calls(ncols: int):
    """(first column, ids, weights) of each call: token e*NB + j routes to expert e
    and is one-hot at column c0 + j."""
    T = E * NB
    ids = (torch.arange(T, dtype=torch.int64) // NB).reshape(T, 1).to(DEV)
    w = torch.ones(T, 1, dtype=torch.float32, device=DEV)
    for c0 in range(0, ncols, NB):
        yield c0, T, ids, w


@pytest.mark.parametrize("block", [32, 128])
def test_down_operands_bitexact_short_tiles(oracle, block):
    L, layer = _layer(block, seed=170 + block)
    got = np.zeros((E, H, I), np.float32)
    for c0, T, ids, w in _calls(I):
        plan = layer.plan(ids, 8)
        sid = plan[0].cpu().numpy()
        act = np.zeros((sid.size, layer.desc.inter_pad), np.float32)
        valid = sid < T
        act[np.nonzero(valid)[0], c0 + sid[valid] % NB] = 1.0
        y = layer.down(torch.as_tensor(act).to(torch.bfloat16).to(DEV), w, plan, 8).float().cpu().numpy()   # [T, H]
        got[:, :, c0:c0 + NB] = y.reshape(E, NB, H).transpose(0, 2, 1)
    want = _rne_bf16(_weights(L, "down_proj", oracle))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{int((got != want).sum())} of {got.size} down operands differ"


@pytest.mark.parametrize("block", [32, 128])
def test_up_operands_bitexact_short_tiles(oracle, block):
    L, layer = _layer(block, seed=180 + block, gate_const=64.0)
    got = np.zeros((E, I, H), np.float32)
    for c0, T, ids, w in _calls(H):
        x = torch.zeros(T, H, dtype=torch.bfloat16)
        x[torch.arange(T), c0 + torch.arange(T) % NB] = 1.0
        plan = layer.plan(ids, 8)
        xs = layer.gather(x.to(DEV), 1, plan, 8)
        act = layer.gate_up(xs, T, 1, plan, 8).float().cpu().numpy()
        sid = plan[0].cpu().numpy()
        rows = np.nonzero(sid < T)[0]
        per = np.zeros((T, I), np.float32)
        per[sid[rows]] = act[rows, :I]
        got[:, :, c0:c0 + NB] = per.reshape(E, NB, I).transpose(0, 2, 1) / 64.0
    want = _rne_bf16(_weights(L, "up_proj", oracle))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{int((got != want).sum())} of {got.size} up operands differ"
