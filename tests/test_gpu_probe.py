"""Bit-exact probes of the weights the grouped GEMM itself consumes.

The dequantization tests check hexmoe_dequant, a separate kernel.  These drive
the GEMM phases (hexmoe_gate_up / hexmoe_down, through the C ABI) with one-hot
activations, so that every output is a single weight times an exact factor:

  down     act row = one-hot at input column c, top-k weight 1.0
           -> y[slot, o] = (W_down[o, c] rounded to the operand type) * 1.0,
              one product accumulated in fp32: exactly RNE16(W_down[o, c])
  up       gate weights all 64.0 (levels 64, scale code 0x38 = 1.0), x one-hot
           at column c -> silu(64) = 64 exactly in fp32, so
              act[slot, o] = RNE16(64 * RNE16(W_up[o, c])) = 64 * RNE16(W_up[o, c])
  gate     up weights all 1.0 -> act[slot, o] = RNE16(silu(RNE16(W_gate[o, c]))),
           checked within one unit in the last place of the 16-bit result
           (silu's exp differs between the GPU and numpy in the last fp32 bit)

Every (expert, row, input) of every projection is covered, for 3- and 4-bit
tiers, scale blocks 32 and 128, bf16 and f16 operands, and tile heights 8 (the
small-batch mma.sync kernels and their precomputed code tables), 16 (tcgen05,
down with split MMA issue) and 128 (tcgen05, one issuer).  The reference value is the
oracle's fp32 dequantization (blackhole/anatomy/hex.py:180-204) rounded to
nearest even.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from helpers import np_tiers

from blackhole_b200 import hex_data as hd

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
E, H, I = 4, 256, 384        # 2 tiers x 2 experts; every input column gets one token per expert


@pytest.fixture(scope="module", autouse=True)
def _clean_error_word():
    from blackhole_b200.hex_moe import device_status
    device_status(0, clear=True)
    yield
    assert device_status(0, clear=True) == 0, "a kernel set the device error word"


def _rne16(a: np.ndarray, dt: torch.dtype) -> np.ndarray:
    return torch.as_tensor(np.ascontiguousarray(a, dtype=np.float32)).to(dt).float().numpy()


def _tiers(block: int, seed: int, gate_const: float | None = None, up_const: float | None = None):
    """Synthetic mixed 3/4-bit layer; optionally every gate / up weight a constant
    (all levels equal to it, scale code 0x38 = 1.0, expert scale 1)."""
    L = hd.synth_layer(E, H, I, "mixed", block, seed=seed)
    for t in L.tiers:
        for name, c in (("gate_proj", gate_const), ("up_proj", up_const)):
            if c is not None:
                p = t[name]
                p["levels"] = torch.full_like(p["levels"], c)
                p["block_scale"] = torch.full_like(p["block_scale"], 0x38)
                p["expert_scale"] = torch.ones_like(p["expert_scale"])
    return L


def _layer(L):
    from blackhole_b200.hex_moe import HexTier, layer_for
    tiers = []
    for t in L.tiers:
        parts = [{q: v.clone().to(DEV) for q, v in t[p].items()} for p in ("gate_proj", "up_proj", "down_proj")]
        tiers.append(HexTier(t["bits"], t["experts"].to(DEV), *parts).prepare(E))
    return layer_for(tiers)


def _expert_weights(L, proj: str, oracle) -> np.ndarray:
    """fp32 weights [E, rows, cols] of one projection in global expert order (oracle)."""
    rows, cols = (H, I) if proj == "down_proj" else (I, H)
    W = np.zeros((E, rows, cols), np.float32)
    for t in np_tiers(L.tiers):
        d = oracle.dequant(t[proj], t["bits"], L.block)
        for local, e in enumerate(t["experts"].tolist()):
            W[e] = d[local]
    return W


def _one_hot_batch(ncol: int):
    """Token t = e * ncol + c routes to expert e (top-1, weight 1); its one-hot column is c."""
    T = E * ncol
    ids = torch.arange(T, dtype=torch.int64).div(ncol, rounding_mode="floor").reshape(T, 1)
    w = torch.ones(T, 1, dtype=torch.float32)
    return T, ids.to(DEV), w.to(DEV)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("block", [32, 128])
@pytest.mark.parametrize("bm", [8, 16, 128])
def test_down_operands_bitexact(oracle, dt, block, bm):
    L = _tiers(block, seed=70 + block + bm)
    layer = _layer(L)
    T, ids, w = _one_hot_batch(I)
    plan = layer.plan(ids, bm)
    sid = plan[0].cpu().numpy()
    ipad = layer.desc.inter_pad
    act = np.zeros((sid.size, ipad), np.float32)
    valid = sid < T
    act[np.nonzero(valid)[0], sid[valid] % I] = 1.0          # plan row r holds slot sid[r]: one-hot at its column
    y = layer.down(torch.as_tensor(act).to(dt).to(DEV), w, plan, bm).float().cpu().numpy()   # [T, H]
    W = _expert_weights(L, "down_proj", oracle)                                          # [E, H, I]
    got = y.reshape(E, I, H).transpose(0, 2, 1)                                          # [E, H(o), I(c)]
    want = _rne16(W, dt)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{int((got != want).sum())} of {got.size} down operands differ"


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("block", [32, 128])
@pytest.mark.parametrize("bm", [8, 16, 128])
def test_up_operands_bitexact(oracle, dt, block, bm):
    L = _tiers(block, seed=80 + block + bm, gate_const=64.0)
    layer = _layer(L)
    T, ids, w = _one_hot_batch(H)
    x = torch.zeros(T, H, dtype=dt)
    x[torch.arange(T), torch.arange(T) % H] = 1.0
    x = x.to(DEV)
    plan = layer.plan(ids, bm)
    xs = layer.gather(x, 1, plan, bm)
    act = layer.gate_up(xs, T, 1, plan, bm).float().cpu().numpy()        # [rows, inter_pad], plan order
    sid = plan[0].cpu().numpy()
    rows = np.nonzero(sid < T)[0]
    got = np.zeros((T, I), np.float32)
    got[sid[rows]] = act[rows, :I]
    got = got.reshape(E, H, I).transpose(0, 2, 1) / 64.0                # [E, I(o), H(c)]
    want = _rne16(_expert_weights(L, "up_proj", oracle), dt)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{int((got != want).sum())} of {got.size} up operands differ"


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("block", [32, 128])
@pytest.mark.parametrize("bm", [8, 64])
def test_gate_operands_within_one_ulp(oracle, dt, block, bm):
    L = _tiers(block, seed=90 + block, up_const=1.0)
    layer = _layer(L)
    T, ids, w = _one_hot_batch(H)
    x = torch.zeros(T, H, dtype=dt)
    x[torch.arange(T), torch.arange(T) % H] = 1.0
    plan = layer.plan(ids, bm)
    xs = layer.gather(x.to(DEV), 1, plan, bm)
    act = layer.gate_up(xs, T, 1, plan, bm).float().cpu().numpy()
    sid = plan[0].cpu().numpy()
    rows = np.nonzero(sid < T)[0]
    got = np.zeros((T, I), np.float32)
    got[sid[rows]] = act[rows, :I]
    got = got.reshape(E, H, I).transpose(0, 2, 1)
    g = _rne16(_expert_weights(L, "gate_proj", oracle), dt).astype(np.float32)
    want = _rne16(g / (np.float32(1.0) + np.exp(-g, dtype=np.float32)), dt)
    # one unit in the last place of the 16-bit value, as int distance of the 16-bit patterns
    gi = torch.as_tensor(got).to(dt).view(torch.int16).int().numpy()
    wi = torch.as_tensor(want).to(dt).view(torch.int16).int().numpy()
    assert np.abs(gi - wi).max() <= 1
    assert (gi == wi).mean() > 0.99
