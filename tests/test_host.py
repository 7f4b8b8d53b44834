"""Host-side logic that needs no GPU: the C-ABI library loads and exports every
symbol the header declares; HexTier.prepare mirrors the reference's checks and
builds the kernel layout; the package fails loudly without CUDA."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch
from conftest import ROOT
from helpers import np_tiers

from blackhole_b200 import hex_data as hd


def header_functions() -> set[str]:
    src = (ROOT / "include" / "hexmoe.h").read_text()
    return set(re.findall(r"HEXMOE_API\s+[\w\s\*]+?\b(hexmoe_\w+)\s*\(", src))


def test_library_exports_every_header_symbol():
    from blackhole_b200 import _lib
    declared = header_functions()
    assert len(declared) >= 12
    assert declared == set(_lib.EXPORTS)
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared:
        assert hasattr(lib, name), name
    assert _lib.lib.hexmoe_abi_version() == 1


def test_noalloc_scratch_constant_matches_header():
    """_lib.NOALLOC_SCRATCH_BYTES mirrors HEXMOE_NOALLOC_SCRATCH_BYTES (the tests probe that limit)."""
    from blackhole_b200 import _lib
    src = (ROOT / "include" / "hexmoe.h").read_text()
    m = re.search(r"#define\s+HEXMOE_NOALLOC_SCRATCH_BYTES\s+\((\d+)u\s*<<\s*(\d+)\)", src)
    assert m, "HEXMOE_NOALLOC_SCRATCH_BYTES not found"
    assert int(m.group(1)) << int(m.group(2)) == _lib.NOALLOC_SCRATCH_BYTES


def test_argument_errors_raise_valueerror_without_gpu():
    from blackhole_b200 import _lib
    rc = _lib.lib.hexmoe_layer_create(None, None)
    assert rc == _lib.HEXMOE_E_ARG and "null" in _lib.last_error()
    with pytest.raises(ValueError):
        _lib.check(rc, "create")
    d = _lib.LayerDesc()
    d.num_experts, d.hidden, d.inter, d.hidden_pad, d.inter_pad, d.block, d.num_tiers = 8, 100, 64, 128, 128, 32, 1
    h = ctypes.c_void_p()
    assert _lib.lib.hexmoe_layer_create(ctypes.byref(d), ctypes.byref(h)) == _lib.HEXMOE_E_ARG   # 100 % 32 != 0
    assert _lib.lib.hexmoe_forward(None, None, 0, 1, 1, None, None, 0, None, 0, 0, None, 0, None) == _lib.HEXMOE_E_ARG
    assert _lib.lib.hexmoe_tile_index(None, 3, 1, 100, 128, None, None) == _lib.HEXMOE_E_ARG    # rows_pad % 128
    assert _lib.lib.hexmoe_tile_index(None, 5, 1, 128, 128, None, None) == _lib.HEXMOE_E_ARG    # bits
    assert _lib.lib.hexmoe_tile_index(None, 3, 1, 128, 128, None, None) == _lib.HEXMOE_E_ARG    # null pointers
    # per-slot forward and row-mapped combine: argument errors before any device work
    assert _lib.lib.hexmoe_forward_slots(None, None, 1, 4, 2, None, None, 0, None, 0, None, 0, None) == _lib.HEXMOE_E_ARG
    assert _lib.lib.hexmoe_combine_rows(None, _lib.BF16, 8, 4, 2, 128, None, None, _lib.BF16, None) == _lib.HEXMOE_E_ARG
    assert _lib.lib.hexmoe_combine_rows(None, _lib.F32, 8, 4, 2, 128, None, None, _lib.BF16, None) == _lib.HEXMOE_E_DTYPE
    assert _lib.lib.hexmoe_align(None, _lib.I32, 100, 0, 16, None, None, None, None, 0, None) == _lib.HEXMOE_E_ARG


def make_tier(E=12, H=128, I=64, bits=3, block=32, seed=0):
    L = hd.synth_layer(E, H, I, str(bits), block, seed)
    t = L.tiers[0]
    from blackhole_b200.hex_moe import HexTier
    return HexTier(t["bits"], t["experts"], dict(t["gate_proj"]), dict(t["up_proj"]), dict(t["down_proj"])), L


def test_prepare_matches_reference_views_and_pads_small_shapes():
    tier, _ = make_tier(E=12, H=128, I=64, bits=3, block=32)
    tier.prepare(12)
    assert tier.gate_proj["idx"].dtype == torch.int32                  # uint32 viewed as int32 (hex_moe.py:187-188)
    assert tier.lookup.tolist() == list(range(12)) and tier.experts.dtype == torch.int32
    assert tier.block == 32 and tier.dims() == (64, 128)
    g = tier.kernel_parts["gate_proj"]
    assert (g["rows_pad"], g["cols_pad"]) == (128, 128)                 # I = 64 padded to one 128-row tile
    assert g["idx"].shape == (12, 128, 128 // 32 * 3)
    assert torch.equal(g["idx"][:, :64], tier.gate_proj["idx"]) and not g["idx"][:, 64:].any()
    assert not g["block_scale"][:, 64:].any()                          # zero scale -> zero weight in padding
    d = tier.kernel_parts["down_proj"]
    assert d["idx"].shape == (12, 128, 128 // 32 * 3) and torch.equal(d["idx"][:, :, :6], tier.down_proj["idx"])


def test_prepare_keeps_production_layout_zero_copy():
    tier, _ = make_tier(E=4, H=256, I=128, bits=4, block=128)
    tier.prepare(4)
    assert tier.block == 128
    for p in ("gate_proj", "up_proj", "down_proj"):
        kp = tier.kernel_parts[p]
        assert kp["idx"].data_ptr() == getattr(tier, p)["idx"].data_ptr()   # read as stored
        assert kp["block_scale"].data_ptr() == getattr(tier, p)["block_scale"].data_ptr()


def test_prepare_rejects_bad_tiers():
    tier, _ = make_tier()
    tier.bits = 5
    with pytest.raises(ValueError):
        tier.prepare(12)
    tier, _ = make_tier()
    tier.gate_proj["block_scale"] = tier.gate_proj["block_scale"][:, :, :1].contiguous()
    with pytest.raises(ValueError):
        tier.prepare(12)


def test_cpu_tensors_fail_loudly():
    from blackhole_b200.hex_moe import align, hex_moe
    tier, L = make_tier()
    tier.prepare(12)
    x = torch.zeros(2, 128, dtype=torch.bfloat16)
    w, ids = hd.synth_routing(2, 12, 4)
    with pytest.raises(ValueError, match="CUDA"):
        hex_moe(x, w, ids, [tier])
    with pytest.raises(ValueError, match="CUDA"):
        align(ids.reshape(-1), 12, 16)


def test_synth_layer_distributions():
    L = hd.synth_layer(8, 256, 512, "mixed", 128, seed=3)
    assert [t["bits"] for t in L.tiers] == [4, 3] and sum(len(t["experts"]) for t in L.tiers) == 8
    lev = L.tiers[0]["gate_proj"]["levels"]
    assert torch.all(lev[:, 1:] >= lev[:, :-1])                              # sorted tables
    assert torch.equal(lev, lev.to(torch.float16).float())                  # fp16-representable
    bs = L.tiers[1]["down_proj"]["block_scale"]
    assert bs.shape == (4, 256, 512 // 128) and bs.dtype == torch.uint8
    w, ids = hd.synth_routing(64, 8, 2, seed=1)
    assert torch.allclose(w.sum(-1), torch.ones(64)) and ids.dtype == torch.int64
    assert hd.tier_bytes(3, 2048, 768, 128) == 1806444                      # bytes per expert, 3-bit, block 128
    npt = np_tiers(L.tiers)
    assert npt[0]["gate_proj"]["idx"].dtype.name == "int32"
