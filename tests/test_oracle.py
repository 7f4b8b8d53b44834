"""The CPU oracle pinned against the reference's golden vectors and known answers.

Known-answer tests restate the reference's own: runtime/tests/test_hex_moe.py:36-61
and tests/test_hex.py:13-20, 43-57, 70-78.  Golden files come from running the
reference itself (tests/golden/make_golden.py)."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden, golden_tiers

from blackhole_b200 import hex_data as hd


def test_fp8_table_matches_reference_dequant(oracle):
    want = golden("fp8_kat.npz")["table"]
    got = oracle.fp8_table()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))       # bitwise, signed zeros included
    # tests/test_hex.py:13-20 values, and the 0x7F / 0xFF quirk (+-480, not NaN)
    assert got[0x38] == 1.0 and got[0x00] == 0.0 and got[0x7F] == 480.0 and got[0xFF] == -480.0
    assert got[0x01] == 0.001953125 and got[0x7E] == 448.0


def test_pack_matches_reference(oracle):
    z = golden("pack.npz")
    for bits in (3, 4):
        words = oracle.pack(z[f"codes{bits}"], bits)
        assert np.array_equal(words.view(np.int32), z[f"words{bits}"])
        assert np.array_equal(oracle.unpack(words, bits, 96), z[f"codes{bits}"])
        # the package's own (torch) packer agrees too
        assert np.array_equal(hd.pack(torch.from_numpy(z[f"codes{bits}"].astype(np.int64)), bits)
                              .view(torch.int32).numpy(), z[f"words{bits}"])


def test_pack_roundtrip_matches_bitstream(oracle):
    """runtime/tests/test_hex_moe.py:36-44: levels = arange, scale code 0x38, es 1."""
    rng = np.random.default_rng(0)
    for bits in (3, 4):
        codes = rng.integers(0, 2 ** bits, (2, 5, 64)).astype(np.uint8)
        words = oracle.pack(codes, bits)
        assert words.shape == (2, 5, 64 // 32 * bits)
        parts = {"idx": words, "block_scale": np.full((2, 5, 2), 0x38, np.uint8),
                 "expert_scale": np.ones(2, np.float32),
                 "levels": np.tile(np.arange(2 ** bits, dtype=np.float32), (2, 1))}
        assert np.array_equal(oracle.dequant(parts, bits), codes.astype(np.float32))


def test_unpack_padding_roundtrip(oracle):
    """tests/test_hex.py:52-57: 70 inputs, padded to 96."""
    rng = np.random.default_rng(3)
    for bits in (3, 4):
        idx = rng.integers(0, 2 ** bits, (5, 70)).astype(np.uint8)
        padded = np.zeros((5, 96), np.uint8)
        padded[:, :70] = idx
        words = oracle.pack(padded, bits)
        assert words.shape == (5, 3 * bits)
        assert np.array_equal(oracle.unpack(words, bits, 96)[:, :70], idx)


@pytest.mark.parametrize("bits", [3, 4])
def test_dequant_bitexact_vs_reference(oracle, bits):
    z = golden(f"dequant_b{bits}.npz")
    got = oracle.dequant(z, bits)
    assert np.array_equal(got.view(np.uint32), z["W"].view(np.uint32))


def test_block128_equals_expanded_block32(oracle):
    rng = np.random.default_rng(1)
    n, rows, cols, bits = 2, 9, 256, 3
    parts = {"idx": rng.integers(0, 2 ** 32, (n, rows, cols // 32 * bits), dtype=np.uint64).astype(np.uint32),
             "block_scale": rng.integers(0, 256, (n, rows, cols // 128)).astype(np.uint8),
             "expert_scale": rng.random(n).astype(np.float32),
             "levels": np.sort(rng.standard_normal((n, 8)).astype(np.float32), -1)}
    w128 = oracle.dequant(parts, bits, block=128)
    p32 = dict(parts, block_scale=np.repeat(parts["block_scale"], 4, axis=-1))
    assert np.array_equal(w128.view(np.uint32), oracle.dequant(p32, bits).view(np.uint32))


def test_align_matches_reference(oracle):
    z = golden("align.npz")
    names = sorted({k.rsplit("_", 1)[0] for k in z if k.endswith("_ids")})
    assert len(names) >= 10
    for name in names:
        n, bm = (int(v) for v in z[f"{name}_meta"])
        sid, eid, npp = oracle.align(z[f"{name}_ids"], n, bm)
        assert np.array_equal(sid, z[f"{name}_sid"]), name
        assert np.array_equal(eid, z[f"{name}_eid"]), name
        assert np.array_equal(npp, z[f"{name}_npp"]), name


def test_align_groups_and_pads(oracle):
    """runtime/tests/test_hex_moe.py:47-61."""
    ids = np.array([2, 0, 0, 2, 2, 1, 3, 0])
    sid, eid, npp = oracle.align(ids, 4, 4)
    S = ids.size
    seen = []
    for b, e in enumerate(eid.tolist()):
        rows = sid[b * 4:(b + 1) * 4].tolist()
        if b * 4 >= int(npp[0]):
            assert e < 0
            continue
        for r in rows:
            if r < S:
                assert ids[r] == e
                seen.append(r)
    assert sorted(seen) == list(range(S))


@pytest.mark.parametrize("T", [1, 3, 40])
@pytest.mark.parametrize("xdt", ["f32", "bf16"])
def test_moe_reference_matches_reference(oracle, T, xdt):
    z = golden(f"moe_ref_T{T}.npz")
    tiers = golden_tiers(z)
    x = z["x32"] if xdt == "f32" else z["xbf16"]
    got = oracle.moe_reference(x, z["w"], z["ids"], tiers, int(z["E"]),
                               act_dtype="float32" if xdt == "f32" else "bfloat16")
    want = z["out_f32"] if xdt == "f32" else z["out_bf16"]
    err = np.abs(got - want).max() / np.abs(want).max()
    # fp32 summation order differs from torch's BLAS; the bf16 case can also move one
    # rounding of h across a bf16 step
    assert err < (2e-6 if xdt == "f32" else 2e-3), err


def test_moe_cfg1_matches_reference(oracle):
    """The tiny benchmark config through block-128 scales, regenerated from seeds."""
    import hashlib
    z = golden("moe_cfg1.npz")
    c = hd.CONFIGS["cfg1"]
    s_layer, s_route, s_x = (int(v) for v in z["seeds"])
    L = hd.synth_layer(c["E"], c["H"], c["I"], c["bits"], c["block"], seed=s_layer)
    w, ids = hd.synth_routing(c["T"][0], c["E"], c["k"], seed=s_route)
    x = hd.synth_x(c["T"][0], c["H"], seed=s_x)

    def digest(*ts):
        h = hashlib.sha256()
        for t in ts:
            h.update(np.ascontiguousarray(t.cpu().numpy()).tobytes())
        return h.hexdigest()

    parts = ("idx", "block_scale", "expert_scale", "levels")
    for t, d in zip(L.tiers, z["tier_digests"]):
        assert digest(*(t[p][q] for p in ("gate_proj", "up_proj", "down_proj") for q in parts), t["experts"]) == d
    assert digest(x.float()) == str(z["x_digest"]) and digest(w, ids) == str(z["route_digest"])
    tiers = [{"bits": t["bits"], "experts": t["experts"].numpy(),
              **{p: {q: t[p][q].numpy() if t[p][q].dtype != torch.uint32 else t[p][q].view(torch.int32).numpy()
                     for q in parts} for p in ("gate_proj", "up_proj", "down_proj")}} for t in L.tiers]
    got = oracle.moe_reference(x.float().numpy(), w.numpy(), ids.numpy(), tiers, c["E"], block=c["block"])
    want = z["out_bf16"]
    assert np.abs(got - want).max() / np.abs(want).max() < 2e-3
    g0 = oracle.dequant(tiers[0]["gate_proj"], tiers[0]["bits"], block=c["block"])
    assert np.array_equal(g0[:, :4].view(np.uint32), z["gate0_rows"].view(np.uint32))


def test_oracle_matches_interpreted_triton_kernel(oracle):
    """Secondary oracle: the reference's own Triton fused path, interpreted, fp32 x."""
    z = golden("triton_interp.npz")
    got = oracle.moe_reference(z["x32"], z["w"], z["ids"], golden_tiers(z), int(z["E"]), act_dtype="float32")
    assert np.abs(got - z["out"]).max() / np.abs(z["out"]).max() < 1e-4
