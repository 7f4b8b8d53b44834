"""The HEX quantizer (hexmoe_quantize, blackhole_b200.quant): the reference's
blackhole/anatomy/hex.py quantize (hex.py:207-227, no Hessian) restated on the
CPU (oracle/hexquant.py) and on the GPU.

CPU: the restatement equals the reference's own outputs (tests/golden/quant.npz,
written by tests/golden/make_golden_quant.py) bit for bit, the fp8 encode
rule, and the C ABI's argument checks.  GPU: the CUDA quantizer equals the
reference outputs bit for bit, a stack equals its matrices quantized one by
one, and its parts dequantize (hexmoe_dequant) to the restatement's weights.
"""

from __future__ import annotations

import ctypes
import hashlib
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden

sys.path.insert(0, str(GOLDEN))
from quant_cases import CASES, case_inputs  # noqa: E402

import hexquant  # noqa: E402  (oracle: test infrastructure)

DEV = torch.device("cuda", 0)


def _inputs(name):
    seed, out, n, L, block, weighted, zero = CASES[name]
    W, energy = case_inputs(seed, out, n, block, weighted, zero)
    z = golden("quant.npz")
    assert hashlib.sha256(W.tobytes()).digest() == z[f"{name}/sha256"].tobytes(), "seeded input changed"
    return W, energy, L, block, z


@pytest.mark.parametrize("name", list(CASES))
def test_restatement_matches_reference_golden(name):
    W, energy, L, block, z = _inputs(name)
    lev, es, codes, idx = hexquant.quantize(W, L, block, energy)
    assert np.array_equal(lev, z[f"{name}/levels"])
    assert es == z[f"{name}/expert_scale"][0]
    assert np.array_equal(codes, z[f"{name}/block_scale"])
    assert np.array_equal(idx, z[f"{name}/codes"])
    assert np.array_equal(hexquant.pack_bits(idx, int(np.log2(L))).view(np.int32), z[f"{name}/idx"])


def test_fp8_encode_rule():
    """Nearest finite e4m3 code, ties to the smaller value; a positive value at
    most half the smallest subnormal rounds to the -0 code (st.py:67-86)."""
    sub = np.float32(2.0 ** -9)
    got = hexquant.fp8_encode(np.array([0.0, sub / 4, sub / 2, sub * 0.75, 448.0, 1e9, 1.0, 1.0625, 1.0626],
                                       np.float32))
    assert got.tolist() == [0x00, 0x80, 0x80, 0x01, 0x7E, 0x7E, 0x38, 0x38, 0x39]


def test_quantize_argument_errors_before_any_device_work():
    from blackhole_b200 import _lib
    L = _lib.lib
    A = (None, None, 0, 20, None, None, None, None, None, None, None, 0, None)
    assert L.hexmoe_quantize(None, 1, 8, 64, 5, 32, *A) == _lib.HEXMOE_E_ARG     # levels
    assert L.hexmoe_quantize(None, 1, 8, 96, 8, 128, *A) == _lib.HEXMOE_E_ARG    # in % block
    assert L.hexmoe_quantize(None, 1, 8, 64, 8, 32, *A) == _lib.HEXMOE_E_ARG     # null pointers
    assert L.hexmoe_quantize_workspace_bytes(1, 8, 96, 128, 0, 0, 0) == 0       # in % block


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(CASES))
def test_quantize_matches_reference_golden(name):
    from blackhole_b200.quant import quantize
    W, energy, L, block, z = _inputs(name)
    got = quantize(torch.from_numpy(W).to(DEV), L, block,
                   torch.from_numpy(energy).to(DEV) if energy is not None else None)
    torch.cuda.synchronize()
    assert np.array_equal(got["levels"].cpu().numpy(), z[f"{name}/levels"])
    assert got["expert_scale"].cpu().numpy()[0] == z[f"{name}/expert_scale"][0]
    assert np.array_equal(got["block_scale"].cpu().numpy(), z[f"{name}/block_scale"])
    assert np.array_equal(got["idx"].view(torch.int32).cpu().numpy(), z[f"{name}/idx"])


@pytest.mark.gpu
@pytest.mark.parametrize("L,block,weighted", [(8, 32, False), (16, 32, True), (8, 128, True)])
def test_stack_equals_matrices_one_by_one(L, block, weighted):
    """Five matrices (one all zero, one with a single huge value) in one call:
    each equals the restatement of the reference on it alone."""
    from blackhole_b200.quant import quantize_stack
    rng = np.random.default_rng(7 + L + block)
    n, out, cols = 5, 48, 256
    W = (rng.standard_normal((n, out, cols)) * 0.03).astype(np.float32)
    W[1] = 0.0
    W[2, 7, 100] = 50.0
    energy = (rng.random((n, cols)).astype(np.float32) + 0.01) if weighted else None
    got = quantize_stack(torch.from_numpy(W).to(DEV), L, block,
                         torch.from_numpy(energy).to(DEV) if weighted else None)
    torch.cuda.synchronize()
    bits = int(np.log2(L))
    for e in range(n):
        lev, es, codes, idx = hexquant.quantize(W[e], L, block, energy[e] if weighted else None)
        assert np.array_equal(got["levels"][e].cpu().numpy(), lev), e
        assert got["expert_scale"][e].item() == es, e
        assert np.array_equal(got["block_scale"][e].cpu().numpy(), codes), e
        assert np.array_equal(got["idx"][e].view(torch.int32).cpu().numpy(), hexquant.pack_bits(idx, bits).view(np.int32)), e


@pytest.mark.gpu
def test_quantized_parts_dequantize_to_the_restatement():
    """The quantizer's parts through hexmoe_dequant (the layer's decode rule) give
    levels[idx] * fp8(code) * es of the restatement, bit for bit: producer and
    consumer of the format agree."""
    from blackhole_b200 import _lib
    from blackhole_b200.quant import quantize_stack
    rng = np.random.default_rng(3)
    n, out, cols, L, block = 3, 64, 256, 8, 32
    W = (rng.standard_normal((n, out, cols)) * 0.02).astype(np.float32)
    parts = quantize_stack(torch.from_numpy(W).to(DEV), L, block)
    outw = torch.empty(n, out, cols, dtype=torch.float32, device=DEV)
    cp = _lib.Parts(parts["idx"].data_ptr(), parts["block_scale"].data_ptr(), parts["expert_scale"].data_ptr(),
                    parts["levels"].data_ptr())
    _lib.check(_lib.lib.hexmoe_dequant(ctypes.byref(cp), 3, block, n, out, cols, out, cols, None, outw.data_ptr(),
                                       _lib.F32, outw.stride(0), outw.stride(1), 0, None), "hexmoe_dequant")
    torch.cuda.synchronize()
    for e in range(n):
        lev, es, codes, idx = hexquant.quantize(W[e], L, block)
        s = hexquant.FP8[codes].astype(np.float32) * np.float32(es)
        want = lev[idx] * np.repeat(s, block, axis=1)
        got = outw[e].cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.astype(np.float32).view(np.uint32)), e


def _q_from(idx: np.ndarray, lev: np.ndarray, codes: np.ndarray, es: float, block: int) -> np.ndarray:
    s = hexquant.FP8[codes].astype(np.float32) * np.float32(es)
    return lev[idx] * np.repeat(s, block, axis=1)


def test_gptq_restatement_matches_reference_golden():
    from quant_cases import GPTQ_CASES, gptq_inputs
    z = golden("quant.npz")
    for name, (seed, out, n, L, block, rows) in GPTQ_CASES.items():
        W, H = gptq_inputs(seed, out, n, rows)
        assert hashlib.sha256(W.tobytes() + H.tobytes()).digest() == z[f"{name}/sha256"].tobytes()
        lev, es, codes, idx = hexquant.quantize(W, L, block, H=H)
        assert np.array_equal(lev, z[f"{name}/levels"]) and np.array_equal(codes, z[f"{name}/block_scale"])
        assert np.array_equal(idx, z[f"{name}/codes"]), name


@pytest.mark.gpu
def test_gptq_matches_reference():
    """GPTQ onto the table on the GPU against the reference's outputs: the table
    and block scales (which GPTQ does not touch) bit for bit; the indices, whose
    error feedback sums in float32 in another order than the reference's, agree
    on at least 99 % of the weights, and the GPTQ objective trace((W-Q) H (W-Q)^T)
    is within 1 % of the reference's and below nearest rounding's."""
    from quant_cases import GPTQ_CASES, gptq_inputs

    from blackhole_b200.quant import quantize
    z = golden("quant.npz")
    for name, (seed, out, n, L, block, rows) in GPTQ_CASES.items():
        W, H = gptq_inputs(seed, out, n, rows)
        got = quantize(torch.from_numpy(W).to(DEV), L, block, H=torch.from_numpy(H).to(DEV))
        torch.cuda.synchronize()
        lev = got["levels"].cpu().numpy()
        codes = got["block_scale"].cpu().numpy()
        es = got["expert_scale"].cpu().numpy()[0]
        assert np.array_equal(lev, z[f"{name}/levels"]) and np.array_equal(codes, z[f"{name}/block_scale"]), name
        bits = int(np.log2(L))
        words = got["idx"].view(torch.int32).cpu().numpy().view(np.uint32)
        mine = _unpack(words, bits, n)
        ref = z[f"{name}/codes"]
        agree = float((mine == ref).mean())
        assert agree >= 0.99, (name, agree)
        e_mine = hexquant.gptq_error(W, _q_from(mine, lev, codes, es, block), H)
        e_ref = hexquant.gptq_error(W, _q_from(ref, lev, codes, es, block), H)
        _, _, _, near = hexquant.quantize(W, L, block)
        e_near = hexquant.gptq_error(W, _q_from(near, lev, codes, es, block), H)
        assert abs(e_mine - e_ref) <= 0.01 * e_ref and e_mine < e_near, (name, e_mine, e_ref, e_near)


def _unpack(words: np.ndarray, bits: int, n: int) -> np.ndarray:
    out = words.shape[0]
    w = words.reshape(out, -1, bits).astype(np.uint64)
    vals = []
    for i in range(32):
        off = i * bits
        wi, sh = off // 32, off % 32
        v = w[:, :, wi] >> np.uint64(sh)
        if sh + bits > 32:
            v |= w[:, :, wi + 1] << np.uint64(32 - sh)
        vals.append(v & np.uint64((1 << bits) - 1))
    return np.stack(vals, -1).reshape(out, -1)[:, :n].astype(np.uint8)
