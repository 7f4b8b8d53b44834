"""The HEX quantizer on the GPU (hexmoe_quantize): the producer side of the format.

Mirrors blackhole/anatomy/hex.py `quantize(W, L, block, energy, H)` (hex.py:207-227)
over a stack of matrices, without a Hessian with the same results bit for bit:
block scales (hex.py:60-70), the weighted k-means level
table fitted on the reference's own sample of the values (hex.py:73-90, numpy
default_rng(0), 2^17 values, drawn here on the host exactly as the reference
draws them), nearest-level indices (hex.py:93-95) packed as the layout's bit
stream (hex.py:136-150).  With a Hessian the indices come from GPTQ onto the
table (hex.py:234-282): the factorizations of its preparation on the device
(torch.linalg, as the reference's gptq_table_torch), the column sweep in
hexmoe_quantize; its float32 sums run in another order than the reference's,
so its indices agree with the reference's up to rounding-order flips.  The
outputs are the parts of one tier's projection (hex_ref.py:1-12), ready for
HexTier.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib

SAMPLE = 1 << 17       # fit_table's sample (hex.py:74)
ITERS = 20             # fit_table's Lloyd iterations (hex.py:74)


def sample_positions(size: int, seed: int = 0, sample: int = SAMPLE) -> np.ndarray | None:
    """The flat positions fit_table fits a matrix of `size` values on (hex.py:79-82):
    None (every value) up to `sample` values, else numpy default_rng(seed) draws."""
    if size <= sample:
        return None
    return np.random.default_rng(seed).integers(0, size, sample)


_SAMPLES: dict = {}


def _sample_on(size: int, dev) -> torch.Tensor | None:
    """sample_positions(size) on `dev`, drawn once per (size, device)."""
    key = (size, str(dev))
    if key not in _SAMPLES:
        pos = sample_positions(size)
        _SAMPLES[key] = torch.as_tensor(pos, dtype=torch.int64, device=dev) if pos is not None else None
    return _SAMPLES[key]


def gptq_prep(W: torch.Tensor, H: torch.Tensor, damp: float = 0.01) -> tuple[torch.Tensor, torch.Tensor]:
    """Per matrix of W [n, out, in] and its Hessian H ([in, in] or [n, in, in],
    sum x x^T): the dead inputs (no activation or an all-zero weight column)
    and the upper Cholesky factor of the damped inverse Hessian as f32, on the
    device: hex.py:234-253 / gptq_table_torch's preparation, damping tripled up
    to six times until both factorizations succeed."""
    n, out, cols = W.shape
    Hd = H.to(device=W.device, dtype=torch.float64)
    if Hd.dim() == 2:
        Hd = Hd.expand(n, cols, cols)
    eye = torch.eye(cols, dtype=torch.float64, device=W.device)
    U = torch.empty(n, cols, cols, dtype=torch.float32, device=W.device)
    dead_all = torch.empty(n, cols, dtype=torch.uint8, device=W.device)
    for e in range(n):
        h = Hd[e].clone()
        if not bool(h.diagonal().any()):
            h = eye.clone()
        dead = (h.diagonal() == 0) | (W[e].abs().amax(0) == 0)
        live = (~dead).to(torch.float64)
        h = h * live[:, None] * live[None, :] + eye * dead.to(torch.float64)[:, None]
        base = float((h.diagonal() * live).sum() / live.sum().clamp(min=1)) or 1.0
        d = damp
        for _ in range(6):
            Lc, info = torch.linalg.cholesky_ex(h + d * base * eye)
            Ue, info2 = torch.linalg.cholesky_ex(torch.cholesky_inverse(Lc), upper=True)
            if int(info) == 0 and int(info2) == 0 and bool(torch.isfinite(Ue).all()):
                break
            d *= 3
        else:
            raise RuntimeError("GPTQ: Hessian not positive definite even with heavy damping")
        U[e] = Ue.to(torch.float32)
        dead_all[e] = dead.to(torch.uint8)
    return U, dead_all


def quantize_stack(W: torch.Tensor, levels: int = 8, block: int = 32, energy: torch.Tensor | None = None,
                   iters: int = ITERS, H: torch.Tensor | None = None, damp: float = 0.01) -> dict:
    """HEX-quantize every matrix of W [n, out, in] (CUDA, cast to f32) as the
    reference quantizes one: returns {"idx" uint32 [n, out, in/32*bits],
    "block_scale" uint8 [n, out, in/block], "expert_scale" f32 [n], "levels" f32
    [n, levels]} on W's device.  energy: [in] or [n, in] per-input mean x^2
    weighting the table fit (the reference's `energy`).  H: [in, in] or [n, in,
    in] Hessians (sum x x^T): GPTQ onto the table instead of nearest rounding
    (the reference's `H`, `damp`)."""
    if not W.is_cuda:
        raise ValueError("quantize_stack runs on CUDA only")
    if W.dim() == 2:
        W = W[None]
    if W.dim() != 3:
        raise ValueError(f"W must be [n, out, in], got {tuple(W.shape)}")
    n, out, cols = W.shape
    if levels not in (8, 16):
        raise ValueError("levels must be 8 or 16")
    if block not in (32, 128) or cols % block:
        raise ValueError(f"block must be 32 or 128 and divide in ({cols})")
    dev = W.device
    Wc = W.to(torch.float32).contiguous()
    en = None
    if energy is not None:
        en = torch.as_tensor(energy, dtype=torch.float32, device=dev)
        en = (en.expand(n, cols) if en.dim() == 1 else en).contiguous()
        if en.shape != (n, cols):
            raise ValueError(f"energy must be [in] or [n, in], got {tuple(energy.shape)}")
    sidx = _sample_on(out * cols, dev)
    ns = 0 if sidx is None else sidx.numel()
    bits = 3 if levels == 8 else 4
    idx = torch.empty(n, out, cols // 32 * bits, dtype=torch.int32, device=dev)
    bs = torch.empty(n, out, cols // block, dtype=torch.uint8, device=dev)
    es = torch.empty(n, dtype=torch.float32, device=dev)
    lev = torch.empty(n, levels, dtype=torch.float32, device=dev)
    hinv, dead = gptq_prep(Wc, H, damp) if H is not None else (None, None)
    nbytes = _lib.lib.hexmoe_quantize_workspace_bytes(n, out, cols, block, ns, int(en is not None), int(H is not None))
    if nbytes == 0:
        raise ValueError("hexmoe_quantize_workspace_bytes: shape not supported")
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    with torch.cuda.device(dev):
        rc = _lib.lib.hexmoe_quantize(p(Wc), n, out, cols, levels, block, p(en), p(sidx), ns, iters, p(hinv), p(dead),
                                      p(idx), p(bs), p(es), p(lev), p(ws), nbytes,
                                      ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    _lib.check(rc, "hexmoe_quantize")
    return {"idx": idx.view(torch.uint32), "block_scale": bs, "expert_scale": es, "levels": lev}


def quantize(W: torch.Tensor, levels: int = 8, block: int = 32, energy: torch.Tensor | None = None,
             H: torch.Tensor | None = None, damp: float = 0.01) -> dict:
    """One matrix [out, in]: the reference's quantize(W, L, block, energy, H, damp)
    parts (Hex.packed(): idx, block_scale, expert_scale [1], levels [L])."""
    parts = quantize_stack(W[None] if W.dim() == 2 else W, levels, block, energy, H=H, damp=damp)
    return {"idx": parts["idx"][0], "block_scale": parts["block_scale"][0], "expert_scale": parts["expert_scale"],
            "levels": parts["levels"][0]}
