"""CPU restatement of the reference HEX quantizer (test infrastructure only).

Follows blackhole/anatomy/hex.py: block_scales (60-70), fit_table (73-90),
nearest (93-95), quantize (207-227), GPTQ onto the table (_prep 234-253,
gptq_table 256-282) and pack_bits (136-150), with the fp8 e4m3 encode of
blackhole/anatomy/st.py:67-86 (nearest finite code, ties to the smaller value).  Written out arithmetic step by
arithmetic step in the precision the reference computes in (float32 arrays,
Python floats where it uses them, float64 sums in the table fit), so that the
CUDA quantizer (hexmoe_quantize) can be checked against it bit for bit; tests
pin this restatement to tests/golden/quant.npz, written by the reference itself.
Only tests/ import this module.
"""

from __future__ import annotations

import numpy as np

FP8_MAX = 448.0
SAMPLE = 1 << 17


def _fp8_table() -> np.ndarray:
    out = np.zeros(256, np.float32)
    for b in range(256):
        s = -1.0 if b >> 7 else 1.0
        e, m = (b >> 3) & 15, b & 7
        if e == 15 and m == 7:
            out[b] = np.nan
        elif e == 0:
            out[b] = s * m / 8 * 2.0 ** -6
        else:
            out[b] = s * (1 + m / 8) * 2.0 ** (e - 7)
    return out


FP8 = _fp8_table()


def fp8_encode(x: np.ndarray) -> np.ndarray:
    """Nearest finite e4m3 code, ties to the smaller value (st.encode)."""
    finite = np.where(np.isfinite(FP8))[0]
    order = finite[np.argsort(FP8[finite], kind="stable")]
    vals = FP8[order]
    xc = np.clip(np.asarray(x, np.float32), -vals[-1], vals[-1])
    i = np.clip(np.searchsorted(vals, xc), 1, len(vals) - 1)
    pick = np.where(np.abs(vals[i - 1] - xc) <= np.abs(vals[i] - xc), i - 1, i)
    return order[pick].astype(np.uint8)


def sample_index(size: int, seed: int = 0, sample: int = SAMPLE) -> np.ndarray | None:
    """The values fit_table draws (with replacement) from a matrix of `size` values."""
    if size <= sample:
        return None
    return np.random.default_rng(seed).integers(0, size, sample)


def quantile_init(x: np.ndarray, L: int) -> np.ndarray:
    """np.quantile(x, linspace(0, 1, L + 2)[1:-1]) (method 'linear'), as float32."""
    return np.quantile(x, np.linspace(0, 1, L + 2)[1:-1]).astype(np.float32)


def gptq_prep(W: np.ndarray, H: np.ndarray, damp: float = 0.01):
    """(W with dead inputs zeroed, the upper Cholesky factor of the damped inverse
    Hessian as float32, the dead-input mask): hex.py:234-253."""
    W = np.asarray(W, np.float32).copy()
    H = np.asarray(H, np.float64).copy()
    n = W.shape[1]
    if not np.any(np.diag(H)):
        H = np.eye(n)
    dead = (np.diag(H) == 0) | (np.abs(W).max(0) == 0)
    live = (~dead).astype(np.float64)
    H = H * live[:, None] * live[None, :] + np.diag(dead.astype(np.float64))
    W[:, dead] = 0
    base = float((np.diag(H) * live).sum() / max(live.sum(), 1)) or 1.0
    d = damp
    for _ in range(6):
        try:
            Lc = np.linalg.cholesky(H + d * base * np.eye(n))
            Hinv = np.linalg.inv(Lc.T) @ np.linalg.inv(Lc)
            U = np.linalg.cholesky(Hinv).T
            if np.isfinite(U).all():
                return W, U.astype(np.float32), dead
        except np.linalg.LinAlgError:
            pass
        d *= 3
    raise RuntimeError("GPTQ: Hessian not positive definite even with heavy damping")


def gptq_table(W: np.ndarray, H: np.ndarray, scales: np.ndarray, levels: np.ndarray, damp: float = 0.01,
               cols: int = 128) -> np.ndarray:
    """Columns rounded onto levels * scales in order, each rounding error spread
    over the columns still to come through the inverse Hessian's factor, in
    blocks of `cols` columns with the later columns updated once per block
    (hex.py:256-282).  Returns the dequantized matrix Q."""
    W, U, dead = gptq_prep(W, H, damp)
    n = W.shape[1]
    Q = np.zeros_like(W)
    mids = (levels[1:] + levels[:-1]) / 2
    for b0 in range(0, n, cols):
        b1 = min(b0 + cols, n)
        Wb = W[:, b0:b1].copy()
        Eb = np.zeros_like(Wb)
        Ub = U[b0:b1, b0:b1]
        for j in range(b1 - b0):
            s = scales[:, b0 + j]
            q = levels[np.searchsorted(mids, np.clip(Wb[:, j] / s, -1, 1))] * s
            Q[:, b0 + j] = q
            e = (Wb[:, j] - q) / Ub[j, j]
            Wb[:, j:] -= e[:, None] * Ub[j, j:][None, :]
            Eb[:, j] = e
        W[:, b1:] -= Eb @ U[b0:b1, b1:]
    Q[:, dead] = 0
    return Q


def gptq_error(W: np.ndarray, Q: np.ndarray, H: np.ndarray) -> float:
    """GPTQ's objective: trace((W - Q) H (W - Q)^T), in float64."""
    D = np.asarray(W, np.float64) - np.asarray(Q, np.float64)
    return float(np.einsum("ij,jk,ik->", D, np.asarray(H, np.float64), D))


def quantize(W: np.ndarray, L: int, block: int, energy: np.ndarray | None = None, iters: int = 20,
             H: np.ndarray | None = None, damp: float = 0.01):
    """(levels f32 [L], expert_scale f32, block-scale codes u8 [out, nblk], codes u8 [out, n]);
    with H [in, in] the codes come from GPTQ onto the table."""
    W = np.asarray(W, np.float32)
    out, n = W.shape
    pad = -n % block
    x = np.pad(W, ((0, 0), (0, pad))).reshape(out, -1, block)
    amax = np.abs(x).max(-1)
    es = max(float(amax.max()) / FP8_MAX, 1e-30)
    blk = FP8[fp8_encode(np.minimum(amax / es, FP8_MAX))] * es
    blk = np.where(blk > 0, blk, 1.0).astype(np.float32)
    xn = np.clip(x / blk[..., None], -1, 1).reshape(out, -1)[:, :n]
    codes = fp8_encode(np.minimum(blk / es, FP8_MAX))
    scales = np.repeat(blk, block, axis=1)[:, :n]
    w = None if energy is None else np.asarray(energy, np.float32)[None, :] * scales ** 2
    # fit_table
    xs = xn.ravel().astype(np.float32)
    ws = None if w is None else w.ravel().astype(np.float32)
    si = sample_index(xs.size)
    if si is not None:
        xs = xs[si]
        ws = ws[si] if ws is not None else None
    if ws is None:
        ws = np.ones_like(xs)
    lev = quantile_init(xs, L)
    for _ in range(iters):
        a = np.searchsorted((lev[1:] + lev[:-1]) / 2, xs)
        num = np.bincount(a, weights=xs * ws, minlength=L)
        den = np.bincount(a, weights=ws, minlength=L)
        lev = np.sort(np.where(den > 0, num / np.maximum(den, 1e-30), lev)).astype(np.float32)
    if H is None:
        idx = np.searchsorted((lev[1:] + lev[:-1]) / 2, np.clip(xn, -1, 1)).astype(np.uint8)
    else:
        Q = gptq_table(W, H, scales, lev, damp)
        idx = np.searchsorted((lev[1:] + lev[:-1]) / 2, np.clip(Q / scales, -1, 1)).astype(np.uint8)
    return lev, np.float32(es), codes, idx


def pack_bits(idx: np.ndarray, bits: int) -> np.ndarray:
    """[out, n] codes -> uint32 [out, n/32*bits]: per 32 inputs one little-endian bit stream."""
    out, n = idx.shape
    x = idx.astype(np.uint64).reshape(out, -1, 32)
    words = np.zeros((out, x.shape[1], bits), np.uint64)
    for i in range(32):
        off = i * bits
        wi, sh = off // 32, off % 32
        words[:, :, wi] |= (x[:, :, i] << sh) & 0xFFFFFFFF
        if sh + bits > 32:
            words[:, :, wi + 1] |= x[:, :, i] >> (32 - sh)
    return words.reshape(out, -1).astype(np.uint32)
