"""hexmoe_forward_noalloc (the forward for callers that cannot allocate device
memory, scratch in a fixed array inside the library) against hexmoe_forward
with a caller workspace, both through the C ABI.

The file name sorts last so pytest collects it after the other GPU tests: the
scratch array is shared and keeps the previous call's contents, and the test
must hold both in a fresh process and after everything else has run.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from helpers import rel_err, within

from blackhole_b200 import _lib
from blackhole_b200 import hex_data as hd

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
E, H, I, K = 16, 512, 256, 4


def _layer():
    from blackhole_b200.hex_moe import HexTier, layer_for
    L = hd.synth_layer(E, H, I, "mixed", 32, seed=11, device=DEV)
    tiers = [HexTier(t["bits"], t["experts"], t["gate_proj"], t["up_proj"], t["down_proj"]).prepare(E)
             for t in L.tiers]
    return layer_for(tiers)


def _inputs(T: int, seed: int):
    w, ids = hd.synth_routing(T, E, K, seed=seed)
    x = hd.synth_x(T, H, seed=seed + 1, device=DEV).to(torch.bfloat16).contiguous()
    return x, w.to(DEV).float().contiguous(), ids.to(DEV).to(torch.int32).contiguous()


def _with_workspace(layer, x, w, ids) -> torch.Tensor:
    T = x.shape[0]
    out = torch.empty(T, H, dtype=torch.float32, device=DEV)
    nbytes = _lib.lib.hexmoe_forward_workspace_bytes(layer.handle, T, K, 0, _lib.BF16)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.lib.hexmoe_forward(layer.handle, x.data_ptr(), _lib.BF16, T, K, w.data_ptr(), ids.data_ptr(),
                                       _lib.I32, out.data_ptr(), _lib.F32, 0, ws.data_ptr(), nbytes, stream),
               "hexmoe_forward")
    torch.cuda.synchronize()
    return out


def _no_alloc(layer, x, w, ids, out: torch.Tensor) -> None:
    T = x.shape[0]
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.lib.hexmoe_forward_noalloc(layer.handle, x.data_ptr(), _lib.BF16, T, K, w.data_ptr(),
                                               ids.data_ptr(), _lib.I32, out.data_ptr(), _lib.F32, 0, stream),
               "hexmoe_forward_noalloc")
    torch.cuda.synchronize()


def test_noalloc_matches_workspace_forward_two_calls():
    """Two calls in a row, each bit-equal to hexmoe_forward with a workspace on
    the same inputs.  A first call at a larger batch with NaN / Inf activations
    leaves poisoned rows all over the shared array; the second, smaller call must
    not see any of them (padding rows of its plan hold whatever the first call
    left, and must never reach `out`)."""
    from blackhole_b200.hex_moe import device_status
    device_status(0, clear=True)
    layer = _layer()
    poison = _inputs(96, 3)[0]
    poison[::3] = float("nan")
    poison[1::3] = float("inf")
    x0, w0, ids0 = poison, *_inputs(96, 3)[1:]
    out0 = torch.empty(96, H, dtype=torch.float32, device=DEV)
    _no_alloc(layer, x0, w0, ids0, out0)
    for T, seed in ((48, 5), (20, 9)):
        x, w, ids = _inputs(T, seed)
        want = _with_workspace(layer, x, w, ids).cpu().numpy()
        out = torch.full((T, H), float("nan"), dtype=torch.float32, device=DEV)
        _no_alloc(layer, x, w, ids, out)
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), rel_err(got, want)
        assert within(got, want)
    assert device_status(0, clear=True) == 0


def test_noalloc_rejects_batches_beyond_its_scratch():
    """The largest batch whose scratch fits runs; one token more is rejected
    with HEXMOE_E_ARG before anything is launched."""
    layer = _layer()
    limit = _lib.NOALLOC_SCRATCH_BYTES
    need = lambda t: _lib.lib.hexmoe_forward_workspace_bytes(layer.handle, t, K, 0, _lib.BF16)   # noqa: E731
    lo, hi = 1, 2
    while need(hi) <= limit:
        lo, hi = hi, hi * 2
    while hi - lo > 1:                      # largest T with need(T) <= limit
        mid = (lo + hi) // 2
        lo, hi = (mid, hi) if need(mid) <= limit else (lo, mid)
    x, w, ids = _inputs(lo, 13)
    out = torch.empty(lo, H, dtype=torch.float32, device=DEV)
    _no_alloc(layer, x, w, ids, out)
    want = _with_workspace(layer, x, w, ids)
    assert torch.equal(out, want)
    T = hi
    x = torch.zeros(T, H, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(T, K, dtype=torch.float32, device=DEV)
    ids = torch.zeros(T, K, dtype=torch.int32, device=DEV)
    out = torch.empty(T, H, dtype=torch.float32, device=DEV)
    with pytest.raises(ValueError, match="scratch bytes"):
        _no_alloc(layer, x, w, ids, out)
