"""ctypes binding of libhexmoe.so (the C ABI in include/hexmoe.h).

The library is built in-tree (blackhole_b200/libhexmoe.so, `make` in the
package directory or __graft_entry__.build()).  There is no fallback: importing
this module without the library raises ImportError.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libhexmoe.so"

HEXMOE_OK, HEXMOE_E_ARG, HEXMOE_E_DTYPE, HEXMOE_E_CUDA, HEXMOE_E_UNSUPPORTED, HEXMOE_E_DEVICE = range(6)
F32, BF16, F16 = 0, 1, 2
I32, I64 = 0, 1
MAX_TIERS = 4
NOALLOC_SCRATCH_BYTES = 32 << 20   # HEXMOE_NOALLOC_SCRATCH_BYTES in include/hexmoe.h

EXPORTS = (
    "hexmoe_abi_version", "hexmoe_last_error", "hexmoe_device_status", "hexmoe_build_expert_map",
    "hexmoe_layer_create", "hexmoe_layer_destroy", "hexmoe_forward_workspace_bytes", "hexmoe_forward",
    "hexmoe_align_workspace_bytes", "hexmoe_align", "hexmoe_dequant", "hexmoe_route_topk",
    "hexmoe_gather", "hexmoe_gate_up", "hexmoe_down", "hexmoe_combine", "hexmoe_forward_noalloc",
    "hexmoe_tile_index", "hexmoe_combine_rows", "hexmoe_forward_slots",
    "hexmoe_ep_init", "hexmoe_ep_handle", "hexmoe_ep_connect", "hexmoe_ep_workspace_bytes", "hexmoe_ep_dispatch",
    "hexmoe_ep_experts", "hexmoe_ep_combine", "hexmoe_ep_forward", "hexmoe_ep_destroy",
    "hexmoe_quantize_workspace_bytes", "hexmoe_quantize",
)
EP_MAX_WORLD = 8          # HEXMOE_EP_MAX_WORLD
EP_HANDLE_BYTES = 64      # HEXMOE_EP_HANDLE_BYTES


class Parts(ctypes.Structure):
    _fields_ = [("idx", ctypes.c_void_p), ("block_scale", ctypes.c_void_p), ("expert_scale", ctypes.c_void_p),
                ("levels", ctypes.c_void_p)]


class Tier(ctypes.Structure):
    _fields_ = [("bits", ctypes.c_int32), ("n", ctypes.c_int32), ("experts", ctypes.c_void_p),
                ("gate", Parts), ("up", Parts), ("down", Parts)]


class LayerDesc(ctypes.Structure):
    _fields_ = [("num_experts", ctypes.c_int32), ("hidden", ctypes.c_int32), ("inter", ctypes.c_int32),
                ("hidden_pad", ctypes.c_int32), ("inter_pad", ctypes.c_int32), ("block", ctypes.c_int32),
                ("num_tiers", ctypes.c_int32), ("tiers", Tier * MAX_TIERS), ("expert_map", ctypes.c_void_p)]


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(f"blackhole_b200: {LIB_PATH.name} is not built (run `make` in "
                          f"{LIB_PATH.parent.parent} or __graft_entry__.build()); there is no non-CUDA fallback")
    L = ctypes.CDLL(str(LIB_PATH), mode=ctypes.RTLD_LOCAL)
    P, I32_, I64_, SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
    sig = {
        "hexmoe_abi_version": (ctypes.c_int, []),
        "hexmoe_last_error": (ctypes.c_char_p, []),
        "hexmoe_device_status": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, P]),
        "hexmoe_build_expert_map": (ctypes.c_int, [P, P, P]),
        "hexmoe_layer_create": (ctypes.c_int, [P, P]),
        "hexmoe_layer_destroy": (ctypes.c_int, [P]),
        "hexmoe_forward_workspace_bytes": (SZ, [P, I64_, I32_, I32_, I32_]),
        "hexmoe_forward": (ctypes.c_int, [P, P, I32_, I64_, I32_, P, P, I32_, P, I32_, I32_, P, SZ, P]),
        "hexmoe_forward_noalloc": (ctypes.c_int, [P, P, I32_, I64_, I32_, P, P, I32_, P, I32_, I32_, P]),
        "hexmoe_forward_slots": (ctypes.c_int, [P, P, I32_, I64_, I32_, P, P, I32_, P, I32_, P, SZ, P]),
        "hexmoe_align_workspace_bytes": (SZ, [I64_, I32_]),
        "hexmoe_align": (ctypes.c_int, [P, I32_, I64_, I32_, I32_, P, P, P, P, SZ, P]),
        "hexmoe_dequant": (ctypes.c_int, [P, I32_, I32_, I32_, I32_, I32_, I32_, I32_, P, P, I32_, I64_, I64_, I64_,
                                          P]),
        "hexmoe_route_topk": (ctypes.c_int, [P, I32_, I64_, I32_, I32_, I32_, P, P, P]),
        "hexmoe_tile_index": (ctypes.c_int, [P, I32_, I32_, I32_, I32_, P, P]),
        "hexmoe_gather": (ctypes.c_int, [P, I32_, I64_, I32_, I32_, I32_, P, P, I32_, P, P]),
        "hexmoe_gate_up": (ctypes.c_int, [P, P, I32_, I64_, I32_, P, P, P, I32_, P, P]),
        "hexmoe_down": (ctypes.c_int, [P, P, I32_, I64_, I32_, P, P, P, P, I32_, P, P]),
        "hexmoe_combine": (ctypes.c_int, [P, I32_, I64_, I32_, I32_, P, I32_, P]),
        "hexmoe_combine_rows": (ctypes.c_int, [P, I32_, I64_, I64_, I32_, I32_, P, P, I32_, P]),
        "hexmoe_ep_init": (ctypes.c_int, [I32_, I32_, I32_, I32_, I32_, I64_, I32_, P]),
        "hexmoe_ep_handle": (ctypes.c_int, [P, P]),
        "hexmoe_ep_connect": (ctypes.c_int, [P, P]),
        "hexmoe_ep_workspace_bytes": (SZ, [P, P, I32_]),
        "hexmoe_ep_dispatch": (ctypes.c_int, [P, P, I32_, I64_, P, P, I32_, P]),
        "hexmoe_ep_experts": (ctypes.c_int, [P, P, I32_, P, SZ, P]),
        "hexmoe_ep_combine": (ctypes.c_int, [P, I64_, P, I32_, P]),
        "hexmoe_ep_forward": (ctypes.c_int, [P, P, P, I32_, I64_, P, P, I32_, P, I32_, I32_, P, SZ, P]),
        "hexmoe_ep_destroy": (ctypes.c_int, [P]),
        "hexmoe_quantize_workspace_bytes": (SZ, [I32_, I32_, I32_, I32_, I64_, I32_, I32_]),
        "hexmoe_quantize": (ctypes.c_int, [P, I32_, I32_, I32_, I32_, I32_, P, P, I64_, I32_, P, P, P, P, P, P, P, SZ,
                                           P]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    return L


lib = _load()


def last_error() -> str:
    return (lib.hexmoe_last_error() or b"").decode(errors="replace")


def check(rc: int, what: str = "hexmoe") -> None:
    """Raise the reference's exception type for a non-OK status (ValueError for
    argument / dtype errors, as the reference's asserts and plugin checks do;
    RuntimeError for CUDA and device failures)."""
    if rc == HEXMOE_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc in (HEXMOE_E_ARG, HEXMOE_E_DTYPE):
        raise ValueError(msg)
    raise RuntimeError(msg)


def device_status(device: int, clear: bool = True) -> int:
    v = ctypes.c_int32(0)
    check(lib.hexmoe_device_status(int(device), int(clear), ctypes.byref(v)), "hexmoe_device_status")
    return int(v.value)


def env_flag(name: str, default: str = "") -> str:
    return os.environ.get(name, default)
