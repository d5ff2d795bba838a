"""ctypes binding of libi8moe.so (the C ABI declared in include/i8moe.h).

The library path follows the reference's loader (int8_hybrid_moe/__init__.py:
21-36): ``INT8_HYBRID_MOE_LIB`` when set, else the in-tree build next to this
file.  A missing library raises at import time, as in the reference; there is
no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import c_char_p, c_float, c_int, c_int64, c_size_t, c_uint32, c_void_p
from pathlib import Path

_DEFAULT_LIB_PATH = str(Path(__file__).resolve().parent / "libi8moe.so")
LIB_PATH = os.environ.get("INT8_HYBRID_MOE_LIB", _DEFAULT_LIB_PATH)

P = c_void_p
I64 = c_int64
I32 = c_int

# name -> (restype, argtypes); must match include/i8moe.h exactly.
PROTOTYPES = {
    "i8moe_abi_version": (I32, []),
    "i8moe_ep_plan": (I32, [P, I64, I64, I64, I64, P, P, P, P]),
    "i8moe_ep_pack": (I32, [P, I64, P, P, I64, P, I64, I64, P, P, P, P]),
    "i8moe_ep_combine": (I32, [P, I32, P, I64, I64, P, I64, P, P]),
    "i8moe_ep_p2p_region_bytes": (I32, [I64, I64, I64, I64, I64, I32, P]),
    "i8moe_ep_ipc_alloc": (I32, [I64, P, P]),
    "i8moe_ep_ipc_open": (I32, [P, P]),
    "i8moe_ep_ipc_close": (I32, [P]),
    "i8moe_ep_ipc_free": (I32, [P]),
    "i8moe_ep_p2p_dispatch": (I32, [P, I32, P, P, P, P, P, P]),
    "i8moe_ep_p2p_wait": (I32, [P, I32, P]),
    "i8moe_ep_p2p_ready": (I32, [P, I32, P]),
    "i8moe_ep_p2p_combine": (I32, [P, I32, I32, P, P, P]),
    "i8moe_ep_p2p_combine_topk": (I32, [P, I32, I32, P, P, P, I64, P, P]),
    "i8moe_last_error": (c_char_p, []),
    "i8moe_device_error": (I32, [I32, ctypes.POINTER(c_uint32), I32]),
    "i8moe_moe_permute_unpermute_supported": (I32, []),
    "i8moe_route_workspace_size": (c_size_t, [I64, I64]),
    "i8moe_moe_permute_metadata": (I32, [P, P, P, I64, I64, I64, I64, P, P, P, P, c_size_t, P]),
    "i8moe_moe_permute_metadata_noalloc": (I32, [P, P, P, I64, I64, I64, I64, P, P, P, P]),
    "i8moe_router_topk": (I32, [P, P, I64, I64, I64, P, P, P]),
    "i8moe_router_route_for_gemm": (I32, [P, P, I64, I64, I64, P, P, P, P, I64, P, P, P, P, P, P,
                                          P, I64, I64, I64, I64, I64, P, c_size_t, P]),
    "i8moe_moe_route_for_gemm": (I32, [P, P, P, I64, I64, I64, I64, P, P, P, P, P, P, P, I64, I64,
                                       I64, I64, I64, P, c_size_t, P]),
    "i8moe_moe_permute": (I32, [P, I32, I64, P, P, P, I64, I64, I64, I64, P, P, P, P, P, c_size_t,
                                P]),
    "i8moe_moe_unpermute": (I32, [P, I32, P, P, P, I64, I64, I64, I64, P, P]),
    "i8moe_silu_and_mul": (I32, [P, P, I32, I64, I64, P]),
    "i8moe_scale_offsets": (I32, [P, I64, I64, P, P]),
    "i8moe_quant_grouped": (I32, [P, I32, I64, I64, P, I64, I64, I64, I64, I64, P, P, P, P, I32,
                                  P]),
    "i8moe_quant_permute": (I32, [P, I32, I64, I64, P, I64, I64, P, I64, I64, I64, I64, I64, P, P,
                                  P, P, I32, P]),
    "i8moe_quant_silu": (I32, [P, I32, I64, I64, P, I64, I64, I64, I64, I64, P, P, P, P, I32, P]),
    "i8moe_quantize_weights": (I32, [P, I32, I64, I64, I64, I64, I64, P, P, P]),
    "i8moe_quantize_scales": (I32, [P, I64, I64, I64, I64, P, P, P]),
    "i8moe_hybrid_grouped_gemm": (I32, [P, P, P, I64, P, P, P, P, P, P, P, I64, P, I32, I64, I64,
                                        I64, I64, I64, I64, I64, P]),
    "i8moe_hybrid_grouped_gemm_silu_quant": (I32, [P, P, P, I64, P, P, P, P, P, P, P, I64, I32,
                                                   I64, I64, I64, I64, I64, I64, I64, I64, P, P,
                                                   P, P]),
    "i8moe_int8_grouped_mm": (I32, [P, P, P, I32, c_float, P, P, P, P, I64, I64, I64, I64, P]),
    "i8moe_gemm_set_cta_pairs": (I32, [I32]),
    "i8moe_int8_mma_peak": (I32, [I64, I32, P, P]),
}

BF16, FP16, FP32, S32 = 0, 1, 2, 3


def _load():
    if not os.path.isfile(LIB_PATH):
        raise RuntimeError(
            f"Cannot find libi8moe.so at {LIB_PATH}.\n"
            "Build it first:  python int8blockwisegemm_b200/_build.py\n"
            "or set INT8_HYBRID_MOE_LIB to the path of the compiled .so.")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


LIB = _load()


def last_error() -> str:
    msg = LIB.i8moe_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str = "") -> None:
    """Raise RuntimeError (the reference's TORCH_CHECK behaviour) on failure."""
    if rc != 0:
        raise RuntimeError(f"{what}: {last_error()}" if what else last_error())


def call(name: str, *args) -> None:
    check(getattr(LIB, name)(*args), name)


def set_cta_pairs(mode: int) -> int:
    """Grouped-GEMM variant: 1 CTA pairs (cta_group::2), 0 one CTA per tile,
    -1 by problem shape (default).  Returns the previous mode."""
    prev = _load().i8moe_gemm_set_cta_pairs(int(mode))
    if prev < -1:
        check(prev, "i8moe_gemm_set_cta_pairs")
    return prev


def device_error(device: int, clear: bool = False) -> int:
    w = c_uint32(0)
    check(LIB.i8moe_device_error(device, ctypes.byref(w), 1 if clear else 0), "device_error")
    return int(w.value)
