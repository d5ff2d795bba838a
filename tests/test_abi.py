"""The C ABI without a GPU: libi8moe.so loads, exports every function that
include/i8moe.h declares with the prototype table the bindings use, and the
argument checks that run before any CUDA call return their documented codes."""

import ctypes
import re

import pytest

from tests.conftest import ROOT

HEADER = ROOT / "include" / "i8moe.h"


def header_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)  # drop comments
    return sorted(set(re.findall(r"\b(i8moe_\w+)\s*\(", text)))


def test_header_declares_functions():
    names = header_functions()
    assert "i8moe_hybrid_grouped_gemm" in names and len(names) >= 15


def test_library_exports_every_header_function():
    from int8blockwisegemm_b200 import _lib
    names = header_functions()
    missing_proto = [n for n in names if n not in _lib.PROTOTYPES]
    assert not missing_proto, f"no ctypes prototype for {missing_proto}"
    extra_proto = [n for n in _lib.PROTOTYPES if n not in names]
    assert not extra_proto, f"prototypes for undeclared functions {extra_proto}"
    raw = ctypes.CDLL(_lib.LIB_PATH)
    for n in names:
        assert hasattr(raw, n), f"libi8moe.so does not export {n}"


def test_calls_that_need_no_gpu():
    from int8blockwisegemm_b200 import _lib
    lib = _lib.LIB
    assert lib.i8moe_abi_version() >= 1
    assert lib.i8moe_moe_permute_unpermute_supported() == 1
    # 2048-key chunks x 2^bits buckets x 4 bytes
    assert lib.i8moe_route_workspace_size(65536, 256) == 32 * 512 * 4
    assert lib.i8moe_route_workspace_size(1, 8) == 1 * 16 * 4
    assert lib.i8moe_route_workspace_size(10, 0) == 0
    # GEMM variant switch: returns the previous mode, rejects other values
    prev = lib.i8moe_gemm_set_cta_pairs(1)
    assert prev in (-1, 0, 1)
    assert lib.i8moe_gemm_set_cta_pairs(0) == 1
    assert lib.i8moe_gemm_set_cta_pairs(2) == -1 and "cta pairs" in _lib.last_error()
    assert lib.i8moe_gemm_set_cta_pairs(prev) == 0


def test_argument_errors_before_any_cuda_call():
    from int8blockwisegemm_b200 import _lib
    lib = _lib.LIB
    rc = lib.i8moe_moe_permute_metadata(None, None, None, 4, 2, 0, 0, None, None, None, None, 0,
                                        None)
    assert rc == -1 and "n_expert" in _lib.last_error()
    rc = lib.i8moe_moe_permute_metadata(None, None, None, 4, 2, 8, 8, None, None, None, None, 0,
                                        None)
    assert rc == -1 and "workspace" in _lib.last_error()


def test_noalloc_rejects_problems_above_its_fixed_scratch():
    from int8blockwisegemm_b200 import _lib
    lib = _lib.LIB
    # 2048 experts -> 4096 buckets x 16 KiB per chunk: 128 chunks fill 2 MiB
    rc = lib.i8moe_moe_permute_metadata_noalloc(None, None, None, 32768, 8, 2048, 2048, None,
                                                None, None, None)
    assert rc == -1
    msg = _lib.last_error()
    assert "fixed" in msg and "i8moe_moe_permute_metadata" in msg
    # a row count n_token * topk that does not fit in int32 is rejected before
    # it is formed
    rc = lib.i8moe_moe_permute_metadata_noalloc(None, None, None, 2**40, 8, 8, 8, None, None,
                                                None, None)
    assert rc == -1 and "int32" in _lib.last_error()


def test_peer_exchange_region_layout():
    """The peer-exchange region layout (a host-side computation): every part
    256-byte aligned, disjoint, inside the region, and bad shapes rejected."""
    import ctypes
    from int8blockwisegemm_b200 import _lib
    from int8blockwisegemm_b200.ep import _Layout
    lib = _lib.LIB
    P, T, k, K = 8, 8192, 8, 2048
    C = P * T
    for combine in (0, 1):  # I8MOE_EP_COMBINE_ROWS, I8MOE_EP_COMBINE_TOPK
        lay = _Layout()
        assert lib.i8moe_ep_p2p_region_bytes(P, C, k, K, 2, combine, ctypes.addressof(lay)) == 0
        parts = [(lay.off_rows, C * K * 2), (lay.off_ids, C * k * 4), (lay.off_w, C * k * 4),
                 (lay.off_out, 2 * lay.out_bytes), (lay.off_mm2, 2 * lay.mm2_bytes),
                 (lay.off_inv, 2 * lay.inv_bytes), (lay.off_inbox, 2 * P * P * 4),
                 (lay.off_flags, 3 * P * 8), (lay.off_epoch, 12)]
        if combine == 0:
            assert lay.out_bytes >= C * K * 2 and lay.mm2_bytes == 0 and lay.inv_bytes == 0
        else:
            assert lay.out_bytes == 0 and lay.mm2_bytes >= C * k * K * 2
            assert lay.inv_bytes >= C * k * 4
        end = 0
        for off, size in parts:
            assert off % 256 == 0 and off >= end, (off, end)
            end = off + size
        assert end <= lay.bytes
    lay = _Layout()
    assert lib.i8moe_ep_p2p_region_bytes(33, 33, k, K, 2, 0, ctypes.addressof(lay)) == -1
    assert "ranks" in _lib.last_error()
    assert lib.i8moe_ep_p2p_region_bytes(P, C, k, K, 4, 0, ctypes.addressof(lay)) == -1
    assert lib.i8moe_ep_p2p_region_bytes(P, C, 33, K, 2, 0, ctypes.addressof(lay)) == -1
    assert lib.i8moe_ep_p2p_region_bytes(P, C, k, K, 2, 2, ctypes.addressof(lay)) == -1
    assert "combine" in _lib.last_error()
