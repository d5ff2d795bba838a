"""GPU test of i8moe_moe_permute_metadata_noalloc, the routing entry point
that takes no workspace (its histogram scratch is a fixed device array in the
library).  It is called twice in a row on different inputs, through the C
ABI, and each result is compared bit for bit with i8moe_moe_permute_metadata
given a caller workspace.  This file is named to be collected last, and it
needs nothing from the other tests, so it passes alone in a fresh process as
well as after them."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(seed, T, k, E, n_local, lo):
    g = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    emap = None
    if n_local < E:
        emap = torch.full((E,), -1, dtype=torch.int32)
        emap[lo:lo + n_local] = torch.arange(n_local, dtype=torch.int32)
    return ids, emap


def _outputs(dev, T, k, n_local):
    R = T * k
    eft = torch.zeros(n_local + 1, dtype=torch.int64, device=dev)
    inv = torch.full((R,), -7, dtype=torch.int32, device=dev)
    pidx = torch.full((R,), R, dtype=torch.int32, device=dev)  # sentinel, as permute.py fills
    return eft, inv, pidx


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def test_noalloc_routing_matches_workspace_entry_point_twice_in_a_row():
    from int8blockwisegemm_b200 import _lib
    lib = _lib.LIB
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream()
    sp = ctypes.c_void_p(stream.cuda_stream)
    cases = [dict(seed=11, T=8192, k=8, E=256, n_local=256, lo=0),
             dict(seed=12, T=1000, k=6, E=64, n_local=32, lo=16)]
    got, want = [], []
    for c in cases:
        ids, emap = _case(c["seed"], c["T"], c["k"], c["E"], c["n_local"], c["lo"])
        ids, emap = ids.to(dev), (emap.to(dev) if emap is not None else None)
        tei = torch.arange(c["T"] * c["k"], dtype=torch.int32, device=dev)
        want_out = _outputs(dev, c["T"], c["k"], c["n_local"])
        ws_bytes = lib.i8moe_route_workspace_size(c["T"] * c["k"], c["E"])
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        _lib.check(lib.i8moe_moe_permute_metadata(
            _ptr(ids), _ptr(tei), _ptr(emap), c["T"], c["k"], c["E"], c["n_local"],
            *map(_ptr, want_out), _ptr(ws), ws_bytes, sp), "moe_permute_metadata")
        want.append(want_out)
        got.append((ids, tei, emap, _outputs(dev, c["T"], c["k"], c["n_local"])))
    # the two allocation-free calls back to back on the stream, reusing the scratch
    for c, (ids, tei, emap, out) in zip(cases, got):
        _lib.check(lib.i8moe_moe_permute_metadata_noalloc(
            _ptr(ids), _ptr(tei), _ptr(emap), c["T"], c["k"], c["E"], c["n_local"],
            *map(_ptr, out), sp), "moe_permute_metadata_noalloc")
    torch.cuda.synchronize()
    for (ids, tei, emap, out), ref in zip(got, want):
        for a, b in zip(out, ref):
            assert torch.equal(a.cpu(), b.cpu())
    assert _lib.device_error(0) == 0
