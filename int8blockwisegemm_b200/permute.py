"""MoE permute / unpermute wrappers with the reference's signatures and
allocations (int8_hybrid_moe/permute.py:9-134): permuted_idx is pre-filled
with the sentinel n_token*topk, token_expert_indices is arange."""

from __future__ import annotations

import torch

from . import ops


def _alloc(n_token: int, topk: int, n_local_expert: int, device):
    rows = n_token * topk
    tei = torch.arange(rows, dtype=torch.int32, device=device).reshape(n_token, topk)
    eft = torch.empty(n_local_expert + 1, dtype=torch.int64, device=device)
    pidx = torch.full((rows,), rows, dtype=torch.int32, device=device)
    inv = torch.empty((n_token, topk), dtype=torch.int32, device=device)
    return tei, eft, pidx, inv


def moe_permute(hidden_states, a1q_scale, topk_ids, n_expert: int, n_local_expert: int = -1,
                expert_map=None, permuted_hidden_states=None):
    """Expand and permute activation rows into expert-contiguous order."""
    n_token, n_hidden = hidden_states.size()
    topk = topk_ids.size(1)
    if n_local_expert == -1:
        n_local_expert = n_expert
    if permuted_hidden_states is None:
        permuted_hidden_states = torch.empty((n_token * topk, n_hidden),
                                             dtype=hidden_states.dtype,
                                             device=hidden_states.device)
    tei, eft, pidx, inv = _alloc(n_token, topk, n_local_expert, hidden_states.device)
    ops.moe_permute(hidden_states, topk_ids.to(torch.int32), tei, expert_map, n_expert,
                    n_local_expert, topk, permuted_hidden_states, eft, inv, pidx)
    if a1q_scale is not None and a1q_scale.dim() > 1:
        a1q_scale = a1q_scale[pidx.clamp(max=n_token * topk - 1) // topk]
    return permuted_hidden_states, a1q_scale, eft, inv.flatten(), pidx


def moe_permute_metadata(hidden_states, topk_ids, n_expert: int, n_local_expert: int = -1,
                         expert_map=None):
    """Routing metadata only (no row copy)."""
    n_token = hidden_states.size(0)
    topk = topk_ids.size(1)
    if n_local_expert == -1:
        n_local_expert = n_expert
    tei, eft, pidx, inv = _alloc(n_token, topk, n_local_expert, hidden_states.device)
    ops.moe_permute_metadata(topk_ids.to(torch.int32), tei, expert_map, n_expert,
                             n_local_expert, topk, eft, inv, pidx)
    return eft, inv.flatten(), pidx


def moe_route_for_gemm(topk_ids, n_token: int, n_expert: int, n_local_expert: int, expert_map,
                       n_out1: int, k1: int, n_out2: int, k2: int, tile_m: int, inv_out=None):
    """Extension: routing metadata plus the int32 expert offsets, both GEMMs'
    problem sizes and the quant scale offsets, from one set of kernels.
    ``inv_out`` (int32, n_token * topk elements, contiguous) receives the
    inverse map instead of a new tensor.

    Returns (expert_first_token_offset, inv_permuted_idx (flat), permuted_idx,
             expert_offsets_i32 [E+1], problem_sizes13, problem_sizes2,
             scale_offsets_i32 [E+1])."""
    topk = topk_ids.size(1)
    dev = topk_ids.device
    # the routing kernels write every permuted_idx slot (sentinel included)
    # and take token_expert_indices as arange when it is omitted: no
    # pre-fill launches on this path
    rows = n_token * topk
    eft = torch.empty(n_local_expert + 1, dtype=torch.int64, device=dev)
    pidx = torch.empty(rows, dtype=torch.int32, device=dev)
    if inv_out is None:
        inv = torch.empty((n_token, topk), dtype=torch.int32, device=dev)
    else:
        assert (inv_out.dtype == torch.int32 and inv_out.is_contiguous()
                and inv_out.numel() == rows and inv_out.device == dev)
        inv = inv_out.view(n_token, topk)
    eo = torch.empty(n_local_expert + 1, dtype=torch.int32, device=dev)
    ps1 = torch.empty((n_local_expert, 3), dtype=torch.int32, device=dev)
    ps2 = torch.empty((n_local_expert, 3), dtype=torch.int32, device=dev)
    so = torch.empty(n_local_expert + 1, dtype=torch.int32, device=dev)
    torch.ops.int8_hybrid_moe.moe_route_for_gemm(
        topk_ids.to(torch.int32), None, expert_map, n_expert, n_local_expert, topk, eft, inv,
        pidx, eo, ps1, ps2, so, n_out1, k1, n_out2, k2, tile_m)
    return eft, inv.flatten(), pidx, eo, ps1, ps2, so


def router_topk(logits, topk: int, bias=None):
    """Extension (the router upstream of the runner): top-k experts of each
    token by logits + bias, weights = softmax of their unbiased logits.
    Returns (topk_weights fp32 [T, k], topk_ids int32 [T, k])."""
    from ._lib import call
    assert logits.dtype == torch.float32 and logits.is_contiguous() and logits.is_cuda
    T, E = logits.shape
    ids = torch.empty(T, topk, dtype=torch.int32, device=logits.device)
    w = torch.empty(T, topk, dtype=torch.float32, device=logits.device)
    if bias is not None:
        assert bias.dtype == torch.float32 and bias.numel() == E and bias.is_contiguous()
    with torch.cuda.device(logits.device):
        call("i8moe_router_topk", logits.data_ptr(),
             bias.data_ptr() if bias is not None else None, T, E, topk, ids.data_ptr(),
             w.data_ptr(), torch.cuda.current_stream(logits.device).cuda_stream)
    return w, ids


def router_route_for_gemm(logits, topk: int, n_local_expert: int, expert_map, n_out1: int,
                          k1: int, n_out2: int, k2: int, tile_m: int, bias=None):
    """Extension: ``router_topk`` and ``moe_route_for_gemm`` in one pass (the
    router kernel also builds the routing histogram).  Returns
    (topk_weights, topk_ids, expert_first_token_offset, inv_permuted_idx
    (flat), permuted_idx, expert_offsets_i32, problem_sizes13,
    problem_sizes2, scale_offsets_i32)."""
    from ._lib import call
    assert logits.dtype == torch.float32 and logits.is_contiguous() and logits.is_cuda
    T, E = logits.shape
    dev = logits.device
    ids = torch.empty(T, topk, dtype=torch.int32, device=dev)
    w = torch.empty(T, topk, dtype=torch.float32, device=dev)
    eft = torch.empty(n_local_expert + 1, dtype=torch.int64, device=dev)
    pidx = torch.empty(T * topk, dtype=torch.int32, device=dev)
    inv = torch.empty((T, topk), dtype=torch.int32, device=dev)
    eo = torch.empty(n_local_expert + 1, dtype=torch.int32, device=dev)
    ps1 = torch.empty((n_local_expert, 3), dtype=torch.int32, device=dev)
    ps2 = torch.empty((n_local_expert, 3), dtype=torch.int32, device=dev)
    so = torch.empty(n_local_expert + 1, dtype=torch.int32, device=dev)
    from ._lib import LIB
    ws = torch.empty(max(1, LIB.i8moe_route_workspace_size(T * topk, E)), dtype=torch.uint8,
                     device=dev)
    emap = expert_map.to(torch.int32).contiguous() if expert_map is not None else None
    with torch.cuda.device(dev):
        call("i8moe_router_route_for_gemm", logits.data_ptr(),
             bias.data_ptr() if bias is not None else None, T, E, topk, ids.data_ptr(),
             w.data_ptr(), None, emap.data_ptr() if emap is not None else None,
             n_local_expert, eft.data_ptr(), inv.data_ptr(), pidx.data_ptr(), eo.data_ptr(),
             ps1.data_ptr(), ps2.data_ptr(), so.data_ptr(), n_out1, k1, n_out2, k2, tile_m,
             ws.data_ptr(), ws.numel(), torch.cuda.current_stream(dev).cuda_stream)
    return w, ids, eft, inv.flatten(), pidx, eo, ps1, ps2, so


def moe_unpermute(out, permuted_hidden_states, topk_weights, inv_permuted_idx,
                  expert_first_token_offset=None) -> None:
    """Top-k weighted reduction back to token order."""
    topk = topk_weights.size(1)
    ops.moe_unpermute(permuted_hidden_states, topk_weights, inv_permuted_idx,
                      expert_first_token_offset, topk, out)
