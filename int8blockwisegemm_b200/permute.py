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
                       n_out1: int, k1: int, n_out2: int, k2: int, tile_m: int):
    """Extension: routing metadata plus the int32 expert offsets, both GEMMs'
    problem sizes and the quant scale offsets, from one set of kernels.

    Returns (expert_first_token_offset, inv_permuted_idx (flat), permuted_idx,
             expert_offsets_i32 [E+1], problem_sizes13, problem_sizes2,
             scale_offsets_i32 [E+1])."""
    topk = topk_ids.size(1)
    dev = topk_ids.device
    tei, eft, pidx, inv = _alloc(n_token, topk, n_local_expert, dev)
    eo = torch.empty(n_local_expert + 1, dtype=torch.int32, device=dev)
    ps1 = torch.empty((n_local_expert, 3), dtype=torch.int32, device=dev)
    ps2 = torch.empty((n_local_expert, 3), dtype=torch.int32, device=dev)
    so = torch.empty(n_local_expert + 1, dtype=torch.int32, device=dev)
    torch.ops.int8_hybrid_moe.moe_route_for_gemm(
        topk_ids.to(torch.int32), tei, expert_map, n_expert, n_local_expert, topk, eft, inv,
        pidx, eo, ps1, ps2, so, n_out1, k1, n_out2, k2, tile_m)
    return eft, inv.flatten(), pidx, eo, ps1, ps2, so


def moe_unpermute(out, permuted_hidden_states, topk_weights, inv_permuted_idx,
                  expert_first_token_offset=None) -> None:
    """Top-k weighted reduction back to token order."""
    topk = topk_weights.size(1)
    ops.moe_unpermute(permuted_hidden_states, topk_weights, inv_permuted_idx,
                      expert_first_token_offset, topk, out)
