"""INT8 hybrid grouped MoE forward (drop-in for the reference's
int8_hybrid_moe/cutlass_runner.py:69-236), on the sm_100a kernels.

The op sequence, the variant choice (tile_m 64 when the average rows per
expert is <= 70, else 128), the workspace aliasing and the environment
switches are the reference's.  With the fused permute+quant path on, the
routing kernels also emit the int32 expert offsets, both problem-size tables
and the quant scale offsets (moe_route_for_gemm), which replaces the
reference's handful of small torch ops between routing and the first GEMM
without changing any value.  No step synchronises with the host, so the
whole forward can be captured in a CUDA graph.
"""

from __future__ import annotations

import os

import torch

from .activation import MoEActivation, apply_moe_activation
from .ops import cutlass_int8_blockwise_hybrid_grouped, cutlass_int8_blockwise_hybrid_grouped_small
from .permute import moe_permute, moe_permute_metadata, moe_route_for_gemm, moe_unpermute
from .quant import (
    _resize_cache,
    fused_permute_quant_int8_hybrid_grouped,
    fused_silu_quant_int8_hybrid_grouped,
    fused_w13_silu_quant_int8_hybrid_grouped,
    moe_kernel_quantize_input_int8_hybrid_grouped,
)

_VARIANT_TILE_M = {"hybrid": 128, "hybrid_small": 64}
_VARIANT_TILE_N = {"hybrid": 64, "hybrid_small": 64}
_VARIANT_TILE_K = {"hybrid": 128, "hybrid_small": 128}

_USE_FUSED_SILU_QUANT_W2: bool = (
    os.environ.get("VLLM_INT8_HYBRID_FUSED_SILU_QUANT", "1").strip() == "1")
_USE_FUSED_PERMUTE_QUANT_W1: bool = (
    os.environ.get("VLLM_INT8_HYBRID_FUSED_PERMUTE_QUANT", "0").strip() == "1")
# SiLU*up + requant inside the w13 GEMM epilogue (no reference counterpart;
# applies when the fused SiLU quant is selected and N is a multiple of 32)
_USE_FUSED_W13_EPILOGUE: bool = (
    os.environ.get("INT8_HYBRID_MOE_FUSED_W13_EPILOGUE", "1").strip() == "1")


def pick_grouped_hybrid_variant(sum_M: int, num_experts: int) -> str:
    """Variant by average rows per expert (cutlass_runner.py:43-50)."""
    if num_experts <= 0:
        return "hybrid"
    return "hybrid_small" if sum_M / num_experts <= 70 else "hybrid"


def _dispatch_grouped_hybrid(variant: str):
    return {"hybrid": cutlass_int8_blockwise_hybrid_grouped,
            "hybrid_small": cutlass_int8_blockwise_hybrid_grouped_small}[variant]


def _variant_tile_m(variant: str) -> int:
    return _VARIANT_TILE_M[variant]


def _expert_offsets_i32(expert_first_token_offset: torch.Tensor) -> torch.Tensor:
    return expert_first_token_offset.to(torch.int32)


def _run_cutlass_int8_hybrid_grouped_moe(
    output: torch.Tensor,
    hidden_states: torch.Tensor,
    w1: torch.Tensor,
    w2: torch.Tensor,
    topk_ids: torch.Tensor,
    topk_weights: torch.Tensor,
    activation: MoEActivation,
    global_num_experts: int,
    expert_map: torch.Tensor | None,
    w1_qscale: torch.Tensor,
    w1_fscale: torch.Tensor,
    w2_qscale: torch.Tensor,
    w2_fscale: torch.Tensor,
    workspace13: torch.Tensor,
    workspace2: torch.Tensor,
    quant_block_size: int,
    super_group_size: int,
    q_max: int,
    *,
    _trace: dict | None = None,
    _tile_m: int | None = None,
    _inv_out: torch.Tensor | None = None,
    _unpermute: bool = True,
) -> None:
    """Full INT8 hybrid grouped MoE forward; writes ``output`` [M, K].

    Keyword-only additions to the reference signature:
    ``_trace``: when a dict is given, every intermediate tensor is stored in
    it for verification.
    ``_tile_m``: forces the quant tile height (64 or 128) instead of the
    rows-per-expert rule; expert parallelism passes the single-GPU choice so
    its quant tiles match a single-GPU run.
    ``_inv_out``: int32 buffer of M * topk elements that receives the
    routing's inverse map.
    ``_unpermute=False``: stop after the w2 GEMM; its rows stay in
    ``workspace2`` ([M * topk, K] at offset 0) and ``output`` is not
    written.  The expert-parallel top-k combine performs the unpermute from
    those rows and ``_inv_out`` on the rank that owns each token."""
    assert activation.is_gated, "Only gated activation is supported"
    assert hidden_states.dtype in (torch.float16, torch.bfloat16, torch.float32)
    assert w1.dtype == torch.int8 and w2.dtype == torch.int8
    assert w1_qscale is not None and w1_fscale is not None
    assert w2_qscale is not None and w2_fscale is not None
    assert global_num_experts != -1

    M = hidden_states.size(0)
    topk = topk_ids.size(1)
    local_E = w1.size(0)
    _, K, N = w2.shape
    assert w1.size(2) == K
    assert w1.size(1) == 2 * N

    mm1_out = _resize_cache(workspace13, (M * topk, N * 2))
    act_out = _resize_cache(workspace2, (M * topk, N))
    mm2_out = _resize_cache(workspace2, (M * topk, K))
    sum_M = M * topk
    num_expert = global_num_experts if expert_map is None else expert_map.size(0)

    variant = pick_grouped_hybrid_variant(sum_M, local_E)
    if _tile_m is not None:
        variant = {128: "hybrid", 64: "hybrid_small"}[_tile_m]
    tile_m = _variant_tile_m(variant)
    gemm = _dispatch_grouped_hybrid(variant)

    if _USE_FUSED_PERMUTE_QUANT_W1:
        (expert_first_token_offset, inv_perm, permuted_idx, expert_offsets, problem_sizes1,
         problem_sizes2, scale_offsets) = moe_route_for_gemm(
            topk_ids, M, num_expert, local_E, expert_map, 2 * N, K, K, N, tile_m,
            inv_out=_inv_out)
        a1q, a1_qscale, a1_fscale, a1_scale_offsets = fused_permute_quant_int8_hybrid_grouped(
            hidden_states, permuted_idx, topk=topk, block_k=quant_block_size, q_max=q_max,
            super_group_size=super_group_size, expert_offsets=expert_offsets, tile_m=tile_m,
            scale_offsets=scale_offsets)
    else:
        a1_perm = _resize_cache(workspace2, (M * topk, K))
        a1, _, expert_first_token_offset, inv_perm, _ = moe_permute(
            hidden_states, None, topk_ids, num_expert, local_E, expert_map,
            permuted_hidden_states=a1_perm)
        expert_offsets = _expert_offsets_i32(expert_first_token_offset)
        counts = expert_offsets[1:] - expert_offsets[:-1]
        problem_sizes1 = torch.empty((local_E, 3), dtype=torch.int32, device=hidden_states.device)
        problem_sizes2 = torch.empty((local_E, 3), dtype=torch.int32, device=hidden_states.device)
        problem_sizes1[:, 0] = counts
        problem_sizes1[:, 1] = 2 * N
        problem_sizes1[:, 2] = K
        problem_sizes2[:, 0] = counts
        problem_sizes2[:, 1] = K
        problem_sizes2[:, 2] = N
        scale_offsets = None
        a1q, a1_qscale, a1_fscale, a1_scale_offsets = (
            moe_kernel_quantize_input_int8_hybrid_grouped(
                a1, block_k=quant_block_size, q_max=q_max, super_group_size=super_group_size,
                expert_offsets=expert_offsets, tile_m=tile_m))

    fuse_w13 = (_USE_FUSED_W13_EPILOGUE and _USE_FUSED_SILU_QUANT_W2
                and activation == MoEActivation.SILU and N % 32 == 0
                and mm1_out.dtype in (torch.bfloat16, torch.float16))
    if fuse_w13:
        # ---- w13 GEMM with SiLU * up + requant in its epilogue ----
        a2q, a2_qscale, a2_fscale, a2_scale_offsets = fused_w13_silu_quant_int8_hybrid_grouped(
            a1q, a1_qscale, a1_fscale, w1, w1_qscale, w1_fscale, expert_offsets,
            problem_sizes1, scale_offsets if scale_offsets is not None else a1_scale_offsets,
            quant_block_size, q_max, super_group_size, tile_m, mm1_out.dtype)
    else:
        # ---- w13 GEMM ----
        gemm(a1q, a1_qscale, a1_fscale, w1, w1_qscale, w1_fscale, expert_offsets,
             problem_sizes1, mm1_out, quant_block_size, super_group_size,
             scale_offsets=a1_scale_offsets)

    # ---- SiLU * up + requant ----
    if fuse_w13:
        pass
    elif _USE_FUSED_SILU_QUANT_W2 and activation == MoEActivation.SILU:
        a2q, a2_qscale, a2_fscale, a2_scale_offsets = fused_silu_quant_int8_hybrid_grouped(
            mm1_out, block_k=quant_block_size, q_max=q_max, super_group_size=super_group_size,
            expert_offsets=expert_offsets, tile_m=tile_m, scale_offsets=scale_offsets)
    else:
        apply_moe_activation(activation, act_out, mm1_out)
        a2q, a2_qscale, a2_fscale, a2_scale_offsets = (
            moe_kernel_quantize_input_int8_hybrid_grouped(
                act_out, block_k=quant_block_size, q_max=q_max,
                super_group_size=super_group_size, expert_offsets=expert_offsets,
                tile_m=tile_m, scale_offsets=scale_offsets))

    # ---- w2 GEMM ----
    gemm(a2q, a2_qscale, a2_fscale, w2, w2_qscale, w2_fscale, expert_offsets, problem_sizes2,
         mm2_out, quant_block_size, super_group_size, scale_offsets=a2_scale_offsets)

    if _trace is not None:
        _trace.update(
            eft=expert_first_token_offset, inv=inv_perm, expert_offsets=expert_offsets,
            problem_sizes1=problem_sizes1, problem_sizes2=problem_sizes2, tile_m=tile_m,
            a1q=a1q, a1_Q=a1_qscale, a1_F=a1_fscale, a1_so=a1_scale_offsets,
            mm1=None if fuse_w13 else mm1_out.clone(), a2q=a2q, a2_Q=a2_qscale, a2_F=a2_fscale, a2_so=a2_scale_offsets,
            mm2=mm2_out.clone(), scale_offsets=scale_offsets)
        if _USE_FUSED_PERMUTE_QUANT_W1:
            _trace["pidx"] = permuted_idx

    if _inv_out is not None and _inv_out.data_ptr() != inv_perm.data_ptr():
        _inv_out.view(-1).copy_(inv_perm.view(-1))
    if not _unpermute:
        return
    moe_unpermute(out=output, permuted_hidden_states=mm2_out, topk_weights=topk_weights,
                  inv_permuted_idx=inv_perm, expert_first_token_offset=expert_first_token_offset)
