"""Python entry points of the compiled ops (names and signatures of the
reference's int8_hybrid_moe/ops.py:14-141), dispatching through
``torch.ops.int8_hybrid_moe``."""

from __future__ import annotations

import torch

_OPS = torch.ops.int8_hybrid_moe


def cutlass_int8_blockwise_hybrid_grouped(A, Q_A, F_A, B, Q_B, F_B, expert_offsets,
                                          problem_sizes, out, quant_block_size: int,
                                          super_group_size: int, scale_offsets=None) -> None:
    """Grouped hybrid INT8 GEMM, A-scale rows per 128 rows of an expert."""
    _OPS.cutlass_int8_blockwise_hybrid_grouped(A, Q_A, F_A, B, Q_B, F_B, expert_offsets,
                                               problem_sizes, out, quant_block_size,
                                               super_group_size, scale_offsets)


def cutlass_int8_blockwise_hybrid_grouped_small(A, Q_A, F_A, B, Q_B, F_B, expert_offsets,
                                                problem_sizes, out, quant_block_size: int,
                                                super_group_size: int,
                                                scale_offsets=None) -> None:
    """Grouped hybrid INT8 GEMM, A-scale rows per 64 rows of an expert."""
    _OPS.cutlass_int8_blockwise_hybrid_grouped_small(A, Q_A, F_A, B, Q_B, F_B, expert_offsets,
                                                     problem_sizes, out, quant_block_size,
                                                     super_group_size, scale_offsets)


def cutlass_int8_blockwise_hybrid_grouped_bias(A, Q_A, F_A, B, Q_B, F_B, expert_offsets,
                                               problem_sizes, out, bias, quant_block_size: int,
                                               super_group_size: int,
                                               scale_offsets=None) -> None:
    _OPS.cutlass_int8_blockwise_hybrid_grouped_bias(A, Q_A, F_A, B, Q_B, F_B, expert_offsets,
                                                    problem_sizes, out, bias, quant_block_size,
                                                    super_group_size, scale_offsets)


def cutlass_int8_blockwise_hybrid_grouped_small_bias(A, Q_A, F_A, B, Q_B, F_B, expert_offsets,
                                                     problem_sizes, out, bias,
                                                     quant_block_size: int,
                                                     super_group_size: int,
                                                     scale_offsets=None) -> None:
    _OPS.cutlass_int8_blockwise_hybrid_grouped_small_bias(A, Q_A, F_A, B, Q_B, F_B,
                                                          expert_offsets, problem_sizes, out,
                                                          bias, quant_block_size,
                                                          super_group_size, scale_offsets)


def cutlass_int8_grouped_mm(a, b, out, a_scale: float, b_scale: float, expert_offsets,
                            problem_sizes) -> None:
    """Per-tensor-scaled grouped INT8 GEMM (out = bf16(a_scale*b_scale*acc))."""
    _OPS.cutlass_int8_grouped_mm(a, b, out, a_scale, b_scale, expert_offsets, problem_sizes)


def int8_grouped_mm_scaled(a, b, out, a_row_scale, b_expert_scale, expert_offsets,
                           problem_sizes) -> None:
    """Extension: per-token activation scale x per-expert weight scale."""
    _OPS.int8_grouped_mm_scaled(a, b, out, a_row_scale, b_expert_scale, expert_offsets,
                                problem_sizes)


def silu_and_mul(output: torch.Tensor, input: torch.Tensor) -> None:
    """output = silu(input[..., :d]) * input[..., d:]."""
    _OPS.silu_and_mul(output, input)


def moe_permute(hidden_states, topk_ids, token_expert_indices, expert_map, n_expert: int,
                n_local_expert: int, topk: int, permuted_hidden_states,
                expert_first_token_offset, inv_permuted_idx, permuted_idx) -> None:
    _OPS.moe_permute(hidden_states, topk_ids, token_expert_indices, expert_map, n_expert,
                     n_local_expert, topk, permuted_hidden_states, expert_first_token_offset,
                     inv_permuted_idx, permuted_idx)


def moe_permute_metadata(topk_ids, token_expert_indices, expert_map, n_expert: int,
                         n_local_expert: int, topk: int, expert_first_token_offset,
                         inv_permuted_idx, permuted_idx) -> None:
    _OPS.moe_permute_metadata(topk_ids, token_expert_indices, expert_map, n_expert,
                              n_local_expert, topk, expert_first_token_offset,
                              inv_permuted_idx, permuted_idx)


def moe_unpermute(permuted_hidden_states, topk_weights, inv_permuted_idx,
                  expert_first_token_offset, topk: int, out) -> None:
    if topk_weights.dtype != torch.float32:
        topk_weights = topk_weights.to(torch.float32)
    _OPS.moe_unpermute(permuted_hidden_states, topk_weights, inv_permuted_idx,
                       expert_first_token_offset, topk, out)


def moe_permute_unpermute_supported() -> bool:
    return _OPS.moe_permute_unpermute_supported()
