"""Activation quantisation entry points with the reference's signatures and
return values (int8_hybrid_moe/quant.py:99-140, 212-277, 360-433, 514-579),
computed by the sm_100a kernels of libi8moe (csrc/quant.cu): two launches,
``quant_rows_kernel`` (the per-(expert M-tile x 128-K block) absmax INT8
quantisation, writing the raw block scales into the Q buffer) and
``scales_to_qf`` (the two-level Q int32 / F fp32 factorisation, in place).

Each function returns ``(qA, Q_A, F_A, scale_offsets_i32)`` with
Q_A [cdiv(M, tile_m) + E, K_blocks] and F_A [same rows, num_super_groups];
only the first scale_offsets[E] rows are written (the reference leaves the
remaining rows of its ``torch.empty`` scale buffer unset as well).
"""

from __future__ import annotations

from math import prod

import torch

from ._lib import BF16, FP16, FP32, call

_DT = {torch.bfloat16: BF16, torch.float16: FP16, torch.float32: FP32}


def cdiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def _resize_cache(x: torch.Tensor, v: tuple[int, ...]) -> torch.Tensor:
    """Shrink a workspace and view it with shape ``v`` (quant.py:26-29)."""
    assert prod(v) <= x.numel(), f"{v} ({prod(v)}) <= {x.shape} ({x.numel()})"
    return x.flatten()[: prod(v)].view(*v)


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _outputs(M: int, K: int, E: int, tile_m: int, block_k: int, super_group_size: int, device):
    kb = cdiv(K, block_k)
    rows = cdiv(M, tile_m) + E
    qA = torch.empty((M, K), dtype=torch.int8, device=device)
    Q = torch.empty((rows, kb), dtype=torch.int32, device=device)
    F = torch.empty((rows, cdiv(kb, super_group_size)), dtype=torch.float32, device=device)
    return qA, Q, F


def _eo32(expert_offsets: torch.Tensor) -> torch.Tensor:
    return expert_offsets if expert_offsets.dtype == torch.int32 else expert_offsets.to(torch.int32)


def quantize_scales_for_hybrid(scale: torch.Tensor, Q_max: int = 64,
                               super_group_size: int | None = None):
    """Two-level scale factorisation: F[r,g] = max(|s[r,g-block]|,1e-12)/Q_max,
    Q = rint(s / F)."""
    assert scale.ndim == 2, "scale must be a 2D tensor [X_blocks, K_blocks]"
    assert scale.dtype == torch.float32, "scale must be float32"
    rows, kb = scale.shape
    if super_group_size is None:
        super_group_size = kb
    nsg = cdiv(kb, super_group_size)
    scale = scale.contiguous()
    Q = torch.empty(rows, kb, dtype=torch.int32, device=scale.device)
    F = torch.empty(rows, nsg, dtype=torch.float32, device=scale.device)
    with torch.cuda.device(scale.device):
        call("i8moe_quantize_scales", scale.data_ptr(), rows, kb, Q_max, super_group_size,
             Q.data_ptr(), F.data_ptr(), _stream(scale))
    return Q, F


def moe_kernel_quantize_input_int8_hybrid_grouped(A, block_k: int, q_max: int,
                                                  super_group_size: int, expert_offsets,
                                                  tile_m: int, scale_offsets=None):
    """Grouped quant of an expert-contiguous [M, K] activation."""
    assert A.ndim == 2 and A.is_contiguous()
    assert A.dtype in _DT
    assert expert_offsets.ndim == 1 and expert_offsets.is_cuda
    assert block_k > 0 and tile_m > 0 and super_group_size > 0
    M, K = A.shape
    eo = _eo32(expert_offsets)
    E = eo.numel() - 1
    qA, Q, F = _outputs(M, K, E, tile_m, block_k, super_group_size, A.device)
    so, ready = _so(scale_offsets, E, A.device)
    with torch.cuda.device(A.device):
        call("i8moe_quant_grouped", A.data_ptr(), _DT[A.dtype], M, K, eo.data_ptr(), E, tile_m,
             block_k, q_max, super_group_size, qA.data_ptr(), Q.data_ptr(), F.data_ptr(),
             so.data_ptr(), ready, _stream(A))
    return qA, Q, F, so[:-1]


def fused_permute_quant_int8_hybrid_grouped(hidden_states, permuted_idx, topk: int,
                                            block_k: int, q_max: int, super_group_size: int,
                                            expert_offsets, tile_m: int, scale_offsets=None):
    """Gather hidden_states[permuted_idx // topk] and quantise in one pass."""
    assert hidden_states.ndim == 2 and hidden_states.is_contiguous()
    assert hidden_states.dtype in _DT
    assert permuted_idx.ndim == 1 and permuted_idx.is_cuda
    assert permuted_idx.dtype == torch.int32
    assert expert_offsets.ndim == 1 and expert_offsets.is_cuda
    assert topk > 0 and block_k > 0 and tile_m > 0 and super_group_size > 0
    n_token, K = hidden_states.shape
    M = permuted_idx.numel()
    eo = _eo32(expert_offsets)
    E = eo.numel() - 1
    qA, Q, F = _outputs(M, K, E, tile_m, block_k, super_group_size, hidden_states.device)
    so, ready = _so(scale_offsets, E, hidden_states.device)
    with torch.cuda.device(hidden_states.device):
        call("i8moe_quant_permute", hidden_states.data_ptr(), _DT[hidden_states.dtype], n_token,
             K, permuted_idx.data_ptr(), M, topk, eo.data_ptr(), E, tile_m, block_k, q_max,
             super_group_size, qA.data_ptr(), Q.data_ptr(), F.data_ptr(), so.data_ptr(), ready,
             _stream(hidden_states))
    return qA, Q, F, so[:-1]


def fused_silu_quant_int8_hybrid_grouped(mm1_out, block_k: int, q_max: int,
                                         super_group_size: int, expert_offsets, tile_m: int,
                                         scale_offsets=None):
    """silu(gate) * up of the w13 output, quantised over the intermediate dim."""
    assert mm1_out.ndim == 2 and mm1_out.is_contiguous()
    assert mm1_out.dtype in _DT
    assert expert_offsets.ndim == 1 and expert_offsets.is_cuda
    assert block_k > 0 and tile_m > 0 and super_group_size > 0
    sum_m, two_n = mm1_out.shape
    assert two_n % 2 == 0, "w13 output must have an even last dim (2*N)"
    N = two_n // 2
    eo = _eo32(expert_offsets)
    E = eo.numel() - 1
    qA, Q, F = _outputs(sum_m, N, E, tile_m, block_k, super_group_size, mm1_out.device)
    so, ready = _so(scale_offsets, E, mm1_out.device)
    with torch.cuda.device(mm1_out.device):
        call("i8moe_quant_silu", mm1_out.data_ptr(), _DT[mm1_out.dtype], sum_m, N,
             eo.data_ptr(), E, tile_m, block_k, q_max, super_group_size, qA.data_ptr(),
             Q.data_ptr(), F.data_ptr(), so.data_ptr(), ready, _stream(mm1_out))
    return qA, Q, F, so[:-1]


def quantize_weights_blockwise_int8(w: torch.Tensor, block_n: int = 64, block_k: int = 128):
    """Blockwise INT8 weights on the device, the reference's weight
    preparation ``_quantize_blockwise_int8`` (bench_int8_hybrid_moe.py:98-120).
    Returns (q int8 [E, N, K], scale fp32 [E, ceil(N/64), ceil(K/128)])."""
    assert w.ndim == 3 and w.is_cuda and w.dtype in _DT
    w = w.contiguous()
    E, N, K = w.shape
    q = torch.empty((E, N, K), dtype=torch.int8, device=w.device)
    scale = torch.empty((E, cdiv(N, block_n), cdiv(K, block_k)), dtype=torch.float32,
                        device=w.device)
    with torch.cuda.device(w.device):
        call("i8moe_quantize_weights", w.data_ptr(), _DT[w.dtype], E, N, K, block_n, block_k,
             q.data_ptr(), scale.data_ptr(), _stream(w))
    return q, scale


def prepare_hybrid_weights(w: torch.Tensor, q_max: int, super_group_size: int,
                           block_n: int = 64, block_k: int = 128):
    """Device version of the reference's weight preparation: blockwise INT8
    weights plus the hybrid (Q, F) factorisation of their scales along K
    (bench_int8_hybrid_moe.py:228-244).  Returns (q [E, N, K] int8,
    Q [E, N/64, Kb] int32, F [E, N/64, num_super_groups] fp32)."""
    q, scale = quantize_weights_blockwise_int8(w, block_n, block_k)
    E, Nb, Kb = scale.shape
    Q, F = quantize_scales_for_hybrid(scale.reshape(E * Nb, Kb), q_max, super_group_size)
    return q, Q.reshape(E, Nb, Kb), F.reshape(E, Nb, -1)


def fused_w13_silu_quant_int8_hybrid_grouped(a_q, a_qscale, a_fscale, w1, w1_qscale, w1_fscale,
                                             expert_offsets, problem_sizes, scale_offsets,
                                             block_k: int, q_max: int, super_group_size: int,
                                             tile_m: int, act_dtype, bias=None):
    """w13 hybrid grouped GEMM with SiLU(gate)*up + INT8 requant fused into its
    epilogue (no reference counterpart; equal to ``cutlass_int8_blockwise_
    hybrid_grouped`` into ``act_dtype`` followed by
    ``fused_silu_quant_int8_hybrid_grouped``, without the [M, 2N]
    intermediate).  ``scale_offsets``: the activation scale offsets for
    ``tile_m``, [E+1] (or [E], completed here).  Returns
    ``(a2q, Q_A2, F_A2, scale_offsets_i32)`` like the quant functions."""
    assert a_q.dtype == torch.int8 and w1.dtype == torch.int8
    assert act_dtype in (torch.bfloat16, torch.float16)
    sum_m, K = a_q.shape
    E, two_n, K2 = w1.shape
    assert K2 == K and two_n % 2 == 0
    N = two_n // 2
    eo = _eo32(expert_offsets)
    assert eo.numel() == E + 1
    dev = a_q.device
    if scale_offsets is not None and scale_offsets.numel() == E + 1:
        so = scale_offsets
    else:
        so = torch.empty(E + 1, dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            call("i8moe_scale_offsets", eo.data_ptr(), E, tile_m, so.data_ptr(), _stream(a_q))
    qA, Q, F = _outputs(sum_m, N, E, tile_m, block_k, super_group_size, dev)
    bias_stride = 0
    if bias is not None:
        assert bias.dtype == torch.float32 and bias.is_contiguous()
        bias_stride = 0 if bias.ndim == 1 else bias.shape[-1]
    with torch.cuda.device(dev):
        call("i8moe_hybrid_grouped_gemm_silu_quant", a_q.data_ptr(), a_qscale.data_ptr(),
             a_fscale.data_ptr(), a_qscale.shape[0], w1.data_ptr(), w1_qscale.data_ptr(),
             w1_fscale.data_ptr(), eo.data_ptr(), problem_sizes.data_ptr(), so.data_ptr(),
             bias.data_ptr() if bias is not None else None, bias_stride, _DT[act_dtype], E,
             sum_m, N, K, block_k, super_group_size, tile_m, q_max, qA.data_ptr(),
             Q.data_ptr(), F.data_ptr(), _stream(a_q))
    return qA, Q, F, so[:-1]


def _so(scale_offsets, E: int, device):
    """Scale-offset buffer [E+1]; ``scale_offsets`` (already computed for the
    same expert offsets and tile_m) is reused as is."""
    if scale_offsets is not None:
        assert scale_offsets.dtype == torch.int32 and scale_offsets.numel() == E + 1
        return scale_offsets, 1
    return torch.empty(E + 1, dtype=torch.int32, device=device), 0
