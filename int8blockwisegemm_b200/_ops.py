"""``torch.ops.int8_hybrid_moe`` registration backed by libi8moe.so.

The ten schemas of the reference (csrc/torch_bindings.cpp:73-132) are
registered verbatim, each with a CUDA implementation that validates its
arguments like the reference's TORCH_CHECKs, then calls the C ABI on the
current stream.  Extension ops with no reference counterpart are added in the
same namespace (moe_route_for_gemm, int8_grouped_mm_scaled).

Nothing here synchronises with the host except ``cutlass_int8_grouped_mm``,
whose reference implementation reads expert_offsets / problem_sizes on the
host to validate them (csrc/int8_grouped_gemm.cu:114-151); set
INT8_HYBRID_MOE_SKIP_HOST_CHECKS=1 (or capture a CUDA graph) to skip that.
"""

from __future__ import annotations

import os

import torch

from . import _lib
from ._lib import BF16, FP16, FP32, S32, call

_DT = {torch.bfloat16: BF16, torch.float16: FP16, torch.float32: FP32}
# GEMM outputs: the reference's bf16, fp16 (extension) and the raw int32
# accumulator (verification extension).
_OUT_DT = {torch.bfloat16: BF16, torch.float16: FP16, torch.int32: S32}

SCHEMAS = {
    "cutlass_int8_grouped_mm":
        "cutlass_int8_grouped_mm(Tensor a, Tensor b, Tensor(a!) out, float a_scale, "
        "float b_scale, Tensor expert_offsets, Tensor problem_sizes) -> ()",
    "cutlass_int8_blockwise_hybrid_grouped":
        "cutlass_int8_blockwise_hybrid_grouped(Tensor a_q, Tensor a_qscale, Tensor a_fscale, "
        "Tensor b_q, Tensor b_qscale, Tensor b_fscale, Tensor expert_offsets, "
        "Tensor problem_sizes, Tensor(a!) out, int quant_block_size, int super_group_size, "
        "Tensor? scale_offsets=None) -> ()",
    "cutlass_int8_blockwise_hybrid_grouped_bias":
        "cutlass_int8_blockwise_hybrid_grouped_bias(Tensor a_q, Tensor a_qscale, "
        "Tensor a_fscale, Tensor b_q, Tensor b_qscale, Tensor b_fscale, Tensor expert_offsets, "
        "Tensor problem_sizes, Tensor(a!) out, Tensor bias, int quant_block_size, "
        "int super_group_size, Tensor? scale_offsets=None) -> ()",
    "cutlass_int8_blockwise_hybrid_grouped_small":
        "cutlass_int8_blockwise_hybrid_grouped_small(Tensor a_q, Tensor a_qscale, "
        "Tensor a_fscale, Tensor b_q, Tensor b_qscale, Tensor b_fscale, Tensor expert_offsets, "
        "Tensor problem_sizes, Tensor(a!) out, int quant_block_size, int super_group_size, "
        "Tensor? scale_offsets=None) -> ()",
    "cutlass_int8_blockwise_hybrid_grouped_small_bias":
        "cutlass_int8_blockwise_hybrid_grouped_small_bias(Tensor a_q, Tensor a_qscale, "
        "Tensor a_fscale, Tensor b_q, Tensor b_qscale, Tensor b_fscale, Tensor expert_offsets, "
        "Tensor problem_sizes, Tensor(a!) out, Tensor bias, int quant_block_size, "
        "int super_group_size, Tensor? scale_offsets=None) -> ()",
    "moe_permute":
        "moe_permute(Tensor input, Tensor topk_ids, Tensor token_expert_indices, "
        "Tensor? expert_map, int n_expert, int n_local_expert, int topk, "
        "Tensor! permuted_input, Tensor! expert_first_token_offset, "
        "Tensor! inv_permuted_idx, Tensor! permuted_idx) -> ()",
    "moe_permute_metadata":
        "moe_permute_metadata(Tensor topk_ids, Tensor token_expert_indices, "
        "Tensor? expert_map, int n_expert, int n_local_expert, int topk, "
        "Tensor! expert_first_token_offset, Tensor! inv_permuted_idx, "
        "Tensor! permuted_idx) -> ()",
    "moe_unpermute":
        "moe_unpermute(Tensor permuted_hidden_states, Tensor topk_weights, "
        "Tensor inv_permuted_idx, Tensor? expert_first_token_offset, int topk, "
        "Tensor! hidden_states) -> ()",
    "moe_permute_unpermute_supported": "moe_permute_unpermute_supported() -> bool",
    "silu_and_mul": "silu_and_mul(Tensor! out, Tensor input) -> ()",
    # ---- extensions (no reference counterpart) ----
    "moe_route_for_gemm":
        "moe_route_for_gemm(Tensor topk_ids, Tensor? token_expert_indices, Tensor? expert_map, "
        "int n_expert, int n_local_expert, int topk, Tensor! expert_first_token_offset, "
        "Tensor! inv_permuted_idx, Tensor! permuted_idx, Tensor! expert_offsets, "
        "Tensor! problem_sizes13, Tensor! problem_sizes2, Tensor! scale_offsets, int n_out1, "
        "int k1, int n_out2, int k2, int tile_m) -> ()",
    "int8_grouped_mm_scaled":
        "int8_grouped_mm_scaled(Tensor a, Tensor b, Tensor(a!) out, Tensor a_row_scale, "
        "Tensor b_expert_scale, Tensor expert_offsets, Tensor problem_sizes) -> ()",
}


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _capturing() -> bool:
    return torch.cuda.is_current_stream_capturing()


# ---------------------------------------------------------------------------
# GEMMs
# ---------------------------------------------------------------------------

def _check_hybrid(a_q, a_qs, a_fs, b_q, b_qs, b_fs, eo, ps, out):
    """int8_hybrid_grouped_gemm.cu:481-565 (check_base_inputs)."""
    ts = (a_q, a_qs, a_fs, b_q, b_qs, b_fs, eo, ps, out)
    _check(all(t.is_cuda for t in ts), "all grouped hybrid tensors must be CUDA tensors")
    _check(all(t.device == a_q.device for t in ts),
           "all grouped hybrid tensors must be on the same device")
    _check(all(t.is_contiguous() for t in ts), "all grouped hybrid tensors must be contiguous")
    _check(a_q.dtype == torch.int8, "a_q must be int8")
    _check(b_q.dtype == torch.int8, "b_q must be int8")
    _check(a_qs.dtype == torch.int32, "a_qscale must be int32")
    _check(b_qs.dtype == torch.int32, "b_qscale must be int32")
    _check(a_fs.dtype == torch.float32, "a_fscale must be float32")
    _check(b_fs.dtype == torch.float32, "b_fscale must be float32")
    _check(eo.dtype == torch.int32, "expert_offsets must be int32")
    _check(ps.dtype == torch.int32, "problem_sizes must be int32")
    _check(out.dtype in _OUT_DT, "out must be bfloat16 (or float16 / int32)")
    _check(a_q.dim() == 2, "a_q must have shape [sum_M, K]")
    _check(a_qs.dim() == 2, "a_qscale must have shape [sum_e ceil(M_e / TileM), K_blocks]")
    _check(a_fs.dim() == 2,
           "a_fscale must have shape [sum_e ceil(M_e / TileM), num_super_groups]")
    _check(b_q.dim() == 3, "b_q must have shape [E, N, K]")
    _check(b_qs.dim() == 3, "b_qscale must have shape [E, ceil(N / TileN), K_blocks]")
    _check(b_fs.dim() == 3, "b_fscale must have shape [E, ceil(N / TileN), num_super_groups]")
    _check(eo.dim() == 1, "expert_offsets must have shape [E + 1]")
    _check(ps.dim() == 2 and ps.size(1) == 3, "problem_sizes must have shape [E, 3]")
    _check(out.dim() == 2, "out must have shape [sum_M, N]")
    E, N, K = b_q.shape
    _check(ps.size(0) == E, "problem_sizes.shape[0] must equal b_q.shape[0]")
    _check(eo.size(0) == E + 1, "expert_offsets must have E + 1 entries")
    _check(a_q.size(1) == K, "a_q.shape[1] must equal b_q.shape[2]")
    _check(out.size(0) == a_q.size(0), "out.shape[0] must equal a_q.shape[0]")
    _check(out.size(1) == N, "out.shape[1] must equal b_q.shape[1]")
    _check(K % 32 == 0, "K must be divisible by 32 for INT8 tensor ops")


def _hybrid(tile_m: int, with_bias: bool):
    def impl(a_q, a_qs, a_fs, b_q, b_qs, b_fs, eo, ps, out, *rest):
        # the dispatcher passes trailing defaulted arguments only when given
        if with_bias:
            bias, qbs, sg = rest[:3]
            so = rest[3] if len(rest) > 3 else None
        else:
            qbs, sg = rest[:2]
            so = rest[2] if len(rest) > 2 else None
            bias = None
        _check_hybrid(a_q, a_qs, a_fs, b_q, b_qs, b_fs, eo, ps, out)
        E, N, K = b_q.shape
        if so is not None:
            _check(so.is_cuda, "scale_offsets must be CUDA")
            _check(so.device == a_q.device, "scale_offsets must share device with a_q")
            _check(so.is_contiguous(), "scale_offsets must be contiguous")
            _check(so.dtype == torch.int32, "scale_offsets must be int32")
            _check(so.dim() == 1, "scale_offsets must have shape [E]")
            _check(so.size(0) == E, "scale_offsets length must equal num experts")
        bias_stride = 0
        if bias is not None:
            _check(bias.is_cuda, "bias must be a CUDA tensor")
            _check(bias.device == a_q.device, "bias must be on the same device")
            _check(bias.is_contiguous(), "bias must be contiguous")
            _check(bias.dtype == torch.float32, "bias must be float32")
            _check((bias.dim() == 1 and bias.size(0) == N)
                   or (bias.dim() == 2 and bias.size(0) == E and bias.size(1) == N),
                   "bias must have shape [N] or [E, N]")
            bias_stride = N if bias.dim() == 2 else 0
        _check(qbs > 0, "quant_block_size must be positive")
        _check(sg > 0, "super_group_size must be positive")
        _check(qbs % 128 == 0, "quant_block_size must be divisible by the selected TileK")
        nqb = -(-K // qbs)
        nsg = -(-nqb // sg)
        nsb = -(-N // 64)
        _check(a_qs.size(1) == nqb, "a_qscale.shape[1] must equal ceil(K / quant_block_size)")
        _check(a_fs.size(1) == nsg, "a_fscale.shape[1] must equal num_super_groups")
        _check(tuple(b_qs.shape) == (E, nsb, nqb),
               "b_qscale must have shape [E, ceil(N / TileN), K_blocks] for the selected variant")
        _check(tuple(b_fs.shape) == (E, nsb, nsg),
               "b_fscale must have shape [E, ceil(N / TileN), num_super_groups] "
               "for the selected variant")
        if a_qs.size(0) * nsb == 0:
            return
        with torch.cuda.device(a_q.device):
            call("i8moe_hybrid_grouped_gemm", a_q.data_ptr(), a_qs.data_ptr(), a_fs.data_ptr(),
                 a_qs.size(0), b_q.data_ptr(), b_qs.data_ptr(), b_fs.data_ptr(), eo.data_ptr(),
                 ps.data_ptr(), _ptr(so), _ptr(bias), bias_stride, out.data_ptr(),
                 _OUT_DT[out.dtype], E, a_q.size(0), N, K, qbs, sg, tile_m, _stream(a_q))
    return impl


def _check_grouped_mm(a, b, out, eo, ps):
    """int8_grouped_gemm.cu:52-94."""
    _check(a.is_cuda and b.is_cuda and out.is_cuda, "a, b, and out must be CUDA tensors")
    _check(eo.is_cuda and ps.is_cuda, "expert_offsets and problem_sizes must be CUDA tensors")
    _check(b.device == a.device and out.device == a.device and eo.device == a.device
           and ps.device == a.device, "all tensors must be on the same CUDA device")
    _check(a.is_contiguous() and b.is_contiguous() and out.is_contiguous(),
           "a, b, and out must be contiguous")
    _check(eo.is_contiguous() and ps.is_contiguous(),
           "expert_offsets and problem_sizes must be contiguous")
    _check(a.dtype == torch.int8, "a must be int8")
    _check(b.dtype == torch.int8, "b must be int8")
    _check(out.dtype in _OUT_DT, "out must be bfloat16 (or float16 / int32)")
    _check(eo.dtype == torch.int32, "expert_offsets must be int32")
    _check(ps.dtype == torch.int32, "problem_sizes must be int32")
    _check(a.dim() == 2, "a must have shape [sum_M, K]")
    _check(b.dim() == 3, "b must have shape [E, N, K]")
    _check(out.dim() == 2, "out must have shape [sum_M, N]")
    _check(ps.dim() == 2 and ps.size(1) == 3, "problem_sizes must have shape [E, 3]")
    _check(eo.dim() == 1, "expert_offsets must have shape [E + 1]")
    E, N, K = b.shape
    _check(ps.size(0) == E, "problem_sizes.shape[0] must equal b.shape[0]")
    _check(eo.size(0) == E + 1, "expert_offsets must have E + 1 entries")
    _check(a.size(1) == K, "a.shape[1] must equal b.shape[2]")
    _check(out.size(0) == a.size(0), "out.shape[0] must equal a.shape[0]")
    _check(out.size(1) == N, "out.shape[1] must equal b.shape[1]")
    _check(K % 32 == 0, "K must be divisible by 32 for INT8 tensor ops")
    if os.environ.get("INT8_HYBRID_MOE_SKIP_HOST_CHECKS", "0") == "1" or _capturing():
        return
    h_off = eo.cpu()
    h_ps = ps.cpu()
    _check(int(h_off[0]) == 0, "expert_offsets[0] must be 0")
    _check(int(h_off[-1]) == a.size(0), "expert_offsets[-1] must equal a.shape[0]")
    d = h_off[1:] - h_off[:-1]
    _check(bool((h_ps[:, 0] == d).all()), "problem_sizes[e, 0] must match expert_offsets delta")
    _check(bool((h_ps[:, 1] == N).all()), "all problems must use N == b.shape[1]")
    _check(bool((h_ps[:, 2] == K).all()), "all problems must use K == b.shape[2]")


def _grouped_mm(a, b, out, a_scale, b_scale, eo, ps):
    _check_grouped_mm(a, b, out, eo, ps)
    E, N, K = b.shape
    alpha = float(torch.tensor(a_scale * b_scale, dtype=torch.float64).float())
    with torch.cuda.device(a.device):
        call("i8moe_int8_grouped_mm", a.data_ptr(), b.data_ptr(), out.data_ptr(),
             _OUT_DT[out.dtype], alpha, None, None, eo.data_ptr(), ps.data_ptr(), E, a.size(0), N, K,
             _stream(a))


def _grouped_mm_scaled(a, b, out, a_row_scale, b_expert_scale, eo, ps):
    _check_grouped_mm(a, b, out, eo, ps)
    E, N, K = b.shape
    _check(a_row_scale.dtype == torch.float32 and a_row_scale.numel() == a.size(0)
           and a_row_scale.is_contiguous(), "a_row_scale must be float32 [sum_M]")
    _check(b_expert_scale.dtype == torch.float32 and b_expert_scale.numel() == E
           and b_expert_scale.is_contiguous(), "b_expert_scale must be float32 [E]")
    with torch.cuda.device(a.device):
        call("i8moe_int8_grouped_mm", a.data_ptr(), b.data_ptr(), out.data_ptr(),
             _OUT_DT[out.dtype], 1.0, a_row_scale.data_ptr(), b_expert_scale.data_ptr(),
             eo.data_ptr(), ps.data_ptr(), E, a.size(0), N, K, _stream(a))


# ---------------------------------------------------------------------------
# permute / unpermute / activation
# ---------------------------------------------------------------------------

def _check_permute_common(topk_ids, tei, eft, inv, n_local):
    """moe_permute_unpermute_op.cu:20-31 / :89-100."""
    _check(eft.dtype == torch.int64, "expert_first_token_offset must be int64")
    _check(topk_ids.dtype == torch.int32, "topk_ids must be int32")
    _check(tei.dtype == torch.int32, "token_expert_indices must be int32")
    _check(inv.dtype == torch.int32, "inv_permuted_idx must be int32")
    _check(eft.size(0) == n_local + 1, "expert_first_token_offset shape != n_local_expert+1")
    _check(inv.shape == tei.shape, "token_expert_indices shape must be same as inv_permuted_idx")
    for t in (topk_ids, tei, eft, inv):
        _check(t.is_cuda and t.is_contiguous(), "moe_permute tensors must be contiguous CUDA")


def _route_ws(R: int, n_expert: int, device) -> torch.Tensor:
    nbytes = int(_lib.LIB.i8moe_route_workspace_size(R, n_expert))
    return torch.empty(max(nbytes, 16), dtype=torch.uint8, device=device)


def _permute_metadata(topk_ids, tei, emap, n_expert, n_local, topk, eft, inv, pidx):
    _check_permute_common(topk_ids, tei, eft, inv, n_local)
    n_token = topk_ids.size(0)
    ws = _route_ws(n_token * topk, n_expert, topk_ids.device)
    with torch.cuda.device(topk_ids.device):
        call("i8moe_moe_permute_metadata", topk_ids.data_ptr(), tei.data_ptr(), _ptr(emap),
             n_token, topk, n_expert, n_local, eft.data_ptr(), inv.data_ptr(), pidx.data_ptr(),
             ws.data_ptr(), ws.numel(), _stream(topk_ids))


def _permute(inp, topk_ids, tei, emap, n_expert, n_local, topk, pin, eft, inv, pidx):
    _check_permute_common(topk_ids, tei, eft, inv, n_local)
    _check(inp.dtype in _DT and pin.dtype == inp.dtype, "moe_permute: unsupported dtype")
    n_token, n_hidden = inp.shape
    ws = _route_ws(n_token * topk, n_expert, inp.device)
    with torch.cuda.device(inp.device):
        call("i8moe_moe_permute", inp.data_ptr(), _DT[inp.dtype], n_hidden, topk_ids.data_ptr(),
             tei.data_ptr(), _ptr(emap), n_token, topk, n_expert, n_local, pin.data_ptr(),
             eft.data_ptr(), inv.data_ptr(), pidx.data_ptr(), ws.data_ptr(), ws.numel(),
             _stream(inp))


def _route_for_gemm(topk_ids, tei, emap, n_expert, n_local, topk, eft, inv, pidx, eo32, ps1,
                    ps2, so, n_out1, k1, n_out2, k2, tile_m):
    # token_expert_indices may be omitted: it is arange(n_token * topk)
    _check_permute_common(topk_ids, tei if tei is not None else inv, eft, inv, n_local)
    n_token = topk_ids.size(0)
    ws = _route_ws(n_token * topk, n_expert, topk_ids.device)
    with torch.cuda.device(topk_ids.device):
        call("i8moe_moe_route_for_gemm", topk_ids.data_ptr(), _ptr(tei), _ptr(emap),
             n_token, topk, n_expert, n_local, eft.data_ptr(), inv.data_ptr(), pidx.data_ptr(),
             eo32.data_ptr(), ps1.data_ptr(), ps2.data_ptr(), so.data_ptr(), n_out1, k1, n_out2,
             k2, tile_m, ws.data_ptr(), ws.numel(), _stream(topk_ids))


def _unpermute(x, w, inv, eft, topk, out):
    """moe_permute_unpermute_op.cu:134-169."""
    _check(x.dtype == out.dtype, "permuted_hidden_states dtype must be same as hidden_states")
    _check(w.dtype == torch.float32,
           f"moe_unpermute: topk_weights must be float32 (got {w.dtype}); the kernel "
           "reinterprets this buffer as float* unconditionally")
    _check(x.dtype in _DT, "moe_unpermute: unsupported dtype")
    n_token, n_hidden = out.shape
    n_local = eft.size(0) - 1 if eft is not None else 0
    with torch.cuda.device(out.device):
        call("i8moe_moe_unpermute", x.data_ptr(), _DT[x.dtype], w.data_ptr(), inv.data_ptr(),
             _ptr(eft), n_local, n_token, topk, n_hidden, out.data_ptr(), _stream(out))


def _silu_and_mul(out, inp):
    _check(inp.dtype in _DT and out.dtype == inp.dtype, "silu_and_mul: unsupported dtype")
    d = inp.size(-1) // 2
    rows = inp.numel() // inp.size(-1) if inp.size(-1) else 0
    if rows == 0:
        return
    with torch.cuda.device(inp.device):
        call("i8moe_silu_and_mul", out.data_ptr(), inp.data_ptr(), _DT[inp.dtype], rows, d,
             _stream(inp))


def _supported() -> bool:
    return bool(_lib.LIB.i8moe_moe_permute_unpermute_supported())


_LIB = None


def register() -> torch.library.Library:
    global _LIB
    if _LIB is not None:
        return _LIB
    lib = torch.library.Library("int8_hybrid_moe", "DEF")
    for schema in SCHEMAS.values():
        lib.define(schema)
    lib.impl("cutlass_int8_grouped_mm", _grouped_mm, "CUDA")
    lib.impl("int8_grouped_mm_scaled", _grouped_mm_scaled, "CUDA")
    lib.impl("cutlass_int8_blockwise_hybrid_grouped", _hybrid(128, False), "CUDA")
    lib.impl("cutlass_int8_blockwise_hybrid_grouped_bias", _hybrid(128, True), "CUDA")
    lib.impl("cutlass_int8_blockwise_hybrid_grouped_small", _hybrid(64, False), "CUDA")
    lib.impl("cutlass_int8_blockwise_hybrid_grouped_small_bias", _hybrid(64, True), "CUDA")
    lib.impl("moe_permute", _permute, "CUDA")
    lib.impl("moe_permute_metadata", _permute_metadata, "CUDA")
    lib.impl("moe_route_for_gemm", _route_for_gemm, "CUDA")
    lib.impl("moe_unpermute", _unpermute, "CUDA")
    lib.impl("silu_and_mul", _silu_and_mul, "CUDA")
    lib.impl("moe_permute_unpermute_supported", _supported, "CompositeExplicitAutograd")
    _LIB = lib
    return lib
