"""CPU restatement of the reference INT8 hybrid MoE forward path (numpy).

TEST INFRASTRUCTURE ONLY.  This module is the parity oracle for the CUDA
path in ``int8blockwisegemm_b200`` and the timed CPU baseline of
``bench.py``.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.
The product path never calls it.

Every function restates one piece of PatchouliTIS/INT8BlockwiseGEMM and
cites the reference file:line it follows (paths relative to the reference
project root).

Pinning.  The quantisation functions (``grouped_blockwise_quant``,
``fused_permute_quant``, ``fused_silu_quant``, ``quantize_scales_for_hybrid``)
and the orchestration in ``moe_forward`` are pinned against golden vectors
produced by running the reference's own Python/Triton code
(``int8_hybrid_moe/quant.py`` kernels in the Triton CPU interpreter,
``int8_hybrid_moe/cutlass_runner.py`` unchanged) -- see
``tests/golden/make_golden.py``.  The routing sort, the CUTLASS hybrid GEMM,
the per-tensor grouped GEMM, ``silu_and_mul`` and the unpermute reduction are
CUDA/CUB/CUTLASS code that cannot run without a GPU and without the absent
CUTLASS submodule; for those the restatement below follows the source and is
"parity unpinned" against the reference's own execution.

Arithmetic conventions:
  * "bf16"/"fp16" tensors are carried as float32 arrays whose values are
    exactly representable in that dtype; ``round_to(x, dtype)`` is the
    round-to-nearest-even conversion the CUDA code performs.
  * int32 arithmetic that may overflow is computed in int64 and wrapped
    modulo 2**32 (the reference uses plain C++ int32 arithmetic).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

# ---------------------------------------------------------------------------
# dtype helpers
# ---------------------------------------------------------------------------

DTYPES = ("bf16", "fp16", "fp32")


def bf16_round(x) -> np.ndarray:
    """float32 -> nearest-even bfloat16, returned as float32 values."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = x.view(np.uint32).astype(np.uint64)
    r = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.nan
    return out


def round_to(x, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` (RNE) and return them as float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "bf16":
        return bf16_round(x)
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "fp32":
        return x.copy()
    raise ValueError(dtype)


def wrap_i32(x) -> np.ndarray:
    """Two's-complement wrap of an integer array to int32."""
    return (np.asarray(x, dtype=np.int64) & 0xFFFFFFFF).astype(np.uint32).view(np.int32)


def fma_f32(a, b, c) -> np.ndarray:
    """float32 fused multiply-add, emulated in float64.

    Exact whenever a*b is exact in float64 (true for fp32 x bf16/fp16
    operands) and the float64 sum needs no rounding; otherwise it can differ
    from a hardware FMA by one float32 ulp through double rounding.
    """
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    c = np.asarray(c, np.float64)
    return (a * b + c).astype(np.float32)


def f32_to_i32(x) -> np.ndarray:
    """float -> int32 with truncation as PTX ``cvt.rzi.s32.f32`` does it:
    NaN -> 0, out-of-range values saturate."""
    x = np.asarray(x, np.float64)
    x = np.where(np.isnan(x), 0.0, np.trunc(x))
    return np.clip(x, -2147483648.0, 2147483647.0).astype(np.int32)


def clamp_f32(x, lo, hi) -> np.ndarray:
    """min(max(x, lo), hi) with NaN-suppressing max/min (PTX max.f32 /
    min.f32 return the non-NaN operand), as Triton's ``tl.clamp`` compiles."""
    return np.fmin(np.fmax(np.asarray(x, np.float32), np.float32(lo)), np.float32(hi))


def cdiv(a: int, b: int) -> int:
    return (a + b - 1) // b


# ---------------------------------------------------------------------------
# Routing / permutation  (csrc/permute_unpermute_kernels/*, csrc/moe_permute_unpermute_op.cu)
# ---------------------------------------------------------------------------


def experts_to_bits(n_expert: int) -> int:
    """Radix-sort key width.  moe_permute_unpermute_kernel.cu:11-15."""
    return int(math.floor(math.log2(2 * n_expert - 1))) + 1


def preprocess_topk_ids(topk_ids: np.ndarray, expert_map: np.ndarray, n_expert: int) -> np.ndarray:
    """Expert-parallel id remap.  moe_permute_unpermute_kernel.cu:132-160.

    A global id whose map entry is -1 (expert not on this rank) becomes
    ``id + n_expert`` so it sorts after every local expert; a local one
    becomes its local index.
    """
    ids = np.asarray(topk_ids, np.int64).reshape(-1)
    local = np.asarray(expert_map, np.int64)[ids]
    out = np.where(local == -1, ids + n_expert, local)
    return wrap_i32(out)


def sort_and_scan(keys: np.ndarray, values: np.ndarray, n_expert: int, n_local: int):
    """Stable key/value sort + per-expert first-row offsets.

    ``cub::DeviceRadixSort::SortPairs`` over bits [0, experts_to_bits) is a
    stable LSD sort on the low key bits (moe_permute_unpermute_kernel.cu:25-57,
    112-130); ``computeExpertFirstTokenOffsetKernel`` then binary-searches the
    sorted keys for every expert in [0, n_local] (:65-97).  For keys in
    [0, 2**bits) -- every id the reference produces -- the binary search equals
    "number of keys < e", which is what is returned here.
    """
    keys = np.asarray(keys, np.int32).reshape(-1)
    values = np.asarray(values, np.int32).reshape(-1)
    bits = experts_to_bits(n_expert)
    masked = keys.astype(np.int64) & ((1 << bits) - 1)
    order = np.argsort(masked, kind="stable")
    sorted_keys = keys[order]
    sorted_vals = values[order]
    sm = masked[order]
    offsets = np.searchsorted(sm, np.arange(n_local + 1), side="left").astype(np.int64)
    return sorted_keys, sorted_vals, offsets


def moe_permute_metadata(topk_ids, token_expert_indices, expert_map, n_expert: int,
                         n_local: int, topk: int):
    """Routing metadata without a row copy.

    Host op: csrc/moe_permute_unpermute_op.cu:81-132; maps:
    moe_permute_unpermute_kernel.inl:80-118; Python wrapper allocations
    (sentinel-filled permuted_idx): int8_hybrid_moe/permute.py:73-115.

    Returns (expert_first_token_offset int64 [n_local+1],
             inv_permuted_idx int32 [T, topk], permuted_idx int32 [T*topk]).
    """
    topk_ids = np.asarray(topk_ids, np.int32)
    T = topk_ids.shape[0]
    R = T * topk
    keys = topk_ids.reshape(-1)
    if expert_map is not None:
        keys = preprocess_topk_ids(keys, expert_map, n_expert)
    _, sorted_vals, offsets = sort_and_scan(keys, token_expert_indices, n_expert, n_local)
    inv = np.empty(R, np.int32)
    permuted_idx = np.full(R, R, np.int32)
    dest = np.arange(R, dtype=np.int64)
    inv[sorted_vals] = dest.astype(np.int32)
    limit = offsets[n_local] if expert_map is not None else R
    keep = dest < limit
    permuted_idx[dest[keep]] = sorted_vals[keep]
    return offsets, inv.reshape(T, topk), permuted_idx


def moe_permute(hidden, topk_ids, token_expert_indices, expert_map, n_expert: int,
                n_local: int, topk: int, permuted_input=None):
    """Routing metadata + row gather.

    csrc/moe_permute_unpermute_op.cu:10-79, expandInputRowsKernel
    moe_permute_unpermute_kernel.inl:3-78.  Rows whose destination is beyond
    the valid count (expert-parallel case) are not written.
    """
    hidden = np.asarray(hidden)
    offsets, inv, permuted_idx = moe_permute_metadata(
        topk_ids, token_expert_indices, expert_map, n_expert, n_local, topk)
    R = permuted_idx.shape[0]
    if permuted_input is None:
        permuted_input = np.zeros((R, hidden.shape[1]), hidden.dtype)
    limit = offsets[n_local] if expert_map is not None else R
    d = np.arange(int(limit))
    permuted_input[d] = hidden[permuted_idx[d] // topk]
    return permuted_input, offsets, inv, permuted_idx


# ---------------------------------------------------------------------------
# Activation quantisation  (int8_hybrid_moe/quant.py)
# ---------------------------------------------------------------------------

ACT_EPS = np.float32(1e-10)     # quant.py:265,420,568
SCALE_EPS = np.float32(1e-12)   # quant.py:137
INT8_MAX = np.float32(127.0)
INT8_MIN = np.float32(-128.0)


def round_half_away(y: np.ndarray) -> np.ndarray:
    """libdevice ``round``: nearest, ties away from zero (quant.py:36-39)."""
    y = np.asarray(y, np.float32)
    t = np.trunc(y)
    return np.where(np.abs(y - t) >= np.float32(0.5), t + np.sign(y), t).astype(np.float32)


def scale_offsets_from(expert_offsets, tile_m: int) -> np.ndarray:
    """Exclusive cumsum of ceil(M_e / tile_m), length E+1 (quant.py:238-242)."""
    eo = np.asarray(expert_offsets, np.int64)
    counts = eo[1:] - eo[:-1]
    sc = np.floor_divide(counts + tile_m - 1, tile_m)
    return np.concatenate([[0], np.cumsum(sc)]).astype(np.int64)


def _tile_rows(expert_offsets, tile_m: int, M: int):
    """Row index of every (scale row, row-in-tile) slot, -1 for masked slots.

    Scale row s belongs to the expert e with so[e] <= s < so[e+1] and covers
    rows [eo[e] + (s-so[e])*tile_m, min(+tile_m, eo[e+1], M))
    (quant.py:169-193, the binary search at :175-185).
    """
    eo = np.asarray(expert_offsets, np.int64)
    so = scale_offsets_from(eo, tile_m)
    S = int(so[-1])
    E = eo.shape[0] - 1
    rows = np.full((S, tile_m), -1, np.int64)
    for e in range(E):
        n_t = int(so[e + 1] - so[e])
        if n_t == 0:
            continue
        start = eo[e] + np.arange(n_t)[:, None] * tile_m + np.arange(tile_m)[None, :]
        valid = (start < eo[e + 1]) & (start < M)
        rows[so[e]:so[e + 1]] = np.where(valid, start, -1)
    return rows, so


def _quant_tiles(x_tiles: np.ndarray, valid: np.ndarray):
    """Per-(tile, K-block) absmax INT8 quant of x_tiles [S, tm, Kb*128]."""
    S, tm, Kp = x_tiles.shape
    Kb = Kp // 128
    xt = np.where(valid, x_tiles, np.float32(0)).reshape(S, tm, Kb, 128)
    absmax = np.abs(xt).max(axis=(1, 3)) if S > 0 else np.zeros((0, Kb), np.float32)
    scale = (np.maximum(absmax, ACT_EPS) / INT8_MAX).astype(np.float32)
    y = xt / scale[:, None, :, None]
    q = round_half_away(clamp_f32(y, INT8_MIN, INT8_MAX)).astype(np.int8)
    return q.reshape(S, tm, Kp), scale


def _quant_generic(get_x, M: int, K: int, expert_offsets, tile_m: int, block_k: int):
    if block_k != 128:
        raise NotImplementedError("the reference pipeline quantises with block_k == 128")
    rows, so = _tile_rows(expert_offsets, tile_m, M)
    S = rows.shape[0]
    Kb = cdiv(K, block_k)
    Kp = Kb * block_k
    flat = rows.reshape(-1)
    valid_r = flat >= 0
    x = np.zeros((flat.shape[0], Kp), np.float32)
    if valid_r.any():
        x[valid_r, :K] = get_x(flat[valid_r])
    colmask = np.zeros(Kp, bool)
    colmask[:K] = True
    valid = (valid_r[:, None] & colmask[None, :]).reshape(S, tile_m, Kp)
    q, scale = _quant_tiles(x.reshape(S, tile_m, Kp), valid)
    qA = np.zeros((M, K), np.int8)
    qf = q.reshape(-1, Kp)
    qA[flat[valid_r]] = qf[valid_r, :K]
    return qA, scale, so


def grouped_blockwise_quant(A, expert_offsets, tile_m: int, block_k: int = 128):
    """Per-(expert M-tile x 128-K block) absmax INT8 quant of an already
    permuted [M, K] activation.  quant.py:147-209 (kernel), :212-277 (host).

    Returns (qA int8 [M,K] -- rows outside every expert left 0,
             scale f32 [total_scale_rows, Kb], scale_offsets int64 [E+1]).
    """
    A = np.asarray(A, np.float32)
    M, K = A.shape
    return _quant_generic(lambda r: A[r], M, K, expert_offsets, tile_m, block_k)


def fused_permute_quant(hidden, permuted_idx, topk: int, expert_offsets, tile_m: int,
                        block_k: int = 128):
    """Gather hidden[permuted_idx // topk] and quantise.  quant.py:284-357,
    host :360-433."""
    hidden = np.asarray(hidden, np.float32)
    pidx = np.asarray(permuted_idx, np.int64)
    M = pidx.shape[0]
    K = hidden.shape[1]
    return _quant_generic(lambda r: hidden[pidx[r] // topk], M, K, expert_offsets, tile_m,
                          block_k)


def silu_mul_native(gate, up, dtype: str) -> np.ndarray:
    """``(g / (1 + exp(-g))).to(dtype) * up`` rounded to ``dtype``
    (quant.py:495-499): SiLU in float32, cast to the storage dtype, product in
    the storage dtype (exact product rounded once)."""
    g = np.asarray(gate, np.float32)
    u = np.asarray(up, np.float32)
    with np.errstate(over="ignore"):
        e = np.exp(-g)
        s = (g / (np.float32(1.0) + e)).astype(np.float32)
    s = round_to(s, dtype)
    return round_to(s * u, dtype)


def fused_silu_quant(mm1_out, expert_offsets, tile_m: int, dtype: str, block_k: int = 128):
    """SiLU(gate)*up + grouped INT8 quant over the intermediate dim.
    quant.py:440-511 (kernel), :514-579 (host)."""
    mm1 = np.asarray(mm1_out, np.float32)
    M, two_n = mm1.shape
    N = two_n // 2

    def get_x(r):
        return silu_mul_native(mm1[r, :N], mm1[r, N:], dtype)

    return _quant_generic(get_x, M, N, expert_offsets, tile_m, block_k)


def quantize_weights_blockwise(w, block_n: int = 64, block_k: int = 128):
    """Blockwise INT8 weights, bench_int8_hybrid_moe.py:98-120: per (expert,
    block_n rows, block_k columns) block, scale = max(absmax, 1e-10) / 127 and
    q = clamp(rint(w / scale), -128, 127) (torch.round: ties to even); the
    zero padding of ragged blocks takes part in the absmax.

    Returns (q int8 [E, N, K], scale f32 [E, ceil(N/block_n), ceil(K/block_k)])."""
    w = np.asarray(w, np.float32)
    E, N, K = w.shape
    nb, kb = -(-N // block_n), -(-K // block_k)
    pad = np.zeros((E, nb * block_n, kb * block_k), np.float32)
    pad[:, :N, :K] = w
    view = pad.reshape(E, nb, block_n, kb, block_k).transpose(0, 1, 3, 2, 4)
    amax = np.abs(view).max(axis=(-1, -2))
    scale = (np.maximum(amax, np.float32(1e-10)) / np.float32(127.0)).astype(np.float32)
    qv = np.clip(np.rint(view / scale[..., None, None]), -128, 127).astype(np.int8)
    q = qv.transpose(0, 1, 3, 2, 4).reshape(E, nb * block_n, kb * block_k)[:, :N, :K]
    return np.ascontiguousarray(q), scale


def quantize_scales_for_hybrid(scale, q_max: int = 64, super_group_size: int | None = None):
    """Two-level (Q int32, F fp32) factorisation of fp32 block scales.
    quant.py:52-96 (kernel), :99-140 (host).

    F[r, g] = max(max_{kb in g} |s[r,kb]|, 1e-12) / q_max;
    Q[r, kb] = rint(s[r,kb] / F[r, g(kb)])  (round half to even).
    """
    s = np.asarray(scale, np.float32)
    rows, Kb = s.shape
    if super_group_size is None:
        super_group_size = Kb
    n_sg = cdiv(Kb, super_group_size)
    Q = np.zeros((rows, Kb), np.int32)
    F = np.zeros((rows, n_sg), np.float32)
    for g in range(n_sg):
        lo, hi = g * super_group_size, min((g + 1) * super_group_size, Kb)
        blk = s[:, lo:hi]
        smax = np.maximum(np.abs(blk).max(axis=1) if rows else np.zeros(0, np.float32), SCALE_EPS)
        fg = (smax / np.float32(q_max)).astype(np.float32)
        F[:, g] = fg
        Q[:, lo:hi] = f32_to_i32(np.rint(blk / fg[:, None]))
    return Q, F


# ---------------------------------------------------------------------------
# GEMMs  (csrc/int8_hybrid_grouped_gemm.cu, csrc/int8_grouped_gemm.cu)
# ---------------------------------------------------------------------------

TILE_N_SCALE = 64     # int8_hybrid_grouped_gemm.cu:211-216 (TileN of both variants)
TILE_K = 128          # ibid.


def _k_tiles(K: int):
    """CUTLASS 2.x predicated iterators visit the partial K residue tile
    first: tiles are [0, r), [r, r+128), ... with r = K - 128*(Kt-1)
    (PredicatedTileAccessIterator residue handling, used by the mainloop at
    int8_hybrid_grouped_gemm.cu:303-306,344-443).  Left-padding K with
    128*Kt - K zeros gives the same tiles with uniform width."""
    Kt = cdiv(K, TILE_K)
    return Kt, Kt * TILE_K - K


def hybrid_grouped_gemm(A, QA, FA, B, QB, FB, expert_offsets, problem_sizes,
                        quant_block_size: int, tile_m: int, scale_offsets=None,
                        bias=None, out_dtype: str = "bf16", out=None, return_w: bool = False):
    """Grouped hybrid INT8 GEMM.  Kernel: int8_hybrid_grouped_gemm.cu:218-479;
    host checks :481-565,614-753.

    For expert e, row r (m-tile cta_m = (r-eo[e])//tile_m), column n
    (64-column scale block j = n//64) and scale row s = so[e] + cta_m:
      P_qb  = sum_{k in q-block qb} A[r,k] * B[e,n,k]                  (:344-432)
      W     = sum_qb (QA[s,qb] * QB[e,j,qb]) * P_qb    int32, wrapping (:433-442)
      out   = dtype_rn(float(W) * (FA[s,0] * FB[e,j,0]))               (:445-453,472-475)
      (_bias variants: float32(float(W) * F) + bias[n], two roundings, :449-458)
    Only the first super-group's F is read (:445-447).

    ``out`` rows that belong to no expert are left untouched.  With
    ``return_w`` the int32 W matrix is returned as well.
    """
    A = np.asarray(A, np.int8)
    B = np.asarray(B, np.int8)
    QA = np.asarray(QA, np.int64)
    QB = np.asarray(QB, np.int64)
    FA = np.asarray(FA, np.float32)
    FB = np.asarray(FB, np.float32)
    eo = np.asarray(expert_offsets, np.int64)
    ps = np.asarray(problem_sizes, np.int64)
    E, N, K = B.shape
    sum_m = A.shape[0]
    if quant_block_size % TILE_K:
        raise ValueError("quant_block_size must be divisible by the selected TileK")
    ktpq = quant_block_size // TILE_K
    Kt, pad = _k_tiles(K)
    nq = cdiv(Kt, ktpq)
    if out is None:
        out = np.zeros((sum_m, N), np.float32)
    W_all = np.zeros((sum_m, N), np.int32) if return_w else None
    if scale_offsets is None:
        m_tiles = np.floor_divide(ps[:, 0] + tile_m - 1, tile_m)
        so = np.concatenate([[0], np.cumsum(m_tiles)[:-1]]).astype(np.int64)
    else:
        so = np.asarray(scale_offsets, np.int64)
    jn = np.arange(N) // TILE_N_SCALE
    for e in range(E):
        m_e = int(ps[e, 0])
        if m_e <= 0:
            continue
        r0 = int(eo[e])
        a_e = np.zeros((m_e, Kt * TILE_K), np.float32)
        a_e[:, pad:] = A[r0:r0 + m_e]
        b_e = np.zeros((N, Kt * TILE_K), np.float32)  # one expert at a time (memory)
        b_e[:, pad:] = B[e]
        a_t = a_e.reshape(m_e, Kt, TILE_K).transpose(1, 0, 2)
        b_t = b_e.reshape(N, Kt, TILE_K).transpose(1, 2, 0)
        P = np.matmul(a_t, b_t)  # [Kt, m_e, N]: exact (|P| < 2**24)
        P = P.astype(np.int64)
        srow = so[e] + np.arange(m_e) // tile_m
        acc = np.zeros((m_e, N), np.int64)
        for qb in range(nq):
            pq = P[qb * ktpq:(qb + 1) * ktpq].sum(axis=0)
            q = wrap_i32(QA[srow, qb][:, None] * QB[e, jn, qb][None, :]).astype(np.int64)
            acc += q * pq
        W = wrap_i32(acc)
        f = (FA[srow, 0][:, None] * FB[e, jn, 0][None, :]).astype(np.float32)
        if bias is None:
            y = (W.astype(np.float32) * f).astype(np.float32)
        else:
            bias = np.asarray(bias, np.float32)
            bvec = bias[e] if bias.ndim == 2 else bias
            y = (W.astype(np.float32) * f).astype(np.float32) + bvec[None, :].astype(np.float32)
        out[r0:r0 + m_e] = round_to(y, out_dtype)
        if return_w:
            W_all[r0:r0 + m_e] = W
    if return_w:
        return out, W_all
    return out


def int8_grouped_mm(a, b, a_scale: float, b_scale: float, expert_offsets, problem_sizes,
                    out=None, a_row_scale=None, b_expert_scale=None, out_dtype: str = "bf16"):
    """Per-tensor-scaled grouped INT8 GEMM.  csrc/int8_grouped_gemm.cu:35-47
    (LinearCombination alpha = float(a_scale*b_scale), beta = 0), :106-220.

      out[r, n] = bf16_rn(float(acc[r,n]) * alpha),  acc = sum_k a[r,k]*b[e,n,k]

    Extension (no reference counterpart; opt-in): with per-token
    ``a_row_scale`` [sum_M] and per-expert ``b_expert_scale`` [E] the factor
    is alpha[r] = float32(a_row_scale[r] * b_expert_scale[e]).
    """
    a = np.asarray(a, np.int8)
    b = np.asarray(b, np.int8)
    eo = np.asarray(expert_offsets, np.int64)
    ps = np.asarray(problem_sizes, np.int64)
    E, N, K = b.shape
    if out is None:
        out = np.zeros((a.shape[0], N), np.float32)
    alpha = np.float32(a_scale * b_scale)
    for e in range(E):
        m_e = int(ps[e, 0])
        if m_e <= 0:
            continue
        r0 = int(eo[e])
        acc = (a[r0:r0 + m_e].astype(np.float64) @ b[e].astype(np.float64).T)
        acc = wrap_i32(acc.astype(np.int64)).astype(np.float32)
        if a_row_scale is not None:
            al = (np.asarray(a_row_scale, np.float32)[r0:r0 + m_e]
                  * np.float32(np.asarray(b_expert_scale, np.float32)[e])).astype(np.float32)
            y = acc * al[:, None]
        else:
            y = acc * alpha
        out[r0:r0 + m_e] = round_to(y.astype(np.float32), out_dtype)
    return out


# ---------------------------------------------------------------------------
# Activation and unpermute  (csrc/activation_kernels.cu, .inl finalize)
# ---------------------------------------------------------------------------


def silu_and_mul(x, dtype: str) -> np.ndarray:
    """out = dtype(silu(x[:, :d])) * x[:, d:]  (activation_kernels.cu:78-145,
    260-265): SiLU in float32, rounded to the storage dtype, then a
    storage-dtype multiply."""
    x = np.asarray(x, np.float32)
    d = x.shape[-1] // 2
    return silu_mul_native(x[..., :d], x[..., d:], dtype)


def moe_unpermute(permuted_hidden, topk_weights, inv_permuted_idx, expert_first_token_offset,
                  topk: int, out_dtype: str) -> np.ndarray:
    """Top-k weighted reduction back to token order.
    finalizeMoeRoutingKernel, moe_permute_unpermute_kernel.inl:132-206;
    host csrc/moe_permute_unpermute_op.cu:134-169.

      acc = 0; for j in 0..topk-1:  if inv[t,j] < valid: acc = fma(w[t,j], x[inv[t,j]], acc)
      out[t] = dtype_rn(acc)
    (the reference's ``acc + w * x`` is contracted to an FMA by nvcc.)
    """
    x = np.asarray(permuted_hidden, np.float32)
    w = np.asarray(topk_weights, np.float32).reshape(-1, topk)
    inv = np.asarray(inv_permuted_idx, np.int64).reshape(-1, topk)
    T = w.shape[0]
    valid = None
    if expert_first_token_offset is not None:
        valid = int(np.asarray(expert_first_token_offset, np.int64)[-1])
    acc = np.zeros((T, x.shape[1]), np.float32)
    for j in range(topk):
        idx = inv[:, j]
        ok = np.ones(T, bool) if valid is None else idx < valid
        safe = np.where(ok, idx, 0)
        upd = fma_f32(w[:, j][:, None], x[safe], acc)
        acc = np.where(ok[:, None], upd, acc)
    return round_to(acc, out_dtype)


# ---------------------------------------------------------------------------
# Orchestration  (int8_hybrid_moe/cutlass_runner.py)
# ---------------------------------------------------------------------------

VARIANT_TILE_M = {"hybrid": 128, "hybrid_small": 64}   # cutlass_runner.py:30


def pick_grouped_hybrid_variant(sum_m: int, num_experts: int) -> str:
    """cutlass_runner.py:43-50."""
    if num_experts <= 0:
        return "hybrid"
    return "hybrid_small" if sum_m / num_experts <= 70 else "hybrid"


@dataclass
class ForwardTrace:
    offsets: np.ndarray
    inv: np.ndarray
    permuted_idx: np.ndarray
    tile_m: int
    a1q: np.ndarray
    a1_scale: np.ndarray
    a1_Q: np.ndarray
    a1_F: np.ndarray
    a1_so: np.ndarray
    mm1: np.ndarray
    w1_acc: np.ndarray
    a2q: np.ndarray
    a2_scale: np.ndarray
    a2_Q: np.ndarray
    a2_F: np.ndarray
    mm2: np.ndarray
    out: np.ndarray


def moe_forward(hidden, w1, w2, topk_ids, topk_weights, w1_q, w1_f, w2_q, w2_f, *,
                dtype: str, global_num_experts: int, expert_map=None,
                quant_block_size: int = 128, super_group_size: int = 256, q_max: int = 16,
                fuse_permute: bool = True, fuse_silu: bool = True,
                trace: bool = False, tile_m: int | None = None):
    """Full INT8 hybrid MoE forward, cutlass_runner.py:69-236.

    Both activation-quant paths (fused permute+quant and permute-then-quant)
    produce the same int8 rows, as do the fused and unfused SiLU paths, so the
    flags only select which restated reference functions are exercised.
    """
    hidden = np.asarray(hidden, np.float32)
    topk_ids = np.asarray(topk_ids, np.int32)
    M, K = hidden.shape
    topk = topk_ids.shape[1]
    local_e = w1.shape[0]
    N = w2.shape[2]
    R = M * topk
    num_expert = global_num_experts if expert_map is None else np.asarray(expert_map).shape[0]
    tei = np.arange(R, dtype=np.int32).reshape(M, topk)
    if fuse_permute:
        offsets, inv, pidx = moe_permute_metadata(topk_ids, tei, expert_map, num_expert,
                                                  local_e, topk)
    else:
        a1, offsets, inv, pidx = moe_permute(hidden, topk_ids, tei, expert_map, num_expert,
                                             local_e, topk)
    eo = offsets.astype(np.int64)
    counts = eo[1:] - eo[:-1]
    ps1 = np.stack([counts, np.full(local_e, 2 * N), np.full(local_e, K)], 1)
    ps2 = np.stack([counts, np.full(local_e, K), np.full(local_e, N)], 1)
    variant = pick_grouped_hybrid_variant(R, local_e)
    tm = VARIANT_TILE_M[variant] if tile_m is None else tile_m  # tile_m: forced (EP tests)
    if fuse_permute:
        a1q, s1, so1 = fused_permute_quant(hidden, pidx, topk, eo, tm)
    else:
        a1q, s1, so1 = grouped_blockwise_quant(a1, eo, tm)
    Q1, F1 = quantize_scales_for_hybrid(s1, q_max, super_group_size)
    mm1, W1 = hybrid_grouped_gemm(a1q, Q1, F1, w1, w1_q, w1_f, eo, ps1, quant_block_size, tm,
                                  scale_offsets=so1[:-1], out_dtype=dtype, return_w=True)
    if fuse_silu:
        a2q, s2, so2 = fused_silu_quant(mm1, eo, tm, dtype)
    else:
        act = silu_and_mul(mm1, dtype)
        a2q, s2, so2 = grouped_blockwise_quant(act, eo, tm)
    Q2, F2 = quantize_scales_for_hybrid(s2, q_max, super_group_size)
    mm2 = hybrid_grouped_gemm(a2q, Q2, F2, w2, w2_q, w2_f, eo, ps2, quant_block_size, tm,
                              scale_offsets=so2[:-1], out_dtype=dtype)
    out = moe_unpermute(mm2, topk_weights, inv.reshape(-1), eo, topk, dtype)
    if not trace:
        return out
    return ForwardTrace(eo, inv, pidx, tm, a1q, s1, Q1, F1, so1, mm1, W1, a2q, s2, Q2, F2, mm2,
                        out)
