"""Parity with the reference's own CUDA code, executed on the same GPU.

oracle/build_ref.py compiles the reference's CUTLASS hybrid grouped GEMM
(csrc/int8_hybrid_grouped_gemm.cu), its per-tensor grouped GEMM
(csrc/int8_grouped_gemm.cu) and its CUB-based permute / unpermute
(csrc/moe_permute_unpermute_op.cu, csrc/permute_unpermute_kernels/) from the
reference source tree into oracle/_ref/libi8moe_ref.so, registered as
torch.ops.int8_hybrid_moe_ref.  These tests give both libraries the same
device inputs and compare:

  * routing: expert_first_token_offset, inv_permuted_idx, permuted_idx and
    the gathered rows of moe_permute -- bit-exact, with and without an EP
    expert_map;
  * the hybrid grouped GEMM: bf16 outputs of w13 and w2 (both tile_m
    variants, with and without bias) on the device's own INT8 activations and
    scales -- bit-exact;
  * the per-tensor grouped GEMM -- bit-exact;
  * the top-k weighted unpermute -- bit-exact (both accumulate in fp32 in
    top-k order).

The reference library is test infrastructure; the tests skip when it has not
been built (it needs the reference sources at build time).  The reference's
GEMM writes bf16 only, so fp16 configurations are not compared here.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from tests.helpers import load_workloads

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
REF_LIB = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libi8moe_ref.so"


@pytest.fixture(scope="module")
def refops():
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/libi8moe_ref.so is not built (python oracle/build_ref.py)")
    torch.ops.load_library(str(REF_LIB))
    return torch.ops.int8_hybrid_moe_ref


@pytest.fixture(scope="module")
def m():
    import int8blockwisegemm_b200 as pkg
    pkg._lib.device_error(0, clear=True)
    yield pkg
    assert pkg._lib.device_error(0) == 0, "a kernel reported a device-side error"


def inputs(name, **kw):
    from dataclasses import replace
    wl = load_workloads()
    cfg = wl.CONFIGS[name]
    if kw:
        cfg = replace(cfg, **kw)
    return cfg, wl.make_inputs(cfg)


def ep_map(E, rank, size):
    per = E // size
    emap = torch.full((E,), -1, dtype=torch.int32)
    emap[rank * per:(rank + 1) * per] = torch.arange(per, dtype=torch.int32)
    return emap.to(DEV), per


def ref_metadata(refops, ids, E, n_local, emap):
    """The reference's permute.moe_permute_metadata (permute.py:73-115)."""
    T, k = ids.shape
    tei = torch.arange(T * k, dtype=torch.int32, device=DEV).reshape(T, k)
    eft = torch.empty(n_local + 1, dtype=torch.int64, device=DEV)
    pidx = torch.full((T * k,), T * k, dtype=torch.int32, device=DEV)
    inv = torch.empty(T, k, dtype=torch.int32, device=DEV)
    refops.permute_metadata(ids, tei, emap, E, n_local, k, eft, inv, pidx)
    return eft, inv.flatten(), pidx


ROUTING_CASES = [("tiny", None), ("ragged", None), ("mid", None), ("decode", None),
                 ("default", None), ("skewed", None), ("large", None), ("tiny", (1, 2)),
                 ("mid", (2, 4)), ("default", (3, 8)), ("skewed", (0, 8))]


@pytest.mark.parametrize("name,ep", ROUTING_CASES,
                         ids=[f"{n}-ep{e[0]}of{e[1]}" if e else n for n, e in ROUTING_CASES])
def test_routing_matches_reference_cuda(m, refops, name, ep):
    cfg, inp = inputs(name)
    ids = inp["topk_ids"].to(DEV)
    emap, n_local = (None, cfg.E) if ep is None else ep_map(cfg.E, *ep)
    r_eft, r_inv, r_pidx = ref_metadata(refops, ids, cfg.E, n_local, emap)
    eft, inv, pidx = m.permute.moe_permute_metadata(inp["hidden"].to(DEV), ids, cfg.E, n_local,
                                                    emap)
    torch.cuda.synchronize()
    assert torch.equal(eft, r_eft)
    assert torch.equal(inv, r_inv)
    assert torch.equal(pidx, r_pidx)


@pytest.mark.parametrize("name,dtype", [("ragged", torch.bfloat16), ("mid", torch.float16),
                                        ("mid", torch.float32), ("default", torch.bfloat16)])
def test_permute_rows_match_reference_cuda(m, refops, name, dtype):
    cfg, inp = inputs(name)
    ids = inp["topk_ids"].to(DEV)
    hidden = inp["hidden"].to(dtype).to(DEV)
    T, k = ids.shape
    R = T * k
    tei = torch.arange(R, dtype=torch.int32, device=DEV).reshape(T, k)
    r_rows = torch.zeros(R, cfg.K, dtype=dtype, device=DEV)
    r_eft = torch.empty(cfg.E + 1, dtype=torch.int64, device=DEV)
    r_inv = torch.empty(T, k, dtype=torch.int32, device=DEV)
    r_pidx = torch.full((R,), R, dtype=torch.int32, device=DEV)
    refops.permute(hidden, ids, tei, None, cfg.E, cfg.E, k, r_rows, r_eft, r_inv, r_pidx)
    rows, _, eft, inv, _ = m.permute.moe_permute(hidden, None, ids, cfg.E, cfg.E, None)
    torch.cuda.synchronize()
    v = int(r_eft[-1])
    assert torch.equal(eft, r_eft)
    assert torch.equal(inv, r_inv.flatten())
    assert torch.equal(rows[:v], r_rows[:v])


def _gemm_case(m, cfg, inp):
    """Runs the unfused forward (so mm1 is materialised) and returns its trace."""
    r = m.cutlass_runner
    r._USE_FUSED_PERMUTE_QUANT_W1 = True
    r._USE_FUSED_SILU_QUANT_W2 = True
    r._USE_FUSED_W13_EPILOGUE = False
    try:
        dt = torch.bfloat16
        T, k = inp["topk_ids"].shape
        R = T * k
        d = {kk: v.to(DEV) for kk, v in inp.items()}
        out = torch.empty(T, cfg.K, dtype=dt, device=DEV)
        tr = {}
        r._run_cutlass_int8_hybrid_grouped_moe(
            out, d["hidden"], d["w13"], d["w2"], d["topk_ids"], d["topk_weights"],
            m.activation.MoEActivation.SILU, cfg.E, None, d["w13_q"], d["w13_f"], d["w2_q"],
            d["w2_f"], torch.empty(R, max(2 * cfg.N, cfg.K), dtype=dt, device=DEV),
            torch.empty(R, max(cfg.N, cfg.K), dtype=dt, device=DEV), cfg.quant_block, cfg.sg,
            cfg.q_max, _trace=tr)
        torch.cuda.synchronize()
    finally:
        r._USE_FUSED_W13_EPILOGUE = True
    return d, tr, out


def _ref_hybrid(refops, tm, bias, a, qa, fa, b, qb, fb, eo, ps, out, cfg, so):
    op = {(128, False): refops.hybrid, (128, True): refops.hybrid_bias,
          (64, False): refops.hybrid_small, (64, True): refops.hybrid_small_bias}[(tm, bias is not None)]
    if bias is None:
        op(a, qa, fa, b, qb, fb, eo, ps, out, cfg.quant_block, cfg.sg, so)
    else:
        op(a, qa, fa, b, qb, fb, eo, ps, out, bias, cfg.quant_block, cfg.sg, so)


GEMM_CASES = ["tiny", "ragged", "mid", "decode", "default"]


@pytest.mark.parametrize("name", GEMM_CASES)
def test_hybrid_gemm_matches_reference_cuda(m, refops, name):
    """mm1 and mm2 of this library's forward against the reference CUTLASS
    kernel run on the same INT8 activations, Q/F scales and offsets."""
    cfg, inp = inputs(name)
    d, tr, _ = _gemm_case(m, cfg, inp)
    E = cfg.E
    tm = tr["tile_m"]
    v = int(tr["eft"][-1])
    R = tr["a1q"].shape[0]
    so1 = tr["a1_so"][:E].contiguous()
    so2 = tr["a2_so"][:E].contiguous()
    mm1 = torch.zeros(R, 2 * cfg.N, dtype=torch.bfloat16, device=DEV)
    _ref_hybrid(refops, tm, None, tr["a1q"], tr["a1_Q"], tr["a1_F"], d["w13"], d["w13_q"],
                d["w13_f"], tr["expert_offsets"], tr["problem_sizes1"], mm1, cfg, so1)
    mm2 = torch.zeros(R, cfg.K, dtype=torch.bfloat16, device=DEV)
    _ref_hybrid(refops, tm, None, tr["a2q"], tr["a2_Q"], tr["a2_F"], d["w2"], d["w2_q"],
                d["w2_f"], tr["expert_offsets"], tr["problem_sizes2"], mm2, cfg, so2)
    torch.cuda.synchronize()
    assert torch.equal(tr["mm1"][:v].view(torch.int16), mm1[:v].view(torch.int16)), "mm1"
    assert torch.equal(tr["mm2"][:v].view(torch.int16), mm2[:v].view(torch.int16)), "mm2"


@pytest.mark.parametrize("name,per_expert", [("tiny", False), ("mid", True), ("ragged", True)])
def test_hybrid_gemm_bias_matches_reference_cuda(m, refops, name, per_expert):
    cfg, inp = inputs(name)
    d, tr, _ = _gemm_case(m, cfg, inp)
    E, N2 = cfg.E, 2 * cfg.N
    g = torch.Generator().manual_seed(11)
    shape = (E, N2) if per_expert else (N2,)
    bias = (torch.randn(*shape, generator=g) * 3.0).to(DEV)
    tm = tr["tile_m"]
    v = int(tr["eft"][-1])
    R = tr["a1q"].shape[0]
    so1 = tr["a1_so"][:E].contiguous()
    args = (tr["a1q"], tr["a1_Q"], tr["a1_F"], d["w13"], d["w13_q"], d["w13_f"],
            tr["expert_offsets"], tr["problem_sizes1"])
    ref_out = torch.zeros(R, N2, dtype=torch.bfloat16, device=DEV)
    _ref_hybrid(refops, tm, bias, *args, ref_out, cfg, so1)
    out = torch.zeros(R, N2, dtype=torch.bfloat16, device=DEV)
    gemm = m.ops.cutlass_int8_blockwise_hybrid_grouped_bias if tm == 128 else \
        m.ops.cutlass_int8_blockwise_hybrid_grouped_small_bias
    gemm(*args, out, bias, cfg.quant_block, cfg.sg, so1)
    torch.cuda.synchronize()
    assert torch.equal(out[:v].view(torch.int16), ref_out[:v].view(torch.int16))


@pytest.mark.parametrize("name", ["ragged", "mid", "default"])
def test_per_tensor_grouped_mm_matches_reference_cuda(m, refops, name):
    cfg, inp = inputs(name)
    d, tr, _ = _gemm_case(m, cfg, inp)
    E = cfg.E
    v = int(tr["eft"][-1])
    R = tr["a1q"].shape[0]
    a_s, b_s = 0.0123, 0.00077
    ref_out = torch.zeros(R, 2 * cfg.N, dtype=torch.bfloat16, device=DEV)
    refops.grouped_mm(tr["a1q"], d["w13"], ref_out, a_s, b_s, tr["expert_offsets"],
                      tr["problem_sizes1"])
    out = torch.zeros(R, 2 * cfg.N, dtype=torch.bfloat16, device=DEV)
    m.ops.cutlass_int8_grouped_mm(tr["a1q"], d["w13"], out, a_s, b_s, tr["expert_offsets"],
                                  tr["problem_sizes1"])
    torch.cuda.synchronize()
    assert torch.equal(out[:v].view(torch.int16), ref_out[:v].view(torch.int16))


@pytest.mark.parametrize("name,ep", [("tiny", None), ("ragged", None), ("mid", None),
                                     ("default", None), ("mid", (1, 4))])
def test_unpermute_matches_reference_cuda(m, refops, name, ep):
    """The top-k weighted unpermute of the forward's own mm2 rows, with the
    EP skip of rows past the local experts' offsets."""
    cfg, inp = inputs(name)
    ids = inp["topk_ids"].to(DEV)
    T, k = ids.shape
    R = T * k
    emap, n_local = (None, cfg.E) if ep is None else ep_map(cfg.E, *ep)
    eft, inv, _ = ref_metadata(refops, ids, cfg.E, n_local, emap)
    g = torch.Generator().manual_seed(5)
    rows = torch.randn(R, cfg.K, generator=g).to(torch.bfloat16).to(DEV)
    w = inp["topk_weights"].to(DEV)
    ref_out = torch.zeros(T, cfg.K, dtype=torch.bfloat16, device=DEV)
    refops.unpermute(rows, w, inv.view(T, k), eft, k, ref_out)
    out = torch.zeros(T, cfg.K, dtype=torch.bfloat16, device=DEV)
    m.permute.moe_unpermute(out, rows, w, inv, eft)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16))
