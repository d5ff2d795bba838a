"""The CPU oracle against golden vectors produced by the reference's own
Python/Triton code (tests/golden/make_golden.py)."""

import numpy as np
import pytest

from oracle import ref_cpu as ref
from tests.conftest import GOLDEN

FWD = ["fwd_tiny", "fwd_tiny_unfused", "fwd_ragged", "fwd_tm128", "fwd_tiny_ep1of2"]


def _load(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def _cfg_inputs(name):
    from tests.helpers import load_workloads
    wl = load_workloads()
    cfg = {"fwd_tiny": "tiny", "fwd_tiny_unfused": "tiny", "fwd_ragged": "ragged",
           "fwd_tm128": "tm128", "fwd_tiny_ep1of2": "tiny"}[name]
    c = wl.CONFIGS[cfg]
    return c, wl.make_inputs(c)


@pytest.mark.parametrize("name", FWD)
def test_forward_matches_reference_runner(name):
    g = _load(name)
    cfg, inp = _cfg_inputs(name)
    np_in = {k: (v.float().numpy() if v.is_floating_point() else v.numpy()) for k, v in inp.items()}
    emap = g.get("expert_map")
    w13, w2 = np_in["w13"], np_in["w2"]
    q13, f13, q2, f2 = np_in["w13_q"], np_in["w13_f"], np_in["w2_q"], np_in["w2_f"]
    if emap is not None:
        local = np.nonzero(emap >= 0)[0]
        sl = slice(int(local[0]), int(local[-1]) + 1)
        w13, w2, q13, f13, q2, f2 = (x[sl] for x in (w13, w2, q13, f13, q2, f2))
    tr = ref.moe_forward(np_in["hidden"], w13, w2, np_in["topk_ids"], np_in["topk_weights"],
                         q13, f13, q2, f2, dtype=cfg.dtype, global_num_experts=cfg.E,
                         expert_map=emap, super_group_size=cfg.sg, q_max=cfg.q_max,
                         fuse_permute=name != "fwd_tiny_unfused",
                         fuse_silu=name != "fwd_tiny_unfused", trace=True)
    v = int(g["valid"])
    rows = g["a1_Q"].shape[0]
    assert tr.tile_m == int(g["tile_m"])
    np.testing.assert_array_equal(tr.offsets, g["eft"])
    np.testing.assert_array_equal(tr.inv, g["inv"])
    np.testing.assert_array_equal(tr.permuted_idx, g["pidx"])
    np.testing.assert_array_equal(tr.a1q[:v], g["a1q"])
    np.testing.assert_array_equal(tr.a1_Q[:rows], g["a1_Q"])
    np.testing.assert_array_equal(tr.a1_F[:rows], g["a1_F"])
    np.testing.assert_array_equal(tr.a1_so[:-1], g["a1_so"])
    np.testing.assert_array_equal(tr.w1_acc[:v], g["w1_acc"])
    np.testing.assert_array_equal(tr.mm1[:v], g["mm1"])
    np.testing.assert_array_equal(tr.a2q[:v], g["a2q"])
    np.testing.assert_array_equal(tr.a2_Q[:rows], g["a2_Q"])
    np.testing.assert_array_equal(tr.a2_F[:rows], g["a2_F"])
    np.testing.assert_array_equal(tr.mm2[:v], g["mm2"])
    np.testing.assert_array_equal(tr.out, g["out"])


@pytest.mark.parametrize("name", ["gq_fp32_tm64", "gq_fp16_tm128", "gq_bf16_tm64_ktail"])
def test_grouped_quant_matches_reference_triton(name):
    g = _load(name)
    qA, scale, so = ref.grouped_blockwise_quant(g["A"], g["eo"], int(g["tile_m"]))
    Q, F = ref.quantize_scales_for_hybrid(scale, 16, 2)
    covered = np.zeros(g["A"].shape[0], bool)
    eo = g["eo"]
    covered[int(eo[0]):int(eo[-1])] = True
    np.testing.assert_array_equal(qA[covered], g["qA"][covered])
    np.testing.assert_array_equal(Q, g["Q"])
    np.testing.assert_array_equal(F, g["F"])
    np.testing.assert_array_equal(so[:-1], g["so"])


@pytest.mark.parametrize("name", ["sq_fp16_tm64", "sq_bf16_tm128"])
def test_silu_quant_matches_reference_triton(name):
    g = _load(name)
    qA, scale, so = ref.fused_silu_quant(g["X"], g["eo"], int(g["tile_m"]), str(g["dtype"]))
    Q, F = ref.quantize_scales_for_hybrid(scale, 16, 256)
    np.testing.assert_array_equal(qA, g["qA"])
    np.testing.assert_array_equal(Q, g["Q"])
    np.testing.assert_array_equal(F, g["F"])


def test_scale_factorisation_matches_reference_triton():
    g = _load("scales_sg3")
    Q, F = ref.quantize_scales_for_hybrid(g["s"], 16, 3)
    np.testing.assert_array_equal(Q, g["Q"])
    np.testing.assert_array_equal(F, g["F"])


@pytest.mark.parametrize("name", ["wq_bf16_ragged", "wq_bf16_even"])
def test_weight_quant_matches_reference_function(name):
    """The weight preparation restated in the oracle equals the reference's own
    _quantize_blockwise_int8 + quantize_scales_for_hybrid outputs."""
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    q, s = ref.quantize_weights_blockwise(g["w"], 64, 128)
    np.testing.assert_array_equal(q, g["q"])
    np.testing.assert_array_equal(s, g["scale"])
    Q, F = ref.quantize_scales_for_hybrid(s.reshape(-1, s.shape[-1]), 16, int(g["sg"]))
    np.testing.assert_array_equal(Q.reshape(g["Q"].shape), g["Q"])
    np.testing.assert_array_equal(F.reshape(g["F"].shape), g["F"])
