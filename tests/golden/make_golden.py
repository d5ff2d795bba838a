"""Generate the golden parity fixtures by running the REFERENCE's own code.

Run in the build container (it needs the reference checkout; it is never run
by the tests or on the GPU box):

    python tests/golden/make_golden.py [--ref PATH]

What runs:
  * ``int8_hybrid_moe/quant.py`` of the reference, unchanged, with its Triton
    kernels executed by Triton's CPU interpreter (``TRITON_INTERPRET=1``).
    The interpreter has no libdevice, so ``libdevice.round`` and
    ``libdevice.rint`` are supplied with their documented CUDA semantics
    (round: nearest, ties away from zero; rint: nearest, ties to even).
  * ``int8_hybrid_moe/{cutlass_runner,permute,ops,activation}.py`` of the
    reference, unchanged, as the orchestration.
  * The reference's C++/CUDA ops (``torch.ops.int8_hybrid_moe.*``: CUB
    routing, CUTLASS GEMMs, unpermute, silu_and_mul) cannot run here -- there
    is no GPU and the CUTLASS submodule is absent -- so they are registered as
    CPU ops backed by ``oracle/ref_cpu.py``.

The script re-executes itself with ``python -O`` because the reference's
host wrappers ``assert tensor.is_cuda``; with ``-O`` those asserts are
stripped and the same code runs on CPU tensors.

  * ``_quantize_blockwise_int8`` of the reference's ``bench_int8_hybrid_moe.py``
    (the weight preparation), taken out of that file with ``ast`` -- the file
    itself imports the CUDA library at module level -- and run unchanged.

Outputs ``tests/golden/*.npz``: routing maps, int8 activations, Q/F scales,
scale offsets, GEMM outputs and the final output of each case, exactly as the
reference code produced them.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import types
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent

if __debug__ and __name__ == "__main__":
    os.execv(sys.executable, [sys.executable, "-O", *sys.argv])

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton.language as tl  # noqa: E402
import triton.language.extra.cuda.libdevice as libdevice  # noqa: E402
from triton.runtime.interpreter import TensorHandle  # noqa: E402

sys.path.insert(0, str(REPO))
from oracle import ref_cpu as ref  # noqa: E402


def _load_file(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


workloads = _load_file("_workloads", REPO / "int8blockwisegemm_b200" / "workloads.py")


# ---------------------------------------------------------------------------
# libdevice for the interpreter
# ---------------------------------------------------------------------------

def _ld_round(x, _semantic=None):
    d = x.handle.data
    t = np.trunc(d)
    r = np.where(np.abs(d - t) >= 0.5, t + np.sign(d), t).astype(d.dtype)
    return tl.core.tensor(TensorHandle(r, x.handle.dtype), x.type)


def _ld_rint(x, _semantic=None):
    d = x.handle.data
    return tl.core.tensor(TensorHandle(np.rint(d).astype(d.dtype), x.handle.dtype), x.type)


libdevice.round = _ld_round
libdevice.rint = _ld_rint


# ---------------------------------------------------------------------------
# bfloat16 arithmetic for the interpreter
# ---------------------------------------------------------------------------
# The interpreter stores bf16 as raw uint16 and (a) casts fp32 -> bf16 by
# truncation and (b) applies numpy arithmetic to the raw bits.  Compiled
# Triton converts with cvt.rn (round to nearest even) and evaluates bf16
# arithmetic as the correctly rounded result of the exact operation.  These
# patches make the interpreter do the same.

from triton.runtime import interpreter as _interp  # noqa: E402


def _bf16_bits_to_f32(bits):
    return (np.asarray(bits).astype(np.uint32) << 16).view(np.float32)


def _f32_to_bf16_bits(x):
    return (ref.bf16_round(np.asarray(x, np.float32)).view(np.uint32) >> 16).astype(np.uint16)


_orig_cast = _interp.InterpreterBuilder.cast_impl
_orig_fp_to_fp = _interp.InterpreterBuilder.create_fp_to_fp
_orig_binary = _interp.InterpreterBuilder.binary_op


def _as_f32(h):
    if h.dtype.scalar == tl.bfloat16:
        return _bf16_bits_to_f32(h.data)
    return h.data.astype(np.float32)


def _cast_impl(self, src, dst_type):
    s, d = src.dtype.scalar, dst_type.scalar
    if s == tl.bfloat16 or d == tl.bfloat16:
        x = _as_f32(src) if s.is_floating() else src.data.astype(np.float32)
        if d == tl.bfloat16:
            return TensorHandle(_f32_to_bf16_bits(x), d)
        return TensorHandle(x.astype(_interp._get_np_dtype(d)), d)
    return _orig_cast(self, src, dst_type)


def _fp_to_fp(self, src, dst_type, rounding_mode):
    if src.dtype.scalar == tl.bfloat16 or dst_type.scalar == tl.bfloat16:
        return _cast_impl(self, src, dst_type)
    return _orig_fp_to_fp(self, src, dst_type, rounding_mode)


def _binary_op(self, lhs, rhs, op):
    if lhs.dtype.scalar == tl.bfloat16:
        out = op(_as_f32(lhs), _as_f32(rhs))
        if out.dtype == np.float32:
            return TensorHandle(_f32_to_bf16_bits(out), tl.bfloat16)
        return TensorHandle(out, lhs.dtype.scalar)
    return _orig_binary(self, lhs, rhs, op)


_interp.InterpreterBuilder.cast_impl = _cast_impl
_interp.InterpreterBuilder.create_fp_to_fp = _fp_to_fp
_interp.InterpreterBuilder.binary_op = _binary_op
for _n in ("create_fp_ext", "create_fp_trunc", "create_si_to_fp", "create_ui_to_fp",
           "create_fp_to_si", "create_fp_to_ui"):
    setattr(_interp.InterpreterBuilder, _n, lambda self, src, dst_type: _cast_impl(self, src,
                                                                                   dst_type))


# ---------------------------------------------------------------------------
# CPU stand-ins for the reference's compiled ops (oracle-backed)
# ---------------------------------------------------------------------------

RECORD: list = []


def _np(t: torch.Tensor) -> np.ndarray:
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.float().numpy()
    return t.numpy()


def _dtype_name(t: torch.Tensor) -> str:
    return {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}[t.dtype]


def _register_ops():
    lib = torch.library.Library("int8_hybrid_moe", "DEF")
    lib.define("cutlass_int8_blockwise_hybrid_grouped(Tensor a_q, Tensor a_qscale, "
               "Tensor a_fscale, Tensor b_q, Tensor b_qscale, Tensor b_fscale, "
               "Tensor expert_offsets, Tensor problem_sizes, Tensor(a!) out, "
               "int quant_block_size, int super_group_size, "
               "Tensor? scale_offsets=None) -> ()")
    lib.define("cutlass_int8_blockwise_hybrid_grouped_small(Tensor a_q, Tensor a_qscale, "
               "Tensor a_fscale, Tensor b_q, Tensor b_qscale, Tensor b_fscale, "
               "Tensor expert_offsets, Tensor problem_sizes, Tensor(a!) out, "
               "int quant_block_size, int super_group_size, "
               "Tensor? scale_offsets=None) -> ()")
    lib.define("moe_permute(Tensor input, Tensor topk_ids, Tensor token_expert_indices, "
               "Tensor? expert_map, int n_expert, int n_local_expert, int topk, "
               "Tensor! permuted_input, Tensor! expert_first_token_offset, "
               "Tensor! inv_permuted_idx, Tensor! permuted_idx) -> ()")
    lib.define("moe_permute_metadata(Tensor topk_ids, Tensor token_expert_indices, "
               "Tensor? expert_map, int n_expert, int n_local_expert, int topk, "
               "Tensor! expert_first_token_offset, Tensor! inv_permuted_idx, "
               "Tensor! permuted_idx) -> ()")
    lib.define("moe_unpermute(Tensor permuted_hidden_states, Tensor topk_weights, "
               "Tensor inv_permuted_idx, Tensor? expert_first_token_offset, int topk, "
               "Tensor! hidden_states) -> ()")
    lib.define("silu_and_mul(Tensor! out, Tensor input) -> ()")

    def gemm(tile_m):
        def impl(a_q, a_qs, a_fs, b_q, b_qs, b_fs, eo, ps, out, qbs, sg, so=None):
            o, w = ref.hybrid_grouped_gemm(
                a_q.numpy(), a_qs.numpy(), a_fs.numpy(), b_q.numpy(), b_qs.numpy(),
                b_fs.numpy(), eo.numpy(), ps.numpy(), qbs, tile_m,
                scale_offsets=None if so is None else so.numpy(),
                out_dtype=_dtype_name(out), return_w=True)
            eon = eo.numpy().astype(np.int64)
            rows = slice(int(eon[0]), int(eon[-1]))
            out[rows] = torch.from_numpy(o[rows]).to(out.dtype)
            RECORD.append(dict(kind="gemm", tile_m=tile_m, a_q=a_q.clone(), a_qs=a_qs.clone(),
                               a_fs=a_fs.clone(), so=None if so is None else so.clone(),
                               out=out.clone(), w=torch.from_numpy(w)))
        return impl

    def permute_meta(topk_ids, tei, emap, n_expert, n_local, topk, eft, inv, pidx):
        o, i, p = ref.moe_permute_metadata(topk_ids.numpy(), tei.numpy(),
                                           None if emap is None else emap.numpy(),
                                           n_expert, n_local, topk)
        eft.copy_(torch.from_numpy(o))
        inv.copy_(torch.from_numpy(i))
        lim = int(o[n_local]) if emap is not None else p.shape[0]
        pidx[:lim] = torch.from_numpy(p[:lim])
        RECORD.append(dict(kind="route", eft=eft.clone(), inv=inv.clone(), pidx=pidx.clone()))

    def permute(inp, topk_ids, tei, emap, n_expert, n_local, topk, pin, eft, inv, pidx):
        permute_meta(topk_ids, tei, emap, n_expert, n_local, topk, eft, inv, pidx)
        lim = int(eft[n_local]) if emap is not None else pidx.shape[0]
        src = pidx[:lim].long() // topk
        pin[:lim] = inp[src]

    def unpermute(x, w, inv, eft, topk, out):
        o = ref.moe_unpermute(_np(x), w.numpy(), inv.numpy(),
                              None if eft is None else eft.numpy(), topk, _dtype_name(out))
        out.copy_(torch.from_numpy(o).to(out.dtype))

    def silu(out, inp):
        out.copy_(torch.from_numpy(ref.silu_and_mul(_np(inp), _dtype_name(inp))).to(out.dtype))

    lib.impl("cutlass_int8_blockwise_hybrid_grouped", gemm(128), "CPU")
    lib.impl("cutlass_int8_blockwise_hybrid_grouped_small", gemm(64), "CPU")
    lib.impl("moe_permute_metadata", permute_meta, "CPU")
    lib.impl("moe_permute", permute, "CPU")
    lib.impl("moe_unpermute", unpermute, "CPU")
    lib.impl("silu_and_mul", silu, "CPU")
    return lib


def _load_reference(ref_root: Path):
    pkg_dir = ref_root / "int8_hybrid_moe"
    pkg = types.ModuleType("int8_hybrid_moe")
    pkg.__path__ = [str(pkg_dir)]
    sys.modules["int8_hybrid_moe"] = pkg
    mods = {}
    for name in ("quant", "ops", "activation", "permute", "cutlass_runner"):
        mods[name] = _load_file(f"int8_hybrid_moe.{name}", pkg_dir / f"{name}.py")
        setattr(pkg, name, mods[name])
    return mods


# ---------------------------------------------------------------------------
# cases
# ---------------------------------------------------------------------------

def run_forward(mods, cfg, fuse_permute: bool, fuse_silu: bool, ep=None):
    """Run the reference runner on ``cfg``; ``ep=(rank, size)`` uses an
    expert_map that keeps experts [rank*E/size, (rank+1)*E/size)."""
    inp = workloads.make_inputs(cfg)
    runner = mods["cutlass_runner"]
    runner._USE_FUSED_PERMUTE_QUANT_W1 = fuse_permute
    runner._USE_FUSED_SILU_QUANT_W2 = fuse_silu
    dt = workloads.TORCH_DTYPE[cfg.dtype]
    T, K, N, E, k = cfg.T, cfg.K, cfg.N, cfg.E, cfg.topk
    expert_map = None
    w13, w2 = inp["w13"], inp["w2"]
    q13, f13, q2, f2 = inp["w13_q"], inp["w13_f"], inp["w2_q"], inp["w2_f"]
    if ep is not None:
        rank, size = ep
        per = E // size
        lo, hi = rank * per, (rank + 1) * per
        expert_map = torch.full((E,), -1, dtype=torch.int32)
        expert_map[lo:hi] = torch.arange(per, dtype=torch.int32)
        w13, w2 = w13[lo:hi].contiguous(), w2[lo:hi].contiguous()
        q13, f13, q2, f2 = (x[lo:hi].contiguous() for x in (q13, f13, q2, f2))
    R = T * k
    ws13 = torch.zeros(R, max(2 * N, K), dtype=dt)
    ws2 = torch.zeros(R, max(N, K), dtype=dt)
    out = torch.zeros(T, K, dtype=dt)
    RECORD.clear()
    runner._run_cutlass_int8_hybrid_grouped_moe(
        output=out, hidden_states=inp["hidden"], w1=w13, w2=w2, topk_ids=inp["topk_ids"],
        topk_weights=inp["topk_weights"], activation=mods["activation"].MoEActivation.SILU,
        global_num_experts=E, expert_map=expert_map, w1_qscale=q13, w1_fscale=f13,
        w2_qscale=q2, w2_fscale=f2, workspace13=ws13, workspace2=ws2,
        quant_block_size=cfg.quant_block, super_group_size=cfg.sg, q_max=cfg.q_max)
    route = [r for r in RECORD if r["kind"] == "route"][0]
    g1, g2 = [r for r in RECORD if r["kind"] == "gemm"]
    eft = route["eft"].numpy()
    valid = int(eft[-1])
    tm = g1["tile_m"]
    so = ref.scale_offsets_from(eft, tm)
    rows = int(so[-1])
    res = dict(
        eft=eft, inv=route["inv"].numpy(), pidx=route["pidx"].numpy(), tile_m=np.int64(tm),
        valid=np.int64(valid),
        a1q=g1["a_q"].numpy()[:valid], a1_Q=g1["a_qs"].numpy()[:rows],
        a1_F=g1["a_fs"].numpy()[:rows], a1_so=g1["so"].numpy(),
        w1_acc=g1["w"].numpy()[:valid], mm1=_np(g1["out"])[:valid],
        a2q=g2["a_q"].numpy()[:valid], a2_Q=g2["a_qs"].numpy()[:rows],
        a2_F=g2["a_fs"].numpy()[:rows], a2_so=g2["so"].numpy(),
        mm2=_np(g2["out"])[:valid], out=_np(out),
    )
    if expert_map is not None:
        res["expert_map"] = expert_map.numpy()
    return res


def quant_cases(mods):
    """Direct calls of the reference quant entry points on edge inputs."""
    q = mods["quant"]
    g = torch.Generator().manual_seed(11)
    cases = {}
    # grouped quant: fp32 / fp16 / bf16 inputs, empty experts, K tail, both tile_m.
    for name, dt, tm, K, counts in (
        ("gq_fp32_tm64", torch.float32, 64, 384, [0, 70, 1, 0, 129, 64]),
        ("gq_fp16_tm128", torch.float16, 128, 256, [300, 0, 17, 128]),
        ("gq_bf16_tm64_ktail", torch.bfloat16, 64, 160, [5, 0, 0, 66, 31]),
    ):
        M = sum(counts)
        A = (torch.randn(M, K, generator=g) * torch.exp(torch.randn(M, 1, generator=g))).to(dt)
        if M > 3:
            A[3] = 0
        eo = torch.tensor([0, *np.cumsum(counts).tolist()], dtype=torch.int32)
        qa, Q, F, so = q.moe_kernel_quantize_input_int8_hybrid_grouped(
            A, block_k=128, q_max=16, super_group_size=2, expert_offsets=eo, tile_m=tm)
        rows = int(ref.scale_offsets_from(eo.numpy(), tm)[-1])
        cases[name] = dict(A=_np(A), dtype=np.array(_dtype_name(A)), eo=eo.numpy(),
                           tile_m=np.int64(tm), qA=qa.numpy(), Q=Q.numpy()[:rows],
                           F=F.numpy()[:rows], so=so.numpy())
    # fused SiLU + quant, fp16 and bf16 inputs.
    for name, dt, tm, N, counts in (
        ("sq_fp16_tm64", torch.float16, 64, 256, [10, 0, 90, 64]),
        ("sq_bf16_tm128", torch.bfloat16, 128, 384, [129, 3, 0, 200]),
    ):
        M = sum(counts)
        X = (torch.randn(M, 2 * N, generator=g) * 3).to(dt)
        eo = torch.tensor([0, *np.cumsum(counts).tolist()], dtype=torch.int32)
        aq, Q, F, so = q.fused_silu_quant_int8_hybrid_grouped(
            X, block_k=128, q_max=16, super_group_size=256, expert_offsets=eo, tile_m=tm)
        rows = int(ref.scale_offsets_from(eo.numpy(), tm)[-1])
        cases[name] = dict(X=_np(X), dtype=np.array(_dtype_name(X)), eo=eo.numpy(),
                           tile_m=np.int64(tm), qA=aq.numpy(), Q=Q.numpy()[:rows],
                           F=F.numpy()[:rows], so=so.numpy())
    # scale factorisation with several super-groups and a ragged last group.
    s = torch.exp(torch.randn(37, 7, generator=g) * 2).float()
    s[0, :] = 0.0
    s[1, 3] = 1e-14
    Qs, Fs = q.quantize_scales_for_hybrid(s, Q_max=16, super_group_size=3)
    cases["scales_sg3"] = dict(s=s.numpy(), Q=Qs.numpy(), F=Fs.numpy())
    return cases


def weight_quant_cases(ref_root: Path, mods):
    """The reference's weight preparation: blockwise INT8 weights
    (bench_int8_hybrid_moe.py:98-120, block 64 x quant_block) and the hybrid
    Q/F factorisation of their scales along K (:233-244)."""
    import ast
    src = (ref_root / "bench_int8_hybrid_moe.py").read_text()
    fn = next(n for n in ast.parse(src).body
              if isinstance(n, ast.FunctionDef) and n.name == "_quantize_blockwise_int8")
    ns = {"torch": torch}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), "bench_int8_hybrid_moe.py", "exec"), ns)
    qblk = ns["_quantize_blockwise_int8"]
    q = mods["quant"]
    g = torch.Generator().manual_seed(4242)
    cases = {}
    for name, (E, N, K, sg) in {"wq_bf16_ragged": (3, 136, 200, 1),
                                "wq_bf16_even": (2, 128, 512, 2)}.items():
        w = (torch.randn(E, N, K, generator=g) * 0.02).to(torch.bfloat16)
        w[1, :64, :128] = 0            # an all-zero block: the 1e-10 scale floor
        w[0, 5, 7] = 0.5               # an outlier that owns its block's absmax
        wq, scale = qblk(w, 64, 128)
        Kb = scale.shape[-1]
        Q, F = q.quantize_scales_for_hybrid(scale.reshape(-1, Kb).contiguous(), Q_max=16,
                                            super_group_size=sg)
        cases[name] = dict(w=_np(w), sg=np.int64(sg), q=wq.numpy(), scale=scale.numpy(),
                           Q=Q.numpy().reshape(E, -1, Kb), F=F.numpy().reshape(E, -1, F.shape[-1]))
    return cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("INT8_HYBRID_MOE_REFERENCE_SRC"),
                    required="INT8_HYBRID_MOE_REFERENCE_SRC" not in os.environ,
                    help="the reference's source tree (its int8_hybrid_moe package and "
                         "benchmark script)")
    ap.add_argument("--only", choices=["all", "weights"], default="all")
    args = ap.parse_args()
    mods = _load_reference(Path(args.ref))
    _keep = _register_ops()  # noqa: F841
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    if args.only == "weights":
        for name, d in weight_quant_cases(Path(args.ref), mods).items():
            np.savez_compressed(HERE / f"{name}.npz", **d)
            print("wrote", name, {k: getattr(v, "shape", None) for k, v in d.items()})
        return
    C = workloads.CONFIGS
    fwd = {
        "fwd_tiny": run_forward(mods, C["tiny"], True, True),
        "fwd_tiny_unfused": run_forward(mods, C["tiny"], False, False),
        "fwd_ragged": run_forward(mods, C["ragged"], True, True),
        "fwd_tm128": run_forward(mods, C["tm128"], True, True),
        "fwd_tiny_ep1of2": run_forward(mods, C["tiny"], True, True, ep=(1, 2)),
    }
    for name, d in {**fwd, **quant_cases(mods), **weight_quant_cases(Path(args.ref), mods)}.items():
        np.savez_compressed(HERE / f"{name}.npz", **d)
        print("wrote", name, {k: getattr(v, "shape", None) for k, v in d.items()})


if __name__ == "__main__":
    main()
