"""Compile the reference's own CUDA kernels into oracle/_ref/ (test checker).

    python oracle/build_ref.py [--reference DIR] [--force] [--verbose]

What it builds: the reference's INT8 hybrid grouped GEMM
(csrc/int8_hybrid_grouped_gemm.cu), its per-tensor grouped GEMM
(csrc/int8_grouped_gemm.cu) and its permute / unpermute ops
(csrc/moe_permute_unpermute_op.cu,
csrc/permute_unpermute_kernels/moe_permute_unpermute_kernel.cu), compiled
from the reference source tree where it lies, plus oracle/ref_bindings.cpp,
which registers them under torch.ops.int8_hybrid_moe_ref (the reference's own
csrc/torch_bindings.cpp would claim the product's namespace).  The result is
oracle/_ref/libi8moe_ref.so, loaded only by the parity tests.

How: nvcc directly on those files (no CMake), with the reference's flags
(--use_fast_math, C++17; CMakeLists.txt:73-85), torch's headers, and the
CUTLASS 2.x headers that ship inside this image (flashinfer's vendored
CUTLASS, version 4.5.0; the reference pins the CUTLASS v4.4.2 submodule,
which is not checked out).  The reference's SM80 kernels (mma.sync s8,
cp.async) are compiled unchanged for sm_100a, the B200 target; its
activation kernels are left out (not on the checked path).

The output goes to oracle/_ref/ only; the reference tree is never written.
When the reference tree is absent (the GPU box), nothing is built and the
prebuilt library, if any, is used as is.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
LIB = OUT / "libi8moe_ref.so"
DEFAULT_REF = Path(os.environ.get("I8MOE_REFERENCE_DIR", "/root/reference"))

REF_SOURCES = [
    "csrc/int8_hybrid_grouped_gemm.cu",
    "csrc/int8_grouped_gemm.cu",
    "csrc/moe_permute_unpermute_op.cu",
    "csrc/permute_unpermute_kernels/moe_permute_unpermute_kernel.cu",
]


def _cutlass_include() -> Path | None:
    try:
        import flashinfer  # noqa: F401  (only to locate its data directory)
    except Exception:
        return None
    import flashinfer as fi
    p = Path(fi.__file__).resolve().parent / "data" / "cutlass" / "include"
    return p if (p / "cutlass" / "cutlass.h").exists() else None


def _torch_flags() -> tuple[list[str], list[str]]:
    import torch
    tdir = Path(torch.__file__).resolve().parent
    inc = [tdir / "include", tdir / "include" / "torch" / "csrc" / "api" / "include",
           Path(sysconfig.get_paths()["include"])]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cflags = [f"-I{p}" for p in inc] + [f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
                                        "-DTORCH_EXTENSION_NAME=i8moe_ref",
                                        "-DTORCH_API_INCLUDE_EXTENSION_H"]
    ldflags = [f"-L{tdir / 'lib'}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
               "-ltorch_cuda", "-Xlinker", f"-rpath,{tdir / 'lib'}"]
    return cflags, ldflags


def _nvcc() -> str:
    return os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


def build(reference: Path = DEFAULT_REF, force: bool = False, verbose: bool = False) -> Path | None:
    """Builds oracle/_ref/libi8moe_ref.so; returns its path, or None when the
    reference tree or the CUTLASS headers are not available here."""
    if not (reference / REF_SOURCES[0]).exists():
        return LIB if LIB.exists() else None
    cutlass = _cutlass_include()
    if cutlass is None:
        return LIB if LIB.exists() else None
    srcs = [reference / s for s in REF_SOURCES] + [HERE / "ref_bindings.cpp"]
    newest_src = max(s.stat().st_mtime for s in srcs)
    if not force and LIB.exists() and LIB.stat().st_mtime >= newest_src:
        return LIB
    OUT.mkdir(exist_ok=True)
    cflags, ldflags = _torch_flags()
    common = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "--expt-extended-lambda", "-DNDEBUG",
              f"-I{reference / 'include'}", f"-I{reference / 'csrc'}", f"-I{cutlass}", *cflags]
    arch = ["-gencode", "arch=compute_100a,code=sm_100a"]

    def compile_one(src: Path) -> Path:
        obj = OUT / (src.name.replace(".", "_") + ".o")
        if obj.exists() and obj.stat().st_mtime >= src.stat().st_mtime and not force:
            return obj
        if src.suffix == ".cu":
            cmd = [_nvcc(), *arch, *common, "--use_fast_math", "-c", str(src), "-o", str(obj)]
        else:
            cmd = [_nvcc(), *common, "-x", "c++", "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout[-4000:]}\n{res.stderr[-4000:]}")
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, srcs))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), *arch, "-shared", "-o", str(tmp), *map(str, objs), *ldflags]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    for o in objs:
        o.unlink()
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=DEFAULT_REF)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(a.reference, a.force, a.verbose))


if __name__ == "__main__":
    sys.exit(main())
