"""Build the reference's own GPU path of the blockwise-FP8 linear into ``oracle/_ref/``.

TEST INFRASTRUCTURE ONLY: the results are a checker and a timed comparator for
``tests/`` and ``bench.py``; the product path (``ltx-2_b200/``) never loads them.

What is built, from the reference checkout where its files lie (nothing is copied
into the repository; ``oracle/_ref/`` is git-ignored and travels to the GPU box as a
build product):

* ``oracle/_ref/blockwise/ref_blockwise_cpp*.so`` -- ``ltx-kernels/csrc/blockwise/
  api.cpp`` + ``kernels/geforce/gemm.cu``: the SM89 ``mma.sync`` CuTe GEMM that the
  reference dispatches on Blackwell (``ltx_kernels/blockwise/linear.py:25-35``), with
  the nvcc flags of the reference's ``setup.py`` (blockwise_nvcc) and
  ``-gencode arch=compute_100a,code=sm_100a``.  The pinned CUTLASS v3.8.0
  (``setup.py``, CUTLASS_REF) is not available offline; the CUTLASS headers vendored
  in site-packages (flashinfer's copy) are used instead.  Two of their headers,
  ``cute/arch/mma_sm89.hpp`` and ``cute/atom/mma_traits_sm89.hpp``, are shadowed by
  empty files in an include overlay: the reference defines its own SM89 atoms
  (``kernels/geforce/mma_sm89_fp16.hpp``) and the newer CUTLASS's copies collide.
* ``oracle/_ref/ops/ref_ops_cpp*.so`` -- ``ltx-kernels/csrc/ops/*``: the q/k RMSNorm +
  RoPE kernels and the FP6 pack/unpack, with the reference's ops_cpp flags
  (``--use_fast_math`` included).
* ``oracle/_ref/py/ltx_kernels/`` -- byte copies of the reference's Python package
  files on the path (``__init__.py``, ``arch.py``, ``all_to_all.py`` and
  ``blockwise/{__init__,triton_ops,functional,linear}.py``) so the GPU box (which has
  no reference checkout) can run the reference's Triton quantiser, torch functions
  and linear module; ``oracle/refpath.py`` loads them.

Usage:  python oracle/build_ref.py [REFERENCE_ROOT] [--force]
``__graft_entry__.build()`` calls this when the reference checkout is present.
"""
from __future__ import annotations

import glob
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
DEFAULT_REF = os.environ.get("LTX2_REFERENCE", "/root/reference")


def _kernels_root(ref_root: str) -> str:
    return os.path.join(ref_root, "packages", "ltx-kernels")


def cutlass_include() -> str:
    """The CUTLASS/CuTe header tree vendored with flashinfer (site-packages)."""
    import flashinfer  # noqa: PLC0415  (only its data directory is used)

    inc = os.path.join(os.path.dirname(flashinfer.__file__), "data", "cutlass", "include")
    if not os.path.exists(os.path.join(inc, "cutlass", "cutlass.h")):
        raise FileNotFoundError(f"no CUTLASS headers at {inc}")
    return inc


def _overlay() -> str:
    """Empty stand-ins for the two CUTLASS SM89 headers the reference redefines."""
    root = os.path.join(OUT, "overlay")
    for rel in ("cute/arch/mma_sm89.hpp", "cute/atom/mma_traits_sm89.hpp"):
        p = os.path.join(root, rel)
        os.makedirs(os.path.dirname(p), exist_ok=True)
        if not os.path.exists(p):
            with open(p, "w") as f:
                f.write("// Shadowed: the reference defines its own SM89 MMA atoms.\n#pragma once\n")
    return root


_HALF_FLAGS = ["-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
               "-U__CUDA_NO_HALF2_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__"]
_GENCODE = ["-gencode=arch=compute_100a,code=sm_100a"]


def _built(dirname: str, name: str) -> str | None:
    hits = glob.glob(os.path.join(OUT, dirname, name + "*.so"))
    return hits[0] if hits else None


def build_gemm(ref_root: str, force: bool = False, verbose: bool = False) -> str:
    from torch.utils.cpp_extension import load  # noqa: PLC0415

    name = "ref_blockwise_cpp"
    if not force and _built("blockwise", name):
        return _built("blockwise", name)
    kr = _kernels_root(ref_root)
    src = os.path.join(kr, "csrc", "blockwise")
    bdir = os.path.join(OUT, "blockwise")
    os.makedirs(bdir, exist_ok=True)
    import torch  # noqa: PLC0415

    abi = f"-D_GLIBCXX_USE_CXX11_ABI={int(torch.compiled_with_cxx11_abi())}"
    load(name=name,
         sources=[os.path.join(src, "api.cpp"), os.path.join(src, "kernels", "geforce", "gemm.cu")],
         extra_include_paths=[_overlay(), src, os.path.join(src, "kernels", "deep_gemm", "include"),
                              cutlass_include(), "/usr/local/cuda/include"],
         extra_cflags=["-O3", "-std=c++17", "-fPIC", "-Wno-psabi", "-Wno-deprecated-declarations", abi],
         extra_cuda_cflags=["-O3", "-std=c++17", "--ptxas-options=-O2", "--expt-relaxed-constexpr",
                            "--expt-extended-lambda", *_HALF_FLAGS, "-DCCCL_DISABLE_CTK_COMPATIBILITY_CHECK",
                            *_GENCODE],
         extra_ldflags=["-lcuda", "-L/usr/local/cuda/lib64/stubs"],
         build_directory=bdir, verbose=verbose, is_python_module=True)
    return _built("blockwise", name)


def build_ops(ref_root: str, force: bool = False, verbose: bool = False) -> str:
    from torch.utils.cpp_extension import load  # noqa: PLC0415

    name = "ref_ops_cpp"
    if not force and _built("ops", name):
        return _built("ops", name)
    src = os.path.join(_kernels_root(ref_root), "csrc", "ops")
    bdir = os.path.join(OUT, "ops")
    os.makedirs(bdir, exist_ok=True)
    files = ["ops_api.cpp", "fp6_bitpack.cpp", "fp6_pack.cu", "rms_norm_rope.cpp", "rms_norm_rope_cuda.cu",
             "rms_norm_split_rope.cpp", "rms_norm_split_rope_cuda.cu"]
    load(name=name, sources=[os.path.join(src, f) for f in files],
         extra_include_paths=[os.path.join(src, "include")],
         extra_cflags=["-O3", "-std=c++17"],
         extra_cuda_cflags=["-O3", "-std=c++17", *_HALF_FLAGS, "--expt-relaxed-constexpr", "--expt-extended-lambda",
                            "--use_fast_math", "-DCCCL_DISABLE_CTK_COMPATIBILITY_CHECK", *_GENCODE],
         build_directory=bdir, verbose=verbose, is_python_module=True)
    return _built("ops", name)


_PY_FILES = ("__init__.py", "arch.py", "all_to_all.py", "blockwise/__init__.py", "blockwise/triton_ops.py",
             "blockwise/functional.py", "blockwise/linear.py")


def copy_python(ref_root: str) -> str:
    src = os.path.join(_kernels_root(ref_root), "src", "ltx_kernels")
    dst = os.path.join(OUT, "py", "ltx_kernels")
    for f in _PY_FILES:
        os.makedirs(os.path.dirname(os.path.join(dst, f)), exist_ok=True)
        shutil.copyfile(os.path.join(src, f), os.path.join(dst, f))
    return os.path.dirname(dst)


def build(ref_root: str = DEFAULT_REF, force: bool = False, verbose: bool = False) -> dict:
    if not os.path.isdir(_kernels_root(ref_root)):
        raise FileNotFoundError(f"no reference checkout at {ref_root}")
    os.makedirs(OUT, exist_ok=True)
    out = {"py": copy_python(ref_root)}
    out["gemm"] = build_gemm(ref_root, force, verbose)
    out["ops"] = build_ops(ref_root, force, verbose)
    return out


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    print(build(args[0] if args else DEFAULT_REF, force="--force" in sys.argv, verbose="--verbose" in sys.argv))
