"""The reference's own implementation of the path, loaded from ``oracle/_ref/``.

TEST INFRASTRUCTURE ONLY: ``tests/`` use it as a checker and ``bench.py`` times it
beside the product; the product path (``ltx-2_b200/``) never imports it.

``oracle/build_ref.py`` builds these from the reference checkout:

* ``gemm()``        -- the compiled ``blockwise_cpp`` module of the reference (its
                       ``fp8_gemm_nt_sm89``, ``ltx-kernels/csrc/blockwise/api.cpp:42-81``).
* ``ops()``         -- the compiled ``ops_cpp`` module (``rms_norm_rope``,
                       ``rms_norm_split_rope``, ``fp6_pack``, ``fp6_unpack``;
                       ``ltx-kernels/csrc/ops/ops_api.cpp``).
* ``triton_ops()``  -- ``ltx_kernels/blockwise/triton_ops.py`` as written.
* ``functional()``  -- ``ltx_kernels/blockwise/functional.py`` as written.

The package under test registers torch ops with the reference's names
(``blockwise::quantize``, ``q8_kernels_ops::rms_norm_rope``, ...), so the reference
modules are executed with ``torch.library.triton_op`` / ``custom_op`` /
``register_fake`` / ``wrap_triton`` replaced by pass-through decorators: their
functions become plain Python callables that launch the same Triton kernels and
call the same compiled functions, without registering anything.
"""
from __future__ import annotations

import contextlib
import glob
import importlib.machinery
import importlib.util
import os
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

_cache: dict = {}


def _so(sub: str, name: str) -> str | None:
    hits = glob.glob(os.path.join(REF_DIR, sub, name + "*.so"))
    return hits[0] if hits else None


PY_ROOT = os.path.join(REF_DIR, "py")  # holds the reference's ltx_kernels package files
_BLOCKWISE_PY = os.path.join(PY_ROOT, "ltx_kernels", "blockwise")


def available(part: str = "all") -> bool:
    """Whether the built reference artefacts are present (``gemm``, ``ops``, ``py`` or ``all``)."""
    have = {"gemm": _so("blockwise", "ref_blockwise_cpp") is not None,
            "ops": _so("ops", "ref_ops_cpp") is not None,
            "py": os.path.exists(os.path.join(_BLOCKWISE_PY, "triton_ops.py"))}
    return all(have.values()) if part == "all" else have[part]


def _load_ext(sub: str, name: str):
    if name in _cache:
        return _cache[name]
    path = _so(sub, name)
    if path is None:
        raise ImportError(f"{name} is not built; run oracle/build_ref.py with the reference checkout")
    import torch  # noqa: F401,PLC0415  (the extension links against torch's libraries)

    loader = importlib.machinery.ExtensionFileLoader(name, path)
    spec = importlib.util.spec_from_file_location(name, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    _cache[name] = mod
    return mod


def gemm():
    return _load_ext("blockwise", "ref_blockwise_cpp")


def ops():
    return _load_ext("ops", "ref_ops_cpp")


@contextlib.contextmanager
def _no_registration():
    import torch.library as tl  # noqa: PLC0415

    def passthrough(*_a, **_k):
        return lambda f: f

    saved = {k: getattr(tl, k) for k in ("triton_op", "custom_op", "register_fake", "wrap_triton")}
    tl.triton_op = passthrough
    tl.custom_op = passthrough
    tl.register_fake = passthrough
    tl.wrap_triton = lambda k: k
    try:
        yield
    finally:
        for k, v in saved.items():
            setattr(tl, k, v)


def _exec_py(modname: str, fname: str, extra_modules: dict | None = None):
    path = os.path.join(_BLOCKWISE_PY, fname)
    if not os.path.exists(path):
        raise ImportError(f"{fname} is not built; run oracle/build_ref.py with the reference checkout")
    spec = importlib.util.spec_from_file_location(modname, path)
    mod = importlib.util.module_from_spec(spec)
    saved = {}
    for k, v in (extra_modules or {}).items():
        saved[k] = sys.modules.get(k)
        sys.modules[k] = v
    try:
        with _no_registration():
            spec.loader.exec_module(mod)
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
    return mod


def triton_ops():
    """The reference's Triton kernels and their host wrappers (triton_ops.py)."""
    if "triton_ops" not in _cache:
        _cache["triton_ops"] = _exec_py("ltxref_triton_ops", "triton_ops.py")
    return _cache["triton_ops"]


def functional(with_cuda_ops: bool = True):
    """The reference's functional.py; ``ops_cpp`` is the built extension, or a stub
    without its functions when ``with_cuda_ops`` is false (the CPU functions
    ``blockwise_quantize_torch`` / ``blockwise_quantize_weights`` need none)."""
    key = f"functional:{with_cuda_ops}"
    if key in _cache:
        return _cache[key]
    if with_cuda_ops:
        ops_mod = ops()
    else:
        ops_mod = types.ModuleType("ops_cpp")
        for a in ("fp6_pack", "fp6_unpack", "rms_norm_rope", "rms_norm_split_rope"):
            setattr(ops_mod, a, None)
    mod = _exec_py("ltxref_functional", "functional.py",
                   {"ops_cpp": ops_mod, "ltx_kernels.blockwise.triton_ops": triton_ops()})
    _cache[key] = mod
    return mod
