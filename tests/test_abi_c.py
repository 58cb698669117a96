"""The C ABI from C: tests/abi_c/consumer.c includes include/ltxfp8.h, links
libltxfp8.so with gcc and calls the entry points that need no GPU."""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

from conftest import REPO


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_c_consumer_builds_links_and_runs(tmp_path):
    from ltx_kernels import _lib
    _lib.load()  # builds nothing; makes sure the library exists
    libdir = os.path.dirname(_lib.LIB_PATH)
    exe = tmp_path / "consumer"
    subprocess.check_call(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(REPO, "include"),
                           os.path.join(REPO, "tests", "abi_c", "consumer.c"), "-o", str(exe),
                           "-L", libdir, "-lltxfp8", f"-Wl,-rpath,{libdir}"])
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    assert "abi_c ok" in out.stdout
