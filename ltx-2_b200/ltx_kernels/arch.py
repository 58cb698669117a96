"""GPU architecture probe (mirrors ltx-kernels/src/ltx_kernels/arch.py:10-31)."""
from __future__ import annotations

import functools

import torch


@functools.lru_cache(maxsize=8)
def _arch_for_device(device_index: int) -> str:
    major, minor = torch.cuda.get_device_capability(device_index)
    if major == 8 and minor < 9:
        return "ampere"
    if major == 8 and minor == 9:
        return "ada"
    if major == 9 and minor == 0:
        return "hopper"
    if major in {10, 12}:
        return "blackwell"
    raise NotImplementedError(f"Unsupported GPU compute capability sm_{major}{minor}.")


def get_device_arch() -> str:
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is not available; blockwise kernels require a CUDA device.")
    return _arch_for_device(torch.cuda.current_device())
