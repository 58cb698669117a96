"""Token sharding of the blockwise-FP8 linears across GPUs of one node.

The linears are row-independent in the token dimension, so every rank runs them
on its own slice of the sequence with replicated FP8 weights and no collective
on the data path.  This mirrors the token partition of the reference's sequence
parallelism (ltx-core/src/ltx_core/multigpu/transformer/sequence_parallel.py):

* ``pad_for_uniform_sharding`` -- zero-pad the sequence to a multiple of the
  world size (``pad_modality_for_uniform_sharding``, sequence_parallel.py:53-100).
  Padded tokens quantise to NaN codes with scale 0, exactly as in the
  reference; their outputs are dropped after the gather.
* ``compute_sequence_partition`` / ``shard_tokens`` -- equal contiguous slices of
  the sequence dimension per rank (sequence_parallel.py:31-49, 158-182).
* ``gather_output_tokens`` -- all-gather of the per-rank outputs along the
  sequence dimension (sequence_parallel.py:185-224), only where a full tensor
  is needed on every rank.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist


def compute_sequence_partition(total_tokens: int, world_size: int) -> List[int]:
    """Uniform per-rank token counts; ``total_tokens`` must divide evenly."""
    if world_size < 1:
        raise ValueError("world_size must be >= 1")
    if total_tokens % world_size != 0:
        raise ValueError(f"total_tokens ({total_tokens}) must be divisible by world_size ({world_size}); "
                         "pad the sequence first")
    return [total_tokens // world_size] * world_size


def compute_sequence_offsets(counts: List[int]) -> List[int]:
    offs, acc = [], 0
    for c in counts:
        offs.append(acc)
        acc += c
    return offs


def pad_for_uniform_sharding(x: torch.Tensor, world_size: int, dim: int = 1) -> Tuple[torch.Tensor, int]:
    """Zero-pad ``x`` along ``dim`` to a multiple of ``world_size``; returns (padded, original length)."""
    t = x.shape[dim]
    pad = (-t) % world_size
    if pad == 0:
        return x, t
    shape = list(x.shape)
    shape[dim] = pad
    return torch.cat([x, torch.zeros(shape, dtype=x.dtype, device=x.device)], dim=dim), t


def shard_tokens(x: torch.Tensor, world_size: int, rank: int, dim: int = 1) -> Tuple[torch.Tensor, List[int]]:
    """This rank's slice of the (already padded) sequence dimension, and all ranks' counts."""
    counts = compute_sequence_partition(x.shape[dim], world_size)
    start = compute_sequence_offsets(counts)[rank]
    return x.narrow(dim, start, counts[rank]), counts


def gather_output_tokens(local: torch.Tensor, counts: List[int], group: Optional[dist.ProcessGroup] = None,
                         dim: int = 1) -> torch.Tensor:
    """All-gather per-rank outputs along ``dim`` (uniform counts, so no re-padding is needed)."""
    if len(set(counts)) != 1:
        raise ValueError("gather_output_tokens expects uniform per-rank counts")
    parts = [torch.empty_like(local) for _ in counts]
    dist.all_gather(parts, local.contiguous(), group=group)
    return torch.cat(parts, dim=dim)


def unpad(x: torch.Tensor, original_len: int, dim: int = 1) -> torch.Tensor:
    return x.narrow(dim, 0, original_len)
