"""Multi-process token sharding on CPU (gloo, world size 2): the host-side logic of
the N-GPU path.  The per-rank linear is the oracle's dequantise-matmul restatement
here (no GPU); on the GPU box the same shards go through the CUDA kernels."""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG, REPO


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_partition_and_padding():
    from ltx_kernels.blockwise.sharding import (compute_sequence_offsets, compute_sequence_partition,
                                                pad_for_uniform_sharding, shard_tokens, unpad)
    assert compute_sequence_partition(12, 4) == [3, 3, 3, 3]
    with pytest.raises(ValueError):
        compute_sequence_partition(10, 4)
    x = torch.arange(2 * 10 * 3, dtype=torch.float32).view(2, 10, 3)
    xp, t = pad_for_uniform_sharding(x, 4)
    assert xp.shape == (2, 12, 3) and t == 10 and torch.all(xp[:, 10:] == 0)
    pieces = [shard_tokens(xp, 4, r)[0] for r in range(4)]
    assert torch.equal(torch.cat(pieces, dim=1), xp)
    assert compute_sequence_offsets([3, 3, 3, 3]) == [0, 3, 6, 9]
    assert torch.equal(unpad(xp, t), x)
    same, t2 = pad_for_uniform_sharding(x[:, :8], 4)
    assert same.shape[1] == 8 and t2 == 8


def _worker(rank: int, world: int, port: int, out_dir: str):
    sys.path[:0] = [PKG, REPO]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O
        from ltx_kernels.blockwise.sharding import gather_output_tokens, pad_for_uniform_sharding, shard_tokens, unpad
        g = torch.Generator().manual_seed(0)
        B, T, K, N = 2, 37, 256, 128
        x = torch.randn(B, T, K, generator=g).to(torch.bfloat16)
        w = torch.randn(N, K, generator=g) * 0.02
        wq, ws = O.quant_weight_128x128(w.numpy())
        xp, t = pad_for_uniform_sharding(x, world)
        local, counts = shard_tokens(xp, world, rank)
        lb = local.contiguous().view(-1, K).view(torch.int16).numpy().view(np.uint16)
        aq, asc = O.quant_act_1x128(lb)
        y = O.gemm_dequant_f32(aq, asc, wq, ws)                     # per-rank linear
        y = torch.from_numpy(y).view(B, counts[rank], N)
        full = unpad(gather_output_tokens(y, counts), t)
        torch.save(full, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_linear_matches_single(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    from oracle import oracle as O
    g = torch.Generator().manual_seed(0)
    B, T, K, N = 2, 37, 256, 128
    x = torch.randn(B, T, K, generator=g).to(torch.bfloat16)
    w = torch.randn(N, K, generator=g) * 0.02
    wq, ws = O.quant_weight_128x128(w.numpy())
    aq, asc = O.quant_act_1x128(x.view(-1, K).view(torch.int16).numpy().view(np.uint16))
    ref = torch.from_numpy(O.gemm_dequant_f32(aq, asc, wq, ws)).view(B, T, N)
    for r in range(world):
        got = torch.load(tmp_path / f"rank{r}.pt")
        assert got.shape == ref.shape
        # Each token's row is computed from the same codes on whichever rank owns it.
        assert torch.equal(got, ref)
