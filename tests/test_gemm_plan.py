"""The GEMM launch plan (split-K of skinny outputs, split of a sparse last wave of
long-K outputs) as the host computes it, without a GPU: ltxfp8_gemm_plan_for_sms
against a restatement of its rules, and the bounds the callers rely on."""
from __future__ import annotations

import ctypes
import itertools
import math

import pytest

SMS = 148           # B200
TILE_M, TILE_N = 128, 256
STATIC_SCRATCH = 32 << 20


def _plan(M, N, K, sms=SMS):
    from ltx_kernels import _lib
    L = _lib.load()
    info = _lib.GemmPlanInfo()
    rc = L.ltxfp8_gemm_plan_for_sms(M, N, K, sms, ctypes.byref(info))
    assert rc == 0, L.ltxfp8_last_error().decode()
    return info.workspace_bytes, info.launches, info.splits, info.split_row0


def _splits(tiles, kb, sms):
    """Cost model of the skinny split: ceil(kb/S) + 6 + 0.105 * units against kb."""
    if kb < 4 or tiles * 2 > sms:
        return 1, kb
    best, best_s = float(kb), 1
    for s in range(2, min(sms // tiles, kb // 2, 16) + 1):
        c = math.ceil(kb / s) + 6.0 + 0.105 * tiles * s
        if c < best:
            best, best_s = c, s
    if best_s < 2:
        return 1, kb
    kbps = math.ceil(kb / best_s)
    return math.ceil(kb / kbps), kbps


def _expected(M, N, K, sms=SMS):
    mt, nt, kb = math.ceil(M / TILE_M), math.ceil(N / TILE_N), K // 128
    tiles = mt * nt
    if tiles * 2 <= sms:
        s, _ = _splits(tiles, kb, sms)
        return (0, tiles, s) if s > 1 else (M, 0, 1)
    rem = tiles % sms
    if kb < 64 or rem == 0 or rem * 2 > sms:
        return M, 0, 1
    tail_mt = math.ceil(rem / nt)
    if tail_mt >= mt or tail_mt * nt * 2 > sms:
        return M, 0, 1
    s, _ = _splits(tail_mt * nt, kb, sms)
    return ((mt - tail_mt) * TILE_M, tail_mt * nt, s) if s > 1 else (M, 0, 1)


SHAPES = list(itertools.product([1, 64, 128, 256, 1000, 2048, 5000, 6144, 24576, 49152],
                                [128, 2048, 4096, 12288, 16384],
                                [128, 512, 2048, 4096, 8192, 16384]))


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_plan_matches_rules(M, N, K):
    ws, launches, splits, row0 = _plan(M, N, K)
    e_row0, e_tiles, e_splits = _expected(M, N, K)
    assert (row0, splits) == (e_row0, e_splits)
    if splits == 1:
        assert ws == 0 and launches == 1 and row0 == M
        return
    assert ws == e_tiles * splits * TILE_M * TILE_N * 4
    assert launches == (3 if row0 > 0 else 2)
    assert 0 <= row0 < M and row0 % TILE_M == 0
    # every split unit runs in one wave, and the scratch fits the static array
    assert e_tiles * splits <= SMS
    assert ws <= STATIC_SCRATCH


def test_plan_examples():
    # skinny outputs with long K split (text rows of an 8-GPU rank; an audio projection)
    assert _plan(256, 4096, 4096)[2] > 1
    assert _plan(128, 2048, 8192)[2] > 1
    # 32 tiles of only 16 K blocks: the reduction would cost more than it saves
    assert _plan(128, 8192, 2048)[2] == 1
    # 8-GPU FFN down shard: full waves unsplit, the last two M-tile rows split 4 ways
    ws, launches, splits, row0 = _plan(6144, 4096, 16384)
    assert (row0, splits, launches) == (5888, 4, 3) and ws == 32 * 4 * TILE_M * TILE_N * 4
    # short K and full-wave shapes are not split
    assert _plan(6144, 4096, 4096)[2] == 1
    assert _plan(24576, 16384, 4096)[2] == 1


def test_plan_rejects_bad_arguments():
    from ltx_kernels import _lib
    L = _lib.load()
    info = _lib.GemmPlanInfo()
    assert L.ltxfp8_gemm_plan_for_sms(128, 100, 256, SMS, ctypes.byref(info)) == _lib.ERR_UNSUPPORTED_SHAPE
    assert L.ltxfp8_gemm_plan_for_sms(128, 256, 256, 0, ctypes.byref(info)) == _lib.ERR_INVALID_ARGUMENT
    assert L.ltxfp8_gemm_plan_for_sms(128, 256, 256, SMS, None) == _lib.ERR_INVALID_ARGUMENT
