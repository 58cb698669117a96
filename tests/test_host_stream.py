"""Host side of the token streamer without a GPU: chunk boundaries."""
from __future__ import annotations

import pytest


@pytest.mark.parametrize("rows,chunk", [(24576, 2048), (3000, 1024), (1000, 4096), (1, 1), (0, 7), (2049, 1024)])
def test_chunk_bounds_cover_rows(rows, chunk):
    from ltx_kernels.blockwise.host_stream import chunk_bounds
    b = chunk_bounds(rows, chunk)
    assert b[0] == 0 and b[-1] == rows
    sizes = [b[i + 1] - b[i] for i in range(len(b) - 1)]
    assert all(0 < s <= chunk for s in sizes) or rows == 0
    assert sum(sizes) == rows
    assert all(s == chunk for s in sizes[:-1])  # only the last chunk is ragged


def test_chunk_bounds_rejects_bad_arguments():
    from ltx_kernels.blockwise.host_stream import chunk_bounds
    with pytest.raises(ValueError):
        chunk_bounds(10, 0)
    with pytest.raises(ValueError):
        chunk_bounds(-1, 4)
