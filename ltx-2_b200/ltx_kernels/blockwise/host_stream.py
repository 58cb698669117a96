"""Token streaming from host memory through a row-independent blockwise layer.

Serving with host-resident activations (offloaded token streams, or a host that
owns the request buffers) pays one PCIe round trip per call: H2D of the bf16
tokens, the layer, D2H of the result.  Run one after the other, the two copies
cost more than the FP8 layers themselves (FFN pair at 24576 tokens: ~3.5 ms each
way at ~57 GB/s against ~4 ms of GEMMs).  The linears of the reference's DiT are
row-independent in the tokens (each output row depends only on its input row:
ltx-core/src/ltx_core/multigpu/transformer/sequence_parallel.py:158-182 shards
them by tokens for the same reason), so a call can be cut into token chunks and
pipelined over three CUDA streams:

    h2d stream      copy chunk i+1 into device slot (i+1) % 2
    compute stream  layer on chunk i (the caller's kernels, on this stream)
    d2h stream      copy the result of chunk i-1 back to the host

Only the first chunk's H2D copy and the last chunk's D2H copy are not hidden.
(Half-size first and last chunks measured no faster: with the three stages this
close in total time, the next full chunk's copy is exposed instead.)

Device input slots are reused only after the compute stream has finished with
them (events).  Chunk outputs stay referenced until the caller's stream has
joined the d2h stream at the end of the call; they are allocated on the compute
stream, whose next work is ordered after that join, so the caching allocator
may reuse them at once (``record_stream`` would defer their reuse to event
polling and make the allocator grow new segments mid-call).  Anything the
caller records after the call (CUDA events, a synchronize) covers all of the
work.  Every kernel
on the path is row-independent and deterministic, so each output row equals the
whole-batch result for that row, bit for bit where the GEMM plan (split-K or not)
is the same at the chunk's row count and at the batch's, and to fp32 summation
order where it differs.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

__all__ = ["chunk_bounds", "stream_tokens", "TokenStreamer"]


def chunk_bounds(rows: int, chunk: int):
    """Row boundaries [0, c, 2c, ..., rows] of a ``rows``-token call cut into chunks of
    at most ``chunk`` tokens."""
    if rows < 0 or chunk < 1:
        raise ValueError("chunk_bounds: rows >= 0 and chunk >= 1 required")
    return list(range(0, rows, chunk)) + [rows]


class TokenStreamer:
    """Reusable streams, events and device input slots for ``stream_tokens``.

    ``fn`` receives each chunk as one sequence of tokens, bf16 ``[1, rows, in_features]``
    (the DiT's ``[B, S, D]`` layout, which ``BlockwiseFP8Linear`` requires), runs on the
    current stream and returns ``[1, rows, out_features]`` or ``[rows, out_features]``;
    it must be row-independent."""

    def __init__(self, fn: Callable[[torch.Tensor], torch.Tensor], in_features: int, chunk_tokens: int,
                 device: Optional[torch.device] = None, in_dtype: torch.dtype = torch.bfloat16):
        if chunk_tokens < 1:
            raise ValueError("chunk_tokens must be >= 1")
        self.fn = fn
        self.chunk = int(chunk_tokens)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.in_features = in_features
        self.in_dtype = in_dtype
        self.h2d = torch.cuda.Stream(self.device)
        self.compute = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        self.slots = [torch.empty((self.chunk, in_features), dtype=in_dtype, device=self.device) for _ in range(2)]
        self.in_ready = [torch.cuda.Event() for _ in range(2)]
        self.in_free = [torch.cuda.Event() for _ in range(2)]

    def bounds(self, rows: int):
        """Row boundaries of the chunks of a ``rows``-token call."""
        return chunk_bounds(rows, self.chunk)

    def __call__(self, x_host: torch.Tensor, out_host: torch.Tensor) -> torch.Tensor:
        if x_host.is_cuda or out_host.is_cuda:
            raise RuntimeError("stream_tokens: x_host and out_host must be host tensors")
        if x_host.dim() != 2 or x_host.shape[1] != self.in_features or x_host.dtype != self.in_dtype:
            raise RuntimeError(f"stream_tokens: x_host must be {self.in_dtype} [rows, {self.in_features}], got "
                               f"{x_host.dtype} {tuple(x_host.shape)}")
        if out_host.dim() != 2 or out_host.shape[0] != x_host.shape[0]:
            raise RuntimeError("stream_tokens: out_host must be [rows, out_features] with the rows of x_host")
        if not (x_host.is_contiguous() and out_host.is_contiguous()):
            raise RuntimeError("stream_tokens: host buffers must be contiguous")
        rows = x_host.shape[0]
        caller = torch.cuda.current_stream(self.device)
        outputs = []  # chunk results, alive until the caller has joined the d2h stream
        for s in (self.h2d, self.compute, self.d2h):
            s.wait_stream(caller)
        fresh = [True, True]
        b = self.bounds(rows)
        for i in range(len(b) - 1):
            r0, r1 = b[i], b[i + 1]
            n = r1 - r0
            slot = i & 1
            xd = self.slots[slot][:n]
            with torch.cuda.stream(self.h2d):
                if not fresh[slot]:
                    self.h2d.wait_event(self.in_free[slot])
                xd.copy_(x_host[r0:r1], non_blocking=True)
                self.in_ready[slot].record(self.h2d)
            fresh[slot] = False
            with torch.cuda.stream(self.compute):
                self.compute.wait_event(self.in_ready[slot])
                y = self.fn(xd.unsqueeze(0))
                self.in_free[slot].record(self.compute)
                if y.dim() == 3 and y.shape[0] == 1:
                    y = y[0]
                if y.dim() != 2 or y.shape[0] != n or y.dtype != out_host.dtype or y.shape[1] != out_host.shape[1]:
                    raise RuntimeError(f"stream_tokens: layer returned {y.dtype} {tuple(y.shape)}, out_host is "
                                       f"{out_host.dtype} [{rows}, {out_host.shape[1]}]")
                outputs.append(y)
            self.d2h.wait_stream(self.compute)
            with torch.cuda.stream(self.d2h):
                out_host[r0:r1].copy_(y, non_blocking=True)
        caller.wait_stream(self.d2h)
        # The device slots are read on the compute stream and written on the h2d
        # stream; the next call's first copies wait for this call's last reads.
        caller.wait_stream(self.compute)
        # Compute-stream work of a later call (which may reuse these blocks) is
        # ordered after the caller's stream, hence after the copies that read them.
        del outputs
        return out_host


def stream_tokens(fn: Callable[[torch.Tensor], torch.Tensor], x_host: torch.Tensor, out_host: torch.Tensor,
                  chunk_tokens: int = 2048, device: Optional[torch.device] = None) -> torch.Tensor:
    """Run the row-independent layer ``fn`` over host tokens ``x_host`` [rows, K] (bf16,
    pinned for overlap) into ``out_host`` [rows, N], chunk by chunk (each chunk handed to
    ``fn`` as ``[1, chunk, K]``), with the copies of neighbouring chunks overlapping the
    layer.  Returns ``out_host``; the caller's current stream is ordered after every copy.

    ``chunk_tokens`` trades pipeline fill (the first H2D and last D2H are not hidden)
    against GEMM efficiency on short chunks; for the DiT FFN pair at 24576 tokens
    2048-token chunks measured best (4.69 ms; 3072: 4.90, 4096: 5.16, unchunked 10.6,
    against 3.7 ms of device work and ~3.6 ms for each copy direction).  For repeated
    calls keep a ``TokenStreamer``."""
    return TokenStreamer(fn, x_host.shape[1], chunk_tokens, device, x_host.dtype)(x_host, out_host)
