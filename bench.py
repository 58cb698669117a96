"""Benchmark of the B200 blockwise-FP8 linear path (BASELINE.json metric).

BASELINE.json's metric is "FP8 blockwise GEMM TFLOPS & % B200 FP8 peak; DiT
linear-stack ms at 1/2/4/8 GPU".  The default workload measures both halves:

* the step: BASELINE config 3, one denoising step of the 48-block dual-stream DiT,
  linears only, CFG batch 2 (28 blockwise-FP8 GEMMs per block), token-sharded over
  the ranks with weights replicated (strong scaling: the step's tokens are split).
  The step runs through the package's public layer modules (``BlockwiseFP8Linear``,
  ``BlockwiseFP8FeedForward``) on the step's quantised token streams; it is captured
  once as a CUDA graph and replayed.  `value` is the whole job's TFLOP/s, `ms_per_step`
  the step time (max over ranks, CUDA events).
* the GEMM: `headline_gemm` is the 24576 x 4096 -> 16384 up projection (bias +
  GELU-tanh + 1x128 requant fused), the shape of BASELINE's >= 70 % target, event-timed
  in isolation (burst) and over a seconds-long loop (sustained, clocks sampled).

`e2e` is the same step with the step's bf16 token streams copied in from pinned host
memory, quantised on the device, run through the stack, and the step's outputs (the
last block's video and audio FFN outputs) copied back, every step.
`gpu_reference` times the reference's own B200 path (its Triton 1x128 quantiser and
its SM89 mma.sync GEMM with fp32 accumulation, built from the reference's sources
into oracle/_ref) on config 0, config 1 and the headline GEMM, beside ours.

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--workload dit_step|ffn|linear|qkv_lora|producers|sweep|fp6]
                    [--impl ours|reference] [--e2e-chunk T] [--m TOKENS]

Multi-GPU (torchrun, one process per GPU): every rank runs its token shard, no
collective on the data path.  `--impl reference` times the reference's CPU torch
path (blockwise_quantize_torch, dequantise, fp32 matmul, bias, bf16; the reference's
own functions from oracle/_ref, else the oracle's restatement) on a bounded sample
of the same workload, on rank 0.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(REPO, "ltx-2_b200"), REPO):
    if _p not in sys.path:
        sys.path.insert(0, _p)

BASELINE_METRIC = "FP8 blockwise GEMM TFLOPS & % B200 FP8 peak; DiT linear-stack ms at 1/2/4/8 GPU"
NOMINAL_FP8_TFLOPS = 4500.0

WORKLOADS = {
    # name: (description, M per GPU, list of (K, N, epilogue))
    "ffn": ("DiT FFN pair (BASELINE config 1): 24576 tokens, 4096->16384 (+bias+GELU-tanh+1x128 requant) "
            "-> 16384->4096 (+bias)", 24576, [(4096, 16384, "gelu_requant"), (16384, 4096, "bias")]),
    "linear": ("single FP8 blockwise linear (BASELINE config 0): 6144 tokens, 4096->4096 (+bias)", 6144,
               [(4096, 4096, "bias")]),
    "qkv_lora": ("QKV projection with runtime LoRA r=128 (BASELINE config 2): 24576 tokens, 4096->12288", 24576,
                 [(4096, 12288, "lora128")]),
}


# one denoising step of the 48-block dual-stream DiT,
# linears only, CFG batch 2.  Token classes: video (2 x 24576), audio (2 x 512),
# text context (2 x 1024).  Per block, 28 blockwise-FP8 GEMMs
# (ltx-core/src/ltx_core/model/transformer/transformer.py:87-417,
# attention.py:508-579, feed_forward.py:6-15; dims from model_configurator.py:46-80):
# (token class, K, N, epilogue, input)
DIT_TOKENS = {"video": 2 * 24576, "audio": 2 * 512, "text": 2 * 1024}
DIT_BLOCKS = 48
DIT_BLOCK_GEMMS = [
    # video stream, hidden 4096
    ("video", 4096, 4096, "bias", "v"), ("video", 4096, 4096, "bias", "v"), ("video", 4096, 4096, "bias", "v"),
    ("video", 4096, 4096, "bias", "v"),                                      # self-attn q, k, v, out
    ("video", 4096, 4096, "bias", "v"), ("text", 4096, 4096, "bias", "t4"),
    ("text", 4096, 4096, "bias", "t4"), ("video", 4096, 4096, "bias", "v"),  # text cross-attn q, k, v, out
    ("video", 4096, 16384, "gelu_requant", "v"), ("video", 16384, 4096, "bias", "ffn_v"),  # FFN
    ("video", 4096, 2048, "bias", "v"), ("audio", 2048, 2048, "bias", "a"),
    ("audio", 2048, 2048, "bias", "a"), ("video", 2048, 4096, "bias", "v2k"),  # audio->video q, k, v, out
    # audio stream, hidden 2048
    ("audio", 2048, 2048, "bias", "a"), ("audio", 2048, 2048, "bias", "a"), ("audio", 2048, 2048, "bias", "a"),
    ("audio", 2048, 2048, "bias", "a"),                                      # self-attn
    ("audio", 2048, 2048, "bias", "a"), ("text", 2048, 2048, "bias", "t2"),
    ("text", 2048, 2048, "bias", "t2"), ("audio", 2048, 2048, "bias", "a"),  # text cross-attn
    ("audio", 2048, 8192, "gelu_requant", "a"), ("audio", 8192, 2048, "bias", "ffn_a"),   # FFN
    ("audio", 2048, 2048, "bias", "a"), ("video", 4096, 2048, "bias", "v"),
    ("video", 4096, 2048, "bias", "v"), ("audio", 2048, 2048, "bias", "a"),  # video->audio q, k, v, out
]
assert len(DIT_BLOCK_GEMMS) == 28
# The step's input token streams: one bf16 tensor per (token class, width) a GEMM reads
# (the FFN down projections read the up projections' requantised hidden state).
DIT_INPUTS = sorted({(c, K) for c, K, N, e, s in DIT_BLOCK_GEMMS if not s.startswith("ffn")})

HEADLINE = (24576, 4096, 16384)  # M, K, N of BASELINE's >= 70 % target (config-1 up projection)


def _env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


# ----------------------------------------------------------------------------- peaks
def measured_peaks() -> dict:
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def fp8_peak(sustained: bool = False):
    """Dense e4m3 tensor peak: twice the measured bf16 GEMM peak (the tensor core's e4m3
    rate is twice its bf16 rate); fallback 2 x 1590 / 2 x 1400 TFLOP/s."""
    mp = measured_peaks()
    key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    if key in mp:
        return 2.0 * float(mp[key]), f"2 x MEASURED_PEAKS.json {key} (of measured)"
    return (2800.0 if sustained else 3180.0), "2 x fallback bf16 (of fallback)"


def hbm_peak():
    mp = measured_peaks()
    if "hbm_gbs" in mp:
        return float(mp["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (of measured)"
    return 6650.0, "fallback 6.65 TB/s (of fallback)"


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, power, reasons = [], 0.0, [], set()
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = max(smax, float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"),
                               parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_median": statistics.median(power) if power else None}


# ----------------------------------------------------------------------------- timing helpers
def _events():
    import torch
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def graphed(fn):
    """`fn` captured once as a CUDA graph; returns the replay callable, or None when `fn`
    cannot be captured.  One replay is one host call, so events around short kernels hold
    their device time rather than the Python per-call overhead (a one-row quantisation
    times at 9 us eager after an L2 flush, 24 us eager back to back)."""
    import torch
    try:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
    except Exception as e:  # noqa: BLE001 -- reported, then timed eagerly
        torch.cuda.synchronize()
        print(f"bench: graph capture failed ({type(e).__name__}: {e}); timing eager calls", file=sys.stderr)
        return None
    return g.replay


def time_launches(fn, reps: int, warmup: int = 3, flush=None, graph: bool = False):
    """Mean device time (ms) of `fn` over `reps` launches, each bracketed by CUDA events on
    the current stream; `flush()` (untimed) runs before each launch when given.  `graph`:
    time replays of `fn` captured as a CUDA graph (falls back to eager calls when the
    capture fails)."""
    import torch
    for _ in range(warmup):
        fn()
    if graph:
        fn = graphed(fn) or fn
        fn()
    evs = [_events() for _ in range(reps)]
    for s, e in evs:
        if flush is not None:
            flush()
        s.record()
        fn()
        e.record()
    torch.cuda.synchronize()
    return sum(s.elapsed_time(e) for s, e in evs) / reps


def time_loop(fn, seconds: float, gpu_index: int):
    """Back-to-back launches of `fn` for about `seconds` (sustained regime, under the power
    cap); returns (mean ms per launch, launches, clocks sampled meanwhile)."""
    import torch
    t = time_launches(fn, 3, warmup=2)
    n = max(5, int(seconds * 1e3 / max(t, 1e-3)))
    clk = ClockSampler(gpu_index).start()
    s, e = _events()
    s.record()
    for _ in range(n):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / n, n, clk.stop()


class L2Flush:
    """Writes a buffer larger than the 126 MB L2 between timed launches of small shapes."""

    def __init__(self, dev):
        import torch
        self.buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def __call__(self):
        self.buf.fill_(1)


# ----------------------------------------------------------------------------- synthetic inputs
def synth_acts(M: int, K: int, g, dev):
    """bf16 ~N(0,1) with a seeded 1 % of channels x20 (BASELINE.json's activations)."""
    import torch
    x = torch.randn(M, K, generator=g, device=dev)
    x[:, torch.randperm(K, generator=g, device=dev)[: max(1, K // 100)]] *= 20.0
    return x.to(torch.bfloat16)


def synth_weight(N: int, K: int, g, dev):
    """~N(0, 0.02), block-quantised by the library's 128 x 128 weight kernel, plus a bias
    ~N(0, 0.01) rounded to bf16 and held in fp32."""
    import torch
    from ltx_kernels.blockwise import ops
    w = torch.randn(N, K, generator=g, device=dev) * 0.02
    wq, ws = ops.quantize_weight_128x128(w)
    del w
    b = (torch.randn(N, generator=g, device=dev) * 0.01).to(torch.bfloat16).float()
    return wq, ws, b


def gemm_alg_bytes(M, K, N, epi) -> float:
    """Algorithmic bytes of one GEMM launch: A + SFA + W + SFB + bias + output."""
    b = M * K + 4 * M * K / 128 + N * K + 4 * N * K / 16384 + 4 * N
    if epi == "gelu_requant":
        b += M * N + 4 * M * N / 128
    else:
        b += 2 * M * N
    if epi.startswith("lora"):
        r = int(epi[4:])
        b += 2 * M * r + 2 * N * r
    return b


def measure_cublas_fp8(dev) -> float | None:
    """cuBLASLt e4m3 GEMM throughput (torch._scaled_mm, 8192^3, best of 10), TFLOP/s:
    an external reference point (per-tensor scales, no block-scale promotion)."""
    import torch
    try:
        n = 8192
        a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
        b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn).t()
        one = torch.ones((), device=dev)
        f = lambda: torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        best = min(time_launches(f, 1, warmup=0) for _ in range(10))
        del a, b
        return 2.0 * n ** 3 / (best * 1e-3) / 1e12
    except Exception:  # noqa: BLE001 - informational
        return None


# ----------------------------------------------------------------------------- the headline GEMM
def headline_gemm(dev, gpu_index: int, sustained_s: float = 3.0, burst_only: bool = False,
                  burst: dict | None = None) -> dict:
    """The 24576 x 4096 -> 16384 up projection with bias + GELU-tanh + 1x128 requant fused:
    burst (event-timed launches; `burst_only` measures just these, on a cool GPU before the
    step loop) and sustained (a seconds-long loop, clocks sampled)."""
    import torch
    from ltx_kernels.blockwise import ops
    M, K, N = HEADLINE
    g = torch.Generator(device=dev).manual_seed(77)
    aq, asc = ops.quantize_1x128(synth_acts(M, K, g, dev))
    wq, ws, b = synth_weight(N, K, g, dev)
    from ltx_kernels import _lib as L
    f = lambda: ops.gemm(aq, asc, wq, ws, b, gelu=True, requant=True, write_d=False)
    if burst is None:
        burst = {"fused": time_launches(f, 10),
                 # the FFN module's path for the same result: plain GEMM to bf16, then GELU + requant
                 "split": time_launches(lambda: ops.gelu_tanh_quantize_1x128(ops.gemm(aq, asc, wq, ws, b),
                                                                            L.QUANT_TRITON), 10),
                 "plain": time_launches(lambda: ops.gemm(aq, asc, wq, ws, b), 10)}
        if burst_only:
            return burst
    burst, split_ms, plain_ms = burst["fused"], burst["split"], burst["plain"]
    sus_ms, n, clk = time_loop(f, sustained_s, gpu_index)
    flops = 2.0 * M * N * K
    pk, pk_src = fp8_peak()
    pks, pks_src = fp8_peak(sustained=True)
    tf, tfs = flops / (burst * 1e-3) / 1e12, flops / (sus_ms * 1e-3) / 1e12
    return {"shape": {"M": M, "K": K, "N": N, "epilogue": "bias + GELU-tanh + 1x128 requant"},
            "kernel": "fp8_blockwise_gemm_kernel<1,1>",
            "burst": {"ms": burst, "tflops": tf, "frac_of_fp8_peak": tf / pk, "peak": pk, "peak_source": pk_src,
                      "frac_of_nominal_4500": tf / NOMINAL_FP8_TFLOPS},
            "sustained": {"ms": sus_ms, "tflops": tfs, "launches": n, "frac_of_fp8_peak": tfs / pks, "peak": pks,
                          "peak_source": pks_src, "clocks": clk},
            "split_chain": {"ms": split_ms, "tflops": flops / (split_ms * 1e-3) / 1e12,
                            "frac_of_fp8_peak": flops / (split_ms * 1e-3) / 1e12 / pk,
                            "path": "GEMM (bias, bf16) + gelu_tanh_quant_kernel: BlockwiseFP8FeedForward's default"},
            "plain_gemm_bf16": {"ms": plain_ms, "tflops": flops / (plain_ms * 1e-3) / 1e12,
                                "frac_of_fp8_peak": flops / (plain_ms * 1e-3) / 1e12 / pk},
            "alg_bytes": gemm_alg_bytes(M, K, N, "gelu_requant"),
            "timing": "burst figures event-timed before the step loop (cool GPU), sustained after it"}


# ----------------------------------------------------------------------------- the reference's GPU path
def gpu_reference_record(dev) -> dict:
    """The reference's own B200 path timed beside ours on identical inputs: its Triton 1x128
    quantiser (triton_ops.py:102-151) and its SM89 mma.sync GEMM with fp32 accumulation
    (linear.py:25-35,98-104; csrc/blockwise/kernels/geforce/gemm.cu), built for sm_100a
    into oracle/_ref.  The reference's FFN runs GELU unfused (torch F.gelu on the bf16
    GEMM output, gelu_approx.py:10) and re-quantises it with the Triton quantiser."""
    import torch
    import torch.nn.functional as F
    from ltx_kernels import _lib as L
    from ltx_kernels.blockwise import ops
    from oracle import refpath
    if not refpath.available():
        return {"available": False, "why": "oracle/_ref not built (needs the reference checkout at build time)"}
    G, T = refpath.gemm(), refpath.triton_ops()
    out = {"available": True, "ref_path": "Triton quant + SM89 mma.sync GEMM (fp32 accumulate), sm_100a build",
           "ours_path": "CUDA quant + tcgen05 GEMM (fused epilogue)"}
    g = torch.Generator(device=dev).manual_seed(5)

    def sm89(a, s, w, ws, b, M, N):
        d = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        G.fp8_gemm_nt_sm89((a, s), (w, ws), d, b, use_fast_accum=False)
        return d

    # headline GEMM shape, bf16 out + bias on both sides
    M, K, N = HEADLINE
    x = synth_acts(M, K, g, dev)
    aq, asc = ops.quantize_1x128(x)
    wq, ws, b = synth_weight(N, K, g, dev)
    t_ref = time_launches(lambda: sm89(aq, asc, wq, ws, b, M, N), 5, warmup=2)
    t_ours = time_launches(lambda: ops.gemm(aq, asc, wq, ws, b), 10)
    fl = 2.0 * M * N * K
    out["gemm_24576x4096x16384_bias_bf16"] = {"ref_ms": t_ref, "ours_ms": t_ours, "ref_tflops": fl / t_ref / 1e9,
                                              "ours_tflops": fl / t_ours / 1e9, "speedup": t_ref / t_ours}
    # config 1: the FFN pair at 24576 tokens
    w2q, w2s, b2 = synth_weight(4096, 16384, g, dev)

    def ref_ffn():
        q, s = T._quant_blockwise_tma_aligned_func(x.view(1, M, K), False)
        h = F.gelu(sm89(q.view(M, K), s, wq, ws, b, M, N), approximate="tanh")
        hq, hs = T._quant_blockwise_tma_aligned_func(h.view(1, M, N), False)
        return sm89(hq.view(M, N), hs, w2q, w2s, b2, M, 4096)

    def our_ffn():  # the FFN module's path (BlockwiseFP8FeedForward)
        q, s = ops.quantize_1x128(x, L.QUANT_TRITON)
        hq, hs = ops.gelu_tanh_quantize_1x128(ops.gemm(q, s, wq, ws, b), L.QUANT_TRITON)
        return ops.gemm(hq, hs, w2q, w2s, b2)

    t_ref, t_ours = time_launches(ref_ffn, 3, warmup=1), time_launches(our_ffn, 10)
    fl = 2 * 2.0 * M * N * K
    out["ffn_config1"] = {"ref_ms": t_ref, "ours_ms": t_ours, "ref_tflops": fl / t_ref / 1e9,
                          "ours_tflops": fl / t_ours / 1e9, "speedup": t_ref / t_ours}
    del w2q, w2s
    # config 0: quantise + one 6144 x 4096 -> 4096 linear
    M0, K0, N0 = 6144, 4096, 4096
    x0 = synth_acts(M0, K0, g, dev)
    w0q, w0s, b0 = synth_weight(N0, K0, g, dev)
    flush = L2Flush(dev)

    def ref_lin():
        q, s = T._quant_blockwise_tma_aligned_func(x0.view(1, M0, K0), False)
        return sm89(q.view(M0, K0), s, w0q, w0s, b0, M0, N0)

    def our_lin():
        q, s = ops.quantize_1x128(x0, L.QUANT_TRITON)
        return ops.gemm(q, s, w0q, w0s, b0)

    t_ref, t_ours = time_launches(ref_lin, 10, flush=flush), time_launches(our_lin, 10, flush=flush)
    fl = 2.0 * M0 * N0 * K0
    out["linear_config0"] = {"ref_ms": t_ref, "ours_ms": t_ours, "ref_tflops": fl / t_ref / 1e9,
                             "ours_tflops": fl / t_ours / 1e9, "speedup": t_ref / t_ours, "l2": "flushed"}
    torch.cuda.synchronize()
    return out


# ----------------------------------------------------------------------------- CPU reference path
def _cpu_threads() -> int:
    import torch
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def cpu_reference_layers(layers, rows: int, seed: int = 0, budget_s: float = 8.0):
    """The reference's CPU torch path over `rows` tokens of a stack of linears, each
    (K, N, epilogue, input key): blockwise_quantize_torch (functional.py:138-144) of the
    bf16 input, dequantise, fp32 matmul with the dequantised blockwise_quantize_weights
    weight (functional.py:128-135, load time, untimed), + fp32 bias, bf16; GELU-tanh in
    torch on bf16 after a gelu_requant layer.  The reference's own functions come from
    oracle/_ref (kind "reference"); without it, the oracle's restatement (kind "port").
    Returns (seconds per pass, flops per pass, threads, kind)."""
    import numpy as np
    import torch
    import torch.nn.functional as F
    from oracle import refpath

    threads = _cpu_threads()
    g = torch.Generator().manual_seed(seed)
    if refpath.available("py"):
        RF = refpath.functional(with_cuda_ops=False)
        kind = "reference"

        def quant(x):  # x bf16 [M, K] -> (e4m3 [M, K], scales [K/128, M])
            q, s = RF.blockwise_quantize_torch(x.view(1, *x.shape))
            return q.view(x.shape), s

        def wquant(w):
            return RF.blockwise_quantize_weights(w)
    else:
        from oracle import oracle as O
        kind = "port"

        def quant(x):
            xb = x.contiguous().view(torch.int16).numpy().view(np.uint16)
            q, s = O.quant_act_1x128(xb)
            return torch.from_numpy(q).view(torch.float8_e4m3fn), torch.from_numpy(s[:, : x.shape[0]].copy())

        def wquant(w):
            q, s = O.quant_weight_128x128(w.numpy())
            return torch.from_numpy(q).view(torch.float8_e4m3fn), torch.from_numpy(s)

    def dequant_act(q, s):
        M, K = q.shape
        return (q.float().view(M, K // 128, 128) * s.t().reshape(M, K // 128, 1)).view(M, K)

    mats, inputs = [], {}
    for K, N, epi, key in layers:
        wq, ws = wquant(torch.randn(N, K, generator=g) * 0.02)
        wd = (wq.float().view(N // 128, 128, K // 128, 128) * ws.view(N // 128, 1, K // 128, 1)).view(N, K)
        b = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16).float()
        mats.append((K, N, epi, key, wd, b))
        if key is not None and key not in inputs:
            x = torch.randn(rows, K, generator=g)
            x[:, torch.randperm(K, generator=g)[: max(1, K // 100)]] *= 20.0
            inputs[key] = x.to(torch.bfloat16)

    def run():
        hidden = None
        for K, N, epi, key, wd, b in mats:
            x = hidden if key is None else inputs[key]
            q, s = quant(x)
            d = (dequant_act(q, s) @ wd.t() + b).to(torch.bfloat16)
            hidden = F.gelu(d, approximate="tanh") if epi == "gelu_requant" else d

    run()
    reps, t0 = 0, time.perf_counter()
    while True:
        run()
        reps += 1
        el = time.perf_counter() - t0
        if el > budget_s or reps >= 50:
            break
    flops = sum(2.0 * rows * N * K for K, N, epi, key, wd, b in mats)
    return el / reps, flops, threads, kind


def dit_cpu_layers():
    """One DiT block as (K, N, epilogue, input key) for cpu_reference_layers; an FFN
    down projection reads the preceding up projection's output (key None)."""
    return [(K, N, e, None if s.startswith("ffn") else (c, K)) for c, K, N, e, s in DIT_BLOCK_GEMMS]


def _dit_cpu_run(layers, rows: dict):
    """One config-3 block through the reference CPU path: each token class's GEMMs as one
    stack on `rows[class]` tokens (an FFN down projection reads its up projection's
    output).  Returns (seconds per block, threads, kind)."""
    total_t, threads, kind = 0.0, 1, "port"
    for seed, cls in enumerate(("video", "audio", "text")):
        sub = [lay for lay, (c, *_rest) in zip(layers, DIT_BLOCK_GEMMS) if c == cls]
        per, _, threads, kind = cpu_reference_layers(sub, rows[cls], seed=seed, budget_s=4.0)
        total_t += per
    return total_t, threads, kind


def dit_flops(toks: dict, blocks: int) -> float:
    return blocks * sum(2.0 * toks[c] * K * N for c, K, N, _, _ in DIT_BLOCK_GEMMS)


# ----------------------------------------------------------------------------- DiT step
def dit_tokens_per_rank(world: int, scaling: str) -> dict:
    """Token rows of each class on one rank: strong scaling splits the fixed step
    (padded up to a multiple of the world size), weak scaling keeps the full step per rank."""
    if scaling == "weak":
        return dict(DIT_TOKENS)
    return {k: -(-v // world) for k, v in DIT_TOKENS.items()}


def build_dit_step(dev, world: int, rank: int, scaling: str, blocks: int = DIT_BLOCKS):
    """The config-3 linear stack on this rank as the package's public layer modules.

    Returns (step, xin, flops, launches, desc, toks): `xin` holds the step's bf16 input
    token streams (one per (class, width) in DIT_INPUTS, device-resident); `step()`
    quantises them (torch.ops.blockwise.quantize, the reference's op) and runs the
    48 blocks, returning the last block's FFN outputs {"video": .., "audio": ..}."""
    import torch
    from ltx_kernels.blockwise import BlockwiseFP8FeedForward, BlockwiseFP8Linear
    from ltx_kernels.blockwise import ops

    toks = dit_tokens_per_rank(world, scaling)
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    xin = {key: synth_acts(toks[key[0]], key[1], g, dev) for key in DIT_INPUTS}

    def linear(K, N):
        wq, ws, b = synth_weight(N, K, g, dev)
        m = BlockwiseFP8Linear(K, N, bias=True, device=dev)
        m.weight.data, m.weight_scale.data, m.bias.data = wq, ws, b
        return m

    layers = []
    for _ in range(blocks):
        blk, pending = [], None
        for cls, K, N, epi, src in DIT_BLOCK_GEMMS:
            if epi == "gelu_requant":
                pending = (cls, K, linear(K, N))
            elif src.startswith("ffn"):
                up_cls, up_K, up = pending
                blk.append(("ffn", up_cls, up_K, BlockwiseFP8FeedForward.from_linears(up, linear(K, N))))
            else:
                blk.append(("linear", cls, K, linear(K, N)))
        layers.append(blk)
    torch.cuda.synchronize(dev)

    # The audio and text layers run on a second stream (forked after the input
    # quantisation, joined at the end; both captured into the step's graph): their skinny
    # GEMMs use the SMs the video GEMMs leave idle in their last, partial waves.
    side = torch.cuda.Stream(dev)

    def step():
        acts = {}
        for (cls, K), x in xin.items():
            q, s = torch.ops.blockwise.quantize(x.view(1, *x.shape), False)
            acts[(cls, K)] = (q, s)
        outs = {}
        main = torch.cuda.current_stream(dev)
        side.wait_stream(main)
        with torch.inference_mode():
            for blk in layers:
                for kind, cls, K, mod in blk:
                    if cls == "video":
                        y = mod(acts[(cls, K)])
                    else:
                        with torch.cuda.stream(side):
                            y = mod(acts[(cls, K)])
                    if kind == "ffn":
                        outs[cls] = y
        main.wait_stream(side)
        return outs

    flops = dit_flops(toks, blocks)
    desc = (f"DiT linear stack (BASELINE config 3): {blocks} blocks x 28 FP8 GEMMs, CFG batch 2, tokens per rank "
            f"video {toks['video']} / audio {toks['audio']} / text {toks['text']} ({scaling} scaling)")
    launches = len(DIT_INPUTS)  # the step's quantiser launches
    for cls, K, N, epi, src in DIT_BLOCK_GEMMS:
        launches += blocks * ops.gemm_plan(toks[cls], N, K, dev)["launches"]
        if epi == "gelu_requant":
            launches += blocks  # the FFN's GELU + requant pass
    return step, xin, flops, launches, desc, toks


def dominant_kernel_roofline(dev, M: int, K: int = 4096, N: int = 16384) -> dict:
    """The step's dominant kernel -- fp8_blockwise_gemm_kernel<0,0> on the video FFN up
    projection (bias, bf16 out; the FFN module's GELU + requant follow in their own pass)
    at this rank's token count -- event-timed in isolation in the same run."""
    import torch
    from ltx_kernels.blockwise import ops
    g = torch.Generator(device=dev).manual_seed(78)
    aq, asc = ops.quantize_1x128(synth_acts(M, K, g, dev))
    wq, ws, b = synth_weight(N, K, g, dev)
    flush = L2Flush(dev) if M * K + N * K < (126 << 20) else None
    ms = time_launches(lambda: ops.gemm(aq, asc, wq, ws, b), 10, flush=flush)
    flops = 2.0 * M * N * K
    pk, src = fp8_peak()
    achieved = flops / (ms * 1e-3) / 1e12
    traffic = None
    try:
        with open(os.path.join(REPO, "profiles", "ncu_traffic.json")) as f:
            tr = json.load(f).get("ffn:gemm_4096x16384_bias")
        if tr:  # captured at 24576 rows; scaled by rows processed
            traffic = tr["bytes_per_launch_at_bench_size"] * M / 24576.0
    except (OSError, ValueError, KeyError):
        traffic = None
    return {"bound": "tensor", "kernel": f"fp8_blockwise_gemm_kernel<0,0> (video FFN up, {M}x{K}->{N}, bias, bf16)",
            "achieved": achieved, "peak": pk, "unit": "TFLOP/s", "frac": achieved / pk, "peak_source": src,
            "frac_of_nominal_4500": achieved / NOMINAL_FP8_TFLOPS, "launch_ms": ms,
            "alg_bytes": gemm_alg_bytes(M, K, N, "bias"), "traffic": traffic,
            "traffic_note": "ncu DRAM bytes of the 24576-row launch scaled by rows" if traffic else None,
            "timing": "isolated launches, CUDA events on the launching stream" + (", L2 flushed" if flush else "")}


def run_dit(args, rank: int, world: int, local: int):
    """Config 3: the DiT linear stack, token-sharded over the ranks (strong scaling by default)."""
    scaling = args.scaling or "strong"
    sample = {"video": 512, "audio": 64, "text": 64}
    toks_rank = dit_tokens_per_rank(world, scaling)
    desc = (f"DiT linear stack (BASELINE config 3): {args.blocks} blocks x 28 FP8 GEMMs, CFG batch 2, tokens per "
            f"rank video {toks_rank['video']} / audio {toks_rank['audio']} / text {toks_rank['text']} "
            f"({scaling} scaling)")
    cfg = {"workload": desc, "tokens_per_rank": toks_rank, "blocks": args.blocks,
           "parallelism": f"token-sharded over {world} GPU(s), weights replicated, no collective",
           "l2": "per-block weights 385 MB > L2; no flush"}
    if args.impl == "reference":
        if rank != 0:
            return
        per, threads, kind = _dit_cpu_run(dit_cpu_layers(), sample)
        fl_sample = dit_flops(sample, 1)
        val = fl_sample / per / 1e12
        total = dit_flops(DIT_TOKENS, args.blocks)
        print(json.dumps({
            "metric": BASELINE_METRIC, "value": val, "unit": "TFLOP/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total / (val * 1e12) * 1e3, "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": "f32 (dequantised e4m3 operands)", "data": "synthetic", "config": cfg,
            "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": threads, "kind": kind,
                             "sample": f"one of {args.blocks} blocks, tokens per class {sample}; the reference's "
                                       "CPU torch path (blockwise_quantize_torch, dequantise, fp32 matmul, bias, "
                                       "bf16, torch GELU); ms_per_step extrapolated to the full step by FLOPs"},
            "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    import torch
    import torch.distributed as dist
    from ltx_kernels.blockwise import ops

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))

    head_burst = headline_gemm(dev, local, burst_only=True) if (world == 1 and not args.no_extras) else None
    step, xin, flops, launches, desc, toks = build_dit_step(dev, world, rank, scaling, args.blocks)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()
    assert ops.device_status() == 0
    # The step is ~1350 launches; at several GPUs most of them are shorter than the
    # host's per-call overhead, so the whole step is captured once as a CUDA graph (the
    # C ABI neither allocates nor synchronises) and replayed.
    graph, outs = None, None
    if not args.no_graph:
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            outs = step()
        for _ in range(2):
            graph.replay()
        barrier()

    def run_step():
        if graph is not None:
            graph.replay()
            return outs
        return step()

    clocks = ClockSampler(local).start()
    barrier()
    t0, t1 = _events()
    t0.record()
    for _ in range(args.steps):
        run_step()
    t1.record()
    barrier()
    elapsed = t0.elapsed_time(t1)
    clk = clocks.stop()

    # End to end: this rank's bf16 token streams come from pinned host memory into the
    # step's input buffers, are quantised and run through the stack on the device, and the
    # step's outputs (last block's video and audio FFN outputs) return to pinned host memory.
    hosts = {key: x.cpu().pin_memory() for key, x in xin.items()}
    last = run_step()
    out_host = {c: torch.empty(t.shape, dtype=t.dtype).pin_memory() for c, t in last.items()}
    e2e_steps = max(1, min(args.steps, 10))
    if graph is not None:
        # Double-buffered, as a serving loop runs it: a second set of input buffers and
        # a second capture of the step reading them (sharing the first graph's memory
        # pool: the two never run at once), so step i+1's H2D (one copy stream) and
        # step i's D2H (another) overlap step i's compute.  Every step's copies stay
        # inside the timed region: the first H2D and the last D2H are exposed.
        xin_a = dict(xin)
        xin_b = {key: torch.empty_like(x) for key, x in xin.items()}
        xin.update(xin_b)
        graph_b = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_b, pool=graph.pool()):
            outs_b = step()
        xin.update(xin_a)
        sets = [(xin_a, graph, outs), (xin_b, graph_b, outs_b)]
        main = torch.cuda.current_stream(dev)
        h2d_s, d2h_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

        def e2e_run(n):
            ev_in = [torch.cuda.Event() for _ in range(2)]
            ev_done = [torch.cuda.Event() for _ in range(2)]
            ev_out = [torch.cuda.Event() for _ in range(2)]
            used = [False, False]
            with torch.cuda.stream(h2d_s):
                h2d_s.wait_stream(main)
                for key, h in hosts.items():
                    sets[0][0][key].copy_(h, non_blocking=True)
                ev_in[0].record(h2d_s)
            for i in range(n):
                cur, nxt = i % 2, (i + 1) % 2
                if i + 1 < n:
                    with torch.cuda.stream(h2d_s):
                        if used[nxt]:
                            h2d_s.wait_event(ev_done[nxt])  # the step that last read these inputs
                        for key, h in hosts.items():
                            sets[nxt][0][key].copy_(h, non_blocking=True)
                        ev_in[nxt].record(h2d_s)
                main.wait_event(ev_in[cur])
                if used[cur]:
                    main.wait_event(ev_out[cur])  # its outputs of two steps ago are copied out
                sets[cur][1].replay()
                ev_done[cur].record(main)
                used[cur] = True
                with torch.cuda.stream(d2h_s):
                    d2h_s.wait_event(ev_done[cur])
                    for c, t in sets[cur][2].items():
                        out_host[c].copy_(t, non_blocking=True)
                    ev_out[cur].record(d2h_s)
            main.wait_stream(d2h_s)
            main.wait_stream(h2d_s)

        e2e_run(2)
        barrier()
        e0, e1 = _events()
        e0.record()
        e2e_run(e2e_steps)
        e1.record()
        barrier()
        del graph_b, outs_b, sets
    else:
        def e2e_step():
            for key, h in hosts.items():
                xin[key].copy_(h, non_blocking=True)
            o = run_step()
            for c, t in o.items():
                out_host[c].copy_(t, non_blocking=True)

        e2e_step()
        barrier()
        e0, e1 = _events()
        e0.record()
        for _ in range(e2e_steps):
            e2e_step()
        e1.record()
        barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    assert ops.device_status() == 0
    if world > 1:
        t = torch.tensor([elapsed, e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed, e2e_ms = t.tolist()
    ms = elapsed / args.steps
    total_flops = dit_flops(DIT_TOKENS, args.blocks) if scaling == "strong" else flops * world
    value = total_flops / (ms * 1e-3) / 1e12
    h2d = sum(h.numel() * h.element_size() for h in hosts.values())
    d2h = sum(h.numel() * h.element_size() for h in out_host.values())
    del graph, outs, last
    torch.cuda.synchronize(dev)
    # Per-rank extras (every rank runs them, so the collectives stay in step).
    roof = dominant_kernel_roofline(dev, toks["video"])
    head = headline_gemm(dev, local, burst=head_burst) if head_burst is not None else None
    gref = gpu_reference_record(dev) if (world == 1 and not args.no_extras) else None
    cublas = measure_cublas_fp8(dev) if (rank == 0 and not args.no_extras) else None
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            per, threads, kind = _dit_cpu_run(dit_cpu_layers(), sample)
            cpu = {"value": dit_flops(sample, 1) / per / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": kind,
                   "sample": f"one block, tokens per class {sample}; the reference's CPU torch path"}
        print(json.dumps({
            "metric": BASELINE_METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "e4m3 x e4m3 -> f32 accumulate, bf16 out",
            "data": "synthetic (seeded; BASELINE.json distributions)", "config": cfg,
            "dit_step_ms": ms,
            "headline_gemm": head,
            "roofline": roof,
            "cublas_fp8_tflops": cublas,
            "gpu_reference": gref,
            "cpu_baseline": cpu,
            "e2e": {"value": total_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "H2D of the step's bf16 token streams into the step's input buffers, "
                           "torch.ops.blockwise.quantize + BlockwiseFP8Linear / BlockwiseFP8FeedForward "
                           "(graph-replayed), D2H of the last block's video and audio outputs"
                           + ("; double-buffered inputs, the next step's H2D and this step's D2H on copy "
                              "streams overlapping its compute" if not args.no_graph else "")},
            "gpu_launches": args.steps * launches,
            "cuda_graph": not args.no_graph,
            "clocks": clk,
        }))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- single-layer workloads
def build_workload(name: str, M: int, dev, seed: int):
    """Seeded synthetic inputs resident on `dev` (BASELINE.json distributions)."""
    import torch
    desc, _, layers = WORKLOADS[name]
    g = torch.Generator(device=dev).manual_seed(seed)
    x = synth_acts(M, layers[0][0], g, dev)
    params = []
    for K, N, epi in layers:
        wq, ws, b = synth_weight(N, K, g, dev)
        lora = None
        if epi.startswith("lora"):
            r = int(epi[4:])
            la = (torch.randn(r, K, generator=g, device=dev) * 0.01).to(torch.bfloat16)
            lb = (torch.randn(N, r, generator=g, device=dev) * 0.01).to(torch.bfloat16)
            lora = (la, lb, 1.0)
        params.append((K, N, epi, wq, ws, b, lora))
    torch.cuda.synchronize(dev)
    return x, params


def flops_of(name: str, M: int) -> float:
    total = 0.0
    for K, N, epi in WORKLOADS[name][2]:
        total += 2.0 * M * N * K
        if epi.startswith("lora"):
            r = int(epi[4:])
            total += 2.0 * M * r * (K + N)
    return total


def build_module(name: str, params, dev):
    """The workload's layers as the package's public modules, sharing the bench's weights."""
    from ltx_kernels.blockwise import BlockwiseFP8FeedForward, BlockwiseFP8Linear, BlockwiseFP8LoRALinear

    def linear(K, N, wq, ws, b, lora=None):
        if lora is None:
            m = BlockwiseFP8Linear(K, N, bias=True, device=dev)
        else:
            la, lb, alpha = lora
            m = BlockwiseFP8LoRALinear(K, N, la.shape[0], alpha=alpha, bias=True, device=dev)
            m.lora_A.data, m.lora_B.data = la, lb
        m.weight.data, m.weight_scale.data, m.bias.data = wq, ws, b
        return m

    mods = [linear(K, N, wq, ws, b, lora) for (K, N, epi, wq, ws, b, lora) in params]
    if name == "ffn":
        return BlockwiseFP8FeedForward.from_linears(mods[0], mods[1])
    assert len(mods) == 1, name
    return mods[0]


def make_step(x, params):
    """Returns step(events=None) running the workload once on the current stream."""
    from ltx_kernels import _lib as L
    from ltx_kernels.blockwise import ops

    def step(ev=None):
        i = 0
        if ev is not None:
            ev[i].record()
        aq, asc = ops.quantize_1x128(x)
        i += 1
        if ev is not None:
            ev[i].record()
        cur = (aq, asc)
        out = None
        for (K, N, epi, wq, ws, b, lora) in params:
            if epi == "gelu_requant":
                # the FFN module's path: up projection to bf16, then torch's GELU + the
                # down projection's 1x128 quantisation in one streaming pass
                h = ops.gemm(cur[0], cur[1], wq, ws, b)
                i += 1
                if ev is not None:
                    ev[i].record()
                cur = ops.gelu_tanh_quantize_1x128(h, L.QUANT_TRITON)
            elif epi.startswith("lora"):
                la, lb, alpha = lora
                ax = ops.lora_a(x, la)
                i += 1
                if ev is not None:
                    ev[i].record()
                out = ops.gemm(cur[0], cur[1], wq, ws, b, lora_ax=ax, lora_b=lb, lora_alpha=alpha)
            else:
                out = ops.gemm(cur[0], cur[1], wq, ws, b)
            i += 1
            if ev is not None:
                ev[i].record()
        return out

    n_events = 2 + len(params) + sum(1 for p in params if p[2].startswith("lora") or p[2] == "gelu_requant")
    return step, n_events


def kernel_names(name: str):
    names = ["quantize_1x128"]
    for K, N, epi in WORKLOADS[name][2]:
        if epi.startswith("lora"):
            names.append(f"lora_a_{K}x{epi[4:]}")
        if epi == "gelu_requant":
            names += [f"gemm_{K}x{N}_bias", f"gelu_tanh_quant_{N}"]
        else:
            names.append(f"gemm_{K}x{N}_{epi}")
    return names


def single_cpu_layers(name: str):
    layers = WORKLOADS[name][2]
    out = []
    for i, (K, N, epi) in enumerate(layers):
        out.append((K, N, "gelu_requant" if epi == "gelu_requant" else "bias", ("x", K) if i == 0 else None))
    return out


def run_single(args, rank: int, world: int, local: int):
    desc, M_default, layers = WORKLOADS[args.workload]
    M = args.m or M_default
    rows = 512 if args.workload != "linear" else 1024
    if args.impl == "reference":
        if rank != 0:
            return
        per, fl, threads, kind = cpu_reference_layers(single_cpu_layers(args.workload), rows)
        val = fl / per / 1e12
        print(json.dumps({
            "metric": f"blockwise-FP8 {args.workload} TFLOP/s", "value": val, "unit": "TFLOP/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": flops_of(args.workload, M) / (val * 1e12) * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (dequantised e4m3 operands)", "data": "synthetic",
            "config": {"workload": desc, "tokens_per_gpu": M},
            "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": threads, "kind": kind,
                             "sample": f"{rows} of {M} tokens per step, same layers; the reference's CPU torch "
                                       "path (runtime LoRA not included)"},
            "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    import torch
    import torch.distributed as dist
    from ltx_kernels.blockwise import ops

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    x, params = build_workload(args.workload, M, dev, seed=1234 + rank)
    step, n_ev = make_step(x, params)
    names = kernel_names(args.workload)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()
    assert ops.device_status() == 0

    clocks = ClockSampler(local).start()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n_ev)] for _ in range(args.steps)]
    barrier()
    t_start, t_end = _events()
    t_start.record()
    for i in range(args.steps):
        step(evs[i])
    t_end.record()
    barrier()
    elapsed = t_start.elapsed_time(t_end)
    per_kernel = [0.0] * (n_ev - 1)
    for i in range(args.steps):
        for j in range(n_ev - 1):
            per_kernel[j] += evs[i][j].elapsed_time(evs[i][j + 1])
    per_kernel = [t / args.steps for t in per_kernel]

    # End to end through the public layer modules over pinned host tokens, streamed in
    # token chunks (ltx_kernels.blockwise.host_stream); --e2e-chunk 0: one whole-batch
    # copy in, the layer, one copy out.
    from ltx_kernels.blockwise.host_stream import TokenStreamer
    x_host = x.cpu().pin_memory()
    out_dim = params[-1][1]
    out_host = torch.empty((M, out_dim), dtype=torch.bfloat16).pin_memory()
    e2e_steps = max(3, min(args.steps, 10))
    layer = build_module(args.workload, params, dev)
    chunk = args.e2e_chunk if args.e2e_chunk > 0 else M
    streamer = TokenStreamer(layer, x.shape[1], chunk, dev)

    def e2e_step():
        with torch.inference_mode():
            streamer(x_host, out_host)

    for _ in range(2):
        e2e_step()
    barrier()
    e0, e1 = _events()
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    clk = clocks.stop()
    assert ops.device_status() == 0
    if world > 1:
        t = torch.tensor([elapsed, e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed, e2e_ms = t.tolist()

    fl = flops_of(args.workload, M)
    ms_per_step = elapsed / args.steps
    gemm_idx = [j for j, n in enumerate(names) if n.startswith("gemm")]
    dom = max(gemm_idx, key=lambda j: per_kernel[j])
    K, N, epi = layers[gemm_idx.index(dom)]
    dom_flops = 2.0 * M * N * K + (2.0 * M * int(epi[4:]) * N if epi.startswith("lora") else 0.0)
    achieved = dom_flops / (per_kernel[dom] * 1e-3) / 1e12
    pk, pk_src = fp8_peak()
    traffic = None
    try:
        with open(os.path.join(REPO, "profiles", "ncu_traffic.json")) as f:
            tr = json.load(f).get(f"{args.workload}:{names[dom]}")
        traffic = tr["bytes_per_launch_at_bench_size"] if tr else None
    except (OSError, ValueError, KeyError):
        traffic = None
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            per, flc, threads, kind = cpu_reference_layers(single_cpu_layers(args.workload), rows)
            cpu = {"value": flc / per / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": kind,
                   "sample": f"{rows} of {M} tokens, same layers, the reference's CPU torch path"}
        print(json.dumps({
            "metric": f"blockwise-FP8 {args.workload} TFLOP/s",
            "value": world * fl / (ms_per_step * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 x e4m3 -> f32 accumulate, bf16 out",
            "data": "synthetic (seeded; BASELINE.json distributions)",
            "config": {"workload": desc, "tokens_per_gpu": M, "layers": [list(l) for l in layers],
                       "parallelism": f"token-sharded dp{world}, weights replicated",
                       "l2": "working set > L2 (x 201 MB + weights + 403 MB fp8 hidden state); no flush"},
            "kernels_ms": {n: round(t, 4) for n, t in zip(names, per_kernel)},
            "roofline": {"bound": "tensor", "kernel": names[dom], "achieved": achieved, "peak": pk,
                         "unit": "TFLOP/s", "frac": achieved / pk, "peak_source": pk_src,
                         "frac_of_nominal_4500": achieved / NOMINAL_FP8_TFLOPS, "traffic": traffic},
            "cpu_baseline": cpu,
            "e2e": {"value": world * fl / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": M * out_dim * 2,
                    "api": f"{type(layer).__name__} via host_stream.TokenStreamer, {chunk}-token chunks"},
            "gpu_launches": args.steps * ((n_ev - 1) + sum(ops.gemm_plan(M, N, K, dev)["launches"] - 1
                                                           for K, N, _ in layers)),
            "clocks": clk,
        }))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- config-4 sweep
SWEEP_M = (128, 512, 2048, 8192, 32768, 65536)
SWEEP_KN = ((2048, 2048), (4096, 4096), (4096, 16384), (16384, 4096))


def run_sweep(args, rank: int, world: int, local: int):
    """M x (K, N) GEMMs (bias, bf16 out), each event-timed in isolation
    (L2 flushed between launches when the working set fits in L2), reported against the
    bound that applies at its arithmetic intensity (HBM GB/s or FP8 TFLOP/s), with the
    reference's SM89 GEMM on the same inputs beside it."""
    import torch
    from ltx_kernels.blockwise import ops
    from oracle import refpath
    if args.impl == "reference" or rank != 0:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the sweep is a GPU roofline map; the reference's "
                              "CPU path is timed by the other workloads"}))
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    G = refpath.gemm() if refpath.available("gemm") else None
    pk, pk_src = fp8_peak()
    bw, bw_src = hbm_peak()
    ridge = pk * 1e12 / (bw * 1e9)
    flush = L2Flush(dev)
    g = torch.Generator(device=dev).manual_seed(9)
    points, tot_fl, tot_ms = [], 0.0, 0.0
    clk = ClockSampler(local).start()
    for K, N in SWEEP_KN:
        wq, ws, b = synth_weight(N, K, g, dev)
        for M in SWEEP_M:
            aq, asc = ops.quantize_1x128(synth_acts(M, K, g, dev))
            small = M * K + N * K + 2 * M * N < (126 << 20)
            f = lambda: ops.gemm(aq, asc, wq, ws, b)
            ms = time_launches(f, 20 if M <= 2048 else 8, flush=flush if small else None, graph=True)
            fl, by = 2.0 * M * N * K, gemm_alg_bytes(M, K, N, "bias")
            ai = fl / by
            bound = "hbm" if ai < ridge else "tensor"
            p = {"M": M, "K": K, "N": N, "ms": ms, "tflops": fl / ms / 1e9, "gbs": by / ms / 1e6,
                 "alg_bytes": by, "intensity": ai, "bound": bound, "launches": ops.gemm_plan(M, N, K, dev)["launches"],
                 "frac": (by / ms / 1e6) / bw if bound == "hbm" else (fl / ms / 1e9) / pk,
                 "l2": "flushed" if small else "working set > L2"}
            if G is not None:
                def ref():
                    d = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
                    G.fp8_gemm_nt_sm89((aq, asc), (wq, ws), d, b, use_fast_accum=False)
                rms = time_launches(ref, 5 if M <= 2048 else 3, warmup=1, flush=flush if small else None, graph=True)
                p["ref_sm89_ms"], p["speedup_vs_sm89"] = rms, rms / ms
            points.append(p)
            tot_fl += fl
            tot_ms += ms
            del aq, asc
        del wq, ws
    c = clk.stop()
    print(json.dumps({
        "metric": "blockwise-FP8 GEMM sweep (BASELINE config 4) TFLOP/s", "value": tot_fl / tot_ms / 1e9,
        "unit": "TFLOP/s", "n_gpus": 1, "steps": 1, "warmup": 3, "ms_per_step": tot_ms, "higher_is_better": True,
        "scaling": "none", "vs_baseline": None, "dtype": "e4m3 x e4m3 -> f32 accumulate, bf16 out",
        "data": "synthetic (seeded; BASELINE.json distributions)",
        "config": {"workload": "config-4 roofline sweep", "M": list(SWEEP_M), "KN": [list(k) for k in SWEEP_KN],
                   "timing": "CUDA-graph replays of each call between CUDA events"},
        "peaks": {"fp8_tflops": pk, "fp8_source": pk_src, "hbm_gbs": bw, "hbm_source": bw_src,
                  "ridge_flop_per_byte": ridge},
        "points": points, "e2e": None, "cpu_baseline": None, "gpu_launches": sum(p["launches"] for p in points) * 8,
        "clocks": c}))


# ----------------------------------------------------------------------------- FP6 weights
FP6_SHAPES = [(128, 4096, 16384), (128, 16384, 4096), (1024, 4096, 4096), (8192, 4096, 16384),
              (24576, 4096, 16384)]


def run_fp6(args, rank: int, world: int, local: int):
    """BlockwiseFP6Linear's GEMM (linear.py:212-250): the 6-bit weight streamed into the
    tensor core (``gemm(..., w_fp6=True)``; with the tensor-core copy kept, and with the
    per-call rewrite of the module's default) against unpack-to-e4m3 + FP8 GEMM (the
    reference's algorithm, on this library's kernels and, when built, on the reference's
    own ops_cpp unpack + SM89 GEMM), bias, bf16 out, each event-timed in isolation."""
    import torch
    from ltx_kernels.blockwise import ops
    from oracle import refpath
    if args.impl == "reference" or rank != 0:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the fp6 workload times GPU paths only; the "
                              "reference's own GPU path is timed beside ours in the same line"}))
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    G = refpath.gemm() if refpath.available("gemm") else None
    R = refpath.ops() if refpath.available("ops") else None
    bw, bw_src = hbm_peak()
    flush = L2Flush(dev)
    g = torch.Generator(device=dev).manual_seed(11)
    points, launches = [], 0
    shapes = [sh for sh in FP6_SHAPES if not args.m or sh[0] == args.m]   # --m: one token count only
    clk = ClockSampler(local).start()
    for M, K, N in shapes:
        w = torch.randn(N, K, generator=g, device=dev) * 0.02
        wq, ws = ops.quantize_weight_128x128(w, scale_max=0.1172)
        del w
        b = (torch.randn(N, generator=g, device=dev) * 0.01).to(torch.bfloat16).float()
        w6 = ops.fp6_pack(wq.view(torch.uint8))
        tc, s6 = ops.fp6_to_tc(w6, ws)
        aq, asc = ops.quantize_1x128(synth_acts(M, K, g, dev))
        reps = 20 if M <= 2048 else 8
        small = M * K + N * K + 2 * M * N < (126 << 20)
        fl = flush if small else None
        d6 = ops.gemm(aq, asc, tc, s6, b, w_fp6=True)
        d8 = ops.gemm(aq, asc, ops.fp6_unpack(w6, K).view(torch.float8_e4m3fn), ws, b)
        same = bool(torch.equal(d6, d8))
        t_tc = time_launches(lambda: ops.gemm(aq, asc, tc, s6, b, w_fp6=True), reps, flush=fl, graph=True)
        t_tr = time_launches(lambda: ops.gemm(aq, asc, *ops.fp6_to_tc(w6, ws), b, w_fp6=True), reps, flush=fl,
                             graph=True)
        t_un = time_launches(lambda: ops.gemm(aq, asc, ops.fp6_unpack(w6, K).view(torch.float8_e4m3fn), ws, b),
                             reps, flush=fl, graph=True)
        t_f8 = time_launches(lambda: ops.gemm(aq, asc, wq, ws, b), reps, flush=fl, graph=True)
        launches += reps * (2 * ops.gemm_plan(M, N, K, dev)["launches"] + 2) * 2
        by = M * K + 4 * M * K // 128 + N * K * 3 // 4 + 4 * (N // 128) * (K // 128) + 4 * N + 2 * M * N
        p = {"M": M, "K": K, "N": N, "bit_identical_to_unpack_fp8": same,
             "fp6_tc_us": t_tc * 1e3, "fp6_per_call_rewrite_us": t_tr * 1e3, "unpack_fp8_us": t_un * 1e3,
             "fp8_weight_us": t_f8 * 1e3, "tflops_fp6_tc": 2.0 * M * N * K / t_tc / 1e9,
             "alg_bytes_fp6": by, "gbs_fp6_tc": by / t_tc / 1e6, "hbm_frac_fp6_tc": by / t_tc / 1e6 / bw,
             "speedup_tc_vs_unpack": t_un / t_tc, "speedup_rewrite_vs_unpack": t_un / t_tr}
        if G is not None and R is not None:
            def ref():
                w8 = R.fp6_unpack(w6, K).view(torch.float8_e4m3fn)
                d = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
                G.fp8_gemm_nt_sm89((aq, asc), (w8, ws), d, b, use_fast_accum=False)
            p["ref_unpack_sm89_us"] = time_launches(ref, 5 if M <= 2048 else 3, warmup=1, flush=fl, graph=True) * 1e3
            p["speedup_tc_vs_ref"] = p["ref_unpack_sm89_us"] / p["fp6_tc_us"]
        points.append(p)
        del wq, ws, w6, tc, s6, aq, asc, d6, d8
    c = clk.stop()
    tot = sum(p["fp6_tc_us"] for p in points)
    fl_tot = sum(2.0 * p["M"] * p["N"] * p["K"] for p in points)
    print(json.dumps({
        "metric": "blockwise FP6-weight GEMM TFLOP/s", "value": fl_tot / tot / 1e6, "unit": "TFLOP/s",
        "n_gpus": 1, "steps": 1, "warmup": 3, "ms_per_step": tot / 1e3, "higher_is_better": True,
        "scaling": "none", "vs_baseline": None, "dtype": "e4m3 x e2m3 (6-bit) -> f32 accumulate, bf16 out",
        "data": "synthetic (seeded; FP6-range weights from the 0.1172 quantiser)",
        "config": {"workload": "BlockwiseFP6Linear GEMM shapes", "shapes": [list(x) for x in shapes],
                   "l2": "flushed between launches when the working set fits in L2",
                   "timing": "CUDA-graph replays of each call between CUDA events"},
        "peaks": {"hbm_gbs": bw, "hbm_source": bw_src}, "points": points, "e2e": None, "cpu_baseline": None,
        "gpu_launches": launches, "clocks": c}))


# ----------------------------------------------------------------------------- producers
PROD_B, PROD_S, PROD_H, PROD_HEADS = 2, 24576, 4096, 32   # config 3 video tokens (CFG batch 2), d = 4096


def producer_bytes(M: int, H: int, heads: int) -> dict:
    """Algorithmic HBM bytes per launch (bf16 = 2 B, e4m3 = 1 B, one fp32 scale per 128)."""
    q = M * H + 4 * M * H // 128
    return {"adanorm_quant": 2 * M * H + q,                 # read x, write codes + scales
            "rms_fma_quant": 3 * 2 * M * H + q,             # read x, y, write x, codes + scales
            "gated_attention_quant": 2 * M * H + 2 * M * heads + q,
            "gelu_quant": 2 * M * H + q}


def cpu_producer_sample(rows: int, seed: int = 0):
    """The four producers restated by the oracle on `rows` tokens; returns (s per row, threads=1)."""
    import numpy as np
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    H = PROD_H
    bf = lambda a: O.f32_to_bf16(a.astype(np.float32))
    x = bf(rng.normal(0, 1, (1, rows, H)))
    y = bf(rng.normal(0, 1, (1, rows, H)))
    p = bf(rng.normal(0, 0.1, (1, 1, H)))
    lg = rng.normal(0, 3, (rows, PROD_HEADS)).astype(np.float32)
    O.adanorm_quant(x[:, :8], p, p)  # build + warm
    t0 = time.perf_counter()
    O.adanorm_quant(x, p, p)
    O.rms_fma(x, y, p)
    O.gated_attention(y[0], lg)
    O.gelu_quant(y[0])
    return (time.perf_counter() - t0) / rows, 1


def run_producers(args, rank: int, world: int, local: int):
    """The fused A-operand producers (adanorm, residual FMA + RMS, gated attention, GELU)
    with 1x128 quant, each once per step over the config-3 video tokens of one rank."""
    B, S, H, heads = PROD_B, PROD_S, PROD_H, PROD_HEADS
    M = B * S
    nbytes = producer_bytes(M, H, heads)
    step_bytes = float(sum(nbytes.values()))
    desc = (f"fused producers + 1x128 quant (adanorm, quant_rms_fma, gated_attention, gelu quant), "
            f"one launch each over {M} tokens x {H} (BASELINE config 3 video stream)")
    if args.impl == "reference":
        if rank != 0:
            return
        rows = 64
        per_row, threads = cpu_producer_sample(rows)
        val = step_bytes / M / per_row / 1e9
        print(json.dumps({
            "metric": "blockwise-FP8 producers GB/s", "value": val, "unit": "GB/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_row * M * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": desc, "tokens_per_gpu": M, "sample_tokens": rows},
            "cpu_baseline": {"value": val, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": f"{rows} of {M} tokens per step, oracle restatement"},
            "e2e": {"value": val, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    import torch
    import torch.distributed as dist
    import ltx_kernels.blockwise.functional as F
    from ltx_kernels.blockwise import ops

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    x = torch.randn(B, S, H, generator=g, device=dev).to(torch.bfloat16)
    y = torch.randn(B, S, H, generator=g, device=dev).to(torch.bfloat16)
    sc = (torch.randn(B, 1, H, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    sh = (torch.randn(B, 1, H, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    z = (torch.randn(B, 1, H, generator=g, device=dev) * 0.01).to(torch.bfloat16)
    logits = (torch.randn(B, S, heads, generator=g, device=dev) * 3).to(torch.bfloat16)
    names = list(nbytes)

    from ltx_kernels import _lib as L

    def step(ev=None, mode=None):
        # the reference's GPU arithmetic (triton mode) unless told otherwise: the default
        # of the reference-named ops
        mode = L.QUANT_TRITON if mode is None else mode
        if ev:
            ev[0].record()
        ops.adanorm_quantize(x, sc, sh, mode)
        if ev:
            ev[1].record()
        ops.rms_fma(x, y, z, True, mode)
        if ev:
            ev[2].record()
        ops.gated_attention(y, logits, True, mode)
        if ev:
            ev[3].record()
        ops.gelu_quantize_1x128(y, mode)
        if ev:
            ev[4].record()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.steps):
        step(evs[i])
    t1.record()
    barrier()
    elapsed = t0.elapsed_time(t1)
    per_kernel = [sum(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(args.steps)) / args.steps
                  for j in range(4)]
    # the same launches in IEEE arithmetic (torch mode), reported beside
    for _ in range(2):
        step(mode=L.QUANT_TORCH)
    barrier()
    evt = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    for i in range(args.steps):
        step(evt[i], L.QUANT_TORCH)
    barrier()
    per_kernel_torch = [sum(evt[i][j].elapsed_time(evt[i][j + 1]) for i in range(args.steps)) / args.steps
                        for j in range(4)]

    # end to end through the reference-named ops: x, y from pinned host memory, codes back
    x_host, y_host = x.cpu().pin_memory(), y.cpu().pin_memory()
    q_host = torch.empty((B, S, H), dtype=torch.uint8).pin_memory()

    def e2e_step():
        xd, yd = x_host.to(dev, non_blocking=True), y_host.to(dev, non_blocking=True)
        F.blockwise_quantize_adanorm_triton(xd, None, sc, sh)
        q, _ = F.blockwise_quantize_rms_fma_triton(xd, yd, z)
        F.gated_attention_triton(yd, logits)
        torch.ops.blockwise.quantize(yd, True)
        q_host.copy_(q.view(torch.uint8), non_blocking=True)

    e2e_steps = max(3, min(args.steps, 10))
    for _ in range(2):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    clk = clocks.stop()
    assert ops.device_status() == 0
    if world > 1:
        t = torch.tensor([elapsed, e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed, e2e_ms = t.tolist()
    ms = elapsed / args.steps
    value = world * step_bytes / (ms * 1e-3) / 1e9
    dom = max(range(4), key=lambda j: per_kernel[j])
    achieved = nbytes[names[dom]] / (per_kernel[dom] * 1e-3) / 1e9
    peak, peak_src = None, None
    mp = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(mp):
        try:
            peak, peak_src = float(json.load(open(mp))["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (of measured)"
        except (ValueError, KeyError):
            peak = None
    if peak is None:
        peak, peak_src = 6650.0, "fallback 6.65 TB/s"
    traffic = None
    tpath = os.path.join(REPO, "profiles", "ncu_traffic.json")
    if os.path.exists(tpath):
        try:
            tr = json.load(open(tpath)).get(f"producers:{names[dom]}")
            traffic = tr["bytes_per_launch_at_bench_size"] if tr else None
        except (ValueError, KeyError):
            traffic = None
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            rows = 64
            per_row, threads = cpu_producer_sample(rows)
            cpu = {"value": step_bytes / M / per_row / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
                   "sample": f"{rows} of {M} tokens, the four producers restated by the oracle (scalar C)"}
        print(json.dumps({
            "metric": "blockwise-FP8 producers GB/s", "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 in, f32 math, e4m3 + f32 scales out",
            "data": "synthetic (seeded)",
            "config": {"workload": desc, "tokens_per_gpu": M, "hidden": H, "heads": heads,
                       "parallelism": f"token-sharded dp{world}", "l2": "working set > L2 (x, y 403 MB each); no flush"},
            "kernels_ms": {n: round(t, 4) for n, t in zip(names, per_kernel)},
            "kernels_gbs": {n: round(nbytes[n] / (t * 1e-3) / 1e9, 1) for n, t in zip(names, per_kernel)},
            "arithmetic": "triton mode (the reference's GPU arithmetic); torch mode in kernels_ms_torch_mode",
            "kernels_ms_torch_mode": {n: round(t, 4) for n, t in zip(names, per_kernel_torch)},
            "kernels_gbs_torch_mode": {n: round(nbytes[n] / (t * 1e-3) / 1e9, 1) for n, t in zip(names, per_kernel_torch)},
            "roofline": {"bound": "hbm", "kernel": names[dom], "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": peak_src, "traffic": traffic},
            "cpu_baseline": cpu,
            "e2e": {"value": world * step_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": 2 * M * H * 2, "d2h_bytes_per_step": M * H},
            "gpu_launches": args.steps * 4,
            "clocks": clk}))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="dit_step",
                    choices=["dit_step"] + sorted(WORKLOADS) + ["producers", "sweep", "fp6"])
    ap.add_argument("--scaling", default=None, choices=["weak", "strong"],
                    help="dit_step: strong (default) splits one step's tokens over the ranks, weak gives every "
                         "rank a full step")
    ap.add_argument("--blocks", type=int, default=DIT_BLOCKS, help="dit_step: transformer blocks per step")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--m", type=int, default=0, help="tokens per GPU (default: the workload's)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="dit_step: skip the headline-GEMM, GPU-reference and cuBLAS measurements")
    ap.add_argument("--e2e-chunk", type=int, default=2048,
                    help="ffn/linear/qkv_lora e2e: tokens per streamed chunk (0: whole batch, copies not overlapped)")
    ap.add_argument("--no-graph", action="store_true", help="dit_step: launch every GEMM from Python instead of "
                                                             "replaying a captured CUDA graph")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = _env_int("RANK", 0)
    world = _env_int("WORLD_SIZE", 1)
    local = _env_int("LOCAL_RANK", 0)
    if args.workload == "dit_step":
        return run_dit(args, rank, world, local)
    if args.workload == "producers":
        return run_producers(args, rank, world, local)
    if args.workload == "sweep":
        return run_sweep(args, rank, world, local)
    if args.workload == "fp6":
        return run_fp6(args, rank, world, local)
    return run_single(args, rank, world, local)


if __name__ == "__main__":
    main()
