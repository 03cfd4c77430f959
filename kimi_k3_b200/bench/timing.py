"""Device timing helpers shared by the benchmarks.

CUDA work is timed with events on the launching stream after warm-up, with a
synchronize on both sides; between timed repeats an L2-sized buffer can be
overwritten so that every repeat starts cold (B200 L2 is 126 MB; the flush
buffer is 256 MB). On CPU the same calls fall back to ``time.perf_counter``.
Roofline fractions use the measured copy bandwidth and cuBLAS bf16 throughput
of ``MEASURED_PEAKS.json`` at the repository root when it exists.
"""
from __future__ import annotations

import json
import os
import resource
import statistics
import sys
import time
from dataclasses import dataclass

import torch

_FLUSH_BYTES = 256 << 20
_flush_buf: dict = {}

# Used when the measured-peaks file is absent: an earlier measurement on B200
# (STREAM-style copy, cuBLAS bf16 8192^3 burst).
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def measured_peaks() -> dict:
    """``{'hbm_gbs', 'bf16_tflops', 'bf16_tflops_sustained', 'source'}``."""
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    path = os.path.join(root, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            data = json.load(fh)
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]),
                "bf16_tflops_sustained": float(data.get("bf16_tflops_sustained", data["bf16_tflops"])),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK_PEAKS, source="fallback")


def flush_l2(device) -> None:
    """Overwrite a buffer twice the size of the L2 cache on ``device``."""
    key = str(device)
    buf = _flush_buf.get(key)
    if buf is None:
        buf = torch.empty(_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
        _flush_buf[key] = buf
    buf.fill_(1.0)


@dataclass
class Timing:
    median_ms: float
    min_ms: float
    samples: list

    def as_dict(self) -> dict:
        return {"median_ms": round(self.median_ms, 4), "min_ms": round(self.min_ms, 4), "repeats": len(self.samples)}


def time_fn(fn, *, device=None, warmup: int = 3, repeats: int = 10, flush: bool = True) -> Timing:
    """Time ``fn()`` per call. CUDA: events around each call (L2 flushed before each one
    when ``flush``); CPU: wall clock."""
    is_cuda = device is not None and torch.device(device).type == "cuda"
    for _ in range(max(warmup, 0)):
        fn()
    samples = []
    if is_cuda:
        torch.cuda.synchronize(device)
        for _ in range(repeats):
            if flush:
                flush_l2(device)
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record()
            fn()
            end.record()
            end.synchronize()
            samples.append(start.elapsed_time(end))
        torch.cuda.synchronize(device)
    else:
        for _ in range(repeats):
            t0 = time.perf_counter()
            fn()
            samples.append((time.perf_counter() - t0) * 1e3)
    return Timing(statistics.median(samples), min(samples), samples)


def roofline(ms: float, *, flops: float | None = None, bytes_moved: float | None = None,
             sustained: bool = False) -> dict:
    """Achieved rates and fractions of the measured peaks for one call of ``ms`` milliseconds."""
    peaks = measured_peaks()
    out = {}
    if flops:
        tflops = flops / (ms * 1e-3) / 1e12
        peak = peaks["bf16_tflops_sustained" if sustained else "bf16_tflops"]
        out.update(tflops=round(tflops, 2), tensor_frac=round(tflops / peak, 4))
    if bytes_moved:
        gbs = bytes_moved / (ms * 1e-3) / 1e9
        out.update(gbs=round(gbs, 1), hbm_frac=round(gbs / peaks["hbm_gbs"], 4))
    out["peaks"] = peaks["source"]
    return out


def process_peak_memory_bytes() -> int:
    """Peak resident set size of this process (bytes)."""
    peak = resource.getrusage(resource.RUSAGE_SELF).ru_maxrss
    return int(peak if sys.platform == "darwin" else peak * 1024)


def device_peak_bytes(device) -> int:
    if device is not None and torch.device(device).type == "cuda":
        return int(torch.cuda.max_memory_allocated(device))
    return 0
