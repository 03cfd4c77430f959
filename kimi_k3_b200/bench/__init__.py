"""Benchmarks: device-timed kernel microbenchmarks and module-level benchmarks.

``python -m kimi_k3_b200.bench kernels <case> ...`` times one hand-written kernel;
``python -m kimi_k3_b200.bench <module> ...`` runs a module benchmark (KDA, MLA, MoE,
MTP, backbone, attention residuals, diagnostics levels) and prints CSV or JSON.
"""
from .timing import flush_l2, measured_peaks, roofline, time_fn

__all__ = ["flush_l2", "measured_peaks", "roofline", "time_fn"]
