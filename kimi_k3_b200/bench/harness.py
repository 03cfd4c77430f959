"""Shared pieces of the benchmark entry point (``bench.py``): clock sampling during the timed
region, rank helpers, seeded synthetic batches.  Nothing here touches a model."""
from __future__ import annotations

import os
import statistics
import subprocess
import threading

import torch


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names, parts[3:7]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world, local):
    torch.cuda.set_device(local)
    if world > 1 and not torch.distributed.is_initialized():
        from datetime import timedelta
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=600),
                                             device_id=torch.device("cuda", local))


def max_over_ranks(value: float) -> float:
    if torch.distributed.is_initialized():
        t = torch.tensor([value], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())
    return value


def barrier():
    if torch.distributed.is_initialized():
        torch.distributed.barrier()


def make_batches(n, batch, seq, vocab, seed, device=None, pin=False):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        ids = torch.randint(0, vocab, (batch, seq + 1), generator=g)
        b = {"input_ids": ids[:, :-1].contiguous(), "labels": ids[:, 1:].contiguous(),
             "attention_mask": torch.ones(batch, seq, dtype=torch.bool)}
        if pin:
            b = {k: v.pin_memory() for k, v in b.items()}
        if device is not None:
            b = {k: v.to(device) for k, v in b.items()}
        out.append(b)
    return out


__all__ = ["ClockSampler", "dist_env", "init_dist", "max_over_ranks", "barrier", "make_batches"]
