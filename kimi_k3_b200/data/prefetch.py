"""Device prefetching: the next batches are pinned and copied host-to-device on a side
CUDA stream while the current step runs (the reference moves each batch synchronously on
the compute stream, ``training/autocast.py:move_batch_to_device``)."""
from __future__ import annotations

from collections import deque

import torch


def _pin(batch: dict) -> dict:
    return {k: (v.pin_memory() if torch.is_tensor(v) and not v.is_pinned() else v) for k, v in batch.items()}


class DevicePrefetcher:
    """Iterate ``loader`` yielding device batches ``depth`` steps ahead of use."""

    def __init__(self, loader, device, depth: int = 2, normalize=None):
        self.loader, self.device, self.depth = loader, torch.device(device), max(1, int(depth))
        self.normalize = normalize
        self.stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None

    def __iter__(self):
        queue = deque()
        it = iter(self.loader)

        def push():
            try:
                raw = next(it)
            except StopIteration:
                return False
            b = self.normalize(raw) if self.normalize else raw
            if self.stream is None:
                queue.append((b, None))
                return True
            b = _pin(b)
            with torch.cuda.stream(self.stream):
                dev = {k: (v.to(self.device, non_blocking=True) if torch.is_tensor(v) else v) for k, v in b.items()}
                ev = torch.cuda.Event()
                ev.record(self.stream)
            queue.append((dev, ev))
            return True

        for _ in range(self.depth):
            if not push():
                break
        while queue:
            b, ev = queue.popleft()
            if ev is not None:
                torch.cuda.current_stream(self.device).wait_event(ev)
                for v in b.values():
                    if torch.is_tensor(v):
                        v.record_stream(torch.cuda.current_stream(self.device))
            push()
            yield b

    def __len__(self):
        return len(self.loader)


__all__ = ["DevicePrefetcher"]
