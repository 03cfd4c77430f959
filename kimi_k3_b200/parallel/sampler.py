"""Resumable distributed sampler over the data-parallel x expert-parallel replicas.

Parity: ``training/distributed/sampler.py:8-38`` (reference): shards the dataset over
``DP * EP`` replicas (tensor-parallel peers see the same data), seeded per epoch, with a
cursor so a resumed run continues from the next unseen sample.
"""
from __future__ import annotations

import math

import torch
from torch.utils.data import Sampler


class StatefulDistributedSampler(Sampler):
    def __init__(self, dataset, num_replicas: int | None = None, rank: int | None = None, shuffle: bool = True,
                 seed: int = 0, drop_last: bool = False):
        import torch.distributed as dist
        if num_replicas is None:
            num_replicas = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
        if rank is None:
            rank = dist.get_rank() if dist.is_available() and dist.is_initialized() else 0
        if num_replicas <= 0 or not 0 <= rank < num_replicas:
            raise ValueError("invalid sampler replica configuration")
        self.dataset = dataset
        self.num_replicas, self.rank = int(num_replicas), int(rank)
        self.shuffle, self.seed, self.drop_last = bool(shuffle), int(seed), bool(drop_last)
        self.epoch = 0
        self.cursor = 0
        n = len(dataset)
        if drop_last and n % num_replicas:
            self.num_samples = n // num_replicas
        else:
            self.num_samples = math.ceil(n / num_replicas)
        self.total_size = self.num_samples * num_replicas

    def _indices(self) -> list:
        n = len(self.dataset)
        if self.shuffle:
            g = torch.Generator().manual_seed(self.seed + self.epoch)
            idx = torch.randperm(n, generator=g).tolist()
        else:
            idx = list(range(n))
        if self.drop_last:
            idx = idx[: self.total_size]
        elif len(idx) < self.total_size:
            pad = self.total_size - len(idx)
            idx += (idx * math.ceil(pad / max(len(idx), 1)))[:pad]
        return idx[self.rank: self.total_size: self.num_replicas]

    def __iter__(self):
        idx = self._indices()[self.cursor:]
        for i in idx:
            self.cursor += 1
            yield i

    def __len__(self) -> int:
        return self.num_samples - self.cursor

    def set_epoch(self, epoch: int) -> None:
        self.epoch = int(epoch)
        self.cursor = 0

    def state_dict(self) -> dict:
        return {"epoch": self.epoch, "cursor": self.cursor, "seed": self.seed, "num_replicas": self.num_replicas,
                "rank": self.rank}

    def load_state_dict(self, state: dict) -> None:
        if int(state.get("num_replicas", self.num_replicas)) != self.num_replicas or \
                int(state.get("seed", self.seed)) != self.seed:
            raise ValueError("sampler state is incompatible with this topology")
        epoch, cursor = int(state["epoch"]), int(state["cursor"])
        if epoch < 0 or cursor < 0:
            raise ValueError("sampler epoch and cursor must be non-negative")
        self.epoch, self.cursor = epoch, cursor


__all__ = ["StatefulDistributedSampler"]
