"""Strict ``data.yaml`` loading and the loader bundle handed to training.

Parity: ``data/yaml_config.py:35-365`` (reference): ``data: {name, kind, dataset, loader}``
with ``kind`` ``synthetic_retrieval`` or ``hf_text``, unknown keys rejected, batch size and
workers only under ``loader``; the bundle carries train/validation loaders, the tokenizer and
a ``train_loader_factory(max_seq_len)`` for the progressive context curriculum; with data or
expert parallelism the loaders use a resumable distributed sampler over the DP x EP replicas.
"""
from __future__ import annotations

from dataclasses import dataclass, replace
from pathlib import Path
from typing import Any, Literal

import torch
from torch.utils.data import DataLoader

from ..config.yaml_utils import ConfigError, dataclass_kwargs, expect_mapping, load_yaml_mapping, reject_unknown_keys
from ..parallel.sampler import StatefulDistributedSampler
from ..train.curriculum import ProgressiveContextCollator
from .synthetic import SyntheticRetrievalConfig, create_synthetic_retrieval_dataloaders
from .text import TextDataloaderConfig, create_text_dataloaders


@dataclass(frozen=True)
class LoaderConfig:
    batch_size: int = 8
    validation_batch_size: int | None = None
    num_workers: int = 0
    shuffle_train: bool = True
    pin_memory: bool | Literal["auto"] = "auto"
    persistent_workers: bool = False
    prefetch_factor: int | None = None
    drop_last: bool = False
    seed: int = 42

    def __post_init__(self) -> None:
        if self.batch_size <= 0:
            raise ValueError("loader.batch_size must be positive")
        if self.validation_batch_size is not None and self.validation_batch_size <= 0:
            raise ValueError("loader.validation_batch_size must be None or positive")
        if self.num_workers < 0:
            raise ValueError("loader.num_workers must be non-negative")
        if self.persistent_workers and self.num_workers == 0:
            raise ValueError("persistent_workers requires loader.num_workers > 0")
        if self.prefetch_factor is not None and (self.prefetch_factor <= 0 or self.num_workers == 0):
            raise ValueError("loader.prefetch_factor must be positive and requires loader.num_workers > 0")
        if self.pin_memory not in (True, False, "auto"):
            raise ValueError("loader.pin_memory must be true, false or 'auto'")

    @property
    def eval_batch_size(self) -> int:
        return self.validation_batch_size or self.batch_size

    @property
    def resolved_pin_memory(self) -> bool:
        return torch.cuda.is_available() if self.pin_memory == "auto" else bool(self.pin_memory)


@dataclass(frozen=True)
class DataPipelineConfig:
    name: str
    kind: Literal["synthetic_retrieval", "hf_text"]
    dataset: Any
    loader: LoaderConfig
    source_path: Path | None = None

    def __post_init__(self) -> None:
        if not self.name:
            raise ValueError("data.name must not be empty")
        if self.kind not in ("synthetic_retrieval", "hf_text"):
            raise ValueError("unsupported data.kind")

    @property
    def max_seq_len(self) -> int:
        b = getattr(self.dataset, "block_size", None)
        if b is None:
            raise ValueError("dataset.block_size must be explicit for YAML pipelines")
        return int(b)


@dataclass
class DataBundle:
    train_loader: DataLoader
    val_loader: DataLoader | None
    tokenizer: Any
    config: DataPipelineConfig
    train_loader_factory: Any

    @property
    def vocab_size(self) -> int:
        v = getattr(self.tokenizer, "vocab_size", None)
        if v is None and hasattr(self.tokenizer, "get_vocab_size"):
            v = self.tokenizer.get_vocab_size()
        if v is None:
            raise ValueError("tokenizer does not expose a vocabulary size")
        return int(v)

    def token_id(self, token: str) -> int | None:
        if hasattr(self.tokenizer, "token_to_id"):
            return self.tokenizer.token_to_id(token)
        attr = {"<pad>": "pad_id", "<bos>": "bos_id", "<eos>": "eos_id"}.get(token)
        return None if attr is None else getattr(self.tokenizer, attr, None)


def data_config_from_mapping(root: dict, source: Path | None = None) -> DataPipelineConfig:
    root = dict(root)
    data = dict(expect_mapping(root, "data", path="root"))
    reject_unknown_keys(root, path="root")
    name = str(data.pop("name", source.stem if source else "data"))
    kind = str(data.pop("kind", data.pop("type", "")))
    ds = dict(expect_mapping(data, "dataset", path="data"))
    lv = dict(expect_mapping(data, "loader", path="data"))
    reject_unknown_keys(data, path="data")
    loader = LoaderConfig(**dataclass_kwargs(lv, LoaderConfig, path="data.loader"))
    misplaced = {"batch_size", "num_workers"} & set(ds)
    if misplaced:
        raise ConfigError(f"configure {', '.join(sorted(misplaced))} only in data.loader, not data.dataset")
    ds.setdefault("batch_size", loader.batch_size)
    ds.setdefault("num_workers", loader.num_workers)
    if kind == "synthetic_retrieval":
        dataset = SyntheticRetrievalConfig(**dataclass_kwargs(ds, SyntheticRetrievalConfig, path="data.dataset"))
        dataset.validate()
    elif kind == "hf_text":
        dataset = TextDataloaderConfig(**dataclass_kwargs(ds, TextDataloaderConfig, path="data.dataset"))
        if dataset.block_size is None:
            raise ConfigError("data.dataset.block_size must be explicit in YAML")
    else:
        raise ConfigError("data.kind must be 'synthetic_retrieval' or 'hf_text'")
    return DataPipelineConfig(name, kind, dataset, loader, source)


def load_data_config(path) -> DataPipelineConfig:
    """Parse and validate a data YAML (no download, no tokenization)."""
    source, root = load_yaml_mapping(path)
    return data_config_from_mapping(root, source)


def _loader(dataset, cfg: LoaderConfig, *, train: bool, max_seq_len: int, pad_token_id: int, ignore_index: int = -100,
            distributed_context=None, length_multiple: int = 1) -> DataLoader:
    collate = ProgressiveContextCollator(max_seq_len, pad_token_id=pad_token_id, ignore_index=ignore_index,
                                         length_multiple=length_multiple)
    # The training loader always samples through the resumable sampler: its shuffle is seeded by
    # (seed, epoch), so a run resumed at epoch e sees exactly the batches it would have seen.
    sampler = None
    ctx = distributed_context
    replicas, rank = 1, 0
    if ctx is not None and getattr(ctx, "initialized", False):
        replicas = ctx.data_replicas if hasattr(ctx, "data_replicas") else ctx.dp_size * ctx.ep_size
        rank = ctx.dp_rank if getattr(ctx, "ep_overlays_tp", False) else ctx.dp_rank * ctx.ep_size + ctx.ep_rank
    if train or replicas > 1:
        sampler = StatefulDistributedSampler(dataset, num_replicas=replicas, rank=rank,
                                             shuffle=cfg.shuffle_train if train else False, seed=cfg.seed,
                                             drop_last=cfg.drop_last if train else False)
    kw = {} if cfg.num_workers == 0 or cfg.prefetch_factor is None else {"prefetch_factor": cfg.prefetch_factor}
    return DataLoader(dataset, batch_size=cfg.batch_size if train else cfg.eval_batch_size,
                      shuffle=cfg.shuffle_train if train and sampler is None else False, sampler=sampler,
                      num_workers=cfg.num_workers, pin_memory=cfg.resolved_pin_memory,
                      persistent_workers=cfg.persistent_workers, drop_last=cfg.drop_last if train else False,
                      generator=torch.Generator().manual_seed(cfg.seed), collate_fn=collate, **kw)


def build_dataloaders_from_yaml(path, *, distributed_context=None, length_multiple: int = 1) -> DataBundle:
    """Build loaders once; ``train_loader_factory(max_seq_len)`` rebuilds for a PCC stage."""
    cfg = load_data_config(path)
    return build_dataloaders(cfg, distributed_context=distributed_context, length_multiple=length_multiple)


def build_dataloaders(cfg: DataPipelineConfig, *, distributed_context=None, length_multiple: int = 1) -> DataBundle:
    ds_cfg = replace(cfg.dataset, batch_size=cfg.loader.batch_size, num_workers=cfg.loader.num_workers)
    if cfg.kind == "synthetic_retrieval":
        raw_train, raw_val, tok = create_synthetic_retrieval_dataloaders(ds_cfg, use_mtp=False)
    else:
        raw_train, raw_val, tok = create_text_dataloaders(ds_cfg, use_mtp=False)
    pad = tok.token_to_id("<pad>") if hasattr(tok, "token_to_id") else tok.pad_id

    def make_train_loader(max_seq_len: int):
        if max_seq_len > cfg.max_seq_len:
            raise ValueError(f"requested context {max_seq_len} exceeds data block_size {cfg.max_seq_len}")
        return _loader(raw_train.dataset, cfg.loader, train=True, max_seq_len=max_seq_len, pad_token_id=int(pad),
                       distributed_context=distributed_context, length_multiple=length_multiple)

    val = None if raw_val is None else _loader(raw_val.dataset, cfg.loader, train=False, max_seq_len=cfg.max_seq_len,
                                               pad_token_id=int(pad), distributed_context=distributed_context)
    return DataBundle(make_train_loader(cfg.max_seq_len), val, tok, cfg, make_train_loader)


def load_tokenizer_from_data_yaml(path):
    """The tokenizer a data YAML would use (synthetic vocabulary or the cached BPE file)."""
    cfg = load_data_config(path)
    if cfg.kind == "synthetic_retrieval":
        from .synthetic import SimpleWordTokenizer
        tok = SimpleWordTokenizer()
        tok.build_vocab(cfg.dataset)
        return tok
    from tokenizers import Tokenizer
    p = cfg.dataset.tokenizer_path
    if p is None or not Path(p).exists():
        raise FileNotFoundError(f"tokenizer file {p!r} not found; build the data pipeline once to train it")
    return Tokenizer.from_file(str(p))


__all__ = ["LoaderConfig", "DataPipelineConfig", "DataBundle", "data_config_from_mapping", "load_data_config",
           "build_dataloaders_from_yaml", "build_dataloaders", "load_tokenizer_from_data_yaml"]
