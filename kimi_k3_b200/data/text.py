"""Causal-LM text corpora: presets, byte-level BPE tokenizer, fixed-length blocks.

Parity: ``data/text_datasets.py:41-442`` (reference): the same presets (wikitext2, tinystories,
ag_news, imdb, minipile, fineweb-edu 10BT, fineweb 10/100/350BT), a byte-level BPE tokenizer
(NFKC, ``<unk> <pad> <bos> <eos>``) trained once and cached, documents wrapped in
``<bos> ... <eos>``, concatenated and cut into ``block + 1`` chunks (inputs / shifted labels).

Offline use: ``load_hf_text_splits`` reads the Hugging Face cache only when no network is
available (``HF_DATASETS_OFFLINE``); ``local_files`` presets (``local:<path or glob>``) read
plain-text files, one document per blank-line separated paragraph.
"""
from __future__ import annotations

import glob
from dataclasses import dataclass
from pathlib import Path
from typing import Iterable, Iterator, Optional

import torch
from torch.utils.data import DataLoader, Dataset


@dataclass(frozen=True)
class HFTextDatasetPreset:
    name: str
    dataset_name: str
    subset: Optional[str]
    text_field: str
    train_split: str
    validation_split: Optional[str]
    recommended_block_size: int
    notes: str


@dataclass(frozen=True)
class TextDataloaderConfig:
    preset_name: str = "wikitext2"
    block_size: Optional[int] = None
    batch_size: int = 8
    num_workers: int = 0
    tokenizer_path: Optional[str | Path] = None
    vocab_size: int = 16_000
    min_frequency: int = 2
    max_tokenizer_documents: Optional[int] = 50_000
    max_train_documents: Optional[int] = 20_000
    max_validation_documents: Optional[int] = 2_000
    streaming: bool = False

    def __post_init__(self) -> None:
        if self.block_size is not None and self.block_size <= 0:
            raise ValueError("block_size must be None or positive")
        if self.batch_size <= 0 or self.num_workers < 0:
            raise ValueError("batch_size must be positive and num_workers non-negative")
        if self.vocab_size <= 0 or self.min_frequency <= 0:
            raise ValueError("tokenizer sizes must be positive")
        for name in ("max_tokenizer_documents", "max_train_documents", "max_validation_documents"):
            v = getattr(self, name)
            if v is not None and v <= 0:
                raise ValueError(f"{name} must be None or positive")


def _p(name, ds, subset, tr, va, block, notes):
    return HFTextDatasetPreset(name, ds, subset, "text", tr, va, block, notes)


HF_TEXT_DATASETS = {p.name: p for p in (
    _p("wikitext2", "Salesforce/wikitext", "wikitext-2-raw-v1", "train", "validation", 256,
       "Small Wikipedia long-form language-modeling benchmark."),
    _p("tinystories", "roneneldan/TinyStories", None, "train", "validation", 256,
       "Simple-story corpus useful for tiny LMs and qualitative generation."),
    _p("ag_news", "fancyzhx/ag_news", None, "train", "test", 128, "Short news articles."),
    _p("imdb", "stanfordnlp/imdb", "plain_text", "train", "test", 256, "Movie reviews."),
    _p("minipile", "JeanKaddour/minipile", None, "train", "validation", 256, "Small diverse pretraining mix."),
    _p("fineweb_edu_10bt_mincols", "EliMC/fineweb-edu-10BT-mincols", None, "train", None, 512,
       "Educational web sample; use streaming or max_*_documents for local runs."),
    _p("fineweb_10bt", "HuggingFaceFW/fineweb", "sample-10BT", "train", None, 2048, "FineWeb 10B-token sample."),
    _p("fineweb_100bt", "HuggingFaceFW/fineweb", "sample-100BT", "train", None, 4096, "FineWeb 100B-token sample."),
    _p("fineweb_350bt", "HuggingFaceFW/fineweb", "sample-350BT", "train", None, 8192, "FineWeb 350B-token sample."),
)}


def available_hf_text_dataset_presets() -> list:
    return sorted(HF_TEXT_DATASETS)


def resolve_hf_text_preset(name: str) -> HFTextDatasetPreset:
    if name.startswith("local:"):
        return HFTextDatasetPreset(name, name[len("local:"):], None, "text", "train", None, 256, "local text files")
    try:
        return HF_TEXT_DATASETS[name]
    except KeyError as exc:
        raise KeyError(f"Unknown dataset preset {name!r}. Available: {sorted(HF_TEXT_DATASETS)}") from exc


def iter_texts(split, text_field: str = "text", max_documents: Optional[int] = None) -> Iterator[str]:
    n = 0
    for ex in split:
        t = ex.get(text_field) if isinstance(ex, dict) else ex
        if isinstance(t, str) and t.strip():
            yield t
            n += 1
            if max_documents is not None and n >= max_documents:
                break


def _local_documents(pattern: str) -> list:
    docs = []
    for f in sorted(glob.glob(pattern)) or ([pattern] if Path(pattern).is_file() else []):
        for para in Path(f).read_text(encoding="utf-8").split("\n\n"):
            if para.strip():
                docs.append({"text": para})
    if not docs:
        raise FileNotFoundError(f"no text documents found for {pattern!r}")
    return docs


def load_hf_text_splits(preset_name: str, *, streaming: bool = False) -> dict:
    preset = resolve_hf_text_preset(preset_name)
    if preset_name.startswith("local:"):
        docs = _local_documents(preset.dataset_name)
        cut = max(1, len(docs) // 20)
        return {"train": docs[cut:] or docs, "validation": docs[:cut]}
    from datasets import load_dataset
    args = (preset.dataset_name,) if preset.subset is None else (preset.dataset_name, preset.subset)
    return load_dataset(*args, streaming=streaming)


def train_byte_level_bpe_tokenizer(texts: Iterable[str], *, vocab_size: int = 16_000, min_frequency: int = 2,
                                   save_path=None):
    from tokenizers import Tokenizer, decoders, models, normalizers, pre_tokenizers, trainers
    tok = Tokenizer(models.BPE(unk_token="<unk>"))
    tok.normalizer = normalizers.Sequence([normalizers.NFKC()])
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=int(vocab_size), min_frequency=int(min_frequency),
                                  special_tokens=["<unk>", "<pad>", "<bos>", "<eos>"])
    tok.train_from_iterator(texts, trainer=trainer)
    if save_path is not None:
        Path(save_path).parent.mkdir(parents=True, exist_ok=True)
        tok.save(str(save_path))
    return tok


def load_or_train_byte_level_tokenizer(train_split, *, text_field: str = "text", tokenizer_path, vocab_size=16_000,
                                       min_frequency=2, max_tokenizer_documents: Optional[int] = 50_000):
    from tokenizers import Tokenizer
    path = Path(tokenizer_path)
    if path.exists():
        return Tokenizer.from_file(str(path))
    return train_byte_level_bpe_tokenizer(iter_texts(train_split, text_field, max_tokenizer_documents),
                                          vocab_size=vocab_size, min_frequency=min_frequency, save_path=path)


class CausalTextDataset(Dataset):
    """Documents -> ``<bos> ids <eos>`` concatenation -> ``[n, block + 1]`` chunks (one tensor)."""

    def __init__(self, texts: Iterable[str], tokenizer, *, block_size: int = 256, max_documents: Optional[int] = None):
        if block_size <= 0:
            raise ValueError(f"block_size must be > 0, got {block_size}")
        self.block_size = int(block_size)
        bos, eos, pad = (tokenizer.token_to_id(t) for t in ("<bos>", "<eos>", "<pad>"))
        if bos is None or eos is None or pad is None:
            raise ValueError("Tokenizer must define <bos>, <eos>, and <pad> tokens.")
        ids: list = []
        for i, text in enumerate(texts):
            if max_documents is not None and i >= max_documents:
                break
            if isinstance(text, str) and text.strip():
                ids.append(bos)
                ids.extend(tokenizer.encode(text).ids)
                ids.append(eos)
        chunk = self.block_size + 1
        if len(ids) < chunk:
            raise ValueError(f"Not enough tokens ({len(ids)}) to build one block of length {chunk}.")
        n = len(ids) // chunk
        blocks = torch.tensor(ids[: n * chunk], dtype=torch.long).view(n, chunk)
        self.input_ids = blocks[:, :-1].contiguous()
        self.labels = blocks[:, 1:].contiguous()

    def __len__(self) -> int:
        return int(self.input_ids.shape[0])

    def __getitem__(self, idx):
        return {"input_ids": self.input_ids[idx], "labels": self.labels[idx]}


def create_hf_text_dataloaders(preset_name: str, *, block_size=None, batch_size: int = 8, num_workers: int = 0,
                               tokenizer_path=None, vocab_size: int = 16_000, min_frequency: int = 2,
                               max_tokenizer_documents=50_000, max_train_documents=20_000,
                               max_validation_documents=2_000, streaming: bool = False):
    preset = resolve_hf_text_preset(preset_name)
    splits = load_hf_text_splits(preset_name, streaming=streaming)
    train = splits[preset.train_split]
    val = splits[preset.validation_split] if preset.validation_split and preset.validation_split in splits else None
    if val is None and preset_name.startswith("local:"):
        val = splits.get("validation")
    block = int(block_size or preset.recommended_block_size)
    path = Path(tokenizer_path or f"data/cache/tokenizers/{preset.name.replace(':', '_').replace('/', '_')}.json")
    tok = load_or_train_byte_level_tokenizer(train, text_field=preset.text_field, tokenizer_path=path,
                                             vocab_size=vocab_size, min_frequency=min_frequency,
                                             max_tokenizer_documents=max_tokenizer_documents)
    pin = torch.cuda.is_available()
    train_ds = CausalTextDataset(iter_texts(train, preset.text_field), tok, block_size=block,
                                 max_documents=max_train_documents)
    val_loader = None
    if val is not None:
        try:
            val_ds = CausalTextDataset(iter_texts(val, preset.text_field), tok, block_size=block,
                                       max_documents=max_validation_documents)
            val_loader = DataLoader(val_ds, batch_size=batch_size, shuffle=False, num_workers=num_workers,
                                    pin_memory=pin)
        except ValueError:
            val_loader = None  # too little validation text for one block
    return (DataLoader(train_ds, batch_size=batch_size, shuffle=True, num_workers=num_workers, pin_memory=pin),
            val_loader, tok)


def create_text_dataloaders(cfg: TextDataloaderConfig, *, use_mtp: bool = False):
    """Uniform entry point (labels are already shifted; MTP targets are derived by the model)."""
    del use_mtp
    return create_hf_text_dataloaders(cfg.preset_name, block_size=cfg.block_size, batch_size=cfg.batch_size,
                                      num_workers=cfg.num_workers, tokenizer_path=cfg.tokenizer_path,
                                      vocab_size=cfg.vocab_size, min_frequency=cfg.min_frequency,
                                      max_tokenizer_documents=cfg.max_tokenizer_documents,
                                      max_train_documents=cfg.max_train_documents,
                                      max_validation_documents=cfg.max_validation_documents, streaming=cfg.streaming)


__all__ = ["HFTextDatasetPreset", "TextDataloaderConfig", "HF_TEXT_DATASETS", "available_hf_text_dataset_presets",
           "resolve_hf_text_preset", "iter_texts", "load_hf_text_splits", "train_byte_level_bpe_tokenizer",
           "load_or_train_byte_level_tokenizer", "CausalTextDataset", "create_hf_text_dataloaders",
           "create_text_dataloaders"]
