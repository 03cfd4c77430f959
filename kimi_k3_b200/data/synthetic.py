"""Deterministic synthetic long-context key-value retrieval data.

Parity: ``data/synthetic_long_context_retrieval.py:41-458`` (reference). The example format
and the random draws that produce each example (a per-index ``random.Random(seed + idx)``,
then key sample, value choices, one filler per fact, a filler run sized to fit the block,
query and answer) follow the reference exactly, so the same configuration yields the same
token sequences in both implementations; the tokenizer (``<pad> <bos> <eos> <unk>``,
structural words, ``key_i``, ``value_i``, ``filler_i``) assigns the same ids.
"""
from __future__ import annotations

import random
from dataclasses import dataclass

import torch
from torch.utils.data import DataLoader, Dataset


@dataclass
class SyntheticRetrievalConfig:
    num_train_examples: int = 50_000
    num_val_examples: int = 5_000
    block_size: int = 64
    min_filler_tokens: int = 64
    max_filler_tokens: int = 420
    num_keys_per_example: int = 8
    vocab_filler_size: int = 550
    num_key_types: int = 128
    num_value_types: int = 256
    batch_size: int = 32
    num_workers: int = 0
    seed: int = 42

    def validate(self) -> None:
        if self.num_train_examples <= 0 or self.num_val_examples <= 0:
            raise ValueError("dataset sizes must be positive")
        if self.block_size <= 0 or self.batch_size <= 0:
            raise ValueError("block_size and batch_size must be positive")
        if self.num_keys_per_example <= 0:
            raise ValueError("num_keys_per_example must be positive")
        if self.num_keys_per_example > self.num_key_types:
            raise ValueError("num_keys_per_example cannot exceed num_key_types")
        if self.min_filler_tokens < 0 or self.max_filler_tokens < self.min_filler_tokens:
            raise ValueError("invalid filler-token range")


STRUCTURAL = ("key", "is", "question", "what", "?", "answer", ":", "noise", "the", "and", "then", "because",
              "context", "remember", "value", "token")


class SimpleWordTokenizer:
    """Whitespace tokenizer over a closed vocabulary."""

    def __init__(self):
        self.special_tokens = ["<pad>", "<bos>", "<eos>", "<unk>"]
        self.token_to_idx: dict = {}
        self.idx_to_token: dict = {}
        for t in self.special_tokens:
            self.add_token(t)

    def add_token(self, token: str) -> None:
        if token not in self.token_to_idx:
            i = len(self.token_to_idx)
            self.token_to_idx[token] = i
            self.idx_to_token[i] = token

    def build_vocab(self, cfg: SyntheticRetrievalConfig) -> None:
        for t in STRUCTURAL:
            self.add_token(t)
        for prefix, n in (("key", cfg.num_key_types), ("value", cfg.num_value_types),
                          ("filler", cfg.vocab_filler_size)):
            for i in range(n):
                self.add_token(f"{prefix}_{i}")

    def encode(self, text: str) -> list:
        unk = self.token_to_idx["<unk>"]
        return [self.token_to_idx.get(t, unk) for t in text.strip().split()]

    def decode(self, ids) -> str:
        return " ".join(self.idx_to_token.get(int(i), "<unk>") for i in ids)

    def token_to_id(self, token: str):
        return self.token_to_idx.get(token)

    @property
    def vocab_size(self) -> int:
        return len(self.token_to_idx)

    @property
    def pad_id(self) -> int:
        return self.token_to_idx["<pad>"]

    @property
    def bos_id(self) -> int:
        return self.token_to_idx["<bos>"]

    @property
    def eos_id(self) -> int:
        return self.token_to_idx["<eos>"]


class SyntheticRetrievalGenerator:
    """``<bos> key_a is value_x filler ... filler... question : what is key_a ? answer : value_x <eos>``."""

    def __init__(self, cfg: SyntheticRetrievalConfig, tokenizer: SimpleWordTokenizer, seed: int = 42):
        cfg.validate()
        self.cfg, self.tokenizer = cfg, tokenizer
        self.rng = random.Random(seed)
        self.keys = [f"key_{i}" for i in range(cfg.num_key_types)]
        self.values = [f"value_{i}" for i in range(cfg.num_value_types)]
        self.fillers = [f"filler_{i}" for i in range(cfg.vocab_filler_size)]

    def _fill(self, n: int) -> list:
        return [self.rng.choice(self.fillers) for _ in range(n)]

    def generate_text_example(self):
        c, rng = self.cfg, self.rng
        keys = rng.sample(self.keys, c.num_keys_per_example)
        vals = [rng.choice(self.values) for _ in range(c.num_keys_per_example)]
        kv = dict(zip(keys, vals))
        query = rng.choice(keys)
        answer = kv[query]
        toks = ["<bos>"]
        for k, v in kv.items():
            toks += [k, "is", v]
            toks += self._fill(1)
        room = max(0, c.block_size + 1 - len(toks) - 10)  # the query/answer/eos suffix needs 10 tokens
        hi = min(c.max_filler_tokens, room)
        lo = min(c.min_filler_tokens, hi)
        n = rng.randint(lo, hi)
        toks += self._fill(n)
        toks += ["question", ":", "what", "is", query, "?", "answer", ":", answer, "<eos>"]
        return " ".join(toks), {"query_key": query, "answer_value": answer, "kv_pairs": kv, "filler_len": n}


class SyntheticRetrievalDataset(Dataset):
    """Map-style: index ``i`` always yields the example of seed ``base_seed + i``."""

    def __init__(self, cfg: SyntheticRetrievalConfig, tokenizer: SimpleWordTokenizer, split: str = "train",
                 mtp_depth: int = 0):
        if split not in ("train", "val"):
            raise ValueError("split must be 'train' or 'val'")
        self.cfg, self.tokenizer, self.split, self.mtp_depth = cfg, tokenizer, split, int(mtp_depth)
        self.num_examples = cfg.num_train_examples if split == "train" else cfg.num_val_examples
        self.base_seed = cfg.seed if split == "train" else cfg.seed + 10_000
        self.pad_id = tokenizer.pad_id
        self.block_size = cfg.block_size

    def __len__(self) -> int:
        return self.num_examples

    def _fit(self, ids: list, n: int) -> list:
        return ids[:n] if len(ids) >= n else ids + [self.pad_id] * (n - len(ids))

    def example_ids(self, idx: int) -> list:
        text, _ = SyntheticRetrievalGenerator(self.cfg, self.tokenizer, seed=self.base_seed + int(idx)) \
            .generate_text_example()
        return self.tokenizer.encode(text)

    def __getitem__(self, idx):
        b = self.block_size
        ids = torch.tensor(self._fit(self.example_ids(idx), b + 1 + self.mtp_depth), dtype=torch.long)
        inp = ids[:b]
        out = {"input_ids": inp, "labels": ids[1:b + 1]}
        if self.mtp_depth:
            out["mtp_labels"] = torch.stack([ids[k:k + b] for k in range(2, 2 + self.mtp_depth)])
        else:
            out["attention_mask"] = inp.ne(self.pad_id)
        return out


class SyntheticRetrievalMTPDataset(SyntheticRetrievalDataset):
    """Adds ``mtp_labels [depth, block]`` (targets x[t+2], x[t+3], ...)."""

    def __init__(self, cfg, tokenizer, split: str = "train", mtp_depth: int = 1):
        super().__init__(cfg, tokenizer, split, mtp_depth=mtp_depth)


def create_synthetic_retrieval_dataloaders(cfg: SyntheticRetrievalConfig | None = None, use_mtp: bool = False,
                                           mtp_depth: int = 1):
    """``(train_loader, val_loader, tokenizer)``."""
    cfg = cfg or SyntheticRetrievalConfig()
    cfg.validate()
    tok = SimpleWordTokenizer()
    tok.build_vocab(cfg)
    depth = mtp_depth if use_mtp else 0
    train = SyntheticRetrievalDataset(cfg, tok, "train", mtp_depth=depth)
    val = SyntheticRetrievalDataset(cfg, tok, "val", mtp_depth=depth)
    pin = torch.cuda.is_available()
    return (DataLoader(train, batch_size=cfg.batch_size, shuffle=True, num_workers=cfg.num_workers, pin_memory=pin),
            DataLoader(val, batch_size=cfg.batch_size, shuffle=False, num_workers=cfg.num_workers, pin_memory=pin),
            tok)


class SyntheticTokenDataset(Dataset):
    """Uniform random token blocks (benchmarks and smoke tests): seeded per index."""

    def __init__(self, num_examples: int, block_size: int, vocab_size: int, seed: int = 0):
        self.n, self.block, self.vocab, self.seed = int(num_examples), int(block_size), int(vocab_size), int(seed)

    def __len__(self) -> int:
        return self.n

    def __getitem__(self, idx):
        g = torch.Generator().manual_seed(self.seed * 1_000_003 + int(idx))
        ids = torch.randint(0, self.vocab, (self.block + 1,), generator=g)
        return {"input_ids": ids[:-1], "labels": ids[1:], "attention_mask": torch.ones(self.block, dtype=torch.bool)}


__all__ = ["SyntheticRetrievalConfig", "SimpleWordTokenizer", "SyntheticRetrievalGenerator",
           "SyntheticRetrievalDataset", "SyntheticRetrievalMTPDataset", "create_synthetic_retrieval_dataloaders",
           "SyntheticTokenDataset"]
