"""Progressive Context Curriculum (PCC): token-count stages of growing context length.

Parity: ``training/context_curriculum/{config,curriculum,batching,loader}.py`` (reference).
Stages are ``(max_seq_len, until_tokens)`` with strictly increasing lengths and token limits
and an open-ended last stage; the state machine only reports the active length (the trainer
rebuilds its loader on a transition, optimizer and scheduler state are preserved); the
collator clips samples to the active length, pads dynamically (right padding) and trims the
batch to its longest valid row. Checkpoint state and its compatibility checks follow the
reference field for field.

B200 addition: ``length_multiple`` rounds the trimmed batch length up (to a multiple, capped
at the stage length) so a stage sees a handful of shapes, each of which can keep a captured
CUDA graph; ``length_multiple=1`` reproduces the reference exactly.
"""
from __future__ import annotations

import inspect
from collections.abc import Callable, Mapping, Sequence
from dataclasses import asdict, dataclass, field
from typing import Literal

import torch
from torch.utils.data._utils.collate import default_collate


# --------------------------------------------------------------------------- config
@dataclass(frozen=True)
class ContextStage:
    max_seq_len: int
    until_tokens: int | None

    def __post_init__(self) -> None:
        if self.max_seq_len <= 0:
            raise ValueError("context stage max_seq_len must be positive")
        if self.until_tokens is not None and self.until_tokens <= 0:
            raise ValueError("context stage until_tokens must be positive")


def default_stages() -> tuple:
    return (ContextStage(512, 20_000_000), ContextStage(1024, 40_000_000), ContextStage(2048, 60_000_000),
            ContextStage(4096, 80_000_000), ContextStage(8192, None))


@dataclass(frozen=True)
class ContextCurriculumConfig:
    enabled: bool = False
    stages: tuple = field(default_factory=default_stages)
    transition_unit: Literal["tokens"] = "tokens"
    reset_dataloader_on_transition: bool = True
    preserve_optimizer_state: bool = True
    preserve_scheduler_state: bool = True

    def __post_init__(self) -> None:
        stages = tuple(ContextStage(**s) if isinstance(s, dict) else s for s in self.stages)
        object.__setattr__(self, "stages", stages)
        if not stages:
            raise ValueError("context curriculum stages must not be empty")
        lens = [s.max_seq_len for s in stages]
        if any(b <= a for a, b in zip(lens, lens[1:])):
            raise ValueError("stage max_seq_len values must strictly increase")
        if stages[-1].until_tokens is not None:
            raise ValueError("the final context stage must be open-ended")
        finite = [s.until_tokens for s in stages[:-1]]
        if any(v is None for v in finite):
            raise ValueError("only the final stage may be open-ended")
        if any(b <= a for a, b in zip(finite, finite[1:])):
            raise ValueError("until_tokens values must strictly increase")
        if self.transition_unit != "tokens":
            raise ValueError("tokens are the only supported transition unit")
        if not self.preserve_optimizer_state:
            raise ValueError("PCC cannot reset optimizer state")
        if not self.preserve_scheduler_state:
            raise ValueError("PCC cannot reset scheduler state")

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: dict) -> "ContextCurriculumConfig":
        return cls(**values)


# --------------------------------------------------------------------------- state machine
@dataclass
class ContextCurriculumState:
    stage_index: int
    max_seq_len: int
    tokens_seen: int
    transition_count: int = 0


@dataclass(frozen=True)
class ContextTransition:
    old_stage_index: int
    new_stage_index: int
    old_max_seq_len: int
    new_max_seq_len: int
    tokens_seen_at_transition: int

    def to_dict(self) -> dict:
        return asdict(self)


class ProgressiveContextCurriculum:
    """Reports the active context length; never touches model, optimizer or scheduler."""

    def __init__(self, config: ContextCurriculumConfig, *, training_max_seq_len: int,
                 model_max_seq_len: int | None = None, mtp_min_seq_len: int = 1):
        if training_max_seq_len <= 0:
            raise ValueError("training_max_seq_len must be positive")
        if model_max_seq_len is not None and model_max_seq_len <= 0:
            raise ValueError("model_max_seq_len must be positive")
        if mtp_min_seq_len <= 0:
            raise ValueError("mtp_min_seq_len must be positive")
        self.config = config
        self.training_max_seq_len = int(training_max_seq_len)
        self.model_max_seq_len = None if model_max_seq_len is None else int(model_max_seq_len)
        self.mtp_min_seq_len = int(mtp_min_seq_len)
        if config.enabled:
            if config.stages[-1].max_seq_len > self._limit():
                raise ValueError("context stage exceeds the model/training max_seq_len")
            if config.stages[0].max_seq_len < self.mtp_min_seq_len:
                raise ValueError("first context stage is too short for enabled MTP")
            start = config.stages[0].max_seq_len
        else:
            start = self._limit()
        self.state = ContextCurriculumState(0, start, 0, 0)
        self.last_transition: ContextTransition | None = None

    def _limit(self) -> int:
        return min(self.training_max_seq_len, self.model_max_seq_len or self.training_max_seq_len)

    @property
    def enabled(self) -> bool:
        return self.config.enabled

    @property
    def stage_index(self) -> int:
        return self.state.stage_index

    def current_max_seq_len(self) -> int:
        return self.state.max_seq_len

    def validate_sequence_length(self, sequence_length: int) -> None:
        if sequence_length > self.current_max_seq_len():
            raise ValueError(f"batch sequence length {sequence_length} exceeds active context length "
                             f"{self.current_max_seq_len()}")

    def validate_valid_tokens(self, valid_tokens_per_sample) -> None:
        if bool((valid_tokens_per_sample < self.mtp_min_seq_len).any()):
            raise ValueError("a context-curriculum sample has too few valid tokens for MTP")

    def stage_for_tokens(self, tokens_seen: int) -> int:
        idx = 0
        stages = self.config.stages
        while idx < len(stages) - 1 and stages[idx].until_tokens is not None and tokens_seen >= stages[idx].until_tokens:
            idx += 1
        return idx

    def update(self, tokens_seen: int) -> bool:
        if tokens_seen < self.state.tokens_seen:
            raise ValueError("context curriculum tokens_seen cannot move backward")
        self.state.tokens_seen = int(tokens_seen)
        self.last_transition = None
        if not self.enabled:
            return False
        old = self.state.stage_index
        new = max(old, self.stage_for_tokens(tokens_seen))
        if new == old:
            return False
        old_len = self.state.max_seq_len
        self.state.stage_index = new
        self.state.max_seq_len = self.config.stages[new].max_seq_len
        self.state.transition_count += 1
        self.last_transition = ContextTransition(old, new, old_len, self.state.max_seq_len, int(tokens_seen))
        return True

    def metrics(self) -> dict:
        s = self.state
        return {"context/stage_index": float(s.stage_index), "context/max_seq_len": float(s.max_seq_len),
                "context/tokens_seen": float(s.tokens_seen), "context/transition_count": float(s.transition_count)}

    def _compat(self) -> dict:
        c = self.config
        return {"enabled": self.enabled, "transition_unit": c.transition_unit,
                "reset_dataloader_on_transition": c.reset_dataloader_on_transition,
                "preserve_optimizer_state": c.preserve_optimizer_state,
                "preserve_scheduler_state": c.preserve_scheduler_state,
                "training_max_seq_len": self.training_max_seq_len, "model_max_seq_len": self.model_max_seq_len,
                "mtp_min_seq_len": self.mtp_min_seq_len}

    def state_dict(self) -> dict:
        s = self.state
        out = {"enabled": self.enabled, "stage_index": s.stage_index, "max_seq_len": s.max_seq_len,
               "tokens_seen": s.tokens_seen, "transition_count": s.transition_count,
               "stages": [asdict(st) for st in self.config.stages]}
        out.update({k: v for k, v in self._compat().items() if k != "enabled"})
        return out

    def load_state_dict(self, values: dict) -> None:
        if values.get("stages") != [asdict(st) for st in self.config.stages]:
            raise ValueError("checkpoint context stage definition is incompatible")
        for name, expected in self._compat().items():
            if values.get(name) != expected:
                raise ValueError(f"checkpoint context curriculum {name} is incompatible")
        index = int(values["stage_index"])
        if not 0 <= index < len(self.config.stages):
            raise ValueError("checkpoint context stage index is invalid")
        if index < self.state.stage_index:
            raise ValueError("checkpoint would move context curriculum backward")
        expected_len = self.config.stages[index].max_seq_len if self.enabled else self._limit()
        if int(values["max_seq_len"]) != expected_len:
            raise ValueError("checkpoint active context length is inconsistent")
        tokens = int(values["tokens_seen"])
        if tokens < 0:
            raise ValueError("checkpoint curriculum tokens_seen is invalid")
        if index != (self.stage_for_tokens(tokens) if self.enabled else 0):
            raise ValueError("checkpoint stage does not match its token count")
        self.state = ContextCurriculumState(index, expected_len, tokens, int(values.get("transition_count", index)))
        self.last_transition = None


# --------------------------------------------------------------------------- batching
SEQUENCE_KEYS = frozenset({"input_ids", "labels", "attention_mask", "segment_ids", "loss_mask", "boundary_mask",
                           "token_weights", "inputs_embeds"})
PAD_VALUES = {"input_ids": None, "labels": None, "attention_mask": False, "segment_ids": -1, "loss_mask": False,
              "boundary_mask": False, "token_weights": 0.0}


def _reject_packed(batch: dict, mask: torch.Tensor) -> None:
    seg = batch.get("segment_ids")
    if seg is None:
        return
    if seg.shape != mask.shape:
        raise ValueError("segment_ids must align with input_ids")
    for row_s, row_m in zip(seg, mask):
        if torch.unique(row_s[row_m]).numel() > 1:
            raise ValueError("packed documents are rejected: KDA/MLA currently have no segment-isolated attention "
                             "kernel")


def _visual_placeholders_kept(original_ids, kept_ids, token_id) -> bool:
    return torch.equal(original_ids.eq(token_id).sum(dim=1), kept_ids.eq(token_id).sum(dim=1))


def truncate_batch_to_context(batch: Mapping, max_seq_len: int, *, ignore_index: int = -100,
                              image_token_id: int | None = None, video_token_id: int | None = None,
                              length_multiple: int = 1):
    """Clip every sequence field to the active context, then to the longest valid row
    (rounded up to ``length_multiple`` when the batch is that wide). Returns ``(batch, stats)``."""
    if max_seq_len <= 0:
        raise ValueError("max_seq_len must be positive")
    ids = batch.get("input_ids")
    if not torch.is_tensor(ids):
        raise ValueError("context batching requires tensor input_ids")
    if ids.ndim != 2:
        raise ValueError("input_ids must have shape [B,T]")
    b, length = ids.shape
    out = dict(batch)
    target = min(length, int(max_seq_len))

    def clip(width):
        for name in SEQUENCE_KEYS:
            v = out.get(name)
            if v is None:
                continue
            if not torch.is_tensor(v):
                raise TypeError(f"{name} must be a tensor")
            if v.shape[0] != b or v.shape[1] < width:
                raise ValueError(f"{name} must align with input_ids")
            out[name] = v[:, :width].contiguous()

    for name in SEQUENCE_KEYS:
        v = out.get(name)
        if v is not None and torch.is_tensor(v) and tuple(v.shape[:2]) != (b, length):
            raise ValueError(f"{name} must align with input_ids")
    clip(target)
    mask = out.get("attention_mask")
    if mask is None:
        mask = out["attention_mask"] = torch.ones(b, target, dtype=torch.bool, device=ids.device)
    elif mask.dtype != torch.bool:
        raise TypeError("attention_mask must be boolean")
    if torch.any(mask.sum(dim=1) == 0):
        raise ValueError("context truncation produced an all-padding sample")
    if mask.shape[1] > 1 and torch.any((~mask[:, :-1]) & mask[:, 1:]):
        raise ValueError("context batching requires right-padded attention_mask rows")
    needed = max(1, min(int(mask.sum(dim=1).max().item()), target))
    if length_multiple > 1:
        needed = min(target, -(-needed // length_multiple) * length_multiple)
    if needed < target:
        clip(needed)
        target = needed
        mask = out["attention_mask"]
    _reject_packed(out, mask)
    seg = out.get("segment_ids")
    if seg is not None and "boundary_mask" not in out:
        bnd = torch.ones_like(mask)
        bnd[:, 1:] = seg[:, 1:].eq(seg[:, :-1])
        out["boundary_mask"] = bnd & mask
    for token_id, values_name in ((image_token_id, "pixel_values"), (video_token_id, "video_values")):
        if token_id is not None and out.get(values_name) is not None and \
                not _visual_placeholders_kept(ids, out["input_ids"], token_id):
            raise ValueError(f"context truncation would detach {values_name} from visual placeholder tokens")
    labels = out.get("labels")
    valid = (mask & labels.ne(ignore_index)).sum() if torch.is_tensor(labels) else mask.sum()
    return out, {"valid_tokens": float(valid.item()),
                 "padding_fraction": float(1.0 - mask.sum().item() / max(mask.numel(), 1)),
                 "sequence_length": float(target)}


def dynamic_collate(samples: Sequence[Mapping], pad_token_id: int, ignore_index: int) -> dict:
    """Right-pad per-sample sequences to the longest one."""
    if not samples:
        raise ValueError("cannot collate an empty sample list")
    lengths = [int(s["input_ids"].shape[0]) for s in samples]
    width = max(lengths)
    pads = dict(PAD_VALUES, input_ids=pad_token_id, labels=ignore_index)
    out = {}
    for name in set().union(*(s.keys() for s in samples)):
        vals = [s.get(name) for s in samples]
        if name in SEQUENCE_KEYS and all(torch.is_tensor(v) for v in vals):
            rows = []
            for v in vals:
                v = v[:width]
                missing = width - v.shape[0]
                if missing:
                    v = torch.cat((v, v.new_full((missing,) + tuple(v.shape[1:]), pads.get(name, 0))), 0)
                rows.append(v)
            out[name] = torch.stack(rows)
        elif all(v is not None for v in vals):
            out[name] = default_collate(vals)
    if "attention_mask" not in out:
        out["attention_mask"] = torch.arange(width)[None, :] < torch.tensor(lengths)[:, None]
    return out


def pad_batch_to(batch: dict, width: int, pad_token_id: int, ignore_index: int) -> dict:
    """Right-pad every ``[B, T, ...]`` sequence field of a collated batch to ``width``."""
    out = dict(batch)
    t = batch["input_ids"].shape[1]
    if width <= t:
        return out
    pads = dict(PAD_VALUES, input_ids=pad_token_id, labels=ignore_index)
    if "attention_mask" not in out:
        out["attention_mask"] = torch.ones_like(batch["input_ids"], dtype=torch.bool)
    for name in SEQUENCE_KEYS:
        v = out.get(name)
        if torch.is_tensor(v) and v.ndim >= 2 and v.shape[1] == t:
            fill = v.new_full((v.shape[0], width - t) + tuple(v.shape[2:]), pads.get(name, 0))
            out[name] = torch.cat((v, fill), dim=1)
    return out


class ProgressiveContextCollator:
    """Clip samples to the active context, collate (dynamic padding by default), trim."""

    def __init__(self, max_seq_len: int, *, base_collator: Callable | None = None, pad_token_id: int = 0,
                 ignore_index: int = -100, image_token_id: int | None = None, video_token_id: int | None = None,
                 length_multiple: int = 1):
        self.max_seq_len = int(max_seq_len)
        self.base_collator = base_collator
        self.pad_token_id = int(pad_token_id)
        self.ignore_index = int(ignore_index)
        self.image_token_id = image_token_id
        self.video_token_id = video_token_id
        self.length_multiple = int(length_multiple)

    def __call__(self, samples):
        clipped = []
        for sample in samples:
            s = dict(sample)
            ids = s.get("input_ids")
            for token_id, values_name in ((self.image_token_id, "pixel_values"), (self.video_token_id, "video_values")):
                if token_id is not None and s.get(values_name) is not None and torch.is_tensor(ids) and \
                        ids.eq(token_id).sum() != ids[: self.max_seq_len].eq(token_id).sum():
                    raise ValueError(f"context truncation would detach {values_name} from visual placeholder tokens")
            for name in SEQUENCE_KEYS:
                v = s.get(name)
                if torch.is_tensor(v) and v.ndim >= 1:
                    s[name] = v[: self.max_seq_len]
            clipped.append(s)
        batch = (self.base_collator(clipped) if self.base_collator is not None
                 else dynamic_collate(clipped, self.pad_token_id, self.ignore_index))
        if self.length_multiple > 1:
            width = batch["input_ids"].shape[1]
            batch = pad_batch_to(batch, min(self.max_seq_len, -(-width // self.length_multiple) * self.length_multiple),
                                 self.pad_token_id, self.ignore_index)
        return truncate_batch_to_context(batch, self.max_seq_len, ignore_index=self.ignore_index,
                                         image_token_id=self.image_token_id, video_token_id=self.video_token_id,
                                         length_multiple=self.length_multiple)[0]


def build_context_loader(factory, max_seq_len: int):
    """Call a loader factory with the active context length (keyword if it accepts one)."""
    if factory is None:
        raise ValueError("a train_loader_factory is required")
    params = inspect.signature(factory).parameters
    if "max_seq_len" in params or any(p.kind is inspect.Parameter.VAR_KEYWORD for p in params.values()):
        return factory(max_seq_len=max_seq_len)
    if any(p.kind in (inspect.Parameter.POSITIONAL_ONLY, inspect.Parameter.POSITIONAL_OR_KEYWORD)
           for p in params.values()):
        return factory(max_seq_len)
    raise TypeError("train_loader_factory must accept max_seq_len as an argument")


__all__ = ["ContextStage", "ContextCurriculumConfig", "ContextCurriculumState", "ContextTransition",
           "ProgressiveContextCurriculum", "truncate_batch_to_context", "dynamic_collate", "pad_batch_to",
           "ProgressiveContextCollator", "build_context_loader", "default_stages", "SEQUENCE_KEYS"]
