"""Serving decode loop: preallocated caches and one CUDA-graph replay per generated token.

:func:`generate_tokens` follows the reference's loop (``inference/generation.py:54-266``): every
token re-enters Python, re-allocates the MLA latent cache (``torch.cat``), builds new KDA state
tensors and launches a few hundred small kernels.  :class:`GraphDecoder` keeps the same model
and the same prefill, then

* moves the prefill cache into serving buffers sized for ``max_length`` tokens: the KDA
  recurrent states and conv histories are advanced IN PLACE by the decode kernels
  (``KDAState(inplace=True)``), the MLA latents live in a :class:`StaticMLACache`
  ``[B, max_length, L]`` that appends one row per step in place;
* captures one decode step -- embedding, every layer, LM head, the fused sampling kernel
  (repetition-penalty bitmap, temperature, top-k, top-p, Philox draw keyed by a device
  counter), EOS bookkeeping and the write of the token into a device output buffer -- in a
  CUDA graph, and replays it once per token.  The host reads the device only every
  ``eos_check_every`` tokens (to stop early) and once at the end.

Finished rows keep decoding (their tokens are replaced by the pad id, as in the reference,
whose outputs for finished rows are also the pad id), so every replay does the same work.
Off CUDA (or with ``use_graph=False``) the same step runs eagerly through the PyTorch paths.
"""
from __future__ import annotations

import contextlib
import copy
import time

import torch
import torch.nn as nn

from ..models.backbone import HybridBackboneCache, HybridLayerCache
from ..models.kda import KDAState
from ..models.mla import MLACache, StaticMLACache
from ..models.primitives import ShortConvState
from ..runtime import sync_free
from .session import cache_summary
from .config import GenerationConfig
from .generation import GenerationOutput, last_prompt_logits
from .sampling import sample_next_token


def _shared_handles(model: nn.Module) -> dict:
    """Deep-copy memo that keeps process groups and symmetric-memory workspaces shared: they are
    process-wide rendezvous objects (a copy of a sharded model talks to the same peers)."""
    import torch.distributed as dist
    memo = {}
    kinds = (dist.ProcessGroup,) if dist.is_available() else ()
    for mod in model.modules():
        for value in vars(mod).values():
            if (kinds and isinstance(value, kinds)) or getattr(value, "_kimi_rendezvous", False):
                memo[id(value)] = value
    return memo


def serving_copy(model: nn.Module, dtype: torch.dtype, *, inplace: bool = False) -> nn.Module:
    """``model`` (or a copy of it, unless ``inplace``) with its projection matrices (every
    ``nn.Linear`` weight and the stacked routed-expert weights) stored in ``dtype``, so decode
    steps under autocast read them without a per-step cast.  Embeddings, norms, conv and decay
    parameters keep their dtype; a LM head tied to the embedding gets its own ``dtype`` copy.
    Process groups and peer-memory workspaces of a sharded model are shared, not copied."""
    from ..models.moe import GroupedRoutedExperts
    m = model if inplace else copy.deepcopy(model, _shared_handles(model))
    for mod in m.modules():
        if isinstance(mod, nn.Linear):
            mod.weight = nn.Parameter(mod.weight.detach().to(dtype), requires_grad=False)
        elif isinstance(mod, GroupedRoutedExperts):
            for name in ("gate_proj", "up_proj", "down_proj"):
                setattr(mod, name, nn.Parameter(getattr(mod, name).detach().to(dtype), requires_grad=False))
    return m.eval()


def _static_layer(lc: HybridLayerCache, max_length: int) -> HybridLayerCache:
    s = lc.state
    if isinstance(s, KDAState):
        return HybridLayerCache("kda", KDAState(s.recurrent_state.float().clone(),
                                                ShortConvState(s.q_conv_state.buffer.clone()),
                                                ShortConvState(s.k_conv_state.buffer.clone()),
                                                ShortConvState(s.v_conv_state.buffer.clone()),
                                                s.sequence_offset.clone(), inplace=True))
    if isinstance(s, MLACache):
        return HybridLayerCache("gated_mla", StaticMLACache.from_cache(s, max_length))
    raise TypeError(f"unsupported layer cache {type(s).__name__}")


def _load_static_layer(static: HybridLayerCache, lc: HybridLayerCache) -> None:
    """Refill a serving layer cache in place from a prefill cache (the captured step keeps
    reading the same tensors)."""
    s, src = static.state, lc.state
    if isinstance(s, KDAState):
        s.recurrent_state.copy_(src.recurrent_state)
        for dst, new in ((s.q_conv_state, src.q_conv_state), (s.k_conv_state, src.k_conv_state),
                         (s.v_conv_state, src.v_conv_state)):
            dst.buffer.copy_(new.buffer)
        s.sequence_offset.copy_(src.sequence_offset)
        return
    t = src.latent_kv.shape[1]
    if t > s.latent_kv.shape[1]:
        raise ValueError(f"prompt of {t} tokens exceeds the serving cache ({s.latent_kv.shape[1]})")
    s.latent_kv[:, :t].copy_(src.latent_kv)
    if src.attention_mask is not None:
        s.latent_kv[:, :t].mul_(src.attention_mask[..., None].to(s.latent_kv.dtype))
    s.sequence_offset.copy_(src.sequence_offset)


def _state_tensors(cache: HybridBackboneCache) -> list:
    out = []
    for lc in cache.layer_caches:
        s = lc.state
        if isinstance(s, KDAState):
            out += [s.recurrent_state, s.q_conv_state.buffer, s.k_conv_state.buffer, s.v_conv_state.buffer,
                    s.sequence_offset]
        else:
            out += [s.latent_kv, s.sequence_offset]
    return out


class GraphDecoder:
    """Greedy or sampled generation with a captured decode step.

    ``max_length`` bounds prompt + generated tokens (the MLA latent buffers are sized for it).
    ``autocast_dtype`` (bf16 by default on CUDA, None to disable) is the compute dtype of the
    prefill and of every decode step; with it the decoder serves from :func:`serving_copy` of the
    model (projection matrices stored in that dtype; ``copy_model=False`` converts the model itself
    instead of a copy, for a model loaded only to serve)."""

    def __init__(self, model, *, max_length: int, generation_config: GenerationConfig | None = None,
                 use_graph: bool | None = None, autocast_dtype: torch.dtype | None = torch.bfloat16,
                 copy_model: bool = True):
        self.max_length = int(max_length)
        self.cfg = generation_config or GenerationConfig()
        dev = next(model.parameters()).device
        self.device = dev
        self.use_graph = (dev.type == "cuda") if use_graph is None else bool(use_graph and dev.type == "cuda")
        self.autocast_dtype = autocast_dtype if dev.type == "cuda" else None
        self.model = (serving_copy(model, self.autocast_dtype, inplace=not copy_model)
                      if self.autocast_dtype is not None else model)
        self.graph = None
        self.replays = 0
        self._key = None

    # ------------------------------------------------------------------ helpers
    def _autocast(self):
        if self.autocast_dtype is None:
            return contextlib.nullcontext()
        return torch.autocast("cuda", dtype=self.autocast_dtype)

    def _sample(self, logits: torch.Tensor) -> torch.Tensor:
        """[B, V] -> [B] int64, on the device without host synchronisation."""
        cfg = self.cfg
        if self.device.type == "cuda":
            from .. import ops
            nxt = ops.sample_tokens(logits, self.seen, cfg, self.seed_offset)
            self.seed_offset[1:].add_(1)
            return nxt
        return sample_next_token(logits.float(), cfg, previous_token_ids=self.history, generator=self.gen)[:, 0]

    def _emit(self, nxt: torch.Tensor) -> None:
        """Record one sampled token per row (pad for finished rows) and feed it back."""
        cfg = self.cfg
        pad = cfg.pad_token_id if cfg.pad_token_id is not None else cfg.eos_token_id
        if pad is not None:
            nxt = torch.where(self.finished, torch.full_like(nxt, int(pad)), nxt)
        # the output column never leaves the buffer, however many steps a caller runs
        col = self.step.clamp(max=self.out.shape[1] - 1)
        self.out.scatter_(1, col.view(1, 1).expand(nxt.shape[0], 1), nxt[:, None])
        self.step.add_(1)
        if cfg.eos_token_id is not None:
            self.finished |= nxt.eq(int(cfg.eos_token_id))
        if self.device.type == "cuda":
            if self.seen is not None:
                from .. import ops
                ops.mark_seen(self.seen, nxt[:, None], self.vocab)
        else:
            self.history = torch.cat((self.history, nxt[:, None]), dim=1)
        self.tok.copy_(nxt[:, None])

    def _decode_step(self) -> None:
        with self._autocast(), sync_free(True, all_valid_mask=True):
            out = self.model(input_ids=self.tok, cache=self.cache, use_cache=True, return_dict=True)
        new = out.cache
        for dst, src in zip(_state_tensors(self.cache), _state_tensors(new)):
            if dst.data_ptr() != src.data_ptr():
                dst.copy_(src)
        self._emit(self._sample(out.logits[:, -1, :]))

    # ------------------------------------------------------------------ API
    @torch.inference_mode()
    def generate(self, input_ids: torch.Tensor, attention_mask: torch.Tensor | None = None, *,
                 prefill_kwargs: dict | None = None) -> GenerationOutput:
        """``prefill_kwargs`` go to the prompt's forward only (``pixel_values``, ``video_values``, their
        counts and masks): the visual inputs are consumed by the prefill, decode steps are text."""
        cfg, model, dev = self.cfg, self.model, self.device
        input_ids = input_ids.to(device=dev, dtype=torch.long)
        if input_ids.ndim != 2 or input_ids.shape[1] == 0:
            raise ValueError("input_ids must have shape [B,T], T > 0")
        if attention_mask is None:
            attention_mask = (torch.ones_like(input_ids, dtype=torch.bool) if cfg.pad_token_id is None
                              else input_ids.ne(cfg.pad_token_id))
        attention_mask = attention_mask.to(dev)
        b, width = input_ids.shape
        steps = cfg.max_new_tokens
        reason = "length"
        if cfg.max_total_tokens is not None and max(cfg.max_total_tokens - width, 0) < steps:
            steps, reason = max(cfg.max_total_tokens - width, 0), "max_total_tokens"
        if width + steps > self.max_length:
            raise ValueError(f"prompt ({width}) + new tokens ({steps}) exceed max_length {self.max_length}")
        was_training = model.training
        model.eval()
        sync = (lambda: torch.cuda.synchronize(dev)) if dev.type == "cuda" else (lambda: None)
        try:
            sync()
            t0 = time.perf_counter()
            with self._autocast():
                pre = model(input_ids=input_ids, attention_mask=attention_mask, use_cache=True, return_dict=True,
                            **(prefill_kwargs or {}))
            logits = last_prompt_logits(pre.logits, attention_mask)
            self.vocab = int(logits.shape[-1])
            pen = cfg.repetition_penalty not in (None, 1)
            # the captured step bakes in the batch shape and the sampling / EOS settings
            key = (b, self.vocab, pen, cfg.do_sample, cfg.temperature, cfg.top_k, cfg.top_p, cfg.repetition_penalty,
                   cfg.eos_token_id, cfg.pad_token_id)
            if self.graph is not None and self._key == key:
                # same batch shape as the captured step: refill its buffers in place, replay it
                for static, lc in zip(self.cache.layer_caches, pre.cache.layer_caches):
                    _load_static_layer(static, lc)
                self.cache = HybridBackboneCache(self.cache.layer_caches, pre.cache.sequence_length)
                for t in (self.tok, self.out, self.step, self.finished):
                    t.zero_()
            else:
                self.release()
                self._key = key
                self.cache = HybridBackboneCache(tuple(_static_layer(lc, self.max_length)
                                                       for lc in pre.cache.layer_caches), pre.cache.sequence_length)
                self.tok = torch.zeros(b, 1, dtype=torch.long, device=dev)
                self.out = torch.zeros(b, self.max_length, dtype=torch.long, device=dev)
                self.step = torch.zeros((), dtype=torch.long, device=dev)
                self.finished = torch.zeros(b, dtype=torch.bool, device=dev)
                self.seen = self.seed_offset = None
            if dev.type == "cuda":
                from .. import ops
                if pen:
                    if self.seen is None:
                        self.seen = torch.zeros(b, (self.vocab + 31) // 32, dtype=torch.int32, device=dev)
                    self.seen.zero_()
                    ops.mark_seen(self.seen, input_ids, self.vocab)
                seed = cfg.seed if cfg.seed is not None else int(torch.randint(0, 2 ** 62, ()).item())
                seed_offset = torch.tensor([seed, 0], dtype=torch.long)
                if self.seed_offset is None:
                    self.seed_offset = seed_offset.to(dev)
                else:
                    self.seed_offset.copy_(seed_offset)
            else:
                self.seen = None
                self.history = input_ids.clone()
                self.gen = torch.Generator().manual_seed(cfg.seed) if cfg.seed is not None else None
            sync()
            prefill_s = time.perf_counter() - t0
            t1 = time.perf_counter()
            n = 0
            if steps > 0:
                self._emit(self._sample(logits))
                n = 1
                if self.use_graph and steps > 1 and self.graph is None:
                    self._capture()
                check = max(int(cfg.eos_check_every), 1)
                while n < steps:
                    if cfg.eos_token_id is not None and n % check == 0 and bool(self.finished.all()):
                        reason = "eos"
                        break
                    if self.graph is not None:
                        self.graph.replay()
                        self.replays += 1
                    else:
                        self._decode_step()
                    n += 1
                if (reason != "eos" and cfg.eos_token_id is not None and n % check == 0
                        and bool(self.finished.all())):
                    reason = "eos"
            sync()
            decode_s = time.perf_counter() - t1
        finally:
            if was_training:
                model.train()
        self.cache = HybridBackboneCache(self.cache.layer_caches, int(self.cache.sequence_lengths.max().item()))
        gen_ids = self.out[:, :n].clone()
        total_s = prefill_s + decode_s
        return GenerationOutput(input_ids, torch.cat((input_ids, gen_ids), 1), gen_ids, None, None, reason,
                                self.cache if cfg.return_cache else None, cache_summary(self.cache), None, width, n,
                                prefill_s, decode_s, total_s, n / decode_s if decode_s > 0 else 0.0,
                                n * b / decode_s if decode_s > 0 else 0.0)

    def _capture(self) -> None:
        """Warm the decode step up eagerly on a side stream (restoring every buffer it advanced),
        then capture it."""
        bufs = _state_tensors(self.cache) + [self.tok, self.out, self.step, self.finished, self.seed_offset]
        if self.seen is not None:
            bufs.append(self.seen)
        snapshot = [t.clone() for t in bufs]
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(2):
                self._decode_step()
        torch.cuda.current_stream(self.device).wait_stream(side)
        for dst, src in zip(bufs, snapshot):
            dst.copy_(src)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._decode_step()
        torch.cuda.synchronize(self.device)

    def release(self) -> None:
        """Drop the captured step (required before destroying a process group it uses)."""
        self.graph = None
        self._key = None


def graph_generate(model, input_ids, *, max_length: int | None = None,
                   generation_config: GenerationConfig | None = None, attention_mask=None,
                   use_graph: bool | None = None, prefill_kwargs: dict | None = None) -> GenerationOutput:
    """One-call form of :class:`GraphDecoder` (``max_length`` defaults to prompt + new tokens)."""
    cfg = generation_config or GenerationConfig()
    ml = max_length if max_length is not None else int(input_ids.shape[1]) + cfg.max_new_tokens
    return GraphDecoder(model, max_length=ml, generation_config=cfg, use_graph=use_graph).generate(
        input_ids, attention_mask, prefill_kwargs=prefill_kwargs)


__all__ = ["GraphDecoder", "graph_generate", "serving_copy"]
