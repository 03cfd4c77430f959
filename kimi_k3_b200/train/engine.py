"""One-optimizer-step training engine used by the trainer loop and ``bench.py``.

A step = (optional pinned host -> device copy) -> bf16 autocast forward with the
fused head losses (no ``[N, V]`` logits) -> backward -> global-norm clip on the
device -> hybrid optimizer -> scheduler -> Quantile-Balancing commit.

Two execution modes:

* eager: the clip coefficient is applied without a host round trip; the host syncs are
  the loss normalisers and the optimizer's single finite-gradient check;
* CUDA graph (``cuda_graph=True``): after ``graph_warmup`` sync-free eager steps the
  whole step (forward, backward, clip, Muon + AdamW + QK-Clip, QB commit) is captured
  once and replayed. Host-side validation runs on the host copy of each batch; the
  finite check becomes a device flag (``found_inf``) that suppresses the update inside
  the graph; the host reads it one step later (scheduler and step counters follow).

Parity: the step semantics follow ``training/train_one_epoch.py:145-330`` (reference)
for a window of one micro-batch.
"""
from __future__ import annotations

from contextlib import nullcontext
from dataclasses import dataclass

import torch

from ..debug import nvtx


class KernelWaitError(RuntimeError):
    """A bounded wait inside one of the framework's kernels gave up during a training step."""


def kernel_status_words(device):
    """The device's default status words of the GEMM and KDA kernels (int32 views), or None."""
    if device.type != "cuda":
        return None
    from ..ops import _loader
    ext = _loader.load()
    if ext is None or not hasattr(ext, "status_words"):
        return None
    with torch.cuda.device(device):
        return ext.status_words()


def clear_kernel_status(device) -> None:
    from ..ops import _loader
    ext = _loader.require()
    with torch.cuda.device(device):
        ext.tc_gemm_status(True)
        ext.kda_tc_status(True)


@dataclass
class StepOutput:
    loss: torch.Tensor          # device scalar (total objective)
    ntp_loss: torch.Tensor
    mtp_loss: torch.Tensor | None
    grad_norm: torch.Tensor     # device scalar, pre-clip
    executed: bool


def move_batch(batch: dict, device, non_blocking: bool = True) -> dict:
    return {k: (v.to(device, non_blocking=non_blocking) if isinstance(v, torch.Tensor) else v)
            for k, v in batch.items()}


@torch.no_grad()
def clip_grad_norm_device(params, max_norm: float | None) -> torch.Tensor:
    """Global L2 norm of the gradients; scales them in place by min(1, max_norm/norm) on device."""
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return torch.zeros(())
    norms = torch._foreach_norm(grads, 2.0)
    total = torch.linalg.vector_norm(torch.stack([n.float() for n in norms]), 2.0)
    if max_norm is not None:
        coef = (max_norm / (total + 1e-6)).clamp(max=1.0)
        torch._foreach_mul_(grads, coef)
    return total


class TrainStepEngine:
    """Runs optimizer steps of a KimiK3 model (single process; the distributed runtime wraps it)."""

    def __init__(self, model, optimizer, *, scheduler=None, grad_clip: float | None = 1.0,
                 amp_dtype: torch.dtype | None = torch.bfloat16, use_mtp: bool = True, moe_controller=None,
                 grad_hook=None, cuda_graph: bool = False, graph_warmup: int = 2, grad_norm_fn=None):
        self.model = model
        self.optimizer = optimizer
        self.scheduler = scheduler
        self.grad_clip = grad_clip
        self.amp_dtype = amp_dtype
        self.use_mtp = use_mtp
        self.moe_controller = moe_controller
        self.grad_hook = grad_hook  # called after backward (gradient reduction in data parallel)
        # global gradient norm of a parallel plan (tensor / expert shards counted once, FSDP shards
        # all-reduced); None: the norm of this process's gradients
        self.grad_norm_fn = grad_norm_fn
        self.device = next(model.parameters()).device
        self._params = [p for p in model.parameters() if p.requires_grad]
        self.cuda_graph = bool(cuda_graph) and self.device.type == "cuda"
        self.graph_warmup = int(graph_warmup)
        self._graph = None
        self._static_in = None
        self._static_out = None
        self._graph_steps = 0
        self._pending = None  # (pinned found_inf copy or None, pinned kernel status, event) of the last step
        self._status_words = kernel_status_words(self.device)

    def _autocast(self, cache_enabled: bool = True):
        if self.amp_dtype is None or self.device.type != "cuda":
            return nullcontext()
        return torch.autocast("cuda", dtype=self.amp_dtype, cache_enabled=cache_enabled)

    def forward_loss(self, batch: dict, *, cache_enabled: bool = True):
        with self._autocast(cache_enabled):
            out = self.model(input_ids=batch["input_ids"], attention_mask=batch.get("attention_mask"),
                             labels=batch["labels"], use_mtp=self.use_mtp, compute_logits=False)
        return out

    # ------------------------------------------------------------------ eager
    def step(self, batch: dict, *, mask_all_valid: bool | None = None) -> StepOutput:
        """One optimizer step. ``mask_all_valid`` tells the CUDA-graph path that the batch's
        attention mask is all True (otherwise it is checked, on the host copy when there is one)."""
        if self.cuda_graph and self._graph_eligible(batch, mask_all_valid):
            return self._graph_step(batch)
        self._resolve_pending()
        if batch["input_ids"].device != self.device:
            batch = move_batch(batch, self.device)
        self.model.train()
        if self.moe_controller is not None:
            self.moe_controller.begin()
        try:
            with nvtx("forward"):
                out = self.forward_loss(batch)
            with nvtx("backward"):
                out.loss.backward()
            if self.grad_hook is not None:
                with nvtx("gradient sync"):
                    self.grad_hook()
            with nvtx("optimizer"):
                gnorm = self._clip()
                report = self.optimizer.step()
            executed = bool(getattr(report, "executed", True))
        except BaseException:
            if self.moe_controller is not None:
                self.moe_controller.discard()
            self.optimizer.zero_grad(set_to_none=True)
            raise
        if executed:
            if self.scheduler is not None:
                self.scheduler.step()
            if self.moe_controller is not None:
                self.moe_controller.commit()
        elif self.moe_controller is not None:
            self.moe_controller.discard()
        self.optimizer.zero_grad(set_to_none=True)
        status = self._status_snapshot()
        if status is not None:
            self._pending = (None, *self._to_host(status))
        lo = out.loss_output
        return StepOutput(out.loss.detach(), lo.ntp.loss.detach(), None if lo.mtp is None else lo.mtp.loss.detach(),
                          gnorm, executed)

    def _clip(self) -> torch.Tensor:
        if self.grad_norm_fn is None:
            return clip_grad_norm_device(self._params, self.grad_clip)
        total = self.grad_norm_fn()
        if self.grad_clip is not None:
            grads = [p.grad.to_local() if hasattr(p.grad, "to_local") else p.grad
                     for p in self._params if p.grad is not None]
            if grads:
                torch._foreach_mul_(grads, (self.grad_clip / (total + 1e-6)).clamp(max=1.0))
        return total

    # ------------------------------------------------------------------ kernel status
    def _status_snapshot(self):
        """Stream-ordered copy of the kernels' status words (int32 [2]: GEMM, KDA) or None."""
        if self._status_words is None:
            return None
        return torch.cat(self._status_words)

    @staticmethod
    def _to_host(t):
        host = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        host.copy_(t, non_blocking=True)
        event = torch.cuda.Event()
        event.record()
        return host, event

    def _check_status(self, status) -> None:
        if status is None:
            return
        gemm, kda = (int(v) for v in status.tolist())
        if gemm or kda:
            clear_kernel_status(self.device)
            raise KernelWaitError(
                f"a bounded wait inside a kernel gave up (GEMM status {gemm}, KDA status {kda}); the results of "
                "the last step are not valid. Codes: 1-4 GEMM pipeline roles, 5 peer flag, 6 drain, 11-31 KDA MMAs")

    # ------------------------------------------------------------------ CUDA graph
    @staticmethod
    def _mask_is_all_valid(batch, hint):
        if hint is not None:
            return bool(hint)
        mask = batch.get("attention_mask")
        if mask is None:
            return False  # the model would derive it from pad ids: let the eager path decide
        return bool(mask.all())  # a host tensor is free; a device tensor costs one sync

    def _graph_eligible(self, batch, hint) -> bool:
        if self._static_in is not None:
            for k, v in self._static_in.items():
                if k in batch and tuple(batch[k].shape) != tuple(v.shape):
                    return False
        return self._mask_is_all_valid(batch, hint)

    def _device_step_body(self, batch, *, cache_enabled: bool):
        """Forward, backward, clip, optimizer and QB commit with no host synchronisation."""
        from ..runtime import sync_free
        with sync_free(all_valid_mask=True):
            if self.moe_controller is not None:
                self.moe_controller.begin()
            with nvtx("forward"):
                out = self.forward_loss(batch, cache_enabled=cache_enabled)
            with nvtx("backward"):
                out.loss.backward()
            if self.grad_hook is not None:
                with nvtx("gradient sync"):
                    self.grad_hook()
            with nvtx("optimizer"):
                gnorm = self._clip()
                found_inf = ~torch.isfinite(gnorm)
                self.optimizer.step(found_inf=found_inf)
            if self.moe_controller is not None:
                self.moe_controller.commit(keep_old=found_inf)
        lo = out.loss_output
        return (out.loss.detach(), lo.ntp.loss.detach(), None if lo.mtp is None else lo.mtp.loss.detach(),
                gnorm.detach(), found_inf)

    def _resolve_pending(self) -> None:
        """Read the previous replay's skip flag; advance the scheduler only for executed steps."""
        if self._pending is None:
            return
        flag, status, event = self._pending
        self._pending = None
        event.synchronize()
        self._check_status(status)
        if flag is None:
            return
        if bool(flag.item()):
            if hasattr(self.optimizer, "undo_step_count"):
                self.optimizer.undo_step_count()
        elif self.scheduler is not None:
            self.scheduler.step()

    def _load_static(self, batch) -> None:
        for k, dst in self._static_in.items():
            src = batch.get(k)
            if src is None:
                dst.fill_(True)
            else:
                dst.copy_(src, non_blocking=True)

    def _graph_step(self, batch) -> StepOutput:
        self._resolve_pending()
        self.model.train()
        mirror = getattr(self.optimizer, "weight_mirror", None)
        if mirror is not None:
            # a master changed outside the optimizer since the last step (checkpoint load, EMA
            # swap): the replay reads the bf16 mirrors, so bring them up to date first
            mirror.refresh_if_stale()
        if self._static_in is None:
            if hasattr(self.optimizer, "use_device_lrs"):
                self.optimizer.use_device_lrs()
            ids = batch["input_ids"]
            self._static_in = {"input_ids": torch.empty(ids.shape, dtype=ids.dtype, device=self.device),
                               "labels": torch.empty(batch["labels"].shape, dtype=batch["labels"].dtype,
                                                     device=self.device),
                               "attention_mask": torch.ones(ids.shape, dtype=torch.bool, device=self.device)}
        self._load_static(batch)
        if self._graph_steps < self.graph_warmup:
            # Sync-free eager steps on a side stream: they fill optimizer state and the
            # kernels' one-time set-up, as capture requires.
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self.optimizer.zero_grad(set_to_none=True)
                res = self._device_step_body(self._static_in, cache_enabled=False)
            torch.cuda.current_stream().wait_stream(side)
            res = (*res, self._status_snapshot())
        else:
            if self._graph is None:
                self.optimizer.zero_grad(set_to_none=True)
                self._graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self._graph):
                    body = self._device_step_body(self._static_in, cache_enabled=False)
                    self._static_out = (*body, self._status_snapshot())
            self._graph.replay()
            res = self._static_out
        self._graph_steps += 1
        loss, ntp, mtp, gnorm, found_inf, status = res
        flag = torch.empty((), dtype=torch.bool, pin_memory=True)
        flag.copy_(found_inf, non_blocking=True)
        host_status = None
        if status is not None:
            host_status = torch.empty(status.shape, dtype=status.dtype, pin_memory=True)
            host_status.copy_(status, non_blocking=True)
        event = torch.cuda.Event()
        event.record()
        self._pending = (flag, host_status, event)
        return StepOutput(loss, ntp, mtp, gnorm, True)

    def finish(self) -> None:
        """Settle the bookkeeping of the last replayed step (call before reading the
        scheduler or saving a checkpoint)."""
        self._resolve_pending()

    def release_graph(self) -> None:
        """Drop the captured graph (required before destroying a process group it uses)."""
        self.finish()
        self._graph = None
        self._static_out = None


class MoEController:
    """Open / commit / discard Quantile-Balancing windows on every balanced MoE layer.

    Parity: ``training/moe_control.py:10-57`` (reference).  ``reducer`` (expert / data
    parallel) makes the window statistics global before the bias update.
    """

    def __init__(self, model, reducer=None):
        from ..models.moe import StableLatentMoE
        raw = model.module if hasattr(model, "module") else model
        self.layers = tuple(m for m in raw.modules()
                            if isinstance(m, StableLatentMoE) and m.config.enable_quantile_balancing)
        self.reducer = reducer
        self.window_open = False

    def begin(self) -> None:
        if self.window_open:
            raise RuntimeError("a Quantile Balancing window is already open")
        for layer in self.layers:
            layer.begin_balance_accumulation()
        self.window_open = True

    def commit(self, keep_old=None):
        """Commit every layer's next bias; ``keep_old`` (device bool) keeps the old biases."""
        if not self.window_open:
            raise RuntimeError("no Quantile Balancing window is open")
        updates = tuple(layer.finalize_and_commit_balance(self.reducer, keep_old=keep_old) for layer in self.layers)
        self.window_open = False
        return updates

    def discard(self) -> None:
        if not self.window_open:
            return
        for layer in self.layers:
            layer.discard_balance_accumulation()
        self.window_open = False

    def assert_clean(self) -> None:
        if self.window_open:
            raise RuntimeError("checkpoint requested with an open QB window")
