"""The generic (architecture-neutral) optimizers: plain Muon, Muon + AdamW by name rules, AdamW.

Parity: ``training/muon_optimizer.py:20-728`` and ``training/adam_optimizer.py:11-62`` (reference).
These predate the Kimi-aware optimizer of :mod:`kimi_k3_b200.train.optimizer` (which assigns
parameters from the model's own registry, runs Per-Head Muon and QK-Clip) and are kept for users who
build an optimizer for any ``nn.Module`` from parameter names alone:

* :class:`Muon` -- momentum (optionally Nesterov), quintic Newton-Schulz orthogonalisation of each
  2-D update, decoupled weight decay, no RMS rescaling of the update (the reference's generic form).
  Matrices of equal shape run their iterations as one batched product.
* :class:`HybridMuonAdamW` -- Muon for the 2-D hidden matrices, AdamW for everything else, one
  object for the training loop (``step``, ``zero_grad``, ``set_lr``, ``state_dict``).
* :func:`assign_parameter` / :func:`build_muon_adamw_parameter_groups` -- the name rules: a trainable
  2-D ``*.weight`` goes to Muon unless its name marks an embedding, a head, a norm or a small control
  tensor; of the rest, vectors, biases, norms, embeddings, heads and controls take no weight decay.
* :func:`build_adamw_parameter_groups` / :func:`build_adamw_optimizer` -- AdamW with decay on 2-D
  weights only (no decay for vectors, biases, embeddings, layer norms and the model's ``lm_head``).
"""
from __future__ import annotations

from typing import Any

import torch
import torch.nn as nn

from .optimizer import NS_COEFFS

# Name fragments that keep a 2-D weight away from Muon; the last group of them also means "no decay".
_NOT_MUON = ("embedding", "embed", "token_embedding", "lm_head", "prediction_head", "norm", "bias", "static_",
             "alpha_", "bias_a", "bias_b", "temperature", "scale", "readout", "depth_loss_weights")
_NO_DECAY = ("lm_head", "prediction_head", "bias_a", "bias_b", "alpha_", "static_", "temperature", "scale",
             "depth_loss_weights", "readout")
_NORM_TYPES = (nn.LayerNorm, nn.BatchNorm1d, nn.BatchNorm2d, nn.BatchNorm3d, nn.GroupNorm, nn.InstanceNorm1d,
               nn.InstanceNorm2d, nn.InstanceNorm3d, nn.LocalResponseNorm)


# --------------------------------------------------------------------------- Newton-Schulz
@torch.no_grad()
def zeropower_via_newtonschulz5(G: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    """Orthogonalised ``G`` (2-D) by ``steps`` quintic Newton-Schulz iterations, in fp32, returned in
    ``G``'s dtype.  A matrix whose norm is at most ``eps`` maps to zeros; NaN / Inf raise."""
    if G.dim() != 2:
        raise ValueError(f"zeropower_via_newtonschulz5 expects a 2D tensor, got shape={tuple(G.shape)}.")
    if steps <= 0:
        raise ValueError(f"steps must be > 0, got {steps}.")
    if eps <= 0:
        raise ValueError(f"eps must be > 0, got {eps}.")
    return _orthogonalise(G.detach()[None], steps, eps)[0]


def _orthogonalise(batch: torch.Tensor, steps: int, eps: float) -> torch.Tensor:
    """``[N, m, n]`` -> the same shape and dtype; each matrix normalised by ``||X|| + eps``."""
    x = batch.float()
    if not torch.isfinite(x).all():
        raise FloatingPointError("Input to zeropower_via_newtonschulz5 contains NaN or Inf.")
    norms = x.flatten(1).norm(dim=1)
    tall = x.shape[-2] > x.shape[-1]
    if tall:
        x = x.transpose(-2, -1)
    x = x / (norms + eps)[:, None, None]
    a, b, c = NS_COEFFS
    for _ in range(steps):
        gram = x @ x.transpose(-2, -1)
        x = a * x + (b * gram + c * (gram @ gram)) @ x
    if tall:
        x = x.transpose(-2, -1)
    x = x * (norms > eps).to(x.dtype)[:, None, None]
    return x.to(batch.dtype)


# --------------------------------------------------------------------------- Muon
class Muon(torch.optim.Optimizer):
    """Muon for 2-D parameters (hidden linear weights, attention projections)."""

    def __init__(self, params, lr: float = 1e-3, momentum: float = 0.95, weight_decay: float = 0.0,
                 nesterov: bool = True, ns_steps: int = 5, eps: float = 1e-7):
        if lr <= 0:
            raise ValueError(f"lr must be > 0, got {lr}.")
        if not 0.0 <= momentum < 1.0:
            raise ValueError(f"momentum must satisfy 0 <= momentum < 1, got {momentum}.")
        if weight_decay < 0:
            raise ValueError(f"weight_decay must be >= 0, got {weight_decay}.")
        if ns_steps <= 0:
            raise ValueError(f"ns_steps must be > 0, got {ns_steps}.")
        if eps <= 0:
            raise ValueError(f"eps must be > 0, got {eps}.")
        super().__init__(params, dict(lr=lr, momentum=momentum, weight_decay=weight_decay, nesterov=nesterov,
                                      ns_steps=ns_steps, eps=eps))
        for group in self.param_groups:
            for p in group["params"]:
                if p.ndim != 2:
                    raise ValueError(f"Muon only supports 2D parameters. Got parameter with shape={tuple(p.shape)}.")

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            by_shape: dict = {}
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.ndim != 2:
                    raise ValueError(f"Muon only supports 2D parameters during step. Got shape={tuple(p.shape)}.")
                g = p.grad.detach()
                if not torch.isfinite(g).all():
                    raise FloatingPointError(f"Non-finite gradient found in Muon parameter with shape={tuple(p.shape)}.")
                buf = self.state[p].get("momentum_buffer")
                if buf is None:
                    buf = self.state[p]["momentum_buffer"] = torch.zeros_like(g)
                buf.mul_(group["momentum"]).add_(g)
                update = g.add(buf, alpha=group["momentum"]) if group["nesterov"] else buf
                by_shape.setdefault((tuple(p.shape), p.dtype, p.device), []).append((p, update))
            lr, wd = group["lr"], group["weight_decay"]
            for items in by_shape.values():  # one batched orthogonalisation per shape
                ortho = _orthogonalise(torch.stack([u for _, u in items]), group["ns_steps"], group["eps"])
                for (p, _), o in zip(items, ortho):
                    if wd != 0.0:
                        p.mul_(1.0 - lr * wd)
                    p.add_(o, alpha=-lr)
        return loss


class HybridMuonAdamW:
    """Muon for the selected 2-D matrices and AdamW for the rest, driven as one optimizer."""

    def __init__(self, muon_optimizer: Muon, adamw_optimizer: torch.optim.AdamW, metadata: dict | None = None):
        self.muon, self.adamw = muon_optimizer, adamw_optimizer
        self.metadata = metadata or {}

    @property
    def param_groups(self):
        """Both optimizers' groups, for inspection (change learning rates with :meth:`set_lr`)."""
        return self.muon.param_groups + self.adamw.param_groups

    @property
    def defaults(self):
        return {"muon": getattr(self.muon, "defaults", {}), "adamw": getattr(self.adamw, "defaults", {})}

    def zero_grad(self, set_to_none: bool = True):
        for opt in (self.muon, self.adamw):
            opt.zero_grad(set_to_none=set_to_none)

    def step(self, closure=None):
        loss = closure() if closure is not None else None
        self.muon.step()
        self.adamw.step()
        return loss

    def set_lr(self, lr: float, muon_lr: float | None = None):
        """AdamW groups take ``lr``; Muon groups take ``muon_lr`` (``lr`` when not given)."""
        if lr <= 0:
            raise ValueError(f"lr must be > 0, got {lr}.")
        if muon_lr is not None and muon_lr <= 0:
            raise ValueError(f"muon_lr must be > 0, got {muon_lr}.")
        for opt, value in ((self.adamw, lr), (self.muon, lr if muon_lr is None else muon_lr)):
            for group in opt.param_groups:
                group["lr"] = value

    def state_dict(self):
        return {"muon": self.muon.state_dict(), "adamw": self.adamw.state_dict(), "metadata": self.metadata}

    def load_state_dict(self, state_dict):
        self.muon.load_state_dict(state_dict["muon"])
        self.adamw.load_state_dict(state_dict["adamw"])
        self.metadata = state_dict.get("metadata", self.metadata)


# --------------------------------------------------------------------------- name rules
def _owners(model: nn.Module) -> dict:
    """Full parameter name -> the module that holds it directly."""
    out = {}
    for mname, module in model.named_modules():
        for pname, _ in module.named_parameters(recurse=False):
            out[f"{mname}.{pname}" if mname else pname] = module
    return out


def _is_embedding(name: str, module) -> bool:
    low = name.lower()
    return "embedding" in low or "embed" in low or "wte" in low or isinstance(module, nn.Embedding)


def _is_norm(name: str, module) -> bool:
    return "norm" in name.lower() or isinstance(module, _NORM_TYPES)


def assign_parameter(name: str, param: torch.Tensor, module: nn.Module | None = None) -> str | None:
    """``"muon"``, ``"adamw_decay"``, ``"adamw_no_decay"`` or None (frozen) for one parameter."""
    if not param.requires_grad:
        return None
    low = name.lower()
    if (param.ndim == 2 and name.endswith(".weight") and not any(k in low for k in _NOT_MUON)
            and not _is_embedding(name, module) and not _is_norm(name, module)):
        return "muon"
    if (param.ndim < 2 or name.endswith(".bias") or _is_norm(name, module) or _is_embedding(name, module)
            or any(k in low for k in _NO_DECAY)):
        return "adamw_no_decay"
    return "adamw_decay"


def should_use_muon(name: str, param: torch.Tensor, module: nn.Module | None = None) -> bool:
    return assign_parameter(name, param, module) == "muon"


def should_use_adamw_no_decay(name: str, param: torch.Tensor, module: nn.Module | None = None) -> bool:
    """True for a trainable parameter that AdamW should not decay (whether or not Muon would take it)."""
    if not param.requires_grad:
        return False
    low = name.lower()
    return (param.ndim < 2 or name.endswith(".bias") or _is_norm(name, module) or _is_embedding(name, module)
            or any(k in low for k in _NO_DECAY))


def build_muon_adamw_parameter_groups(model: nn.Module, adamw_weight_decay: float = 0.1,
                                      muon_weight_decay: float = 0.0, verbose: bool = False):
    """``(muon_groups, adamw_groups, metadata)``: every trainable parameter in exactly one group."""
    if adamw_weight_decay < 0:
        raise ValueError(f"adamw_weight_decay must be >= 0, got {adamw_weight_decay}.")
    if muon_weight_decay < 0:
        raise ValueError(f"muon_weight_decay must be >= 0, got {muon_weight_decay}.")
    owners = _owners(model)
    buckets = {"muon": ([], []), "adamw_decay": ([], []), "adamw_no_decay": ([], [])}
    seen = set()
    for name, param in model.named_parameters():
        kind = assign_parameter(name, param, owners.get(name))
        if kind is None:
            continue
        if id(param) in seen:
            raise RuntimeError(f"Duplicate parameter assignment detected for parameter: {name}")
        seen.add(id(param))
        buckets[kind][0].append(param)
        buckets[kind][1].append(name)
    missing = [n for n, p in model.named_parameters() if p.requires_grad and id(p) not in seen]
    if missing:
        raise RuntimeError(f"Some trainable parameters were not assigned to any optimizer group: {missing[:20]}")
    (mp, mn), (dp, dn), (np_, nn_) = buckets["muon"], buckets["adamw_decay"], buckets["adamw_no_decay"]
    muon_groups = [{"params": mp, "weight_decay": muon_weight_decay, "group_name": "muon"}]
    adamw_groups = [{"params": dp, "weight_decay": adamw_weight_decay, "group_name": "adamw_decay"},
                    {"params": np_, "weight_decay": 0.0, "group_name": "adamw_no_decay"}]
    count = lambda ps: int(sum(p.numel() for p in ps))  # noqa: E731
    meta: dict[str, Any] = {
        "num_muon_tensors": len(mp), "num_adamw_decay_tensors": len(dp), "num_adamw_no_decay_tensors": len(np_),
        "num_adamw_tensors": len(dp) + len(np_), "num_muon_params": count(mp), "num_adamw_decay_params": count(dp),
        "num_adamw_no_decay_params": count(np_), "num_adamw_params": count(dp) + count(np_),
        "muon_names": mn, "adamw_decay_names": dn, "adamw_no_decay_names": nn_}
    meta["total_trainable_params"] = meta["num_muon_params"] + meta["num_adamw_params"]
    if verbose:
        print(f"Hybrid Muon + AdamW: Muon {meta['num_muon_tensors']} tensors / {meta['num_muon_params']:,} params, "
              f"AdamW {meta['num_adamw_tensors']} tensors / {meta['num_adamw_params']:,} params "
              f"({meta['num_adamw_no_decay_tensors']} without decay)")
    return muon_groups, adamw_groups, meta


def build_muon_adamw_optimizer(model: nn.Module, learning_rate: float = 3e-4, weight_decay: float = 0.1,
                               betas: tuple = (0.9, 0.95), eps: float = 1e-8, muon_lr: float | None = None,
                               muon_momentum: float = 0.95, muon_nesterov: bool = True, muon_ns_steps: int = 5,
                               muon_eps: float = 1e-7, muon_weight_decay: float = 0.0, verbose: bool = False):
    """``(HybridMuonAdamW, metadata)`` for ``model`` by the name rules."""
    if learning_rate <= 0:
        raise ValueError(f"learning_rate must be > 0, got {learning_rate}.")
    if muon_lr is not None and muon_lr <= 0:
        raise ValueError(f"muon_lr must be > 0 if provided, got {muon_lr}.")
    if weight_decay < 0:
        raise ValueError(f"weight_decay must be >= 0, got {weight_decay}.")
    if len(betas) != 2:
        raise ValueError(f"betas must have length 2, got {betas}.")
    mlr = learning_rate if muon_lr is None else muon_lr
    muon_groups, adamw_groups, meta = build_muon_adamw_parameter_groups(model, weight_decay, muon_weight_decay,
                                                                        verbose)
    if meta["num_muon_tensors"] == 0:
        raise RuntimeError("No parameters were assigned to Muon. Check should_use_muon exclusions or model "
                           "architecture.")
    muon = Muon(muon_groups, lr=mlr, momentum=muon_momentum, weight_decay=muon_weight_decay,
                nesterov=muon_nesterov, ns_steps=muon_ns_steps, eps=muon_eps)
    adamw = torch.optim.AdamW(adamw_groups, lr=learning_rate, betas=betas, eps=eps)
    meta.update(optimizer_type="muon_adamw", learning_rate=learning_rate, muon_lr=mlr, adamw_lr=learning_rate,
                weight_decay=weight_decay, muon_weight_decay=muon_weight_decay, muon_momentum=muon_momentum,
                muon_nesterov=muon_nesterov, muon_ns_steps=muon_ns_steps, muon_eps=muon_eps)
    return HybridMuonAdamW(muon, adamw, meta), meta


# --------------------------------------------------------------------------- AdamW
def build_adamw_parameter_groups(model: nn.Module, weight_decay: float = 0.1):
    """``(groups, info)``: decay on weights of two or more dimensions, none on the rest."""
    if weight_decay < 0:
        raise ValueError("weight_decay must be non-negative")
    owners = _owners(model)
    head = getattr(model, "lm_head", None)
    decay, no_decay, dn, nn_ = [], [], [], []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        module = owners.get(name)
        plain = (p.ndim < 2 or name.endswith(".bias") or isinstance(module, (nn.Embedding, nn.LayerNorm))
                 or "norm" in name.lower() or module is head)
        (no_decay if plain else decay).append(p)
        (nn_ if plain else dn).append(name)
    groups = [{"params": decay, "weight_decay": weight_decay, "group_name": "decay"},
              {"params": no_decay, "weight_decay": 0.0, "group_name": "no_decay"}]
    return groups, {"decay_names": dn, "no_decay_names": nn_, "num_decay_params": sum(p.numel() for p in decay),
                    "num_no_decay_params": sum(p.numel() for p in no_decay)}


def build_adamw_optimizer(model: nn.Module, learning_rate: float = 3e-4, weight_decay: float = 0.1,
                          betas: tuple = (0.9, 0.95), eps: float = 1e-8):
    if learning_rate <= 0:
        raise ValueError("learning_rate must be positive")
    groups, info = build_adamw_parameter_groups(model, weight_decay)
    return torch.optim.AdamW(groups, lr=learning_rate, betas=betas, eps=eps), info


__all__ = ["zeropower_via_newtonschulz5", "Muon", "HybridMuonAdamW", "assign_parameter", "should_use_muon",
           "should_use_adamw_no_decay", "build_muon_adamw_parameter_groups", "build_muon_adamw_optimizer",
           "build_adamw_parameter_groups", "build_adamw_optimizer"]
