"""Hybrid optimizer: (Per-Head) Muon for matrices + AdamW for the rest + QK-Clip.

Parity targets (reference paths):
  * ``training/optimizer/newton_schulz.py:11-74``   quintic NS (a, b, c) = (3.4445, -4.7750, 2.0315)
  * ``training/optimizer/muon.py:17-142``           momentum, Nesterov, decoupled decay, RMS match
  * ``training/optimizer/per_head_muon.py:14-159``  per-head orthogonalisation of q/k/v
  * ``training/optimizer/parameter_registry.py``    family assignment + fingerprint
  * ``training/optimizer/qk_clip.py:39-162``        rescale W_q / W_k by sqrt(tau / s)
  * ``training/optimizer/hybrid.py:28-255``         transactional step, state dict
  * ``training/optimizer/config.py``                KimiOptimizerConfig

B200 design: every Muon matrix (a plain 2-D weight, one head block of a q/k/v
projection, or one expert of a stacked ``[E, H, L]`` weight) is placed in a bucket
of equal-shape matrices; each step runs one batched Newton-Schulz per bucket
(``torch.baddbmm`` chains) instead of one small GEMM chain per matrix/head.  The
non-finite check, the update metrics and QK-Clip all stay on the device; the host
reads them in one transfer when a report is requested.
"""
from __future__ import annotations

import hashlib
import json
import math
from dataclasses import asdict, dataclass, field
from typing import Literal

import torch
import torch.nn as nn

from ..runtime import host_checks

NS_COEFFS = (3.4445, -4.7750, 2.0315)


# --------------------------------------------------------------------------- config
@dataclass(frozen=True)
class KimiOptimizerConfig:
    kind: Literal["adamw", "muon_adamw", "per_head_muon_adamw"] = "per_head_muon_adamw"
    adamw_lr: float = 3e-4
    adamw_betas: tuple = (0.9, 0.95)
    adamw_eps: float = 1e-8
    muon_lr: float | None = None
    muon_momentum: float = 0.95
    muon_nesterov: bool = True
    muon_ns_steps: int = 5
    muon_ns_eps: float = 1e-7
    muon_update_rms_scaling: bool = True
    weight_decay: float = 0.1
    muon_weight_decay: float | None = None
    per_head_qkv: bool = True
    qk_clip_enabled: bool = True
    qk_clip_threshold: float = 100.0
    qk_clip_eps: float = 1e-6
    qk_clip_every_steps: int = 1
    qk_clip_kda_experimental: bool = False
    fail_on_unclassified_matrix: bool = True
    muon_ns_dtype: str = "auto"

    def __post_init__(self) -> None:
        object.__setattr__(self, "adamw_betas", tuple(self.adamw_betas))
        if self.kind not in ("adamw", "muon_adamw", "per_head_muon_adamw"):
            raise ValueError("unknown optimizer kind")
        if self.adamw_lr <= 0 or self.adamw_eps <= 0:
            raise ValueError("AdamW learning rate and epsilon must be positive")
        if len(self.adamw_betas) != 2 or not all(0 <= v < 1 for v in self.adamw_betas):
            raise ValueError("adamw_betas must contain two values in [0, 1)")
        if self.muon_lr is not None and self.muon_lr <= 0:
            raise ValueError("muon_lr must be None or positive")
        if not 0 <= self.muon_momentum < 1:
            raise ValueError("muon_momentum must be in [0, 1)")
        if self.muon_ns_steps <= 0 or self.muon_ns_eps <= 0:
            raise ValueError("Newton-Schulz steps and epsilon must be positive")
        if self.weight_decay < 0 or (self.muon_weight_decay is not None and self.muon_weight_decay < 0):
            raise ValueError("weight decay must be non-negative")
        if self.qk_clip_threshold <= 0 or self.qk_clip_eps <= 0 or self.qk_clip_every_steps <= 0:
            raise ValueError("invalid QK-Clip configuration")
        if self.kind == "per_head_muon_adamw" and not self.per_head_qkv:
            raise ValueError("canonical Per-Head Muon requires per_head_qkv=True")
        if self.muon_ns_dtype not in ("auto", "float32", "bfloat16"):
            raise ValueError("muon_ns_dtype must be auto, float32 or bfloat16")

    @property
    def resolved_muon_lr(self) -> float:
        return self.adamw_lr if self.muon_lr is None else self.muon_lr

    @property
    def resolved_muon_weight_decay(self) -> float:
        return self.weight_decay if self.muon_weight_decay is None else self.muon_weight_decay

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: dict) -> "KimiOptimizerConfig":
        return cls(**values)


# --------------------------------------------------------------------------- Newton-Schulz
@torch.no_grad()
def zeropower_via_newton_schulz(matrix: torch.Tensor, *, steps: int = 5, eps: float = 1e-7,
                                output_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Single-matrix quintic Newton-Schulz orthogonalisation (fp32)."""
    if matrix.ndim != 2:
        raise ValueError("Newton-Schulz input must be a 2D matrix")
    if steps <= 0 or eps <= 0:
        raise ValueError("steps and eps must be positive")
    out = batched_newton_schulz(matrix.detach()[None].float(), steps=steps, eps=eps, dtype=torch.float32)[0]
    if not torch.isfinite(matrix).all():
        raise FloatingPointError("Newton-Schulz input contains NaN or Inf")
    return out.to(dtype=output_dtype or matrix.dtype)


@torch.no_grad()
def batched_newton_schulz(x: torch.Tensor, *, steps: int = 5, eps: float = 1e-7,
                          dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Orthogonalise a batch ``[N, m, n]`` of matrices; all-zero matrices map to zero.

    Tall matrices are transposed so the Gram matrix is the small side.
    """
    transposed = x.shape[-2] > x.shape[-1]
    w = x.transpose(-2, -1) if transposed else x
    norms = w.float().flatten(1).norm(dim=1)
    w = (w.float() / norms.clamp_min(eps)[:, None, None]).to(dtype)
    w = newton_schulz_iterations(w, steps)
    w = w.float() * (norms > eps).to(torch.float32)[:, None, None]
    return w.transpose(-2, -1) if transposed else w


def newton_schulz_iterations(w: torch.Tensor, steps: int, *, transpose_out: bool = False,
                             tensor_cores: bool = False) -> torch.Tensor:
    """The quintic iterations on an already normalised batch ``[N, m, n]`` with ``m <= n``.

    Each step is ``X <- (a I + b G + c G^2) X`` with ``G = X X^T``: the small ``[m, m]`` polynomial
    takes the ``a I`` term on its diagonal, so the big product is a plain batched GEMM (no copy of
    X into the output as ``a X + P X`` would need).  ``transpose_out`` returns ``X^T`` [N, n, m]
    contiguous, computed by the last step as ``X^T P`` (P is symmetric) instead of a transpose copy.

    ``tensor_cores=True`` runs the products on this package's grouped tcgen05 GEMM
    (:func:`_ns_iterations_tc`).  On the t4_wikitext Muon buckets (522 x [64, 640], 425 x
    [640, 320], 221 x [320, 640], ...) it measured 6.5 ms per optimizer step against 3.9 ms for the
    batched library GEMMs: the matrices are padded to 128-row tiles (64 -> 128, 320 -> 384) and the
    128-wide tiles are load-bound, so the default stays on the batched GEMMs."""
    if tensor_cores and _ns_on_tensor_cores(w):
        return _ns_iterations_tc(w, steps, transpose_out)
    a, b, c = NS_COEFFS
    for i in range(steps):
        gram = w @ w.transpose(-2, -1)
        poly = torch.baddbmm(gram, gram, gram, beta=b, alpha=c)  # b*G + c*G@G
        poly.diagonal(dim1=-2, dim2=-1).add_(a)                   # + a*I
        if transpose_out and i == steps - 1:
            return torch.bmm(w.transpose(-2, -1), poly)
        w = torch.bmm(poly, w)
    return w.transpose(-2, -1).contiguous() if transpose_out else w


def _ns_on_tensor_cores(w: torch.Tensor) -> bool:
    from .. import ops
    return (w.is_cuda and w.dtype == torch.bfloat16 and w.ndim == 3 and w.shape[-1] % 8 == 0 and w.numel() > 0
            and ops.use_kernels(w))


_NS_OFFSETS: dict = {}


def _ns_tile_n(n: int) -> int:
    """Output tile width with the least padding (256 on a tie: fewer tiles)."""
    return 256 if (-n) % 256 <= (-n) % 128 else 128


def _ns_iterations_tc(w: torch.Tensor, steps: int, transpose_out: bool) -> torch.Tensor:
    """The quintic iterations on this package's grouped tcgen05 GEMM (bf16 operands, fp32
    accumulation).  Each matrix of the batch is one row segment of the grouped product, padded to
    a multiple of 128 rows with zeros; the padding stays zero through every step (its rows of
    ``P = a I + b G + c G^2`` are ``a e_i`` and meet zero rows of X).  Per step: ``G = X X^T`` and
    ``G2 = G G^T`` (G is symmetric) with both operands K-major, the polynomial in one elementwise
    kernel, and ``X <- P X`` with X as the MN-major operand."""
    from ..ops import _loader
    C = _loader.require()
    e, m, n = w.shape
    mp = -(-m // 128) * 128
    x = torch.zeros(e, mp, n, dtype=torch.bfloat16, device=w.device)
    x[:, :m].copy_(w)
    key = (e, mp, w.device)
    offs = _NS_OFFSETS.get(key)
    if offs is None:
        offs = _NS_OFFSETS[key] = (torch.arange(e + 1, dtype=torch.int32) * mp).to(w.device)
    a, b, c = NS_COEFFS
    bn_g, bn_x = _ns_tile_n(mp), _ns_tile_n(n)
    rows = e * mp
    for _ in range(steps):
        g = C.tc_gemm_grouped(1, x.view(rows, n), x, None, False, False, offs, rows, mp, n, 0, None, False, 0.0,
                              0.0, None, None, 0, bn_g, uniform_rows=mp)[0]
        g2 = C.tc_gemm_grouped(1, g, g.view(e, mp, mp), None, False, False, offs, rows, mp, mp, 0, None, False, 0.0,
                               0.0, None, None, 0, bn_g, uniform_rows=mp)[0]
        poly = C.ns_poly(g, g2, a, b, c)
        x = C.tc_gemm_grouped(1, poly, x, None, False, True, offs, rows, n, mp, 0, None, False, 0.0, 0.0, None, None,
                              0, bn_x, uniform_rows=mp)[0].view(e, mp, n)
    out = x[:, :m]
    return out.transpose(-2, -1) if transpose_out else out


@torch.no_grad()
def match_update_rms(orthogonal_update, reference=None, *, mode="shape", eps=1e-12):
    if mode == "shape":
        return orthogonal_update * (max(orthogonal_update.shape[-2:]) ** 0.5)
    if mode != "reference_rms":
        raise ValueError("unknown update RMS matching mode")
    if reference is None or reference.shape != orthogonal_update.shape:
        raise ValueError("reference_rms mode requires a matching reference")
    target = reference.float().square().mean().sqrt()
    current = orthogonal_update.float().square().mean().sqrt()
    if float(current) <= eps:
        return torch.zeros_like(orthogonal_update)
    return orthogonal_update * (target / current).to(orthogonal_update.dtype)


# --------------------------------------------------------------------------- head layouts
@dataclass(frozen=True)
class HeadMatrixLayout:
    num_heads: int
    head_dim: int
    head_axis: int
    input_dim: int
    output_dim: int
    packed_kind: str = "separate"
    qkv_slices: tuple | None = None

    def __post_init__(self) -> None:
        if self.num_heads <= 0 or self.head_dim <= 0 or self.head_axis not in (0, 1):
            raise ValueError("invalid head layout")
        if self.packed_kind == "fused_qkv" and self.qkv_slices is None:
            raise ValueError("fused_qkv layout requires explicit slices")

    def validate(self, matrix: torch.Tensor) -> None:
        if matrix.ndim != 2 or tuple(matrix.shape) != (self.output_dim, self.input_dim):
            raise ValueError("matrix shape does not match the head layout")
        if self.packed_kind == "separate" and matrix.shape[self.head_axis] != self.num_heads * self.head_dim:
            raise ValueError("head axis does not equal num_heads * head_dim")

    def head_blocks(self, matrix: torch.Tensor) -> torch.Tensor:
        """``[num_heads, head_dim, in]`` (axis 0) or ``[num_heads, out, head_dim]`` (axis 1) view/copy."""
        if self.head_axis == 0:
            return matrix.reshape(self.num_heads, self.head_dim, matrix.shape[1])
        return matrix.reshape(matrix.shape[0], self.num_heads, self.head_dim).permute(1, 0, 2)


def split_head_matrix(matrix, layout: HeadMatrixLayout):
    layout.validate(matrix)
    blocks = layout.head_blocks(matrix)
    return tuple(blocks[i] for i in range(layout.num_heads))


def merge_head_matrix(blocks, layout: HeadMatrixLayout):
    st = torch.stack(tuple(blocks))
    if layout.head_axis == 0:
        return st.reshape(layout.output_dim, layout.input_dim)
    return st.permute(1, 0, 2).reshape(layout.output_dim, layout.input_dim)


@torch.no_grad()
def per_head_orthogonalize(matrix, layout: HeadMatrixLayout, *, steps, eps, rms_scaling=True):
    """Orthogonalise each head block independently (batched NS); returns (update, metrics)."""
    layout.validate(matrix)
    blocks = layout.head_blocks(matrix).float()
    raw = blocks.flatten(1).square().mean(1).sqrt()
    ortho = batched_newton_schulz(blocks, steps=steps, eps=eps)
    orms = ortho.flatten(1).square().mean(1).sqrt()
    if rms_scaling:
        ortho = ortho * (max(ortho.shape[-2:]) ** 0.5)
    final = ortho.flatten(1).square().mean(1).sqrt()
    out = merge_head_matrix(list(ortho), layout)

    def summary(v, label):
        v = v.double()
        mean, std = float(v.mean()), float(v.std(unbiased=False))
        return {f"per_head_muon/{label}_mean": mean, f"per_head_muon/{label}_std": std,
                f"per_head_muon/{label}_min": float(v.min()), f"per_head_muon/{label}_max": float(v.max()),
                f"per_head_muon/{label}_median": float(v.median()), f"per_head_muon/{label}_cv": std / max(mean, eps)}

    metrics = {}
    metrics.update(summary(raw, "raw_momentum_rms"))
    metrics.update(summary(orms, "orthogonal_update_rms"))
    metrics.update(summary(final, "head_update_rms"))
    fd = final.double()
    metrics["per_head_muon/head_update_rms_max_to_median"] = float(fd.max()) / max(float(fd.median()), eps)
    metrics["per_head_muon/fraction_heads_near_zero_update"] = float((fd <= eps).double().mean())
    return out.to(matrix.dtype), metrics


# --------------------------------------------------------------------------- registry
OptimizerFamily = Literal["adamw_decay", "adamw_no_decay", "muon", "per_head_muon"]


@dataclass(frozen=True)
class MatrixParameterSpec:
    parameter_name: str
    parameter: nn.Parameter
    owner_module_name: str
    role: str
    optimizer_family: str
    apply_weight_decay: bool
    head_layout: HeadMatrixLayout | None = None

    def fingerprint_record(self) -> dict:
        layout = None
        if self.head_layout is not None:
            hl = self.head_layout
            layout = {"num_heads": hl.num_heads, "head_dim": hl.head_dim, "head_axis": hl.head_axis,
                      "input_dim": hl.input_dim, "output_dim": hl.output_dim, "packed_kind": hl.packed_kind}
        return {"name": self.parameter_name, "shape": list(self.parameter.shape), "role": self.role,
                "family": self.optimizer_family, "weight_decay": self.apply_weight_decay, "head_layout": layout}


@dataclass(frozen=True)
class ParameterAssignmentReport:
    specs: tuple
    numel_by_family: dict
    tensor_count_by_family: dict
    percentages_by_family: dict
    missing: tuple
    duplicates: tuple
    ambiguous: tuple
    fingerprint: str

    @property
    def total_numel(self) -> int:
        return sum(self.numel_by_family.values())

    def names_for(self, family: str) -> tuple:
        return tuple(s.parameter_name for s in self.specs if s.optimizer_family == family)

    def to_dict(self) -> dict:
        return {"numel_by_family": dict(self.numel_by_family), "tensor_count_by_family": dict(self.tensor_count_by_family),
                "percentages_by_family": dict(self.percentages_by_family), "missing": list(self.missing),
                "duplicates": list(self.duplicates), "ambiguous": list(self.ambiguous),
                "fingerprint": self.fingerprint, "specs": [s.fingerprint_record() for s in self.specs]}


def _qkv_layout(owner_name, owner, modules):
    from ..models.kda import KDAProjections
    from ..models.mla import LatentKVProjection, MLAProjections
    spec = getattr(owner, "_kimi_head_spec", None)
    if spec is not None:
        nh, hd = spec
        return getattr(owner, "_kimi_role"), HeadMatrixLayout(nh, hd, 0, owner.in_features, owner.local_out_features)
    parent_name, _, attr = owner_name.rpartition(".")
    parent = modules.get(parent_name)
    if isinstance(parent, KDAProjections) and attr in ("q_proj", "k_proj", "v_proj"):
        role = {"q_proj": "attention_q", "k_proj": "attention_k", "v_proj": "attention_v"}[attr]
        hd = parent.config.value_head_dim if attr == "v_proj" else parent.config.key_head_dim
    elif isinstance(parent, MLAProjections) and attr == "query":
        role, hd = "attention_q", parent.config.q_head_dim
    elif isinstance(parent, LatentKVProjection) and attr in ("key_up", "value_up"):
        role = "attention_k" if attr == "key_up" else "attention_v"
        hd = parent.config.q_head_dim if attr == "key_up" else parent.config.v_head_dim
    else:
        return None
    return role, HeadMatrixLayout(parent.config.num_heads, hd, 0, owner.in_features, owner.out_features)


def _is_norm(name, owner):
    return "norm" in name.lower() or isinstance(owner, (nn.LayerNorm, nn.BatchNorm1d, nn.BatchNorm2d, nn.GroupNorm))


def build_parameter_registry(model: nn.Module, *, kind: str = "per_head_muon_adamw",
                             strict: bool = True) -> ParameterAssignmentReport:
    """Assign every trainable tensor to one optimizer family (reference rules).

    Stacked routed-expert weights (``[E, H, L]``) are Muon matrices (one per expert).
    """
    from ..models.moe import GroupedRoutedExperts
    modules = dict(model.named_modules())
    owner_by_name = {}
    for mname, module in modules.items():
        for local, _ in module.named_parameters(recurse=False):
            owner_by_name[f"{mname}.{local}" if mname else local] = (mname, module)
    specs, seen, duplicates, ambiguous = [], {}, [], []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        if id(p) in seen:
            duplicates.append(name)
            continue
        seen[id(p)] = name
        owner_name, owner = owner_by_name[name]
        qkv = _qkv_layout(owner_name, owner, modules)
        role, layout = "other", None
        explicit = getattr(owner, "_kimi_role", None)
        parallel_linear = bool(getattr(owner, "_kimi_parallel_linear", False))
        no_decay = (p.ndim < 2 or name.endswith(".bias") or isinstance(owner, nn.Embedding) or _is_norm(name, owner)
                    or "lm_head" in name or "pseudo_query" in name or explicit in ("embedding", "lm_head"))
        stacked = isinstance(owner, GroupedRoutedExperts)
        if qkv is not None:
            role, layout = qkv
        elif stacked:
            role = "moe_routed_expert"
        elif explicit is not None:
            role = explicit
        elif isinstance(owner, nn.Embedding):
            role = "embedding"
        elif "lm_head" in name:
            role = "lm_head"
        elif _is_norm(name, owner):
            role = "norm"
        elif isinstance(owner, nn.Linear):
            low = name.lower()
            if ".router." in low:
                role = "moe_router"
            elif "shared_experts" in low:
                role = "moe_shared_expert"
            elif "routed_experts" in low:
                role = "moe_routed_expert"
            elif "output_proj" in low:
                role = "attention_o"
            elif low.startswith("mtp.") or ".mtp." in low:
                role = "mtp_matrix"
            else:
                role = "dense_matrix"
        matrix_like = (isinstance(owner, nn.Linear) or parallel_linear) and p.ndim == 2
        if kind == "adamw":
            family = "adamw_no_decay" if no_decay else "adamw_decay"
        elif layout is not None and kind == "per_head_muon_adamw":
            family = "per_head_muon"
        elif (matrix_like and not no_decay and role != "moe_router") or (stacked and p.ndim == 3):
            family = "muon"
        else:
            family = "adamw_no_decay" if no_decay else "adamw_decay"
        if strict and matrix_like and role == "other":
            ambiguous.append(name)
        specs.append(MatrixParameterSpec(name, p, owner_name, role, family,
                                         family in ("adamw_decay", "muon", "per_head_muon"),
                                         layout if family == "per_head_muon" else None))
    trainable = {id(p): n for n, p in model.named_parameters() if p.requires_grad}
    assigned = {id(s.parameter) for s in specs}
    missing = tuple(n for i, n in trainable.items() if i not in assigned)
    if strict and (missing or duplicates or ambiguous):
        raise RuntimeError(f"invalid parameter registry: missing={missing}, duplicates={duplicates}, "
                           f"ambiguous={ambiguous}")
    fams = ("adamw_decay", "adamw_no_decay", "muon", "per_head_muon")
    numel = {f: sum(s.parameter.numel() for s in specs if s.optimizer_family == f) for f in fams}
    count = {f: sum(1 for s in specs if s.optimizer_family == f) for f in fams}
    total = max(sum(numel.values()), 1)
    pct = {f: 100.0 * numel[f] / total for f in fams}
    fp = hashlib.sha256(json.dumps([s.fingerprint_record() for s in specs], sort_keys=True).encode()).hexdigest()
    return ParameterAssignmentReport(tuple(specs), numel, count, pct, missing, tuple(duplicates), tuple(ambiguous), fp)


# --------------------------------------------------------------------------- Muon
@dataclass
class _MatrixSlot:
    param: torch.Tensor
    count: int           # matrices contributed by this parameter
    rows: int
    cols: int
    to_blocks: callable  # tensor shaped like param -> [count, rows, cols]
    from_blocks: callable
    per_head: bool = False  # head blocks along dim 0 (Per-Head Muon)


class KimiMuon(torch.optim.Optimizer):
    """Muon over equal-shape matrix buckets (batched Newton-Schulz per bucket)."""

    def __init__(self, params, *, lr, momentum, nesterov, ns_steps, eps, weight_decay, update_rms_scaling,
                 spec_by_parameter: dict, ns_dtype: str = "auto"):
        if lr <= 0 or not 0 <= momentum < 1 or ns_steps <= 0 or eps <= 0 or weight_decay < 0:
            raise ValueError("invalid Muon configuration")
        super().__init__(params, dict(lr=lr, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps, eps=eps,
                                      weight_decay=weight_decay, update_rms_scaling=update_rms_scaling))
        self.spec_by_parameter = spec_by_parameter
        self.ns_dtype = ns_dtype
        self.last_update_metrics: dict = {}
        self._metric_tensors: dict = {}
        self._buckets = None
        self._slots = {}
        for group in self.param_groups:
            for p in group["params"]:
                if p.ndim not in (2, 3):
                    raise ValueError("Muon parameters must be 2D (or stacked 3D experts)")
                self._slots[id(p)] = self._make_slot(p)

    def _make_slot(self, p) -> _MatrixSlot:
        spec = self.spec_by_parameter.get(id(p))
        if spec is not None and spec.optimizer_family == "per_head_muon" and spec.head_layout is not None \
                and spec.head_layout.head_axis == 0 and spec.head_layout.packed_kind == "separate":
            hl = spec.head_layout
            return _MatrixSlot(p, hl.num_heads, hl.head_dim, p.shape[1],
                               lambda t, hl=hl: t.reshape(hl.num_heads, hl.head_dim, t.shape[-1]),
                               lambda b, p=p: b.reshape(p.shape), per_head=True)
        if p.ndim == 3:
            return _MatrixSlot(p, p.shape[0], p.shape[1], p.shape[2], lambda t: t, lambda b: b)
        return _MatrixSlot(p, 1, p.shape[0], p.shape[1], lambda t: t[None], lambda b: b[0])

    def _resolved_ns_dtype(self, device) -> torch.dtype:
        if self.ns_dtype == "float32" or (self.ns_dtype == "auto" and device.type != "cuda"):
            return torch.float32
        return torch.bfloat16

    def restrict_to(self, param_ids) -> None:
        """Sharded data parallelism: this rank updates (and keeps state for) only these
        parameters; the others are broadcast by their owners after the step."""
        self._owned = set(param_ids)
        self._buckets = None

    def _mine(self, p) -> bool:
        owned = getattr(self, "_owned", None)
        return owned is None or id(p) in owned

    def _tp_gathered(self, p) -> bool:
        """A tensor-parallel shard whose Newton-Schulz needs the whole matrix: split over a group of
        more than one rank, and not a per-head slot whose heads all live on this rank."""
        group = getattr(p, "_kimi_tp_group", None)
        if group is None or not torch.distributed.is_initialized() or torch.distributed.get_world_size(group) < 2:
            return False
        slot = self._slots[id(p)]
        return not (slot.per_head and getattr(p, "_kimi_tp_dim", 0) == 0)

    @torch.no_grad()
    def _step_tp_gathered(self, skip, metrics) -> None:
        """Momentum stays per shard; the momentum-updated shards are all-gathered along their split
        dimension, orthogonalised as whole matrices (the same update as one process computes) and
        each rank applies its own slice.  Shards of equal shape, split dimension and group move as
        one batch: one all-gather and one batched Newton-Schulz per batch."""
        import torch.distributed as dist
        for group in self.param_groups:
            lr, mom, wd = group["lr"], group["momentum"], group["weight_decay"]
            batches: dict = {}
            for p in group["params"]:
                if p.grad is None or not self._mine(p) or not self._tp_gathered(p):
                    continue
                key = (id(p._kimi_tp_group), p._kimi_tp_dim, tuple(p.shape), p.dtype, p.device)
                batches.setdefault(key, []).append(p)
            for ps in batches.values():
                tp, dim = ps[0]._kimi_tp_group, ps[0]._kimi_tp_dim
                world, rank = dist.get_world_size(tp), dist.get_rank(tp)
                raws = []
                for p in ps:
                    st = self.state[p]
                    buf = st.get("momentum_buffer")
                    if buf is None:
                        buf = st["momentum_buffer"] = torch.zeros_like(p)
                    g = p.grad.to(buf.dtype)
                    if skip is not None:
                        g = torch.where(skip, torch.zeros((), device=g.device, dtype=g.dtype), g)
                        buf.mul_(torch.where(skip, 1.0, mom).to(buf.dtype)).add_(g)
                    else:
                        buf.mul_(mom).add_(g)
                    raws.append(g.add(buf, alpha=mom) if group["nesterov"] else buf)
                local = torch.stack(raws)                               # [n, r, c]
                n = local.shape[0]
                parts = torch.empty((world * n,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
                dist.all_gather_into_tensor(parts, local.contiguous(), group=tp)  # rank-major blocks of n
                full = torch.cat(parts.view((world,) + tuple(local.shape)).unbind(0), dim + 1)  # [n, R, C]
                ortho = batched_newton_schulz(full.float(), steps=group["ns_steps"], eps=group["eps"],
                                              dtype=self._resolved_ns_dtype(local.device))
                scale = max(full.shape[1:]) ** 0.5 if group["update_rms_scaling"] else 1.0
                metrics["raw"].append(full.float().flatten(1).square().mean(1).sqrt())
                metrics["ortho"].append(ortho.flatten(1).square().mean(1).sqrt())
                metrics["scaled"].append(metrics["ortho"][-1] * scale)
                upd = torch.chunk(ortho, world, dim=dim + 1)[rank].to(ps[0].dtype).mul_(scale)
                lr_eff = torch.where(skip, 0.0, lr) if skip is not None else lr
                if wd:
                    torch._foreach_mul_(ps, 1.0 - lr_eff * wd)
                if torch.is_tensor(lr_eff):
                    upd.mul_((-lr_eff).to(upd.dtype))
                    torch._foreach_add_(ps, list(upd.unbind(0)))
                else:
                    torch._foreach_add_(ps, list(upd.unbind(0)), alpha=-lr_eff)
                pn = torch.stack(torch._foreach_norm(ps)).float() / (ps[0].numel() ** 0.5)
                lr_v = lr if torch.is_tensor(lr) else torch.tensor(float(lr), device=pn.device)
                metrics["ratio"].append(lr_v * metrics["scaled"][-1] / pn.clamp_min(group["eps"]))

    def _ensure_buckets(self) -> list:
        """Per-parameter momentum buffers become views into one tensor per bucket, so a step
        is a handful of launches per bucket instead of a dozen per parameter."""
        if self._buckets is not None:
            return self._buckets
        keyed: dict = {}
        for gi, group in enumerate(self.param_groups):
            for p in group["params"]:
                if not self._mine(p) or self._tp_gathered(p):
                    continue
                slot = self._slots[id(p)]
                keyed.setdefault((gi, slot.rows, slot.cols, p.device, p.dtype), []).append(p)
        buckets = []
        for (gi, rows, cols, dev, dt), ps in keyed.items():
            count = sum(self._slots[id(p)].count for p in ps)
            mom = torch.zeros(count, rows, cols, device=dev, dtype=dt)
            off = 0
            for p in ps:
                slot = self._slots[id(p)]
                view = slot.from_blocks(mom[off:off + slot.count])
                old = self.state[p].get("momentum_buffer")
                if old is not None:
                    view.copy_(old)
                self.state[p]["momentum_buffer"] = view
                off += slot.count
            sqrt_numel = torch.tensor([float(p.numel()) for p in ps], device=dev).sqrt()
            buckets.append((gi, rows, cols, ps, mom, sqrt_numel))
        self._buckets = buckets
        return buckets

    def load_state_dict(self, state_dict):
        super().load_state_dict(state_dict)
        self._buckets = None  # re-view the loaded per-parameter buffers on the next step

    @torch.no_grad()
    def step(self, closure=None, *, skip: torch.Tensor | None = None):
        """One Muon step. ``skip`` (device bool scalar) turns the step into a no-op on the
        device (momentum, weight decay and update all suppressed) without a host branch."""
        if closure is not None:
            with torch.enable_grad():
                closure()
        if any(_is_dtensor(p) for g in self.param_groups for p in g["params"]):
            return self._step_sharded(skip)
        if any(p.grad is None for g in self.param_groups for p in g["params"] if self._mine(p)):
            if skip is not None:
                raise RuntimeError("device-flag Muon steps need a gradient for every parameter")
            return self._step_sparse()
        metrics = {"raw": [], "ortho": [], "scaled": [], "ratio": []}
        for bi, (gi, rows, cols, ps, mom_buf, numel) in enumerate(self._ensure_buckets()):
            group = self.param_groups[gi]
            lr, mom, wd = group["lr"], group["momentum"], group["weight_decay"]
            slots = [self._slots[id(p)] for p in ps]
            if self._fused_ok(mom_buf, rows, cols):
                self._fused_bucket_step(bi, group, rows, cols, ps, slots, mom_buf, numel, skip, metrics)
                continue
            g = torch.cat([s.to_blocks(p.grad).to(mom_buf.dtype) for p, s in zip(ps, slots)], 0)
            if skip is not None:
                g = torch.where(skip, torch.zeros((), device=g.device, dtype=g.dtype), g)
                mom_buf.mul_(torch.where(skip, 1.0, mom).to(mom_buf.dtype)).add_(g)
            else:
                mom_buf.mul_(mom).add_(g)
            raw = g.add(mom_buf, alpha=mom) if group["nesterov"] else mom_buf
            ortho = batched_newton_schulz(raw, steps=group["ns_steps"], eps=group["eps"],
                                          dtype=self._resolved_ns_dtype(mom_buf.device))
            metrics["raw"].append(raw.float().flatten(1).square().mean(1).sqrt())
            metrics["ortho"].append(ortho.flatten(1).square().mean(1).sqrt())
            scale = max(rows, cols) ** 0.5 if group["update_rms_scaling"] else 1.0
            metrics["scaled"].append(metrics["ortho"][-1] * scale)
            upd = ortho.to(mom_buf.dtype).mul_(scale)
            views, off = [], 0
            for p, s in zip(ps, slots):
                views.append(s.from_blocks(upd[off:off + s.count]))
                off += s.count
            unorm = torch.stack(torch._foreach_norm(views)).float()
            pnorm = torch.stack(torch._foreach_norm(ps)).float()
            metrics["ratio"].append(lr * unorm / (pnorm.clamp_min(1e-30) / numel).clamp_min(group["eps"]) / numel)
            lr_eff = torch.where(skip, 0.0, lr) if skip is not None else lr
            if wd:
                torch._foreach_mul_(ps, 1.0 - lr_eff * wd)
            if torch.is_tensor(lr_eff):
                upd.mul_(-lr_eff)
                torch._foreach_add_(ps, views)
            else:
                torch._foreach_add_(ps, views, alpha=-lr_eff)
        self._step_tp_gathered(skip, metrics)
        self._metric_tensors = {k: torch.cat(v) for k, v in metrics.items() if v}
        self.last_update_metrics = {}
        return self._metric_tensors

    # ---- fused CUDA path: two passes over the bucket around the Newton-Schulz GEMMs
    @staticmethod
    def _fused_ok(mom_buf, rows, cols) -> bool:
        if not mom_buf.is_cuda or mom_buf.dtype != torch.float32 or (rows * cols) % 4:
            return False
        from .. import ops
        return ops.use_kernels(mom_buf)

    def _bucket_tables(self, bi, ps, slots, device):
        """Per-matrix parameter pointers and the matrix -> parameter map of bucket ``bi`` (cached;
        parameters never move)."""
        tables = getattr(self, "_fused_tables", None)
        if tables is None:
            tables = self._fused_tables = {}
        key = (bi, tuple(p.data_ptr() for p in ps))
        hit = tables.get(bi)
        if hit is not None and hit[0] == key:
            return hit[1], hit[2]
        ptrs, owner = [], []
        for j, (p, s) in enumerate(zip(ps, slots)):
            step = s.rows * s.cols * p.element_size()
            ptrs.extend(p.data_ptr() + m * step for m in range(s.count))
            owner.extend([j] * s.count)
        ptr_t = torch.tensor(ptrs, dtype=torch.int64, device=device)
        own_t = torch.tensor(owner, dtype=torch.int64, device=device)
        tables[bi] = (key, ptr_t, own_t)
        return ptr_t, own_t

    def _fused_bucket_step(self, bi, group, rows, cols, ps, slots, mom_buf, numel, skip, metrics):
        from ..ops import _loader
        C = _loader.require()
        dev = mom_buf.device
        count, mn = mom_buf.shape[0], rows * cols
        lr, wd = group["lr"], group["weight_decay"]
        g = torch.cat([s.to_blocks(p.grad).to(torch.float32) for p, s in zip(ps, slots)], 0)
        x = torch.empty(count, rows, cols, dtype=torch.bfloat16, device=dev)
        sumsq = torch.zeros(count, dtype=torch.float32, device=dev)
        C.muon_momentum(g, mom_buf, x, sumsq, float(group["momentum"]), bool(group["nesterov"]), skip)
        C.muon_normalize(x, sumsq, float(group["eps"]))
        transposed = rows > cols
        o = newton_schulz_iterations(x.transpose(-2, -1) if transposed else x, group["ns_steps"],
                                     transpose_out=transposed).contiguous()
        scale = max(rows, cols) ** 0.5 if group["update_rms_scaling"] else 1.0
        lr_t = lr.reshape(()).float() if torch.is_tensor(lr) else torch.full((), float(lr), device=dev)
        ptr_t, own_t = self._bucket_tables(bi, ps, slots, dev)
        stats = torch.zeros(count, 3, dtype=torch.float32, device=dev)
        C.muon_apply(o, ptr_t, sumsq, lr_t, float(wd), float(scale), float(group["eps"]), skip, stats)
        metrics["raw"].append((sumsq / mn).sqrt())
        ortho = (stats[:, 0] / mn).sqrt()
        metrics["ortho"].append(ortho)
        metrics["scaled"].append(ortho * scale)
        per = torch.zeros(len(ps), 2, dtype=torch.float32, device=dev).index_add_(0, own_t, stats[:, 1:])
        unorm, pnorm = per[:, 0].sqrt(), per[:, 1].sqrt()
        metrics["ratio"].append(lr_t * unorm / (pnorm.clamp_min(1e-30) / numel).clamp_min(group["eps"]) / numel)

    @torch.no_grad()
    def _step_sharded(self, skip=None):
        """Fully sharded parameters (DTensor shards along dim 0): momentum per local shard; the
        momentum-updated matrix is all-gathered, orthogonalised whole (Newton-Schulz needs the full
        matrix), and every rank applies its own rows of the update."""
        from torch.distributed.tensor import DTensor
        metrics = {"raw": [], "ortho": [], "scaled": [], "ratio": []}
        for group in self.param_groups:
            lr, mom, wd = group["lr"], group["momentum"], group["weight_decay"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                sharded = isinstance(p, DTensor)
                pl = p.to_local() if sharded else p
                g = p.grad.to_local() if isinstance(p.grad, DTensor) else p.grad
                st = self.state[p]
                buf = st.get("momentum_buffer")
                if buf is None:
                    buf = st["momentum_buffer"] = torch.zeros_like(pl)
                g = g.to(buf.dtype)
                if skip is not None:
                    g = torch.where(skip, torch.zeros((), device=g.device, dtype=g.dtype), g)
                    buf.mul_(torch.where(skip, 1.0, mom).to(buf.dtype)).add_(g)
                else:
                    buf.mul_(mom).add_(g)
                raw = g.add(buf, alpha=mom) if group["nesterov"] else buf
                if sharded:
                    raw_full = DTensor.from_local(raw, p.device_mesh, p.placements, shape=p.shape,
                                                  stride=p.stride()).full_tensor()
                else:
                    raw_full = raw
                slot = self._slots[id(p)]
                blocks = slot.to_blocks(raw_full).float()
                ortho = batched_newton_schulz(blocks, steps=group["ns_steps"], eps=group["eps"],
                                              dtype=self._resolved_ns_dtype(p.device))
                scale = max(slot.rows, slot.cols) ** 0.5 if group["update_rms_scaling"] else 1.0
                metrics["raw"].append(blocks.flatten(1).square().mean(1).sqrt())
                metrics["ortho"].append(ortho.flatten(1).square().mean(1).sqrt())
                metrics["scaled"].append(metrics["ortho"][-1] * scale)
                upd = slot.from_blocks(ortho).to(pl.dtype).mul_(scale)
                if sharded:
                    mesh = p.device_mesh
                    upd = torch.chunk(upd, mesh.size(), dim=0)[mesh.get_local_rank()]
                lr_eff = torch.where(skip, 0.0, lr) if skip is not None else lr
                if wd:
                    pl.mul_(1.0 - lr_eff * wd)
                if torch.is_tensor(lr_eff):
                    pl.add_(upd * (-lr_eff).to(upd.dtype))
                else:
                    pl.add_(upd, alpha=-lr_eff)
                prms = pl.float().square().mean().sqrt().clamp_min(group["eps"])  # this rank's rows
                lr_v = lr if torch.is_tensor(lr) else torch.tensor(float(lr), device=prms.device)
                metrics["ratio"].append((lr_v * metrics["scaled"][-1].mean() / prms)[None])
        self._metric_tensors = {k: torch.cat(v) for k, v in metrics.items() if v}
        self.last_update_metrics = {}
        return self._metric_tensors

    @torch.no_grad()
    def _step_sparse(self):
        """Parameters without gradients this step keep their momentum untouched (reference
        behaviour); the others are processed matrix by matrix."""
        self._ensure_buckets()
        metrics = {"raw": [], "ortho": [], "scaled": [], "ratio": []}
        for group in self.param_groups:
            lr, mom, wd = group["lr"], group["momentum"], group["weight_decay"]
            for p in group["params"]:
                if p.grad is None or not self._mine(p) or self._tp_gathered(p):
                    continue
                slot = self._slots[id(p)]
                buf = self.state[p]["momentum_buffer"]
                buf.mul_(mom).add_(p.grad)
                raw = p.grad.add(buf, alpha=mom) if group["nesterov"] else buf
                ortho = batched_newton_schulz(slot.to_blocks(raw).float(), steps=group["ns_steps"], eps=group["eps"],
                                              dtype=self._resolved_ns_dtype(p.device))
                metrics["raw"].append(slot.to_blocks(raw).float().flatten(1).square().mean(1).sqrt())
                metrics["ortho"].append(ortho.flatten(1).square().mean(1).sqrt())
                if group["update_rms_scaling"]:
                    ortho = ortho * (max(slot.rows, slot.cols) ** 0.5)
                metrics["scaled"].append(ortho.flatten(1).square().mean(1).sqrt())
                upd = slot.from_blocks(ortho).to(p.dtype)
                prms = p.float().square().mean().sqrt()
                metrics["ratio"].append((lr * upd.float().square().mean().sqrt() / prms.clamp_min(group["eps"]))[None])
                if wd:
                    p.mul_(1.0 - lr * wd)
                p.add_(upd, alpha=-lr)
        self._step_tp_gathered(None, metrics)
        self._metric_tensors = {k: torch.cat(v) for k, v in metrics.items() if v}
        self.last_update_metrics = {}
        return self._metric_tensors

    def update_metrics(self) -> dict:
        """Materialise the last step's update statistics (one device-to-host copy)."""
        if not self._metric_tensors:
            return {}
        keys = ("raw", "ortho", "scaled", "ratio")
        vals = torch.stack([self._metric_tensors[k].float().mean() for k in keys]).tolist()
        raw, ortho, scaled, ratio = vals
        self.last_update_metrics = {"muon/raw_update_rms": raw, "muon/orthogonal_update_rms": ortho,
                                    "muon/scaled_update_rms": scaled, "muon/ns_gain": scaled / max(raw, 1e-12),
                                    "muon/update_to_parameter_ratio": ratio}
        return self.last_update_metrics


def _is_dtensor(p) -> bool:
    try:
        from torch.distributed.tensor import DTensor
    except ImportError:  # pragma: no cover
        return False
    return isinstance(p, DTensor)


# --------------------------------------------------------------------------- QK-Clip
@dataclass
class QKClipReport:
    applied: bool
    events: int
    fraction_layers_clipped: float
    max_preclip_scale: float
    max_postclip_scale: float
    mean_rescale_factor: float
    min_rescale_factor: float
    consecutive_steps_active: int

    def metrics(self) -> dict:
        return {"qk_clip/applied": float(self.applied), "qk_clip/events": float(self.events),
                "qk_clip/fraction_layers_clipped": self.fraction_layers_clipped,
                "qk_clip/max_preclip_scale": self.max_preclip_scale,
                "qk_clip/max_postclip_scale": self.max_postclip_scale,
                "qk_clip/mean_rescale_factor": self.mean_rescale_factor,
                "qk_clip/min_rescale_factor": self.min_rescale_factor,
                "qk_clip/consecutive_steps_active": float(self.consecutive_steps_active)}


class QKClipController:
    """After each step: if ``s = rms(q) rms(k) sqrt(d) > tau`` scale W_q and W_k by ``sqrt(tau/s)``.

    Scales of every MLA layer are stacked, reduced (MAX over the TP group) in one
    collective and applied on the device.
    """

    def __init__(self, model, *, threshold, eps=1e-6, every_steps=1, include_kda_experimental=False):
        from ..models.kda import KimiDeltaAttention
        from ..models.mla import GatedMLA
        if threshold <= 0 or eps <= 0 or every_steps <= 0:
            raise ValueError("invalid QK-Clip configuration")
        self.threshold, self.eps, self.every_steps = float(threshold), float(eps), int(every_steps)
        self.layers = []
        for name, m in model.named_modules():
            custom = getattr(m, "_kimi_qk_weights", None)
            if custom is not None:
                self.layers.append((name, m, custom[0], custom[1]))
            elif isinstance(m, GatedMLA):
                self.layers.append((name, m, m.projections.query.weight, m.projections.latent_kv.key_up.weight))
            elif include_kda_experimental and isinstance(m, KimiDeltaAttention):
                self.layers.append((name, m, m.projections.q_proj.weight, m.projections.k_proj.weight))
        self.total_events = 0
        self.consecutive_steps_active = 0
        self._pending = None
        self.replica_group = None  # data-parallel group: scales are MAX-reduced over it as well

    @torch.no_grad()
    def apply(self, step: int, *, materialize: bool = True, skip: torch.Tensor | None = None):
        if step % self.every_steps:
            return QKClipReport(False, 0, 0.0, 0.0, 0.0, 1.0, 1.0, self.consecutive_steps_active)
        active = [(m, wq, wk) for _, m, wq, wk in self.layers if getattr(m, "_last_qk_scale", None) is not None]
        if not active:
            return QKClipReport(False, 0, 0.0, 0.0, 0.0, 1.0, 1.0, self.consecutive_steps_active)
        scales = torch.stack([m._last_qk_scale.detach().float().reshape(()) for m, _, _ in active])
        group = getattr(active[0][0], "_kimi_qk_group", None)
        if group is not None and torch.distributed.is_initialized() and torch.distributed.get_world_size(group) > 1:
            torch.distributed.all_reduce(scales, op=torch.distributed.ReduceOp.MAX, group=group)
        # replicas (data parallel) and shards (fully sharded) of one matrix must take the same factor
        if self.replica_group is not None and torch.distributed.get_world_size(self.replica_group) > 1:
            torch.distributed.all_reduce(scales, op=torch.distributed.ReduceOp.MAX, group=self.replica_group)
        corr = torch.where(scales > self.threshold, self.threshold / scales.clamp_min(self.eps),
                           torch.ones_like(scales)).clamp(max=1.0)
        if skip is not None:  # the optimizer step was suppressed on the device: no clipping either
            corr = torch.where(skip, torch.ones_like(corr), corr)
        sym = corr.sqrt()
        for i, (_, wq, wk) in enumerate(active):
            for w in (wq, wk):
                (w.to_local() if _is_dtensor(w) else w).mul_(sym[i].to(w.dtype))
        self._pending = (scales, corr, len(self.layers))
        return self.report() if materialize else None

    def report(self) -> QKClipReport:
        if self._pending is None:
            return QKClipReport(False, 0, 0.0, 0.0, 0.0, 1.0, 1.0, self.consecutive_steps_active)
        scales, corr, n = self._pending
        self._pending = None
        s, c = scales.tolist(), corr.tolist()
        if any(not math.isfinite(v) for v in s):
            raise FloatingPointError("QK scale proxy is non-finite")
        factors = [f for f, v in zip(c, s) if v > self.threshold]
        events = len(factors)
        self.total_events += events
        self.consecutive_steps_active = self.consecutive_steps_active + 1 if events else 0
        return QKClipReport(bool(events), events, events / max(n, 1), max(s, default=0.0),
                            max([min(v, self.threshold) for v in s], default=0.0),
                            sum(factors) / len(factors) if factors else 1.0, min(factors, default=1.0),
                            self.consecutive_steps_active)

    def state_dict(self) -> dict:
        return {"threshold": self.threshold, "eps": self.eps, "every_steps": self.every_steps,
                "total_events": self.total_events, "consecutive_steps_active": self.consecutive_steps_active}

    def load_state_dict(self, state: dict) -> None:
        for key in ("threshold", "eps", "every_steps"):
            if float(state[key]) != float(getattr(self, key)):
                raise ValueError(f"QK-Clip {key} is incompatible")
        self.total_events = int(state["total_events"])
        self.consecutive_steps_active = int(state["consecutive_steps_active"])


# --------------------------------------------------------------------------- hybrid
@dataclass
class OptimizerStepReport:
    executed: bool
    adamw_lr: float
    muon_lr: float
    qk_clip_applied: bool
    qk_clip_events: int
    nonfinite_parameters: int
    update_metrics: dict = field(default_factory=dict)


def _all_finite(tensors) -> torch.Tensor:
    """Single device boolean: every tensor is finite."""
    if not tensors:
        return torch.ones((), dtype=torch.bool)
    tensors = [t.to_local() if _is_dtensor(t) else t for t in tensors]  # a shard is finite iff its rows are
    norms = torch._foreach_norm([t.float() if t.dtype not in (torch.float32, torch.float64) else t
                                 for t in tensors], 2.0)
    return torch.isfinite(torch.stack(norms)).all()


class KimiHybridOptimizer:
    """Muon (matrices) + AdamW (rest) + QK-Clip; a non-finite gradient skips the whole step."""

    def __init__(self, muon, adamw, report, config, qk_clip, mirror=None):
        self.muon, self.adamw, self.report, self.config, self.qk_clip = muon, adamw, report, config, qk_clip
        # bf16 copies of the projection weights read by the tensor-core GEMMs; rewritten (one
        # launch) at the end of every step, after Muon, AdamW and QK-Clip have written the masters
        self.weight_mirror = mirror
        self.step_number = 0
        self.last_step_report: OptimizerStepReport | None = None
        self.last_skip: torch.Tensor | None = None

    @property
    def param_groups(self):
        return self.muon.param_groups + self.adamw.param_groups

    @property
    def defaults(self):
        return {"muon": self.muon.defaults, "adamw": self.adamw.defaults}

    def zero_grad(self, set_to_none: bool = True) -> None:
        self.muon.zero_grad(set_to_none=set_to_none)
        self.adamw.zero_grad(set_to_none=set_to_none)

    @torch.no_grad()
    def step(self, closure=None, *, gradients_known_finite: bool = False,
             found_inf: torch.Tensor | None = None) -> OptimizerStepReport:
        """One hybrid step; a non-finite gradient skips it (reference: ``hybrid.py:59-112``).

        Host mode: one finite check read on the host decides. Device mode (``found_inf`` given,
        or inside :func:`kimi_k3_b200.runtime.sync_free`): the flag stays on the device and
        suppresses Muon, AdamW (``found_inf`` of the fused kernel) and QK-Clip without a host
        branch; ``last_skip`` holds it for the caller to read later.
        """
        if closure is not None:
            with torch.enable_grad():
                closure()
        params = [p for g in self.param_groups for p in g["params"] if p.grad is not None]
        if found_inf is not None or not host_checks():
            if found_inf is None:
                found_inf = ~_all_finite([p.grad for p in params])
            skip = found_inf.reshape(()).to(torch.bool)
            self.muon.step(skip=skip)
            self.adamw.found_inf = skip.to(torch.float32)
            try:
                self.adamw.step()
            finally:
                del self.adamw.found_inf
            self.step_number += 1
            if self.qk_clip is not None:
                self.qk_clip.apply(self.step_number, materialize=False, skip=skip)
            self.refresh_weight_mirror()
            self.last_skip = skip
            rep = OptimizerStepReport(True, self.adamw.param_groups[0]["lr"], self.muon.param_groups[0]["lr"], False,
                                      0, 0, {})
            self.last_step_report = rep
            return rep
        self.last_skip = None
        if not gradients_known_finite:
            if not bool(_all_finite([p.grad for p in params])):
                bad = sum(int(not torch.isfinite(p.grad).all()) for p in params)
                rep = OptimizerStepReport(False, self.adamw.param_groups[0]["lr"], self.muon.param_groups[0]["lr"],
                                          False, 0, bad, {})
                self.last_step_report = rep
                return rep
        self.muon.step()
        self.adamw.step()
        self.step_number += 1
        if self.qk_clip is not None:
            self.qk_clip.apply(self.step_number, materialize=False)
        self.refresh_weight_mirror()
        rep = OptimizerStepReport(True, self.adamw.param_groups[0]["lr"], self.muon.param_groups[0]["lr"], False, 0,
                                  0, {})
        self.last_step_report = rep
        return rep

    def refresh_weight_mirror(self) -> None:
        """Rewrite the bf16 weight mirrors from the fp32 masters (stream-ordered, one launch).  The
        optimizer calls it after every update; sharded data parallelism calls it again after the
        owners' broadcasts."""
        if self.weight_mirror is not None:
            self.weight_mirror.refresh()

    def restrict_to(self, param_ids) -> None:
        """Update only ``param_ids`` (sharded data parallelism): Muon keeps state for its owned
        matrices; AdamW skips the others because their gradients are dropped before its step."""
        self._owned = set(param_ids)
        self.muon.restrict_to(self._owned)

    def drop_foreign_gradients(self) -> None:
        owned = getattr(self, "_owned", None)
        if owned is None:
            return
        for g in self.param_groups:
            for p in g["params"]:
                if id(p) not in owned:
                    p.grad = None

    def undo_step_count(self) -> None:
        """A device-mode step turned out to be skipped: the host step counter steps back."""
        self.step_number = max(0, self.step_number - 1)

    def use_device_lrs(self) -> None:
        """Move every learning rate into a device tensor (read by replayed CUDA graphs).

        The scheduler then updates them in place; AdamW switches to its capturable form.
        """
        for opt in (self.muon, self.adamw):
            for g in opt.param_groups:
                dev = g["params"][0].device if g["params"] else torch.device("cpu")
                if not torch.is_tensor(g["lr"]):
                    g["lr"] = torch.tensor(float(g["lr"]), device=dev, dtype=torch.float32)
        for g in self.adamw.param_groups:
            g["capturable"] = True
            for p in g["params"]:
                st = self.adamw.state.get(p)
                if st and "step" in st and st["step"].device != p.device:
                    st["step"] = st["step"].to(p.device)

    def materialize_report(self) -> OptimizerStepReport:
        """Fill the last report's metrics (Muon statistics, QK-Clip) with one host sync each."""
        rep = self.last_step_report
        if rep is None or not rep.executed:
            return rep
        metrics = dict(self.muon.update_metrics())
        if self.qk_clip is not None:
            clip = self.qk_clip.report()
            metrics.update(clip.metrics())
            rep.qk_clip_applied, rep.qk_clip_events = clip.applied, clip.events
        rep.update_metrics = metrics
        return rep

    def set_lr(self, lr: float, muon_lr: float | None = None) -> None:
        if lr < 0 or (muon_lr is not None and muon_lr < 0):
            raise ValueError("learning rates must be non-negative")
        def assign(g, v):
            if torch.is_tensor(g["lr"]):
                g["lr"].fill_(v)
            else:
                g["lr"] = v
        for g in self.adamw.param_groups:
            assign(g, lr)
        for g in self.muon.param_groups:
            assign(g, lr if muon_lr is None else muon_lr)

    def set_lrs(self, *, adamw_lr: float, muon_lr: float) -> None:
        self.set_lr(adamw_lr, muon_lr)

    def get_lrs(self) -> dict:
        return {"adamw_lr": float(self.adamw.param_groups[0]["lr"]), "muon_lr": float(self.muon.param_groups[0]["lr"])}

    def parameter_assignment_report(self):
        return self.report

    def state_dict(self) -> dict:
        return {"format_version": 1, "muon": self.muon.state_dict(), "adamw": self.adamw.state_dict(),
                "parameter_registry_fingerprint": self.report.fingerprint, "parameter_registry": self.report.to_dict(),
                "config": self.config.to_dict(),
                "qk_clip": None if self.qk_clip is None else self.qk_clip.state_dict(),
                "step_number": self.step_number}

    def load_state_dict(self, state: dict, strict: bool = True) -> None:
        if strict and state.get("parameter_registry_fingerprint") != self.report.fingerprint:
            raise ValueError("optimizer parameter registry fingerprint mismatch")
        self.muon.load_state_dict(state["muon"])
        self.adamw.load_state_dict(state["adamw"])
        if self.qk_clip is not None and state.get("qk_clip") is not None:
            self.qk_clip.load_state_dict(state["qk_clip"])
        self.step_number = int(state.get("step_number", 0))


def build_kimi_optimizer(model, config: KimiOptimizerConfig | None = None):
    """Build ``(optimizer, registry)``: AdamW only, or Muon/Per-Head Muon + AdamW (+ QK-Clip)."""
    config = config or KimiOptimizerConfig()
    reg = build_parameter_registry(model, kind=config.kind, strict=config.fail_on_unclassified_matrix)
    decay = [s.parameter for s in reg.specs if s.optimizer_family == "adamw_decay"]
    no_decay = [s.parameter for s in reg.specs if s.optimizer_family == "adamw_no_decay"]
    fused = bool(decay + no_decay) and all(p.is_cuda and not _is_dtensor(p) for p in decay + no_decay)
    groups = [{"params": decay, "weight_decay": config.weight_decay, "group_name": "adamw_decay"},
              {"params": no_decay, "weight_decay": 0.0, "group_name": "adamw_no_decay"}]
    if config.kind == "adamw":
        return torch.optim.AdamW(groups, lr=config.adamw_lr, betas=config.adamw_betas, eps=config.adamw_eps,
                                 fused=fused or None), reg
    muon_specs = [s for s in reg.specs if s.optimizer_family in ("muon", "per_head_muon")]
    if not muon_specs:
        raise RuntimeError("Kimi optimizer found no Muon matrices")
    muon = KimiMuon([{"params": [s.parameter for s in muon_specs]}], lr=config.resolved_muon_lr,
                    momentum=config.muon_momentum, nesterov=config.muon_nesterov, ns_steps=config.muon_ns_steps,
                    eps=config.muon_ns_eps, weight_decay=config.resolved_muon_weight_decay,
                    update_rms_scaling=config.muon_update_rms_scaling,
                    spec_by_parameter={id(s.parameter): s for s in muon_specs}, ns_dtype=config.muon_ns_dtype)
    adamw = torch.optim.AdamW(groups, lr=config.adamw_lr, betas=config.adamw_betas, eps=config.adamw_eps,
                              fused=fused or None)
    qk = (QKClipController(model, threshold=config.qk_clip_threshold, eps=config.qk_clip_eps,
                           every_steps=config.qk_clip_every_steps,
                           include_kda_experimental=config.qk_clip_kda_experimental)
          if config.qk_clip_enabled else None)
    return KimiHybridOptimizer(muon, adamw, reg, config, qk, mirror=build_weight_mirror(model)), reg


def build_weight_mirror(model):
    """bf16 mirrors of the model's projection weights (every ``nn.Linear`` weight and the stacked
    routed-expert matrices) when they live on CUDA and the native kernels are enabled; else None.
    Weights a module declares in ``projection_groups()`` share one buffer per group (the fused GEMM
    reads them as one matrix)."""
    from .. import ops
    from ..ops.mirror import WeightMirror
    if any(_is_dtensor(p) for p in model.parameters()):
        return None  # fully sharded: weights exist whole only while their unit runs
    weights, seen = [], set()
    for mod in model.modules():
        cands = []
        if isinstance(mod, nn.Linear):
            cands.append(mod.weight)
        cands.extend(p for _, p in mod.named_parameters(recurse=False) if p.ndim == 3)
        for p in cands:
            if id(p) not in seen and p.is_cuda and p.dtype == torch.float32:
                seen.add(id(p))
                weights.append(p)
    if not weights or not ops.use_kernels(weights[0]):
        return None
    groups = []
    for mod in model.modules():
        declare = getattr(mod, "projection_groups", None)
        if callable(declare):
            groups.extend(declare())
    return WeightMirror(weights, groups=groups)


__all__ = [
    "KimiOptimizerConfig", "zeropower_via_newton_schulz", "batched_newton_schulz", "match_update_rms",
    "HeadMatrixLayout", "split_head_matrix", "merge_head_matrix", "per_head_orthogonalize", "MatrixParameterSpec",
    "ParameterAssignmentReport", "build_parameter_registry", "KimiMuon", "QKClipReport", "QKClipController",
    "OptimizerStepReport", "KimiHybridOptimizer", "build_kimi_optimizer", "build_weight_mirror",
]
