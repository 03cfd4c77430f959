"""Module-level benchmarks: KDA, Gated MLA, Stable LatentMoE, MTP, the hybrid backbone,
Attention Residuals and the training-diagnostics levels.

They mirror the reference's benchmark scripts (``benchmarks/benchmark_kda.py``,
``benchmark_mla.py``, ``benchmark_stable_latent_moe.py``, ``benchmark_mtp.py``,
``benchmark_hybrid_backbone.py``, ``benchmark_attention_residuals.py`` and
``scripts/benchmark_training_diagnostics.py``): same default shapes, same CSV / JSON
columns. Two differences: ``--device cuda`` runs them on the GPU with the sm_100a
kernels and times each call with CUDA events (``time_fn``), and the byte columns report
device peak memory there instead of the process RSS.
"""
from __future__ import annotations

import argparse
import json
import math
import statistics

import torch
import torch.nn as nn

from .timing import device_peak_bytes, process_peak_memory_bytes, time_fn


def _device(name: str | None) -> torch.device:
    if name:
        return torch.device(name)
    return torch.device("cuda" if torch.cuda.is_available() else "cpu")


def _peak(device) -> int:
    return device_peak_bytes(device) if device.type == "cuda" else process_peak_memory_bytes()


def _secs(fn, device, repeats, warmup=1) -> float:
    with torch.inference_mode():
        return time_fn(fn, device=device, warmup=warmup, repeats=repeats, flush=False).min_ms / 1e3


def _common(p: argparse.ArgumentParser) -> argparse.ArgumentParser:
    p.add_argument("--device", default=None, help="cpu or cuda (default: cuda when available)")
    return p


# --------------------------------------------------------------------------- KDA
def kda_state_elements(state) -> int:
    return sum(t.numel() for t in (state.recurrent_state, state.q_conv_state.buffer, state.k_conv_state.buffer,
                                   state.v_conv_state.buffer, state.sequence_offset))


def bench_kda(argv=None) -> list:
    """``length,recurrent_seconds,chunkwise_seconds,decode_ms,state_elements`` (reference
    ``benchmarks/benchmark_kda.py:43-80``)."""
    from ..models.kda import KDAConfig, KimiDeltaAttention
    p = _common(argparse.ArgumentParser(description="KDA recurrent vs chunkwise vs decode"))
    p.add_argument("--lengths", nargs="+", type=int, default=[64, 256, 1024, 4096])
    p.add_argument("--repeats", type=int, default=1)
    p.add_argument("--d-model", type=int, default=16)
    p.add_argument("--heads", type=int, default=2)
    p.add_argument("--key-head-dim", type=int, default=4)
    p.add_argument("--value-head-dim", type=int, default=8)
    args = p.parse_args(argv)
    dev = _device(args.device)
    torch.manual_seed(0)
    model = KimiDeltaAttention(KDAConfig(d_model=args.d_model, num_heads=args.heads, key_head_dim=args.key_head_dim,
                                         value_head_dim=args.value_head_dim, chunk_size=64,
                                         secondary_tile_size=16)).to(dev).eval()
    rows = []
    print("length,recurrent_seconds,chunkwise_seconds,decode_ms,state_elements")
    for length in args.lengths:
        hidden = torch.randn(1, length, args.d_model, device=dev)
        res = {}
        for mode in ("recurrent", "chunkwise"):
            res[mode] = _secs(lambda: model(hidden, mode=mode, output_final_state=True), dev, args.repeats)
        with torch.inference_mode():
            chunk_state = model(hidden, mode="chunkwise", output_final_state=True).state
            rec_state = model(hidden, mode="recurrent", output_final_state=True).state
        token = hidden[:, :1]
        decode = _secs(lambda: model(token, state=chunk_state.clone(), mode="decode"), dev, 1, warmup=0)
        if kda_state_elements(rec_state) != kda_state_elements(chunk_state):
            raise AssertionError("recurrent and chunkwise states differ in size")
        row = (length, res["recurrent"], res["chunkwise"], decode * 1e3, kda_state_elements(chunk_state))
        print(f"{row[0]},{row[1]:.6f},{row[2]:.6f},{row[3]:.3f},{row[4]}")
        rows.append(row)
    return rows


# --------------------------------------------------------------------------- MLA
def bench_mla(argv=None) -> list:
    """``length,seconds,decode_ms,latent_elements,full_kv_elements,compression_ratio``
    (reference ``benchmarks/benchmark_mla.py:28-61``)."""
    from ..models.mla import GatedMLA, GatedMLAConfig
    p = _common(argparse.ArgumentParser(description="Gated MLA prefill and latent-cache decode"))
    p.add_argument("--lengths", nargs="+", type=int, default=[64, 256, 1024])
    p.add_argument("--repeats", type=int, default=3)
    args = p.parse_args(argv)
    dev = _device(args.device)
    torch.manual_seed(0)
    cfg = GatedMLAConfig(d_model=64, num_heads=4, q_head_dim=16, v_head_dim=16, kv_latent_dim=32)
    model = GatedMLA(cfg).to(dev).eval()
    rows = []
    print("length,seconds,decode_ms,latent_elements,full_kv_elements,compression_ratio")
    for length in args.lengths:
        hidden = torch.randn(1, length, cfg.d_model, device=dev)
        secs = _secs(lambda: model(hidden, use_cache=True), dev, args.repeats)
        with torch.inference_mode():
            prefill = model(hidden, use_cache=True)
        token = torch.randn(1, 1, cfg.d_model, device=dev)
        decode = _secs(lambda: model(token, cache=prefill.cache, use_cache=True), dev, 1, warmup=0)
        row = (length, secs, decode * 1e3, prefill.cache.cache_elements, length * cfg.full_kv_width,
               cfg.cache_compression_ratio)
        print(f"{row[0]},{row[1]:.6f},{row[2]:.3f},{row[3]},{row[4]},{row[5]:.3f}")
        rows.append(row)
    return rows


# --------------------------------------------------------------------------- MoE
def _make_moe(backend, top_k, experts, d_model, latent_dim):
    from ..models.moe import StableLatentMoE, StableLatentMoEConfig
    return StableLatentMoE(StableLatentMoEConfig(
        d_model=d_model, latent_dim=latent_dim, num_shared_experts=2, num_routed_experts=experts,
        routed_experts_per_token=top_k, shared_expert_hidden_dim=2 * d_model, routed_expert_hidden_dim=2 * latent_dim,
        routing_backend=backend, enable_quantile_balancing=top_k < experts))


def bench_moe(argv=None) -> list:
    """``backend,routing,tokens,top_k,forward_ms,forward_backward_ms,assignments,
    zero_load_experts,load_cv,process_peak_bytes`` (reference
    ``benchmarks/benchmark_stable_latent_moe.py:88-150``)."""
    p = _common(argparse.ArgumentParser(description="Stable LatentMoE reference vs vectorized dispatch"))
    p.add_argument("--tokens", nargs="+", type=int, default=[1, 64, 256])
    p.add_argument("--top-k", nargs="+", type=int, default=[1, 2])
    p.add_argument("--experts", type=int, default=8)
    p.add_argument("--d-model", type=int, default=32)
    p.add_argument("--latent-dim", type=int, default=16)
    p.add_argument("--repeats", type=int, default=3)
    args = p.parse_args(argv)
    dev = _device(args.device)
    torch.manual_seed(0)
    rows = []
    print("backend,routing,tokens,top_k,forward_ms,forward_backward_ms,assignments,zero_load_experts,load_cv,"
          "process_peak_bytes")
    for top_k in args.top_k:
        for tokens in args.tokens:
            inputs = torch.randn(tokens, args.d_model, device=dev)
            for routing in ("natural", "imbalanced"):
                ref = _make_moe("reference", top_k, args.experts, args.d_model, args.latent_dim).to(dev)
                vec = _make_moe("vectorized", top_k, args.experts, args.d_model, args.latent_dim).to(dev)
                vec.load_state_dict(ref.state_dict())
                for backend, model in (("reference", ref), ("vectorized", vec)):
                    if routing == "imbalanced":
                        with torch.no_grad():
                            model.routing_bias.copy_(torch.linspace(4.0, -4.0, args.experts, device=dev))
                    fwd = _secs(lambda: model(inputs, return_router_diagnostics=True), dev, args.repeats)
                    with torch.inference_mode():
                        out = model(inputs, return_router_diagnostics=True)

                    def fwd_bwd():
                        value = inputs.detach().clone().requires_grad_()
                        model.zero_grad(set_to_none=True)
                        model(value).square().mean().backward()

                    bwd = time_fn(fwd_bwd, device=dev, warmup=1, repeats=args.repeats, flush=False).min_ms / 1e3
                    d = out.diagnostics
                    row = (backend, routing, tokens, top_k, fwd * 1e3, bwd * 1e3, int(d.num_assignments),
                           int(d.zero_load_experts), float(d.coefficient_of_variation), _peak(dev))
                    print(f"{row[0]},{row[1]},{row[2]},{row[3]},{row[4]:.3f},{row[5]:.3f},{row[6]},{row[7]},"
                          f"{row[8]:.4f},{row[9]}")
                    rows.append(row)
    return rows


# --------------------------------------------------------------------------- MTP
def build_mtp_modules(vocab_size: int = 128, d_model: int = 16):
    """Embedding, one-repeat KimiBlock, tied LM head and MTP head (reference
    ``benchmarks/benchmark_mtp.py:19-81``)."""
    from ..models.attnres import AttentionResidualConfig
    from ..models.backbone import KimiBlock, KimiBlockConfig
    from ..models.kda import KDAConfig
    from ..models.mla import GatedMLAConfig
    from ..models.moe import StableLatentMoEConfig
    from ..models.mtp import KimiMTPConfig, KimiMTPHead
    kda = KDAConfig(d_model=d_model, num_heads=2, key_head_dim=4, value_head_dim=d_model // 2,
                    short_conv_kernel_size=2, chunk_size=8, secondary_tile_size=4, decay_initializer="zeros")
    mla = GatedMLAConfig(d_model=d_model, num_heads=2, q_head_dim=4, v_head_dim=d_model // 2, kv_latent_dim=8,
                         attention_backend="manual")
    moe = StableLatentMoEConfig(d_model=d_model, latent_dim=d_model // 2, num_shared_experts=2, num_routed_experts=4,
                                routed_experts_per_token=2, shared_expert_hidden_dim=12, routed_expert_hidden_dim=10)
    ar = AttentionResidualConfig(d_model, mode="block", sublayers_per_depth_block=4)
    cfg = KimiMTPConfig(d_model=d_model, vocab_size=vocab_size, kda_config=kda, mla_config=mla,
                        stable_latent_moe_config=moe, attention_residual_config=ar)
    emb = nn.Embedding(vocab_size, d_model)
    head = nn.Linear(d_model, vocab_size, bias=False)
    head.weight = emb.weight
    block = KimiBlock(KimiBlockConfig(d_model=d_model, num_pattern_repeats=1, kda_config=kda, mla_config=mla,
                                      stable_latent_moe_config=moe, attention_residual_config=ar))
    return emb.eval(), block.eval(), head.eval(), KimiMTPHead(cfg, emb, head).eval()


def bench_mtp(argv=None) -> dict:
    """Main-only vs main + MTP latency and the MTP head's unique parameters (reference
    ``benchmarks/benchmark_mtp.py:93-126``)."""
    from ..models.mtp import mtp_parameter_counts
    p = _common(argparse.ArgumentParser(description="MTP latency overhead"))
    p.add_argument("--batch-size", type=int, default=2)
    p.add_argument("--tokens", type=int, default=32)
    p.add_argument("--iterations", type=int, default=10)
    args = p.parse_args(argv)
    dev = _device(args.device)
    torch.manual_seed(0)
    if dev.type == "cpu":
        torch.set_num_threads(1)
    emb, block, head, mtp = build_mtp_modules()
    emb, block, head, mtp = (m.to(dev) for m in (emb, block, head, mtp))
    ids = torch.randint(0, mtp.config.vocab_size, (args.batch_size, args.tokens), device=dev)

    def main_only():
        return head(block(emb(ids)).last_hidden_state)

    def main_with_mtp():
        hidden = block(emb(ids)).last_hidden_state
        return head(hidden), mtp(hidden, ids).logits

    with torch.inference_mode():
        t_main = statistics.median(time_fn(main_only, device=dev, warmup=1, repeats=args.iterations,
                                           flush=False).samples) / 1e3
        t_both = statistics.median(time_fn(main_with_mtp, device=dev, warmup=1, repeats=args.iterations,
                                           flush=False).samples) / 1e3
    counts = mtp_parameter_counts(mtp)
    overhead = 100.0 * (t_both / t_main - 1.0)
    print(f"main_only_median_ms={1e3 * t_main:.3f}")
    print(f"main_plus_mtp_median_ms={1e3 * t_both:.3f}")
    print(f"mtp_latency_overhead_percent={overhead:.2f}")
    print(f"unique_mtp_parameters={counts['unique_mtp_total']}")
    return {"main_only_s": t_main, "main_plus_mtp_s": t_both, "overhead_percent": overhead, **counts}


# --------------------------------------------------------------------------- backbone
def _hybrid_backbone(groups: int, attnres=None, d_model: int = 32, heads: int = 4):
    from ..models.backbone import HybridAttentionBackbone, HybridBackboneConfig
    from ..models.kda import KDAConfig
    from ..models.mla import GatedMLAConfig
    return HybridAttentionBackbone(HybridBackboneConfig(
        d_model=d_model, num_hybrid_groups=groups, mlp_hidden_dim=64,
        kda_config=KDAConfig(d_model=d_model, num_heads=heads, key_head_dim=4, value_head_dim=8,
                             short_conv_kernel_size=4, chunk_size=64, secondary_tile_size=16),
        mla_config=GatedMLAConfig(d_model=d_model, num_heads=heads, q_head_dim=8, v_head_dim=8, kv_latent_dim=16),
        attention_residual_config=attnres)).eval()


def backbone_cache_bytes(cache) -> int:
    total = 0
    for layer in cache.layer_caches:
        if layer.attention_type == "kda":
            s = layer.state
            tensors = (s.recurrent_state, s.q_conv_state.buffer, s.k_conv_state.buffer, s.v_conv_state.buffer)
        else:
            tensors = (layer.state.latent_kv,)
        total += sum(t.numel() * t.element_size() for t in tensors)
    return total


def bench_backbone(argv=None) -> list:
    """``groups,length,full_seconds,prefill_seconds,decode_ms,cache_elements,cache_bytes,
    process_peak_bytes`` (reference ``benchmarks/benchmark_hybrid_backbone.py:103-160``)."""
    p = _common(argparse.ArgumentParser(description="Hybrid backbone full / prefill / decode"))
    p.add_argument("--groups", nargs="+", type=int, default=[1, 2, 4])
    p.add_argument("--lengths", nargs="+", type=int, default=[64, 256])
    p.add_argument("--repeats", type=int, default=2)
    args = p.parse_args(argv)
    dev = _device(args.device)
    torch.manual_seed(0)
    rows = []
    print("groups,length,full_seconds,prefill_seconds,decode_ms,cache_elements,cache_bytes,process_peak_bytes")
    for groups in args.groups:
        model = _hybrid_backbone(groups).to(dev)
        for length in args.lengths:
            hidden = torch.randn(1, length, model.config.d_model, device=dev)
            full = _secs(lambda: model(hidden, mode="full"), dev, args.repeats)
            pre = _secs(lambda: model(hidden, mode="prefill", use_cache=True), dev, args.repeats)
            with torch.inference_mode():
                prefill = model(hidden, mode="prefill", use_cache=True)
            token = torch.randn(1, 1, model.config.d_model, device=dev)
            dec = _secs(lambda: model(token, cache=prefill.cache, mode="decode", use_cache=True), dev, args.repeats)
            row = (groups, length, full, pre, dec * 1e3, prefill.cache.total_elements,
                   backbone_cache_bytes(prefill.cache), _peak(dev))
            print(f"{row[0]},{row[1]},{row[2]:.6f},{row[3]:.6f},{row[4]:.3f},{row[5]},{row[6]},{row[7]}")
            rows.append(row)
    return rows


# --------------------------------------------------------------------------- Attention Residuals
class DepthMixMicrostack(nn.Module):
    """``2 * layers`` linear+tanh sublayers mixed by standard residuals, Full AttnRes or
    Block AttnRes (eager or two-phase); returns the output, the peak source elements, the
    conceptual source reads and the inter-block scans (reference
    ``benchmarks/benchmark_attention_residuals.py:46-160``)."""

    def __init__(self, d_model: int, transformer_layers: int, mode: str, backend: str, block_size: int):
        super().__init__()
        from ..models.attnres import (AttentionResidualSite, BlockAttentionResidualController, DepthSiteMetadata,
                                      FullAttentionResidualController)
        self.mode, self.backend, self.block_size = mode, backend, block_size
        self.transforms = nn.ModuleList(nn.Linear(d_model, d_model, bias=False) for _ in range(2 * transformer_layers))
        if mode == "standard":
            self.sites, self.final_site, self.controller = nn.ModuleList(), None, None
            return
        n = 2 * transformer_layers
        self.sites = nn.ModuleList(
            AttentionResidualSite(d_model, metadata=DepthSiteMetadata(
                site_index=i, transformer_layer_index=i // 2, site_kind="pre_attention" if i % 2 == 0 else "pre_ffn",
                attention_type="kda", hybrid_group_index=None, position_in_hybrid_group=None,
                depth_block_index=i // block_size if mode == "block" else None,
                position_in_depth_block=i % block_size if mode == "block" else None))
            for i in range(n))
        self.final_site = AttentionResidualSite(d_model, metadata=DepthSiteMetadata(
            n, None, "final_output", None, None, None, None, None))
        self.controller = (FullAttentionResidualController() if mode == "full"
                           else BlockAttentionResidualController(block_size, backend))

    def forward(self, embedding):
        from ..models.attnres import FullAttentionResidualState
        if self.mode == "standard":
            hidden = embedding
            for tr in self.transforms:
                hidden = hidden + torch.tanh(tr(hidden))
            return hidden, 2 * embedding.numel(), 2 * len(self.transforms), 0
        state = self.controller.initialize(embedding)
        by_block: dict = {}
        if self.mode == "block":
            for site in self.sites:
                by_block.setdefault(site.metadata.depth_block_index, []).append(site)
        by_block = {k: tuple(v) for k, v in by_block.items()}
        peak = state.source_elements
        reads = 0
        full = isinstance(state, FullAttentionResidualState)
        for site, tr in zip(self.sites, self.transforms):
            if self.mode == "block":
                self.controller.prepare_depth_block(state, by_block[site.metadata.depth_block_index])
            reads += len(state.sources) if full else 1 + len(state.completed_blocks) + int(state.partial_block is not None)
            mixed = self.controller.mix_for_site(site, state).mixed_state
            self.controller.append_output(state, torch.tanh(tr(mixed)))
            peak = max(peak, state.source_elements)
        reads += len(state.sources) if full else 1 + math.ceil(len(self.sites) / self.block_size)
        out = self.controller.finalize(state, self.final_site).mixed_state
        peak = max(peak, state.source_elements)
        return out, peak, reads, (0 if full else state.inter_block_scan_count)


def bench_attnres(argv=None) -> list:
    """Depth-mixing microstack CSV, then decode through the integrated backbone (reference
    ``benchmarks/benchmark_attention_residuals.py:222-296``)."""
    from ..models.attnres import AttentionResidualConfig
    p = _common(argparse.ArgumentParser(description="Attention Residuals depth mixing and decode"))
    p.add_argument("--layers", nargs="+", type=int, default=[2, 4, 8, 16])
    p.add_argument("--lengths", nargs="+", type=int, default=[1, 64, 256])
    p.add_argument("--decode-contexts", nargs="+", type=int, default=[64, 256])
    p.add_argument("--d-model", type=int, default=32)
    p.add_argument("--block-size", type=int, default=4)
    p.add_argument("--repeats", type=int, default=3)
    args = p.parse_args(argv)
    dev = _device(args.device)
    torch.manual_seed(0)
    modes = (("standard", "eager"), ("full", "eager"), ("block", "eager"), ("block", "two_phase"))
    rows = []
    print("kind,mode,backend,layers,length,seconds,peak_source_bytes,conceptual_source_reads,inter_block_scans")
    for layers in args.layers:
        for length in args.lengths:
            hidden = torch.randn(1, length, args.d_model, device=dev)
            for mode, backend in modes:
                stack = DepthMixMicrostack(args.d_model, layers, mode, backend, args.block_size).to(dev).eval()
                secs = _secs(lambda: stack(hidden), dev, args.repeats)
                with torch.inference_mode():
                    _, peak, reads, scans = stack(hidden)
                row = ("depth", mode, backend, layers, length, secs, peak * hidden.element_size(), reads, scans)
                print(f"depth,{mode},{backend},{layers},{length},{secs:.6f},{row[6]},{reads},{scans}")
                rows.append(row)
    print("kind,mode,backend,context,decode_ms,persistent_cache_elements,persistent_cache_bytes,attnres_cache_entries")
    for mode, backend in modes:
        cfg = None
        if mode == "full":
            cfg = AttentionResidualConfig(32, mode="full", sublayers_per_depth_block=None)
        elif mode == "block":
            cfg = AttentionResidualConfig(32, mode="block", sublayers_per_depth_block=4, backend=backend)
        model = _hybrid_backbone(1, cfg).to(dev)
        for context in args.decode_contexts:
            hidden = torch.randn(1, context, 32, device=dev)
            with torch.inference_mode():
                prefill = model(hidden, mode="prefill", use_cache=True)
            token = torch.randn(1, 1, 32, device=dev)
            secs = _secs(lambda: model(token, cache=prefill.cache, mode="decode", use_cache=True), dev, args.repeats)
            with torch.inference_mode():
                decoded = model(token, cache=prefill.cache, mode="decode", use_cache=True)
            row = ("decode", mode, backend, context, secs * 1e3, decoded.cache.total_elements,
                   backbone_cache_bytes(decoded.cache), 0)
            print(f"decode,{mode},{backend},{context},{row[4]:.3f},{row[5]},{row[6]},0")
            rows.append(row)
    return rows


# --------------------------------------------------------------------------- diagnostics levels
def _percentile90(values):
    ordered = sorted(values)
    return ordered[min(len(ordered) - 1, int(0.9 * len(ordered)))]


def run_diagnostics_mode(mode: str, context: int, steps: int, device) -> dict:
    """One short training run at a diagnostics level (off / cheap / standard / deep);
    reference ``scripts/benchmark_training_diagnostics.py:28-112``."""
    import time
    from torch.utils.data import DataLoader
    from .. import KimiK3, kimi_k3_cpu_tiny_config
    from ..train.diagnostics import DiagnosticsConfig, KimiDiagnosticCollector
    from ..train.loop import train_one_epoch
    from ..train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
    torch.manual_seed(17)
    model = KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False)).to(device)
    optimizer, registry = build_kimi_optimizer(model, KimiOptimizerConfig(qk_clip_enabled=True))
    intervals = {"cheap": (steps + 1, steps + 1), "standard": (1, steps + 1), "deep": (steps + 1, 1)}
    collector = None
    if mode != "off":
        standard, deep = intervals[mode]
        collector = KimiDiagnosticCollector(model, DiagnosticsConfig(cheap_every_steps=1, standard_every_steps=standard,
                                                                     deep_every_steps=deep),
                                            parameter_specs=registry.specs)
    gen = torch.Generator().manual_seed(123)
    batches = [{"input_ids": torch.randint(5, 128, (context,), generator=gen),
                "labels": torch.randint(5, 128, (context,), generator=gen),
                "attention_mask": torch.ones(context, dtype=torch.bool)} for _ in range(steps)]
    metrics = []
    if device.type == "cuda":
        torch.cuda.reset_peak_memory_stats(device)
        torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    train_one_epoch(model, DataLoader(batches, batch_size=1), optimizer, device=device, diagnostics=collector,
                    max_batches=steps, use_mtp=True, on_optimizer_step=lambda m: metrics.append(dict(m)))
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    elapsed = time.perf_counter() - t0
    times = [m["train/step_time_ms"] for m in metrics]
    tokens = sum(m["tokens"] for m in metrics)
    return {"mode": mode, "context": context, "steps": steps, "median_step_time_ms": statistics.median(times),
            "p90_step_time_ms": _percentile90(times), "tokens_per_second": tokens / elapsed,
            "max_allocated_gpu_mb": torch.cuda.max_memory_allocated(device) / 1024 ** 2 if device.type == "cuda" else 0.0,
            "persistent_diagnostic_bytes": max((m.get("diagnostics/persistent_gpu_bytes", 0.0) for m in metrics),
                                               default=0.0),
            "scalars": max((m.get("diagnostics/scalars_emitted", 0.0) for m in metrics), default=0.0)}


def bench_diagnostics(argv=None) -> list:
    p = _common(argparse.ArgumentParser(description="training step time at each diagnostics level"))
    p.add_argument("--contexts", type=int, nargs="+", default=[512, 2048])
    p.add_argument("--steps", type=int, default=5)
    args = p.parse_args(argv)
    dev = _device(args.device)
    rows = []
    for context in args.contexts:
        base = run_diagnostics_mode("off", context, args.steps, dev)
        rows.append({**base, "overhead_vs_off": 0.0})
        for mode in ("cheap", "standard", "deep"):
            r = run_diagnostics_mode(mode, context, args.steps, dev)
            r["overhead_vs_off"] = r["median_step_time_ms"] / max(base["median_step_time_ms"], 1e-12) - 1.0
            rows.append(r)
    print(json.dumps(rows, indent=2))
    return rows


BENCHMARKS = {"kda": bench_kda, "mla": bench_mla, "moe": bench_moe, "mtp": bench_mtp, "backbone": bench_backbone,
              "attnres": bench_attnres, "diagnostics": bench_diagnostics}


# --------------------------------------------------------------------------- one flagship step, per kernel
def bench_step_profile(argv=None) -> str:
    """Per-kernel device time of one eager training step of the flagship model (the
    ``t4_wikitext`` architecture with vocab 50,257, batch 16 x 1024 tokens), from the torch
    profiler's CUDA activity after three warm-up steps. Shares, not absolute times, are what
    this table is for: the profiler serialises nothing but adds host overhead."""
    import time
    from torch.profiler import ProfilerActivity, profile
    from ..config.profiles import profile_model_config
    from ..models import KimiK3
    from ..train.engine import MoEController, TrainStepEngine
    from ..train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
    p = argparse.ArgumentParser(description="per-kernel profile of one training step")
    p.add_argument("--batch", type=int, default=16)
    p.add_argument("--seq-len", type=int, default=1024)
    p.add_argument("--vocab", type=int, default=50257)
    p.add_argument("--top", type=int, default=40)
    p.add_argument("--shapes", action="store_true", help="group the table by input shapes")
    args = p.parse_args(argv)
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    model = KimiK3(profile_model_config("t4_wikitext", vocab_size=args.vocab)).to(dev)
    opt, _ = build_kimi_optimizer(model, KimiOptimizerConfig(muon_lr=0.02, adamw_lr=3e-4, qk_clip_enabled=True))
    eng = TrainStepEngine(model, opt, grad_clip=1.0, moe_controller=MoEController(model))
    gen = torch.Generator().manual_seed(1)
    ids = torch.randint(3, args.vocab, (args.batch, args.seq_len), generator=gen).to(dev)
    batch = {"input_ids": ids, "labels": ids.clone(),
             "attention_mask": torch.ones_like(ids, dtype=torch.bool)}
    for _ in range(3):
        eng.step(batch, mask_all_valid=True)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], record_shapes=args.shapes) as prof:
        t0 = time.perf_counter()
        eng.step(batch, mask_all_valid=True)
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) * 1e3
    table = prof.key_averages(group_by_input_shape=args.shapes).table(
        sort_by="self_cuda_time_total" if args.shapes else "cuda_time_total", row_limit=args.top,
        max_name_column_width=60, max_shapes_column_width=90)
    print(f"step wall ms {wall:.1f}")
    print(table)
    return table


BENCHMARKS["step"] = bench_step_profile


def bench_decode(argv=None) -> list:
    """Serving decode throughput of the flagship architecture (``t4_wikitext``, vocab 50,257,
    random-init weights): prefill a batch of prompts, then generate ``--new-tokens`` per row.
    Rows: the CUDA-graph decoder (:class:`GraphDecoder`, bf16, one graph replay per token) and the
    reference-style loop (:func:`generate_tokens` under the same bf16 autocast: a new cache per
    token and every kernel launched from Python).  Decode time is the host time between two device
    synchronisations around the token loop."""
    import contextlib
    from ..config.profiles import profile_model_config
    from ..infer import GenerationConfig, GraphDecoder, generate_tokens
    from ..models import KimiK3
    p = argparse.ArgumentParser(description="decode throughput")
    p.add_argument("--batch", type=int, default=16)
    p.add_argument("--prompt", type=int, default=512)
    p.add_argument("--new-tokens", type=int, default=128)
    p.add_argument("--vocab", type=int, default=50257)
    p.add_argument("--sample", action="store_true", help="top-k 50 / top-p 0.9 sampling instead of greedy")
    p.add_argument("--skip-eager", action="store_true")
    p.add_argument("--profile", action="store_true", help="print the per-kernel table of eager decode steps")
    args = p.parse_args(argv)
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    model = KimiK3(profile_model_config("t4_wikitext", vocab_size=args.vocab)).to(dev).eval()
    ids = torch.randint(3, args.vocab, (args.batch, args.prompt), device=dev)
    cfg = GenerationConfig(max_new_tokens=args.new_tokens, do_sample=args.sample, top_k=50 if args.sample else None,
                           top_p=0.9 if args.sample else None, seed=0)
    rows = []

    def run(name, fn, new_tokens):
        fn()  # warm-up (and graph capture)
        torch.cuda.synchronize()
        out = fn()
        torch.cuda.synchronize()
        rows.append({"impl": name, "batch": args.batch, "prompt": args.prompt, "new_tokens": new_tokens,
                     "prefill_ms": round(out.prefill_seconds * 1e3, 3),
                     "decode_ms_per_token": round(out.decode_seconds * 1e3 / max(out.generated_tokens, 1), 4),
                     "decode_tokens_per_s": round(out.batch_tokens_per_second, 1)})
        print(json.dumps(rows[-1]))

    dec = GraphDecoder(model, max_length=args.prompt + args.new_tokens, generation_config=cfg)
    if args.profile:
        from torch.profiler import ProfilerActivity, profile
        eager_dec = GraphDecoder(model, max_length=args.prompt + 16, use_graph=False,
                                 generation_config=GenerationConfig(max_new_tokens=2))
        eager_dec.generate(ids)
        with torch.inference_mode():
            eager_dec._decode_step()
            torch.cuda.synchronize()
            with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], record_shapes=True) as prof:
                for _ in range(4):
                    eager_dec._decode_step()
                torch.cuda.synchronize()
        print("four eager decode steps")
        print(prof.key_averages(group_by_input_shape=True).table(sort_by="self_cuda_time_total", row_limit=30,
                                                                 max_name_column_width=60,
                                                                 max_shapes_column_width=80))
    run("cuda_graph_decoder", lambda: dec.generate(ids), args.new_tokens)
    if not args.skip_eager:
        n = min(args.new_tokens, 32)
        ecfg = GenerationConfig(max_new_tokens=n, do_sample=args.sample, top_k=cfg.top_k, top_p=cfg.top_p, seed=0)

        def eager():
            with torch.autocast("cuda", dtype=torch.bfloat16):
                return generate_tokens(model, ids, generation_config=ecfg)
        run("eager_reference_loop", eager, n)
    return rows


BENCHMARKS["decode"] = bench_decode


def bench_ep(argv=None) -> list:
    """Expert-parallel routed experts, forward + backward, per rank ``--tokens`` tokens of width
    ``--latent`` routed top-``--topk`` over ``--experts`` SiTU-GLU experts (hidden ``--hidden``)
    split over all ranks.  Compares the device-initiated NVLink exchange (``ep_fused``: dispatch
    into the owners' grouped inputs, combine in the down-GEMM epilogue) with the NCCL
    all-to-all path of :class:`ExpertParallelMoE`.  Run under torchrun (one rank per GPU); times
    are CUDA events on each rank, the max over ranks is reported."""
    import datetime
    import os
    from types import SimpleNamespace
    import torch.distributed as dist
    from ..models.moe import GroupedRoutedExperts, StableLatentMoE  # noqa: F401
    from ..parallel.ep_fused import EPWorkspace, fused_ep_experts
    from ..parallel.expert_parallel import exchange_counts, _a2a
    from .. import ops
    p = argparse.ArgumentParser(description="expert-parallel exchange")
    p.add_argument("--tokens", type=int, default=16384)
    p.add_argument("--latent", type=int, default=320)
    p.add_argument("--hidden", type=int, default=640)
    p.add_argument("--experts", type=int, default=12)
    p.add_argument("--topk", type=int, default=2)
    p.add_argument("--repeats", type=int, default=20)
    args = p.parse_args(argv)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dev = torch.device("cuda", torch.cuda.current_device())
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev,
                                rank=rank, world_size=world)
    m, l, h, e, k = args.tokens, args.latent, args.hidden, args.experts, args.topk
    per = e // world
    g = torch.Generator(device=dev).manual_seed(1 + rank)
    x = torch.randn(m, l, device=dev, generator=g).bfloat16()
    sel = torch.stack([torch.randperm(e, device=dev, generator=g)[:k] for _ in range(m)]) if m <= 4096 else \
        torch.topk(torch.rand(m, e, device=dev, generator=g), k, -1).indices
    w = torch.softmax(torch.randn(m, k, device=dev, generator=g), -1)
    gw = torch.Generator(device=dev).manual_seed(0)
    wg, wu, wd = (torch.randn(*s, device=dev, generator=gw) * 0.05 for s in ((per, h, l), (per, h, l), (per, l, h)))
    dout = torch.randn(m, l, device=dev, generator=g)
    ex = SimpleNamespace(gate_proj=wg.requires_grad_(), up_proj=wu.requires_grad_(), down_proj=wd.requires_grad_())
    ws = EPWorkspace(None, dev, tokens=m, top_k=k, latent=l, num_experts=e)
    xr, wr = x.clone().requires_grad_(), w.clone().requires_grad_()

    def fused():
        y = fused_ep_experts(xr, sel, wr, ex, ws, 4.0, 25.0)
        y.backward(dout)

    def nccl():
        flat_e = sel.reshape(-1)
        flat_t = torch.arange(m, device=dev).repeat_interleave(k)
        owner = torch.div(flat_e, per, rounding_mode="floor")
        order = torch.argsort(owner, stable=True)
        send = torch.bincount(owner, minlength=world).to(torch.int64)
        ins = send.tolist()
        outs = exchange_counts(send, None)
        rows = xr.index_select(0, flat_t[order])
        meta = torch.stack(((flat_e[order] - owner[order] * per).float(), wr.reshape(-1)[order]), 1)
        r_lat = _a2a(rows, outs, ins, None)
        r_meta = _a2a(meta, outs, ins, None)
        out = ops.moe_grouped_experts(r_lat, r_meta[:, 0].round().long()[:, None], r_meta[:, 1:2], ex.gate_proj,
                                      ex.up_proj, ex.down_proj, 4.0, 25.0)
        back = _a2a(out, ins, outs, None)
        y = torch.zeros(m, l, device=dev).index_add(0, flat_t[order], back)
        y.backward(dout)

    rows_out = []
    for name, fn in (("nvlink_fused", fused), ("nccl_all_to_all", nccl)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.repeats):
            fn()
        t1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([t0.elapsed_time(t1) / args.repeats], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.barrier()
        rows_out.append({"bench": "ep", "impl": name, "ranks": world, "tokens_per_rank": m, "latent": l,
                         "hidden": h, "experts": e, "top_k": k, "fwd_bwd_ms_max_over_ranks": round(ms.item(), 4),
                         "bytes_crossing_nvlink_per_rank_fwd": int(m * k * (world - 1) / world * (l * 2 + l * 4))})
        if rank == 0:
            print(json.dumps(rows_out[-1]), flush=True)
    ws.check()
    del ws
    dist.barrier()
    dist.destroy_process_group()
    return rows_out


BENCHMARKS["ep"] = bench_ep


def bench_allgather_gemm(argv=None) -> list:
    """Sequence-parallel column projection ``all_gather(x) @ W^T``: the fused kernel (A tiles
    TMA-loaded from the owners' shards over NVLink) against NCCL all-gather + the same GEMM.
    Run under torchrun; CUDA-event time per call, max over ranks."""
    import datetime
    import os
    import torch.distributed as dist
    from ..parallel.symmetric import AllGatherWorkspace, fused_allgather_matmul
    from ..ops import _loader
    p = argparse.ArgumentParser(description="fused all-gather GEMM")
    p.add_argument("--shard-rows", type=int, default=8192, help="rows per rank")
    p.add_argument("--k", type=int, default=640)
    p.add_argument("--cols-out", type=int, default=1920)
    p.add_argument("--repeats", type=int, default=50)
    args = p.parse_args(argv)
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dev = torch.device("cuda", torch.cuda.current_device())
    if not dist.is_initialized():
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    C = _loader.require()
    x = torch.randn(args.shard_rows, args.k, device=dev).bfloat16()
    w = torch.randn(args.cols_out, args.k, device=dev).bfloat16()
    ws = AllGatherWorkspace(None, dev, rows=args.shard_rows, cols=args.k)
    full = torch.empty(world * args.shard_rows, args.k, device=dev, dtype=torch.bfloat16)
    out = torch.empty(world * args.shard_rows, args.cols_out, device=dev, dtype=torch.bfloat16)
    bn = 256 if args.cols_out >= 256 else 128

    def fused():
        fused_allgather_matmul(x, w, ws, out=out)

    def nccl():
        dist.all_gather_into_tensor(full, x)
        C.tc_gemm_dense(full, w, False, False, False, bn, out)

    rows_out = []
    for name, fn in (("fused_allgather_gemm", fused), ("nccl_allgather_then_gemm", nccl)):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.repeats):
            fn()
        t1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([t0.elapsed_time(t1) / args.repeats], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        flops = 2.0 * world * args.shard_rows * args.k * args.cols_out
        rows_out.append({"bench": "allgather_gemm", "impl": name, "ranks": world, "rows_per_rank": args.shard_rows,
                         "k": args.k, "n": args.cols_out, "ms_max_over_ranks": round(ms.item(), 4),
                         "tflops": round(flops / ms.item() / 1e9, 1)})
        if rank == 0:
            print(json.dumps(rows_out[-1]), flush=True)
    ws.check()
    del ws
    dist.barrier()
    dist.destroy_process_group()
    return rows_out


BENCHMARKS["allgather_gemm"] = bench_allgather_gemm
