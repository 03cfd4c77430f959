"""Benchmark configurations beside the single-GPU flagship (``bench.py --config NAME``).

Every configuration has two arms with the same data, shapes, optimizer settings and timing:

* ``ours``: this package's models, kernels, engine and parallel runtime;
* ``reference``: the unmodified reference installed under ``baseline/_ref``, driven only
  through its public API (model builder, ``parallelize_kimi_model`` / ``wrap_data_parallel``,
  ``train_one_epoch``, ``inference_autoregressive`` / ``generate_tokens``).

Configurations (shapes from the reference's profiles; synthetic data, random-init weights):

``cpu_smoke``    cpu_smoke model on CPU in fp32: Muon + AdamW steps on synthetic key-value
                 retrieval sequences (batch 4, length 32, seed 0), then cached greedy decode
                 of 8 tokens.  Timed on the host clock (there is no device).
``gpu24_tp_ep``  gpu_24gb model, complete-head TP2 x EP(N/2) (2, 4, 8 GPUs), sequence 1,024,
                 global batch 32 sequences (fixed: strong scaling); EP ranks are data replicas.
                 Ours runs the fused GEMM + all-reduce output projections and the device-
                 initiated NVLink expert exchange.
``gpu48_fsdp``   gpu_48gb model, fully sharded data parallelism over N GPUs (N = 1: unsharded),
                 progressive context 2,048 -> 8,192 at 16,384 tokens per GPU per step (8 x 2,048,
                 then 2 x 8,192; weak scaling); the value is total tokens over total time.
``gpu80_infer``  gpu_80gb text stack, cached inference over N GPUs: prefill 64 prompts x 4,096
                 tokens, then 512 greedy decode steps.  Ours: TP-N attention with EP-N experts on
                 the same ranks (served from one captured CUDA graph per token); the reference's
                 topology rule (world = DP x TP x EP) admits TP-N or EP-N but not both, so its arm
                 runs TP-N.  Reports batch decode tokens/s (value), per-sequence decode tokens/s
                 (the reference's definition) and p50 time to first token.

Device time: CUDA events around the timed steps on the compute stream with a barrier and a
synchronize on both sides, max over ranks.  Inference splits prefill and decode with the
generation API's own synchronised clocks (max over ranks).
"""
from __future__ import annotations

import os
import statistics
import sys
import time

import torch

from .harness import ClockSampler, barrier, max_over_ranks

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF_DIR = os.path.join(_ROOT, "baseline", "_ref")
CONFIGS = ("cpu_smoke", "gpu24_tp_ep", "gpu48_fsdp", "gpu80_infer")


def optimizer_settings(**over):
    """The profiles' training.yaml optimizer values (per-head Muon + Muon + AdamW, QK-Clip)."""
    s = dict(kind="per_head_muon_adamw", adamw_lr=3e-4, adamw_betas=(0.9, 0.95), adamw_eps=1e-8, muon_lr=3e-4,
             muon_momentum=0.95, muon_nesterov=True, muon_ns_steps=5, muon_ns_eps=1e-7, muon_update_rms_scaling=True,
             weight_decay=0.1, per_head_qkv=True, qk_clip_enabled=True, qk_clip_threshold=100.0,
             qk_clip_every_steps=1)
    s.update(over)
    return s


def _reference_importable() -> None:
    if not os.path.isdir(os.path.join(REF_DIR, "src")):
        raise FileNotFoundError("baseline/_ref is not installed")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)


def _token_batches(n, batch, seq, vocab, seed, device=None):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        ids = torch.randint(0, vocab, (batch, seq + 1), generator=g)
        b = {"input_ids": ids[:, :-1].contiguous(), "labels": ids[:, 1:].contiguous(),
             "attention_mask": torch.ones(batch, seq, dtype=torch.bool)}
        out.append({k: v.to(device) for k, v in b.items()} if device is not None else b)
    return out


def _dist_dict(world, *, tp=1, ep=1, dp_mode="none", overlay=False, ours=False):
    """The ``distributed:`` mapping both arms load (``fused`` keys only on ours)."""
    d = {"enabled": world > 1, "backend": "nccl", "timeout_seconds": 600,
         "data_parallel": {"mode": dp_mode, "size": world if dp_mode != "none" else 1},
         "tensor_parallel": {"enabled": tp > 1, "size": tp},
         "expert_parallel": {"enabled": ep > 1, "size": ep}}
    if ours:
        if tp > 1:
            d["tensor_parallel"]["fused_output_reduce"] = True
        if ep > 1:
            d["expert_parallel"].update(dispatch="nvlink_fused", overlay_tensor_parallel=overlay)
    return d


class _ReferenceTimer:
    """``on_optimizer_step`` callback of the reference's ``train_one_epoch``: opens the timed
    region after ``warmup`` steps and closes it ``steps`` later."""

    def __init__(self, warmup, steps, local, sample_clocks=True):
        self.warmup, self.steps, self.n = warmup, steps, 0
        self.ev0, self.ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.sampler = ClockSampler(local) if sample_clocks else None
        self.t0 = self.t1 = None

    def __call__(self, _metrics):
        self.n += 1
        if self.n == self.warmup:
            torch.cuda.synchronize()
            barrier()
            if self.sampler is not None:
                self.sampler.start()
            torch.cuda.synchronize()
            barrier()
            self.t0 = time.perf_counter()
            self.ev0.record()
        elif self.n == self.warmup + self.steps:
            self.ev1.record()
            torch.cuda.synchronize()
            self.t1 = time.perf_counter()
            barrier()

    def result(self):
        clocks = self.sampler.stop() if self.sampler is not None else None
        return self.ev0.elapsed_time(self.ev1) / self.steps, (self.t1 - self.t0) * 1e3 / self.steps, clocks


def _reference_train(ref_train, model, opt, make_batches, args, local, **kw):
    """Time the reference's ``train_one_epoch`` over ``warmup + steps`` optimizer steps.

    Falls back, in this order and saying so in the returned note, to what the reference itself
    offers: fp32 when its bf16 autocast path raises (its AttnRes rejects mixed depth-source dtypes),
    and gradient accumulation over 2, 4 or 8 micro-batches (its ``grad_accum_steps``) when the full
    per-replica batch runs out of device memory.  ``make_batches(n, micro)`` returns ``n`` batches of
    ``1 / micro`` of the per-replica batch.  Returns (device ms, host ms, clocks, note)."""
    notes, amp = [], True
    for micro in (1, 2, 4, 8):
        batches = make_batches((args.warmup + args.steps) * micro, micro)
        while True:
            timer = _ReferenceTimer(args.warmup, args.steps, local)
            oom = False
            try:
                ref_train(model, batches, opt, amp_enabled=amp, amp_dtype="bf16", grad_accum_steps=micro,
                          max_batches=len(batches), on_optimizer_step=timer, **kw)
                if micro > 1:
                    notes.append(f"the full batch exceeds device memory in the reference; {micro} accumulated "
                                 "micro-batches per step")
                ms, host, clocks = timer.result()
                return ms, host, clocks, "; ".join(notes) or None
            except TypeError as exc:
                if not amp:
                    raise
                amp = False
                notes.append(f"reference bf16 autocast fails ({str(exc)[:100]}); measured in fp32")
            except torch.OutOfMemoryError:
                oom = True
            if oom:  # outside the handler, so the failed step's frames are gone before the cache is freed
                if timer.sampler is not None:
                    timer.sampler.stop()
                opt.zero_grad(set_to_none=True)
                torch.cuda.empty_cache()
                break
    raise torch.OutOfMemoryError("the reference runs out of device memory even with 8 micro-batches per step")


def _time_engine(engine, dev_batches, host_batches, warmup, steps, local):
    """Device-timed steps, then the same count end to end (pinned inputs in, loss out)."""
    for i in range(warmup):
        engine.step(dev_batches[i % len(dev_batches)], mask_all_valid=True)
    torch.cuda.synchronize()
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    torch.cuda.synchronize()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(steps):
        engine.step(dev_batches[i % len(dev_batches)], mask_all_valid=True)
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()  # device-timed loop only (its polls would slow the synchronising loop below)
    ms = ev0.elapsed_time(ev1) / steps
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    loss = None
    for i in range(steps):
        out = engine.step(host_batches[i % len(host_batches)], mask_all_valid=True)
        loss = float(out.loss.item())
    engine.finish()
    torch.cuda.synchronize()
    barrier()
    e2e = (time.perf_counter() - t0) * 1e3 / steps
    return ms, e2e, clocks, loss


# =========================================================================== cpu_smoke
CPU_SMOKE_BATCH, CPU_SMOKE_SEQ, CPU_SMOKE_DECODE = 4, 32, 8


def _retrieval_batches(n):
    """Synthetic key -> value retrieval sequences of the cpu_smoke data profile, seed 0."""
    from ..data.synthetic import SimpleWordTokenizer, SyntheticRetrievalConfig, SyntheticRetrievalDataset
    cfg = SyntheticRetrievalConfig(num_train_examples=n * CPU_SMOKE_BATCH, num_val_examples=1,
                                   block_size=CPU_SMOKE_SEQ, min_filler_tokens=4, max_filler_tokens=12,
                                   num_keys_per_example=2, vocab_filler_size=32, num_key_types=8, num_value_types=16,
                                   batch_size=CPU_SMOKE_BATCH, seed=0)
    tok = SimpleWordTokenizer()
    tok.build_vocab(cfg)
    ds = SyntheticRetrievalDataset(cfg, tok, "train")
    out = []
    for b in range(n):
        rows = [ds[b * CPU_SMOKE_BATCH + i] for i in range(CPU_SMOKE_BATCH)]
        out.append({k: torch.stack([r[k] for r in rows]) for k in rows[0]})
    return out


def run_cpu_smoke(args, impl):
    from ..config.profiles import profile_model_mapping
    torch.manual_seed(0)
    batches = _retrieval_batches(args.warmup + args.steps)
    mapping = profile_model_mapping("cpu_smoke")
    opt_kw = optimizer_settings(adamw_lr=1e-3, muon_lr=0.01)
    prompt = batches[0]["input_ids"]
    if impl == "ours":
        from ..config.model_yaml import build_model_config_from_mapping
        from ..infer import GenerationConfig, generate_tokens
        from ..models import KimiK3
        from ..train.engine import MoEController, TrainStepEngine
        from ..train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
        model = KimiK3(build_model_config_from_mapping(mapping))
        opt, _ = build_kimi_optimizer(model, KimiOptimizerConfig(**opt_kw))
        engine = TrainStepEngine(model, opt, grad_clip=1.0, amp_dtype=None, use_mtp=True,
                                 moe_controller=MoEController(model))
        for b in batches[:args.warmup]:
            engine.step(b)
        t0 = time.perf_counter()
        loss = None
        for b in batches[args.warmup:]:
            loss = float(engine.step(b).loss)
        step_ms = (time.perf_counter() - t0) * 1e3 / args.steps
        gen = generate_tokens(model, prompt, generation_config=GenerationConfig(
            max_new_tokens=CPU_SMOKE_DECODE, do_sample=False, device="cpu"))
    else:
        _reference_importable()
        from inference.config import GenerationConfig as RefGen
        from inference.generation import generate_tokens as ref_generate
        from src.kimi_k3.yaml_config import build_model_config_from_mapping as ref_build
        from src.kimi_k3_mini import KimiK3 as RefKimiK3
        from training.moe_control import MoEController as RefMoEController
        from training.optimizer import KimiOptimizerConfig as RefOptConfig
        from training.optimizer import build_kimi_optimizer as ref_build_optimizer
        from training.train_one_epoch import train_one_epoch as ref_train
        model = RefKimiK3(ref_build(mapping))
        opt, _ = ref_build_optimizer(model, RefOptConfig(**opt_kw))
        stamps = []
        ref_train(model, batches, opt, device=torch.device("cpu"), amp_enabled=False, grad_clip=1.0,
                  max_batches=len(batches), use_mtp=True, moe_controller=RefMoEController(model),
                  on_optimizer_step=lambda _m: stamps.append(time.perf_counter()))
        step_ms = (stamps[-1] - stamps[args.warmup - 1]) * 1e3 / args.steps
        loss = None
        gen = ref_generate(model, prompt, generation_config=RefGen(max_new_tokens=CPU_SMOKE_DECODE, do_sample=False,
                                                                   device="cpu"))
    tokens = CPU_SMOKE_BATCH * CPU_SMOKE_SEQ
    return {"metric": "train_tokens_per_s", "unit": "tokens/s", "value": round(tokens / (step_ms / 1e3), 1),
            "ms_per_step": round(step_ms, 3), "n_gpus": 0, "device": "cpu", "dtype": "fp32", "scaling": None,
            "higher_is_better": True, "last_loss": None if loss is None else round(loss, 4),
            "decode": {"generated_tokens": int(gen.generated_tokens), "prefill_ms": round(gen.prefill_seconds * 1e3, 3),
                       "decode_ms": round(gen.decode_seconds * 1e3, 3),
                       "tokens_per_s_per_sequence": round(gen.tokens_per_second, 2)},
            "data": "synthetic key-value retrieval sequences (seed 0), random-init weights",
            "config": {"model": "cpu_smoke", "global_batch": CPU_SMOKE_BATCH, "seq_len": CPU_SMOKE_SEQ,
                       "parallelism": "none", "timing": "host clock (CPU)"}}


# =========================================================================== gpu24_tp_ep
GPU24_SEQ, GPU24_GLOBAL_BATCH = 1024, 32


def run_gpu24_tp_ep(args, world, rank, local, impl):
    if world < 2 or world % 2:
        raise ValueError("gpu24_tp_ep runs TP2 x EP(N/2): N must be 2, 4 or 8")
    tp, ep = 2, world // 2
    replicas = ep
    per_replica = GPU24_GLOBAL_BATCH // replicas
    dev = torch.device("cuda", local)
    from ..config.profiles import profile_model_config, profile_model_mapping
    d = _dist_dict(world, tp=tp, ep=ep, ours=impl == "ours")
    note = None
    if impl == "ours":
        from ..models import KimiK3
        from ..parallel.config import distributed_config_from_dict
        from ..parallel.environment import setup_distributed
        from ..parallel.parallelize import parallelize_kimi_model
        from ..train.engine import MoEController, TrainStepEngine
        from ..train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
        dcfg = distributed_config_from_dict(d)
        ctx = setup_distributed(dcfg)
        torch.manual_seed(1337)
        with torch.device(dev):
            model = KimiK3(profile_model_config("gpu_24gb"))
        plan = parallelize_kimi_model(model, dcfg, ctx)
        plan.broadcast_parameters()
        opt, _ = build_kimi_optimizer(model, KimiOptimizerConfig(**optimizer_settings()))
        engine = TrainStepEngine(model, opt, grad_clip=1.0, amp_dtype=torch.bfloat16, use_mtp=True,
                                 moe_controller=MoEController(model, reducer=plan.qb_reducer()),
                                 grad_hook=plan.sync_gradients, grad_norm_fn=plan.grad_norm)
        vocab = model.config.vocab_size
        replica = ctx.ep_rank
        dev_b = _token_batches(2, per_replica, GPU24_SEQ, vocab, 1000 + replica, dev)
        host_b = [{k: v.pin_memory() for k, v in b.items()}
                  for b in _token_batches(2, per_replica, GPU24_SEQ, vocab, 2000 + replica)]
        ms, e2e, clocks, loss = _time_engine(engine, dev_b, host_b, args.warmup, args.steps, local)
    else:
        _reference_importable()
        from src.kimi_k3.yaml_config import build_model_config_from_mapping as ref_build
        from src.kimi_k3_mini import KimiK3 as RefKimiK3
        from training.distributed.config import distributed_config_from_dict as ref_dist
        from training.distributed.environment import initialize_distributed
        from training.distributed.mesh import build_device_mesh
        from training.distributed.parallelize import parallelize_kimi_model as ref_parallelize
        from training.distributed.wrapping import broadcast_model_state, wrap_data_parallel
        from training.moe_control import MoEController as RefMoEController
        from training.optimizer import KimiOptimizerConfig as RefOptConfig
        from training.optimizer import build_kimi_optimizer as ref_build_optimizer
        from training.train_one_epoch import train_one_epoch as ref_train
        dcfg = ref_dist(d)
        ctx = build_device_mesh(initialize_distributed(dcfg), dcfg)
        torch.manual_seed(1337)
        with torch.device(dev):
            model = RefKimiK3(ref_build(profile_model_mapping("gpu_24gb")))
        broadcast_model_state(model, ctx)
        ref_parallelize(model, dcfg, ctx)
        model.to(dev)
        model = wrap_data_parallel(model, dcfg, ctx, training_precision="bf16")
        raw = model.module if hasattr(model, "module") else model
        opt, _ = ref_build_optimizer(raw, RefOptConfig(**optimizer_settings()))
        vocab = raw.config.vocab_size

        def make(n, micro):
            return _token_batches(n, per_replica // micro, GPU24_SEQ, vocab, 1000 + ctx.ep_rank)
        ms, e2e, clocks, note = _reference_train(ref_train, model, opt, make, args, local, device=dev, grad_clip=1.0,
                                                 use_mtp=True, moe_controller=RefMoEController(model),
                                                 distributed_context=ctx)
        loss = None
    ms, e2e = max_over_ranks(ms), max_over_ranks(e2e)
    tokens = GPU24_GLOBAL_BATCH * GPU24_SEQ
    h2d = per_replica * GPU24_SEQ * (8 + 8 + 1)
    line = {"metric": "train_tokens_per_s", "unit": "tokens/s", "value": round(tokens / (ms / 1e3), 1),
            "ms_per_step": round(ms, 3), "n_gpus": world, "dtype": "fp32" if note and "fp32" in note else "bf16",
            "scaling": "strong", "higher_is_better": True, "clocks": clocks,
            "e2e": {"value": round(tokens / (e2e / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(e2e, 3),
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4},
            "data": "synthetic uniform token ids (seeded per data replica), random-init weights",
            "config": {"model": "gpu_24gb-shaped Kimi K3 (MTP on)", "global_batch": GPU24_GLOBAL_BATCH,
                       "seq_len": GPU24_SEQ, "parallelism": f"tp{tp}xep{ep}",
                       "l2": "per-step working set >> 126 MB L2"}}
    if loss is not None:
        line["last_loss"] = round(loss, 4)
    if note:
        line["note"] = note
    _close(ctx)
    return line


# =========================================================================== gpu48_fsdp
GPU48_STAGES = ((2048, 8), (8192, 2))  # (sequence length, sequences per GPU): 16,384 tokens per GPU


def run_gpu48_fsdp(args, world, rank, local, impl):
    dev = torch.device("cuda", local)
    from ..config.profiles import profile_model_config, profile_model_mapping
    d = _dist_dict(world, dp_mode="fsdp" if world > 1 else "none")
    stage_ms, stage_e2e, clocks_all, note, loss = [], [], [], None, None
    if impl == "ours":
        from ..models import KimiK3
        from ..parallel.config import distributed_config_from_dict
        from ..parallel.data_parallel import QBReducer
        from ..parallel.environment import setup_distributed
        from ..parallel.fsdp import shard_kimi_model, sharded_grad_norm
        from ..train.engine import MoEController, TrainStepEngine
        from ..train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
        dcfg = distributed_config_from_dict(d)
        ctx = setup_distributed(dcfg)
        torch.manual_seed(1337)
        with torch.device(dev):
            model = KimiK3(profile_model_config("gpu_48gb"))
        if world > 1:
            import torch.distributed as dist
            for p in model.parameters():
                dist.broadcast(p.data, src=0)
            shard_kimi_model(model, dcfg, ctx)
        opt, _ = build_kimi_optimizer(model, KimiOptimizerConfig(**optimizer_settings()))
        params = [p for p in model.parameters() if p.requires_grad]
        if world > 1 and getattr(opt, "qk_clip", None) is not None:
            opt.qk_clip.replica_group = ctx.dp_group
        vocab = model.config.vocab_size
        for si, (seq, bpg) in enumerate(GPU48_STAGES):
            # one engine per context stage; a single GPU captures each stage's step in a CUDA graph
            engine = TrainStepEngine(model, opt, grad_clip=1.0, amp_dtype=torch.bfloat16, use_mtp=True,
                                     moe_controller=MoEController(model, reducer=QBReducer(ctx.dp_group)
                                                                  if world > 1 else None),
                                     grad_norm_fn=(lambda: sharded_grad_norm(params)) if world > 1 else None,
                                     cuda_graph=world == 1 and not args.no_graph)
            dev_b = _token_batches(2, bpg, seq, vocab, 1000 + 10 * rank + si, dev)
            host_b = [{k: v.pin_memory() for k, v in b.items()}
                      for b in _token_batches(2, bpg, seq, vocab, 2000 + 10 * rank + si)]
            ms, e2e, clocks, loss = _time_engine(engine, dev_b, host_b, args.warmup, args.steps, local)
            engine.release_graph()
            del engine
            stage_ms.append(max_over_ranks(ms))
            stage_e2e.append(max_over_ranks(e2e))
            clocks_all.append(clocks)
    else:
        _reference_importable()
        from src.kimi_k3.yaml_config import build_model_config_from_mapping as ref_build
        from src.kimi_k3_mini import KimiK3 as RefKimiK3
        from training.distributed.config import distributed_config_from_dict as ref_dist
        from training.distributed.environment import initialize_distributed
        from training.distributed.mesh import build_device_mesh
        from training.distributed.wrapping import broadcast_model_state, wrap_data_parallel
        from training.moe_control import MoEController as RefMoEController
        from training.optimizer import KimiOptimizerConfig as RefOptConfig
        from training.optimizer import build_kimi_optimizer as ref_build_optimizer
        from training.train_one_epoch import train_one_epoch as ref_train
        dcfg = ref_dist(d)
        ctx = build_device_mesh(initialize_distributed(dcfg), dcfg)
        torch.manual_seed(1337)
        with torch.device(dev):
            model = RefKimiK3(ref_build(profile_model_mapping("gpu_48gb")))
        if world > 1:
            broadcast_model_state(model, ctx)
            model = wrap_data_parallel(model, dcfg, ctx, training_precision="bf16")
        raw = model.module if hasattr(model, "module") else model
        try:
            opt, _ = ref_build_optimizer(model, RefOptConfig(**optimizer_settings()))
        except ValueError as exc:
            # FSDP hands the reference's Muon flattened parameter shards, which it rejects
            note = f"reference Muon rejects FSDP parameter shards ({exc}); measured with AdamW only"
            opt, _ = ref_build_optimizer(model, RefOptConfig(**optimizer_settings(kind="adamw")))
        vocab = raw.config.vocab_size
        for si, (seq, bpg) in enumerate(GPU48_STAGES):
            def make(n, micro, seq=seq, bpg=bpg, si=si):
                return _token_batches(n, max(bpg // micro, 1), seq, vocab, 1000 + 10 * rank + si)
            ms, e2e, clocks, stage_note = _reference_train(ref_train, model, opt, make, args, local, device=dev,
                                                           grad_clip=1.0, use_mtp=True,
                                                           moe_controller=RefMoEController(model),
                                                           distributed_context=ctx)
            if stage_note:
                note = "; ".join(x for x in (note, f"stage {seq}: {stage_note}") if x)
            stage_ms.append(max_over_ranks(ms))
            stage_e2e.append(max_over_ranks(e2e))
            clocks_all.append(clocks)
    tokens = [seq * bpg * world for seq, bpg in GPU48_STAGES]
    total_ms, total_e2e = sum(stage_ms), sum(stage_e2e)
    value = sum(tokens) / (total_ms / 1e3)
    line = {"metric": "train_tokens_per_s", "unit": "tokens/s", "value": round(value, 1),
            "ms_per_step": round(total_ms / len(stage_ms), 3), "n_gpus": world,
            "dtype": "fp32" if note and "fp32" in note else "bf16", "scaling": "weak", "higher_is_better": True,
            "clocks": clocks_all[-1],
            "stages": [{"seq_len": seq, "seqs_per_gpu": bpg, "ms_per_step": round(ms, 3),
                        "tokens_per_s": round(t / (ms / 1e3), 1)}
                       for (seq, bpg), ms, t in zip(GPU48_STAGES, stage_ms, tokens)],
            "e2e": {"value": round(sum(tokens) / (total_e2e / 1e3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": 16384 * 17, "d2h_bytes_per_step": 4},
            "data": "synthetic uniform token ids (seeded per rank), random-init weights",
            "config": {"model": "gpu_48gb-shaped Kimi K3 text stack (MTP on)", "tokens_per_gpu_step": 16384,
                       "seq_len": "2048 then 8192 (progressive context)",
                       "parallelism": f"fsdp{world}" if world > 1 else "single GPU",
                       "l2": "per-step working set >> 126 MB L2"}}
    if loss is not None:
        line["last_loss"] = round(loss, 4)
    if note:
        line["note"] = note
    _close(ctx)
    return line


# =========================================================================== gpu80_infer
GPU80_PROMPTS, GPU80_PROMPT_LEN = 64, 4096


def run_gpu80_infer(args, world, rank, local, impl):
    dev = torch.device("cuda", local)
    decode_steps = args.decode_steps
    repeats = max(1, args.steps)
    from ..config.profiles import profile_model_config, profile_model_mapping
    g = torch.Generator().manual_seed(4242)
    vocab = profile_model_mapping("gpu_80gb")["model"]["vocab_size"]
    prompts = torch.randint(3, vocab, (GPU80_PROMPTS, GPU80_PROMPT_LEN), generator=g)
    prompts_pinned = prompts.pin_memory()
    note = None
    if impl == "ours":
        from ..infer import GenerationConfig, GraphDecoder
        from ..infer.distributed import graph_capturable, prepare_distributed_model
        from ..models import KimiK3
        from ..parallel.config import distributed_config_from_dict
        from ..parallel.environment import setup_distributed
        d = _dist_dict(world, tp=world, ep=world, overlay=True, ours=True)
        dcfg = distributed_config_from_dict(d)
        ctx = setup_distributed(dcfg)
        torch.manual_seed(1337)
        with torch.device(dev):
            model = KimiK3(profile_model_config("gpu_80gb"))
        model = prepare_distributed_model(model, dcfg, ctx).requires_grad_(False).eval()
        parallelism = f"tp{world}+ep{world} (same ranks)" if world > 1 else "single GPU"

        # one serving decoder: the decode step is captured on the first generation (the warm-up)
        # and replayed by every later one with the same batch shape
        decoder = GraphDecoder(model, max_length=GPU80_PROMPT_LEN + decode_steps,
                               generation_config=GenerationConfig(do_sample=False, device=str(dev)),
                               use_graph=graph_capturable(model), copy_model=False)

        def generate(steps):
            decoder.cfg = GenerationConfig(max_new_tokens=steps, do_sample=False, device=str(dev), eos_token_id=None,
                                           return_cache=False)
            ids = prompts_pinned.to(dev, non_blocking=True)
            out = decoder.generate(ids)
            return out, out.generated_ids.cpu()  # device -> host read of the result
    else:
        _reference_importable()
        from inference.config import GenerationConfig as RefGen
        from inference.generation import generate_tokens as ref_generate
        from src.kimi_k3.yaml_config import build_model_config_from_mapping as ref_build
        from src.kimi_k3_mini import KimiK3 as RefKimiK3
        from training.distributed.config import distributed_config_from_dict as ref_dist
        from training.distributed.environment import initialize_distributed
        from training.distributed.mesh import build_device_mesh
        from training.distributed.parallelize import parallelize_kimi_model as ref_parallelize
        d = _dist_dict(world, tp=world)
        dcfg = ref_dist(d)
        ctx = build_device_mesh(initialize_distributed(dcfg), dcfg)
        torch.manual_seed(1337)
        with torch.device(dev):
            model = RefKimiK3(ref_build(profile_model_mapping("gpu_80gb")))
        if world > 1:
            ref_parallelize(model, dcfg, ctx)
        model.to(dev).eval()
        parallelism = f"tp{world}" if world > 1 else "single GPU"
        state = {"model": model.to(torch.bfloat16)}

        def generate(steps):
            cfg = RefGen(max_new_tokens=steps, do_sample=False, device=str(dev), return_cache=False)
            with torch.inference_mode():
                out = ref_generate(state["model"], prompts_pinned.to(dev, non_blocking=True), generation_config=cfg)
            return out, out.generated_ids.cpu()

        try:
            generate(2)
        except RuntimeError as exc:
            # this profile keeps the MLA attention output in fp32 (keep_attention_output_fp32), which
            # the bf16 output projection rejects: the reference serves it in fp32
            if "dtype" not in str(exc):
                raise
            note = f"reference bf16 weights fail ({str(exc)[:120]}); measured in fp32"
            state["model"] = state["model"].float()
            torch.cuda.empty_cache()

    # warm-up: one short generation (kernels' one-time set-up, workspaces, allocator)
    generate(4)
    torch.cuda.synchronize()
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    ttft, decode_s, generated = [], [], 0
    for _ in range(repeats):
        torch.cuda.synchronize()
        barrier()
        out, toks = generate(decode_steps)
        ttft.append(max_over_ranks(out.prefill_seconds))
        decode_s.append(max_over_ranks(out.decode_seconds))
        generated = int(toks.shape[1])
    clocks = sampler.stop()
    if impl == "ours":
        from ..parallel.expert_parallel import release_shared_workspaces
        decoder.release()  # the captured step holds NCCL calls: drop it before the process group
        release_shared_workspaces()
    dec = statistics.median(decode_s)
    batch_tps = GPU80_PROMPTS * generated / dec if dec > 0 else 0.0
    line = {"metric": "decode_tokens_per_s", "unit": "tokens/s", "value": round(batch_tps, 1),
            "ms_per_step": round(dec * 1e3 / max(generated, 1), 3), "n_gpus": world,
            "dtype": "bf16" if note is None else "fp32",
            "scaling": "strong", "higher_is_better": True, "clocks": clocks,
            "ttft_p50_ms": round(statistics.median(ttft) * 1e3, 2),
            "decode_tokens_per_s_per_sequence": round(generated / dec if dec > 0 else 0.0, 2),
            "generated_tokens": generated, "repeats": repeats,
            "e2e": {"value": round(GPU80_PROMPTS * generated / (dec + statistics.median(ttft)), 1),
                    "unit": "tokens/s (prefill + decode)", "h2d_bytes_per_step": int(prompts.numel() * 8),
                    "d2h_bytes_per_step": GPU80_PROMPTS * generated * 8},
            "data": "synthetic uniform prompt ids (seed 4242), random-init weights",
            "config": {"model": "gpu_80gb-shaped Kimi K3 text stack", "prompts": GPU80_PROMPTS,
                       "prompt_len": GPU80_PROMPT_LEN, "decode_steps": decode_steps, "parallelism": parallelism,
                       "timing": "generation API clocks (synchronised), max over ranks"}}
    if note:
        line["note"] = note
    _close(ctx)
    return line


def _close(ctx) -> None:
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        barrier()
        dist.destroy_process_group()


def run_config(args, world, rank, local):
    """Run ``args.config`` for ``args.impl``; returns the JSON line (every rank)."""
    if args.config == "cpu_smoke":
        line = run_cpu_smoke(args, args.impl)
    else:
        if not torch.cuda.is_available():
            raise RuntimeError("no CUDA device")
        torch.cuda.set_device(local)
        fn = {"gpu24_tp_ep": run_gpu24_tp_ep, "gpu48_fsdp": run_gpu48_fsdp, "gpu80_infer": run_gpu80_infer}[args.config]
        line = fn(args, world, rank, local, args.impl)
    line.update({"steps": args.steps, "warmup": args.warmup, "vs_baseline": None, "bench_config": args.config})
    if args.impl == "reference":
        line["impl"] = "reference"
    return line


__all__ = ["CONFIGS", "run_config", "optimizer_settings"]
