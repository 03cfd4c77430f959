"""Tensor- and expert-parallel inference.

Parity: ``scripts/infer_kimi.py:98-141`` (reference): the ``distributed:`` section of an
inference YAML (TP / EP only; ``inference/yaml_config.py:34-40`` rejects DDP / FSDP) is applied
by initialising the process group, building the rank mesh, loading the checkpoint on this
rank's device and sharding the model in place with the training plan, then every rank runs the
same generation; rank 0 reports.

What each rank holds after :func:`prepare_distributed_model`:

* tensor parallelism: whole KDA heads (recurrent state ``[B, H/TP, K, V]`` and conv history per
  rank) and whole MLA heads over a replicated latent cache (the latent compression is
  replicated, so every rank appends the same latent row: ``mla_cache_layout: replicated``);
  the vocabulary-sharded LM head gathers the logits, so sampling sees the full distribution
  and, driven by the same seed and counter, picks the same token on every rank;
* expert parallelism: a block of routed experts; the (token, slot) rows go to their owners and
  back inside each MoE layer (NCCL all-to-alls, or the device-initiated NVLink exchange when
  ``expert_parallel.dispatch: nvlink_fused``).  With ``overlay_tensor_parallel`` the EP group is
  the TP group and each rank routes its block of the shared tokens.

:class:`~kimi_k3_b200.infer.graph_decode.GraphDecoder` captures the sharded decode step in a
CUDA graph like the single-GPU one.  The NCCL all-to-all needs split sizes on the host and
cannot be captured, so captured decode steps with EP use the ``nvlink_fused`` exchange;
:func:`graph_capturable` reports whether a sharded model can be captured.
"""
from __future__ import annotations

from dataclasses import replace

import torch
import torch.nn as nn


def prepare_distributed_model(model: nn.Module, config, context) -> nn.Module:
    """Shard ``model`` in place for inference over ``context`` (no-op when distributed is off)."""
    if not config.enabled:
        return model
    if config.data_parallel.mode != "none":
        raise ValueError("distributed inference does not use DDP/FSDP")
    from ..parallel.parallelize import parallelize_kimi_model
    raw = model.module if hasattr(model, "module") else model
    parallelize_kimi_model(raw, config, context)
    raw.requires_grad_(False).eval()
    return raw


def graph_capturable(model: nn.Module) -> bool:
    """False when an expert-parallel MoE of ``model`` exchanges rows with host-sized all-to-alls."""
    from ..parallel.expert_parallel import ExpertParallelMoE
    from ..parallel.tensor_parallel import group_size
    for m in model.modules():
        if isinstance(m, ExpertParallelMoE) and group_size(m.group) > 1 and not m.device_exchange:
            return False
    return True


def run_distributed_generation(model_config_path, checkpoint_path, prompt, inference_yaml, *, tokenizer=None,
                               precision: str = "model", use_graph: bool = False, max_length: int | None = None):
    """Initialise the mesh from ``inference_yaml.distributed``, load, shard, generate.

    Returns ``(output, context)``; the caller reports on ``context.is_global_zero`` and closes
    the context."""
    from ..parallel.environment import setup_distributed
    from .config import ModelLoadConfig
    from .generation import inference_autoregressive
    from .session import encode_prompt, load_kimi_checkpoint
    dist_cfg = inference_yaml.distributed
    context = setup_distributed(dist_cfg)
    gen = inference_yaml.generation
    device = str(context.device) if dist_cfg.enabled else gen.device
    loaded = load_kimi_checkpoint(model_config_path, checkpoint_path, tokenizer=tokenizer,
                                  load_config=ModelLoadConfig(device=device, precision=precision))
    model = prepare_distributed_model(loaded.model, dist_cfg, context)
    gen = replace(gen, device=str(next(model.parameters()).device))
    if use_graph and torch.device(gen.device).type == "cuda":
        from .graph_decode import GraphDecoder
        ids = encode_prompt(prompt, tokenizer=tokenizer, add_bos_token=gen.add_bos_token)
        ml = max_length or int(ids.shape[1]) + gen.max_new_tokens
        dec = GraphDecoder(model, max_length=ml, generation_config=gen, use_graph=graph_capturable(model))
        out = dec.generate(ids)
        dec.release()
    else:
        out = inference_autoregressive(model, prompt, tokenizer=tokenizer, generation_config=gen)
    return out, context


__all__ = ["prepare_distributed_model", "graph_capturable", "run_distributed_generation"]
