"""Built-in model profiles (the shapes named by the benchmark configurations).

Each entry is a model-YAML mapping in the reference schema (``model: {...}``) so the
same strict builder handles files and built-ins; ``write_profile`` emits it as a
``model.yaml``.  Shapes follow the reference's ``config/kimi_full_pipeline/<profile>``
model files (dimensions listed per profile below).
"""
from __future__ import annotations

import copy
from pathlib import Path

import yaml


def _text_model(name, vocab, d, heads, groups, latent, n_shared, n_routed, top_k, shared_h, routed_h,
                ar_backend="two_phase", mtp_backend="eager", special=True):
    m = {"name": name, "architecture": "kimi_k3", "vocab_size": vocab, "d_model": d, "num_heads": heads,
         "num_hybrid_groups": groups, "attention_pattern": ["kda", "kda", "kda", "gated_mla"],
         "add_final_gated_mla": True, "tie_word_embeddings": True, "initializer_range": 0.02,
         "kda": {"key_head_dim": 64, "short_conv_kernel_size": 4, "chunk_size": 64, "secondary_tile_size": 16,
                 "accumulate_state_in_fp32": True},
         "mla": {"q_head_dim": 64, "kv_latent_dim": d, "attention_backend": "auto"},
         "moe": {"latent_dim": latent, "num_shared_experts": n_shared, "num_routed_experts": n_routed,
                 "routed_experts_per_token": top_k, "shared_expert_hidden_dim": shared_h,
                 "routed_expert_hidden_dim": routed_h, "routing_backend": "vectorized",
                 "quantile_backend": "histogram", "enable_quantile_balancing": True},
         "attention_residual": {"mode": "block", "sublayers_per_depth_block": 8, "backend": ar_backend},
         "vision": {"enabled": False},
         "mtp": {"enabled": True, "loss_weight": 0.1,
                 "attention_residual": {"mode": "block", "sublayers_per_depth_block": 8, "backend": mtp_backend}}}
    if special:
        m.update({"pad_token_id": 0, "bos_token_id": 1, "eos_token_id": 2})
    return {"model": m}


MODEL_PROFILES = {
    # d 640, 10 heads, 3 groups (9 KDA + 4 MLA), MoE latent 320, 12 experts top-2, MTP  (~212.9M params at V=16000)
    "t4_wikitext": _text_model("kimi_k3_t4_wikitext_213m", 16000, 640, 10, 3, 320, 1, 12, 2, 960, 640),
    # d 768, 12 heads, 3 groups, latent 384, 16 experts top-4
    "gpu_24gb": _text_model("kimi_k3_24gb_text", 32000, 768, 12, 3, 384, 1, 16, 4, 1024, 768),
    # d 1024, 16 heads, 4 groups, latent 512, 32 experts top-4, 2 shared (text stack of the multimodal profile)
    "gpu_48gb": _text_model("kimi_k3_48gb_text", 64000, 1024, 16, 4, 512, 2, 32, 4, 1536, 1024),
    # d 1536, 24 heads, 6 groups, latent 768, 64 experts top-8, 2 shared (text stack)
    "gpu_80gb": _text_model("kimi_k3_gpu_80gb_text", 64000, 1536, 24, 6, 768, 2, 64, 8, 2048, 1536,
                            mtp_backend="two_phase"),
}

CPU_SMOKE = {"model": {
    "name": "kimi_k3_cpu_tiny", "architecture": "kimi_k3", "vocab_size": 128, "d_model": 16, "num_heads": 2,
    "num_hybrid_groups": 1, "attention_pattern": ["kda", "kda", "kda", "gated_mla"], "add_final_gated_mla": True,
    "pad_token_id": 0, "bos_token_id": 1, "eos_token_id": 2, "image_token_id": 3, "video_token_id": 4,
    "tie_word_embeddings": True,
    "kda": {"key_head_dim": 4, "short_conv_kernel_size": 4, "chunk_size": 64, "secondary_tile_size": 16},
    "mla": {"q_head_dim": 4, "kv_latent_dim": 8, "attention_backend": "auto"},
    "moe": {"latent_dim": 8, "num_shared_experts": 1, "num_routed_experts": 4, "routed_experts_per_token": 2,
            "shared_expert_hidden_dim": 20, "routed_expert_hidden_dim": 16},
    "attention_residual": {"mode": "block", "sublayers_per_depth_block": 4, "backend": "eager"},
    "vision": {"enabled": True, "type": "moonvit", "image_size": 16, "patch_size": 4, "embed_dim": 16, "depth": 2,
               "num_heads": 4, "use_cls_token": False, "use_pixel_shuffle": True, "projector": {"hidden_dim": 32}},
    "mtp": {"enabled": True, "loss_weight": 0.1,
            "attention_residual": {"mode": "block", "sublayers_per_depth_block": 4, "backend": "eager"}}}}
MODEL_PROFILES["cpu_smoke"] = CPU_SMOKE


def profile_model_mapping(name: str) -> dict:
    if name not in MODEL_PROFILES:
        raise KeyError(f"unknown model profile {name!r}; known: {sorted(MODEL_PROFILES)}")
    return copy.deepcopy(MODEL_PROFILES[name])


def profile_model_config(name: str, *, vocab_size: int | None = None):
    from .model_yaml import build_model_config_from_mapping
    return build_model_config_from_mapping(profile_model_mapping(name), vocab_size_override=vocab_size)


def write_profile(name: str, directory: str | Path) -> Path:
    path = Path(directory) / "model.yaml"
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(yaml.safe_dump(profile_model_mapping(name), sort_keys=False))
    return path


__all__ = ["MODEL_PROFILES", "profile_model_mapping", "profile_model_config", "write_profile"]


# --------------------------------------------------------------------------- full pipelines
# B200 recipes: bf16 autocast, large micro-batches (HBM3e holds them), no gradient
# accumulation unless the global batch asks for it, native kernels on.
def _training(run, *, max_seq_len, epochs=1, accum=1, precision="bf16", muon_lr=0.02, adamw_lr=3e-4, curriculum=None,
              distributed=None, use_mtp=True, diagnostics_light=True):
    t = {"runtime": {"device": "auto", "total_steps": None, "verbose": True, "use_ema": False, "ema_decay": 0.999,
                     "eval_use_ema": False},
         "training": {"epochs": epochs, "gradient_accumulation_steps": accum, "precision": precision,
                      "grad_clip_norm": 1.0, "use_mtp": use_mtp, "max_batches_per_epoch": None,
                      "max_eval_batches": 64, "log_every_steps": 10, "eval_every_epochs": 1,
                      "checkpoint_every_epochs": 1, "prediction_every_epochs": 1, "seed": 1337,
                      "deterministic": False, "max_seq_len": max_seq_len},
         "loss": {"ignore_index": -100, "label_smoothing": 0.0, "mtp_loss_weight": 0.1},
         "optimizer": {"kind": "per_head_muon_adamw", "adamw_lr": adamw_lr, "adamw_betas": [0.9, 0.95],
                       "adamw_eps": 1.0e-8, "muon_lr": muon_lr, "muon_momentum": 0.95, "muon_nesterov": True,
                       "muon_ns_steps": 5, "muon_ns_eps": 1.0e-7, "muon_update_rms_scaling": True,
                       "weight_decay": 0.1, "per_head_qkv": True, "qk_clip_enabled": True,
                       "qk_clip_threshold": 100.0, "qk_clip_every_steps": 1},
         "scheduler": {"kind": "cosine", "warmup_ratio": 0.01, "warmup_steps": None, "min_lr_ratio": 0.1},
         "diagnostics": {"enabled": True, "cheap_every_steps": 1, "standard_every_steps": 50 if diagnostics_light else 10,
                         "deep_every_steps": 1000, "sample_layers_per_standard_step": 2 if diagnostics_light else 8,
                         "sample_tokens_per_layer": 64, "sample_parameters_per_group": 4,
                         "sample_elements_per_parameter": 64, "max_diagnostic_time_fraction": 0.03,
                         "max_persistent_gpu_bytes": 4194304, "alert_patience_steps": 5},
         "context_curriculum": curriculum or {"enabled": False},
         "checkpoint": {"output_dir": f"checkpoints/{run}", "run_name": f"kimi_k3_{run}", "keep_last_n": 3,
                        "save_optimizer": True, "save_rng_state": True, "atomic_write": True, "resume_from": None},
         "prediction": {"sample_index": 0, "max_tokens": 32},
         "kernels": {"native_kernels": True, "fused_head_loss": True, "muon_ns_dtype": "auto"}}
    if distributed:
        t["distributed"] = distributed
    return t


def _data_text(name, block, batch, preset="wikitext2", vocab=16000):
    return {"data": {"name": name, "kind": "hf_text",
                     "dataset": {"preset_name": preset, "block_size": block,
                                 "tokenizer_path": f"data/cache/tokenizers/{preset}_{vocab}.json", "vocab_size": vocab,
                                 "min_frequency": 2, "max_tokenizer_documents": None, "max_train_documents": None,
                                 "max_validation_documents": None, "streaming": False},
                     "loader": {"batch_size": batch, "validation_batch_size": batch, "num_workers": 2,
                                "shuffle_train": True, "pin_memory": "auto", "persistent_workers": True,
                                "prefetch_factor": 2, "drop_last": False, "seed": 42}}}


def _data_synthetic(name, block, batch, n_train=50_000, n_val=2_000, **kw):
    ds = {"num_train_examples": n_train, "num_val_examples": n_val, "block_size": block, "min_filler_tokens": 64,
          "max_filler_tokens": max(64, block - 64), "num_keys_per_example": 8, "vocab_filler_size": 550,
          "num_key_types": 128, "num_value_types": 256, "seed": 42}
    ds.update(kw)
    return {"data": {"name": name, "kind": "synthetic_retrieval", "dataset": ds,
                     "loader": {"batch_size": batch, "num_workers": 0, "shuffle_train": True, "pin_memory": "auto",
                                "persistent_workers": False, "drop_last": False, "seed": 42}}}


def _dist(dp=1, tp=1, ep=1, mode=None, overlay=False):
    return {"enabled": dp * tp * (1 if overlay else ep) > 1, "backend": "auto", "init_method": "env",
            "timeout_seconds": 1800,
            "data_parallel": {"mode": mode or ("ddp" if dp > 1 else "none"), "size": dp},
            "tensor_parallel": {"enabled": tp > 1, "size": tp, "shard_embeddings": True, "shard_lm_head": True,
                                "sequence_parallel_norms": False, "shard_kda_heads": True, "shard_mla_heads": True,
                                "shard_moe_latent_projections": False, "mla_cache_layout": "replicated"},
            "expert_parallel": {"enabled": ep > 1, "size": ep, "dispatch": "all_to_all",
                                "expert_placement": "contiguous", "shared_experts": "replicated", "drop_tokens": False,
                                "capacity_factor": None, "overlay_tensor_parallel": overlay},
            "pipeline_parallel": {"enabled": False, "size": 1}, "context_parallel": {"enabled": False, "size": 1},
            "checkpoint": {"format": "distributed", "async_save": False, "save_rng_per_rank": True},
            "diagnostics": {"aggregate_across_data_parallel": True, "log_rank": 0, "per_rank_debug": False}}


INFERENCE_GREEDY = {"inference": {"max_new_tokens": 128, "do_sample": False, "temperature": 1.0, "top_k": None,
                                  "top_p": None, "repetition_penalty": None, "eos_token_id": None,
                                  "pad_token_id": None, "add_bos_token": True, "skip_special_tokens": True,
                                  "seed": 1337, "device": "auto", "return_scores": False, "return_cache": True,
                                  "max_total_tokens": None},
                    "distributed": {"enabled": False}}
_PCC = {"enabled": True, "stages": [{"max_seq_len": 2048, "until_tokens": 200_000_000},
                                    {"max_seq_len": 4096, "until_tokens": 400_000_000},
                                    {"max_seq_len": 8192, "until_tokens": None}],
        "transition_unit": "tokens", "reset_dataloader_on_transition": True, "preserve_optimizer_state": True,
        "preserve_scheduler_state": True}

PIPELINES = {
    "cpu_smoke": ("cpu_smoke", _training("cpu_smoke", max_seq_len=32, precision="fp32", muon_lr=0.01,
                                         diagnostics_light=False),
                  {"data": {"name": "synthetic_cpu_smoke", "kind": "synthetic_retrieval",
                            "dataset": {"num_train_examples": 32, "num_val_examples": 8, "block_size": 32,
                                        "min_filler_tokens": 4, "max_filler_tokens": 12, "num_keys_per_example": 2,
                                        "vocab_filler_size": 32, "num_key_types": 8, "num_value_types": 16,
                                        "seed": 7},
                            "loader": {"batch_size": 4, "num_workers": 0, "shuffle_train": True, "pin_memory": False,
                                       "persistent_workers": False, "drop_last": False, "seed": 7}}}),
    "t4_wikitext": ("t4_wikitext", _training("t4_wikitext_213m", max_seq_len=1024, epochs=3),
                    _data_text("wikitext2_1024", 1024, 16)),
    "t4_retrieval": ("t4_wikitext", _training("t4_retrieval", max_seq_len=1024),
                     _data_synthetic("synthetic_retrieval_1024", 1024, 16)),
    "gpu_24gb": ("gpu_24gb", _training("gpu_24gb", max_seq_len=2048), _data_text("fineweb_edu_2048", 2048, 16,
                                                                                 "fineweb_edu_10bt_mincols", 32000)),
    "gpu_48gb": ("gpu_48gb", _training("gpu_48gb", max_seq_len=8192, curriculum=_PCC),
                 _data_text("fineweb_10bt_8192", 8192, 4, "fineweb_10bt", 64000)),
    "gpu_80gb": ("gpu_80gb", _training("gpu_80gb", max_seq_len=4096), _data_text("fineweb_4096", 4096, 8,
                                                                                 "fineweb_100bt", 64000)),
    "distributed_ddp_2x": ("t4_wikitext", _training("ddp_2x", max_seq_len=1024, distributed=_dist(dp=2)),
                           _data_text("wikitext2_1024", 1024, 16)),
    "distributed_fsdp_8x_48gb": ("gpu_48gb", _training("fsdp_8x_48gb", max_seq_len=8192, curriculum=_PCC,
                                                       distributed=_dist(dp=8, mode="fsdp")),
                                 _data_text("fineweb_10bt_8192", 8192, 4, "fineweb_10bt", 64000)),
    "distributed_tp_2x_24gb": ("gpu_24gb", _training("tp_2x_24gb", max_seq_len=2048, distributed=_dist(tp=2)),
                               _data_text("fineweb_edu_2048", 2048, 16, "fineweb_edu_10bt_mincols", 32000)),
    "distributed_tp_ep_4x_24gb": ("gpu_24gb", _training("tp_ep_4x_24gb", max_seq_len=2048,
                                                        distributed=_dist(tp=2, ep=2)),
                                  _data_text("fineweb_edu_2048", 2048, 16, "fineweb_edu_10bt_mincols", 32000)),
    "distributed_ep8_tp8_80gb": ("gpu_80gb", _training("ep8_tp8_80gb", max_seq_len=4096,
                                                       distributed=_dist(tp=8, ep=8, overlay=True)),
                                 _data_text("fineweb_4096", 4096, 8, "fineweb_100bt", 64000)),
}


def write_pipeline(name: str, directory) -> Path:
    """Write ``model.yaml``, ``training.yaml``, ``data.yaml`` and ``inference.yaml`` of a pipeline."""
    if name not in PIPELINES:
        raise KeyError(f"unknown pipeline profile {name!r}; known: {sorted(PIPELINES)}")
    model_name, training, data = PIPELINES[name]
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    model = profile_model_mapping(model_name)
    tv = data["data"]["dataset"].get("vocab_size")
    if tv is not None:
        model["model"]["vocab_size"] = tv
    for fname, mapping in (("model.yaml", model), ("training.yaml", training), ("data.yaml", data),
                           ("inference.yaml", INFERENCE_GREEDY)):
        (d / fname).write_text(yaml.safe_dump(mapping, sort_keys=False))
    return d


def write_all_pipelines(root) -> list:
    return [write_pipeline(n, Path(root) / n) for n in PIPELINES]


__all__ += ["PIPELINES", "write_pipeline", "write_all_pipelines", "INFERENCE_GREEDY"]

if __name__ == "__main__":
    import sys
    for p in write_all_pipelines(sys.argv[1] if len(sys.argv) > 1 else "configs/kimi_full_pipeline"):
        print(p)
