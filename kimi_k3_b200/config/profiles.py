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
