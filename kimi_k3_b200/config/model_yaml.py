"""Strict model YAML schema -> typed ``KimiK3Config`` (no weights allocated).

Parity: ``src/kimi_k3/yaml_config.py:66-302`` (reference).  The schema is the
reference's, so its profile ``model.yaml`` files load unchanged:
``model: {architecture: kimi_k3, d_model, vocab_size (int | auto), num_heads,
num_hybrid_groups, attention_pattern, add_final_gated_mla, special ids,
kda: {...}, mla: {...}, moe: {...}, attention_residual: {...}, vision: {...}, mtp: {...}}``.
Head dimensions and ``d_model`` are injected into the sub-configs; a data
vocabulary larger than the model vocabulary is rejected.
"""
from __future__ import annotations

from pathlib import Path
from typing import Any

from ..models.attnres import AttentionResidualConfig
from ..models.backbone import KimiBlockConfig
from ..models.kda import KDAConfig
from ..models.kimi_k3 import KimiK3Config, VisionProjectorConfig, vision_output_dim
from ..models.mla import GatedMLAConfig
from ..models.moe import StableLatentMoEConfig
from ..models.mtp import KimiMTPConfig
from ..models.vision import VisionEncoderConfig
from ..models.vision_ablations import HierarchicalVisionConfig, SwinVisionConfig
from .yaml_utils import ConfigError, dataclass_kwargs, expect_mapping, load_yaml_mapping, reject_unknown_keys


def _component(values, typ, *, path, injected):
    merged = {**injected, **values}
    try:
        return typ(**dataclass_kwargs(merged, typ, path=path))
    except (TypeError, ValueError) as exc:
        if isinstance(exc, ConfigError):
            raise
        raise ConfigError(f"{path}: {exc}") from exc


def _special_ids(model: dict, data_bundle) -> dict:
    use_data = bool(model.pop("use_data_special_tokens", False))
    vals = {n: model.pop(n, None) for n in ("pad_token_id", "bos_token_id", "eos_token_id", "image_token_id",
                                            "video_token_id")}
    if use_data and data_bundle is not None:
        for name, tok in (("pad_token_id", "<pad>"), ("bos_token_id", "<bos>"), ("eos_token_id", "<eos>")):
            resolved = data_bundle.token_id(tok)
            if resolved is not None:
                vals[name] = int(resolved)
    return vals


TOP_LEVEL_FIELDS = {"tie_word_embeddings", "use_bias_in_lm_head", "vision_token_integration", "freeze_vision_encoder",
                    "return_dict", "output_hidden_states", "output_attentions", "output_router_diagnostics",
                    "output_attnres_diagnostics"}


def build_model_config_from_mapping(values: dict[str, Any], *, data_bundle=None,
                                    vocab_size_override: int | None = None) -> KimiK3Config:
    root = dict(values)
    model = expect_mapping(root, "model", path="root")
    reject_unknown_keys(root, path="root")
    if model.pop("architecture", None) != "kimi_k3":
        raise ConfigError("model.architecture must be 'kimi_k3'")
    model.pop("name", None)
    d_model = int(model.pop("d_model"))
    vocab_value = model.pop("vocab_size")
    if vocab_size_override is not None:
        vocab = int(vocab_size_override)
    elif vocab_value == "auto":
        if data_bundle is None:
            raise ConfigError("vocab_size=auto requires data_bundle")
        vocab = data_bundle.vocab_size
    else:
        vocab = int(vocab_value)
    if data_bundle is not None and data_bundle.vocab_size > vocab:
        raise ConfigError(f"data vocabulary ({data_bundle.vocab_size}) exceeds model vocab_size ({vocab})")
    special = _special_ids(model, data_bundle)
    heads = int(model.pop("num_heads"))
    if d_model % heads:
        raise ConfigError("model.d_model must be divisible by num_heads")
    vdim = d_model // heads
    groups = int(model.pop("num_hybrid_groups"))
    pattern = tuple(model.pop("attention_pattern", ("kda", "kda", "kda", "gated_mla")))
    add_final = bool(model.pop("add_final_gated_mla", True))
    kda_v = expect_mapping(model, "kda", path="model")
    kda = _component(kda_v, KDAConfig, path="model.kda",
                     injected={"d_model": d_model, "num_heads": heads, "key_head_dim": int(kda_v.pop("key_head_dim")),
                               "value_head_dim": vdim})
    mla_v = expect_mapping(model, "mla", path="model")
    mla = _component(mla_v, GatedMLAConfig, path="model.mla",
                     injected={"d_model": d_model, "num_heads": heads, "q_head_dim": int(mla_v.pop("q_head_dim")),
                               "v_head_dim": vdim, "kv_latent_dim": int(mla_v.pop("kv_latent_dim"))})
    moe = _component(expect_mapping(model, "moe", path="model"), StableLatentMoEConfig, path="model.moe",
                     injected={"d_model": d_model})
    attnres = _component(expect_mapping(model, "attention_residual", path="model"), AttentionResidualConfig,
                         path="model.attention_residual", injected={"d_model": d_model})
    init_range = float(model.pop("initializer_range", 0.02))
    backbone = KimiBlockConfig(d_model=d_model, num_pattern_repeats=groups, kda_config=kda, mla_config=mla,
                               stable_latent_moe_config=moe, attention_residual_config=attnres,
                               attention_pattern=pattern, add_final_gated_mla=add_final,
                               rms_norm_eps=float(model.pop("rms_norm_eps", 1e-6)),
                               residual_dropout=float(model.pop("residual_dropout", 0.0)), init_std=init_range)
    vis_v = expect_mapping(model, "vision", path="model", required=False)
    enable_vision = bool(vis_v.pop("enabled", False))
    use_ps = bool(vis_v.pop("use_pixel_shuffle", True))
    vision = projector = None
    if enable_vision:
        vtype = vis_v.pop("type", "moonvit")
        proj_v = vis_v.pop("projector", {})
        classes = {"moonvit": VisionEncoderConfig, "hierarchical": HierarchicalVisionConfig, "swin": SwinVisionConfig}
        if vtype not in classes:
            raise ConfigError(f"unsupported model.vision.type: {vtype}")
        for key in ("embed_dims", "depths", "num_heads"):
            if isinstance(vis_v.get(key), list):
                vis_v[key] = tuple(vis_v[key])
        vision = classes[vtype](**dataclass_kwargs(vis_v, classes[vtype], path="model.vision"))
        width = vision_output_dim(vision)
        if not isinstance(proj_v, dict):
            raise ConfigError("model.vision.projector must be a mapping")
        defaults = {"input_dim": width * (4 if use_ps else 1), "hidden_dim": max(d_model, width), "output_dim": d_model}
        projector = VisionProjectorConfig(**dataclass_kwargs({**defaults, **proj_v}, VisionProjectorConfig,
                                                             path="model.vision.projector"))
    else:
        reject_unknown_keys(vis_v, path="model.vision")
    mtp_v = expect_mapping(model, "mtp", path="model", required=False)
    enable_mtp = bool(mtp_v.pop("enabled", True))
    mtp = None
    if enable_mtp:
        ar_v = mtp_v.pop("attention_residual", {"mode": "block", "sublayers_per_depth_block": 8, "backend": "eager"})
        if not isinstance(ar_v, dict):
            raise ConfigError("model.mtp.attention_residual must be a mapping")
        mtp_ar = _component(ar_v, AttentionResidualConfig, path="model.mtp.attention_residual",
                            injected={"d_model": d_model})
        mtp = KimiMTPConfig(d_model=d_model, vocab_size=vocab, kda_config=kda, mla_config=mla,
                            stable_latent_moe_config=moe, attention_residual_config=mtp_ar,
                            **dataclass_kwargs(mtp_v, KimiMTPConfig, path="model.mtp"))
    else:
        reject_unknown_keys(mtp_v, path="model.mtp")
    top = {k: model.pop(k) for k in tuple(model) if k in TOP_LEVEL_FIELDS}
    reject_unknown_keys(model, path="model")
    return KimiK3Config(vocab_size=vocab, d_model=d_model, backbone=backbone, **special, vision=vision,
                        vision_projector=projector, mtp=mtp, enable_vision=enable_vision, enable_mtp=enable_mtp,
                        vision_use_pixel_shuffle=use_ps, initializer_range=init_range, **top)


def load_model_config(path: str | Path, *, data_bundle=None, vocab_size_override: int | None = None) -> KimiK3Config:
    _, values = load_yaml_mapping(path)
    return build_model_config_from_mapping(values, data_bundle=data_bundle, vocab_size_override=vocab_size_override)


def build_model_from_yaml(path: str | Path, *, data_bundle=None, vocab_size_override: int | None = None):
    from ..models.kimi_k3 import KimiK3
    return KimiK3(load_model_config(path, data_bundle=data_bundle, vocab_size_override=vocab_size_override))


__all__ = ["build_model_config_from_mapping", "load_model_config", "build_model_from_yaml"]
