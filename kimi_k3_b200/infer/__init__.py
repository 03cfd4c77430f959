"""Inference: cached generation, sampling, checkpoint loading, audits, YAML configuration."""
from .audit import compare_full_vs_cached_logits
from .cache import cache_memory_bytes, cache_summary, validate_kimi_cache
from .config import GenerationConfig, ModelLoadConfig
from .generation import (GenerationOutput, decode_one_token, generate_tokens, inference_autoregressive,
                         prefill_prompt)
from .graph_decode import GraphDecoder, graph_generate
from .loading import LoadedKimiCheckpoint, load_kimi_checkpoint
from .sampling import apply_repetition_penalty, sample_next_token, top_k_filter, top_p_filter
from .tokenization import decode_token_ids, encode_prompt, tokenizer_token_id
from .yaml_config import InferenceYamlConfig, load_generation_config, load_inference_yaml_config
