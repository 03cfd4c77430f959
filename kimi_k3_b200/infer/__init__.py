"""Inference: cached generation, sampling, checkpoint loading, audits, YAML configuration."""
from .config import GenerationConfig, ModelLoadConfig
from .generation import (GenerationOutput, decode_one_token, generate_tokens, inference_autoregressive,
                         prefill_prompt)
from .graph_decode import GraphDecoder, graph_generate
from .sampling import apply_repetition_penalty, sample_next_token, top_k_filter, top_p_filter
from .session import (CacheReport, InferenceSession, LoadedKimiCheckpoint, TextCodec, cache_memory_bytes,
                      cache_summary, compare_full_vs_cached_logits, decode_token_ids, encode_prompt,
                      load_kimi_checkpoint, tokenizer_token_id, validate_kimi_cache)
from .yaml_config import InferenceYamlConfig, load_generation_config, load_inference_yaml_config
