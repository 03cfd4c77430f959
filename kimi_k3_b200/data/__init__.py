"""Data pipelines: synthetic retrieval, causal text corpora, YAML loader bundles, prefetching."""
from .synthetic import (SimpleWordTokenizer, SyntheticRetrievalConfig, SyntheticRetrievalDataset,
                        SyntheticRetrievalGenerator, SyntheticRetrievalMTPDataset, SyntheticTokenDataset,
                        create_synthetic_retrieval_dataloaders)
from .text import (CausalTextDataset, HF_TEXT_DATASETS, TextDataloaderConfig, available_hf_text_dataset_presets,
                   create_hf_text_dataloaders, create_text_dataloaders, train_byte_level_bpe_tokenizer)
from .yaml_config import (DataBundle, DataPipelineConfig, LoaderConfig, build_dataloaders, build_dataloaders_from_yaml,
                          load_data_config, load_tokenizer_from_data_yaml)
from .prefetch import DevicePrefetcher
from .inspection import summarize_lm_batch, summarize_tensor
