"""Data pipelines: synthetic retrieval parity with the reference, YAML bundles, text blocks,
context-curriculum loader factory, distributed sampler, device prefetcher (CPU)."""
import textwrap

import pytest
import torch

from _oracle import needs_reference, ref
from kimi_k3_b200.data import (CausalTextDataset, DevicePrefetcher, SyntheticRetrievalConfig,
                               build_dataloaders_from_yaml, create_synthetic_retrieval_dataloaders, load_data_config,
                               summarize_lm_batch, train_byte_level_bpe_tokenizer)
from kimi_k3_b200.parallel.sampler import StatefulDistributedSampler

SMOKE = SyntheticRetrievalConfig(num_train_examples=32, num_val_examples=8, block_size=32, min_filler_tokens=4,
                                 max_filler_tokens=12, num_keys_per_example=2, vocab_filler_size=32, num_key_types=8,
                                 num_value_types=16, batch_size=4, seed=7)


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("mtp", [False, True])
def test_synthetic_examples_match_reference(mtp):
    ref()
    from data.synthetic_long_context_retrieval import SyntheticRetrievalConfig as RC
    from data.synthetic_long_context_retrieval import create_synthetic_retrieval_dataloaders as rcreate
    import dataclasses
    rl, rv, rt = rcreate(RC(**dataclasses.asdict(SMOKE)), use_mtp=mtp)
    ol, ov, ot = create_synthetic_retrieval_dataloaders(SMOKE, use_mtp=mtp)
    assert rt.token_to_idx == ot.token_to_idx
    for i in range(len(rl.dataset)):
        a, b = rl.dataset[i], ol.dataset[i]
        for k in a:
            assert torch.equal(a[k], b[k]), (i, k)
    assert torch.equal(rv.dataset[3]["input_ids"], ov.dataset[3]["input_ids"])


def test_yaml_bundle_and_context_factory(tmp_path):
    p = tmp_path / "data.yaml"
    p.write_text(textwrap.dedent("""
        data:
          name: smoke
          kind: synthetic_retrieval
          dataset: {num_train_examples: 32, num_val_examples: 8, block_size: 32, min_filler_tokens: 4,
                    max_filler_tokens: 12, num_keys_per_example: 2, vocab_filler_size: 32, num_key_types: 8,
                    num_value_types: 16, seed: 7}
          loader: {batch_size: 4, num_workers: 0, shuffle_train: true, pin_memory: false, seed: 7}
        """))
    cfg = load_data_config(p)
    assert cfg.max_seq_len == 32 and cfg.loader.batch_size == 4
    bundle = build_dataloaders_from_yaml(p)
    b = next(iter(bundle.train_loader))
    assert b["input_ids"].shape[0] == 4 and b["input_ids"].shape[1] <= 32
    short = next(iter(bundle.train_loader_factory(16)))
    assert short["input_ids"].shape[1] <= 16
    with pytest.raises(ValueError):
        bundle.train_loader_factory(64)
    assert bundle.token_id("<pad>") == 0 and bundle.vocab_size > 50
    s = summarize_lm_batch(b)
    assert s["batch_size"] == 4
    bad = tmp_path / "bad.yaml"
    bad.write_text(p.read_text().replace("seed: 7}", "seed: 7, typo: 1}", 1))
    with pytest.raises(Exception):
        load_data_config(bad)


def test_text_blocks_and_bpe_tokenizer(tmp_path):
    docs = [f"document number {i} talks about kimi delta attention and latent experts." * 3 for i in range(40)]
    tok = train_byte_level_bpe_tokenizer(docs, vocab_size=300, min_frequency=1, save_path=tmp_path / "tok.json")
    ds = CausalTextDataset(docs, tok, block_size=16)
    item = ds[0]
    assert item["input_ids"].shape == (16,) and torch.equal(ds.input_ids[1, 1:], ds.labels[1, :-1])
    assert int(ds.input_ids[0, 0]) == tok.token_to_id("<bos>")


def test_distributed_sampler_shards_and_resumes():
    data = list(range(10))
    s0 = StatefulDistributedSampler(data, num_replicas=2, rank=0, shuffle=True, seed=3)
    s1 = StatefulDistributedSampler(data, num_replicas=2, rank=1, shuffle=True, seed=3)
    a, b = list(s0), list(s1)
    assert sorted(a + b) == data
    s0.set_epoch(1)
    it = iter(s0)
    first = [next(it), next(it)]
    state = s0.state_dict()
    rest = list(it)
    s2 = StatefulDistributedSampler(data, num_replicas=2, rank=0, shuffle=True, seed=3)
    s2.load_state_dict(state)
    assert list(s2) == rest and len(first) == 2


def test_device_prefetcher_cpu_passthrough():
    loader, _, _ = create_synthetic_retrieval_dataloaders(SMOKE)
    got = list(DevicePrefetcher(loader, "cpu"))
    assert len(got) == len(loader) and got[0]["input_ids"].shape[0] == 4
