"""The module benchmarks run on CPU with the reference's CSV columns; MTP parameter
accounting matches the reference on the reference benchmark's modules."""
import io
from contextlib import redirect_stdout

import pytest
import torch

from _oracle import needs_reference, ref


def _run(fn, argv):
    buf = io.StringIO()
    with redirect_stdout(buf):
        rows = fn(argv)
    return rows, buf.getvalue().strip().splitlines()


def test_kda_benchmark_columns():
    from kimi_k3_b200.bench.modules import bench_kda
    rows, lines = _run(bench_kda, ["--device", "cpu", "--lengths", "64", "100"])
    assert lines[0] == "length,recurrent_seconds,chunkwise_seconds,decode_ms,state_elements"
    assert [r[0] for r in rows] == [64, 100]
    assert rows[0][4] == rows[1][4]  # the state does not grow with the context


def test_mla_benchmark_compression():
    from kimi_k3_b200.bench.modules import bench_mla
    rows, lines = _run(bench_mla, ["--device", "cpu", "--lengths", "32", "--repeats", "1"])
    assert lines[0].startswith("length,seconds,decode_ms,latent_elements")
    length, _, _, latent, full_kv, ratio = rows[0]
    assert latent * ratio == full_kv and latent == 32 * 32


def test_moe_benchmark_backends_agree():
    from kimi_k3_b200.bench.modules import bench_moe
    rows, _ = _run(bench_moe, ["--device", "cpu", "--tokens", "16", "--top-k", "2", "--repeats", "1"])
    assert len(rows) == 4
    by = {(r[0], r[1]): r for r in rows}
    for routing in ("natural", "imbalanced"):
        a, b = by[("reference", routing)], by[("vectorized", routing)]
        assert a[6:9] == b[6:9]  # assignments, zero-load experts, load CV
    assert by[("reference", "imbalanced")][7] > 0


def test_backbone_and_attnres_benchmarks():
    from kimi_k3_b200.bench.modules import bench_attnres, bench_backbone
    rows, _ = _run(bench_backbone, ["--device", "cpu", "--groups", "1", "--lengths", "16", "--repeats", "1"])
    assert rows[0][5] > 0 and rows[0][6] > 0
    rows, _ = _run(bench_attnres, ["--device", "cpu", "--layers", "2", "--lengths", "4", "--decode-contexts", "8",
                                   "--repeats", "1"])
    depth = {(r[1], r[2]): r for r in rows if r[0] == "depth"}
    assert depth[("full", "eager")][7] > depth[("block", "eager")][7]  # full AttnRes reads more sources
    assert depth[("block", "two_phase")][8] > 0 and depth[("block", "eager")][8] == 0


def _reference_mtp_head(vocab_size=128, d_model=16):
    """The reference benchmark's MTP modules, built through the reference API."""
    ref()
    import torch.nn as nn
    from src.attention_residuals import AttentionResidualConfig
    from src.kda import KDAConfig
    from src.mla import GatedMLAConfig
    from src.mtp import KimiMTPConfig, KimiMTPHead
    from src.stable_latent_moe import StableLatentMoEConfig
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
    return KimiMTPHead(cfg, emb, head)


@needs_reference
def test_mtp_parameter_counts_match_reference():
    ref()
    from src.mtp import mtp_parameter_counts as ref_counts
    from kimi_k3_b200.bench.modules import bench_mtp, build_mtp_modules
    from kimi_k3_b200.models.mtp import mtp_parameter_counts
    theirs = ref_counts(_reference_mtp_head())
    torch.manual_seed(0)
    _, _, _, head = build_mtp_modules()
    ours = mtp_parameter_counts(head)
    assert ours == theirs
    assert ours["unique_mtp_total"] == ours["fusion"] + ours["block"] > 0
    assert ours["shared_embedding_lm_overlap"] == ours["shared_lm_head"]  # tied weights
    out, lines = _run(bench_mtp, ["--device", "cpu", "--iterations", "2"])
    assert lines[-1] == f"unique_mtp_parameters={ours['unique_mtp_total']}"


@pytest.mark.slow
@pytest.mark.parametrize("impl", ["ours", "reference"])
def test_bench_cpu_smoke_prints_one_json_line(impl):
    """``bench.py --config cpu_smoke`` (both arms) prints a single JSON result line with the metric,
    its value and unit, the step time and the decode figures."""
    import json
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if impl == "reference":
        from conftest import reference_available
        if not reference_available():
            pytest.skip("reference package not installed")
    proc = subprocess.run([sys.executable, "bench.py", "--config", "cpu_smoke", "--steps", "2", "--warmup", "3",
                           "--impl", impl], cwd=root, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    out = json.loads(lines[0])
    assert out["metric"] == "train_tokens_per_s" and out["unit"] == "tokens/s" and out["value"] > 0
    assert out["steps"] == 2 and out["warmup"] == 3 and out["higher_is_better"] is True
    assert out["decode"]["generated_tokens"] == 8
    assert (out.get("impl") == "reference") == (impl == "reference")
