"""Tensor- and expert-parallel inference on CPU (gloo ranks) against one process.

A float64 tiny model generates greedily (cached prefill + decode) in one process; the same
weights sharded over two ranks (TP, EP, EP overlaid on TP) must produce the same tokens and
the same per-step logits, through the eager generation loop and through the serving decoder.
The inference YAML path (``distributed:`` section, checkpoint on disk) is exercised end to end.
"""
import os

import pytest
import torch

from _dist_harness import run_ranks

STEPS = 6


def _model():
    from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
    cfg = kimi_k3_cpu_tiny_config(enable_vision=False)
    torch.manual_seed(0)
    return KimiK3(cfg).double().eval()


def _prompt():
    g = torch.Generator().manual_seed(3)
    return torch.randint(5, 128, (2, 9), generator=g)


def _generate(model, decoder: bool):
    from kimi_k3_b200.infer import GenerationConfig, GraphDecoder, generate_tokens
    cfg = GenerationConfig(max_new_tokens=STEPS, do_sample=False, return_scores=True, device="cpu")
    ids = _prompt()
    if decoder:
        out = GraphDecoder(model, max_length=ids.shape[1] + STEPS, generation_config=cfg, use_graph=False,
                           autocast_dtype=None).generate(ids)
        return out.sequences, None
    out = generate_tokens(model, ids, generation_config=cfg)
    return out.sequences, torch.stack(out.scores)


def _layout_config(layout, world):
    from kimi_k3_b200.parallel.config import distributed_config_from_dict
    cfg = {"enabled": True, "backend": "gloo", "timeout_seconds": 120}
    if layout in ("tp", "tp_ep_overlay"):
        cfg["tensor_parallel"] = {"enabled": True, "size": world}
    if layout == "ep":
        cfg["expert_parallel"] = {"enabled": True, "size": world}
    if layout == "tp_ep_overlay":
        cfg["expert_parallel"] = {"enabled": True, "size": world, "overlay_tensor_parallel": True}
    return distributed_config_from_dict(cfg)


def _rank(rank, world, layout):
    from kimi_k3_b200.infer.distributed import graph_capturable, prepare_distributed_model
    from kimi_k3_b200.parallel.environment import setup_distributed
    dcfg = _layout_config(layout, world)
    ctx = setup_distributed(dcfg)
    model = prepare_distributed_model(_model(), dcfg, ctx)
    seq, scores = _generate(model, decoder=False)
    seq_dec, _ = _generate(model, decoder=True)
    capturable = graph_capturable(model)
    # the serving copy of a sharded model shares its process groups instead of copying them
    from kimi_k3_b200.infer.graph_decode import serving_copy
    seq_copy, _ = _generate(serving_copy(model, torch.float64), decoder=False)
    assert torch.equal(seq_copy, seq)
    ctx.close()
    return seq, scores, seq_dec, capturable


@pytest.mark.parametrize("layout", ["tp", "ep", "tp_ep_overlay"])
def test_sharded_generation_matches_single_process(layout):
    ref_seq, ref_scores = _generate(_model(), decoder=False)
    ref_dec, _ = _generate(_model(), decoder=True)
    assert torch.equal(ref_seq, ref_dec)
    for seq, scores, seq_dec, capturable in run_ranks(_rank, 2, layout):
        assert torch.equal(seq, ref_seq), layout
        assert torch.equal(seq_dec, ref_seq), layout
        # logits of every step: vocabulary-parallel head gathered, float64 end to end
        assert (scores - ref_scores).abs().max().item() < 1e-9, layout
        # the NCCL-style all-to-all exchange sizes its splits on the host: not capturable
        assert capturable == (layout == "tp")


def _yaml_rank(rank, world, root):
    from kimi_k3_b200.infer import load_inference_yaml_config
    from kimi_k3_b200.infer.distributed import run_distributed_generation
    iy = load_inference_yaml_config(os.path.join(root, "inference.yaml"))
    out, ctx = run_distributed_generation(os.path.join(root, "model.yaml"), os.path.join(root, "ckpt.pt"),
                                          [int(x) for x in _prompt()[0]], iy)
    seq = out.sequences.clone()
    world_size = ctx.world_size
    ctx.close()
    return seq, world_size


def test_inference_yaml_distributed_section(tmp_path):
    from kimi_k3_b200.config.model_yaml import build_model_from_yaml
    from kimi_k3_b200.config.profiles import write_pipeline
    from kimi_k3_b200.infer import GenerationConfig, generate_tokens
    write_pipeline("cpu_smoke", tmp_path)
    model = build_model_from_yaml(tmp_path / "model.yaml")
    torch.save({"model_state_dict": model.state_dict(), "format_version": 1}, tmp_path / "ckpt.pt")
    (tmp_path / "inference.yaml").write_text(
        "inference:\n  max_new_tokens: 5\n  do_sample: false\n  add_bos_token: false\n  device: cpu\n"
        "distributed:\n  enabled: true\n  backend: gloo\n  data_parallel: {mode: none, size: 1}\n"
        "  tensor_parallel: {enabled: true, size: 2}\n  expert_parallel: {enabled: false, size: 1}\n")
    model.eval()
    ids = _prompt()[:1]
    ref = generate_tokens(model, ids, generation_config=GenerationConfig(max_new_tokens=5, device="cpu")).sequences
    for seq, world_size in run_ranks(_yaml_rank, 2, str(tmp_path)):
        assert world_size == 2
        assert torch.equal(seq, ref)


def test_cli_infer_single_process(tmp_path, capsys):
    """``python -m kimi_k3_b200 infer`` without a distributed section: token-id prompt, greedy."""
    from kimi_k3_b200.cli import main
    from kimi_k3_b200.config.model_yaml import build_model_from_yaml
    from kimi_k3_b200.config.profiles import write_pipeline
    write_pipeline("cpu_smoke", tmp_path)
    model = build_model_from_yaml(tmp_path / "model.yaml")
    torch.save({"model_state_dict": model.state_dict(), "format_version": 1}, tmp_path / "ckpt.pt")
    assert main(["infer", "--model-config", str(tmp_path / "model.yaml"), "--checkpoint", str(tmp_path / "ckpt.pt"),
                 "--prompt", "5 17 9 33", "--max-new-tokens", "3"]) == 0
    out = capsys.readouterr().out.splitlines()
    import json
    stats = json.loads(out[-1])
    assert stats["world_size"] == 1 and stats["finish_reason"] in ("length", "eos")
    assert out[0].startswith("[[5, 17, 9, 33")
