"""Configuration checks on CPU: every built-in pipeline profile loads, validates and matches the committed
YAML; strict unknown-key rejection; the CLI's validate / train --validate-only / profiles commands; the
reference's own loaders read the generated model and data YAMLs to the same configs.

Reference behaviour: ``configuration/yaml_utils.py`` (strict mappings), ``src/kimi_k3/yaml_config.py:66-295``
(model YAML), ``data/yaml_config.py:138`` (data YAML), ``scripts/validate_*.py`` (CLI summaries).
"""
import json
from pathlib import Path

import pytest
import yaml

from _oracle import needs_reference, ref
from kimi_k3_b200.cli import main
from kimi_k3_b200.config.model_yaml import build_model_config_from_mapping, load_model_config
from kimi_k3_b200.config.profiles import PIPELINES, write_all_pipelines, write_pipeline
from kimi_k3_b200.config.yaml_utils import ConfigError, resolve_kimi_pipeline_profile
from kimi_k3_b200.data import load_data_config
from kimi_k3_b200.train.config import load_training_config, validate_pipeline_compatibility

ROOT = Path(__file__).resolve().parents[1]
COMMITTED = ROOT / "configs" / "kimi_full_pipeline"
NAMES = sorted(PIPELINES)


@pytest.fixture(scope="module")
def generated(tmp_path_factory):
    out = tmp_path_factory.mktemp("pipelines")
    write_all_pipelines(out)
    return out


@pytest.mark.parametrize("name", NAMES)
def test_profile_loads_and_validates(generated, name):
    paths = resolve_kimi_pipeline_profile(generated / name)
    t = load_training_config(paths.training)
    d = load_data_config(paths.data)
    m = load_model_config(paths.model)
    validate_pipeline_compatibility(t, model_config=m, data_config=d)
    assert m.d_model > 0 and m.vocab_size > 0
    if t.distributed.enabled:
        assert t.distributed.logical_world_size >= 2


@pytest.mark.parametrize("name", NAMES)
def test_committed_profile_matches_the_generator(generated, name):
    for part in ("model.yaml", "data.yaml", "training.yaml"):
        committed = COMMITTED / name / part
        if not committed.is_file():
            pytest.skip(f"{name}/{part} is not committed")
        assert yaml.safe_load(committed.read_text()) == yaml.safe_load((generated / name / part).read_text()), part


@pytest.mark.parametrize("part,loader", [("model.yaml", load_model_config), ("data.yaml", load_data_config),
                                         ("training.yaml", load_training_config)])
def test_unknown_keys_are_rejected(generated, tmp_path, part, loader):
    src = yaml.safe_load((generated / "cpu_smoke" / part).read_text())
    top = next(iter(src))
    bad = dict(src)
    if isinstance(bad[top], dict):
        bad[top] = {**bad[top], "definitely_not_a_key": 1}
    else:
        bad["definitely_not_a_key"] = 1
    p = tmp_path / part
    p.write_text(yaml.safe_dump(bad))
    with pytest.raises((ConfigError, ValueError, TypeError)):
        loader(p)


def test_model_mapping_rejects_a_data_vocab_larger_than_the_model(generated):
    values = yaml.safe_load((generated / "cpu_smoke" / "model.yaml").read_text())
    cfg = build_model_config_from_mapping(values)
    assert cfg.vocab_size > 0

    class Bundle:
        vocab_size = cfg.vocab_size + 1
        pad_token_id, bos_token_id, eos_token_id = 0, 1, 2
    fixed = dict(values)
    fixed["model"] = {**fixed["model"], "vocab_size": cfg.vocab_size}
    with pytest.raises((ConfigError, ValueError)):
        build_model_config_from_mapping(fixed, data_bundle=Bundle())


def test_missing_profile_directory_is_reported(tmp_path):
    with pytest.raises((ConfigError, FileNotFoundError, ValueError)):
        resolve_kimi_pipeline_profile(tmp_path / "nope")


# --------------------------------------------------------------------------- CLI
@pytest.mark.parametrize("name", NAMES)
def test_cli_validate_prints_a_summary(generated, name, capsys):
    d = generated / name
    assert main(["validate", "--data-config", str(d / "data.yaml"), "--model-config", str(d / "model.yaml"),
                 "--training-config", str(d / "training.yaml")]) == 0
    out = json.loads(capsys.readouterr().out)
    assert set(out) >= {"data", "model", "distributed"}
    if out["distributed"]["enabled"]:
        assert out["launch"].startswith("torchrun") and str(out["distributed"]["world_size"]) in out["launch"]


@pytest.mark.parametrize("name", ["cpu_smoke", "t4_wikitext", "gpu_80gb", "distributed_tp_ep_4x_24gb"])
def test_cli_train_validate_only(generated, name, capsys):
    assert main(["train", "--profile", str(generated / name), "--validate-only"]) == 0
    out = json.loads(capsys.readouterr().out)
    assert out["model_d_model"] > 0 and out["distributed_world"] >= 1


def test_cli_argument_errors(generated):
    with pytest.raises(SystemExit):
        main(["train", "--profile", str(generated / "cpu_smoke"), "--model-config", "x.yaml", "--validate-only"])
    with pytest.raises(SystemExit):
        main(["train", "--model-config", "x.yaml", "--validate-only"])
    with pytest.raises(SystemExit):
        main(["unknown-command"])


def test_cli_profiles_writes_every_pipeline(tmp_path, capsys):
    assert main(["profiles", "--output", str(tmp_path)]) == 0
    printed = capsys.readouterr().out.split()
    assert len(printed) == len(NAMES)
    for name in NAMES:
        assert (tmp_path / name / "model.yaml").is_file()
    single = write_pipeline("cpu_smoke", tmp_path / "one")
    assert Path(single).exists()


# --------------------------------------------------------------------------- reference loaders
@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("name", NAMES)
def test_reference_loaders_read_the_generated_model_and_data_yaml(generated, name):
    ref()
    from data.yaml_config import load_data_config as ref_data
    from src.kimi_k3.yaml_config import load_model_config as ref_model
    d = generated / name
    assert ref_model(d / "model.yaml").to_dict() == load_model_config(d / "model.yaml").to_dict()
    theirs, ours = ref_data(d / "data.yaml"), load_data_config(d / "data.yaml")
    assert theirs.name == ours.name


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("vision_type,extra", [
    ("moonvit", dict(image_size=16, patch_size=4, embed_dim=16, depth=1, num_heads=4)),
    ("hierarchical", dict(image_size=32, patch_size=4, embed_dims=[8, 16], depths=[1, 1], num_heads=[2, 4])),
    ("swin", dict(image_size=32, patch_size=4, embed_dims=[8, 16], depths=[2, 2], num_heads=[2, 4], window_size=2)),
])
def test_model_yaml_vision_types_match_reference(generated, vision_type, extra):
    import copy
    ref()
    from src.kimi_k3.yaml_config import build_model_config_from_mapping as rbuild
    values = yaml.safe_load((generated / "cpu_smoke" / "model.yaml").read_text())
    values["model"]["vision"] = {"enabled": True, "type": vision_type, **extra, "projector": {"hidden_dim": 32}}
    ours = build_model_config_from_mapping(copy.deepcopy(values))
    assert ours.to_dict() == rbuild(copy.deepcopy(values)).to_dict()
    bad = copy.deepcopy(values)
    bad["model"]["vision"]["type"] = "convnext"
    with pytest.raises((ConfigError, ValueError)):
        build_model_config_from_mapping(bad)
