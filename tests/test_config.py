"""Config surface: the 29B YAMLs load, legacy keys map, unknown/duplicate keys fail, CLI wins."""
import os

import pytest

from pan2_b200.config import parse_training_config

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PRE = os.path.join(ROOT, "config", "pretrain_29B_720p.yaml")


def test_pretrain_yaml_loads():
    c = parse_training_config(["--config", PRE])
    assert c.transformer_config_overrides["num_layers"] == 44
    assert c.learning_rate == 2e-5 and c.lr_scheduler_type == "cosine_decay" and c.cp_size == 4
    assert c.packed_joint_token_budget == 110576 and c.hybrid_shard is True
    assert c.snr_type.value == "lognorm" and c.train_timestep_shift == 9.0


def test_cli_overrides_yaml():
    c = parse_training_config(["--config", PRE, "--learning_rate", "3e-4", "--sp_size", "2", "--no_anomaly"])
    assert c.learning_rate == 3e-4 and c.cp_size == 2 and c.anomaly_detection is False


def test_unknown_and_duplicate_keys(tmp_path):
    bad = tmp_path / "bad.yaml"
    bad.write_text("training:\n  not_an_option: 1\n")
    with pytest.raises(ValueError, match="is not an option"):
        parse_training_config(["--config", str(bad)])
    dup = tmp_path / "dup.yaml"
    dup.write_text("a:\n  learning_rate: 1.0e-4\nb:\n  learning_rate: 2.0e-4\n")
    with pytest.raises(ValueError, match="twice"):
        parse_training_config(["--config", str(dup)])


def test_legacy_keys_and_checks(tmp_path):
    y = tmp_path / "legacy.yaml"
    y.write_text("x:\n  sp_size: 2\n  i2v_prob: 0.25\n  single_stream_only: true\n")
    c = parse_training_config(["--config", str(y)])
    assert c.cp_size == 2 and c.image_cond_prob == 0.25
    with pytest.raises(ValueError):
        parse_training_config(["--image_cond_prob", "0.8", "--video_cond_prob", "0.5"])
    with pytest.raises(ValueError):
        parse_training_config(["--pretrained_transformer_path", "/nonexistent"])
