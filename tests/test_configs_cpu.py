"""The YAML run configurations (one per benchmark configuration, plus the reference's own
run) load into a valid ModelConfig and TrainArgs."""
import glob
import os
import sys

import pytest

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, HERE)

FILES = sorted(glob.glob(os.path.join(HERE, "atomic_ai_hybrid_b200", "configs", "*.yaml")))


def test_there_is_a_file_per_configuration():
    names = {os.path.basename(f) for f in FILES}
    assert {"config1_tiny_cpu.yaml", "config3_hybrid_1b.yaml", "config4_hybrid_7b_ep8.yaml",
            "config5_hybrid_long_tp8.yaml", "reference.yaml"} <= names


@pytest.mark.parametrize("path", FILES, ids=[os.path.basename(f) for f in FILES])
def test_config_loads(path):
    import train
    from atomic_ai_hybrid_b200.config import load_yaml_config
    cfg = load_yaml_config(path)
    cfg.validate()
    args = train.apply_yaml_train_section(train.parse(["--config", path]))
    assert args.seq_len > 0 and args.global_batch > 0
    if "long" in path:
        assert args.tensor_parallel == 8 and args.expert_parallel == 8 and args.remat
        assert cfg.d_model == 4096 and cfg.num_layers == 48
    # a flag given on the command line wins over the file
    args = train.apply_yaml_train_section(train.parse(["--config", path, "--seq-len", "128"]))
    assert args.seq_len == 128
