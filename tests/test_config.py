from pathlib import Path

import pytest
import yaml

from packbalance_b200.config import DataConfig, ModelConfig, TrainConfig, config_to_dict, load_config, save_config

CONFIG_DIR = Path(__file__).resolve().parents[1] / "configs"


def test_roundtrip(tmp_path: Path) -> None:
    cfg = load_config(CONFIG_DIR / "tiny.yaml")
    save_config(cfg, tmp_path / "c.yaml")
    assert config_to_dict(load_config(tmp_path / "c.yaml")) == config_to_dict(cfg)


def test_unknown_keys_rejected(tmp_path: Path) -> None:
    p = tmp_path / "bad.yaml"
    p.write_text(yaml.safe_dump({"model": {"d_modle": 3}}))
    with pytest.raises(ValueError):
        load_config(p)
    p.write_text(yaml.safe_dump({"optim": {}}))
    with pytest.raises(ValueError):
        load_config(p)


@pytest.mark.parametrize("name", sorted(p.name for p in CONFIG_DIR.glob("*.yaml")))
def test_shipped_configs_load(name: str) -> None:
    load_config(CONFIG_DIR / name)


def test_reference_schema_keys_accepted() -> None:
    ModelConfig(dropout=0.1, attention_backend="flex", compile_attention=True)
    DataConfig(drop_last=False, tokenizer="x", persistent_workers=False)
    TrainConfig(keep_last=3, compile=True, find_unused_parameters=True, bucket_cap_mb=10)


def test_validation() -> None:
    with pytest.raises(ValueError):
        ModelConfig(d_model=30, n_heads=4)
    with pytest.raises(ValueError):
        DataConfig(mode="nope")
    with pytest.raises(ValueError):
        TrainConfig(dtype="fp8")
    assert abs(DataConfig(synthetic_median=256.0).lognormal_mu - 5.545) < 1e-3


def test_overrides_parse_yaml_values_and_validate() -> None:
    from packbalance_b200.config import PackBalanceConfig, apply_overrides

    cfg = apply_overrides(PackBalanceConfig(), ["train.fsdp_weight_windows=2", "train.grad_reduce_dtype=bf16",
                                                "model.tie_embeddings=false", "data.seq_len=1024"])
    assert cfg.train.fsdp_weight_windows == 2 and cfg.train.grad_reduce_dtype == "bf16"
    assert cfg.model.tie_embeddings is False and cfg.data.seq_len == 1024
    for bad in ("train.nope=1", "train.fsdp_weight_windows", "nope.x=1", "train.fsdp_weight_windows=1",
                "train.fsdp_weight_windows=-2",
                "train.grad_reduce_dtype=fp16"):
        with pytest.raises(ValueError):
            apply_overrides(PackBalanceConfig(), [bad])


def test_overrides_coerce_float_fields() -> None:
    from packbalance_b200.config import PackBalanceConfig, apply_overrides

    cfg = apply_overrides(PackBalanceConfig(), ["train.lr=3e-4", "train.grad_clip=2", "train.min_lr=1.5e-5"])
    assert cfg.train.lr == 3e-4 and isinstance(cfg.train.lr, float)
    assert cfg.train.grad_clip == 2.0 and isinstance(cfg.train.grad_clip, float)
    assert cfg.train.min_lr == 1.5e-5
    with pytest.raises(ValueError):
        apply_overrides(PackBalanceConfig(), ["train.lr=fast"])
