from pathlib import Path

import torch

from packbalance_b200.config import ModelConfig
from packbalance_b200.models.llama import LlamaForCausalLM
from packbalance_b200.parallel.flat import FlatParameters
from packbalance_b200.parallel.optim import FlatAdamW
from packbalance_b200.train.checkpoint import committed_checkpoints, find_latest_checkpoint, load_checkpoint, save_checkpoint
from packbalance_b200.utils import AsyncCheckpointWriter


def _make(cfg):
    m = LlamaForCausalLM(cfg)
    f = FlatParameters(m)
    return m, FlatAdamW(f, lr=1e-3)


def test_save_load_roundtrip_and_reference_format(tmp_path: Path, model_cfg: ModelConfig) -> None:
    torch.manual_seed(0)
    m, o = _make(model_cfg)
    m.flat = None
    o.flat.grad.normal_()
    o.step()
    d = save_checkpoint(m, o, 7, tmp_path / "ckpt", fsdp=False, extra={"loss": 1.5})
    state = torch.load(d / "state.pt", weights_only=False)
    assert set(state) == {"model", "optimizer", "step", "extra"} and state["step"] == 7
    assert (d / "meta.json").exists()
    m2, o2 = _make(model_cfg)
    meta = load_checkpoint(d, m2, o2, fsdp=False, device=torch.device("cpu"))
    assert meta["step"] == 7 and meta["loss"] == 1.5
    for a, b in zip(m.state_dict().values(), m2.state_dict().values()):
        torch.testing.assert_close(a, b)
    torch.testing.assert_close(o.exp_avg, o2.exp_avg)
    # A plain torch model + AdamW (the reference's objects) can read the same file.
    ref = LlamaForCausalLM(model_cfg)
    ref.load_state_dict(state["model"])
    torch.optim.AdamW(ref.parameters()).load_state_dict(state["optimizer"])


def test_torn_checkpoint_is_skipped_and_pruning(tmp_path: Path, model_cfg: ModelConfig) -> None:
    m, o = _make(model_cfg)
    root = tmp_path / "checkpoints"
    writer = AsyncCheckpointWriter()
    for step in (1, 2, 3):
        save_checkpoint(m, o, step, root, fsdp=False, async_writer=writer, keep_last=2)
        writer.wait()
    assert [p.name for p in committed_checkpoints(root)] == ["step_0000002", "step_0000003"]
    torn = root / "step_0000009"
    torn.mkdir()
    (torn / "state.pt.tmp").write_bytes(b"partial")
    assert find_latest_checkpoint(tmp_path).name == "step_0000003"
