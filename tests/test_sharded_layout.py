"""Layout of the native sharded engine (host-side arithmetic, CPU)."""

from dataclasses import replace

import pytest

from packbalance_b200.config import ModelConfig
from packbalance_b200.models.llama import LlamaForCausalLM
from packbalance_b200.parallel.sharded import ALIGN, plan_layout


@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("tie", [True, False])
def test_layout_covers_every_parameter_once(model_cfg: ModelConfig, world: int, tie: bool) -> None:
    model = LlamaForCausalLM(replace(model_cfg, tie_embeddings=tie))
    lay = plan_layout(model, world)
    names = [n for n, p in model.named_parameters()]
    slots = lay.rep + [s for u in lay.units for s in u.slots]
    assert sorted(s.name for s in slots) == sorted(names)
    # non-overlapping, in increasing order, norms first
    spans = sorted((s.offset, s.offset + s.numel) for s in slots)
    assert all(a[1] <= b[0] for a, b in zip(spans, spans[1:]))
    assert all(s.offset + s.numel <= lay.rep_n for s in lay.rep)
    assert all(s.name.endswith("norm.weight") for s in lay.rep)
    soff = 0
    for u in lay.units:
        assert u.unit0 % ALIGN == 0 and u.cs % ALIGN == 0 and u.cs * world >= u.span
        assert u.soff == soff
        soff += u.cs
        assert all(u.unit0 <= s.offset and s.offset + s.numel <= u.unit0 + u.span for s in u.slots)
        # gather segments lie in the unit and cover every weight of it
        covered = sum(hi - lo for lo, hi in u.segments)
        assert covered == u.span and all(u.unit0 <= lo < hi <= u.unit0 + u.span for lo, hi in u.segments)
    assert soff == lay.shard_numel
    assert lay.units[0].name == "embed" and (lay.units[-1].name == "head") == (not tie)


def test_layer_segments_follow_the_fused_gemms(model_cfg: ModelConfig) -> None:
    model = LlamaForCausalLM(model_cfg)
    lay = plan_layout(model, 2)
    layer = next(u for u in lay.units if u.name == "layer0")
    names = [s.name.split(".")[-2] for s in layer.slots]
    assert names == ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"]
    (qlo, qhi), (glo, ghi) = layer.segments
    assert qlo == layer.slots[0].offset and qhi == layer.slots[3].offset + layer.slots[3].numel
    assert glo == layer.slots[4].offset and ghi == layer.slots[6].offset + layer.slots[6].numel


def test_8b_config_fits_on_b200_at_8_ranks() -> None:
    """benchmark config #5 (Llama-3-8B shape) on 8 ranks: the sharded engine's persistent
    buffers per rank (bf16 gathered weights, fp32 gradient, fp32 master + moments +
    reduced-gradient shards) leave most of a B200's 180 GB for activations.  Built on
    the meta device: no memory is allocated."""
    from pathlib import Path

    import torch

    from packbalance_b200.config import load_config

    cfg = load_config(Path(__file__).resolve().parents[1] / "configs" / "b5_8b_fsdp.yaml")
    with torch.device("meta"):
        model = LlamaForCausalLM(cfg.model)
    n = sum(p.numel() for p in model.parameters())
    assert 7.9e9 < n < 8.1e9
    lay = plan_layout(model, 8)
    assert lay.numel >= n and lay.numel - n < 0.001 * n  # padding stays small
    assert lay.shard_numel * 8 >= n - lay.rep_n
    per_rank = 2 * lay.numel + 4 * lay.numel + 16 * lay.shard_numel
    assert per_rank < 70e9, per_rank / 1e9


@pytest.mark.parametrize("windows", [0, 2, 3])
def test_gradient_windows_rotate_in_backward_order(model_cfg: ModelConfig, windows: int) -> None:
    from packbalance_b200.parallel.sharded import plan_grad_storage

    cfg = replace(model_cfg, n_layers=5, tie_embeddings=False)
    lay = plan_layout(LlamaForCausalLM(cfg), 4)
    st = plan_grad_storage(lay, 4, windows)
    layers = [u for u in lay.units if u.name.startswith("layer")]
    fixed = [u for u in lay.units if not u.name.startswith("layer")]
    if windows == 0:
        assert st.windows == 0 and all(u.gwin == -1 for u in lay.units)
        assert st.fixed_numel == lay.numel  # every unit keeps its own storage
    else:
        assert st.windows == windows and st.win_numel == max(4 * u.cs for u in layers)
        # backward order (last layer first) cycles through the windows
        assert [u.gwin for u in reversed(layers)] == [i % windows for i in range(len(layers))]
        assert all(u.goff == u.gwin * st.win_numel for u in layers)
    if windows == 0:
        assert all(u.goff == u.unit0 for u in lay.units)  # the layout itself
    else:
        # fixed-buffer units: after the norms, disjoint, in order
        off = lay.rep_n
        for u in fixed:
            assert u.gwin == -1 and u.goff == off
            off += 4 * u.cs
        assert st.fixed_numel == off


def test_8b_gradient_windows_shrink_the_per_rank_footprint() -> None:
    """Config #5 on 8 ranks: three rotating windows instead of a model-size fp32
    gradient buffer."""
    from pathlib import Path

    import torch

    from packbalance_b200.config import load_config
    from packbalance_b200.parallel.sharded import ShardedParameters, plan_grad_storage

    cfg = load_config(Path(__file__).resolve().parents[1] / "configs" / "b5_8b_fsdp.yaml")
    with torch.device("meta"):
        model = LlamaForCausalLM(cfg.model)
    lay = plan_layout(model, 8)
    st = plan_grad_storage(lay, 8, ShardedParameters.GRAD_WINDOWS)
    grad_bytes = 4 * (st.fixed_numel + st.windows * st.win_numel)
    assert grad_bytes < 0.25 * 4 * lay.numel, grad_bytes / 1e9  # vs a full fp32 gradient
    per_rank = 2 * lay.numel + grad_bytes + 16 * lay.shard_numel
    assert per_rank < 40e9, per_rank / 1e9


@pytest.mark.parametrize("windows", [0, 2, 3])
def test_weight_windows_place_layers_in_forward_order(model_cfg: ModelConfig, windows: int) -> None:
    from packbalance_b200.parallel.sharded import plan_weight_storage

    cfg = replace(model_cfg, n_layers=5, tie_embeddings=False)
    lay = plan_layout(LlamaForCausalLM(cfg), 4)
    st = plan_weight_storage(lay, 4, windows)
    layers = [u for u in lay.units if u.name.startswith("layer")]
    fixed = [u for u in lay.units if not u.name.startswith("layer")]
    # units with their own place: disjoint, in order, from 0
    placed = lay.units if windows == 0 else fixed
    off = 0
    for u in placed:
        assert u.wwin == -1 and u.woff == off
        off += 4 * u.cs
    assert st.fixed_numel == off
    if windows == 0:
        assert st.windows == 0 and st.numel == off
    else:
        assert st.windows == windows and st.win_numel == max(4 * u.cs for u in layers)
        # forward order cycles through the windows; every window fits its largest layer
        assert [u.wwin for u in layers] == [i % windows for i in range(len(layers))]
        assert all(u.woff == st.fixed_numel + u.wwin * st.win_numel for u in layers)
        assert st.numel == st.fixed_numel + windows * st.win_numel
    with pytest.raises(ValueError):
        plan_weight_storage(lay, 4, 1)


def test_8b_weight_windows_shrink_the_per_rank_footprint() -> None:
    """Config #5 on 8 ranks with two weight windows: the gathered bf16 weights are the
    embedding, the head and two layers instead of the whole model."""
    from pathlib import Path

    import torch

    from packbalance_b200.config import load_config
    from packbalance_b200.parallel.sharded import ShardedParameters, plan_grad_storage, plan_weight_storage

    cfg = load_config(Path(__file__).resolve().parents[1] / "configs" / "b5_8b_fsdp.yaml")
    with torch.device("meta"):
        model = LlamaForCausalLM(cfg.model)
    lay = plan_layout(model, 8)
    gs = plan_grad_storage(lay, 8, ShardedParameters.GRAD_WINDOWS)
    ws = plan_weight_storage(lay, 8, 2)
    weight_bytes = 2 * ws.numel
    assert weight_bytes < 0.2 * 2 * lay.numel, weight_bytes / 1e9  # vs persistent bf16 weights
    grad_bytes = 4 * (gs.fixed_numel + gs.windows * gs.win_numel)
    per_rank = weight_bytes + grad_bytes + 18 * lay.shard_numel
    assert per_rank < 30e9, per_rank / 1e9  # 41 GB with persistent weights


def test_auto_weight_windows_keeps_small_models_persistent() -> None:
    """fsdp_weight_windows: -1 keeps the gathered bf16 weights while they fit in a quarter
    of the device (1.1B and 8B on a 180 GB B200), else rotates two windows (30B)."""
    from packbalance_b200.parallel.sharded import auto_weight_windows

    b200 = 183_359 * 2**20
    assert auto_weight_windows(1_100_000_000, b200) == 0
    assert auto_weight_windows(8_000_000_000, b200) == 0
    assert auto_weight_windows(30_000_000_000, b200) == 2
    assert auto_weight_windows(8_000_000_000, 40 * 2**30) == 2
