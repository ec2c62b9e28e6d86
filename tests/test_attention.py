import pytest
import torch
import torch.nn.functional as F

from packbalance_b200.config import DataConfig, ModelConfig
from packbalance_b200.data.cost import FlopModel
from packbalance_b200.data.dataset import PackedDataset
from packbalance_b200.data.packer import build_packs
from packbalance_b200.data.store import TokenStore
from packbalance_b200.models.attention import doc_start_from_doc_ids, eager_attention
from packbalance_b200.models.llama import LlamaModel
from packbalance_b200.ops.attention import attention_plan, doc_end_from_start
from packbalance_b200.ops.reference import varlen_attention_reference


def test_eager_attention_matches_dense_mask() -> None:
    torch.manual_seed(0)
    q, k, v = (torch.randn(1, 2, 8, 4) for _ in range(3))
    doc_ids = torch.tensor([[0, 0, 0, 1, 1, 2, 2, 2]])
    mask = (doc_ids == doc_ids.T) & torch.tril(torch.ones(8, 8, dtype=torch.bool))
    ref = F.scaled_dot_product_attention(q, k, v, attn_mask=mask[None, None])
    torch.testing.assert_close(eager_attention(q, k, v, doc_ids), ref, atol=1e-5, rtol=1e-5)


def test_varlen_reference_matches_eager_gqa() -> None:
    torch.manual_seed(0)
    t, h, hk, d = 40, 4, 2, 8
    q, k, v = torch.randn(t, h, d), torch.randn(t, hk, d), torch.randn(t, hk, d)
    doc_ids = torch.tensor([0] * 7 + [1] * 20 + [2] * 13)
    ds = doc_start_from_doc_ids(doc_ids)
    ref = eager_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None], v.transpose(0, 1)[None], doc_ids[None])
    out = varlen_attention_reference(q, k, v, ds)
    torch.testing.assert_close(out, ref[0].transpose(0, 1), atol=1e-5, rtol=1e-5)


def test_packed_model_matches_isolated_documents(
    store: TokenStore, data_cfg: DataConfig, model_cfg: ModelConfig, flop_model: FlopModel
) -> None:
    torch.manual_seed(0)
    pack = next(p for p in build_packs(store, data_cfg, flop_model) if len(p.segments) >= 2)
    item = PackedDataset(store, [pack], data_cfg)[0]
    model = LlamaModel(model_cfg).eval()
    with torch.no_grad():
        packed = model(item["input_ids"][None], item["position_ids"][None], item["doc_ids"][None])
        off = 0
        for seg in pack.segments:
            toks = torch.from_numpy(store.read(seg.start, seg.length))
            iso = model(toks[None], torch.arange(seg.length)[None], torch.zeros(1, seg.length, dtype=torch.long))
            torch.testing.assert_close(packed[0, off : off + seg.length], iso[0], atol=1e-5, rtol=1e-5)
            off += seg.length


def test_doc_start_and_end() -> None:
    ids = torch.tensor([[0, 0, 1, 1, 1, -1], [0, 1, 1, 1, 2, 2]])
    ds = doc_start_from_doc_ids(ids)
    assert ds.tolist() == [0, 0, 2, 2, 2, 5, 6, 7, 7, 7, 10, 10]
    assert doc_end_from_start(ds).tolist() == [1, 1, 4, 4, 4, 5, 6, 9, 9, 9, 11, 11]


def test_attention_plan_orders_by_cost() -> None:
    ds = torch.cat([torch.zeros(1024, dtype=torch.int32), torch.arange(1024, 1024 + 256, dtype=torch.int32)])
    # one CTA: the dealt order is the cost order itself
    plan = attention_plan(ds, n_heads=2, n_kv_heads=1, n_ctas=1)
    fwd = plan["fwd"]
    assert fwd.shape == (10 * 2, 3)
    # The last q tile of the 1024-token document sees 8 key tiles and comes first.
    assert fwd[0].tolist() == [7, 0, 0] and fwd[-1].tolist() == [9, 1, 9]
    bwd = plan["bwd"]
    assert bwd.shape == (10 * 2, 3)
    assert bwd[0].tolist() == [0, 0, 7] and bwd[1].tolist() == [0, 1, 7]


@pytest.mark.parametrize("backend", ["eager", "auto"])
def test_generate_shape(model_cfg: ModelConfig, backend: str) -> None:
    from dataclasses import replace

    from packbalance_b200.models.llama import LlamaForCausalLM

    torch.manual_seed(0)
    model = LlamaForCausalLM(replace(model_cfg, attention_backend=backend))
    out = model.generate(torch.randint(0, model_cfg.vocab_size, (1, 4)), max_new_tokens=4, temperature=0.0)
    assert out.shape == (1, 8)


def test_host_plan_matches_device_plan() -> None:
    """The numpy plan the trainer builds with the batch equals the torch plan."""
    import numpy as np

    from packbalance_b200.ops.attention import attention_plan, attention_plan_host

    rng = np.random.default_rng(3)
    for t in (1000, 1024, 4099):
        lens, tot = [], 0
        while tot < t:
            n = int(min(rng.integers(1, 700), t - tot))
            lens.append(n)
            tot += n
        ds = np.concatenate([np.full(n, s) for n, s in zip(lens, np.cumsum([0] + lens[:-1]))]).astype(np.int32)
        dev = attention_plan(torch.from_numpy(ds), 6, 2)
        host = attention_plan_host(ds, 6)
        for k in ("fwd", "bwd", "doc_start", "doc_end"):
            assert torch.equal(dev[k], host[k]), (t, k)
        if t % 8:
            padded = np.concatenate([ds, np.arange(t, -(-t // 8) * 8)]).astype(np.int32)
            devp = attention_plan(torch.from_numpy(padded), 6, 2)
            for k in ("fwd", "bwd", "doc_start", "doc_end"):
                assert torch.equal(devp[k], host["padded"][k]), (t, k)


def test_plan_deals_every_item_once_and_balances() -> None:
    """The dealt work lists are a permutation of the cost-sorted items, and the busiest
    persistent CTA's cost stays near the mean on a skewed document mix."""
    import numpy as np

    from packbalance_b200.ops.attention import TILE, _deal_order, attention_plan_host

    for n, g in ((768, 148), (100, 148), (1000, 37)):
        d = _deal_order(n, g)
        assert sorted(d.tolist()) == list(range(n))
    rng = np.random.default_rng(0)
    lens = np.clip(rng.lognormal(np.log(256), 1.2, 200).astype(int), 16, 2048)
    ds = np.concatenate([np.full(n, s) for n, s in zip(lens, np.cumsum(np.r_[0, lens[:-1]]))])[:8192]
    plan = attention_plan_host(ds, 12, 148)
    fwd = plan["fwd"].numpy()
    assert len({(int(a), int(b)) for a, b, _ in fwd}) == fwd.shape[0] == (8192 // TILE) * 12
    cost = (fwd[:, 0] - fwd[:, 2] + 1).astype(float)
    loads = np.bincount(np.arange(len(cost)) % 148, weights=cost, minlength=148)
    assert loads.max() / loads.mean() < 1.12


def test_plan_covers_exactly_the_needed_tiles_property() -> None:
    """For random packed layouts (one-token documents, documents crossing tiles, ragged
    ends), every forward item (q tile, head, first kv tile) starts at the kv tile of the
    tile's earliest document start, every backward item (kv tile, head, last q tile)
    ends at the q tile of the kv tile's latest document end, and each (tile, head) pair
    appears exactly once in each list; brute force over the dense mask."""
    import numpy as np
    from hypothesis import given, settings
    from hypothesis import strategies as st

    from packbalance_b200.ops.attention import TILE, attention_plan_host

    @settings(max_examples=40, deadline=None)
    @given(st.lists(st.integers(1, 300), min_size=1, max_size=30), st.integers(1, 4), st.integers(1, 148))
    def check(lengths, heads, ctas):
        ds = np.concatenate([np.full(n, s) for n, s in zip(lengths, np.cumsum([0] + lengths[:-1]))]).astype(np.int64)
        t = ds.size
        nt = -(-t // TILE)
        plan = attention_plan_host(ds, heads, ctas)
        fwd, bwd = plan["fwd"].numpy(), plan["bwd"].numpy()
        assert sorted((int(a), int(b)) for a, b, _ in fwd) == [(i, h) for i in range(nt) for h in range(heads)]
        assert sorted((int(a), int(b)) for a, b, _ in bwd) == [(i, h) for i in range(nt) for h in range(heads)]
        q = np.arange(t)
        allowed = (q[None, :] >= ds[:, None]) & (q[None, :] <= q[:, None])  # [query, key]
        for qt, _, kt0 in fwd:
            rows = allowed[qt * TILE : (qt + 1) * TILE]
            need = np.nonzero(rows.any(axis=0))[0] // TILE
            assert kt0 == need.min() and need.max() <= qt
        for kt, _, qhi in bwd:
            cols = allowed[:, kt * TILE : (kt + 1) * TILE]
            need = np.nonzero(cols.any(axis=1))[0] // TILE
            assert qhi == need.max() and need.min() >= kt

    check()
