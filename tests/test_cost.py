import numpy as np

from packbalance_b200.data.cost import FlopModel, cost_stats


def test_cost_model_properties(flop_model: FlopModel) -> None:
    assert flop_model.head_dim == 8
    assert flop_model.d_kv == 16
    assert flop_model.linear_params > 0
    assert flop_model.total_params >= flop_model.linear_params
    assert flop_model.attention_flops_coeff > 0


def test_attention_cost_is_quadratic(flop_model: FlopModel) -> None:
    one = flop_model.pack_cost([256])
    two = flop_model.pack_cost([128, 128])
    assert one > two
    assert np.isclose(one - two, flop_model.attention_flops_coeff * (256**2 - 2 * 128**2))


def test_padded_cost_exceeds_packed(flop_model: FlopModel) -> None:
    assert flop_model.padded_batch_cost([32] * 4, pad_len=64) > flop_model.pack_cost([32] * 4)


def test_doc_cost_vectorised(flop_model: FlopModel) -> None:
    lens = np.array([5, 17, 64])
    np.testing.assert_allclose(flop_model.doc_cost(lens), [flop_model.pack_cost([n]) for n in lens])


def test_cost_stats() -> None:
    s = cost_stats([1.0, 2.0, 3.0])
    assert s["mean"] == 2.0 and s["max"] == 3.0 and s["cv"] > 0
    assert cost_stats([])["mean"] == 0.0
