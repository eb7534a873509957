"""The Laguna router family in the oracle: the reference's own hermetic tests
(crates/model-serving/tests/laguna_hermetic/routing.rs) ported as data, plus
the exp-based sigmoid and tanh the router uses."""
import math

import numpy as np
import pytest

from oracle import oracle as O


def sig(x):
    return 1.0 / (1.0 + math.exp(-x))


def route(logits, K, bias=None, softcap=0.0, normalize=False):
    return O.route_laguna_experts(np.asarray([logits], np.float32), K, correction_bias=bias,
                                  softcap=softcap, normalize=normalize)


def test_correction_bias_selects_but_original_scores_are_gathered():
    # routing.rs:9-21: expert 0 wins only through its bias; its weight stays 0.5
    ids, sc = route([0.0, 2.0, -2.0, 0.5], 2, bias=np.array([2.0, 0, 0, 0], np.float32))
    assert ids.tolist() == [[0, 1]]
    assert abs(sc[0, 0] - sig(0.0)) < 1e-6 and abs(sc[0, 1] - sig(2.0)) < 1e-6


def test_equal_selection_scores_break_toward_the_lower_id():
    ids, _ = route([0.0, 0.0, -4.0], 1)  # routing.rs:23-29
    assert ids.tolist() == [[0]]


def test_softcap_applies_before_sigmoid():
    # routing.rs:31-43: 2 * tanh(30 / 2) caps the logit
    assert abs(O.lib().ao_tanhf(15.0) * 2.0 - 2.0 * math.tanh(15.0)) < 1e-6
    _, raw = route([30.0, 0.0], 1)
    _, capped = route([30.0, 0.0], 1, softcap=2.0)
    assert raw[0, 0] > capped[0, 0]
    assert abs(capped[0, 0] - sig(2.0 * math.tanh(15.0))) < 1e-6


def test_normalisation_of_the_selected_scores():
    _, raw = route([1.0, 0.0, -1.0], 2)  # routing.rs:45-56
    _, nrm = route([1.0, 0.0, -1.0], 2, normalize=True)
    assert abs(float(nrm.sum()) - 1.0) < 1e-6
    assert abs(nrm[0, 0] - raw[0, 0] / raw.sum()) < 1e-6


def test_invalid_geometry_is_rejected():
    with pytest.raises(ValueError):
        route([0.0, 0.0], 3)  # top-K above the router dimension (routing.rs:58-63)
    with pytest.raises(ValueError):
        route([0.0, 0.0], 1, softcap=-1.0)


def test_exp_based_sigmoid_and_tanh_are_accurate():
    lib = O.lib()
    for x in np.linspace(-20, 20, 801):
        x = float(np.float32(x))
        assert abs(lib.ao_sigmoid_plainf(x) - sig(x)) <= 2e-7 * max(sig(x), 1e-30) + 1e-12
        assert abs(lib.ao_tanhf(x) - math.tanh(x)) <= 4e-7


def test_laguna_block_runs_on_the_oracle():
    from astronomical_b200 import synthetic

    cfg = dict(synthetic.LAGUNA)
    w = synthetic.make_block_weights(cfg, seed=3)
    x = synthetic.make_hidden_states(12, cfg["hidden"], seed=4)
    y, ids, sc = O.moe_block_forward(w, x)
    assert sc.dtype == np.float32 and np.allclose(sc.sum(1), 1.0, atol=1e-6)
    # the bias only ranks: the selected experts are the top-K of sigmoid + bias
    logits = O.matmul_bf16_nt(x, w["router_w"])
    ids2, sc2 = O.route_laguna_experts(logits, cfg["top_k"], w["router_correction_bias"])
    assert np.array_equal(ids, ids2) and np.array_equal(sc, sc2)
