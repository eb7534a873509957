"""Known-answer tests of the reference, ported as data and run against the CPU
oracle.  Each test names the reference test it restates (paths relative to the
reference project root).  These pin the oracle before it is trusted as the
checker for the CUDA path."""
import math

import numpy as np
import pytest

from oracle import oracle as O
from astronomical_b200.synthetic import bf16_to_f32, f32_to_bf16, pack_affine, unpack_affine


def close(actual, expected, tol):
    actual = np.asarray(actual, np.float64).ravel()
    expected = np.asarray(expected, np.float64).ravel()
    assert actual.shape == expected.shape
    scale = np.maximum(np.abs(expected), 1.0)
    assert np.all(np.abs(actual - expected) <= tol * scale), (actual, expected)


# crates/model-serving/tests/direct_mlx/qwen3_5_moe/routing_and_combination.rs:12-68
def test_route_normalize_and_combine_selected_and_shared_experts():
    logits = np.array([[0.0, math.log(2.0), math.log(3.0), math.log(4.0)]], np.float32)
    ids, scores = O.route_experts(logits, top_k=2, normalize=True)
    close(np.sort(scores.ravel()), [3.0 / 7.0, 4.0 / 7.0], 1e-6)
    expert_outputs = np.array([[0, 0], [0, 0], [7, 14], [14, 21]], np.float32)
    selected = expert_outputs[ids[0]][None]  # [T=1, K=2, D=2]
    sparse = O.unsorted_expert_weighted_sum(selected, scores)
    combined = O.combine_sparse_and_shared(sparse, np.array([[2.0, 4.0]], np.float32),
                                           np.array([[0.0]], np.float32))
    close(combined, [12.0, 20.0], 1e-6)


# routing_and_combination.rs:70-107 and direct_mlx/sparse_experts.rs:33-64
def test_bf16_expert_outputs_with_f32_scores_keep_bf16():
    outs = f32_to_bf16(np.array([[[2.0, 4.0], [6.0, 8.0]]], np.float32))
    scores = np.array([[0.25, 0.75]], np.float32)
    red = O.unsorted_expert_weighted_sum(outs, scores)
    assert red.dtype == np.uint16  # bf16 result
    close(bf16_to_f32(red), [5.0, 7.0], 1e-5)


# routing_and_combination.rs:109-182
def test_sort_expert_assignments_and_restore_order():
    x = np.array([[10.0, 11.0], [20.0, 21.0]], np.float32)
    ids = np.array([[5, 0, 4], [1, 3, 2]], np.uint32)
    s = O.sort_expert_assignments(ids, experts=6)
    sorted_states = x[s["sorted_tokens"]]
    close(sorted_states, [10, 11, 20, 21, 20, 21, 20, 21, 10, 11, 10, 11], 1e-6)
    assert s["sorted_ids"].tolist() == [0, 1, 2, 3, 4, 5]
    assert s["inverse_order"].tolist() == [5, 0, 4, 1, 3, 2]
    assert s["sorted_order"].tolist() == [1, 3, 5, 4, 2, 0]
    assert s["expert_offsets"].tolist() == [0, 1, 2, 3, 4, 5, 6]
    sorted_outputs = np.array([[100, 101], [110, 111], [120, 121], [130, 131], [140, 141],
                               [150, 151]], np.float32)
    restored = sorted_outputs[s["inverse_order"]]
    close(restored, [150, 151, 100, 101, 140, 141, 110, 111, 130, 131, 120, 121], 1e-6)


# routing_and_combination.rs:184-228; direct_mlx/sparse_experts.rs:87-173
def test_sorted_weighted_sum_without_restoring():
    sorted_outputs = np.array([[100, 101], [110, 111], [120, 121], [130, 131], [140, 141],
                               [150, 151]], np.float32)
    inverse = np.array([5, 0, 4, 1, 3, 2], np.uint32)
    scores = np.array([[0.1, 0.2, 0.7], [0.25, 0.25, 0.5]], np.float32)
    out = O.sorted_expert_weighted_sum(sorted_outputs, inverse, scores)
    close(out, [133.0, 134.0, 120.0, 121.0], 1e-5)
    restored = sorted_outputs[inverse].reshape(2, 3, 2)
    close(O.unsorted_expert_weighted_sum(restored, scores), [133.0, 134.0, 120.0, 121.0], 1e-5)
    # bf16 outputs (values are exact in bf16) give the same answer
    out16 = O.sorted_expert_weighted_sum(f32_to_bf16(sorted_outputs), inverse, scores)
    close(bf16_to_f32(out16), [133.0, 134.0, 120.0, 121.0], 1e-5)


# crates/runtime-integration/tests/direct_mlx/quantized_operations.rs:5-61, :63-124, :126-160
def test_affine_qmm_known_answers():
    x = f32_to_bf16(np.arange(1, 65, dtype=np.float32)[None])
    w4 = np.array([[0x11111111] * 8, [0x22222222] * 8], np.uint32)
    one, zero = f32_to_bf16(np.ones((2, 1))), f32_to_bf16(np.zeros((2, 1)))
    y = O.gather_qmm(x, w4, one, zero, group=64, bits=4)
    assert bf16_to_f32(y).tolist() == [[2080.0, 4160.0]]
    w8 = np.array([[0x01010101] * 16, [0x02020202] * 16], np.uint32)
    y = O.gather_qmm(x, w8, one, zero, group=64, bits=8)
    assert bf16_to_f32(y).tolist() == [[2080.0, 4160.0]]
    ones = f32_to_bf16(np.ones((1, 64)))
    w5 = np.zeros((2, 10), np.uint32)
    y = O.gather_qmm(ones, w5, f32_to_bf16(np.ones((2, 2))), f32_to_bf16(np.zeros((2, 2))),
                     group=32, bits=5)
    assert bf16_to_f32(y).tolist() == [[0.0, 0.0]]


# quantized_operations.rs:255-306
def test_gather_qmm_selected_experts_known_answer():
    x = f32_to_bf16(np.arange(1, 65, dtype=np.float32)[None])
    words = []
    for v in (0x11111111, 0x22222222, 0x55555555, 0x66666666, 0x33333333, 0x44444444):
        words += [v] * 8
    packed = np.array(words, np.uint32).reshape(3, 2, 8)
    one, zero = f32_to_bf16(np.ones((3, 2, 1))), f32_to_bf16(np.zeros((3, 2, 1)))
    y = O.gather_qmm(x, packed, one, zero, group=64, bits=4, rhs_experts=[2, 0], lhs_rows=[0, 0])
    assert bf16_to_f32(y).ravel().tolist() == [6240.0, 8320.0, 2080.0, 4160.0]


def simple_affine_quantize(w: np.ndarray, group: int, bits: int):
    """Affine quantiser for fixtures: per group scale=(max-min)/(2^b-1), bias=min.
    (The reference asks MLX's quantize; which quantiser made the codes does not
    matter to the qmm-versus-dequantise comparison below.)"""
    rows, in_f = w.shape[:-1], w.shape[-1]
    g = w.reshape(rows + (in_f // group, group)).astype(np.float64)
    lo, hi = g.min(-1, keepdims=True), g.max(-1, keepdims=True)
    n_bins = 2**bits - 1
    scale = np.maximum((hi - lo) / n_bins, 1e-7)
    s16 = f32_to_bf16(scale[..., 0])
    b16 = f32_to_bf16(lo[..., 0])
    q = np.clip(np.rint((g - bf16_to_f32(b16)[..., None]) / bf16_to_f32(s16)[..., None]), 0,
                n_bins).astype(np.uint32).reshape(rows + (in_f,))
    return pack_affine(q, bits), s16, b16


def dense_matmul_bf16(x, w):
    """x [n, in] bf16 bits, w [out, in] bf16 bits -> fp32-accumulated bf16 (oracle matmul)."""
    return O.matmul_bf16_nt(x, w)


# crates/model-serving/tests/direct_mlx/sparse_expert_projection.rs:233-338
@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
def test_gather_qmm_matches_dequantized_reference(group, bits):
    E, out_f = 3, 2
    idx = np.arange(E * out_f * group)
    src = (idx // (out_f * group)) * 0.2 + ((idx % 13) - 6.0) * 0.03
    src = src.reshape(E, out_f, group)
    packed, s, b = simple_affine_quantize(src, group, bits)
    a_idx = np.arange(E * group)
    x = f32_to_bf16((0.1 + (a_idx % 17) * 0.015).reshape(E, group))
    sel = [0, 1, 2] if bits % 2 == 0 else [2, 0, 1]
    y = O.gather_qmm(x, packed, s, b, group, bits, rhs_experts=sel, lhs_rows=[0, 1, 2])
    deq = O.dequantize_affine(packed, s, b, group, bits)  # [E, out, in] bf16
    ref = np.stack([dense_matmul_bf16(x[i:i + 1], deq[sel[i]])[0] for i in range(E)])
    close(bf16_to_f32(y), bf16_to_f32(ref), 3e-3)


# quantized_operations.rs:174-253 (2-bit, g64, out=67 "slow" qmv width)
def test_bf16_affine_qmv_odd_output_width():
    in_f, out_f = 256, 67
    x = f32_to_bf16((0.02 * (np.arange(in_f) % 13 + 1))[None])
    src = (0.05 * ((np.arange(out_f * in_f) % 17) - 8.0)).reshape(out_f, in_f)
    packed, s, b = simple_affine_quantize(src, 64, 2)
    y = O.gather_qmm(x, packed, s, b, 64, 2)
    ref = dense_matmul_bf16(x, O.dequantize_affine(packed, s, b, 64, 2))
    assert np.max(np.abs(bf16_to_f32(y) - bf16_to_f32(ref))) <= 2e-2


# sparse_expert_projection.rs:55-230 (sorted vs original order, affine storage)
@pytest.mark.parametrize("E,T,K,out_f", [(1, 1, 1, 3), (3, 2, 2, 5), (5, 3, 4, 7)])
def test_sorted_and_unsorted_paths_agree(E, T, K, out_f):
    in_f = 64
    rng = np.random.default_rng(E * 100 + T)
    src = ((np.arange(E * out_f * in_f) % 11) - 5.0).reshape(E, out_f, in_f) * 0.0625
    packed, s, b = simple_affine_quantize(src, 64, 4)
    x = f32_to_bf16((0.25 + np.arange(T * in_f) * 0.125 / 16).reshape(T, in_f))
    ids = ((np.arange(T * K) * 2 + 1) % E).astype(np.uint32).reshape(T, K)
    unsorted = O.gather_qmm(x, packed, s, b, 64, 4, rhs_experts=ids.ravel(),
                            lhs_rows=np.repeat(np.arange(T), K))
    st = O.sort_expert_assignments(ids, E)
    sorted_out = O.gather_qmm(x, packed, s, b, 64, 4, rhs_experts=st["sorted_ids"],
                              lhs_rows=st["sorted_tokens"])
    assert np.array_equal(sorted_out[st["inverse_order"]], unsorted)
    scores = f32_to_bf16(np.full((T, K), 1.0 / K, np.float32))
    a = O.sorted_expert_weighted_sum(sorted_out, st["inverse_order"], scores)
    u = O.unsorted_expert_weighted_sum(unsorted.reshape(T, K, out_f), scores)
    close(bf16_to_f32(a), bf16_to_f32(u), 2e-2)
    del rng


# sparse_experts.rs:176-237; sparse_expert_projection.rs:340-388
def test_empty_assignment_sets():
    s = O.sort_expert_assignments(np.zeros((1, 0), np.uint32), experts=4)
    assert s["sorted_ids"].size == 0 and s["expert_offsets"].tolist() == [0] * 5
    red = O.unsorted_expert_weighted_sum(np.zeros((1, 0, 2), np.float32),
                                         np.zeros((1, 0), np.float32))
    assert red.tolist() == [[0.0, 0.0]]
    src = np.full((2, 2, 32), 0.25)
    packed, sc, bi = simple_affine_quantize(src, 32, 4)
    y = O.gather_qmm(np.zeros((0, 32), np.uint16), packed, sc, bi, 32, 4,
                     rhs_experts=np.zeros(0, np.uint32), lhs_rows=np.zeros(0, np.uint32))
    assert y.shape == (0, 2)


# crates/model-serving/tests/hermetic/sparse_experts.rs:5-36
def test_invert_assignment_order():
    st, inv = O.invert_assignment_order([1, 3, 5, 4, 2, 0])
    assert st == O.OK and inv.tolist() == [5, 0, 4, 1, 3, 2]
    st, inv = O.invert_assignment_order(np.zeros(0, np.uint32))
    assert st == O.OK and inv.size == 0
    assert O.invert_assignment_order([0, 0])[0] == O.ERR_DUPLICATE_SLOT
    assert O.invert_assignment_order([0, 2])[0] == O.ERR_OUT_OF_RANGE_SLOT


# crates/runtime-integration/tests/direct_mlx/compiled_swiglu.rs:5-52
def test_swiglu_matches_silu_times_input():
    for g, u in (([-1.0, 0.0, 1.0, 0.5], [2.0, 3.0, 4.0, 5.0]),
                 ([2.0, -2.0, 0.5, -0.5, 1.5, -1.5, 0.25, -0.25, 3.0, -3.0],
                  [1.0, 2.0, 3.0, 4.0, 0.5, 1.5, 2.5, 3.5, 0.75, 1.25])):
        gb, ub = f32_to_bf16(g), f32_to_bf16(u)
        out = bf16_to_f32(O.swiglu(gb, ub))
        gf, uf = bf16_to_f32(gb).astype(np.float64), bf16_to_f32(ub).astype(np.float64)
        silu = gf / (1.0 + np.exp(-gf))
        close(out, silu * uf, 1e-2)


# crates/model-serving/tests/direct_mlx/qwen3_5_moe/resident_gate_up_fusion.rs:14-255
def test_fused_gate_up_equals_separate():
    rng = np.random.default_rng(3)
    E, I, H = 4, 16, 128
    gq = rng.integers(0, 2**32, size=(E, I, H // 8), dtype=np.uint64).astype(np.uint32)
    uq = rng.integers(0, 2**32, size=(E, I, H // 8), dtype=np.uint64).astype(np.uint32)
    gs = f32_to_bf16(np.abs(rng.normal(0, 0.01, (E, I, H // 64))))
    us = f32_to_bf16(np.abs(rng.normal(0, 0.01, (E, I, H // 64))))
    gb, ub = f32_to_bf16(-8 * bf16_to_f32(gs)), f32_to_bf16(-8 * bf16_to_f32(us))
    x = f32_to_bf16(rng.normal(0, 1, (5, H)))
    sel = np.array([3, 1, 0, 3, 2], np.uint32)
    fused = O.gather_qmm(x, np.concatenate([gq, uq], 1), np.concatenate([gs, us], 1),
                         np.concatenate([gb, ub], 1), 64, 4, rhs_experts=sel, lhs_rows=np.arange(5))
    g = O.gather_qmm(x, gq, gs, gb, 64, 4, rhs_experts=sel, lhs_rows=np.arange(5))
    u = O.gather_qmm(x, uq, us, ub, 64, 4, rhs_experts=sel, lhs_rows=np.arange(5))
    assert np.array_equal(fused[:, :I], g) and np.array_equal(fused[:, I:], u)


def test_pack_unpack_roundtrip_all_bits():
    rng = np.random.default_rng(0)
    for bits in (2, 3, 4, 5, 6, 8):
        q = rng.integers(0, 2**bits, size=(3, 64))
        assert np.array_equal(unpack_affine(pack_affine(q, bits), bits), q)


def test_expf_accuracy_and_special_values():
    x = np.linspace(-87.0, 88.0, 200001, dtype=np.float32)
    got = O.expf(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    rel = np.abs(got - ref) / ref
    assert rel.max() < 2.5e-7  # within ~2 ulp of fp32
    sp = O.expf(np.array([0.0, -100.0, 100.0, -np.inf], np.float32))
    assert sp[0] == 1.0 and sp[1] == 0.0 and np.isinf(sp[2]) and sp[3] == 0.0


def test_route_tie_policy_prefers_lower_expert_id():
    # equal bf16 probabilities: the canonical order picks the lower id first
    logits = f32_to_bf16(np.zeros((2, 8), np.float32))
    ids, scores = O.route_experts(logits, top_k=3)
    assert ids.tolist() == [[0, 1, 2], [0, 1, 2]]
    close(bf16_to_f32(scores), np.full(6, 1.0 / 3.0), 4e-3)
