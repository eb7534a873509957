"""Parity of every stage of the CUDA path against the CPU oracle, through the C ABI.

Integer and elementwise stages (routing ids/scores, sort, SwiGLU, weighted sums,
combination) must be bit-exact; the gathered projections must agree to one bf16
ulp (the only difference is the fp32 accumulation order)."""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O  # noqa: E402
from astronomical_b200 import moe  # noqa: E402
from astronomical_b200._lib import AstroMoeError  # noqa: E402
from astronomical_b200.synthetic import bf16_to_f32, f32_to_bf16  # noqa: E402
from tests.helpers import (assert_bf16_ulps, bf16_tensor, to_np_bf16, to_np_u32,  # noqa: E402
                           u32_tensor)

pytestmark = pytest.mark.gpu


def _logits(T, E, seed, kind):
    rng = np.random.default_rng(seed)
    if kind == "normal":
        return rng.normal(0, 1, (T, E)).astype(np.float32)
    if kind == "ties":  # few distinct values: many exact ties at the K boundary
        return (rng.integers(0, 4, (T, E)) * 0.25).astype(np.float32)
    if kind == "router":  # the block's own scale: N(0,1) x N(0,0.02) over 2048
        return rng.normal(0, 0.9, (T, E)).astype(np.float32)
    raise ValueError(kind)


@pytest.mark.parametrize("T,E,K", [(4096, 256, 8), (513, 128, 8), (77, 160, 10), (5, 4, 2),
                                   (64, 1024, 32), (3, 1, 1)])
@pytest.mark.parametrize("kind", ["normal", "ties", "router"])
@pytest.mark.parametrize("normalize", [True, False])
def test_route_bf16_bit_exact(T, E, K, kind, normalize):
    lg = f32_to_bf16(_logits(T, E, T * 7 + E, kind))
    ids_o, sc_o = O.route_experts(lg, K, normalize)
    ids, sc = moe.qwen3_5_moe_route_experts(bf16_tensor(lg), K, normalize)
    torch.cuda.synchronize()
    assert np.array_equal(to_np_u32(ids), ids_o)
    assert np.array_equal(to_np_bf16(sc), sc_o)


@pytest.mark.parametrize("dt", [np.float32, np.float16])
def test_route_f32_f16_bit_exact(dt):
    lg = _logits(1000, 256, 3, "normal").astype(dt)
    ids_o, sc_o = O.route_experts(lg, 8, True)
    ids, sc = moe.qwen3_5_moe_route_experts(torch.from_numpy(lg).cuda(), 8, True)
    assert np.array_equal(to_np_u32(ids), ids_o)
    assert np.array_equal(sc.cpu().numpy(), sc_o)


def test_route_known_answer():
    # routing_and_combination.rs:12-68
    lg = torch.tensor([[0.0, math.log(2.0), math.log(3.0), math.log(4.0)]], device="cuda")
    ids, sc = moe.qwen3_5_moe_route_experts(lg, 2, True)
    assert ids.cpu().tolist() == [[3, 2]]
    got = sorted(sc.cpu().tolist()[0])
    assert abs(got[0] - 3 / 7) <= 1e-6 and abs(got[1] - 4 / 7) <= 1e-6


@pytest.mark.parametrize("T,E,K", [(4096, 256, 8), (77, 160, 10), (5, 4, 2), (64, 1024, 32)])
@pytest.mark.parametrize("kind", ["normal", "ties", "router"])
@pytest.mark.parametrize("bias,softcap,normalize", [(False, 0.0, True), (True, 0.0, True),
                                                    (True, 2.5, False), (False, 1.0, True)])
def test_route_laguna_bit_exact(T, E, K, kind, bias, softcap, normalize):
    # laguna/moe/router.rs:11-60 against the oracle's restatement of the CPU owner
    lg = f32_to_bf16(_logits(T, E, T * 11 + E, kind))
    b = np.random.default_rng(E).normal(0, 0.05, E).astype(np.float32) if bias else None
    ids_o, sc_o = O.route_laguna_experts(lg, K, b, softcap, normalize)
    ids, sc = moe.route_laguna_experts(bf16_tensor(lg), K,
                                       None if b is None else torch.from_numpy(b).cuda(),
                                       softcap, normalize)
    torch.cuda.synchronize()
    assert np.array_equal(to_np_u32(ids), ids_o)
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), sc_o.view(np.uint32))


def test_route_laguna_known_answers():
    # laguna_hermetic/routing.rs:9-56
    lg = torch.tensor([[0.0, 2.0, -2.0, 0.5]], device="cuda")
    ids, sc = moe.route_laguna_experts(lg, 2, torch.tensor([2.0, 0, 0, 0], device="cuda"),
                                       normalize=False)
    assert ids.cpu().tolist() == [[0, 1]]
    assert abs(sc[0, 0].item() - 0.5) < 1e-6 and abs(sc[0, 1].item() - 1 / (1 + math.exp(-2))) < 1e-6
    ids, _ = moe.route_laguna_experts(torch.tensor([[0.0, 0.0, -4.0]], device="cuda"), 1)
    assert ids.cpu().tolist() == [[0]]
    _, nrm = moe.route_laguna_experts(torch.tensor([[1.0, 0.0, -1.0]], device="cuda"), 2)
    assert abs(nrm.sum().item() - 1.0) < 1e-6
    with pytest.raises(AstroMoeError):
        moe.route_laguna_experts(torch.zeros((1, 2), device="cuda"), 3)


def test_route_rejects_bad_arguments():
    lg = torch.zeros((2, 4), device="cuda")
    with pytest.raises(AstroMoeError):
        moe.qwen3_5_moe_route_experts(lg, 5, True)
    with pytest.raises(AstroMoeError):
        moe.qwen3_5_moe_route_experts(torch.zeros(4, device="cuda"), 2, True)


@pytest.mark.parametrize("T,K,E,skew", [(4096, 8, 256, 0.0), (4096, 8, 256, 3.0), (16, 8, 256, 0.0),
                                        (1, 8, 256, 0.0), (1000, 10, 1024, 1.0), (7, 3, 5, 0.0),
                                        (16384, 8, 256, 0.0)])
def test_sort_bit_exact(T, K, E, skew):
    rng = np.random.default_rng(T + K + E)
    p = np.exp(-skew * np.arange(E) / E)
    p /= p.sum()
    ids = rng.choice(E, size=(T, K), p=p).astype(np.uint32)
    ref = O.sort_expert_assignments(ids, E)
    x = torch.zeros((T, 8), dtype=torch.bfloat16, device="cuda")
    got = moe.sort_expert_assignments(x, u32_tensor(ids), experts=E)
    torch.cuda.synchronize()
    assert np.array_equal(to_np_u32(got.sorted_order), ref["sorted_order"])
    assert np.array_equal(to_np_u32(got.inverse_order), ref["inverse_order"])
    assert np.array_equal(to_np_u32(got.sorted_indices), ref["sorted_ids"])
    assert np.array_equal(to_np_u32(got.expert_offsets), ref["expert_offsets"])


def test_sort_known_answer_and_states():
    # routing_and_combination.rs:109-182
    x8 = torch.zeros((2, 8), dtype=torch.bfloat16, device="cuda")
    x8[0, 0], x8[0, 1], x8[1, 0], x8[1, 1] = 10, 11, 20, 21
    ids = u32_tensor(np.array([[5, 0, 4], [1, 3, 2]], np.uint32))
    s = moe.sort_expert_assignments(x8, ids, experts=6)
    assert to_np_u32(s.sorted_indices).tolist() == [0, 1, 2, 3, 4, 5]
    assert to_np_u32(s.inverse_order).tolist() == [5, 0, 4, 1, 3, 2]
    st = bf16_to_f32(to_np_bf16(s.sorted_states[:, 0, :2])).ravel().tolist()
    assert st == [10, 11, 20, 21, 20, 21, 20, 21, 10, 11, 10, 11]
    outs = torch.tensor([[100, 101], [110, 111], [120, 121], [130, 131], [140, 141], [150, 151]],
                        dtype=torch.float32, device="cuda").reshape(6, 1, 2)
    restored = moe.restore_expert_assignment_order(outs, s.inverse_order, [1, 2, 3])
    assert restored.reshape(-1).tolist() == [150, 151, 100, 101, 140, 141, 110, 111, 130, 131,
                                             120, 121]


def test_sort_empty_and_invalid_ids():
    x = torch.zeros((1, 8), dtype=torch.bfloat16, device="cuda")
    s = moe.sort_expert_assignments(x, torch.zeros((1, 0), dtype=torch.int32, device="cuda"),
                                    experts=4)
    assert s.sorted_states.shape == (0, 1, 8)
    moe.device_status(0, reset=True)
    ids = u32_tensor(np.array([[1, 7]], np.uint32))  # 7 >= E: recorded, skipped
    moe.sort_expert_assignments(torch.zeros((1, 8), dtype=torch.bfloat16, device="cuda"), ids,
                                experts=4)
    assert moe.device_status(0, reset=True) & 1


def _qweights(rng, E, out_f, in_f, bits):
    words = in_f * bits // 32
    if bits in (2, 4, 8):
        q = rng.integers(0, 2**32, size=(E, out_f, words), dtype=np.uint64).astype(np.uint32)
    else:
        from astronomical_b200.synthetic import pack_affine
        q = pack_affine(rng.integers(0, 2**bits, size=(E, out_f, in_f)), bits)
    return q


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("sorted_flag", [True, False])
def test_gather_qmm_matches_oracle(bits, group, sorted_flag):
    rng = np.random.default_rng(bits * 10 + group)
    E, out_f, in_f, n = 5, 96, 256, 37
    q = _qweights(rng, E, out_f, in_f, bits)
    s = f32_to_bf16(np.abs(rng.normal(0, 0.01, (E, out_f, in_f // group))))
    b = f32_to_bf16(-(2 ** (bits - 1)) * bf16_to_f32(s))
    x = f32_to_bf16(rng.normal(0, 1, (11, in_f)))
    rhs = rng.integers(0, E, n).astype(np.uint32)
    if sorted_flag:
        rhs = np.sort(rhs)
    lhs = rng.integers(0, 11, n).astype(np.uint32)
    ref = O.gather_qmm(x, q, s, b, group, bits, rhs_experts=rhs, lhs_rows=lhs)
    proj = moe.AffineProjection(u32_tensor(q), bf16_tensor(s), bf16_tensor(b), group, bits)
    order = (moe.ExpertAssignmentOrder.SORTED_BY_EXPERT if sorted_flag
             else moe.ExpertAssignmentOrder.ORIGINAL)
    got = moe.gather_expert_projection(bf16_tensor(x), proj, u32_tensor(rhs), order,
                                       lhs_indices=u32_tensor(lhs))
    torch.cuda.synchronize()
    assert_bf16_ulps(to_np_bf16(got), ref, ulps=1.0, max_frac=0.05)


def test_qmm_and_gather_known_answers():
    # quantized_operations.rs:5-61 and :255-306
    x = bf16_tensor(f32_to_bf16(np.arange(1, 65, dtype=np.float32)[None]))
    w4 = u32_tensor(np.array([[0x11111111] * 8, [0x22222222] * 8], np.uint32))
    one = bf16_tensor(f32_to_bf16(np.ones((2, 1))))
    zero = bf16_tensor(f32_to_bf16(np.zeros((2, 1))))
    y = moe.gather_expert_projection(x, moe.AffineProjection(w4, one, zero, 64, 4), None,
                                     moe.ExpertAssignmentOrder.ORIGINAL)
    assert y.float().cpu().tolist() == [[2080.0, 4160.0]]
    words = []
    for v in (0x11111111, 0x22222222, 0x55555555, 0x66666666, 0x33333333, 0x44444444):
        words += [v] * 8
    packed = u32_tensor(np.array(words, np.uint32).reshape(3, 2, 8))
    one3 = bf16_tensor(f32_to_bf16(np.ones((3, 2, 1))))
    zero3 = bf16_tensor(f32_to_bf16(np.zeros((3, 2, 1))))
    y = moe.gather_expert_projection(x, moe.AffineProjection(packed, one3, zero3, 64, 4),
                                     u32_tensor(np.array([2, 0], np.uint32)),
                                     moe.ExpertAssignmentOrder.ORIGINAL,
                                     lhs_indices=u32_tensor(np.array([0, 0], np.uint32)))
    assert y.float().cpu().ravel().tolist() == [6240.0, 8320.0, 2080.0, 4160.0]


def test_swiglu_bit_exact():
    rng = np.random.default_rng(5)
    g = f32_to_bf16(rng.normal(0, 3, 100000))
    u = f32_to_bf16(rng.normal(0, 3, 100000))
    got = moe.apply_compiled_swiglu(bf16_tensor(g), bf16_tensor(u))
    assert np.array_equal(to_np_bf16(got), O.swiglu(g, u))


@pytest.mark.parametrize("odt,sdt", [("bf16", "bf16"), ("bf16", "f32"), ("f32", "f32"),
                                     ("f32", "bf16"), ("f16", "f16")])
def test_weighted_sums_bit_exact(odt, sdt):
    rng = np.random.default_rng(9)
    T, K, D = 300, 8, 136
    conv = {"bf16": (lambda a: f32_to_bf16(a), lambda a: bf16_tensor(a)),
            "f32": (lambda a: a.astype(np.float32), lambda a: torch.from_numpy(a).cuda()),
            "f16": (lambda a: a.astype(np.float16), lambda a: torch.from_numpy(a).cuda())}
    outs = conv[odt][0](rng.normal(0, 1, (T * K, D)).astype(np.float32))
    scores = conv[sdt][0](rng.random((T, K)).astype(np.float32))
    inv = rng.permutation(T * K).astype(np.uint32)
    ref = O.sorted_expert_weighted_sum(outs, inv, scores)
    got = moe.sorted_expert_weighted_sum(conv[odt][1](outs), u32_tensor(inv), conv[sdt][1](scores))
    g = to_np_bf16(got) if odt == "bf16" else got.cpu().numpy()
    assert np.array_equal(g, ref)
    ref_u = O.unsorted_expert_weighted_sum(outs.reshape(T, K, D), scores)
    got_u = moe.unsorted_expert_weighted_sum(conv[odt][1](outs).reshape(T, K, D),
                                             conv[sdt][1](scores))
    gu = to_np_bf16(got_u) if odt == "bf16" else got_u.cpu().numpy()
    assert np.array_equal(gu, ref_u)


def test_weighted_sum_known_answer():
    # routing_and_combination.rs:184-228
    outs = torch.tensor([[100, 101], [110, 111], [120, 121], [130, 131], [140, 141], [150, 151]],
                        dtype=torch.float32, device="cuda").reshape(6, 1, 2)
    inv = u32_tensor(np.array([5, 0, 4, 1, 3, 2], np.uint32))
    sc = torch.tensor([[0.1, 0.2, 0.7], [0.25, 0.25, 0.5]], device="cuda")
    got = moe.sorted_expert_weighted_sum(outs, inv, sc).cpu().ravel().tolist()
    assert all(abs(a - b) <= 1e-5 * max(1, abs(b)) for a, b in zip(got, [133, 134, 120, 121]))


def test_combine_bit_exact_and_known_answer():
    rng = np.random.default_rng(2)
    T, D = 100, 64
    sp, sh = f32_to_bf16(rng.normal(0, 1, (T, D))), f32_to_bf16(rng.normal(0, 1, (T, D)))
    gl = f32_to_bf16(rng.normal(0, 2, (T, 1)))
    ref = O.combine_sparse_and_shared(sp, sh, gl)
    from astronomical_b200 import _lib
    out = torch.empty((T, D), dtype=torch.bfloat16, device="cuda")
    a, b_, c = bf16_tensor(sp), bf16_tensor(sh), bf16_tensor(gl)
    _lib.check(_lib.lib().astro_moe_combine_sparse_and_shared(
        a.data_ptr(), b_.data_ptr(), c.data_ptr(), 1, T, D, out.data_ptr(),
        torch.cuda.current_stream().cuda_stream))
    assert np.array_equal(to_np_bf16(out), ref)
    # routing_and_combination.rs:12-68, combined [12, 20]
    sel = torch.tensor([[[14.0, 21.0], [7.0, 14.0]]], device="cuda")
    scr = torch.tensor([[4 / 7, 3 / 7]], device="cuda")
    comb = moe.qwen3_5_moe_combine_experts(sel, scr, torch.tensor([[2.0, 4.0]], device="cuda"),
                                           torch.tensor([[0.0]], device="cuda"))
    assert all(abs(a - b) <= 1e-5 * b for a, b in zip(comb.cpu().ravel().tolist(), [12.0, 20.0]))


def test_invert_assignment_order_host():
    assert moe.invert_assignment_order([1, 3, 5, 4, 2, 0]) == [5, 0, 4, 1, 3, 2]
    with pytest.raises(moe.SparseExpertError):
        moe.invert_assignment_order([0, 0])
