"""Whole-block parity: astro_moe_block_forward against the CPU oracle, from the
same hidden states (no intermediate of the GPU is fed to the oracle).

Every block call reports the kernels it ran (astro_moe_ctx_last_block_path); the
oracle is then run with those kernels' accumulation arithmetic (oracle/oracle.py
arith_for_kernels, oracle/astro_oracle.h AO_DOT_*), and router logits, selected
experts, scores, sort offsets and the block output must be identical bit for
bit.  The same output is also compared with the oracle's canonical order
(sequential fma): the spread between two valid accumulation orders, reported
under the reference's own convention (tests/helpers.py reference_metrics) and
held to relative L2 1e-3."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O  # noqa: E402
from astronomical_b200 import moe, synthetic  # noqa: E402
from tests.helpers import (MAX_ABS, REL_L2, bf16_tensor, oracle_arith, record_parity,  # noqa: E402
                           reference_metrics, to_np_bf16, to_np_u32)

pytestmark = pytest.mark.gpu


def small_cfg(**kw):
    cfg = dict(synthetic.CONFIGS[1])
    cfg.update(kw)
    return cfg


def block(w, path, **kw):
    use_tc, decode, fused = path
    return moe.Qwen3_5MoEBlock(w, use_tensor_cores=use_tc, decode_max_tokens=decode,
                               decode_fused=fused, **kw)


def expert_sets_differ(a, b):
    return int((np.sort(a, 1) != np.sort(b, 1)).any(1).sum())


def compare_block(w, x, y, taps, kernels, subset=None, case="block", canonical=True, T=None):
    """Bit-exact comparison of one block call with the oracle run from x with the
    call's kernels' arithmetic, then the spread against the canonical order."""
    cfg = w["config"]
    T = x.shape[0] if T is None else T
    logits = to_np_bf16(taps["router_logits"])
    ids = to_np_u32(taps["selected_indices"])
    scores = (taps["selected_scores"].cpu().numpy() if cfg.get("router") == "laguna"
              else to_np_bf16(taps["selected_scores"]))
    offs = to_np_u32(taps["expert_offsets"])
    got = to_np_bf16(y)
    arith = oracle_arith(kernels)
    sub = np.arange(T) if subset is None else np.asarray(subset)
    router_w = w["router_w"] if "router_w" in w else O.dequantize_affine(
        w["router_q"], w["router_s"], w["router_b"], w["router_group"], w["router_bits"])
    # a1: router logits from x with the router kernel's arithmetic
    ref_logits = O.matmul_bf16_nt(x[sub], router_w, mode=arith["router"])
    assert np.array_equal(logits[sub], ref_logits), (kernels, int((logits[sub] != ref_logits).sum()))
    # a2-a9 from x (no override): routing, sort and the block output
    y_ref, ids_ref, sc_ref = O.moe_block_forward(w, x, token_subset=subset, arith=arith)
    assert np.array_equal(ids[sub], ids_ref)
    assert np.array_equal(scores[sub], sc_ref)
    if subset is None:
        srt = O.sort_expert_assignments(ids_ref, cfg["experts"])
        assert np.array_equal(offs[:cfg["experts"] + 1], srt["expert_offsets"])
    exact = reference_metrics(got[sub], y_ref)
    assert exact["n_differ"] == 0, (kernels, exact)
    assert exact["scaled_max_abs"] <= MAX_ABS and exact["rel_l2"] <= REL_L2
    fields = dict(T=T, rows=int(sub.size), kernels=kernels, arith=arith, exact=exact)
    if canonical:
        # the canonical order: routing and outputs of another valid accumulation order
        y_c, ids_c, _ = O.moe_block_forward(w, x, token_subset=subset)
        canon = reference_metrics(got[sub], y_c)
        logits_c = O.matmul_bf16_nt(x[sub], router_w)
        fields.update(canonical=canon, canonical_logits_differ=int((logits[sub] != logits_c).sum()),
                      canonical_expert_sets_differ=expert_sets_differ(ids[sub], ids_c))
        assert canon["rel_l2"] <= REL_L2, canon
    record_parity(case, **fields)
    return fields


def run_and_compare(cfg, T, seed=0, subset=None, fuse=False, path=(0, 0, 0), case="block",
                    canonical=True, weights=None):
    w = synthetic.make_block_weights(cfg, seed=seed) if weights is None else weights
    x = synthetic.make_hidden_states(T, cfg["hidden"], seed=seed + 1, zipf=bool(cfg.get("zipf")))
    blk = block(w, path, max_tokens=T, fuse_gate_up=fuse)
    y, taps = blk.forward(bf16_tensor(x), taps=True)
    blk.synchronize()
    kernels = blk.last_path()
    blk.close()
    return compare_block(w, x, y, taps, kernels, subset=subset, case=case, canonical=canonical)


# path = (use_tensor_cores, decode_max_tokens, decode_fused): the tcgen05 grouped
# GEMMs, the CUDA-core grouped GEMV, the separate decode kernels (taken here up
# to 1024 tokens so that segments of many rows are covered too), and the fused
# decode kernel (T <= 64; larger T falls through to the separate decode kernels)
PATHS = [pytest.param((1, -1, -1), id="tcgen05"), pytest.param((-1, -1, -1), id="cudacore"),
         pytest.param((0, 1024, -1), id="decode"), pytest.param((0, 1024, 0), id="fused")]


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("seed", [0, 1, 2, 3, 4])
def test_block_config0_shape(path, seed):
    cfg = dict(synthetic.CONFIGS[0])
    run_and_compare(cfg, 32, seed=seed, path=path, case="config0")


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("T", [1, 4, 7, 8, 16, 64, 200, 777])
def test_block_config1_shape_small_T(T, path):
    # T*K < 64 takes the unsorted weighted sum (routing.rs:13), T >= 8 the sorted one
    run_and_compare(small_cfg(), T, seed=T, path=path, case="config1_small_T")


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("seed", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("T", [1, 4, 16, 64])
def test_block_decode_zipf(T, seed, path):
    cfg = dict(synthetic.CONFIGS[2])
    cfg["tokens"] = T
    run_and_compare(cfg, T, seed=100 + 10 * seed + T, path=path, case="config2_decode")


@pytest.mark.parametrize("path", PATHS)
def test_block_fused_gate_up_equals_separate(path):
    # resident_gate_up_fusion.rs: fusing gate||up must not change any value
    cfg = small_cfg()
    w = synthetic.make_block_weights(cfg, seed=4)
    x = bf16_tensor(synthetic.make_hidden_states(96, cfg["hidden"], seed=5))
    a = block(w, path, max_tokens=96, fuse_gate_up=False)
    b = block(w, path, max_tokens=96, fuse_gate_up=True)
    ya, yb = a.forward(x), b.forward(x)
    torch.cuda.synchronize()
    assert torch.equal(ya, yb)
    a.close()
    b.close()


# T=4096, the headline shape, on all rows.  The decode and fused paths take the
# tcgen05 GEMMs at this size, so the two distinct kernel sets are covered; the
# separate decode GEMVs are covered on all rows at 1024 tokens (segments of many
# rows each).
@pytest.mark.parametrize("path", [PATHS[0], PATHS[1]])
def test_block_full_size_config1_all_rows(path):
    run_and_compare(small_cfg(), 4096, seed=11, path=path, case="config1_full")


def test_block_decode_gemv_1024_all_rows():
    run_and_compare(small_cfg(), 1024, seed=13, path=(0, 1024, -1), case="config1_decode_1024")


# The gate/up GEMM takes units of two weight-row blocks from 64 rows per segment
# on average: segments that fill a tile partly (T = 1900, about 66 rows each) and
# skewed routing with segments of several tiles beside nearly empty ones (T =
# 2048, Zipf hidden states), all rows.
@pytest.mark.parametrize("T,zipf", [(1900, None), (2048, 1.1)])
def test_block_paired_gate_up_units_all_rows(T, zipf):
    run_and_compare(small_cfg(zipf=zipf), T, seed=17, path=(1, -1, -1), case="config1_paired")


@pytest.mark.parametrize("path", PATHS)
def test_block_paths_agree_within_tolerance(path):
    """The two GPU paths compute the same block (different accumulation order)."""
    cfg = small_cfg()
    w = synthetic.make_block_weights(cfg, seed=21)
    x = bf16_tensor(synthetic.make_hidden_states(1024, cfg["hidden"], seed=22))
    a = block(w, (1, -1, -1), max_tokens=1024)
    b = block(w, path, max_tokens=1024)
    ya, ta = a.forward(x, taps=True)
    yb, tb = b.forward(x, taps=True)
    torch.cuda.synchronize()
    if torch.equal(ta["router_logits"], tb["router_logits"]):
        assert torch.equal(ta["selected_indices"], tb["selected_indices"])
    a.close()
    b.close()


@pytest.mark.parametrize("path", PATHS)
def test_block_deterministic_and_empty(path):
    cfg = small_cfg()
    w = synthetic.make_block_weights(cfg, seed=8)
    blk = block(w, path, max_tokens=512)
    x = bf16_tensor(synthetic.make_hidden_states(512, cfg["hidden"], seed=9))
    y1 = blk.forward(x)
    y2 = blk.forward(x)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)  # no atomics anywhere: bitwise reproducible
    empty = blk.forward(x[:0])
    assert empty.shape == (0, cfg["hidden"])
    blk.close()


def test_block_host_entry_matches_device_entry():
    cfg = small_cfg()
    w = synthetic.make_block_weights(cfg, seed=12)
    blk = moe.Qwen3_5MoEBlock(w, max_tokens=256)
    x = bf16_tensor(synthetic.make_hidden_states(256, cfg["hidden"], seed=13))
    y = blk.forward(x)
    hx = x.cpu().pin_memory()
    hy = torch.empty_like(hx).pin_memory()
    blk.forward_host(hx, hy)
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), hy)
    blk.close()


def test_block_host_async_calls_match_device_entry():
    """Four overlapping asynchronous host-buffer calls (the staging slots are
    reused twice) each equal the device entry point on their own input."""
    cfg = small_cfg()
    w = synthetic.make_block_weights(cfg, seed=14)
    blk = moe.Qwen3_5MoEBlock(w, max_tokens=384)
    xs = [bf16_tensor(synthetic.make_hidden_states(384, cfg["hidden"], seed=20 + i)) for i in range(4)]
    want = [blk.forward(x) for x in xs]
    torch.cuda.synchronize()
    hin = [x.cpu().pin_memory() for x in xs]
    hout = [torch.empty_like(h).pin_memory() for h in hin]
    for i in range(4):
        blk.forward_host_async(hin[i], hout[i])
    blk.synchronize_host()
    for h, y in zip(hout, want):
        assert torch.equal(h, y.cpu())
    blk.close()


# Each reference projection carries its own quantisation (Qwen3_5AffineWeights,
# qwen3_5/model/decoder_layer_weights.rs:15-26) and the router and shared-expert
# gate may be affine (feed_forward_weights.rs:10-14): the block must equal the
# oracle bit for bit in every mix, whichever kernels each mix selects.
QUANTS = [
    pytest.param({"router": (8, 64), "shared_gate": (8, 64)}, id="affine-router-and-gate-8bit"),
    pytest.param({"router": (4, 64)}, id="affine-router-4bit"),
    pytest.param({"down": (8, 64), "sdown": (8, 64)}, id="down-8bit"),
    pytest.param({"sgate": (8, 64), "sup": (8, 64), "sdown": (8, 64)}, id="shared-8bit-separate"),
    pytest.param({"gate": (8, 128), "up": (8, 128), "down": (3, 32), "sgate": (6, 64),
                  "sup": (6, 64), "sdown": (2, 32), "router": (5, 32), "shared_gate": (6, 128)},
                 id="every-projection-its-own"),
]


@pytest.mark.parametrize("quant", QUANTS)
@pytest.mark.parametrize("T", [5, 64, 300])
def test_block_per_projection_quantisation(quant, T):
    cfg = small_cfg()
    w = synthetic.make_block_weights(cfg, seed=40 + T, quant=quant)
    f = run_and_compare(cfg, T, seed=40 + T, weights=w, case="per_projection_quant")
    kernels = f["kernels"]
    separate = "sgate" in quant and "gate" not in quant
    if separate:
        assert kernels["shared_expert"] == "grouped_gemv"
    if "gate" in quant or "down" in quant:
        assert kernels["experts"] == "grouped_gemv"


def test_gate_and_up_must_share_their_quantisation():
    cfg = small_cfg()
    w = synthetic.make_block_weights(cfg, seed=3, quant={"gate": (8, 64)})
    with pytest.raises(moe.AstroMoeError, match="gate and up"):
        moe.Qwen3_5MoEBlock(w, max_tokens=8)


# The Laguna router family (laguna/moe/router.rs, resident.rs:60-100) on the same
# sort, GEMMs and combine: sigmoid scores with a selection-only correction bias,
# fp32 scores, routed sum scaled by 2.5, ungated shared expert.
@pytest.mark.parametrize("path", [PATHS[0], PATHS[1], PATHS[2]])
@pytest.mark.parametrize("T", [1, 7, 64, 512])
def test_block_laguna_router(T, path):
    cfg = dict(synthetic.LAGUNA)
    f = run_and_compare(cfg, T, seed=500 + T, path=path, case="laguna")
    assert f["kernels"]["gate_logit"] == "none"


def test_block_laguna_softcap_and_no_shared_expert():
    cfg = dict(synthetic.LAGUNA, router_logit_softcap=1.5, shared_intermediate=0)
    run_and_compare(cfg, 96, seed=7, case="laguna_softcap")
