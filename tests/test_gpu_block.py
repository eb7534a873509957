"""Whole-block parity: astro_moe_block_forward against the CPU oracle.

Routing is compared bit-exactly on the GPU's own router logits (the router
projection is a floating-point GEMM whose accumulation order differs from the
CPU's, so its bf16 logits may differ by an ulp; given the same logits the
selected experts, scores and expert offsets are identical).  Block outputs must
meet the north-star tolerance: max-abs 2e-2 and relative L2 1e-3 in bf16."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O  # noqa: E402
from astronomical_b200 import moe, synthetic  # noqa: E402
from tests.helpers import assert_block_close, bf16_tensor, to_np_bf16, to_np_u32  # noqa: E402

pytestmark = pytest.mark.gpu


def small_cfg(**kw):
    cfg = dict(synthetic.CONFIGS[1])
    cfg.update(kw)
    return cfg


def block(w, path, **kw):
    use_tc, decode, fused = path
    return moe.Qwen3_5MoEBlock(w, use_tensor_cores=use_tc, decode_max_tokens=decode,
                               decode_fused=fused, **kw)


def run_and_compare(cfg, T, seed=0, subset=None, fuse=False, path=(0, 0, 0)):
    w = synthetic.make_block_weights(cfg, seed=seed)
    x = synthetic.make_hidden_states(T, cfg["hidden"], seed=seed + 1, zipf=bool(cfg.get("zipf")))
    blk = block(w, path, max_tokens=T, fuse_gate_up=fuse)
    y, taps = blk.forward(bf16_tensor(x), taps=True)
    blk.synchronize()
    logits = to_np_bf16(taps["router_logits"])
    ids = to_np_u32(taps["selected_indices"])
    scores = to_np_bf16(taps["selected_scores"])
    offs = to_np_u32(taps["expert_offsets"])
    got = to_np_bf16(y)
    # router projection: a floating-point GEMM (tensor-core fp32 accumulation
    # differs from the oracle's sequential fma), held to the block tolerance
    sub = np.arange(T) if subset is None else np.asarray(subset)
    ref_logits = O.matmul_bf16_nt(x[sub], w["router_w"])
    assert_block_close(logits[sub], ref_logits)
    # routing / sort: bit-exact given the same logits
    ids_o, sc_o = O.route_experts(logits, cfg["top_k"], cfg.get("normalize", True))
    assert np.array_equal(ids, ids_o)
    assert np.array_equal(scores, sc_o)
    srt = O.sort_expert_assignments(ids_o, cfg["experts"])
    assert np.array_equal(offs[:cfg["experts"] + 1], srt["expert_offsets"])
    # block output on the same logits
    y_ref, ids_r, _, sp, sg = O.moe_block_forward(w, x, token_subset=subset,
                                                  logits_override=logits, terms=True)
    assert np.array_equal(ids_r, ids[sub])
    metrics = assert_block_close(got[sub], y_ref, terms=(sp, sg))
    blk.close()
    return metrics


# path = (use_tensor_cores, decode_max_tokens, decode_fused): the tcgen05 grouped
# GEMMs, the CUDA-core grouped GEMV, the separate decode kernels (taken here up
# to 1024 tokens so that segments of many rows are covered too), and the fused
# decode kernel (T <= 64; larger T falls through to the separate decode kernels)
PATHS = [pytest.param((1, -1, -1), id="tcgen05"), pytest.param((-1, -1, -1), id="cudacore"),
         pytest.param((0, 1024, -1), id="decode"), pytest.param((0, 1024, 0), id="fused")]


@pytest.mark.parametrize("path", PATHS)
def test_block_config0_shape(path):
    cfg = dict(synthetic.CONFIGS[0])
    run_and_compare(cfg, 32, path=path)


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("T", [1, 4, 7, 8, 16, 64, 200, 777])
def test_block_config1_shape_small_T(T, path):
    # T*K < 64 takes the unsorted weighted sum (routing.rs:13), T >= 8 the sorted one
    run_and_compare(small_cfg(), T, seed=T, path=path)


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("T", [1, 4, 16, 64])
def test_block_decode_zipf(T, path):
    cfg = dict(synthetic.CONFIGS[2])
    cfg["tokens"] = T
    run_and_compare(cfg, T, seed=100 + T, path=path)


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


@pytest.mark.parametrize("path", PATHS)
def test_block_full_size_config1_subset(path):
    """T=4096 (the headline shape): every output row depends only on its own
    token, so the oracle checks a sample of 48 rows of the full-size run."""
    rng = np.random.default_rng(7)
    subset = np.sort(rng.choice(4096, 48, replace=False))
    run_and_compare(small_cfg(), 4096, seed=11, subset=subset, path=path)


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
