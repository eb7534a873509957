"""Decode-path properties beyond oracle parity (which test_gpu_block covers):
the fused decode kernel routes bit-identically to the separate decode kernels
(up to 64 tokens) and each equals the oracle run with its own accumulation
arithmetic bit for bit, and a stack of block calls captured in a CUDA graph
replays bit-identically to eager calls."""
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O  # noqa: E402
from astronomical_b200 import moe, synthetic  # noqa: E402
from tests.helpers import bf16_tensor, oracle_arith, to_np_bf16  # noqa: E402

pytestmark = pytest.mark.gpu


def _x(T, seed):
    return bf16_tensor(synthetic.make_hidden_states(T, 2048, seed=seed, zipf=True))


@pytest.mark.parametrize("T", [1, 3, 8, 16, 17, 40, 64])
def test_fused_decode_matches_separate_kernels(T):
    # up to 16 tokens the fused kernel stages all token rows at once, above it
    # stages each segment's rows 16 at a time
    cfg = dict(synthetic.CONFIGS[2])
    w = synthetic.make_block_weights(cfg, seed=30 + T)
    fused = moe.Qwen3_5MoEBlock(w, max_tokens=64, decode_max_tokens=64, decode_fused=0)
    split = moe.Qwen3_5MoEBlock(w, max_tokens=64, decode_max_tokens=64, decode_fused=-1)
    x_np = synthetic.make_hidden_states(T, 2048, seed=40 + T, zipf=True)
    x = bf16_tensor(x_np)
    ya, ta = fused.forward(x, taps=True)
    path_a = fused.last_path()
    yb, tb = split.forward(x, taps=True)
    path_b = split.last_path()
    torch.cuda.synchronize()
    assert path_a["experts"] == "fused_decode" and path_b["experts"] == "decode_gemv"
    assert fused.read_attribution()["kernel_launches"] == 1
    # the two router GEMVs add in the same order: identical logits, so routing
    # and sort are bit-identical
    assert torch.equal(ta["router_logits"], tb["router_logits"])
    assert torch.equal(ta["selected_indices"], tb["selected_indices"])
    assert torch.equal(ta["selected_scores"], tb["selected_scores"])
    assert torch.equal(ta["expert_offsets"], tb["expert_offsets"])
    # the projections add their products in different orders (tensor-core tiles
    # against fma chains): each path equals the oracle, from x, run with its own
    # kernels' arithmetic
    for path, y in ((path_a, ya), (path_b, yb)):
        arith = oracle_arith(path)
        y_ref, _, _ = O.moe_block_forward(w, x_np, arith=arith)
        assert (to_np_bf16(y) == y_ref).all(), arith
    fused.close()
    split.close()


@pytest.mark.parametrize("fused", [0, -1])
def test_decode_stack_graph_replay_equals_eager(fused):
    cfg = dict(synthetic.CONFIGS[2])
    blocks = [moe.Qwen3_5MoEBlock(synthetic.make_block_weights_torch(cfg, seed=50 + l, device="cuda"),
                                  max_tokens=4, decode_fused=fused) for l in range(3)]
    x = _x(4, 60)
    eager = [b.forward(x) for b in blocks]
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        outs = [b.forward(x) for b in blocks]
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for a, b in zip(outs, eager):
        assert torch.equal(a, b)
    assert moe.device_status(0, reset=True) == 0
    del g
    for b in blocks:
        b.close()
