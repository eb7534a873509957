"""A checkpoint written with the reference's tensor names (sharded SafeTensors
+ index + per-module quantisation) runs through the GPU block and equals the
oracle bit for bit, and the paged stack built from it equals the resident
blocks."""
import json
import os

import pytest

torch = pytest.importorskip("torch")

from astronomical_b200 import checkpoint as ck  # noqa: E402
from astronomical_b200 import moe, paging, synthetic  # noqa: E402
from tests.helpers import bf16_tensor  # noqa: E402
from tests.test_checkpoint_cpu import write_checkpoint  # noqa: E402
from tests.test_gpu_block import compare_block  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("quant", [None, {"router": (8, 64), "shared_gate": (8, 64)},
                                   {"down": (8, 64), "sdown": (8, 64)}])
@pytest.mark.parametrize("T", [8, 512])
def test_checkpoint_block_matches_oracle(tmp_path, quant, T):
    cfg = dict(synthetic.CONFIGS[1])
    layers = [synthetic.make_block_weights(cfg, seed=60 + i, quant=quant) for i in range(2)]
    d = write_checkpoint(tmp_path, layers, cfg)
    c = ck.Checkpoint(d)
    for li in range(2):
        w = c.moe_layer(li)
        x = synthetic.make_hidden_states(T, cfg["hidden"], seed=70 + li)
        blk = moe.Qwen3_5MoEBlock(w, max_tokens=T)
        y, taps = blk.forward(bf16_tensor(x), taps=True)
        blk.synchronize()
        kernels = blk.last_path()
        blk.close()
        compare_block(w, x, y, taps, kernels, case="checkpoint", canonical=False)


def test_paged_stack_from_checkpoint_equals_resident(tmp_path):
    cfg = dict(synthetic.CONFIGS[2])
    layers = [synthetic.make_block_weights(cfg, seed=80 + i) for i in range(2)]
    c = ck.Checkpoint(write_checkpoint(tmp_path, layers, cfg))
    loaded = [c.moe_layer(i) for i in range(2)]
    store = paging.pack_expert_pages(loaded)
    P = paging.page_bytes(cfg)
    stack = paging.PagedMoEStack(loaded, store, cache_bytes=24 * P)
    resident = [moe.Qwen3_5MoEBlock(w, max_tokens=64, decode_max_tokens=64, decode_fused=-1)
                for w in loaded]
    for T in (1, 8):
        x = bf16_tensor(synthetic.make_hidden_states(T, 2048, seed=90 + T, zipf=True))
        for li in range(2):
            y = stack.forward(li, x)
            y_ref = resident[li].forward(x)
            torch.cuda.synchronize()
            assert torch.equal(y, y_ref)
    stack.close()
    for b in resident:
        b.close()
