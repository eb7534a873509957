"""Expert paging on the GPU: a paged stack must produce exactly what the resident
block computes with the same decode kernels, while its page cache admits, hits
and evicts pages (a cache far smaller than the expert store forces evictions)."""
import pytest

torch = pytest.importorskip("torch")

from astronomical_b200 import moe, paging, synthetic  # noqa: E402
from tests.helpers import bf16_tensor  # noqa: E402

pytestmark = pytest.mark.gpu


def test_paged_stack_equals_resident_blocks_and_counts_pages():
    cfg = dict(synthetic.CONFIGS[2])
    L = 3
    layers = [synthetic.make_block_weights_torch(cfg, seed=200 + l, device="cuda") for l in range(L)]
    store = paging.pack_expert_pages(layers)
    P = paging.page_bytes(cfg)
    stack = paging.PagedMoEStack(layers, store, cache_bytes=40 * P)
    resident = [moe.Qwen3_5MoEBlock(w, max_tokens=64, decode_max_tokens=64, decode_fused=-1)
                for w in layers]
    seen = set()
    for rep in range(3):
        for T in (1, 8, 5):
            x = bf16_tensor(synthetic.make_hidden_states(T, 2048, seed=300 + T, zipf=True))
            for l in range(L):
                y = stack.forward(l, x)
                y_ref, taps = resident[l].forward(x, taps=True)
                torch.cuda.synchronize()
                assert torch.equal(y, y_ref), (rep, T, l)
                seen |= {(l, int(e)) for e in torch.unique(taps["selected_indices"]).tolist()}
    s = stack.stats()
    assert s["hits"] + s["misses"] == s["lookups"]
    assert s["bytes_h2d"] == s["misses"] * P
    assert s["resident_pages"] <= 40 and s["capacity_pages"] == 40
    assert s["misses"] >= min(len(seen), 40)      # every page needed at least one admission
    assert s["evictions"] == s["misses"] - s["resident_pages"]
    if len(seen) > 40:
        assert s["evictions"] > 0
    assert s["copy_ms"] > 0
    # a call that copied pages ran the copied experts' second launch; every call
    # after the first of a layer that found all its pages resident did not
    assert s["calls"] == 3 * 3 * L
    assert 0 < s["split_calls"] <= s["calls"] and s["split_calls"] <= s["misses"]
    x = bf16_tensor(synthetic.make_hidden_states(1, 2048, seed=301, zipf=True))
    stack.forward(0, x)
    before = stack.stats()
    stack.forward(0, x)  # same token, same layer: every page it needs is resident
    after = stack.stats()
    assert after["misses"] == before["misses"] and after["split_calls"] == before["split_calls"]
    assert after["calls"] == before["calls"] + 1
    assert moe.device_status(0, reset=True) == 0
    stack.close()
    for b in resident:
        b.close()
