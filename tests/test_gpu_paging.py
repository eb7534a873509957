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


def _config1_layers(n, seed):
    cfg = dict(synthetic.CONFIGS[1])
    return cfg, [synthetic.make_block_weights_torch(cfg, seed=seed + l, device="cuda")
                 for l in range(n)]


def test_paged_prefill_equals_resident_block():
    """Calls of more than 64 tokens bring in all their pages and run the tcgen05
    grouped GEMMs over the cache: bit-identical to the resident block (same
    kernels and arithmetic), while the cache (300 pages, two layers of 256
    experts) evicts the other layer's pages."""
    cfg, layers = _config1_layers(2, seed=500)
    store = paging.pack_expert_pages(layers)
    P = paging.page_bytes(cfg)
    stack = paging.PagedMoEStack(layers, store, cache_bytes=300 * P, max_tokens=1024)
    resident = [moe.Qwen3_5MoEBlock(w, max_tokens=1024) for w in layers]
    for T, zipf in ((1024, False), (300, True), (65, False), (1024, False)):
        x = bf16_tensor(synthetic.make_hidden_states(T, cfg["hidden"], seed=600 + T, zipf=zipf))
        for l in range(2):
            y = stack.forward(l, x)
            assert stack.last_path()["experts"] == "tcgen05_gemm"
            y_ref = resident[l].forward(x)
            torch.cuda.synchronize()
            assert resident[l].last_path()["experts"] == "tcgen05_gemm"
            assert torch.equal(y, y_ref), (T, zipf, l)
    s = stack.stats()
    assert s["evictions"] > 0 and s["capacity_pages"] == 300
    assert s["bytes_h2d"] == s["misses"] * P
    # decode calls on the same cache still take the split decode path
    x = bf16_tensor(synthetic.make_hidden_states(4, cfg["hidden"], seed=7, zipf=True))
    y = stack.forward(1, x)
    assert stack.last_path()["experts"] == "decode_gemv"
    assert torch.isfinite(y.float()).all()
    assert moe.device_status(0, reset=True) == 0
    stack.close()
    for b in resident:
        b.close()


def test_paged_call_larger_than_the_cache_is_refused():
    """A call whose routed experts need more pages than the cache holds fails with
    the memory-limit status (a call never evicts its own pages), and the stack
    keeps working for calls that fit."""
    cfg, layers = _config1_layers(1, seed=700)
    store = paging.pack_expert_pages(layers)
    P = paging.page_bytes(cfg)
    stack = paging.PagedMoEStack(layers, store, cache_bytes=64 * P, max_tokens=512)
    x = bf16_tensor(synthetic.make_hidden_states(512, cfg["hidden"], seed=8))
    with pytest.raises(moe.AstroMoeError, match="cannot hold"):
        stack.forward(0, x)
    resident = moe.Qwen3_5MoEBlock(layers[0], max_tokens=64, decode_max_tokens=64,
                                   decode_fused=-1)
    x1 = bf16_tensor(synthetic.make_hidden_states(2, cfg["hidden"], seed=9))
    y = stack.forward(0, x1)
    y_ref = resident.forward(x1)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    stack.close()
    resident.close()
