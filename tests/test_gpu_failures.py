"""Failure detection without faulting, trapping or hanging a GPU.

- Device waits: the library's bounded waits (the fused decode kernel's
  completion-counter wait and the tcgen05 pipeline's mbarrier wait) are made to
  run out with a 1 ms limit on a condition nothing satisfies; the kernel records
  ASTRO_MOE_DEVICE_WAIT_TIMEOUT in the caller's status word and returns, and the
  context stays usable (a block call afterwards is correct).
- Expert paging: a page copy failure injected on the host makes the paged call
  return an error without writing its output and without leaving a stale page
  (the next call copies it again and equals the resident block); a cache ceiling
  below one page is rejected at creation (mlx_runtime_types.rs:129-133,
  ActiveMemoryLimitExceeded).
- Bad inputs found on the device (expert id >= E) are recorded, not trapped.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from astronomical_b200 import _lib, moe, paging, synthetic  # noqa: E402
from tests.helpers import bf16_tensor  # noqa: E402

pytestmark = pytest.mark.gpu

WAIT_TIMEOUT = 2  # ASTRO_MOE_DEVICE_WAIT_TIMEOUT


def _probe(kind, target, flag_value=0, limit_ns=1_000_000):
    flag = torch.full((1,), flag_value, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    result = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    rc = _lib.lib().astro_moe_wait_probe(kind, ctypes.c_void_p(flag.data_ptr()), target, limit_ns,
                                         ctypes.c_void_p(status.data_ptr()),
                                         ctypes.c_void_p(result.data_ptr()), None)
    assert rc == 0, _lib.lib().astro_moe_last_error()
    torch.cuda.synchronize()
    return int(result.item()), int(status.item())


@pytest.mark.parametrize("kind", [0, 1])
def test_bounded_waits_run_out_and_report(kind):
    # the condition never holds: the wait gives up after 1 ms with the timeout bit
    res, st = _probe(kind, target=1, flag_value=0)
    assert res == 0 and st & WAIT_TIMEOUT
    # the condition holds: no timeout
    res, st = _probe(kind, target=1 if kind == 0 else 2, flag_value=1)
    assert res == 1 and st == 0


def test_context_usable_after_a_timed_out_wait():
    _probe(0, target=5, flag_value=0)
    cfg = dict(synthetic.CONFIGS[1])
    w = synthetic.make_block_weights(cfg, seed=3)
    blk = moe.Qwen3_5MoEBlock(w, max_tokens=32)
    x = bf16_tensor(synthetic.make_hidden_states(32, 2048, seed=4))
    y1 = blk.forward(x)
    y2 = blk.forward(x)
    blk.synchronize()  # raises if the library's own status word recorded anything
    assert torch.equal(y1, y2) and torch.isfinite(y1.float()).all()
    blk.close()


def test_wait_probe_rejects_bad_arguments():
    lib = _lib.lib()
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    p = ctypes.c_void_p(status.data_ptr())
    assert lib.astro_moe_wait_probe(0, None, 1, 1000, p, p, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.astro_moe_wait_probe(0, p, 1, 3_000_000_000, p, p, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.astro_moe_wait_probe(5, p, 1, 1000, p, p, None) == _lib.ERR_INVALID_ARGUMENT


def _paged(L=2, cache_pages=24, policy="lru"):
    cfg = dict(synthetic.CONFIGS[2])
    layers = [synthetic.make_block_weights_torch(cfg, seed=210 + l, device="cuda") for l in range(L)]
    store = paging.pack_expert_pages(layers)
    P = paging.page_bytes(cfg)
    return cfg, layers, store, paging.PagedMoEStack(layers, store, cache_bytes=cache_pages * P,
                                                    policy=policy)


def test_injected_page_copy_failure_is_an_error_and_leaves_no_stale_page():
    cfg, layers, store, stack = _paged()
    resident = moe.Qwen3_5MoEBlock(layers[0], max_tokens=64, decode_max_tokens=64, decode_fused=-1)
    x = bf16_tensor(synthetic.make_hidden_states(8, 2048, seed=5, zipf=True))
    stack.inject_copy_failures(3)
    with pytest.raises(moe.AstroMoeError) as e:
        stack.forward(0, x)
    assert e.value.status == _lib.ERR_CUDA and "page copy" in str(e.value)
    s = stack.stats()
    assert s["copy_failures"] == 3
    # the failed experts hold no page: the next call copies them and is correct
    y = stack.forward(0, x)
    y_ref = resident.forward(x)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    assert stack.stats()["copy_failures"] == 3
    stack.close()
    resident.close()


def test_cache_ceiling_below_one_page_is_rejected():
    cfg = dict(synthetic.CONFIGS[2])
    layers = [synthetic.make_block_weights_torch(cfg, seed=1, device="cuda")]
    store = paging.pack_expert_pages(layers)
    with pytest.raises(moe.AstroMoeError) as e:
        paging.PagedMoEStack(layers, store, cache_bytes=paging.page_bytes(cfg) - 1)
    assert e.value.status == _lib.ERR_MEMORY_LIMIT and "holds no" in str(e.value)


@pytest.mark.parametrize("policy", ["lru", "demand"])
def test_pager_policies_compute_the_resident_block(policy):
    cfg, layers, store, stack = _paged(L=3, cache_pages=30, policy=policy)
    resident = [moe.Qwen3_5MoEBlock(w, max_tokens=64, decode_max_tokens=64, decode_fused=-1)
                for w in layers]
    for rep in range(3):
        for T in (1, 8):
            x = bf16_tensor(synthetic.make_hidden_states(T, 2048, seed=400 + T + rep, zipf=True))
            for l in range(3):
                y = stack.forward(l, x)
                assert torch.equal(y, resident[l].forward(x)), (policy, rep, T, l)
    s = stack.stats()
    assert s["hits"] + s["misses"] == s["lookups"] and s["resident_pages"] <= 30
    stack.close()
    for b in resident:
        b.close()


def test_bad_expert_ids_are_recorded_not_trapped():
    ids = torch.tensor([[1, 7]], dtype=torch.int32, device="cuda")  # 7 >= 4 experts
    x = torch.zeros((1, 1, 1, 8), dtype=torch.bfloat16, device="cuda")
    moe.device_status(0, reset=True)
    moe.sort_expert_assignments(x, ids, experts=4)
    torch.cuda.synchronize()
    assert moe.device_status(0, reset=True) & 1  # ASTRO_MOE_DEVICE_BAD_EXPERT_ID
