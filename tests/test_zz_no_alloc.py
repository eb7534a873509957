"""astro_moe_sort_expert_assignments_no_alloc against the allocating sort.

The no-alloc entry point serves callers that cannot allocate device memory
(a process whose own caching allocator holds all of HBM, or a latency-bound loop
that cannot take the synchronisation cudaMalloc/cudaFree may cause); its scratch
is a fixed 256 KiB device array shared by every call on a GPU.  The sort is
integer work, so its outputs must equal the allocating entry point's bit for
bit.  Two calls in a row with different shapes check that what the first call
left in the shared array does not leak into the second.

This file is named to be collected last, so a run that stops at the first
failure has run every other test before it.
"""
import ctypes

import numpy as np
import pytest
import torch

from astronomical_b200 import _lib

ASTRO_MOE_OK = 0
ASTRO_MOE_ERR_UNSUPPORTED = 4
ASTRO_MOE_DEVICE_BAD_EXPERT_ID = 1
SCRATCH_BYTES = 262144


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _ids(T, K, E, seed):
    rng = np.random.default_rng(seed)
    p = np.exp(-2.0 * np.arange(E) / E)
    p /= p.sum()
    return rng.choice(E, size=(T, K), p=p).astype(np.uint32)


def _sort(fn_name, ids_np, E, with_offsets=True, status=None):
    lib = _lib.lib()
    T, K = ids_np.shape
    n = T * K
    ids = torch.from_numpy(ids_np.view(np.int32)).cuda()
    outs = [torch.full((max(n, 1),), -1, dtype=torch.int32, device="cuda") for _ in range(4)]
    offs = torch.full((E + 1,), -1, dtype=torch.int32, device="cuda") if with_offsets else None
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = [_p(ids), T, K, E, *map(_p, outs), _p(offs)]
    if fn_name.endswith("no_alloc"):
        args.append(_p(status))
    rc = getattr(lib, fn_name)(*args, stream)
    assert rc == ASTRO_MOE_OK, lib.astro_moe_last_error().decode()
    torch.cuda.synchronize()
    res = [o[:n].cpu().numpy() for o in outs]
    if offs is not None:
        res.append(offs.cpu().numpy())
    return res


@pytest.mark.gpu
def test_no_alloc_sort_matches_allocating_sort_on_two_calls():
    # first the prefill shape (4096 tokens x top-8 of 256 experts), then a
    # smaller, ragged one that reuses the array the first call filled
    for T, K, E, seed in ((4096, 8, 256, 1), (777, 8, 256, 2)):
        ids = _ids(T, K, E, seed)
        want = _sort("astro_moe_sort_expert_assignments", ids, E)
        got = _sort("astro_moe_sort_expert_assignments_no_alloc", ids, E)
        for w, g in zip(want, got):
            assert np.array_equal(w, g)


@pytest.mark.gpu
def test_no_alloc_sort_without_offsets_and_bad_ids():
    ids = _ids(64, 8, 32, 3)
    want = _sort("astro_moe_sort_expert_assignments", ids, 32, with_offsets=False)
    got = _sort("astro_moe_sort_expert_assignments_no_alloc", ids, 32, with_offsets=False)
    for w, g in zip(want, got):
        assert np.array_equal(w, g)
    # an id >= experts is skipped and reported in the caller's status word
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    bad = np.array([[1, 7]], np.uint32)
    _sort("astro_moe_sort_expert_assignments_no_alloc", bad, 4, status=status)
    assert int(status.item()) & ASTRO_MOE_DEVICE_BAD_EXPERT_ID


@pytest.mark.gpu
def test_no_alloc_sort_without_offsets_on_many_tiles_after_a_larger_call():
    # without an offsets output the offsets live in the array right after the
    # per-tile histograms; a multi-tile call (777 x 8 = 3 tiles) right after a
    # larger one must not see what that call left there
    big = _ids(4096, 8, 256, 5)
    _sort("astro_moe_sort_expert_assignments_no_alloc", big, 256)
    ids = _ids(777, 8, 256, 6)
    want = _sort("astro_moe_sort_expert_assignments", ids, 256, with_offsets=False)
    got = _sort("astro_moe_sort_expert_assignments_no_alloc", ids, 256, with_offsets=False)
    for w, g in zip(want, got):
        assert np.array_equal(w, g)


@pytest.mark.gpu
@pytest.mark.parametrize("with_offsets", [True, False])
def test_no_alloc_sort_at_the_largest_accepted_size(with_offsets):
    # 256 tiles x 256 experts x 4 B = 262,144 B exactly with an offsets output;
    # 254 tiles when the offsets (4 x 257 B) share the array
    E = 256
    n = (256 if with_offsets else 254) * 2048
    ids = _ids(n // 8, 8, E, 7)
    want = _sort("astro_moe_sort_expert_assignments", ids, E, with_offsets=with_offsets)
    got = _sort("astro_moe_sort_expert_assignments_no_alloc", ids, E, with_offsets=with_offsets)
    for w, g in zip(want, got):
        assert np.array_equal(w, g)


@pytest.mark.parametrize("with_offsets", [True, False])
def test_no_alloc_sort_rejects_one_tile_past_the_limit(with_offsets):
    # host-side check, before any CUDA call: the smallest size over the limit
    lib = _lib.lib()
    E = 256
    n = (256 if with_offsets else 254) * 2048 + 1
    need = 4 * E * -(-n // 2048) + (0 if with_offsets else 4 * (E + 1))
    assert need > SCRATCH_BYTES
    assert need - 4 * E <= SCRATCH_BYTES  # one tile fewer fits
    fake = ctypes.c_void_p(256)  # never dereferenced: the call fails first
    rc = lib.astro_moe_sort_expert_assignments_no_alloc(fake, n, 1, E, fake, fake, fake, fake,
                                                        fake if with_offsets else None, None, None)
    assert rc == ASTRO_MOE_ERR_UNSUPPORTED
    assert "static array" in lib.astro_moe_last_error().decode()


def test_no_alloc_sort_rejects_sizes_beyond_the_array():
    # host-side check, before any CUDA call: 4 * 256 * ceil(n / 2048) bytes of
    # histograms exceed 256 KiB past 522,240 assignments
    lib = _lib.lib()
    tokens, K, E = 65536, 16, 256
    assert 4 * E * -(-(tokens * K) // 2048) > SCRATCH_BYTES
    fake = ctypes.c_void_p(256)  # never dereferenced: the call fails first
    rc = lib.astro_moe_sort_expert_assignments_no_alloc(fake, tokens, K, E, fake, fake, fake, fake,
                                                        fake, None, None)
    assert rc == ASTRO_MOE_ERR_UNSUPPORTED
    assert "static array" in lib.astro_moe_last_error().decode()
