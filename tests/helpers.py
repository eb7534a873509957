"""Shared helpers for the parity tests (comparison metrics and array plumbing)."""
from __future__ import annotations

import numpy as np

from astronomical_b200.synthetic import bf16_to_f32, f32_to_bf16

# north-star tolerances for block outputs in bf16
MAX_ABS = 2e-2
REL_L2 = 1e-3


def to_np_bf16(t) -> np.ndarray:
    """torch bf16 tensor -> uint16 bit patterns."""
    import torch

    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def to_np_u32(t) -> np.ndarray:
    import torch

    return t.detach().contiguous().view(torch.int32).cpu().numpy().view(np.uint32)


def bf16_tensor(a, device="cuda"):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(
        torch.bfloat16).to(device)


def u32_tensor(a, device="cuda"):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint32).view(np.int32)).to(device)


def bf16_ulp(x: np.ndarray) -> np.ndarray:
    """Spacing of bf16 numbers at |x| (8 significant bits)."""
    ax = np.abs(x.astype(np.float64))
    ax = np.maximum(ax, np.float64(np.finfo(np.float32).tiny))
    return np.exp2(np.floor(np.log2(ax)) - 7)


def assert_bf16_ulps(a_bits, b_bits, ulps: float = 1.0, max_frac: float = 0.02):
    """Every element within `ulps` bf16 ulps, and at most `max_frac` differing."""
    a = bf16_to_f32(a_bits).astype(np.float64)
    b = bf16_to_f32(b_bits).astype(np.float64)
    assert a.shape == b.shape
    diff = np.abs(a - b)
    tol = ulps * bf16_ulp(np.maximum(np.abs(a), np.abs(b)))
    bad = diff > tol
    assert not bad.any(), f"{bad.sum()} elements beyond {ulps} ulp; worst {diff.max()}"
    frac = float((diff > 0).mean()) if diff.size else 0.0
    assert frac <= max_frac, f"{frac:.4f} of elements differ"


def block_metrics(got_bits, ref_bits, terms=None):
    """(raw max-abs, scaled max-abs, relative L2).

    The scaled error divides by max(1, magnitude): the comparison convention of
    the reference's own bf16 tests (crates/model-serving/tests/direct_mlx/
    sparse_expert_projection.rs:33-44, assert_f32_close scales by
    max(|expected|, 1)).  The magnitude is that of the terms entering the block's
    last addition, |sparse| + |gated shared| (both bf16 values of the oracle), when
    they are given: y can cancel to ~1 while the gated shared term is ~15, and one
    bf16 ulp of that term (0.06) then moves y by more than 2e-2 absolute."""
    g = bf16_to_f32(got_bits).astype(np.float64)
    r = bf16_to_f32(ref_bits).astype(np.float64)
    if not g.size:
        return 0.0, 0.0, 0.0
    d = np.abs(g - r)
    max_abs = float(d.max())
    mag = np.abs(r)
    if terms is not None:
        mag = np.maximum(mag, sum(np.abs(bf16_to_f32(t).astype(np.float64)) for t in terms))
    scaled = float((d / np.maximum(mag, 1.0)).max())
    rel_l2 = float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30))
    return max_abs, scaled, rel_l2


def assert_block_close(got_bits, ref_bits, terms=None):
    """max-abs 2e-2 (scaled, see block_metrics) and rel-L2 1e-3."""
    max_abs, scaled, rel_l2 = block_metrics(got_bits, ref_bits, terms)
    assert scaled <= MAX_ABS and rel_l2 <= REL_L2, (max_abs, scaled, rel_l2)
    return max_abs, scaled, rel_l2


# the oracle's accumulation arithmetic for the kernels of one block call
from oracle.oracle import arith_for_kernels as oracle_arith  # noqa: E402


def reference_metrics(got_bits, ref_bits):
    """The reference's comparison convention (assert_f32_close,
    crates/model-serving/tests/direct_mlx/sparse_expert_projection.rs:32-44):
    |got - expected| <= tol * max(|expected|, 1).  Returns raw max-abs, the
    largest scaled error, relative L2, the count of elements beyond 2e-2 and the
    count of elements that differ at all."""
    g = bf16_to_f32(got_bits).astype(np.float64)
    r = bf16_to_f32(ref_bits).astype(np.float64)
    if not g.size:
        return dict(raw_max_abs=0.0, scaled_max_abs=0.0, rel_l2=0.0, n_beyond=0, n_differ=0, n=0)
    d = np.abs(g - r)
    scaled = d / np.maximum(np.abs(r), 1.0)
    return dict(raw_max_abs=float(d.max()), scaled_max_abs=float(scaled.max()),
                rel_l2=float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30)),
                n_beyond=int((scaled > MAX_ABS).sum()), n_differ=int((d > 0).sum()), n=int(d.size))


def record_parity(case: str, **fields) -> None:
    """Appends one JSON line to $ASTRO_PARITY_LOG (when set): the figures behind
    the committed parity summary."""
    import json
    import os

    path = os.environ.get("ASTRO_PARITY_LOG")
    if not path:
        return
    with open(path, "a") as f:
        f.write(json.dumps(dict(case=case, **fields)) + "\n")


__all__ = ["oracle_arith", "reference_metrics", "record_parity", "to_np_bf16", "to_np_u32", "bf16_tensor", "u32_tensor", "assert_bf16_ulps",
           "block_metrics", "assert_block_close", "bf16_to_f32", "f32_to_bf16", "MAX_ABS",
           "REL_L2"]
