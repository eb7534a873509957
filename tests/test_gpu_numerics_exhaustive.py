"""The packed arithmetic of the tcgen05 gate/up epilogue against the scalar steps
that match the oracle, over whole input spaces on the device
(astro_moe_numerics_check): the Markstein reciprocal of [1, 2] against the
correctly rounded one, the branch-free exp of x <= 0 against expf_cw, the
bf16x2 multiply against the rounded fp32 product, and the packed SwiGLU against
the scalar SwiGLU for every (gate, up) pair of bf16.  The scalar SwiGLU itself is
bit-exact against the oracle (test_gpu_stages.py), so the chain pins the packed
form to the oracle.
"""
import ctypes

import pytest

torch = pytest.importorskip("torch")

from astronomical_b200 import _lib  # noqa: E402

pytestmark = pytest.mark.gpu

CHECKS = {
    0: "reciprocal of every fp32 in [1, 2]",
    1: "exp of every fp32 x <= 0",
    2: "bf16x2 multiply of every bf16 pair",
    3: "packed SwiGLU of every (gate, up) bf16 pair",
}


@pytest.mark.parametrize("which", sorted(CHECKS))
def test_packed_epilogue_arithmetic_is_exact(which):
    count = torch.zeros(1, dtype=torch.int64, device="cuda")
    first = torch.zeros(1, dtype=torch.int32, device="cuda")
    lib = _lib.lib()
    rc = lib.astro_moe_numerics_check(which, ctypes.c_void_p(count.data_ptr()),
                                      ctypes.c_void_p(first.data_ptr()), None)
    assert rc == 0, lib.astro_moe_last_error()
    torch.cuda.synchronize()
    n, f = int(count.item()), int(first.item()) & 0xffffffff
    assert n == 0, f"{CHECKS[which]}: {n} mismatches, first at input {f:#x}"
    assert f == 0xffffffff


def test_numerics_check_rejects_bad_arguments():
    lib = _lib.lib()
    count = torch.zeros(1, dtype=torch.int64, device="cuda")
    assert lib.astro_moe_numerics_check(7, ctypes.c_void_p(count.data_ptr()),
                                        ctypes.c_void_p(count.data_ptr()), None) != 0
    assert lib.astro_moe_numerics_check(0, None, None, None) != 0
