"""The oracle's model of the tensor cores' fp32 accumulation (ao_tc_step, used by
the AO_DOT_TC and AO_DOT_TC_QUARTERS modes) against the hardware.

Both instructions the library's GEMMs issue (tcgen05.mma kind::f16 and mma.sync
m16n8k16, bf16 operands) run D = C + A.B^T through astro_moe_tensor_core_probe
on seeded operands, and every fp32 result must equal the model's bit for bit.
Operands cover exponents of +-14 (products and sums spread over ~60 binades,
where truncation and cancellation show), N(0,1) values (the block's regime),
accumulators far above and below the products, chains of up to 1024 K, and the
case without an initial accumulator.
"""
import ctypes
import zlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O  # noqa: E402
from astronomical_b200 import _lib  # noqa: E402

pytestmark = pytest.mark.gpu


def _operands(rng, shape, kind):
    if kind == "normal":
        return O.f32_to_bf16(rng.normal(0, 1, size=shape).astype(np.float32))
    lo, hi = (-14, 15) if kind == "wide" else (-3, 4)
    m = rng.uniform(1.0, 2.0, size=shape) * rng.choice([-1, 1], size=shape)
    return O.f32_to_bf16((m * np.exp2(rng.integers(lo, hi, size=shape))).astype(np.float32))


def _acc(rng, shape, kind):
    m = rng.uniform(1.0, 2.0, size=shape) * rng.choice([-1, 1], size=shape)
    lo, hi = (-20, 21) if kind == "wide" else (-4, 5)
    return (m * np.exp2(rng.integers(lo, hi, size=shape))).astype(np.float32)


def _dev(a):
    a = np.ascontiguousarray(a)
    return torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).cuda()


def _run(instruction, A, B, C, n, k16, accumulate):
    dA, dB, dC = _dev(A), _dev(B), _dev(C)
    dD = torch.full(C.shape, float("nan"), dtype=torch.float32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _lib.lib().astro_moe_tensor_core_probe(
        instruction, ctypes.c_void_p(dA.data_ptr()), ctypes.c_void_p(dB.data_ptr()),
        ctypes.c_void_p(dC.data_ptr()), ctypes.c_void_p(dD.data_ptr()), A.shape[0], n, k16,
        accumulate, ctypes.c_void_p(status.data_ptr()), None)
    assert rc == 0, _lib.lib().astro_moe_last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return dD.cpu().numpy()


def _model(A, B, C, accumulate):
    """Model result for every (problem, row, column): the step chain over K."""
    P, M, K = A.shape
    N = B.shape[1]
    a = np.broadcast_to(O.bf16_to_f32(A)[:, :, None, :], (P, M, N, K)).reshape(-1, K)
    b = np.broadcast_to(O.bf16_to_f32(B)[:, None, :, :], (P, M, N, K)).reshape(-1, K)
    c = C.reshape(-1) if accumulate else None
    return O.tc_chain(a, b, c).reshape(P, M, N)


CASES = [  # (operand kind, accumulator kind or None, k16)
    ("wide", "wide", 1), ("wide", None, 1), ("normal", "narrow", 1), ("narrow", "wide", 1),
    ("wide", "wide", 4), ("normal", None, 16), ("wide", "wide", 16)]


@pytest.mark.parametrize("kind,acc,k16", CASES)
def test_tcgen05_mma_matches_the_model(kind, acc, k16):
    rng = np.random.default_rng(zlib.crc32(f"tc{kind}{acc}{k16}".encode()))
    P, N, K = 24, (32 if k16 == 4 else 16), 16 * k16
    A = _operands(rng, (P, 128, K), kind)
    B = _operands(rng, (P, N, K), kind)
    C = _acc(rng, (P, 128, N), acc or "narrow")
    got = _run(0, A, B, C, N, k16, int(acc is not None))
    want = _model(A, B, C, acc is not None)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        int((got.view(np.uint32) != want.view(np.uint32)).sum())


@pytest.mark.parametrize("kind,acc,k16", [c for c in CASES if c[1] is not None] +
                         [("normal", "narrow", 64)])
def test_mma_sync_matches_the_model(kind, acc, k16):
    rng = np.random.default_rng(zlib.crc32(f"mma{kind}{acc}{k16}".encode()))
    P, K = (2048 if k16 <= 4 else 256), 16 * k16
    A = _operands(rng, (P, 16, K), kind)
    B = _operands(rng, (P, 8, K), kind)
    C = _acc(rng, (P, 16, 8), acc)
    got = _run(1, A, B, C, 8, k16, 1)
    want = _model(A, B, C, True)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        int((got.view(np.uint32) != want.view(np.uint32)).sum())
