"""Writes tests/golden/tensor_core_steps.npz: single tensor-core accumulation
steps (16 bf16 products + an fp32 accumulator) and the fp32 results a B200
returned for them through astro_moe_tensor_core_probe (tcgen05.mma and
mma.sync).  tests/test_oracle_tc_model.py checks the oracle's model of the step
against these on CPU.  Run on a B200:

    python tests/golden/make_tensor_core_steps.py tests/golden/tensor_core_steps.npz
"""
import ctypes
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from astronomical_b200 import _lib  # noqa: E402


def bf16(v):
    u = np.asarray(v, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def operands(rng, shape, kind):
    if kind == "normal":
        return bf16(rng.normal(0, 1, size=shape))
    lo, hi = (-14, 15) if kind == "wide" else (-3, 4)
    m = rng.uniform(1.0, 2.0, size=shape) * rng.choice([-1, 1], size=shape)
    return bf16(m * np.exp2(rng.integers(lo, hi, size=shape)))


def accumulators(rng, shape, kind):
    m = rng.uniform(1.0, 2.0, size=shape) * rng.choice([-1, 1], size=shape)
    lo, hi = (-20, 21) if kind == "wide" else (-4, 5)
    return (m * np.exp2(rng.integers(lo, hi, size=shape))).astype(np.float32)


def dev(a):
    a = np.ascontiguousarray(a)
    return torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).cuda()


def probe(instruction, A, B, C, n):
    dA, dB, dC = dev(A), dev(B), dev(C)
    dD = torch.empty(C.shape, dtype=torch.float32, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _lib.lib().astro_moe_tensor_core_probe(
        instruction, ctypes.c_void_p(dA.data_ptr()), ctypes.c_void_p(dB.data_ptr()),
        ctypes.c_void_p(dC.data_ptr()), ctypes.c_void_p(dD.data_ptr()), A.shape[0], n, 1, 1,
        ctypes.c_void_p(st.data_ptr()), None)
    torch.cuda.synchronize()
    assert rc == 0 and int(st.item()) == 0
    return dD.cpu().numpy()


def main(out):
    rng = np.random.default_rng(2026)
    a_all, b_all, c_all, d_all, inst = [], [], [], [], []
    for kind, acc in (("wide", "wide"), ("normal", "narrow"), ("narrow", "wide")):
        A = operands(rng, (2, 128, 16), kind)
        B = operands(rng, (2, 16, 16), kind)
        C = accumulators(rng, (2, 128, 16), acc)
        D = probe(0, A, B, C, 16)
        A2 = operands(rng, (64, 16, 16), kind)
        B2 = operands(rng, (64, 8, 16), kind)
        C2 = accumulators(rng, (64, 16, 8), acc)
        D2 = probe(1, A2, B2, C2, 8)
        for i, (AA, BB, CC, DD) in enumerate(((A, B, C, D), (A2, B2, C2, D2))):
            P, M, _ = AA.shape
            N = BB.shape[1]
            pick = rng.choice(P * M * N, 500, replace=False)
            p, r = np.divmod(pick, M * N)
            m, n = np.divmod(r, N)
            a_all.append(AA[p, m])
            b_all.append(BB[p, n])
            c_all.append(CC[p, m, n])
            d_all.append(DD[p, m, n])
            inst.append(np.full(500, i, np.uint8))
    np.savez_compressed(out, a=np.concatenate(a_all), b=np.concatenate(b_all),
                        c=np.concatenate(c_all), d=np.concatenate(d_all),
                        instruction=np.concatenate(inst))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(os.path.dirname(__file__),
                                                            "tensor_core_steps.npz"))
