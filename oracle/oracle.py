"""ctypes wrapper around oracle/liboracle.so -- the CPU restatement of the
reference's sorted-MoE block.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and by
the CPU-baseline leg of bench.py, always as the checker.  The product package
(astronomical_b200) never imports this module.

Arrays are numpy; bf16 values travel as uint16 bit patterns.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

BF16, F16, F32 = 1, 2, 3
OK, ERR_INVALID_ARGUMENT, ERR_DUPLICATE_SLOT, ERR_OUT_OF_RANGE_SLOT = 0, 1, 8, 9

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        src = os.path.join(_HERE, "astro_oracle.c")
        if not os.path.exists(_LIB_PATH) or (
            os.path.exists(src) and os.path.getmtime(src) > os.path.getmtime(_LIB_PATH)
        ):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


def _declare(l: ctypes.CDLL) -> None:
    P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    l.ao_f32_to_bf16.argtypes, l.ao_f32_to_bf16.restype = [ctypes.c_float], ctypes.c_uint16
    l.ao_bf16_to_f32.argtypes, l.ao_bf16_to_f32.restype = [ctypes.c_uint16], ctypes.c_float
    l.ao_expf.argtypes, l.ao_expf.restype = [ctypes.c_float], ctypes.c_float
    l.ao_sigmoidf.argtypes, l.ao_sigmoidf.restype = [ctypes.c_float], ctypes.c_float
    l.ao_expf_batch.argtypes, l.ao_expf_batch.restype = [P, I64, P], None
    l.ao_matmul_bf16_nt.argtypes, l.ao_matmul_bf16_nt.restype = [P, P, I64, I64, I64, P], None
    l.ao_route_experts.argtypes = [P, I, I64, I, I, I, P, P]
    l.ao_route_experts.restype = I
    l.ao_sort_expert_assignments.argtypes = [P, I64, I, I, P, P, P, P, P]
    l.ao_sort_expert_assignments.restype = I
    l.ao_invert_assignment_order.argtypes, l.ao_invert_assignment_order.restype = [P, I64, P], I
    l.ao_dequantize_affine.argtypes = [P, P, P, I64, I, I, I, P]
    l.ao_dequantize_affine.restype = I
    l.ao_gather_qmm.argtypes = [P, P, P, I64, I, P, P, P, I, I, I, I, P]
    l.ao_gather_qmm.restype = I
    l.ao_swiglu.argtypes, l.ao_swiglu.restype = [P, P, I64, P], None
    l.ao_sorted_expert_weighted_sum.argtypes = [P, I, P, P, I, I64, I, I64, P]
    l.ao_sorted_expert_weighted_sum.restype = I
    l.ao_unsorted_expert_weighted_sum.argtypes = [P, I, P, I, I64, I, I64, P]
    l.ao_unsorted_expert_weighted_sum.restype = I
    l.ao_combine_sparse_and_shared.argtypes = [P, P, P, I, I64, I64, P]
    l.ao_combine_sparse_and_shared.restype = None
    l.ao_moe_block_forward.argtypes = [P, P, I64, P, I64, P, P, P, P, I]
    l.ao_moe_block_forward.restype = I
    l.ao_moe_block_forward_terms.argtypes = [P, P, I64, P, I64, P, P, P, P, P, P, I]
    l.ao_moe_block_forward_terms.restype = I
    l.ao_tc_step.argtypes, l.ao_tc_step.restype = [ctypes.c_float, P, P], ctypes.c_float
    l.ao_route_laguna_experts.argtypes = [P, I, I64, I, I, P, ctypes.c_float, I, P, P]
    l.ao_route_laguna_experts.restype = I
    l.ao_sigmoid_plainf.argtypes, l.ao_sigmoid_plainf.restype = [ctypes.c_float], ctypes.c_float
    l.ao_tanhf.argtypes, l.ao_tanhf.restype = [ctypes.c_float], ctypes.c_float
    l.ao_dot.argtypes, l.ao_dot.restype = [P, P, I64, I], ctypes.c_float
    l.ao_tc_chain_batch.argtypes, l.ao_tc_chain_batch.restype = [P, P, P, I64, I64, P], None
    l.ao_matmul_bf16_nt_mode.argtypes = [P, P, I64, I64, I64, I, P]
    l.ao_matmul_bf16_nt_mode.restype = None


class BlockWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "hidden", "experts", "top_k", "intermediate", "shared_intermediate", "group", "bits",
        "normalize")] + [(n, ctypes.c_void_p) for n in (
            "router_w",
            "gate_q", "gate_s", "gate_b", "up_q", "up_s", "up_b", "down_q", "down_s", "down_b",
            "sgate_q", "sgate_s", "sgate_b", "sup_q", "sup_s", "sup_b", "sdown_q", "sdown_s",
            "sdown_b", "shared_gate_w")] + [
        ("proj_bits", ctypes.c_int * 6), ("proj_group", ctypes.c_int * 6),
        ("router_q", ctypes.c_void_p), ("router_s", ctypes.c_void_p), ("router_b", ctypes.c_void_p),
        ("router_bits", ctypes.c_int), ("router_group", ctypes.c_int),
        ("shared_gate_q", ctypes.c_void_p), ("shared_gate_s", ctypes.c_void_p),
        ("shared_gate_b", ctypes.c_void_p), ("shared_gate_bits", ctypes.c_int),
        ("shared_gate_group", ctypes.c_int), ("arith", ctypes.c_int * 6),
        ("router_kind", ctypes.c_int), ("router_logit_softcap", ctypes.c_float),
        ("routed_scaling_factor", ctypes.c_float), ("router_correction_bias", ctypes.c_void_p)]


# accumulation modes of a dot product (AO_DOT_* in astro_oracle.h)
DOT = dict(seq=0, tc=1, tc_quarters=2, slices8=3, lanes8=4, decode32=5, decode16=6, chunk32=7)
# the order of the six modes a block takes
ARITH_STAGES = ("router", "gate_logit", "gate_up", "down", "shared_gate_up", "shared_down")
PROJ_NAMES = ("gate", "up", "down", "sgate", "sup", "sdown")

# Accumulation arithmetic of each kernel of libastro_moe, as AO_DOT_* modes: the
# parity tests ask the library which kernels a block call ran
# (astro_moe_ctx_last_block_path) and run the oracle with the same arithmetic,
# so every stage compares bit for bit.
_ROUTER_ARITH = {"tcgen05_gemm": "tc", "fused_decode": "slices8", "router_gemv": "slices8",
                 "simt_gemm": "seq"}
_GATE_LOGIT_ARITH = {"fused_decode": "slices8", "route": "lanes8", "none": "seq"}
_EXPERT_ARITH = {"tcgen05_gemm": ("tc", "tc"), "fused_decode": ("tc_quarters", "tc_quarters"),
                 "decode_gemv": ("decode32", "decode16"), "grouped_gemv": ("chunk32", "chunk32"),
                 "none": ("seq", "seq")}


def arith_for_kernels(path: dict) -> dict:
    """Oracle accumulation modes for a block call's kernels (router, gate_logit,
    experts, shared_expert names as the library reports them)."""
    gu, dn = _EXPERT_ARITH[path["experts"]]
    sgu, sdn = _EXPERT_ARITH[path["shared_expert"]]
    return dict(router=_ROUTER_ARITH[path["router"]], gate_logit=_GATE_LOGIT_ARITH[path["gate_logit"]],
                gate_up=gu, down=dn, shared_gate_up=sgu, shared_down=sdn)


def arith_codes(arith) -> list:
    """arith: None (all canonical), a dict stage -> mode name, or a 6-sequence."""
    if arith is None:
        return [0] * 6
    if isinstance(arith, dict):
        unknown = set(arith) - set(ARITH_STAGES)
        if unknown:
            raise ValueError(f"unknown stages {sorted(unknown)}")
        vals = [arith.get(k, "seq") for k in ARITH_STAGES]
    else:
        vals = list(arith)
    return [DOT[a] if isinstance(a, str) else int(a) for a in vals]


def _p(a):
    return None if a is None else a.ctypes.data


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ---------------------------------------------------------------- bf16 helpers
def f32_to_bf16(a) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def dtype_code(a: np.ndarray, bf16: bool) -> int:
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.float16:
        return F16
    if a.dtype == np.uint16 and bf16:
        return BF16
    raise TypeError(f"unsupported dtype {a.dtype}")


# ---------------------------------------------------------------- functions
def expf(x) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty_like(x)
    lib().ao_expf_batch(_p(x), x.size, _p(out))
    return out


def _mode(mode) -> int:
    return DOT[mode] if isinstance(mode, str) else int(mode)


def matmul_bf16_nt(x, w, mode="seq") -> np.ndarray:
    """bf16(x . w^T) with the accumulation `mode` (a DOT name)."""
    x, w = _c(x, np.uint16), _c(w, np.uint16)
    out = np.empty((x.shape[0], w.shape[0]), np.uint16)
    lib().ao_matmul_bf16_nt_mode(_p(x), _p(w), x.shape[0], w.shape[0], x.shape[1], _mode(mode),
                                 _p(out))
    return out


def tc_step(c: float, a, b) -> float:
    """One tensor-core accumulation step over 16 bf16-valued products."""
    a, b = _c(a, np.float32), _c(b, np.float32)
    assert a.size == 16 and b.size == 16
    return float(np.float32(lib().ao_tc_step(float(np.float32(c)), _p(a), _p(b))))


def tc_chain(a, b, c=None) -> np.ndarray:
    """a, b float32 [count, n] (bf16 values): the tensor-core step chain per row,
    from c [count] (None: zero)."""
    a, b = _c(a, np.float32), _c(b, np.float32)
    count, n = a.shape
    cc = None if c is None else _c(c, np.float32)
    out = np.empty(count, np.float32)
    lib().ao_tc_chain_batch(_p(a), _p(b), _p(cc), count, n, _p(out))
    return out


def dot(a, b, mode="seq") -> float:
    a, b = _c(a, np.float32), _c(b, np.float32)
    return float(np.float32(lib().ao_dot(_p(a), _p(b), a.size, _mode(mode))))


def route_experts(logits, top_k: int, normalize: bool = True, bf16: bool = True):
    """logits [T, E] (uint16 bf16 bits, float16 or float32) -> (ids u32 [T,K], scores)."""
    logits = np.ascontiguousarray(logits)
    code = dtype_code(logits, bf16)
    T, E = logits.shape
    ids = np.empty((T, top_k), np.uint32)
    scores = np.empty((T, top_k), logits.dtype)
    st = lib().ao_route_experts(_p(logits), code, T, E, top_k, int(normalize), _p(ids), _p(scores))
    if st != OK:
        raise ValueError(f"route_experts status {st}")
    return ids, scores


def route_laguna_experts(logits, top_k: int, correction_bias=None, softcap: float = 0.0,
                         normalize: bool = True, bf16: bool = True):
    """Laguna router (laguna/moe/router_selection.rs:47-107): logits [T, E] ->
    (ids u32 [T, K], fp32 original scores [T, K])."""
    logits = np.ascontiguousarray(logits)
    code = dtype_code(logits, bf16)
    T, E = logits.shape
    ids = np.empty((T, top_k), np.uint32)
    scores = np.empty((T, top_k), np.float32)
    b = None if correction_bias is None else _c(correction_bias, np.float32)
    st = lib().ao_route_laguna_experts(_p(logits), code, T, E, top_k, _p(b), float(softcap),
                                       int(normalize), _p(ids), _p(scores))
    if st != OK:
        raise ValueError(f"route_laguna_experts status {st}")
    return ids, scores


def sort_expert_assignments(ids, experts: int):
    ids = _c(ids, np.uint32)
    T, K = ids.shape if ids.ndim == 2 else (ids.shape[0], 1)
    n = T * K
    outs = [np.empty(max(n, 0), np.uint32) for _ in range(4)]
    offs = np.empty(experts + 1, np.uint32)
    st = lib().ao_sort_expert_assignments(_p(ids), T, K, experts, *[_p(o) for o in outs], _p(offs))
    if st != OK:
        raise ValueError(f"sort_expert_assignments status {st}")
    order, inverse, sorted_ids, sorted_tokens = outs
    return dict(sorted_order=order, inverse_order=inverse, sorted_ids=sorted_ids,
                sorted_tokens=sorted_tokens, expert_offsets=offs)


def invert_assignment_order(order):
    order = _c(order, np.uint32)
    inv = np.empty_like(order)
    st = lib().ao_invert_assignment_order(_p(order), order.size, _p(inv))
    return st, inv


def dequantize_affine(packed, scales, biases, group: int, bits: int) -> np.ndarray:
    packed, scales, biases = _c(packed, np.uint32), _c(scales, np.uint16), _c(biases, np.uint16)
    in_features = packed.shape[-1] * 32 // bits
    rows = int(np.prod(packed.shape[:-1]))
    out = np.empty(packed.shape[:-1] + (in_features,), np.uint16)
    st = lib().ao_dequantize_affine(_p(packed), _p(scales), _p(biases), rows, in_features, group,
                                    bits, _p(out))
    if st != OK:
        raise ValueError(f"dequantize_affine status {st}")
    return out


def gather_qmm(x, packed, scales, biases, group: int, bits: int, rhs_experts=None, lhs_rows=None):
    """y[n] = x[lhs_rows[n]] . dequant(W[rhs_experts[n]])^T  (bf16 in, bf16 out)."""
    x = _c(x, np.uint16)
    packed, scales, biases = _c(packed, np.uint32), _c(scales, np.uint16), _c(biases, np.uint16)
    if packed.ndim == 2:
        packed, scales, biases = packed[None], scales[None], biases[None]
    E, out_f, words = packed.shape
    in_f = words * 32 // bits
    rhs = None if rhs_experts is None else _c(rhs_experts, np.uint32)
    lhs = None if lhs_rows is None else _c(lhs_rows, np.uint32)
    n = rhs.size if rhs is not None else (lhs.size if lhs is not None else x.shape[0])
    y = np.empty((n, out_f), np.uint16)
    st = lib().ao_gather_qmm(_p(x), _p(lhs), _p(rhs), n, in_f, _p(packed), _p(scales), _p(biases),
                             E, out_f, group, bits, _p(y))
    if st != OK:
        raise ValueError(f"gather_qmm status {st}")
    return y


def swiglu(gate, up) -> np.ndarray:
    gate, up = _c(gate, np.uint16), _c(up, np.uint16)
    out = np.empty_like(gate)
    lib().ao_swiglu(_p(gate), _p(up), gate.size, _p(out))
    return out


def sorted_expert_weighted_sum(sorted_outputs, inverse_order, scores, bf16=True):
    so = np.ascontiguousarray(sorted_outputs)
    sc = np.ascontiguousarray(scores)
    inv = _c(inverse_order, np.uint32)
    T, K = sc.shape
    D = so.shape[-1]
    out = np.empty((T, D), so.dtype)
    st = lib().ao_sorted_expert_weighted_sum(_p(so), dtype_code(so, bf16), _p(inv), _p(sc),
                                             dtype_code(sc, bf16), T, K, D, _p(out))
    if st != OK:
        raise ValueError(f"sorted_expert_weighted_sum status {st}")
    return out


def unsorted_expert_weighted_sum(outputs, scores, bf16=True):
    o = np.ascontiguousarray(outputs)
    sc = np.ascontiguousarray(scores)
    T, K = sc.shape
    D = o.shape[-1]
    out = np.empty((T, D), o.dtype)
    st = lib().ao_unsorted_expert_weighted_sum(_p(o), dtype_code(o, bf16), _p(sc),
                                               dtype_code(sc, bf16), T, K, D, _p(out))
    if st != OK:
        raise ValueError(f"unsorted_expert_weighted_sum status {st}")
    return out


def combine_sparse_and_shared(sparse, shared, gate_logits, bf16=True):
    s, sh, g = (np.ascontiguousarray(a) for a in (sparse, shared, gate_logits))
    T, D = s.shape
    out = np.empty_like(s)
    lib().ao_combine_sparse_and_shared(_p(s), _p(sh), _p(g), dtype_code(s, bf16), T, D, _p(out))
    return out


def moe_block_forward(weights: dict, x, token_subset=None, logits_override=None,
                      num_threads: int = 0, terms: bool = False, arith=None):
    """Whole block on CPU.  weights: dict from astronomical_b200.synthetic (MLX layout).
    Returns (y bf16 [n, H], ids [n, K], scores bf16 [n, K]) for the listed tokens, plus
    (sparse, gated_shared) -- the bf16 terms of the final addition -- when terms=True.
    arith: accumulation modes per stage (see arith_codes); None = canonical order.
    Optional weight keys: "<proj>_bits" / "<proj>_group" per projection
    (gate, up, down, sgate, sup, sdown), an affine router ("router_q", "router_s",
    "router_b", "router_bits", "router_group") and an affine shared-expert gate
    ("shared_gate_q", .._s, .._b, .._bits, .._group)."""
    cfg = weights["config"]
    x = _c(x, np.uint16)
    T, H = x.shape
    keep = []

    def arr(name, dtype):
        a = weights.get(name)
        if a is None:
            return None
        a = _c(a, dtype)
        keep.append(a)
        return a.ctypes.data

    bw = BlockWeights(
        hidden=H, experts=cfg["experts"], top_k=cfg["top_k"], intermediate=cfg["intermediate"],
        shared_intermediate=cfg.get("shared_intermediate", 0), group=cfg["group"],
        bits=cfg["bits"], normalize=int(cfg.get("normalize", True)),
        router_w=arr("router_w", np.uint16),
        gate_q=arr("gate_q", np.uint32), gate_s=arr("gate_s", np.uint16),
        gate_b=arr("gate_b", np.uint16),
        up_q=arr("up_q", np.uint32), up_s=arr("up_s", np.uint16), up_b=arr("up_b", np.uint16),
        down_q=arr("down_q", np.uint32), down_s=arr("down_s", np.uint16),
        down_b=arr("down_b", np.uint16),
        sgate_q=arr("sgate_q", np.uint32), sgate_s=arr("sgate_s", np.uint16),
        sgate_b=arr("sgate_b", np.uint16),
        sup_q=arr("sup_q", np.uint32), sup_s=arr("sup_s", np.uint16), sup_b=arr("sup_b", np.uint16),
        sdown_q=arr("sdown_q", np.uint32), sdown_s=arr("sdown_s", np.uint16),
        sdown_b=arr("sdown_b", np.uint16),
        shared_gate_w=arr("shared_gate_w", np.uint16),
        proj_bits=(ctypes.c_int * 6)(*[int(weights.get(f"{n}_bits", 0)) for n in PROJ_NAMES]),
        proj_group=(ctypes.c_int * 6)(*[int(weights.get(f"{n}_group", 0)) for n in PROJ_NAMES]),
        router_q=arr("router_q", np.uint32), router_s=arr("router_s", np.uint16),
        router_b=arr("router_b", np.uint16), router_bits=int(weights.get("router_bits", 0)),
        router_group=int(weights.get("router_group", 0)),
        shared_gate_q=arr("shared_gate_q", np.uint32), shared_gate_s=arr("shared_gate_s", np.uint16),
        shared_gate_b=arr("shared_gate_b", np.uint16),
        shared_gate_bits=int(weights.get("shared_gate_bits", 0)),
        shared_gate_group=int(weights.get("shared_gate_group", 0)),
        arith=(ctypes.c_int * 6)(*arith_codes(arith)),
        router_kind=1 if cfg.get("router") == "laguna" else 0,
        router_logit_softcap=float(cfg.get("router_logit_softcap", 0.0)),
        routed_scaling_factor=float(cfg.get("routed_scaling_factor", 1.0)),
        router_correction_bias=arr("router_correction_bias", np.float32))
    sub = None if token_subset is None else _c(token_subset, np.int64)
    n = T if sub is None else sub.size
    K = cfg["top_k"]
    y = np.empty((n, H), np.uint16)
    ids = np.empty((n, K), np.uint32)
    sc = np.empty((n, K), np.float32 if cfg.get("router") == "laguna" else np.uint16)
    lo = None if logits_override is None else _c(logits_override, np.uint16)
    sp = np.empty((n, H), np.uint16) if terms else None
    sg = np.empty((n, H), np.uint16) if terms else None
    st = lib().ao_moe_block_forward_terms(ctypes.byref(bw), _p(x), T, _p(sub), n, _p(lo), _p(y),
                                          _p(ids), _p(sc), _p(sp), _p(sg), num_threads)
    if st != OK:
        raise ValueError(f"moe_block_forward status {st}")
    if terms:
        return y, ids, sc, sp, sg
    return y, ids, sc
