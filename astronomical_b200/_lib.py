"""ctypes binding of libastro_moe.so (the C ABI in include/astro_moe.h).

The library is built in-tree by astronomical_b200.build; there is no fallback:
if the shared object is missing or fails to load, every call raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libastro_moe.so")

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_CUDA = 2
ERR_OUT_OF_MEMORY = 3
ERR_UNSUPPORTED = 4
ERR_DEVICE_STATUS = 5
ERR_NOT_REGISTERED = 6
ERR_NCCL = 7
ERR_DUPLICATE_SLOT = 8
ERR_OUT_OF_RANGE_SLOT = 9
ERR_MEMORY_LIMIT = 10

DTYPE_BF16, DTYPE_F16, DTYPE_F32 = 1, 2, 3


class AstroMoeError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[status {status}] {message}")
        self.status = status


class Options(ctypes.Structure):
    _fields_ = [("max_tokens", ctypes.c_int64), ("sorted_threshold", ctypes.c_int32),
                ("use_tensor_cores", ctypes.c_int32), ("decode_max_tokens", ctypes.c_int64),
                ("decode_fused", ctypes.c_int64), ("reserved", ctypes.c_int64 * 4)]


class Affine(ctypes.Structure):
    _fields_ = [("packed", ctypes.c_void_p), ("scales", ctypes.c_void_p),
                ("biases", ctypes.c_void_p), ("bits", ctypes.c_int32),
                ("group_size", ctypes.c_int32)]


class LayerWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "hidden", "experts", "top_k", "intermediate", "shared_intermediate", "group_size",
        "bits", "normalize_top_k", "gate_up_fused")] + [
        ("router_weight", ctypes.c_void_p), ("gate", Affine), ("up", Affine), ("down", Affine),
        ("shared_gate", Affine), ("shared_up", Affine), ("shared_down", Affine),
        ("shared_expert_gate", ctypes.c_void_p), ("router_affine", Affine),
        ("shared_expert_gate_affine", Affine), ("router_kind", ctypes.c_int32),
        ("router_logit_softcap", ctypes.c_float), ("routed_scaling_factor", ctypes.c_float),
        ("router_correction_bias", ctypes.c_void_p)]

ROUTER_SOFTMAX, ROUTER_SIGMOID = 0, 1
PAGER_LRU, PAGER_DEMAND = 0, 1


class BlockTaps(ctypes.Structure):
    _fields_ = [("router_logits", ctypes.c_void_p), ("selected_indices", ctypes.c_void_p),
                ("selected_scores", ctypes.c_void_p), ("expert_offsets", ctypes.c_void_p)]


# kernels a block call ran (ASTRO_MOE_KERNEL_*)
KERNEL_NAMES = {0: "none", 1: "tcgen05_gemm", 2: "fused_decode", 3: "decode_gemv",
                4: "grouped_gemv", 5: "router_gemv", 6: "simt_gemm", 7: "route"}


class BlockPath(ctypes.Structure):
    _fields_ = [("router", ctypes.c_int32), ("gate_logit", ctypes.c_int32),
                ("experts", ctypes.c_int32), ("shared_expert", ctypes.c_int32)]

    def as_dict(self):
        return {n: KERNEL_NAMES.get(getattr(self, n), str(getattr(self, n))) for n, _ in self._fields_}


class PagerStats(ctypes.Structure):
    _fields_ = [("lookups", ctypes.c_int64), ("hits", ctypes.c_int64), ("misses", ctypes.c_int64),
                ("evictions", ctypes.c_int64), ("bytes_h2d", ctypes.c_int64),
                ("copy_ms", ctypes.c_double), ("resident_pages", ctypes.c_int64),
                ("capacity_pages", ctypes.c_int64), ("calls", ctypes.c_int64),
                ("split_calls", ctypes.c_int64), ("copy_failures", ctypes.c_int64)]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


class Attribution(ctypes.Structure):
    _fields_ = [("calls", ctypes.c_int64), ("kernel_launches", ctypes.c_int64),
                ("router_projection_ms", ctypes.c_double),
                ("assignment_preparation_ms", ctypes.c_double), ("gate_up_ms", ctypes.c_double),
                ("down_ms", ctypes.c_double), ("weighted_reduction_ms", ctypes.c_double)]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


_lib = None

# every entry point of include/astro_moe.h: (name, argtypes)
_P, _I32, _I64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
SIGNATURES = {
    "astro_moe_last_error": ([], ctypes.c_char_p),
    "astro_moe_abi_version": ([], ctypes.c_int),
    "astro_moe_device_status": ([_I32, _P, _I32], ctypes.c_int),
    "astro_moe_tensor_core_probe": ([_I32, _P, _P, _P, _P, _I64, _I32, _I32, _I32, _P, _P],
                                    ctypes.c_int),
    "astro_moe_wait_probe": ([_I32, _P, ctypes.c_uint32, _I64, _P, _P, _P], ctypes.c_int),
    "astro_moe_numerics_check": ([_I32, _P, _P, _P], ctypes.c_int),
    "astro_moe_route_experts": ([_P, _I32, _I64, _I32, _I32, _I32, _P, _P, _P], ctypes.c_int),
    "astro_moe_route_laguna_experts": ([_P, _I32, _I64, _I32, _I32, _P, ctypes.c_double, _I32,
                                        _P, _P, _P], ctypes.c_int),
    "astro_moe_sort_expert_assignments": ([_P, _I64, _I32, _I32, _P, _P, _P, _P, _P, _P],
                                          ctypes.c_int),
    "astro_moe_sort_expert_assignments_no_alloc": (
        [_P, _I64, _I32, _I32, _P, _P, _P, _P, _P, _P, _P], ctypes.c_int),
    "astro_moe_take_rows": ([_P, _I64, _I32, _P, _I64, _P, _P], ctypes.c_int),
    "astro_moe_gather_qmm": ([_P, _I64, _I32, _P, _P, _I64, _P, _P, _P, _I32, _I32, _I32, _I32,
                              _I32, _P, _P], ctypes.c_int),
    "astro_moe_quantized_matmul": ([_P, _I64, _I32, _P, _P, _P, _I32, _I32, _I32, _P, _P],
                                   ctypes.c_int),
    "astro_moe_dequantize_affine": ([_P, _P, _P, _I64, _I32, _I32, _I32, _P, _P], ctypes.c_int),
    "astro_moe_swiglu": ([_P, _P, _I64, _P, _P], ctypes.c_int),
    "astro_moe_sorted_expert_weighted_sum": ([_P, _I32, _P, _P, _I32, _I64, _I32, _I64, _P, _P],
                                             ctypes.c_int),
    "astro_moe_unsorted_expert_weighted_sum": ([_P, _I32, _P, _I32, _I64, _I32, _I64, _P, _P],
                                               ctypes.c_int),
    "astro_moe_combine_sparse_and_shared": ([_P, _P, _P, _I32, _I64, _I64, _P, _P], ctypes.c_int),
    "astro_moe_invert_assignment_order": ([_P, _I64, _P], ctypes.c_int),
    "astro_moe_ctx_create": ([_I32, _P, ctypes.POINTER(Options), ctypes.POINTER(_P)],
                             ctypes.c_int),
    "astro_moe_ctx_destroy": ([_P], ctypes.c_int),
    "astro_moe_ctx_set_stream": ([_P, _P], ctypes.c_int),
    "astro_moe_ctx_synchronize": ([_P], ctypes.c_int),
    "astro_moe_register_layer": ([_P, _I32, ctypes.POINTER(LayerWeights)], ctypes.c_int),
    "astro_moe_block_forward": ([_P, _I32, _P, _I64, _P], ctypes.c_int),
    "astro_moe_block_forward_taps": ([_P, _I32, _P, _I64, _P, ctypes.POINTER(BlockTaps)],
                                     ctypes.c_int),
    "astro_moe_block_forward_host": ([_P, _I32, _P, _I64, _P], ctypes.c_int),
    "astro_moe_block_forward_host_async": ([_P, _I32, _P, _I64, _P], ctypes.c_int),
    "astro_moe_host_synchronize": ([_P], ctypes.c_int),
    "astro_moe_ctx_last_block_path": ([_P, ctypes.POINTER(BlockPath)], ctypes.c_int),
    "astro_moe_ctx_set_attribution": ([_P, _I32], ctypes.c_int),
    "astro_moe_ctx_read_attribution": ([_P, ctypes.POINTER(Attribution), _I32], ctypes.c_int),
    "astro_moe_ep_register_layer": ([_P, _I32, ctypes.POINTER(LayerWeights), _I32, _I32],
                                    ctypes.c_int),
    "astro_moe_ep_dispatch": ([_P, _I32, _P, _I64, _P, _P], ctypes.c_int),
    "astro_moe_ep_experts": ([_P, _I32, _P, _P, _I32, _I64, _P, _I64, _P], ctypes.c_int),
    "astro_moe_ep_combine": ([_P, _I32, _P, _I64, _P], ctypes.c_int),
    "astro_moe_ep_exchange_create": ([_P, _I32, _I32, _I32, _I64, _I64, _P], ctypes.c_int),
    "astro_moe_ep_exchange_connect": ([_P, _P], ctypes.c_int),
    "astro_moe_ep_exchange_buffers": ([_P, ctypes.POINTER(ctypes.c_void_p),
                                       ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "astro_moe_ep_route": ([_P, _I32, _P, _I64, _P], ctypes.c_int),
    "astro_moe_ep_push": ([_P, _I32, _P, _I64, _P, _P], ctypes.c_int),
    "astro_moe_ep_experts_push": ([_P, _I32, _P, _I64, _P, _I64, _P, _P], ctypes.c_int),
    "astro_moe_ep_post_counts": ([_P, _I32, _P], ctypes.c_int),
    "astro_moe_ep_push_dev": ([_P, _I32, _P, _I64], ctypes.c_int),
    "astro_moe_ep_experts_dev": ([_P, _I32, _P, _I64], ctypes.c_int),
    "astro_moe_ep_exchange_counts": ([_P, _P], ctypes.c_int),
    "astro_moe_page_bytes": ([_I32, _I32, _I32, _I32], ctypes.c_int64),
    "astro_moe_pager_create": ([_P, _I32, _I32, _I32, _I32, _I32, _I32, _P, _I64,
                                ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "astro_moe_pager_destroy": ([_P], ctypes.c_int),
    "astro_moe_pager_set_policy": ([_P, _I32], ctypes.c_int),
    "astro_moe_pager_inject_copy_failures": ([_P, _I64], ctypes.c_int),
    "astro_moe_pager_read_stats": ([_P, ctypes.POINTER(PagerStats), _I32], ctypes.c_int),
    "astro_moe_register_paged_layer": ([_P, _I32, ctypes.POINTER(LayerWeights), _P], ctypes.c_int),
    "astro_moe_paged_block_forward": ([_P, _I32, _P, _I64, _P], ctypes.c_int),
}


def lib() -> ctypes.CDLL:
    """Load the in-tree shared object (raises if it is absent: no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing; run astronomical_b200.build.build()")
        l = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(l, name)
            fn.argtypes, fn.restype = args, res
        _lib = l
    return _lib


def check(status: int) -> None:
    if status != OK:
        msg = lib().astro_moe_last_error()
        raise AstroMoeError(status, msg.decode() if msg else "")
