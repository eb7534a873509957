"""Host-side mirror of the reference's sorted-MoE operators, over the C ABI.

Function names, argument meaning and error behaviour follow the reference
(paths relative to the reference project root):

* ``qwen3_5_moe_route_experts``      -- qwen3_5_moe/model/routing.rs:16-49
* ``sort_expert_assignments``        -- sparse_experts/assignment_sort.rs:24-97
* ``restore_expert_assignment_order``-- sparse_experts/assignment_sort.rs:103-138
* ``invert_assignment_order``        -- sparse_experts/assignment_permutation.rs:10-41
* ``gather_expert_projection``       -- sparse_experts/gathered_projection.rs:84-131
* ``sorted_expert_weighted_sum``     -- sparse_experts/weighted_sum.rs:75-92
* ``unsorted_expert_weighted_sum``   -- sparse_experts/weighted_sum.rs:46-60
* ``apply_compiled_swiglu``          -- runtime-integration/src/mlx_compiled_swiglu.rs:32-42
* ``qwen3_5_moe_combine_experts``    -- qwen3_5_moe/model/output_combination.rs:7-32
* ``Qwen3_5MoEBlock.forward``        -- Qwen3_5Model::forward_qwen3_5_moe, forward.rs:19-127

Device memory, streams and dtypes come from torch (plumbing only); all compute
runs in libastro_moe.so.  Errors raise ``AstroMoeError`` (the analogue of
MlxRuntimeError) or ``SparseExpertError``.
"""
from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np
import torch

from . import _lib
from ._lib import AstroMoeError, check

__all__ = [
    "AstroMoeError", "SparseExpertError", "ExpertAssignmentOrder", "AffineProjection",
    "SortedExpertAssignments", "qwen3_5_moe_route_experts", "sort_expert_assignments",
    "restore_expert_assignment_order", "invert_assignment_order", "gather_expert_projection",
    "sorted_expert_weighted_sum", "unsorted_expert_weighted_sum", "apply_compiled_swiglu",
    "qwen3_5_moe_combine_experts", "Qwen3_5MoEBlock", "device_status",
]


class SparseExpertError(ValueError):
    """SparseExpertError::InvalidAssignmentGeometry (sparse_experts/error.rs)."""


class ExpertAssignmentOrder(enum.Enum):
    """gathered_projection.rs:24-38: a promise about work the caller already did."""
    ORIGINAL = 0
    SORTED_BY_EXPERT = 1

    def uses_sorted_indices(self) -> bool:
        return self is ExpertAssignmentOrder.SORTED_BY_EXPERT


@dataclass
class AffineProjection:
    """StackedExpertProjection::Affine: MLX layout, borrowed (never copied)."""
    packed_weights: torch.Tensor  # int32/uint32 [E, out, in*bits/32]
    scales: torch.Tensor          # bf16 [E, out, in/group]
    biases: torch.Tensor          # bf16 [E, out, in/group]
    group_size: int = 64
    bits: int = 4

    @property
    def experts(self) -> int:
        return self.packed_weights.shape[0] if self.packed_weights.dim() == 3 else 1

    @property
    def out_features(self) -> int:
        return self.packed_weights.shape[-2]

    @property
    def in_features(self) -> int:
        return self.packed_weights.shape[-1] * 32 // self.bits


@dataclass
class SortedExpertAssignments:
    sorted_states: torch.Tensor
    sorted_indices: torch.Tensor
    inverse_order: torch.Tensor
    sorted_order: torch.Tensor
    expert_offsets: torch.Tensor


_DT = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16,
       torch.float32: _lib.DTYPE_F32}


def _stream(t: Optional[torch.Tensor] = None) -> int:
    dev = t.device if t is not None else torch.device("cuda")
    return torch.cuda.current_stream(dev).cuda_stream


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _dtype(t: torch.Tensor) -> int:
    if t.dtype not in _DT:
        raise AstroMoeError(_lib.ERR_INVALID_ARGUMENT, f"unsupported dtype {t.dtype}")
    return _DT[t.dtype]


def _u32(t: torch.Tensor) -> torch.Tensor:
    """uint32 payloads travel in int32/uint32 tensors (same bits)."""
    if t.dtype not in (torch.int32, torch.uint32):
        raise AstroMoeError(_lib.ERR_INVALID_ARGUMENT, f"index arrays must be 32-bit, got {t.dtype}")
    return t.contiguous()


def device_status(device: int = 0, reset: bool = True) -> int:
    st = ctypes.c_uint32(0)
    check(_lib.lib().astro_moe_device_status(device, ctypes.byref(st), int(reset)))
    return st.value


def qwen3_5_moe_route_experts(router_logits: torch.Tensor, expert_count_per_token: int,
                              should_normalize_scores: bool = True):
    """softmax -> top-K (value desc, id asc) -> optional renormalisation."""
    shape = list(router_logits.shape)
    if len(shape) < 2:
        raise AstroMoeError(_lib.ERR_INVALID_ARGUMENT,
                            "router logits must include token and expert dimensions")
    E = shape[-1]
    T = int(np.prod(shape[:-1]))
    logits = router_logits.contiguous()
    ids = torch.empty(shape[:-1] + [expert_count_per_token], dtype=torch.int32,
                      device=logits.device)
    scores = torch.empty(shape[:-1] + [expert_count_per_token], dtype=logits.dtype,
                         device=logits.device)
    check(_lib.lib().astro_moe_route_experts(_ptr(logits), _dtype(logits), T, E,
                                             expert_count_per_token, int(should_normalize_scores),
                                             _ptr(ids), _ptr(scores), _stream(logits)))
    return ids, scores


def route_laguna_experts(router_logits: torch.Tensor, experts_per_token: int,
                         correction_bias: Optional[torch.Tensor] = None,
                         router_logit_softcap: float = 0.0, normalize: bool = True):
    """Laguna routing (laguna/moe/router.rs:11-60): sigmoid scores (optionally
    softcapped), correction bias for the ranking only, original fp32 scores of
    the K winners (optionally renormalised)."""
    shape = list(router_logits.shape)
    if len(shape) < 2:
        raise AstroMoeError(_lib.ERR_INVALID_ARGUMENT,
                            "router logits must include token and expert dimensions")
    E = shape[-1]
    T = int(np.prod(shape[:-1]))
    logits = router_logits.contiguous()
    bias = None if correction_bias is None else correction_bias.to(torch.float32).contiguous()
    if bias is not None and bias.numel() != E:
        raise AstroMoeError(_lib.ERR_INVALID_ARGUMENT,
                            "Laguna correction bias must have one value per expert")
    ids = torch.empty(shape[:-1] + [experts_per_token], dtype=torch.int32, device=logits.device)
    scores = torch.empty(shape[:-1] + [experts_per_token], dtype=torch.float32,
                         device=logits.device)
    check(_lib.lib().astro_moe_route_laguna_experts(
        _ptr(logits), _dtype(logits), T, E, experts_per_token,
        _ptr(bias) if bias is not None else None, float(router_logit_softcap), int(normalize),
        _ptr(ids), _ptr(scores), _stream(logits)))
    return ids, scores


def sort_expert_assignments(expanded_states: torch.Tensor, selected_indices: torch.Tensor,
                            experts: Optional[int] = None) -> SortedExpertAssignments:
    """Stable sort by expert id; gathers the token rows (take) like the reference."""
    K = selected_indices.shape[-1] if selected_indices.dim() else 0
    n = selected_indices.numel()
    H = expanded_states.shape[-1]
    T = expanded_states.numel() // H if H else 0
    dev = expanded_states.device
    if K <= 0 and n == 0:
        empty = torch.empty(0, dtype=torch.int32, device=dev)
        return SortedExpertAssignments(expanded_states.new_zeros((0, 1, H)), empty, empty, empty,
                                       torch.zeros(1 if experts is None else experts + 1,
                                                   dtype=torch.int32, device=dev))
    if n % K != 0 or n // K != T:
        raise SparseExpertError("expert assignments do not match expanded hidden-state tokens")
    ids = _u32(selected_indices).reshape(-1)
    if experts is None:
        experts = int(ids.max().item()) + 1 if n else 1
    order = torch.empty(n, dtype=torch.int32, device=dev)
    inverse = torch.empty(n, dtype=torch.int32, device=dev)
    sorted_ids = torch.empty(n, dtype=torch.int32, device=dev)
    sorted_tokens = torch.empty(n, dtype=torch.int32, device=dev)
    offsets = torch.empty(experts + 1, dtype=torch.int32, device=dev)
    st = _stream(expanded_states)
    check(_lib.lib().astro_moe_sort_expert_assignments(_ptr(ids), n // K, K, experts, _ptr(order),
                                                       _ptr(inverse), _ptr(sorted_ids),
                                                       _ptr(sorted_tokens), _ptr(offsets), st))
    states = expanded_states.reshape(T, H).contiguous()
    if states.dtype == torch.bfloat16 and H % 8 == 0:
        sorted_states = torch.empty((n, H), dtype=states.dtype, device=dev)
        check(_lib.lib().astro_moe_take_rows(_ptr(states), T, H, _ptr(sorted_tokens), n,
                                             _ptr(sorted_states), st))
    else:
        sorted_states = states.index_select(0, sorted_tokens.long())
    return SortedExpertAssignments(sorted_states.reshape(n, 1, H), sorted_ids, inverse, order,
                                   offsets)


def restore_expert_assignment_order(sorted_outputs: torch.Tensor, inverse_order: torch.Tensor,
                                    selected_index_shape: Sequence[int]) -> torch.Tensor:
    n = int(np.prod(selected_index_shape)) if len(selected_index_shape) else 0
    D = sorted_outputs.shape[-1]
    if n == 0:
        return sorted_outputs.new_zeros(list(selected_index_shape) + [D])
    if sorted_outputs.shape[0] != n or inverse_order.numel() != n:
        raise SparseExpertError("sorted expert outputs and inverse order have incompatible shapes")
    return sorted_outputs.reshape(n, D).index_select(0, inverse_order.long()).reshape(
        list(selected_index_shape) + [D])


def invert_assignment_order(sorted_order: Sequence[int]) -> list:
    arr = np.ascontiguousarray(np.asarray(sorted_order, dtype=np.uint32))
    inv = np.empty_like(arr)
    st = _lib.lib().astro_moe_invert_assignment_order(arr.ctypes.data, arr.size, inv.ctypes.data)
    if st != _lib.OK:
        raise SparseExpertError(_lib.lib().astro_moe_last_error().decode())
    return inv.tolist()


def gather_expert_projection(activations: torch.Tensor, projection: AffineProjection,
                             selected_expert_indices: Optional[torch.Tensor],
                             assignment_order: ExpertAssignmentOrder,
                             lhs_indices: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[n] = activations[lhs[n]] . dequant(W[rhs[n]])^T (bf16 activations)."""
    if activations.dtype != torch.bfloat16:
        raise AstroMoeError(_lib.ERR_UNSUPPORTED, "activations must be bfloat16")
    in_f = projection.in_features
    x = activations.reshape(-1, in_f).contiguous()
    rhs = None if selected_expert_indices is None else _u32(selected_expert_indices).reshape(-1)
    lhs = None if lhs_indices is None else _u32(lhs_indices).reshape(-1)
    n = rhs.numel() if rhs is not None else (lhs.numel() if lhs is not None else x.shape[0])
    out = torch.empty((n, projection.out_features), dtype=torch.bfloat16, device=x.device)
    if n == 0:
        return out
    check(_lib.lib().astro_moe_gather_qmm(
        _ptr(x), x.shape[0], in_f, _ptr(lhs), _ptr(rhs), n, _ptr(projection.packed_weights),
        _ptr(projection.scales), _ptr(projection.biases), projection.experts,
        projection.out_features, projection.group_size, projection.bits,
        int(assignment_order.uses_sorted_indices()), _ptr(out), _stream(x)))
    return out


def apply_compiled_swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    g, u = gate.contiguous(), up.contiguous()
    out = torch.empty_like(g)
    check(_lib.lib().astro_moe_swiglu(_ptr(g), _ptr(u), g.numel(), _ptr(out), _stream(g)))
    return out


def sorted_expert_weighted_sum(sorted_expert_outputs: torch.Tensor, inverse_order: torch.Tensor,
                               selected_scores: torch.Tensor) -> torch.Tensor:
    so = sorted_expert_outputs.contiguous()
    sc = selected_scores.contiguous()
    K = sc.shape[-1]
    n = sc.numel()
    D = so.shape[-1]
    if K == 0 or n == 0:
        return so.new_zeros(list(sc.shape[:-1]) + [D])
    if so.numel() // D != n or inverse_order.numel() != n:
        raise SparseExpertError("sorted expert outputs and inverse order must match selected scores")
    out = torch.empty(list(sc.shape[:-1]) + [D], dtype=so.dtype, device=so.device)
    check(_lib.lib().astro_moe_sorted_expert_weighted_sum(
        _ptr(so), _dtype(so), _ptr(_u32(inverse_order)), _ptr(sc), _dtype(sc), n // K, K, D,
        _ptr(out), _stream(so)))
    return out


def unsorted_expert_weighted_sum(selected_expert_outputs: torch.Tensor,
                                 selected_scores: torch.Tensor) -> torch.Tensor:
    o = selected_expert_outputs.contiguous()
    sc = selected_scores.contiguous()
    K = sc.shape[-1]
    D = o.shape[-1]
    T = sc.numel() // K if K else int(np.prod(sc.shape[:-1]))
    out = torch.empty(list(sc.shape[:-1]) + [D], dtype=o.dtype, device=o.device)
    check(_lib.lib().astro_moe_unsorted_expert_weighted_sum(_ptr(o), _dtype(o), _ptr(sc),
                                                            _dtype(sc), T, K, D, _ptr(out),
                                                            _stream(o)))
    return out


def qwen3_5_moe_combine_experts(selected_expert_outputs, selected_scores, shared_expert_output,
                                shared_expert_gate_logits):
    sparse = unsorted_expert_weighted_sum(selected_expert_outputs, selected_scores)
    s, sh, g = (t.contiguous() for t in (sparse, shared_expert_output, shared_expert_gate_logits))
    D = s.shape[-1]
    out = torch.empty_like(s)
    check(_lib.lib().astro_moe_combine_sparse_and_shared(_ptr(s), _ptr(sh), _ptr(g), _dtype(s),
                                                         s.numel() // D, D, _ptr(out),
                                                         _stream(s)))
    return out


# weight-dict keys holding bf16 arrays (everything else is packed uint32 codes)
def _is_bf16_key(k: str) -> bool:
    return k.endswith("_s") or k.endswith("_b") or k in ("router_w", "shared_gate_w")


def device_weights(weights: dict, device, keys=None) -> dict:
    """The array entries of a weight dict (MLX layout) on `device`; integer
    entries (per-projection "<name>_bits" / "<name>_group") are kept as they are."""
    out = {}
    for k, v in weights.items():
        if k == "config" or v is None or (keys is not None and k not in keys):
            continue
        out[k] = int(v) if isinstance(v, (int, np.integer)) else _to_dev(v, device, _is_bf16_key(k))
    return out


def layer_weights_struct(t: dict, cfg: dict, experts: int, fuse_gate_up: bool = False,
                         routed: bool = True) -> "_lib.LayerWeights":
    """astro_moe_layer_weights over device tensors `t` (keys of
    synthetic.make_block_weights): projections gate/up/down/sgate/sup/sdown with
    optional "<name>_bits" / "<name>_group", a bf16 router ("router_w") or an
    affine one ("router_q/_s/_b" + "router_bits/_group"), a bf16 shared-expert
    gate ("shared_gate_w") or an affine one ("shared_gate_q/_s/_b" + bits/group).
    routed=False leaves the routed stacks empty (a paged layer)."""
    def aff(prefix):
        if prefix + "_q" not in t:
            return _lib.Affine()
        return _lib.Affine(t[prefix + "_q"].data_ptr(), t[prefix + "_s"].data_ptr(),
                           t[prefix + "_b"].data_ptr(), int(t.get(prefix + "_bits", 0)),
                           int(t.get(prefix + "_group", 0)))

    lw = _lib.LayerWeights()
    lw.hidden, lw.experts, lw.top_k = cfg["hidden"], experts, cfg["top_k"]
    lw.intermediate = cfg["intermediate"]
    lw.shared_intermediate = cfg.get("shared_intermediate", 0)
    lw.group_size, lw.bits = cfg["group"], cfg["bits"]
    lw.normalize_top_k = int(cfg.get("normalize", True))
    lw.gate_up_fused = int(fuse_gate_up and routed)
    lw.router_weight = t["router_w"].data_ptr() if "router_w" in t else None
    lw.router_affine = aff("router")
    if routed:
        lw.gate = aff("gate")
        lw.up = aff("up") if not fuse_gate_up else _lib.Affine()
        lw.down = aff("down")
    lw.shared_gate, lw.shared_up, lw.shared_down = aff("sgate"), aff("sup"), aff("sdown")
    lw.shared_expert_gate = t["shared_gate_w"].data_ptr() if "shared_gate_w" in t else None
    lw.shared_expert_gate_affine = aff("shared_gate")
    # Laguna router family (laguna/moe/router.rs): sigmoid scores, selection-only
    # correction bias, optional logit softcap, routed scaling, ungated shared expert
    if cfg.get("router") == "laguna":
        lw.router_kind = _lib.ROUTER_SIGMOID
        lw.router_logit_softcap = float(cfg.get("router_logit_softcap", 0.0))
        lw.routed_scaling_factor = float(cfg.get("routed_scaling_factor", 1.0))
        lw.router_correction_bias = (t["router_correction_bias"].data_ptr()
                                     if "router_correction_bias" in t else None)
    return lw


def _to_dev(a, device, bf16=False):
    if isinstance(a, torch.Tensor):
        t = a.to(device)
    else:
        arr = np.ascontiguousarray(a)
        if not arr.flags.writeable:  # a read-only checkpoint memmap: torch wants its own copy
            arr = np.array(arr)
        if arr.dtype == np.uint32:
            arr = arr.view(np.int32)
        t = torch.from_numpy(arr).to(device)
    if bf16 and t.dtype in (torch.uint16, torch.int16):
        t = t.view(torch.bfloat16)
    if t.dtype == torch.uint32:
        t = t.view(torch.int32)
    return t.contiguous()


class Qwen3_5MoEBlock:
    """One resident MoE block on one GPU: forward_qwen3_5_moe over libastro_moe.

    ``weights``: dict in MLX layout (numpy or torch), keys as produced by
    astronomical_b200.synthetic.make_block_weights.  Tensors are kept on the
    device for the block's lifetime (the library only borrows them).
    """

    def __init__(self, weights: dict, device: int = 0, max_tokens: int = 4096,
                 use_tensor_cores: int = 0, fuse_gate_up: bool = False, layer: int = 0,
                 decode_max_tokens: int = 0, decode_fused: int = 0):
        cfg = weights["config"]
        self.cfg = dict(cfg)
        self.device = torch.device("cuda", device)
        self.layer = layer
        dev = self.device
        t = device_weights(weights, dev)
        if fuse_gate_up:
            # resident_gate_up_fusion.rs:221-260: concatenate along the output axis
            t["gate_q"] = torch.cat([t["gate_q"], t.pop("up_q")], 1).contiguous()
            t["gate_s"] = torch.cat([t["gate_s"], t.pop("up_s")], 1).contiguous()
            t["gate_b"] = torch.cat([t["gate_b"], t.pop("up_b")], 1).contiguous()
        self.tensors = t
        self.fused = fuse_gate_up
        opts = _lib.Options()
        opts.max_tokens = max_tokens
        opts.sorted_threshold = 0
        opts.use_tensor_cores = use_tensor_cores
        opts.decode_max_tokens = decode_max_tokens
        opts.decode_fused = decode_fused
        ctx = ctypes.c_void_p()
        with torch.cuda.device(dev):
            check(_lib.lib().astro_moe_ctx_create(device, ctypes.c_void_p(
                torch.cuda.current_stream(dev).cuda_stream), ctypes.byref(opts), ctypes.byref(ctx)))
        self.ctx = ctx

        lw = layer_weights_struct(t, cfg, cfg["experts"], fuse_gate_up=fuse_gate_up)
        self._lw = lw
        check(_lib.lib().astro_moe_register_layer(self.ctx, layer, ctypes.byref(lw)))

    def close(self):
        if getattr(self, "ctx", None):
            _lib.lib().astro_moe_ctx_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _bind_stream(self):
        check(_lib.lib().astro_moe_ctx_set_stream(
            self.ctx, ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)))

    def forward(self, hidden_states: torch.Tensor, taps: bool = False):
        """hidden_states bf16 [..., T, H] -> bf16 [..., T, H] (stream-ordered)."""
        H = self.cfg["hidden"]
        x = hidden_states.reshape(-1, H).contiguous()
        T = x.shape[0]
        out = torch.empty_like(x)
        self._bind_stream()
        if not taps:
            check(_lib.lib().astro_moe_block_forward(self.ctx, self.layer, _ptr(x), T, _ptr(out)))
            return out.reshape(hidden_states.shape)
        E, K = self.cfg["experts"], self.cfg["top_k"]
        tp = {
            "router_logits": torch.empty((T, E), dtype=torch.bfloat16, device=x.device),
            "selected_indices": torch.empty((T, K), dtype=torch.int32, device=x.device),
            "selected_scores": torch.empty((T, K), dtype=torch.float32 if self.cfg.get("router") ==
                                           "laguna" else torch.bfloat16, device=x.device),
            "expert_offsets": torch.empty(E + 2, dtype=torch.int32, device=x.device),
        }
        ct = _lib.BlockTaps(*(tp[k].data_ptr() for k in ("router_logits", "selected_indices",
                                                          "selected_scores", "expert_offsets")))
        check(_lib.lib().astro_moe_block_forward_taps(self.ctx, self.layer, _ptr(x), T, _ptr(out),
                                                      ctypes.byref(ct)))
        return out.reshape(hidden_states.shape), tp

    __call__ = forward

    def forward_host(self, host_hidden: torch.Tensor, host_out: torch.Tensor) -> None:
        """Host buffers in and out (copies inside the call), synchronising."""
        T = host_hidden.numel() // self.cfg["hidden"]
        self._bind_stream()
        check(_lib.lib().astro_moe_block_forward_host(self.ctx, self.layer, _ptr(host_hidden), T,
                                                      _ptr(host_out)))

    def forward_host_async(self, host_hidden: torch.Tensor, host_out: torch.Tensor) -> None:
        """Host buffers in and out without synchronising (call synchronize_host);
        consecutive calls overlap their copies with each other's compute."""
        T = host_hidden.numel() // self.cfg["hidden"]
        self._bind_stream()
        check(_lib.lib().astro_moe_block_forward_host_async(self.ctx, self.layer,
                                                            _ptr(host_hidden), T, _ptr(host_out)))

    def synchronize_host(self) -> None:
        check(_lib.lib().astro_moe_host_synchronize(self.ctx))

    def last_path(self) -> dict:
        """Kernels the last block call ran, per stage (router, gate_logit, experts,
        shared_expert), by name."""
        p = _lib.BlockPath()
        check(_lib.lib().astro_moe_ctx_last_block_path(self.ctx, ctypes.byref(p)))
        return p.as_dict()

    def set_attribution(self, enabled: bool) -> None:
        check(_lib.lib().astro_moe_ctx_set_attribution(self.ctx, int(enabled)))

    def read_attribution(self, reset: bool = True) -> dict:
        a = _lib.Attribution()
        check(_lib.lib().astro_moe_ctx_read_attribution(self.ctx, ctypes.byref(a), int(reset)))
        return a.as_dict()

    def synchronize(self) -> None:
        check(_lib.lib().astro_moe_ctx_synchronize(self.ctx))
