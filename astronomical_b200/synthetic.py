"""Seeded synthetic inputs and weights with the shapes and value distributions of
the benchmark configurations (no checkpoints or datasets are available offline).

Weights use MLX's affine layout, the layout the reference loads from its
checkpoints (qwen3_5_moe/expert_residency/resident_gate_up_fusion.rs:221-260):
packed uint32 ``[E, out, in*bits/32]`` with element j of a row at bit j*bits of
the row's little-endian bit stream, scales and biases bf16 ``[E, out, in/group]``,
and ``w = scale * q + bias``.

Distributions (all configs): activations ~ N(0, 1); router weight ~ N(0, 0.02);
q uniform on 0..15; scales = |N(0, 0.01)|; biases = -8 * scale.  The decode
sweep's Zipf(1.1) expert skew is realised inside the router projection: hidden
feature 0 of every token is set to 1.0 and router column 0 holds the per-expert
bias b_e = ln p(pi(e)), p(r) ~ r^-1.1, pi a seeded permutation.  The block's
arithmetic is therefore unchanged (no extra bias op) while expert load is skewed.

bf16 values are carried as uint16 bit patterns in numpy arrays.
"""
from __future__ import annotations

import numpy as np

CONFIGS = {
    # config 0: CPU plumbing check
    0: dict(tokens=32, hidden=2048, experts=128, top_k=8, intermediate=768,
            shared_intermediate=0, group=64, bits=4, normalize=True, zipf=None),
    # config 1: Qwen3.6-35B-A3B-shaped prefill block (the headline)
    1: dict(tokens=4096, hidden=2048, experts=256, top_k=8, intermediate=512,
            shared_intermediate=512, group=64, bits=4, normalize=True, zipf=None),
    # config 2: decode sweep of the config-1 block with Zipf(1.1) routing skew
    2: dict(tokens=(1, 4, 16, 64), hidden=2048, experts=256, top_k=8, intermediate=512,
            shared_intermediate=512, group=64, bits=4, normalize=True, zipf=1.1),
}


# Laguna-shaped variant of config 1 (laguna/moe: 256 experts, sigmoid router with
# a selection-only correction bias, routed_scaling_factor 2.5, an ungated shared
# expert of the routed width); the same block kernels, another router family
LAGUNA = dict(tokens=512, hidden=2048, experts=256, top_k=8, intermediate=512,
              shared_intermediate=512, group=64, bits=4, normalize=True, zipf=None,
              router="laguna", router_logit_softcap=0.0, routed_scaling_factor=2.5)


def f32_to_bf16(a) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(h) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def pack_affine(q: np.ndarray, bits: int = 4) -> np.ndarray:
    """Pack integer codes [..., in] into MLX's uint32 rows (little-endian bit stream)."""
    q = np.asarray(q, dtype=np.uint64)
    in_f = q.shape[-1]
    assert (in_f * bits) % 32 == 0
    flat = q.reshape(-1, in_f)
    words = in_f * bits // 32
    out = np.zeros((flat.shape[0], words), np.uint64)
    for j in range(in_f):
        bit = j * bits
        w, b = divmod(bit, 32)
        out[:, w] |= (flat[:, j] << np.uint64(b)) & np.uint64(0xFFFFFFFF)
        if b + bits > 32:
            out[:, w + 1] |= flat[:, j] >> np.uint64(32 - b)
    return out.astype(np.uint32).reshape(q.shape[:-1] + (words,))


def unpack_affine(packed: np.ndarray, bits: int = 4) -> np.ndarray:
    packed = np.asarray(packed, dtype=np.uint32)
    words = packed.shape[-1]
    in_f = words * 32 // bits
    flat = packed.reshape(-1, words).astype(np.uint64)
    out = np.zeros((flat.shape[0], in_f), np.uint8)
    for j in range(in_f):
        bit = j * bits
        w, b = divmod(bit, 32)
        v = flat[:, w] >> np.uint64(b)
        if b + bits > 32:
            v |= flat[:, w + 1] << np.uint64(32 - b)
        out[:, j] = (v & np.uint64((1 << bits) - 1)).astype(np.uint8)
    return out.reshape(packed.shape[:-1] + (in_f,))


def _affine(rng, shape_rows, in_f, group, bits):
    """Random q (uniform 0..2^bits-1), |N(0,0.01 * 16/2^bits)| scales and
    -2^(bits-1)*scale biases (for 4 bits: |N(0,0.01)| and -8*scale), so every bit
    width spans about the same weight range."""
    words = in_f * bits // 32
    if bits in (2, 4, 8):
        # uniformly random words have independent uniform fields
        q = rng.integers(0, 2**32, size=shape_rows + (words,), dtype=np.uint64).astype(np.uint32)
    else:
        q = pack_affine(rng.integers(0, 2**bits, size=shape_rows + (in_f,)), bits)
    s = f32_to_bf16(np.abs(rng.normal(0.0, 0.01 * 16.0 / 2**bits,
                                      size=shape_rows + (in_f // group,))))
    b = f32_to_bf16(-float(2 ** (bits - 1)) * bf16_to_f32(s))
    return q, s, b


def quantize_affine(w, bits: int, group: int):
    """MLX-style affine quantisation of float rows [..., in]: per group of
    `group` elements scale = (max - min) / (2^bits - 1), bias = min (both bf16),
    q = round((w - bias) / scale) clipped to the code range.  Returns (packed
    uint32, scales bf16 bits, biases bf16 bits)."""
    w = np.asarray(w, np.float32)
    rows = w.shape[:-1]
    in_f = w.shape[-1]
    g = w.reshape(rows + (in_f // group, group))
    lo, hi = g.min(-1), g.max(-1)
    scale = f32_to_bf16(np.maximum(hi - lo, 1e-8) / (2 ** bits - 1))
    bias = f32_to_bf16(lo)
    sf, bf = bf16_to_f32(scale)[..., None], bf16_to_f32(bias)[..., None]
    q = np.clip(np.rint((g - bf) / sf), 0, 2 ** bits - 1).astype(np.uint32)
    return pack_affine(q.reshape(rows + (in_f,)), bits), scale, bias


# projections whose quantisation make_block_weights can override
QUANT_NAMES = ("gate", "up", "down", "sgate", "sup", "sdown", "router", "shared_gate")


def zipf_router_bias(experts: int, s: float, rng) -> np.ndarray:
    ranks = np.arange(1, experts + 1, dtype=np.float64)
    p = ranks ** (-s)
    p /= p.sum()
    perm = rng.permutation(experts)
    return np.log(p[perm])  # b_e = ln p(pi(e))


def make_block_weights(cfg: dict, seed: int = 0, quant: dict | None = None) -> dict:
    """Router, routed experts (separate gate/up, MLX layout) and optional shared expert.

    quant maps a projection (QUANT_NAMES) to its own (bits, group): the routed and
    shared projections are then drawn with that profile and carry "<name>_bits" /
    "<name>_group" keys, and "router" / "shared_gate" replace the bf16 router or
    shared-expert gate by an MLX-style affine quantisation of the same values
    ("<name>_q/_s/_b", as the reference's Qwen3_5MoERouterGateWeights::Affine)."""
    rng = np.random.default_rng(seed)
    H, E, I = cfg["hidden"], cfg["experts"], cfg["intermediate"]
    Is, G, B = cfg.get("shared_intermediate", 0), cfg["group"], cfg["bits"]
    w = {"config": dict(cfg)}
    router = rng.normal(0.0, 0.02, size=(E, H))
    if cfg.get("zipf"):
        router[:, 0] = zipf_router_bias(E, cfg["zipf"], rng)
    w["router_w"] = f32_to_bf16(router)
    w["gate_q"], w["gate_s"], w["gate_b"] = _affine(rng, (E, I), H, G, B)
    w["up_q"], w["up_s"], w["up_b"] = _affine(rng, (E, I), H, G, B)
    w["down_q"], w["down_s"], w["down_b"] = _affine(rng, (E, H), I, G, B)
    if Is:
        w["sgate_q"], w["sgate_s"], w["sgate_b"] = _affine(rng, (Is,), H, G, B)
        w["sup_q"], w["sup_s"], w["sup_b"] = _affine(rng, (Is,), H, G, B)
        w["sdown_q"], w["sdown_s"], w["sdown_b"] = _affine(rng, (H,), Is, G, B)
        w["shared_gate_w"] = f32_to_bf16(rng.normal(0.0, 0.02, size=(1, H)))
    if cfg.get("router") == "laguna":
        # a per-expert correction bias of the size sigmoid scores move by
        brng = np.random.default_rng([seed, 99])
        w["router_correction_bias"] = brng.normal(0.0, 0.05, size=E).astype(np.float32)
        w.pop("shared_gate_w", None)  # the Laguna shared expert is ungated
    for name, (bits, group) in (quant or {}).items():
        if name not in QUANT_NAMES:
            raise ValueError(f"unknown projection {name}")
        if name == "shared_gate" and not Is:
            continue
        if name in ("router", "shared_gate"):
            dense = w.pop("router_w" if name == "router" else "shared_gate_w")
            w[name + "_q"], w[name + "_s"], w[name + "_b"] = quantize_affine(
                bf16_to_f32(dense), bits, group)
        else:
            if name in ("sgate", "sup", "sdown") and not Is:
                continue
            qrng = np.random.default_rng([seed, QUANT_NAMES.index(name), bits, group])
            rows, in_f = {"gate": ((E, I), H), "up": ((E, I), H), "down": ((E, H), I),
                          "sgate": ((Is,), H), "sup": ((Is,), H), "sdown": ((H,), Is)}[name]
            w[name + "_q"], w[name + "_s"], w[name + "_b"] = _affine(qrng, rows, in_f, group, bits)
        w[name + "_bits"], w[name + "_group"] = int(bits), int(group)
    return w


def make_hidden_states(tokens: int, hidden: int, seed: int = 1, zipf: bool = False) -> np.ndarray:
    rng = np.random.default_rng(seed)
    x = rng.normal(0.0, 1.0, size=(tokens, hidden)).astype(np.float32)
    if zipf:
        x[:, 0] = 1.0
    return f32_to_bf16(x)


def make_block_weights_torch(cfg: dict, seed: int, device):
    """Same distributions, generated on the device with torch (for full-size runs)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    H, E, I = cfg["hidden"], cfg["experts"], cfg["intermediate"]
    Is, G, B = cfg.get("shared_intermediate", 0), cfg["group"], cfg["bits"]
    assert B in (2, 4, 8)

    def affine(rows, in_f):
        words = in_f * B // 32
        q = torch.randint(-2**31, 2**31 - 1, rows + (words,), generator=g, device=device,
                          dtype=torch.int64).to(torch.int32)
        s = torch.randn(rows + (in_f // G,), generator=g, device=device).mul_(0.01).abs_()
        s = s.to(torch.bfloat16)
        b = (s.float() * -8.0).to(torch.bfloat16)
        return q, s, b

    w = {"config": dict(cfg)}
    router = torch.randn((E, H), generator=g, device=device) * 0.02
    if cfg.get("zipf"):
        rng = np.random.default_rng(seed)
        router[:, 0] = torch.tensor(zipf_router_bias(E, cfg["zipf"], rng), device=device,
                                    dtype=torch.float32)
    w["router_w"] = router.to(torch.bfloat16)
    w["gate_q"], w["gate_s"], w["gate_b"] = affine((E, I), H)
    w["up_q"], w["up_s"], w["up_b"] = affine((E, I), H)
    w["down_q"], w["down_s"], w["down_b"] = affine((E, H), I)
    if Is:
        w["sgate_q"], w["sgate_s"], w["sgate_b"] = affine((Is,), H)
        w["sup_q"], w["sup_s"], w["sup_b"] = affine((Is,), H)
        w["sdown_q"], w["sdown_s"], w["sdown_b"] = affine((H,), Is)
        w["shared_gate_w"] = (torch.randn((1, H), generator=g, device=device) * 0.02).to(
            torch.bfloat16)
    return w
