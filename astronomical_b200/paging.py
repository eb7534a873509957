"""Expert paging (config 4): routed experts in pinned host memory, an LRU page
cache in HBM under a byte ceiling.

Mirrors the reference's ``Qwen3_5ExpertPager`` and the paged branch of
``forward_qwen3_5_moe`` (qwen3_5_moe/expert_paging/expert_pager/mod.rs:55-224,
model/forward.rs:229-312): route, find the routed experts, admit the pages that
are not resident, run the experts.  The reference reads missing pages from SSD
with ``pread``; here the whole expert store is pinned host memory and missing
pages are copied with ``cudaMemcpyAsync`` on the pager's own stream.  A page is
one (layer, expert): its gate, up and down codes, scales and biases, contiguous
(``astro_moe_page_bytes`` bytes; 1,769,472 for the Qwen3.6-35B-A3B block).
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import numpy as np
import torch

from . import _lib, moe
from .moe import _ptr, _to_dev, check

__all__ = ["page_bytes", "pack_layer", "pack_expert_pages", "PagedMoEStack"]

# tensor order inside a page (matches astro_moe_pager_create)
_PAGE_ORDER = ("gate_q", "up_q", "down_q", "gate_s", "gate_b", "up_s", "up_b", "down_s", "down_b")


def page_bytes(cfg: dict) -> int:
    return int(_lib.lib().astro_moe_page_bytes(cfg["hidden"], cfg["intermediate"], cfg["group"],
                                               cfg["bits"]))


def _bytes_per_expert(a) -> torch.Tensor:
    if not isinstance(a, torch.Tensor):
        a = np.asarray(a)
        if not a.flags.writeable:  # memory-mapped checkpoint tensors: torch wants writable
            a = a.copy()
    t = torch.as_tensor(a) if not isinstance(a, torch.Tensor) else a
    t = t.detach().contiguous()
    return t.view(torch.uint8).reshape(t.shape[0], -1)


def pack_layer(pages: torch.Tensor, w: dict) -> None:
    """Writes one layer's expert pages into ``pages`` [experts, page_bytes]."""
    off = 0
    for name in _PAGE_ORDER:
        b = _bytes_per_expert(w[name])
        pages[:, off:off + b.shape[1]].copy_(b)
        off += b.shape[1]
    assert off == pages.shape[1], (off, pages.shape[1])


def pack_expert_pages(layers: Sequence[dict], pin: bool = True) -> torch.Tensor:
    """Host store [layers, experts, page_bytes] (uint8, pinned unless pin=False)
    from MLX-layout stacks (numpy or torch, host or device)."""
    cfg = layers[0]["config"]
    E, P = cfg["experts"], page_bytes(cfg)
    store = torch.empty((len(layers), E, P), dtype=torch.uint8, pin_memory=pin)
    for li, w in enumerate(layers):
        pack_layer(store[li], w)
    return store


class PagedMoEStack:
    """Paged MoE layers on one GPU: routers, shared experts and their gates are
    resident; routed experts come from ``store`` through an HBM page cache of at
    most ``cache_bytes``.  Calls of up to 64 tokens (decode) compute the resident
    experts while the missing pages copy; longer calls (prefill) bring in every
    page they route to and run the tensor-core grouped GEMMs over the cache, so a
    call's pages must fit in it."""

    def __init__(self, layers: Sequence[dict], store: torch.Tensor, cache_bytes: int,
                 device: int = 0, policy: str = "lru", max_tokens: int = 64):
        cfg = layers[0]["config"]
        self.cfg = dict(cfg)
        self.device = torch.device("cuda", device)
        self.store = store  # must stay alive: the pager reads it
        opts = _lib.Options()
        opts.max_tokens = int(max_tokens)
        ctx = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(_lib.lib().astro_moe_ctx_create(device, ctypes.c_void_p(
                torch.cuda.current_stream(self.device).cuda_stream), ctypes.byref(opts),
                ctypes.byref(ctx)))
        self.ctx = ctx
        pg = ctypes.c_void_p()
        check(_lib.lib().astro_moe_pager_create(
            self.ctx, len(layers), cfg["experts"], cfg["hidden"], cfg["intermediate"], cfg["group"],
            cfg["bits"], ctypes.c_void_p(store.data_ptr()), int(cache_bytes), ctypes.byref(pg)))
        self.pager = pg
        self.set_policy(policy)
        self._keep = []
        for li, w in enumerate(layers):
            t = moe.device_weights(w, self.device, keys=[k for k in w if not k.startswith(
                ("gate_", "up_", "down_"))])
            self._keep.append(t)
            lw = moe.layer_weights_struct(t, cfg, cfg["experts"], routed=False)
            check(_lib.lib().astro_moe_register_paged_layer(self.ctx, li, ctypes.byref(lw),
                                                            self.pager))

    def set_policy(self, policy: str) -> None:
        """Page retention: "lru" or "demand" (least-routed page evicted first)."""
        codes = {"lru": _lib.PAGER_LRU, "demand": _lib.PAGER_DEMAND}
        if policy not in codes:
            raise ValueError(f"unknown pager policy {policy!r}")
        check(_lib.lib().astro_moe_pager_set_policy(self.pager, codes[policy]))
        self.policy = policy

    def inject_copy_failures(self, count: int) -> None:
        """Failure testing: the next `count` page copies fail on the host."""
        check(_lib.lib().astro_moe_pager_inject_copy_failures(self.pager, int(count)))

    def forward(self, layer: int, x: torch.Tensor) -> torch.Tensor:
        out = torch.empty_like(x)
        check(_lib.lib().astro_moe_ctx_set_stream(
            self.ctx, ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)))
        check(_lib.lib().astro_moe_paged_block_forward(self.ctx, layer, _ptr(x), x.shape[0],
                                                       _ptr(out)))
        return out

    def last_path(self) -> dict:
        """Kernels the last paged call ran, per stage, by name."""
        p = _lib.BlockPath()
        check(_lib.lib().astro_moe_ctx_last_block_path(self.ctx, ctypes.byref(p)))
        return p.as_dict()

    def stats(self, reset: bool = False) -> dict:
        s = _lib.PagerStats()
        check(_lib.lib().astro_moe_pager_read_stats(self.pager, ctypes.byref(s), int(reset)))
        return s.as_dict()

    def close(self):
        if getattr(self, "ctx", None):
            _lib.lib().astro_moe_ctx_destroy(self.ctx)
            self.ctx = None
        if getattr(self, "pager", None):
            _lib.lib().astro_moe_pager_destroy(self.pager)
            self.pager = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
