"""Expert-parallel MoE block over the GPUs of one node (config 3).

The reference runs the sorted MoE block on one device (MLX); this module splits
the same block, ``Qwen3_5Model::forward_qwen3_5_moe`` (qwen3_5_moe/model/
forward.rs:19-127), across ``world`` ranks with one process per GPU:

* experts are block-partitioned: rank r owns experts [r*E/world, (r+1)*E/world);
  the router and the shared expert are replicated, tokens stay data-parallel;
* each rank routes and stably sorts its own tokens over all experts; since the
  sort groups rows by expert, the rows bound for each rank are contiguous;
* per-expert counts go out with one all-to-all, then the token rows with an
  all-to-all-v (NCCL over NVLink/NVSwitch through torch.distributed);
* the receiving rank permutes the rows into expert-major order, appends its own
  tokens as the shared expert's segment and runs the grouped GEMMs;
* the outputs travel back with the reverse all-to-all-v, and the source rank
  forms the router-weighted sum plus the gated shared expert.

Every token's output is computed with the single-GPU block's arithmetic, so an
expert-parallel run reproduces ``Qwen3_5MoEBlock`` on the same tokens.

The exchange logic (``ExpertParallelBlock``) is independent of where the expert
arithmetic runs: it drives any object with ``dispatch`` / ``experts`` /
``combine`` (``CudaExpertShard`` here, an oracle-backed stand-in in the CPU
tests, which run it over gloo ranks).
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import _lib, moe
from .moe import _ptr, check

__all__ = ["expert_range", "local_expert_weights", "CudaExpertShard", "ExpertParallelBlock",
           "ExpertParallelStack", "PeerFailure", "PeerWatchdog"]


class PeerFailure(RuntimeError):
    """A peer rank stopped heart-beating or left; ``ranks`` lists them."""

    def __init__(self, ranks, reason):
        super().__init__(f"expert-parallel peer rank(s) {sorted(ranks)} {reason}")
        self.ranks = sorted(ranks)
        self.reason = reason


class PeerWatchdog:
    """Host-side liveness of the expert-parallel ranks, so a rank learns that a
    peer died or left before it launches the next layer's collectives (which
    would otherwise wait until the process group's timeout).

    A background thread bumps this rank's heartbeat counter in the process
    group's store every ``interval`` seconds and reads the peers' counters and
    departure notices; ``check()`` (called by ExpertParallelBlock before each
    layer) raises PeerFailure when a peer announced its departure with
    ``leave()`` or its counter has not moved for ``timeout`` seconds.  A peer
    that dies in the middle of a layer is caught by the process group's own
    (short) timeout instead.  ``abort()`` tears the process group down without
    waiting on the peers; since check() runs between layers, no collective is
    in flight then.  The thread touches only the store, never a GPU."""

    def __init__(self, store, rank: int, world: int, interval: float = 0.05,
                 timeout: float = 2.0, prefix: str = "astro_moe_ep"):
        import threading
        import time

        self.store, self.rank, self.world = store, rank, world
        self.interval, self.timeout, self.prefix = interval, timeout, prefix
        self._time = time.monotonic
        self._lock = threading.Lock()
        self._stop = threading.Event()
        now = self._time()
        self._seen = {r: (-1, now) for r in range(world) if r != rank}  # (count, last change)
        self._left = set()
        self._beat()
        self._poll()
        self._thread = threading.Thread(target=self._run, name="astro-moe-heartbeat", daemon=True)
        self._thread.start()

    def _key(self, what, r):
        return f"{self.prefix}/{what}/{r}"

    def _beat(self):
        self.store.add(self._key("hb", self.rank), 1)

    def _poll(self):
        now = self._time()
        for r in list(self._seen):
            left = self.store.add(self._key("left", r), 0) > 0
            count = self.store.add(self._key("hb", r), 0)
            with self._lock:
                if left:
                    self._left.add(r)
                if count != self._seen[r][0]:
                    self._seen[r] = (count, now)

    def _run(self):
        while not self._stop.wait(self.interval):
            try:
                self._beat()
                self._poll()
            except Exception:  # the store went away: nothing left to report to
                return

    def check(self) -> None:
        now = self._time()
        with self._lock:
            left = sorted(self._left)
            dead = [r for r, (_, since) in self._seen.items()
                    if r not in self._left and now - since > self.timeout]
        if left:
            raise PeerFailure(left, "left")
        if dead:
            raise PeerFailure(dead, f"sent no heartbeat for {self.timeout:.1f} s")

    def stop(self) -> None:
        """Stops this rank's heartbeat (its peers will see it go silent)."""
        self._stop.set()
        self._thread.join(timeout=1.0)

    def leave(self) -> None:
        """Announces that this rank leaves between layers, then stops beating."""
        self.store.add(self._key("left", self.rank), 1)
        self.stop()

    @staticmethod
    def abort(group=None) -> None:
        """Destroys the process group without a final collective (NCCL's
        communicators are aborted by the backend on destruction)."""
        if dist.is_initialized():
            pg = group or dist.group.WORLD
            abort = getattr(pg, "abort", None)
            try:
                if callable(abort):
                    abort()
            finally:
                dist.destroy_process_group(group)


def expert_range(rank: int, world: int, experts: int) -> Tuple[int, int]:
    """(first, count) of the experts rank `rank` owns; experts % world == 0."""
    if experts % world != 0:
        raise ValueError(f"{experts} experts do not split evenly over {world} ranks")
    n = experts // world
    return rank * n, n


def local_expert_weights(weights: dict, first: int, count: int) -> dict:
    """The layer's weights with only experts [first, first + count) in the routed
    stacks (router, shared expert and its gate unchanged)."""
    out = {"config": dict(weights["config"])}
    for k, v in weights.items():
        if k == "config" or v is None:
            continue
        if k.split("_")[0] in ("gate", "up", "down"):
            out[k] = v[first:first + count]
            if isinstance(out[k], torch.Tensor):
                out[k] = out[k].contiguous()
        else:
            out[k] = v
    return out


class CudaExpertShard:
    """This rank's part of expert-parallel MoE layers on its GPU (libastro_moe).

    ``layers``: per layer, the weights dict of astronomical_b200.synthetic (full
    router, shared expert; routed stacks may be full or already local)."""

    def __init__(self, layers: Sequence[dict], rank: int, world: int, device: int = 0,
                 use_tensor_cores: int = 0, max_tokens: int = 4096):
        self.rank, self.world = rank, world
        self.device = torch.device("cuda", device)
        cfg = layers[0]["config"]
        self.cfg = dict(cfg)
        self.E = cfg["experts"]
        self.first, self.count = expert_range(rank, world, self.E)
        opts = _lib.Options()
        opts.max_tokens = max_tokens
        opts.use_tensor_cores = use_tensor_cores
        ctx = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(_lib.lib().astro_moe_ctx_create(device, ctypes.c_void_p(
                torch.cuda.current_stream(self.device).cuda_stream), ctypes.byref(opts),
                ctypes.byref(ctx)))
        self.ctx = ctx
        self._keep = []
        for li, w in enumerate(layers):
            if w["gate_q"].shape[0] != self.count:
                w = local_expert_weights(w, self.first, self.count)
            self._register(li, w)

    def _register(self, layer: int, w: dict):
        dev = self.device
        t = moe.device_weights(w, dev)
        self._keep.append(t)
        lw = moe.layer_weights_struct(t, self.cfg, self.E)
        check(_lib.lib().astro_moe_ep_register_layer(self.ctx, layer, ctypes.byref(lw),
                                                     self.first, self.count))

    def _bind(self):
        check(_lib.lib().astro_moe_ctx_set_stream(
            self.ctx, ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)))

    # -- the three compute steps of one layer ------------------------------------
    def dispatch(self, layer: int, x: torch.Tensor):
        T, H = x.shape
        K = self.cfg["top_k"]
        send = torch.empty((T * K, H), dtype=torch.bfloat16, device=x.device)
        offsets = torch.empty(self.E + 1, dtype=torch.int32, device=x.device)
        self._bind()
        check(_lib.lib().astro_moe_ep_dispatch(self.ctx, layer, _ptr(x), T, _ptr(send),
                                               _ptr(offsets)))
        return send, offsets

    def experts(self, layer: int, recv_rows: torch.Tensor, recv_counts: torch.Tensor,
                recv_total: int, x: torch.Tensor) -> torch.Tensor:
        out = torch.empty_like(recv_rows)
        self._bind()
        check(_lib.lib().astro_moe_ep_experts(self.ctx, layer, _ptr(recv_rows), _ptr(recv_counts),
                                              self.world, recv_total, _ptr(x), x.shape[0],
                                              _ptr(out)))
        return out

    def combine(self, layer: int, returned: Optional[torch.Tensor], T: int) -> torch.Tensor:
        """returned=None: the rows the peer exchange stored in this rank's return buffer."""
        out = torch.empty((T, self.cfg["hidden"]), dtype=torch.bfloat16, device=self.device)
        self._bind()
        check(_lib.lib().astro_moe_ep_combine(self.ctx, layer, _ptr(returned), T, _ptr(out)))
        return out

    # -- peer-memory exchange ------------------------------------------------------
    def connect_exchange(self, max_tokens: int, group=None) -> None:
        """Allocates this rank's receive / return buffers, trades IPC handles with
        the other ranks (all-gather) and maps theirs."""
        K, H = self.cfg["top_k"], self.cfg["hidden"]
        handles = (ctypes.c_ubyte * 192)()
        check(_lib.lib().astro_moe_ep_exchange_create(self.ctx, self.world, self.rank, H,
                                                      self.world * max_tokens * K, max_tokens * K,
                                                      ctypes.byref(handles)))
        mine = torch.tensor(bytearray(handles), dtype=torch.uint8, device=self.device)
        everyone = torch.empty((self.world, 192), dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(everyone, mine, group=group)
        buf = bytes(everyone.cpu().numpy().tobytes())
        arr = (ctypes.c_ubyte * len(buf)).from_buffer_copy(buf)
        check(_lib.lib().astro_moe_ep_exchange_connect(self.ctx, ctypes.byref(arr)))

    def route(self, layer: int, x: torch.Tensor) -> torch.Tensor:
        offsets = torch.empty(self.E + 1, dtype=torch.int32, device=x.device)
        self._bind()
        check(_lib.lib().astro_moe_ep_route(self.ctx, layer, _ptr(x), x.shape[0], _ptr(offsets)))
        return offsets

    @staticmethod
    def _i64(vals):
        return (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])

    def push(self, layer: int, x: torch.Tensor, send_starts, dest_offsets) -> None:
        self._bind()
        check(_lib.lib().astro_moe_ep_push(self.ctx, layer, _ptr(x), x.shape[0],
                                           self._i64(send_starts), self._i64(dest_offsets)))

    def experts_push(self, layer: int, recv_counts: torch.Tensor, recv_total: int, x: torch.Tensor,
                     recv_starts, return_offsets) -> None:
        self._bind()
        check(_lib.lib().astro_moe_ep_experts_push(self.ctx, layer, _ptr(recv_counts), recv_total,
                                                   _ptr(x), x.shape[0], self._i64(recv_starts),
                                                   self._i64(return_offsets)))

    def post_counts(self, layer: int, offsets: torch.Tensor) -> None:
        self._bind()
        check(_lib.lib().astro_moe_ep_post_counts(self.ctx, layer, _ptr(offsets)))

    def push_dev(self, layer: int, x: torch.Tensor) -> None:
        self._bind()
        check(_lib.lib().astro_moe_ep_push_dev(self.ctx, layer, _ptr(x), x.shape[0]))

    def experts_dev(self, layer: int, x: torch.Tensor) -> None:
        self._bind()
        check(_lib.lib().astro_moe_ep_experts_dev(self.ctx, layer, _ptr(x), x.shape[0]))

    def exchange_counts(self):
        """[world][world] rows rank s sent rank d in the last layer (synchronises)."""
        m = (ctypes.c_uint32 * (self.world * self.world))()
        check(_lib.lib().astro_moe_ep_exchange_counts(self.ctx, m))
        return [[m[s * self.world + d] for d in range(self.world)] for s in range(self.world)]

    def kernel_launches(self, reset: bool = True) -> int:
        a = _lib.Attribution()
        check(_lib.lib().astro_moe_ctx_read_attribution(self.ctx, ctypes.byref(a), int(reset)))
        return int(a.kernel_launches)

    def close(self):
        if getattr(self, "ctx", None):
            _lib.lib().astro_moe_ctx_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ExpertParallelBlock:
    """One layer's exchange: dispatch -> all-to-all -> experts -> all-to-all -> combine.

    ``shard`` provides dispatch/experts/combine for this rank; ``group`` is the
    process group of the `world` ranks (default: the world group)."""

    def __init__(self, shard, rank: int, world: int, experts: int, group=None,
                 exchange: str = "nccl", watchdog: Optional[PeerWatchdog] = None):
        """exchange: "nccl" (all-to-all-v of rows through torch.distributed),
        "peer" (rows stored into the peers' buffers by the dispatch and expert
        kernels, placements computed on the device from count mailboxes: no host
        synchronisation), or "peer_host" (the same stores, placements computed on
        the host after reading the counts back).  The peer modes need
        ``shard.connect_exchange`` first."""
        self.shard, self.rank, self.world, self.E = shard, rank, world, experts
        self.El = expert_range(rank, world, experts)[1]
        self.group = group
        self.exchange = exchange if world > 1 else "nccl"
        self.last_splits: Optional[Tuple[List[int], List[int]]] = None
        self._flag = None
        self.watchdog = watchdog

    def plan(self, offsets: torch.Tensor):
        """Per-expert counts out, per-source counts in; returns host splits and the
        device counts [world][El] this rank receives."""
        counts = (offsets[1:] - offsets[:-1]).to(torch.int32).contiguous()
        if self.world == 1:
            recv_counts = counts
        else:
            recv_counts = torch.empty(self.world * self.El, dtype=torch.int32, device=offsets.device)
            dist.all_to_all_single(recv_counts, counts, group=self.group)
        offs_h = offsets.cpu()
        rc_h = recv_counts.cpu()
        send_splits = [int(offs_h[(r + 1) * self.El] - offs_h[r * self.El]) for r in range(self.world)]
        recv_splits = [int(v) for v in rc_h.view(self.world, self.El).sum(1)]
        return send_splits, recv_splits, recv_counts

    def _barrier(self, device):
        # stream-ordered: no rank passes until every rank's prior kernels finished
        if self._flag is None:
            self._flag = torch.zeros(1, dtype=torch.int32, device=device)
        dist.all_reduce(self._flag, group=self.group)

    def _forward_peer(self, layer: int, x: torch.Tensor, mark) -> torch.Tensor:
        T, W, me = x.shape[0], self.world, self.rank
        offsets = self.shard.route(layer, x)
        mark("dispatch")
        counts = (offsets[1:] - offsets[:-1]).to(torch.int32).contiguous()
        recv_counts = torch.empty(W * self.El, dtype=torch.int32, device=x.device)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        per_dest = counts.view(W, self.El).sum(1).to(torch.int32)
        M = torch.empty(W * W, dtype=torch.int32, device=x.device)  # flat: NCCL and gloo
        dist.all_gather_into_tensor(M, per_dest, group=self.group)
        Mh = M.view(W, W).cpu().tolist()  # Mh[s][d]: rows rank s sends to rank d
        send_starts = [sum(Mh[me][:d]) for d in range(W)]
        dest_offsets = [sum(Mh[s][d] for s in range(me)) for d in range(W)]
        recv_starts = [sum(Mh[s][me] for s in range(q)) for q in range(W)]
        return_offsets = [sum(Mh[s][:me]) for s in range(W)]
        recv_total = sum(Mh[s][me] for s in range(W))
        self.last_splits = ([Mh[me][d] for d in range(W)], [Mh[s][me] for s in range(W)])
        self.shard.push(layer, x, send_starts, dest_offsets)
        self._barrier(x.device)
        mark("exchange_out")
        self.shard.experts_push(layer, recv_counts, recv_total, x, recv_starts, return_offsets)
        mark("experts")
        self._barrier(x.device)
        mark("exchange_back")
        y = self.shard.combine(layer, None, T)
        mark("combine")
        return y

    def _forward_peer_dev(self, layer: int, x: torch.Tensor, mark) -> torch.Tensor:
        offsets = self.shard.route(layer, x)
        self.shard.post_counts(layer, offsets)
        mark("dispatch")
        self._barrier(x.device)
        self.shard.push_dev(layer, x)
        self._barrier(x.device)
        mark("exchange_out")
        self.shard.experts_dev(layer, x)
        mark("experts")
        self._barrier(x.device)
        mark("exchange_back")
        y = self.shard.combine(layer, None, x.shape[0])
        mark("combine")
        return y

    def splits(self):
        """(rows this rank sent each rank, rows it received from each rank) of the last layer."""
        if self.exchange == "peer":
            M = self.shard.exchange_counts()
            return ([M[self.rank][d] for d in range(self.world)],
                    [M[s][self.rank] for s in range(self.world)])
        return self.last_splits

    def forward_host(self, layer: int, hx: torch.Tensor, hy: Optional[torch.Tensor] = None,
                     device=None) -> torch.Tensor:
        """The layer on host buffers: ``hx`` (this rank's tokens, pinned for an
        asynchronous upload) is copied to ``device``, the layer runs there and
        its output is copied into ``hy`` (pinned, same shape as ``hx``; a new host
        tensor when omitted).  The copies are queued on the current stream; with
        ``hy`` given the call does not wait for them."""
        x = hx.to(device if device is not None else hx.device, non_blocking=True)
        y = self.forward(layer, x)
        if hy is None:
            return y.cpu()
        hy.copy_(y, non_blocking=True)
        return hy

    def forward(self, layer: int, x: torch.Tensor, marks=None) -> torch.Tensor:
        """``marks``: optional callable recording a named point (stage timing)."""
        T = x.shape[0]
        mark = marks or (lambda name: None)
        if self.watchdog is not None:
            self.watchdog.check()  # raises PeerFailure before any collective of this layer
        if self.exchange == "peer":
            return self._forward_peer_dev(layer, x, mark)
        if self.exchange == "peer_host":
            return self._forward_peer(layer, x, mark)
        send, offsets = self.shard.dispatch(layer, x)
        mark("dispatch")
        send_splits, recv_splits, recv_counts = self.plan(offsets)
        self.last_splits = (send_splits, recv_splits)
        recv_total = sum(recv_splits)
        if self.world == 1:
            recv = send
        else:
            recv = send.new_empty((recv_total,) + tuple(send.shape[1:]))
            dist.all_to_all_single(recv, send, recv_splits, send_splits, group=self.group)
        mark("exchange_out")
        out_rows = self.shard.experts(layer, recv, recv_counts, recv_total, x)
        mark("experts")
        if self.world == 1:
            returned = out_rows
        else:
            returned = torch.empty_like(send)
            dist.all_to_all_single(returned, out_rows, send_splits, recv_splits, group=self.group)
        mark("exchange_back")
        y = self.shard.combine(layer, returned, T)
        mark("combine")
        return y


class ExpertParallelStack:
    """A stack of expert-parallel MoE layers (config 3: the decoder's attention is
    replaced by identity, so every layer reads the same hidden states)."""

    def __init__(self, shard, rank: int, world: int, experts: int, layers: int, group=None):
        self.block = ExpertParallelBlock(shard, rank, world, experts, group)
        self.layers = layers

    def forward(self, x: torch.Tensor) -> List[torch.Tensor]:
        return [self.block.forward(l, x) for l in range(self.layers)]
