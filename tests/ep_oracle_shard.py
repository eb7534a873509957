"""Test infrastructure: the expert arithmetic of an expert-parallel rank computed
by the CPU oracle, with the dispatch / experts / combine interface of
astronomical_b200.ep.CudaExpertShard.  Rows travel as int32 tensors holding two
bf16 bit patterns each (gloo's all-to-all has no 16-bit integer type), so gloo
moves them unchanged."""
import numpy as np
import torch

from oracle import oracle as O


def _np(t):
    return t.numpy().view(np.uint16) if isinstance(t, torch.Tensor) else t


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32))


class OracleExpertShard:
    def __init__(self, layers, rank, world):
        self.layers = layers
        self.rank, self.world = rank, world
        cfg = layers[0]["config"]
        self.cfg = cfg
        self.E, self.K = cfg["experts"], cfg["top_k"]
        self.El = self.E // world
        self.first = rank * self.El
        self.state = {}

    def dispatch(self, layer, x):
        w = self.layers[layer]
        xs = _np(x)
        logits = O.matmul_bf16_nt(xs, w["router_w"])
        ids, scores = O.route_experts(logits, self.K, self.cfg.get("normalize", True))
        srt = O.sort_expert_assignments(ids, self.E)
        send = xs[srt["sorted_tokens"].astype(np.int64)]
        self.state[layer] = dict(ids=ids, scores=scores, srt=srt)
        return _t(send), torch.from_numpy(srt["expert_offsets"].astype(np.int32))

    def experts(self, layer, recv, recv_counts, recv_total, x):
        w = self.layers[layer]
        G, B = self.cfg["group"], self.cfg["bits"]
        rows = _np(recv)
        counts = recv_counts.numpy().reshape(self.world, self.El)
        experts = np.concatenate([np.full(int(counts[s, e]), self.first + e, np.uint32)
                                  for s in range(self.world) for e in range(self.El)]
                                 + [np.zeros(0, np.uint32)])
        assert experts.size == recv_total
        if recv_total:
            gate = O.gather_qmm(rows, w["gate_q"], w["gate_s"], w["gate_b"], G, B, rhs_experts=experts)
            up = O.gather_qmm(rows, w["up_q"], w["up_s"], w["up_b"], G, B, rhs_experts=experts)
            act = O.swiglu(gate, up)
            out = O.gather_qmm(act, w["down_q"], w["down_s"], w["down_b"], G, B, rhs_experts=experts)
        else:
            out = np.zeros((0, rows.shape[1]), np.uint16)
        st = self.state[layer]
        if self.cfg.get("shared_intermediate", 0):
            xs = _np(x)
            sg = O.gather_qmm(xs, w["sgate_q"], w["sgate_s"], w["sgate_b"], G, B)
            su = O.gather_qmm(xs, w["sup_q"], w["sup_s"], w["sup_b"], G, B)
            st["shared"] = O.gather_qmm(O.swiglu(sg, su), w["sdown_q"], w["sdown_s"], w["sdown_b"], G, B)
            st["gate_logit"] = O.matmul_bf16_nt(xs, w["shared_gate_w"])
        return _t(out)

    def combine(self, layer, returned, T):
        st = self.state[layer]
        rows = _np(returned)
        inv = st["srt"]["inverse_order"]
        if T * self.K >= 64:
            sparse = O.sorted_expert_weighted_sum(rows, inv, st["scores"])
        else:
            slots = rows[inv.astype(np.int64)].reshape(T, self.K, -1)
            sparse = O.unsorted_expert_weighted_sum(slots, st["scores"])
        if "shared" in st:
            sparse = O.combine_sparse_and_shared(sparse, st["shared"], st["gate_logit"])
        return _t(sparse)


class PeerOracleShard(OracleExpertShard):
    """The peer exchange of ExpertParallelBlock(exchange="peer_host") with the
    oracle's arithmetic.  Each rank's receive and return buffers are files mapped
    by every rank (np.memmap), standing in for the CUDA IPC mappings of
    astro_moe_ep_exchange_connect; push and experts_push store rows at the
    placements the block computes, as astro_moe_ep_push (the rows for rank d go
    to d's receive buffer at dest_offsets[d]) and astro_moe_ep_experts_push (the
    rows received from rank s return to s's return buffer at return_offsets[s])
    do.  The block's collectives order the stores, as on the GPUs."""

    def connect_exchange(self, max_tokens, directory, group=None):
        import torch.distributed as dist

        H, K = self.cfg["hidden"], self.cfg["top_k"]
        self.recv_rows, self.ret_rows = self.world * max_tokens * K, max_tokens * K

        def path(kind, r):
            return f"{directory}/{kind}_{r}.bin"

        np.memmap(path("recv", self.rank), np.uint16, "w+", shape=(self.recv_rows, H)).flush()
        np.memmap(path("ret", self.rank), np.uint16, "w+", shape=(self.ret_rows, H)).flush()
        dist.barrier(group=group)
        self.recv = [np.memmap(path("recv", r), np.uint16, "r+", shape=(self.recv_rows, H))
                     for r in range(self.world)]
        self.ret = [np.memmap(path("ret", r), np.uint16, "r+", shape=(self.ret_rows, H))
                    for r in range(self.world)]

    def route(self, layer, x):
        send, offsets = self.dispatch(layer, x)
        self.state[layer]["send"] = _np(send)
        return offsets

    def push(self, layer, x, send_starts, dest_offsets):
        st = self.state[layer]
        offs = st["srt"]["expert_offsets"].astype(np.int64)
        for d in range(self.world):
            n = int(offs[(d + 1) * self.El] - offs[d * self.El])
            a, b = int(send_starts[d]), int(dest_offsets[d])
            assert b + n <= self.recv_rows
            self.recv[d][b:b + n] = st["send"][a:a + n]
            self.recv[d].flush()

    def experts_push(self, layer, recv_counts, recv_total, x, recv_starts, return_offsets):
        assert recv_total <= self.recv_rows
        rows = np.array(self.recv[self.rank][:recv_total])
        out = _np(self.experts(layer, _t(rows), recv_counts, recv_total, x))
        per_source = recv_counts.numpy().reshape(self.world, self.El).sum(1)
        for s in range(self.world):
            n, a, b = int(per_source[s]), int(recv_starts[s]), int(return_offsets[s])
            assert b + n <= self.ret_rows
            self.ret[s][b:b + n] = out[a:a + n]
            self.ret[s].flush()

    def combine(self, layer, returned, T):
        if returned is None:  # the peers stored this rank's rows in its return buffer
            returned = _t(np.array(self.ret[self.rank][:T * self.K]))
        return super().combine(layer, returned, T)
