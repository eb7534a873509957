"""Expert-parallel exchange logic on CPU: 2, 4 or 8 gloo ranks run
astronomical_b200.ep.ExpertParallelBlock with the oracle's expert arithmetic, and
every token's output must equal the single-process oracle block bit for bit
(routing, sort, dispatch splits, the expert-major permutation on the receiving
side, the return all-to-all and the combine all line up)."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from astronomical_b200 import synthetic

CFG = dict(tokens=0, hidden=128, experts=8, top_k=2, intermediate=64, shared_intermediate=64,
           group=64, bits=4, normalize=True, zipf=None)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, T, layers, outdir, skew):
    from astronomical_b200.ep import ExpertParallelBlock
    from tests.ep_oracle_shard import OracleExpertShard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = dict(CFG, zipf=skew)
    ws = [synthetic.make_block_weights(cfg, seed=10 + l) for l in range(layers)]
    x_all = synthetic.make_hidden_states(T * world, cfg["hidden"], seed=99, zipf=bool(skew))
    x = torch.from_numpy(np.ascontiguousarray(x_all[rank * T:(rank + 1) * T]).view(np.int32))
    block = ExpertParallelBlock(OracleExpertShard(ws, rank, world), rank, world, cfg["experts"])
    for l in range(layers):
        y = block.forward(l, x)
        np.save(os.path.join(outdir, f"y_{rank}_{l}.npy"), y.numpy().view(np.uint16))
    np.save(os.path.join(outdir, f"splits_{rank}.npy"), np.array(block.last_splits))
    # the host-buffer entry: the same layer into a caller's output buffer
    hy = torch.empty_like(x)
    block.forward_host(layers - 1, x.clone(), hy)
    np.save(os.path.join(outdir, f"yh_{rank}.npy"), hy.numpy().view(np.uint16))
    dist.destroy_process_group()


# world 8 is the scaling run's size: one expert per rank; with 2 tokens per rank
# most ranks receive no rows from most others
@pytest.mark.parametrize("T,skew,world", [(40, None, 2), (3, None, 2), (24, 1.1, 2), (16, 1.1, 4),
                                          (12, 1.1, 8), (2, None, 8)])
def test_expert_parallel_exchange_matches_single_process_oracle(T, skew, world):
    from oracle import oracle as O

    layers = 2
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, world, port, T, layers, d, skew))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        cfg = dict(CFG, zipf=skew)
        x_all = synthetic.make_hidden_states(T * world, cfg["hidden"], seed=99, zipf=bool(skew))
        for l in range(layers):
            w = synthetic.make_block_weights(cfg, seed=10 + l)
            got = np.concatenate([np.load(os.path.join(d, f"y_{r}_{l}.npy")) for r in range(world)])
            # the oracle block over each rank's own tokens (the sorted/unsorted
            # switch depends on a rank's assignment count, as on one GPU)
            want = np.concatenate([O.moe_block_forward(w, x_all[r * T:(r + 1) * T])[0]
                                   for r in range(world)])
            assert np.array_equal(got, want)
        for r in range(world):
            assert np.array_equal(np.load(os.path.join(d, f"yh_{r}.npy")),
                                  np.load(os.path.join(d, f"y_{r}_{layers - 1}.npy")))
        # rows sent by rank a to rank b are the rows rank b received from rank a
        sp = [np.load(os.path.join(d, f"splits_{r}.npy")) for r in range(world)]
        for a in range(world):
            for b in range(world):
                assert sp[a][0][b] == sp[b][1][a]


def _rank_main_peer(rank, world, port, T, layers, outdir, skew):
    from astronomical_b200.ep import ExpertParallelBlock
    from tests.ep_oracle_shard import PeerOracleShard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = dict(CFG, zipf=skew)
    ws = [synthetic.make_block_weights(cfg, seed=10 + l) for l in range(layers)]
    x_all = synthetic.make_hidden_states(T * world, cfg["hidden"], seed=99, zipf=bool(skew))
    x = torch.from_numpy(np.ascontiguousarray(x_all[rank * T:(rank + 1) * T]).view(np.int32))
    shard = PeerOracleShard(ws, rank, world)
    shard.connect_exchange(T, outdir)
    block = ExpertParallelBlock(shard, rank, world, cfg["experts"], exchange="peer_host")
    for l in range(layers):
        y = block.forward(l, x)
        np.save(os.path.join(outdir, f"y_{rank}_{l}.npy"), y.numpy().view(np.uint16))
    np.save(os.path.join(outdir, f"splits_{rank}.npy"), np.array(block.last_splits))
    dist.destroy_process_group()


@pytest.mark.parametrize("T,skew,world", [(40, None, 2), (16, 1.1, 4), (12, 1.1, 8), (2, None, 8)])
def test_peer_exchange_placements_match_single_process_oracle(T, skew, world):
    """The peer exchange's host-computed placements (each rank's send starts, its
    offsets in every destination's receive buffer, the receive starts per source
    and the return offsets) move every row to the right place and back."""
    from oracle import oracle as O

    layers = 2
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_rank_main_peer, args=(r, world, port, T, layers, d, skew))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        cfg = dict(CFG, zipf=skew)
        x_all = synthetic.make_hidden_states(T * world, cfg["hidden"], seed=99, zipf=bool(skew))
        for l in range(layers):
            w = synthetic.make_block_weights(cfg, seed=10 + l)
            got = np.concatenate([np.load(os.path.join(d, f"y_{r}_{l}.npy")) for r in range(world)])
            want = np.concatenate([O.moe_block_forward(w, x_all[r * T:(r + 1) * T])[0]
                                   for r in range(world)])
            assert np.array_equal(got, want)
        sp = [np.load(os.path.join(d, f"splits_{r}.npy")) for r in range(world)]
        for a in range(world):
            for b in range(world):
                assert sp[a][0][b] == sp[b][1][a]

