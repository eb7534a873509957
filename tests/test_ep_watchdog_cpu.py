"""Peer failure detection for the expert-parallel block on CPU (gloo ranks as
processes; no GPU): a rank that dies between layers without a word, and a rank
that leaves cleanly, are both noticed by the survivor on the host before it
launches the next layer's collectives -- it raises PeerFailure within the
watchdog timeout instead of waiting for the process group's -- and the survivor
aborts its process group and exits normally."""
import datetime
import os
import socket
import tempfile
import time

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


def _rank_main(rank, world, port, mode, outdir):
    from astronomical_b200.ep import ExpertParallelBlock, PeerFailure, PeerWatchdog
    from tests.ep_oracle_shard import OracleExpertShard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    # the process group's own timeout is long: detection must come from the watchdog
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    store = dist.distributed_c10d._get_default_store()
    wd = PeerWatchdog(store, rank, world, interval=0.05, timeout=1.0)
    ws = [synthetic.make_block_weights(CFG, seed=10 + l) for l in range(3)]
    x_all = synthetic.make_hidden_states(8 * world, CFG["hidden"], seed=99)
    x = torch.from_numpy(np.ascontiguousarray(x_all[rank * 8:(rank + 1) * 8]).view(np.int32))
    block = ExpertParallelBlock(OracleExpertShard(ws, rank, world), rank, world, CFG["experts"],
                                watchdog=wd)
    block.forward(0, x)  # one layer together
    dist.barrier()
    if rank == world - 1:
        if mode == "leave":
            wd.leave()
            os._exit(0)  # between layers, nothing in flight
        wd.stop()  # dies silently: its heartbeat stops ...
        time.sleep(30)  # ... and it never joins the next layer
        os._exit(3)
    t0 = time.monotonic()
    outcome = "no failure seen"
    try:
        for l in range(1, 3):
            time.sleep(1.5)  # this rank's other work between MoE layers
            block.forward(l, x)
    except PeerFailure as e:
        outcome = f"{e.reason}|{e.ranks}"
    took = time.monotonic() - t0
    with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
        f.write(f"{outcome}\n{took}\n")
    PeerWatchdog.abort()
    wd.stop()
    os._exit(0)


@pytest.mark.parametrize("mode", ["die", "leave"])
def test_survivor_detects_a_lost_peer_between_layers(mode):
    world = 2
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, d)) for r in range(world)]
        for p in procs:
            p.start()
        procs[0].join(timeout=60)
        assert procs[0].exitcode == 0
        for p in procs[1:]:
            if p.is_alive():
                p.kill()
            p.join(timeout=10)
        outcome, took = open(os.path.join(d, "rank0.txt")).read().split("\n")[:2]
        if mode == "leave":
            assert outcome.startswith("left|[1]")
        else:
            assert outcome.startswith("sent no heartbeat") and outcome.endswith("[1]")
        # noticed at the next layer boundary, long before the group's 60 s timeout
        assert float(took) < 5.0
