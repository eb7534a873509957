"""Expert parallelism on real GPUs: ranks over NCCL, each holding 256/world
experts of the config-1 block, must reproduce the single-GPU block on their own
tokens (routing bit-exact, outputs within the block tolerance).  Needs at least
two GPUs; runs the ranks as child processes with NVLS off and a short
process-group timeout."""
import os
import socket
import tempfile
from datetime import timedelta

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, T, outdir, zipf, exchange):
    import torch.distributed as dist

    from astronomical_b200 import moe, synthetic
    from astronomical_b200.ep import CudaExpertShard, ExpertParallelBlock

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    cfg = dict(synthetic.CONFIGS[2 if zipf else 1])
    layers = [synthetic.make_block_weights_torch(cfg, seed=77 + l, device=dev) for l in range(2)]
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    x = torch.randn((T, cfg["hidden"]), generator=g, device=dev).to(torch.bfloat16)
    if zipf:
        x[:, 0] = 1.0
    shard = CudaExpertShard(layers, rank, world, device=rank, max_tokens=T)
    if exchange != "nccl":
        shard.connect_exchange(T)
    block = ExpertParallelBlock(shard, rank, world, cfg["experts"], exchange=exchange)
    for l in range(2):
        y = block.forward(l, x)
        ref = moe.Qwen3_5MoEBlock(layers[l], device=rank, max_tokens=T)
        y_ref = ref.forward(x)
        torch.cuda.synchronize()
        np.save(os.path.join(outdir, f"y_{rank}_{l}.npy"), y.view(torch.int16).cpu().numpy())
        np.save(os.path.join(outdir, f"r_{rank}_{l}.npy"), y_ref.view(torch.int16).cpu().numpy())
        ref.close()
    torch.cuda.synchronize()
    dist.barrier()  # no peer still uses this rank's exchange buffers
    shard.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("exchange", ["nccl", "peer_host", "peer"])
@pytest.mark.parametrize("T,zipf", [(512, False), (96, True)])
def test_expert_parallel_matches_single_gpu_block(T, zipf, exchange, world):
    import torch.multiprocessing as mp

    from tests.helpers import assert_block_close

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, world, port, T, d, zipf, exchange))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=600)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        for r in range(world):
            for l in range(2):
                got = np.load(os.path.join(d, f"y_{r}_{l}.npy")).view(np.uint16)
                ref = np.load(os.path.join(d, f"r_{r}_{l}.npy")).view(np.uint16)
                # the same arithmetic per row: expected bit-identical, held to the
                # block tolerance
                assert_block_close(got, ref)


def _rank_oracle(rank, world, port, T, rows, outdir):
    """One rank of the device-planned peer exchange on the config-1 block (numpy
    weights, identical on every rank), then the oracle from this rank's hidden
    states on a subset of its rows, with the arithmetic of the kernels the
    single-GPU block ran at this T."""
    import json

    import torch.distributed as dist

    from astronomical_b200 import moe, synthetic
    from astronomical_b200.ep import CudaExpertShard, ExpertParallelBlock
    from oracle import oracle as O
    from tests.helpers import oracle_arith, reference_metrics, to_np_bf16

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=120))
    cfg = dict(synthetic.CONFIGS[1])
    w = synthetic.make_block_weights(cfg, seed=91)
    x_np = synthetic.make_hidden_states(T, cfg["hidden"], seed=500 + rank)
    x = torch.from_numpy(x_np.view(np.int16)).view(torch.bfloat16).to(dev)
    shard = CudaExpertShard([w], rank, world, device=rank, max_tokens=T)
    shard.connect_exchange(T)
    block = ExpertParallelBlock(shard, rank, world, cfg["experts"], exchange="peer")
    y = block.forward(0, x)
    ref = moe.Qwen3_5MoEBlock(w, device=rank, max_tokens=T)
    y_ref = ref.forward(x)
    kernels = ref.last_path()
    torch.cuda.synchronize()
    same = bool(torch.equal(y, y_ref))
    got = to_np_bf16(y)
    ref.close()
    dist.barrier()  # no peer still uses this rank's exchange buffers
    shard.close()
    dist.destroy_process_group()
    sub = np.unique(np.linspace(0, T - 1, rows).astype(np.int64))
    y_or, _, _ = O.moe_block_forward(w, x_np, token_subset=sub, arith=oracle_arith(kernels))
    m = reference_metrics(got[sub], y_or)
    with open(os.path.join(outdir, f"oracle_{rank}.json"), "w") as f:
        json.dump(dict(same_as_single_gpu=same, kernels=kernels, rows=int(sub.size), **m), f)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_expert_parallel_matches_oracle(world):
    """Expert parallelism at config-1 size (4096 tokens per rank, 256 / world
    experts per GPU, the device-planned peer exchange) against the oracle run
    from each rank's hidden states: bit-exact on a 256-row subset of every rank,
    and bit-identical to the single-GPU block on all rows."""
    import json

    import torch.multiprocessing as mp

    from tests.helpers import record_parity

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_rank_oracle, args=(r, world, port, 4096, 256, d))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=900)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        for r in range(world):
            with open(os.path.join(d, f"oracle_{r}.json")) as f:
                res = json.load(f)
            record_parity(f"ep_world{world}_rank{r}", **res)
            assert res["same_as_single_gpu"], (world, r, res)
            assert res["n_differ"] == 0, (world, r, res)
