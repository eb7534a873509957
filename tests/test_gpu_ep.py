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
