"""Row-sharded pool across real GPUs: one process per GPU, peers mapped with
CUDA IPC handles exchanged over a gloo group, the three phases run as one
call on each rank.  Each rank's output must match the single-GPU layer on
its own tokens with the whole table (slots and weights identical, outputs
within 1e-5 relative).  Skipped on a box with fewer GPUs than ranks: ranks
that wait on each other never share a GPU."""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir, vdt_name):
    import datetime

    import torch.distributed as dist

    from model_b200 import MemoryLayer, MemoryPool
    from model_b200.shard import ShardedMemoryLayer, connect, shard_values

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        vdt = getattr(torch, vdt_name)
        pool = MemoryPool(n_sub_keys=128, heads=4, d_key=128, d_value=128, top_k=16)
        layer = MemoryLayer(pool, d_model=128, layer=1)
        params = layer.init(0, values_dtype=vdt)                      # same seed: same table on every rank
        M = 777
        h = torch.randn(M, 128, device="cuda", generator=torch.Generator("cuda").manual_seed(5 + rank))
        comm = connect(pool.config(M, vdt, 128))
        local = dict(params, pool=dict(params["pool"], values=shard_values(params["pool"]["values"], rank, world)))
        sharded = ShardedMemoryLayer(layer, comm)
        for i in range(4):   # plain and split (overlapped halves) calls, alternating
            y, mem, aux = sharded.apply(local, h, check=True, split=bool(i % 2))
        torch.cuda.synchronize()
        dist.barrier()
        y0, mem0, aux0 = layer.apply(params, h, check=True)
        torch.cuda.synchronize()
        same = bool(torch.equal(aux["slots"], aux0["slots"]) and torch.equal(aux["weights"], aux0["weights"]))
        e_mem = float((mem - mem0).abs().max() / mem0.abs().max())
        e_y = float((y - y0).abs().max() / y0.abs().max())
        np.save(os.path.join(outdir, f"r{rank}.npy"), np.array([float(same), e_mem, e_y]))
        dist.barrier()
        comm.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("vdt_name", ["float32", "bfloat16"])
def test_sharded_across_gpus(world, vdt_name, tmp_path):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), vdt_name), nprocs=world, join=True)
    for rank in range(world):
        same, e_mem, e_y = np.load(tmp_path / f"r{rank}.npy")
        assert same == 1.0, f"rank {rank}: routing differs"
        assert e_mem <= 1e-5 and e_y <= 1e-5, f"rank {rank}: mem {e_mem:.2e} y {e_y:.2e}"
