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
        # 2600 tokens: 21 score tiles, so the split calls take the overlapped
        # path (second half's score beside the first half's gather)
        M = 2600
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


def _row_worker(rank, world, port, outdir):
    import datetime

    import torch.distributed as dist

    from model_b200 import _lib as L
    from model_b200.shard import connect
    from model_b200.sparse import sharded_rowwise_adagrad
    from oracle import memlayer_ref as ref

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        n_sub, H, k, d, lr, clip, rest = 64, 4, 8, 64, 0.05, 1.0, 0.25
        N = n_sub * n_sub
        rng = np.random.default_rng(1)                              # same table on every rank
        values = rng.standard_normal((N, d)).astype(np.float32)
        acc = (rng.random(N) * 0.1).astype(np.float32)
        per = []
        for r in range(world):                                       # every rank's reads (seeded)
            rr = np.random.default_rng(50 + r)
            M = 40 + 17 * r
            hot = np.random.default_rng(3).permutation(N)
            s = hot[np.minimum(rr.zipf(1.1, size=(M, H, k)), N) - 1].astype(np.int32)
            w = rr.random((M, H, k)).astype(np.float32)
            g = (rr.standard_normal((M, d)) * 0.1).astype(np.float32)
            per.append((s, w, g))
        cfg = L.MemlayerConfig(tokens=40 + 17 * (world - 1), heads=H, n_sub_keys=n_sub, d_key=16, d_value=d,
                               top_k=k, d_model=16, values_dtype=L.F32, routing_noise=0.0, min_temperature=1.0,
                               max_temperature=1.0)
        comm = connect(cfg, n_reads=1)
        v = torch.from_numpy(values[rank::world].copy()).cuda()
        a = torch.from_numpy(acc[rank::world].copy()).cuda()
        s, w, g = per[rank]
        out = sharded_rowwise_adagrad(v, a, {"slots": [torch.from_numpy(s).cuda()],
                                             "weights": [torch.from_numpy(w).cuda()]},
                                      {0: torch.from_numpy(g).cuda()}, [0], comm, lr=lr, grad_clip=clip,
                                      rest_sq_norm=torch.tensor([rest]), check=True)
        torch.cuda.synchronize()
        dist.barrier()
        uniq, rows = ref.fetched_row_grads_sharded(per, N)
        scale = ref.clip_scale(rest, rows, clip)
        ref.rowwise_adagrad(values, acc, uniq, rows * scale, lr)
        e_v = float(np.abs(v.cpu().numpy() - values[rank::world]).max() / np.abs(values).max())
        e_a = float(np.abs(a.cpu().numpy() - acc[rank::world]).max() / np.abs(acc).max())
        e_s = abs(float(out["clip_scale"]) - float(scale)) / float(scale)
        np.save(os.path.join(outdir, f"row{rank}.npy"), np.array([e_v, e_a, e_s]))
        dist.barrier()
        comm.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_owner_sharded_update_across_gpus(world, tmp_path):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_row_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for rank in range(world):
        e_v, e_a, e_s = np.load(tmp_path / f"row{rank}.npy")
        assert e_v <= 1e-5 and e_a <= 1e-5 and e_s <= 1e-6, f"rank {rank}: {e_v:.2e} {e_a:.2e} {e_s:.2e}"


def _bwd_worker(rank, world, port, outdir):
    import datetime

    import torch.distributed as dist

    from model_b200 import MemoryLayer, MemoryPool
    from model_b200.shard import ShardedMemoryLayer, connect, shard_values

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        pool = MemoryPool(n_sub_keys=128, heads=4, d_key=128, d_value=128, top_k=16, min_temperature=5.0)
        layer = MemoryLayer(pool, d_model=128, layer=1)
        params = layer.init(0)                                        # same seed: same weights on every rank
        M = 300 + 77 * rank
        gen = torch.Generator("cuda").manual_seed(9 + rank)
        h = torch.randn(M, 128, device="cuda", generator=gen)
        dy = torch.randn(M, 128, device="cuda", generator=gen)
        comm = connect(pool.config(300 + 77 * (world - 1), torch.float32, 128))
        local = dict(params, pool=dict(params["pool"], values=shard_values(params["pool"]["values"], rank, world)))
        sharded = ShardedMemoryLayer(layer, comm)
        for _ in range(2):                                            # two steps on one communicator
            y, mem, aux, ctx = sharded.apply_train(local, h, train=False, check=True)
            g = sharded.backward(ctx, dy, balance_coef=0.3, check=True)
        torch.cuda.synchronize()
        dist.barrier()
        y0, mem0, aux0, ctx0 = layer.apply_train(params, h, train=False, check=True)
        g0 = layer.backward(ctx0, dy, balance_coef=0.3, check=True)
        torch.cuda.synchronize()
        errs = [0.0 if torch.equal(aux["slots"], aux0["slots"]) else 1.0]
        for a, b in ((g["h"], g0["h"]), (g["probe"], g0["probe"]),
                     (g["router_1"]["kernel"], g0["router_1"]["kernel"]),
                     (g["mem_gate_1"]["kernel"], g0["mem_gate_1"]["kernel"]),
                     (g["mem_out_1"]["kernel"], g0["mem_out_1"]["kernel"]),
                     (g["pool"]["sub_keys"], g0["pool"]["sub_keys"]),
                     (g["pool"]["log_temperature"], g0["pool"]["log_temperature"])):
            errs.append(float((a - b).abs().max() / b.abs().max().clamp_min(1e-12)))
        np.save(os.path.join(outdir, f"bwd{rank}.npy"), np.array(errs))
        dist.barrier()
        comm.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_backward_across_gpus(world, tmp_path):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_bwd_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for rank in range(world):
        errs = np.load(tmp_path / f"bwd{rank}.npy")
        assert errs[0] == 0.0, f"rank {rank}: routing differs"
        assert (errs[1:] <= 1e-5).all(), f"rank {rank}: gradient errors {errs[1:]}"


def _staged_worker(rank, world, port, outdir):
    import datetime

    import torch.distributed as dist

    from model_b200 import MemoryLayer, MemoryPool
    from model_b200.shard import StagedCall, shard_values

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        pool = MemoryPool(n_sub_keys=128, heads=4, d_key=128, d_value=128, top_k=16)
        layer = MemoryLayer(pool, d_model=128, layer=1)
        params = layer.init(0)                                        # same seed: same table on every rank
        M = 777
        h = torch.randn(M, 128, device="cuda", generator=torch.Generator("cuda").manual_seed(5 + rank))
        local = dict(params, pool=dict(params["pool"], values=shard_values(params["pool"]["values"], rank, world)))
        call = StagedCall(layer, local, h, rank, world)
        for _ in range(3):                                            # buffers reused across calls
            call.run()
        call.check()
        y, mem, aux = call.result()
        torch.cuda.synchronize()
        y0, mem0, aux0 = layer.apply(params, h, check=True)
        torch.cuda.synchronize()
        same = bool(torch.equal(aux["slots"], aux0["slots"]) and torch.equal(aux["weights"], aux0["weights"]))
        e_mem = float((mem - mem0).abs().max() / mem0.abs().max())
        e_y = float((y - y0).abs().max() / y0.abs().max())
        np.save(os.path.join(outdir, f"st{rank}.npy"), np.array([float(same), e_mem, e_y]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_staged_nccl_exchange_across_gpus(world, tmp_path):
    """The NCCL-staged exchange (all-gather of the routing entries,
    reduce-scatter of the partial rows) against the single-GPU layer."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_staged_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for rank in range(world):
        same, e_mem, e_y = np.load(tmp_path / f"st{rank}.npy")
        assert same == 1.0, f"rank {rank}: routing differs"
        assert e_mem <= 1e-5 and e_y <= 1e-5, f"rank {rank}: mem {e_mem:.2e} y {e_y:.2e}"
