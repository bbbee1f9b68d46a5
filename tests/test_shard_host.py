"""Host-side logic of the row-sharded pool, on CPU: the striping of the value
table, the C ABI's argument checks and sizes (no CUDA call is reached), and
world-size-2 gloo runs of the sharded read -- every rank gathers the rows it
owns for every rank's tokens and the token owner adds the partials in rank
order -- and of the sharded backward's dot exchange, checked against the
single-table oracle."""

import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch

from model_b200 import _lib as L
from model_b200.shard import exchange_handles, owner_of, shard_rows, shard_values


def test_shard_rows_matches_library():
    lib = L.lib()
    for N in (0, 1, 7, 64, 262144, 1000003):
        for world in (1, 2, 3, 4, 8):
            rows = [shard_rows(N, r, world) for r in range(world)]
            assert sum(rows) == N
            for r in range(world):
                assert lib.memlayer_shard_rows(N, r, world) == rows[r]


def test_shard_values_partition_the_table():
    t = torch.arange(50 * 3, dtype=torch.float32).reshape(50, 3)
    for world in (1, 2, 4, 8):
        parts = [shard_values(t, r, world) for r in range(world)]
        slots = torch.arange(50)
        own, row = owner_of(slots, world)
        for s in range(50):
            assert torch.equal(parts[int(own[s])][int(row[s])], t[s])


def _cfg(**kw):
    base = dict(tokens=64, heads=4, n_sub_keys=64, d_key=64, d_value=64, top_k=16, d_model=64,
                values_dtype=L.F32, routing_noise=0.0, min_temperature=10.0, max_temperature=100.0)
    base.update(kw)
    return L.MemlayerConfig(**base)


def test_comm_create_rejects_bad_ranks():
    lib = L.lib()
    h = C.c_void_p()
    for rank, world in ((0, 0), (0, 9), (-1, 2), (2, 2)):
        assert lib.memlayer_shard_comm_create(C.byref(_cfg()), rank, world, C.byref(h)) == L.ERR_BAD_SHAPE
        assert not h.value
    assert lib.memlayer_shard_comm_create(C.byref(_cfg()), 0, 2, None) == L.ERR_BAD_POINTER
    assert lib.memlayer_shard_comm_create(C.byref(_cfg(d_value=66)), 0, 2, C.byref(h)) == L.ERR_UNSUPPORTED
    assert lib.memlayer_shard_comm_destroy(None) == L.ERR_BAD_POINTER


def test_sharded_workspace_and_entry_checks():
    lib = L.lib()
    single, two, eight = C.c_size_t(), C.c_size_t(), C.c_size_t()
    cfg = _cfg()
    assert lib.memlayer_layer_workspace_size(C.byref(cfg), C.byref(single)) == L.OK
    assert lib.memlayer_shard_workspace_size(C.byref(cfg), 2, 1, C.byref(two)) == L.OK
    assert lib.memlayer_shard_workspace_size(C.byref(cfg), 8, 1, C.byref(eight)) == L.OK
    assert single.value < two.value <= eight.value
    assert lib.memlayer_shard_workspace_size(C.byref(cfg), 9, 1, C.byref(two)) == L.ERR_BAD_SHAPE
    la = L.MemlayerLayerArgs()
    assert lib.memlayer_layer_forward_sharded(C.byref(cfg), C.byref(la), None, L.PHASE_ALL, None, 0,
                                              None) == L.ERR_BAD_POINTER


def test_sharded_backward_needs_the_forward_statistics_for_the_balance_term():
    import types

    from model_b200.shard import ShardedBackward
    call = types.SimpleNamespace(stats=False)      # a forward run without routing statistics
    with pytest.raises(ValueError, match="stats=True"):
        ShardedBackward(call, torch.zeros(1, 4), balance_coef=0.1)


# ---------------------------------------------------------------------------
# world-size-2 gloo run of the sharded read
# ---------------------------------------------------------------------------
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir):
    import torch.distributed as dist

    from oracle import memlayer_ref as ref

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # handle exchange: every rank sees every handle in rank order
        got = exchange_handles(bytes([rank]) * L.IPC_HANDLE_BYTES)
        assert got == [bytes([r]) * L.IPC_HANDLE_BYTES for r in range(world)]

        cfg = ref.PoolConfig(n_sub_keys=16, heads=2, d_key=16, d_value=8, top_k=4)
        rng = np.random.default_rng(0)
        N, d, M = cfg.pool_size, cfg.d_value, 24
        sub_keys = rng.standard_normal((cfg.heads, 2, 16, 8)).astype(np.float32)
        values = (rng.standard_normal((N, d)) * 0.02).astype(np.float32)
        local = values[rank::world]                                    # this rank's rows
        q = np.random.default_rng(100 + rank).standard_normal((M, cfg.heads, cfg.d_key)).astype(np.float32)
        r = ref.route(cfg, q, sub_keys, float(np.log(10.0)))
        slots, weights = r["slots"].astype(np.int64), ref.softmax(r["slot_scores"]).astype(np.float32)

        # every owner sees every rank's (slot, weight) entries
        all_s = [torch.empty(M, cfg.heads, cfg.top_k, dtype=torch.int64) for _ in range(world)]
        all_w = [torch.empty(M, cfg.heads, cfg.top_k) for _ in range(world)]
        dist.all_gather(all_s, torch.from_numpy(slots))
        dist.all_gather(all_w, torch.from_numpy(weights))
        # owner side: partial row per (source rank, token) from local rows only
        part = np.zeros((world, M, d), np.float32)
        for src in range(world):
            s, w = all_s[src].numpy(), all_w[src].numpy()
            own, row = s % world, s // world
            for m in range(M):
                for h in range(cfg.heads):
                    for j in range(cfg.top_k):
                        if own[m, h, j] == rank:
                            part[src, m] += w[m, h, j] * local[row[m, h, j]]
        # token-owner side: partials from every owner, summed in rank order
        parts = [torch.empty(world, M, d) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(part))
        out = np.zeros((M, d), np.float32)
        for o in range(world):
            out += parts[o][rank].numpy()
        want = ref.gather_mix(values, slots, weights)
        np.save(os.path.join(outdir, f"err{rank}.npy"),
                np.array([np.abs(out - want).max() / np.abs(want).max()]))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_sharded_read(tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for rank in range(2):
        assert float(np.load(tmp_path / f"err{rank}.npy")[0]) <= 1e-6


# ---------------------------------------------------------------------------
# gloo runs (2 and 3 ranks) of the sharded backward's exchange: every rank sends
# its probe rows, each owner returns probe . row for its entries of every
# rank's reads in inbox order (per (source, token, owner): heads in order,
# then lanes), and the reader maps the dots back to (head, lane) as the
# routing backward does -- checked against the whole-table dots
# ---------------------------------------------------------------------------
def _inbox_order(own, o):
    """(head, lane) of each entry of owner `o` for one token, in inbox order."""
    return [(h, j) for h in range(own.shape[0]) for j in range(own.shape[1]) if own[h, j] == o]


def _bwd_worker(rank, world, port, outdir):
    import torch.distributed as dist

    from oracle import memlayer_ref as ref

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = ref.PoolConfig(n_sub_keys=16, heads=2, d_key=16, d_value=8, top_k=4)
        rng = np.random.default_rng(0)
        N, d, M, H, k = cfg.pool_size, cfg.d_value, 24, cfg.heads, cfg.top_k
        sub_keys = rng.standard_normal((H, 2, 16, 8)).astype(np.float32)
        values = rng.standard_normal((N, d))
        local = values[rank::world]
        q = np.random.default_rng(100 + rank).standard_normal((M, H, cfg.d_key)).astype(np.float32)
        read = (ref.route(cfg, q, sub_keys, float(np.log(10.0)))["slots"].astype(np.int64) + N // 2 + 1) % N
        probe = np.random.default_rng(200 + rank).standard_normal((M, d))
        # ROUTE: every owner sees every rank's reads and probe rows
        all_r = [torch.empty(M, H, k, dtype=torch.int64) for _ in range(world)]
        all_p = [torch.empty(M, d, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(all_r, torch.from_numpy(read))
        dist.all_gather(all_p, torch.from_numpy(probe))
        # GATHER: this owner's dots per (source, token), in inbox order
        dots = np.zeros((world, M, H * k))
        for src in range(world):
            rs, pr = all_r[src].numpy(), all_p[src].numpy()
            for m in range(M):
                for i, (h, j) in enumerate(_inbox_order(rs[m] % world, rank)):
                    dots[src, m, i] = pr[m] @ local[rs[m, h, j] // world]
        back = [torch.empty(world, M, H * k, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(back, torch.from_numpy(dots))
        # REDUCE: the reader finds each read's dot from its owner's list
        dw = np.zeros((M, H, k))
        for m in range(M):
            for o in range(world):
                for i, (h, j) in enumerate(_inbox_order(read[m] % world, o)):
                    dw[m, h, j] = back[o][rank, m, i].item()
        want = np.einsum("md,mhkd->mhk", probe, values[read])
        np.save(os.path.join(outdir, f"bwd{rank}.npy"), np.array([np.abs(dw - want).max() / np.abs(want).max()]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_ranks_sharded_backward_dots(world, tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_bwd_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for rank in range(world):
        assert float(np.load(tmp_path / f"bwd{rank}.npy")[0]) <= 1e-12
