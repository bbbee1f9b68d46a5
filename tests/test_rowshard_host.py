"""Host side of the owner-sharded row update (train.py:175-206 replaced by
pushes to the row owners), on CPU: the oracle's data-parallel merge, the C
ABI's argument checks (no CUDA call is reached), and a world-size-2 gloo run
of the owner decomposition -- every rank merges its own fetches, sends each
merged row to the rank that owns it, the owner sums the rows in source-rank
order, the clip uses the sum of every owner's squared norm -- checked
against the oracle's replicated update."""

import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch

from model_b200 import _lib as L
from oracle import memlayer_ref as ref


def _reads(rng, M, H, k, d, N):
    s = rng.integers(0, N, (M, H, k))
    w = rng.random((M, H, k)).astype(np.float32)
    g = rng.standard_normal((M, d)).astype(np.float32)
    return s, w, g


def test_dp_merge_equals_single_device_merge():
    rng = np.random.default_rng(0)
    N, H, k, d = 256, 2, 4, 8
    per = [_reads(rng, M, H, k, d, N) for M in (13, 0, 40)]
    u, r = ref.fetched_row_grads_sharded(per, N)
    s_all = np.concatenate([p[0] for p in per])
    w_all = np.concatenate([p[1] for p in per])
    g_all = np.concatenate([p[2] for p in per])
    u1, r1 = ref.fetched_row_grads(s_all, w_all, g_all, N)
    np.testing.assert_array_equal(u, u1)
    np.testing.assert_allclose(r, r1, rtol=1e-5, atol=1e-6)
    # one device: exactly the single-device merge
    u2, r2 = ref.fetched_row_grads_sharded(per[2:], N)
    u3, r3 = ref.fetched_row_grads(*per[2], N)
    np.testing.assert_array_equal(u2, u3)
    np.testing.assert_array_equal(r2, r3)


def _cfg(**kw):
    base = dict(tokens=64, heads=2, n_sub_keys=16, d_key=16, d_value=8, top_k=4, d_model=16,
                values_dtype=L.F32, routing_noise=0.0, min_temperature=10.0, max_temperature=100.0)
    base.update(kw)
    return L.MemlayerConfig(**base)


def test_rowgrad_comm_and_entry_checks():
    lib = L.lib()
    h = C.c_void_p()
    for n_reads, rank, world in ((0, 0, 2), (9, 0, 2), (1, 2, 2), (1, 0, 9), (1, -1, 2)):
        assert lib.memlayer_shard_comm_create_rowgrad(C.byref(_cfg()), n_reads, rank, world,
                                                      C.byref(h)) == L.ERR_BAD_SHAPE
        assert not h.value
    assert lib.memlayer_shard_comm_create_rowgrad(C.byref(_cfg(values_dtype=L.F16)), 1, 0, 2,
                                                  C.byref(h)) == L.ERR_UNSUPPORTED
    assert lib.memlayer_shard_comm_create_rowgrad(C.byref(_cfg(d_value=6)), 1, 0, 2, C.byref(h)) == L.ERR_UNSUPPORTED
    assert lib.memlayer_shard_comm_create_rowgrad(C.byref(_cfg()), 1, 0, 2, None) == L.ERR_BAD_POINTER
    nb = C.c_size_t()
    assert lib.memlayer_shard_rowgrad_workspace_size(None, 10, C.byref(nb)) == L.ERR_BAD_POINTER
    a = L.MemlayerAdagradArgs()
    assert lib.memlayer_row_adagrad_sharded(C.byref(_cfg()), None, 1, C.byref(a), None, L.PHASE_ALL, None, 0,
                                            None) == L.ERR_BAD_POINTER


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        N, H, k, d, lr, clip, rest = 256, 2, 4, 8, 0.05, 1.0, 0.3
        rng = np.random.default_rng(0)                     # same table on every rank
        values = rng.standard_normal((N, d)).astype(np.float32)
        acc = rng.random(N).astype(np.float32)
        per = [_reads(np.random.default_rng(10 + r), M, H, k, d, N) for r, M in enumerate((30, 17))]
        # ROUTE: local merge, each merged row to its owner (all_gather stands in for the peer stores)
        u, rows = ref.fetched_row_grads(*per[rank], N)
        lists_u = [None] * world
        lists_r = [None] * world
        dist.all_gather_object(lists_u, u)
        dist.all_gather_object(lists_r, rows)
        # GATHER: the owner's rows, contributions summed in source-rank order
        mine = {}
        for src in range(world):
            for s, row in zip(lists_u[src], lists_r[src]):
                if s % world == rank:
                    mine[s] = mine[s] + row if s in mine else row.astype(np.float32).copy()
        own_u = np.array(sorted(mine), np.int64)
        own_r = np.stack([mine[s] for s in own_u]) if len(own_u) else np.zeros((0, d), np.float32)
        sq = torch.tensor([float(np.sum(own_r.astype(np.float64) ** 2))], dtype=torch.float64)
        sqs = [torch.empty(1, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(sqs, sq)
        # REDUCE: global norm from the owners' partials in rank order, update the owned rows
        gn = np.sqrt(sum(float(x) for x in sqs) + rest)
        scale = np.float32(min(1.0, clip / (gn + 1e-6)))
        local_v, local_a = values[rank::world].copy(), acc[rank::world].copy()
        ref.rowwise_adagrad(local_v, local_a, own_u // world, own_r * scale, lr)
        # the reference: replicated merge + update of the whole table
        ru, rr = ref.fetched_row_grads_sharded(per, N)
        want_scale = ref.clip_scale(rest, rr, clip)
        wv, wa = values.copy(), acc.copy()
        ref.rowwise_adagrad(wv, wa, ru, rr * want_scale, lr)
        ev = np.abs(local_v - wv[rank::world]).max() / np.abs(wv).max()
        ea = np.abs(local_a - wa[rank::world]).max() / np.abs(wa).max()
        np.save(os.path.join(outdir, f"r{rank}.npy"), np.array([ev, ea, abs(float(scale) - float(want_scale))]))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_owner_sharded_update(tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for rank in range(2):
        ev, ea, es = np.load(tmp_path / f"r{rank}.npy")
        assert ev <= 1e-6 and ea <= 1e-6 and es <= 1e-7
