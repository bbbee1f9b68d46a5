"""The bounded waits of the row-sharded path, made to run out on one GPU.

A rank that never arrives is emulated by wiring two communicators to each
other in this process and running only rank 0's phases: rank 1 launches
nothing, so every flag rank 0 waits on stays unset.  With the wait budget
cut to 1 ms (memlayer_shard_comm_set_wait_budget), rank 0's waits give up,
record their code in the call's status word (31: inbox of the forward, 33:
row-update inbox, 35: probe rows of the backward), later waits of the call
give up at once, and the call returns promptly.  No kernel waits on a later
launch; nothing faults.  Afterwards the GPU is checked to be usable: a
complete sharded call on fresh communicators must match the single-GPU
layer."""

import re
import time

import numpy as np
import pytest
import torch

from model_b200 import _lib as L

pytestmark = pytest.mark.gpu

BUDGET_S = 1e-3


def _layer(n=64, H=4, dk=64, d=64, k=16, dm=64):
    from model_b200 import MemoryLayer, MemoryPool
    layer = MemoryLayer(MemoryPool(n_sub_keys=n, heads=H, d_key=dk, d_value=d, top_k=k), d_model=dm, layer=1)
    return layer, layer.init(0)


def _local(params, r, world):
    from model_b200.shard import shard_values
    return dict(params, pool=dict(params["pool"], values=shard_values(params["pool"]["values"], r, world)))


def _status(exc):
    m = re.search(r"device status (\d+)", str(exc))
    return int(m.group(1)) if m else None


def _healthy_after():
    """A complete two-rank call on fresh communicators still matches the single-GPU layer."""
    from test_shard_gpu import _run
    layer, params = _layer()
    hs = [torch.randn(100, 64, device="cuda", generator=torch.Generator("cuda").manual_seed(7 + r))
          for r in range(2)]
    got = _run(layer, params, hs, 2, repeats=1)
    for h, (y, mem, aux) in zip(hs, got):
        y0, mem0, aux0 = layer.apply(params, h, check=True)
        torch.cuda.synchronize()
        assert torch.equal(aux["slots"], aux0["slots"])
        np.testing.assert_allclose(y.cpu().numpy(), y0.cpu().numpy(), rtol=0, atol=1e-5 * float(y0.abs().max()))


def test_wait_budget_is_checked_on_the_host():
    from model_b200.shard import emulated_comms
    layer, params = _layer()
    comms = emulated_comms(layer.pool.config(16, torch.float32, 64), 2)
    try:
        for bad in (0.0, 1e-7, 61.0):
            with pytest.raises(L.MemlayerError):
                comms[0].set_wait_budget(bad)
        comms[0].set_wait_budget(0.5)
    finally:
        for c in comms:
            c.close()


def test_forward_wait_on_a_rank_that_never_routes():
    from model_b200.shard import ShardedCall, emulated_comms
    layer, params = _layer()
    h = torch.randn(200, 64, device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    comms = emulated_comms(layer.pool.config(200, torch.float32, 64), 2)
    try:
        for c in comms:
            c.set_wait_budget(BUDGET_S)
        call = ShardedCall(layer, comms[0], _local(params, 0, 2), h)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for ph in (L.PHASE_ROUTE, L.PHASE_GATHER, L.PHASE_REDUCE):
            call.run(ph)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        with pytest.raises(L.DeviceError) as e:
            call.check()
        assert _status(e.value) == 31, str(e.value)      # the gather's wait on rank 1's inbox gave up first
        assert elapsed < 0.5, f"the call took {elapsed:.3f} s with a 1 ms wait budget"
    finally:
        torch.cuda.synchronize()
        for c in comms:
            c.close()
    _healthy_after()


def test_row_update_wait_on_a_rank_that_never_pushes():
    from model_b200.shard import emulated_comms
    from model_b200.sparse import ShardedRowUpdate
    n_sub, H, k, d, M = 32, 4, 8, 64, 50
    N = n_sub * n_sub
    rng = np.random.default_rng(3)
    cfg = L.MemlayerConfig(tokens=M, heads=H, n_sub_keys=n_sub, d_key=16, d_value=d, top_k=k, d_model=16,
                           values_dtype=L.F32, routing_noise=0.0, min_temperature=1.0, max_temperature=1.0)
    comms = emulated_comms(cfg, 2, n_reads=1)
    try:
        for c in comms:
            c.set_wait_budget(BUDGET_S)
        values = torch.from_numpy(rng.standard_normal((N, d)).astype(np.float32)[0::2].copy()).cuda()
        acc = torch.zeros(values.shape[0], device="cuda")
        aux = {"slots": [torch.from_numpy(rng.integers(0, N, (M, H, k)).astype(np.int32)).cuda()],
               "weights": [torch.from_numpy(rng.random((M, H, k)).astype(np.float32)).cuda()]}
        up = ShardedRowUpdate(comms[0], values, acc, aux, {0: torch.randn(M, d, device="cuda")}, [0], lr=0.01,
                              grad_clip=1.0)
        before = values.clone()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for ph in (L.PHASE_ROUTE, L.PHASE_GATHER, L.PHASE_REDUCE):
            up.run(ph)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        with pytest.raises(L.DeviceError) as e:
            up.check()
        assert _status(e.value) == 33, str(e.value)
        assert elapsed < 0.5, f"the call took {elapsed:.3f} s with a 1 ms wait budget"
        assert torch.equal(values, before), "a failed step must not update rows"
    finally:
        torch.cuda.synchronize()
        for c in comms:
            c.close()
    _healthy_after()


def test_backward_wait_on_a_rank_that_never_publishes_its_probe():
    from model_b200.shard import ShardedBackward, ShardedCall, emulated_comms
    layer, params = _layer()
    hs = [torch.randn(120, 64, device="cuda", generator=torch.Generator("cuda").manual_seed(11 + r))
          for r in range(2)]
    comms = emulated_comms(layer.pool.config(120, torch.float32, 64), 2)
    try:
        calls = [ShardedCall(layer, comms[r], _local(params, r, 2), hs[r], stats=True) for r in range(2)]
        for ph in (L.PHASE_ROUTE, L.PHASE_GATHER, L.PHASE_REDUCE):    # a complete forward on both ranks
            for c in calls:
                c.run(ph)
        torch.cuda.synchronize()
        for c in calls:
            c.check()
        for c in comms:
            c.set_wait_budget(BUDGET_S)
        bw = ShardedBackward(calls[0], torch.randn(120, 64, device="cuda"))
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for ph in (L.PHASE_ROUTE, L.PHASE_GATHER, L.PHASE_REDUCE):    # rank 1 never starts its backward
            bw.run(ph)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        with pytest.raises(L.DeviceError) as e:
            bw.check()
        assert _status(e.value) == 35, str(e.value)
        assert elapsed < 0.5, f"the call took {elapsed:.3f} s with a 1 ms wait budget"
    finally:
        torch.cuda.synchronize()
        for c in comms:
            c.close()
    _healthy_after()
