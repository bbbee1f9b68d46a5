"""Backward of the row-sharded memory layer on one GPU (emulated ranks wired
to each other's buffers, one phase at a time on one stream, so no kernel
waits on a later launch).  Each rank's gradients must equal the single-GPU
backward (memlayer_layer_backward) on the same tokens with the whole table:
the per-read dots are computed in the same order (so the routing gradient
is the same), and only the read output, summed over owners in rank order
in the forward, differs in rounding -- every gradient within 1e-5 of its
largest entry.  The single-GPU backward itself is pinned to the oracle
elsewhere."""

import pytest
import torch

from model_b200 import _lib as L

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _layer(n=64, H=4, dk=64, d=64, k=16, dm=64, seed=0, vdt=torch.float32, **kw):
    from model_b200 import MemoryLayer, MemoryPool
    pool = MemoryPool(n_sub_keys=n, heads=H, d_key=dk, d_value=d, top_k=k, min_temperature=5.0, **kw)
    layer = MemoryLayer(pool, d_model=dm, layer=1)
    params = layer.init(seed, values_dtype=vdt)
    with torch.no_grad():
        for name in ("router_1", "mem_gate_1", "mem_out_1"):
            params[name]["bias"].normal_(0.0, 0.1, generator=torch.Generator("cuda").manual_seed(seed))
    return layer, params


def _rand(shape, seed):
    return torch.randn(*shape, device="cuda", generator=torch.Generator("cuda").manual_seed(seed))


def _flat(g):
    return {"h": g["h"], "w_router": g["router_1"]["kernel"], "b_router": g["router_1"]["bias"],
            "sub_keys": g["pool"]["sub_keys"], "log_temperature": g["pool"]["log_temperature"],
            "w_gate": g["mem_gate_1"]["kernel"], "b_gate": g["mem_gate_1"]["bias"],
            "w_out": g["mem_out_1"]["kernel"], "b_out": g["mem_out_1"]["bias"], "probe": g["probe"]}


def _run(layer, params, hs, dys, world, bal, steps=2, rtp=False, **kw):
    """`steps` forward + backward rounds on the same communicators; the
    gradients of the last one, per rank."""
    from model_b200.shard import ShardedBackward, ShardedCall, emulated_comms, shard_values
    cap = max(1, max(h.shape[0] for h in hs))
    cfg = layer.pool.config(cap, params["pool"]["values"].dtype, layer.d_model)
    comms = emulated_comms(cfg, world)
    out = []
    try:
        for _ in range(steps):
            calls = []
            for r in range(world):
                p = dict(params)
                p["pool"] = dict(params["pool"], values=shard_values(params["pool"]["values"], r, world))
                calls.append(ShardedCall(layer, comms[r], p, hs[r], stats=True, **kw))
            for ph in (L.PHASE_ROUTE, L.PHASE_GATHER, L.PHASE_REDUCE):
                for c in calls:
                    c.run(ph)
            bws = [ShardedBackward(c, dy, balance_coef=bal, route_through_pool=rtp) for c, dy in zip(calls, dys)]
            for ph in (L.PHASE_ROUTE, L.PHASE_GATHER, L.PHASE_REDUCE):
                for b in bws:
                    b.run(ph)
            torch.cuda.synchronize()
            for c, b in zip(calls, bws):
                c.check()
                b.check()
        out = [({k: v.clone() for k, v in _flat(b.result()).items()}, c.result()[2]) for c, b in zip(calls, bws)]
    finally:
        torch.cuda.synchronize()
        for c in comms:
            c.close()
    return out


def _compare(layer, params, hs, dys, got, bal, rtp=False, **kw):
    for r, (h, dy, (g, aux)) in enumerate(zip(hs, dys, got)):
        y0, mem0, aux0, ctx = layer.apply_train(params, h, train=False, check=True, **kw)
        want = _flat(layer.backward(ctx, dy, balance_coef=bal, route_through_pool=rtp, check=True))
        torch.cuda.synchronize()
        assert torch.equal(aux["slots"], aux0["slots"]), f"rank {r}: slots differ"
        for name, w in want.items():
            a = g[name]
            assert a.shape == w.shape, name
            if w.numel() == 0:
                continue
            scale = w.abs().max().clamp_min(1e-12)
            err = ((a - w).abs().max() / scale).item()
            assert err <= TOL, f"rank {r} {name}: {err:.2e} of max |grad| {scale.item():.3e}"


@pytest.mark.parametrize("world", [1, 2, 3, 4])
@pytest.mark.parametrize("bal", [0.0, 0.5])
def test_sharded_backward_matches_single_gpu(world, bal):
    layer, params = _layer(seed=world)
    hs = [_rand((150 + 37 * r, 64), 10 * world + r) for r in range(world)]
    dys = [_rand((h.shape[0], 64), 100 + 10 * world + r) for r, h in enumerate(hs)]
    got = _run(layer, params, hs, dys, world, bal)
    _compare(layer, params, hs, dys, got, bal)


def test_sharded_backward_half_table_shuffle_and_empty_rank():
    layer, params = _layer(n=48, H=2, dk=32, d=96, k=8, dm=40, seed=7, vdt=torch.bfloat16, query_scale=True)
    hs = [_rand((90, 40), 1), _rand((0, 40), 2), _rand((133, 40), 3)]
    dys = [_rand((h.shape[0], 40), 10 + r) for r, h in enumerate(hs)]
    got = _run(layer, params, hs, dys, 3, 0.3, rtp=True, shuffle_reads=True)
    _compare(layer, params, hs, dys, got, 0.3, rtp=True, shuffle_reads=True)


def test_sharded_backward_once_per_forward():
    from model_b200.shard import ShardedBackward, ShardedCall, emulated_comms
    layer, params = _layer(seed=3)
    h, dy = _rand((20, 64), 4), _rand((20, 64), 5)
    cfg = layer.pool.config(20, params["pool"]["values"].dtype, layer.d_model)
    (comm,) = emulated_comms(cfg, 1)
    try:
        call = ShardedCall(layer, comm, params, h, stats=True)
        first = ShardedBackward(call, dy)
        with pytest.raises(L.MemlayerError):   # no forward has run on the communicator yet
            first.run(L.PHASE_ROUTE)
        call.run(L.PHASE_ALL)
        first.run(L.PHASE_ALL)
        with pytest.raises(L.MemlayerError):   # the inbox of that forward has served its backward
            ShardedBackward(call, dy).run(L.PHASE_ROUTE)
        torch.cuda.synchronize()
        first.check()
    finally:
        torch.cuda.synchronize()
        comm.close()
