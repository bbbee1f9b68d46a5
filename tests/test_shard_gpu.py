"""Row-sharded pool on one GPU: every rank of a `world`-rank communicator is
driven from this process (emulated ranks wired to each other's buffers), one
phase at a time on one stream, so no kernel ever waits on a later launch.
Each rank's result must equal the single-GPU memory layer on the same
tokens with the whole table: slot ids and weights identical (same routing
kernels), pool output and layer output within 1e-5 relative (only the
order of the float32 sums differs)."""

import numpy as np
import pytest
import torch

from parity import OUT_RTOL_F32, assert_rel, check_slots

pytestmark = pytest.mark.gpu


def _layer(n=64, H=4, dk=64, d=64, k=16, dm=64, seed=0, vdt=torch.float32, **kw):
    from model_b200 import MemoryLayer, MemoryPool
    pool = MemoryPool(n_sub_keys=n, heads=H, d_key=dk, d_value=d, top_k=k, **kw)
    layer = MemoryLayer(pool, d_model=dm, layer=1)
    return layer, layer.init(seed, values_dtype=vdt)


def _run(layer, params, hs, world, repeats=2, split=False, **kw):
    from model_b200 import _lib as L
    from model_b200.shard import ShardedCall, emulated_comms, shard_values
    cap = max(1, max(h.shape[0] for h in hs))
    cfg = layer.pool.config(cap, params["pool"]["values"].dtype, layer.d_model)
    comms = emulated_comms(cfg, world)
    calls = []
    for r in range(world):
        p = dict(params)
        p["pool"] = dict(params["pool"], values=shard_values(params["pool"]["values"], r, world))
        calls.append(ShardedCall(layer, comms[r], p, hs[r], **kw))
    for _ in range(repeats):           # later calls reuse the buffers with a new epoch
        for ph in (L.PHASE_ROUTE, L.PHASE_GATHER, L.PHASE_REDUCE):
            for c in calls:
                c.run(ph | (L.PHASE_SPLIT if split else 0))
    torch.cuda.synchronize()
    for c in calls:
        c.check()
    res = [tuple(t.clone() if isinstance(t, torch.Tensor) else t for t in c.result()[:2]) + (c.result()[2],)
           for c in calls]
    for c in comms:
        c.close()
    return res


def _hidden(M, dm, seed):
    g = torch.Generator("cuda").manual_seed(seed)
    return torch.randn(M, dm, device="cuda", generator=g)


def _compare(layer, params, hs, got, **kw):
    for r, (h, (y, mem, aux)) in enumerate(zip(hs, got)):
        y0, mem0, aux0 = layer.apply(params, h, check=True, **kw)
        torch.cuda.synchronize()
        assert torch.equal(aux["slots"], aux0["slots"]), f"rank {r}: slots differ"
        assert torch.equal(aux["weights"], aux0["weights"]), f"rank {r}: weights differ"
        if h.shape[0]:
            assert_rel(mem.cpu().numpy(), mem0.cpu().numpy(), OUT_RTOL_F32, f"rank {r} mem")
            assert_rel(y.cpu().numpy(), y0.cpu().numpy(), OUT_RTOL_F32, f"rank {r} y")


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_sharded_matches_single_gpu(world):
    layer, params = _layer()
    hs = [_hidden(300, 64, 10 + r) for r in range(world)]
    _compare(layer, params, hs, _run(layer, params, hs, world))


@pytest.mark.parametrize("vdt", [torch.bfloat16, torch.float16])
def test_sharded_half_tables(vdt):
    layer, params = _layer(vdt=vdt, d=128)
    hs = [_hidden(257, 64, 30 + r) for r in range(4)]
    _compare(layer, params, hs, _run(layer, params, hs, 4))


def test_sharded_ragged_and_empty_ranks():
    """Ranks with different token counts, one with none."""
    layer, params = _layer()
    hs = [_hidden(m, 64, 50 + r) for r, m in enumerate((300, 0, 129, 7))]
    _compare(layer, params, hs, _run(layer, params, hs, 4))


def test_sharded_shuffle_reads_and_k32():
    layer, params = _layer(n=128, H=8, dk=128, d=64, k=32)
    hs = [_hidden(200, 64, 70 + r) for r in range(2)]
    _compare(layer, params, hs, _run(layer, params, hs, 2, shuffle_reads=True), shuffle_reads=True)


def test_sharded_cfg0_shapes_against_oracle():
    """configs[0] shapes on 4 emulated ranks, 1024 tokens each; rank 0's pool
    output against the CPU oracle on the full table."""
    from oracle import memlayer_ref as ref
    layer, params = _layer(n=512, H=4, dk=256, d=256, k=16, dm=256, seed=3)
    hs = [_hidden(1024, 256, 90 + r) for r in range(4)]
    got = _run(layer, params, hs, 4)
    _compare(layer, params, hs, got)
    P = layer.pool
    cfg = ref.PoolConfig(n_sub_keys=P.n_sub_keys, heads=P.heads, d_key=P.d_key, d_value=P.d_value, top_k=P.top_k)
    h = hs[0][:64].cpu().numpy()
    q = ref.dense(h, params["router_1"]["kernel"].cpu().numpy(), params["router_1"]["bias"].cpu().numpy())
    out, aux = ref.pool_forward(cfg, q.reshape(64, P.heads, P.d_key), params["pool"]["sub_keys"].cpu().numpy(),
                                float(params["pool"]["log_temperature"]), params["pool"]["values"].cpu().numpy(),
                                with_stats=False)
    r = ref.route(cfg, q.reshape(64, P.heads, P.d_key), params["pool"]["sub_keys"].cpu().numpy(),
                  float(params["pool"]["log_temperature"]))
    check_slots(got[0][2]["slots"][:64].cpu().numpy(), aux["slots"], r["scores"], P.n_sub_keys)
    assert_rel(got[0][1][:64].cpu().numpy(), out, OUT_RTOL_F32, "mem vs oracle")


@pytest.mark.parametrize("world", [2, 8])
def test_sharded_split_halves(world):
    """MEMLAYER_PHASE_SPLIT: the exchange in two token halves (phase by
    phase here: both halves' pushes, both gathers, both reduces)."""
    layer, params = _layer()
    hs = [_hidden(m, 64, 110 + r) for r, m in enumerate([301, 0, 1, 129, 300, 7, 64, 2][:world])]
    _compare(layer, params, hs, _run(layer, params, hs, world, split=True))
