"""The row-sharded forward with a staged exchange (memlayer_layer_forward_staged)
on one GPU: every rank is driven from this process and the two collectives
are emulated with torch ops (concatenation for the all-gather, a sum in rank
order for the reduce-scatter); nothing waits on anything.  Each rank must
match the single-GPU layer on its own tokens with the whole table (slots and
weights identical, outputs within 1e-5 relative for float32 tables), and
its read output must equal the peer-store exchange's bit for bit: both sum
the same partial rows in rank order."""

import pytest
import torch

from parity import OUT_RTOL_F32, OUT_RTOL_HALF, assert_rel

pytestmark = pytest.mark.gpu


def _layer(n=64, H=4, dk=64, d=64, k=16, dm=64, seed=0, vdt=torch.float32, **kw):
    from model_b200 import MemoryLayer, MemoryPool
    pool = MemoryPool(n_sub_keys=n, heads=H, d_key=dk, d_value=d, top_k=k, **kw)
    layer = MemoryLayer(pool, d_model=dm, layer=1)
    return layer, layer.init(seed, values_dtype=vdt)


def _staged(layer, params, hs, world, repeats=2, **kw):
    from model_b200 import _lib as L
    from model_b200.shard import StagedCall, shard_values
    calls = []
    for r in range(world):
        p = dict(params)
        p["pool"] = dict(params["pool"], values=shard_values(params["pool"]["values"], r, world))
        calls.append(StagedCall(layer, p, hs[r], r, world, **kw))
    for _ in range(repeats):
        for c in calls:
            c.phase(L.PHASE_ROUTE)
        mine = torch.stack([c.route[c.rank] for c in calls])          # all-gather
        for c in calls:
            c.route.copy_(mine)
        for c in calls:
            c.phase(L.PHASE_GATHER)
        for c in calls:                                               # reduce-scatter, rank order
            acc = torch.zeros_like(c.mem_in)
            for o in calls:
                acc += o.partials[c.rank]
            c.mem_in.copy_(acc)
        for c in calls:
            c.phase(L.PHASE_REDUCE)
    torch.cuda.synchronize()
    for c in calls:
        c.check()
    return [c.result() for c in calls]


def _hidden(M, dm, seed):
    g = torch.Generator("cuda").manual_seed(seed)
    return torch.randn(M, dm, device="cuda", generator=g)


@pytest.mark.parametrize("world", [1, 2, 3, 4])
def test_staged_matches_single_gpu_and_peer_store(world):
    from test_shard_gpu import _run
    layer, params = _layer()
    hs = [_hidden(300, 64, 10 + r) for r in range(world)]
    got = _staged(layer, params, hs, world)
    p2p = _run(layer, params, hs, world)
    for r, (h, (y, mem, aux)) in enumerate(zip(hs, got)):
        y0, mem0, aux0 = layer.apply(params, h, check=True)
        torch.cuda.synchronize()
        assert torch.equal(aux["slots"], aux0["slots"]), f"rank {r}: slots differ"
        assert torch.equal(aux["weights"], aux0["weights"]), f"rank {r}: weights differ"
        assert_rel(mem.cpu().numpy(), mem0.cpu().numpy(), OUT_RTOL_F32, f"rank {r} mem")
        assert_rel(y.cpu().numpy(), y0.cpu().numpy(), OUT_RTOL_F32, f"rank {r} y")
        assert torch.equal(mem, p2p[r][1]), f"rank {r}: staged and peer-store reads differ"


@pytest.mark.parametrize("vdt", [torch.bfloat16, torch.float16])
def test_staged_half_tables_shuffle_and_k32(vdt):
    layer, params = _layer(n=64, H=8, dk=64, d=32, k=32, vdt=vdt)
    hs = [_hidden(257, 64, 20 + r) for r in range(3)]
    got = _staged(layer, params, hs, 3, shuffle_reads=True)
    for r, (h, (y, mem, aux)) in enumerate(zip(hs, got)):
        y0, mem0, aux0 = layer.apply(params, h, check=True, shuffle_reads=True)
        torch.cuda.synchronize()
        assert torch.equal(aux["slots"], aux0["slots"])
        assert_rel(mem.cpu().numpy(), mem0.cpu().numpy(), OUT_RTOL_HALF, f"rank {r} mem")
        assert_rel(y.cpu().numpy(), y0.cpu().numpy(), OUT_RTOL_F32, f"rank {r} y")


def test_staged_cfg0_shapes_tensor_core_path():
    """configs[0] layer shapes (d_key 256, n 512, k 16, d 256) at 2 ranks of
    2048 tokens: the tensor-core projections and score kernel feed ROUTE."""
    layer, params = _layer(n=512, H=4, dk=256, d=256, k=16, dm=256)
    hs = [_hidden(2048, 256, 30 + r) for r in range(2)]
    got = _staged(layer, params, hs, 2, repeats=1)
    for r, (h, (y, mem, aux)) in enumerate(zip(hs, got)):
        y0, mem0, aux0 = layer.apply(params, h, check=True)
        torch.cuda.synchronize()
        assert torch.equal(aux["slots"], aux0["slots"])
        assert_rel(y.cpu().numpy(), y0.cpu().numpy(), OUT_RTOL_F32, f"rank {r} y")
