"""The C ABI library: loads, exports every declared symbol, and rejects bad
arguments on the host (these calls return before touching a GPU)."""

import ctypes as C
import glob
import os
import re

import pytest

from model_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(\w+)\s*\(", text, flags=re.M)
    return sorted(set(n for n in names if n.startswith(("memlayer_", "mlshard_"))))


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    names = declared_functions()
    assert "memlayer_pool_forward" in names and "memlayer_layer_forward" in names
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ but not exported"
    assert lib.memlayer_abi_version() == 1


def test_struct_sizes_match_header_layout():
    # int64 + 12 * 4-byte fields
    assert C.sizeof(L.MemlayerConfig) == 8 + 12 * 4
    assert C.sizeof(L.MemlayerPoolArgs) == 5 * 8 + 4 * 3 + 4 + 10 * 8  # 4 bytes of padding before `out`
    assert C.sizeof(L.MemlayerLayerArgs) == 9 * 8 + C.sizeof(L.MemlayerPoolArgs)
    assert C.sizeof(L.MemlayerRead) == 4 * 8
    assert C.sizeof(L.MemlayerAdagradArgs) == 2 * 8 + 2 * 4 + 3 * 8
    assert C.sizeof(L.MemlayerLayerGrads) == 8 + 4 + 4 + 8 + 10 * 8   # dy, coef, flag, forward ws, 10 outputs
    assert C.sizeof(L.MemlayerStagedArgs) == 5 * 8 + 2 * 4


def cfg(**kw):
    base = dict(tokens=8192, heads=4, n_sub_keys=512, d_key=256, d_value=256, top_k=16, d_model=256,
                values_dtype=L.F32, routing_noise=1.0, min_temperature=10.0, max_temperature=100.0,
                query_scale=0, balance_temperature_grad=0)
    base.update(kw)
    return L.MemlayerConfig(**base)


def ws_size(c, layer=False):
    n = C.c_size_t()
    f = L.lib().memlayer_layer_workspace_size if layer else L.lib().memlayer_pool_workspace_size
    return f(C.byref(c), C.byref(n)), n.value


def test_workspace_size_scales_with_tokens():
    st, a = ws_size(cfg(tokens=1024))
    st2, b = ws_size(cfg(tokens=2048))
    assert st == st2 == L.OK and 0 < a < b
    st, c = ws_size(cfg(tokens=1024), layer=True)
    assert st == L.OK and c > a


@pytest.mark.parametrize("bad,status", [
    (dict(d_key=7), L.ERR_BAD_SHAPE),                  # memory.py:95 d_key must be even
    (dict(top_k=513), L.ERR_BAD_SHAPE),                # memory.py:96 top_k <= n_sub_keys
    (dict(heads=0), L.ERR_BAD_SHAPE),
    (dict(tokens=-1), L.ERR_BAD_SHAPE),
    (dict(n_sub_keys=50000), L.ERR_BAD_SHAPE),         # n*n must fit int32 slot ids
    (dict(top_k=33, n_sub_keys=64), L.ERR_UNSUPPORTED),
    (dict(values_dtype=7), L.ERR_UNSUPPORTED),
    (dict(values_dtype=L.F16, d_value=12), L.ERR_UNSUPPORTED),
    (dict(min_temperature=0.0), L.ERR_BAD_SHAPE),
])
def test_bad_configs_are_rejected_on_the_host(bad, status):
    st, _ = ws_size(cfg(**bad))
    assert st == status
    a = L.MemlayerPoolArgs()
    assert L.lib().memlayer_pool_forward(C.byref(cfg(**bad)), C.byref(a), None, 0, None) == status


def test_missing_pointers_and_workspace_are_rejected():
    c = cfg(tokens=16)
    a = L.MemlayerPoolArgs()  # all NULL
    assert L.lib().memlayer_pool_forward(C.byref(c), C.byref(a), None, 0, None) == L.ERR_BAD_POINTER
    # every pointer set (never dereferenced: the workspace check fails first)
    fake = 1 << 20
    a = L.MemlayerPoolArgs(queries=fake, sub_keys=fake, log_temperature=fake, values=fake, out=fake,
                           slots=fake, weights=fake)
    assert L.lib().memlayer_pool_forward(C.byref(c), C.byref(a), None, 0, None) == L.ERR_WORKSPACE
    _, need = ws_size(c)
    assert L.lib().memlayer_pool_forward(C.byref(c), C.byref(a), fake, 1024, None) == L.ERR_WORKSPACE
    assert L.lib().memlayer_pool_forward(C.byref(c), C.byref(a), fake + 8, need, None) == L.ERR_WORKSPACE
    # training with selection noise but no Gumbel sample
    a.train = 1
    a.noise_scale = 1.0
    assert L.lib().memlayer_pool_forward(C.byref(c), C.byref(a), fake, need, None) == L.ERR_BAD_POINTER


def test_status_strings():
    for s in range(7):
        assert L.status_string(s)
    assert "unknown" in L.status_string(99)


def test_pool_mirror_keeps_reference_assertions():
    from model_b200 import MemoryPool
    with pytest.raises(AssertionError):
        MemoryPool(n_sub_keys=16, heads=2, d_key=7, d_value=12, top_k=4)
    with pytest.raises(AssertionError):
        MemoryPool(n_sub_keys=4, heads=2, d_key=8, d_value=12, top_k=5)
    pool = MemoryPool(n_sub_keys=16, heads=2, d_key=8, d_value=12, top_k=4)
    import torch
    with pytest.raises(TypeError):
        pool.apply({"params": {}}, torch.zeros(3, 2, 8))  # CPU tensor: no CPU path


def test_prepared_layer_call_refuses_an_unprepared_workspace():
    # no memlayer_layer_forward ran on this workspace: refused before any launch
    c = cfg(tokens=4)
    nb = C.c_size_t()
    assert L.lib().memlayer_layer_workspace_size(C.byref(c), C.byref(nb)) == L.OK
    la = L.MemlayerLayerArgs(h=256, w_router=256, w_gate=256, w_out=256, y=256,
                             pool=L.MemlayerPoolArgs(sub_keys=256, log_temperature=256, values=256))
    assert L.lib().memlayer_layer_forward_prepared(C.byref(c), C.byref(la), 1 << 20, nb.value,
                                                   None) == L.ERR_WORKSPACE
    assert L.lib().memlayer_layer_forward_prepared(C.byref(c), None, 1 << 20, nb.value, None) == L.ERR_BAD_POINTER


def test_layer_backward_arguments_rejected_on_the_host():
    lib = L.lib()
    c = cfg(tokens=64, d_key=64, d_value=64, d_model=64)
    nb = C.c_size_t()
    assert lib.memlayer_layer_backward_workspace_size(C.byref(c), 1, C.byref(nb)) == L.OK
    nb0 = C.c_size_t()
    assert lib.memlayer_layer_backward_workspace_size(C.byref(c), 0, C.byref(nb0)) == L.OK
    assert nb0.value < nb.value                                     # the balance term's buffers
    assert lib.memlayer_layer_backward_workspace_size(C.byref(cfg(d_key=6)), 0, C.byref(nb0)) == L.ERR_UNSUPPORTED
    la = L.MemlayerLayerArgs(h=256, w_router=256, w_gate=256, w_out=256, y=256,
                             pool=L.MemlayerPoolArgs(sub_keys=256, log_temperature=256, values=256, slots=256,
                                                     weights=256))
    g = L.MemlayerLayerGrads(dy=256, balance_coef=0.0)
    assert lib.memlayer_layer_backward(C.byref(c), None, C.byref(g), 1 << 20, nb.value, None) == L.ERR_BAD_POINTER
    assert lib.memlayer_layer_backward(C.byref(c), C.byref(la), None, 1 << 20, nb.value, None) == L.ERR_BAD_POINTER
    # the balance term needs the forward's workspace and its balance_loss output
    gb = L.MemlayerLayerGrads(dy=256, balance_coef=0.01)
    assert lib.memlayer_layer_backward(C.byref(c), C.byref(la), C.byref(gb), 1 << 20, nb.value,
                                       None) == L.ERR_BAD_POINTER
    # workspace missing, short or misaligned
    assert lib.memlayer_layer_backward(C.byref(c), C.byref(la), C.byref(g), None, nb.value, None) == L.ERR_WORKSPACE
    assert lib.memlayer_layer_backward(C.byref(c), C.byref(la), C.byref(g), 1 << 20, 64, None) == L.ERR_WORKSPACE
    assert lib.memlayer_layer_backward(C.byref(c), C.byref(la), C.byref(g), (1 << 20) + 16, nb.value,
                                       None) == L.ERR_WORKSPACE


def test_sharded_layer_backward_arguments_rejected_on_the_host():
    lib = L.lib()
    c = cfg(tokens=64, d_key=64, d_value=64, d_model=64)
    la = L.MemlayerLayerArgs(h=256, w_router=256, w_gate=256, w_out=256, y=256, mem=256,
                             pool=L.MemlayerPoolArgs(sub_keys=256, log_temperature=256, values=256, slots=256,
                                                     weights=256))
    g = L.MemlayerLayerGrads(dy=256, balance_coef=0.0)
    nb = C.c_size_t()
    assert lib.memlayer_layer_backward_workspace_size(C.byref(c), 0, C.byref(nb)) == L.OK
    # no communicator
    assert lib.memlayer_layer_backward_sharded(C.byref(c), C.byref(la), C.byref(g), None, L.PHASE_ALL, 1 << 20,
                                               nb.value, None) == L.ERR_BAD_POINTER
    # phases outside ROUTE / GATHER / REDUCE are refused before the communicator is read
    not_a_comm = C.create_string_buffer(64)
    for phases in (0, L.PHASE_ALL | L.PHASE_SPLIT, 16):
        assert lib.memlayer_layer_backward_sharded(C.byref(c), C.byref(la), C.byref(g), C.addressof(not_a_comm),
                                                   phases, 1 << 20, nb.value, None) == L.ERR_BAD_SHAPE


def test_sharded_phase_masks_that_cannot_complete_are_refused():
    """REDUCE with ROUTE but without GATHER would wait for this rank's own
    gather, which no later launch of the call runs: refused on the host,
    before the communicator is read."""
    lib = L.lib()
    c = cfg(tokens=64, d_key=64, d_value=64, d_model=64)
    not_a_comm = C.addressof(C.create_string_buffer(64))
    la = L.MemlayerLayerArgs(h=256, w_router=256, w_gate=256, w_out=256, y=256, mem=256,
                             pool=L.MemlayerPoolArgs(sub_keys=256, log_temperature=256, values=256, slots=256,
                                                     weights=256))
    g = L.MemlayerLayerGrads(dy=256, balance_coef=0.0)
    bad = L.PHASE_ROUTE | L.PHASE_REDUCE
    assert lib.memlayer_layer_backward_sharded(C.byref(c), C.byref(la), C.byref(g), not_a_comm, bad, 1 << 20,
                                               1 << 30, None) == L.ERR_BAD_SHAPE
    assert lib.memlayer_layer_forward_sharded(C.byref(c), C.byref(la), not_a_comm, bad, 1 << 20, 1 << 30,
                                              None) == L.ERR_BAD_SHAPE
    assert lib.memlayer_layer_forward_sharded(C.byref(c), C.byref(la), not_a_comm, bad | L.PHASE_SPLIT, 1 << 20,
                                              1 << 30, None) == L.ERR_BAD_SHAPE
    pa = la.pool
    assert lib.memlayer_pool_forward_sharded(C.byref(c), C.byref(pa), not_a_comm, bad, 1 << 20, 1 << 30,
                                             None) == L.ERR_BAD_SHAPE
    assert lib.memlayer_shard_comm_set_wait_budget(None, 1000000) == L.ERR_BAD_POINTER


def test_staged_exchange_arguments_rejected_on_the_host():
    lib = L.lib()
    c = cfg(tokens=64, d_key=64, d_value=64, d_model=64)
    nb = C.c_size_t()
    assert lib.memlayer_layer_workspace_size(C.byref(c), C.byref(nb)) == L.OK
    la = L.MemlayerLayerArgs(h=256, w_router=256, w_gate=256, w_out=256, y=256,
                             pool=L.MemlayerPoolArgs(sub_keys=256, log_temperature=256, values=256, slots=256,
                                                     weights=256))
    ok = dict(all_slots=256, all_weights=256, partials=256, mem=256, rank=0, world=2)
    f = lib.memlayer_layer_forward_staged

    def call(phases=L.PHASE_ROUTE, ws=1 << 20, nbytes=None, args=la, **kw):
        x = L.MemlayerStagedArgs(**dict(ok, **kw))
        return f(C.byref(c), C.byref(args) if args is not None else None, C.byref(x), phases, ws,
                 nb.value if nbytes is None else nbytes, None)

    assert call(args=None) == L.ERR_BAD_POINTER
    for phases in (0, 8, L.PHASE_ALL | L.PHASE_SPLIT):
        assert call(phases=phases) == L.ERR_BAD_SHAPE
    for rank, world in ((0, 0), (2, 2), (-1, 2), (0, 9)):
        assert call(rank=rank, world=world) == L.ERR_BAD_SHAPE
    assert call(route_stride=-1) == L.ERR_BAD_SHAPE
    assert call(route_stride=64 * 4 * 16 - 1) == L.ERR_BAD_SHAPE        # shorter than one rank's entries
    assert call(partials=256 + 8) == L.ERR_BAD_POINTER                   # misaligned
    assert call(phases=L.PHASE_GATHER, all_slots=None) == L.ERR_BAD_POINTER
    assert call(phases=L.PHASE_REDUCE, mem=None) == L.ERR_BAD_POINTER
    assert call(ws=None) == L.ERR_WORKSPACE
    assert call(nbytes=64) == L.ERR_WORKSPACE
    assert call(ws=(1 << 20) + 16) == L.ERR_WORKSPACE
