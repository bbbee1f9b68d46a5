"""The value table in page-locked host memory (memory.py:180-183 with
host_pool.fetch, host_pool.py:206-220): MemoryPool(host_pool=name) reads
through memlayer_pool_forward_host_table, which must give exactly the
outputs, slots, weights and statistics of the device-table forward on the
same rows (the mix runs in the same order), and match the oracle."""

import ctypes as C

import numpy as np
import pytest
import torch

from model_b200 import MemoryPool
from model_b200 import _lib as L
from model_b200.host_table import HostTable
from oracle import memlayer_ref as ref

pytestmark = pytest.mark.gpu


def _pair(n_sub, H, dk, d, k, dtype, seed=0):
    host_pool = MemoryPool(n_sub_keys=n_sub, heads=H, d_key=dk, d_value=d, top_k=k)
    params = host_pool.init(seed, values_dtype=dtype)
    table = HostTable(n_sub * n_sub, d, dtype=dtype, seed=seed)
    table.values.copy_(params["params"]["values"].cpu())
    pool_h = MemoryPool(n_sub_keys=n_sub, heads=H, d_key=dk, d_value=d, top_k=k, host_pool=table.name)
    return host_pool, pool_h, params, table


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("shuffle", [False, True])
@pytest.mark.parametrize("M", [5, 128, 300])   # 160 / 4096 fetches: one-CTA dedup; 9600: radix sort
def test_host_table_matches_device_table(dtype, shuffle, M):
    pool_d, pool_h, params, table = _pair(64, 4, 64, 64, 8, dtype)
    q = torch.randn(M, 4, 64, device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    out_d, aux_d = pool_d.apply(params, q, shuffle_reads=shuffle, check=True)
    pv = {k: v for k, v in params["params"].items() if k != "values"}   # no values param with a host pool
    out_h, aux_h = pool_h.apply({"params": pv}, q, shuffle_reads=shuffle, check=True)
    torch.cuda.synchronize()
    assert torch.equal(out_d, out_h)
    for key in ("slots", "weights", "slot_counts", "subkey_counts", "balance_loss", "top1_weight"):
        assert torch.equal(aux_d[key], aux_h[key]), key
    table.close()


def test_host_table_against_oracle_and_ragged_shapes():
    pool_d, pool_h, params, table = _pair(48, 2, 32, 40, 16, torch.float32, seed=3)
    for M in (1, 7, 129):
        q = torch.randn(M, 2, 32, device="cuda", generator=torch.Generator("cuda").manual_seed(M))
        pv = {k: v for k, v in params["params"].items() if k != "values"}
        out, aux = pool_h.apply({"params": pv}, q, check=True)
        cfg = ref.PoolConfig(n_sub_keys=48, heads=2, d_key=32, d_value=40, top_k=16)
        want = ref.gather_mix(table.values.numpy(), aux["slots"].cpu().numpy().astype(np.int64),
                              aux["weights"].cpu().numpy())
        np.testing.assert_allclose(out.cpu().numpy(), want, rtol=1e-5, atol=1e-6 * np.abs(want).max())
    table.close()


def test_host_table_rejects_pageable_memory():
    pool = MemoryPool(n_sub_keys=16, heads=2, d_key=16, d_value=8, top_k=4)
    cfg = pool.config(4, torch.float32)
    pageable = np.zeros((256, 8), np.float32)       # not page-locked: the GPU cannot read it
    q = torch.zeros(4, 2, 16, device="cuda")
    sk = torch.zeros(2, 2, 16, 8, device="cuda")
    lt = torch.zeros(1, device="cuda")
    out = torch.empty(4, 8, device="cuda")
    sl = torch.empty(4, 2, 4, dtype=torch.int32, device="cuda")
    w = torch.empty(4, 2, 4, device="cuda")
    a = L.MemlayerPoolArgs(queries=q.data_ptr(), sub_keys=sk.data_ptr(), log_temperature=lt.data_ptr(),
                           values=pageable.ctypes.data, out=out.data_ptr(), slots=sl.data_ptr(), weights=w.data_ptr())
    nb = C.c_size_t()
    assert L.lib().memlayer_host_table_workspace_size(C.byref(cfg), C.byref(nb)) == L.OK
    ws = torch.empty(nb.value, dtype=torch.uint8, device="cuda")
    assert L.lib().memlayer_pool_forward_host_table(C.byref(cfg), C.byref(a), ws.data_ptr(), nb.value,
                                                    None) == L.ERR_BAD_POINTER


def test_host_table_loads_reference_snapshot(tmp_path):
    rng = np.random.default_rng(0)
    vals = rng.standard_normal((256, 8)).astype(np.float16)
    np.save(tmp_path / "values.npy", vals)
    t = HostTable(256, 8, path=str(tmp_path), dtype=torch.float16)
    assert t.values.is_pinned() and np.array_equal(t.values.numpy(), vals)
    t.save(str(tmp_path / "snap"))
    assert np.array_equal(np.load(tmp_path / "snap" / "values.npy"), vals)
    t.close()
