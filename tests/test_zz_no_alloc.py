"""memlayer_pool_forward_noalloc: the MemoryPool forward for callers that
cannot allocate or pass a device workspace (its workspace is a fixed array
inside the library).  Checked through the C ABI against the regular entry
point, which gets a caller-allocated workspace, on two calls in a row.

This file is collected last on purpose: the entry point's first call on a
device sets up the array's address, and the test must pass both alone in a
fresh process and after every other test."""

import ctypes as C

import numpy as np
import pytest
import torch

from model_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _cfg(M):
    return L.MemlayerConfig(tokens=M, heads=4, n_sub_keys=256, d_key=128, d_value=64, top_k=16, d_model=0,
                            values_dtype=L.F32, routing_noise=1.0, min_temperature=10.0, max_temperature=100.0,
                            query_scale=0, balance_temperature_grad=0)


def _run(entry, cfg, q, sk, lt, vals, ws=None):
    M = cfg.tokens
    out = torch.empty(M, 64, device="cuda")
    slots = torch.empty(M, 4, 16, dtype=torch.int32, device="cuda")
    weights = torch.empty(M, 4, 16, device="cuda")
    top1 = torch.empty(1, device="cuda")
    a = L.MemlayerPoolArgs(queries=q.data_ptr(), sub_keys=sk.data_ptr(), log_temperature=lt.data_ptr(),
                           values=vals.data_ptr(), out=out.data_ptr(), slots=slots.data_ptr(),
                           weights=weights.data_ptr(), top1_weight=top1.data_ptr())
    s = torch.cuda.current_stream().cuda_stream
    lib = L.lib()
    if entry == "noalloc":
        f = lib.memlayer_pool_forward_noalloc
        f.restype = C.c_int32
        f.argtypes = [C.POINTER(L.MemlayerConfig), C.POINTER(L.MemlayerPoolArgs), C.c_void_p]
        L.check(f(C.byref(cfg), C.byref(a), s), "memlayer_pool_forward_noalloc")
    else:
        L.check(lib.memlayer_pool_forward(C.byref(cfg), C.byref(a), ws.data_ptr(), ws.numel(), s),
                "memlayer_pool_forward")
    torch.cuda.synchronize()
    return out.cpu().numpy(), slots.cpu().numpy(), weights.cpu().numpy(), float(top1.cpu())


def test_noalloc_matches_workspace_entry_twice():
    g = torch.Generator(device="cuda").manual_seed(5)
    sk = torch.randn(4, 2, 256, 64, device="cuda", generator=g)
    lt = torch.full((1,), float(np.log(10.0)), device="cuda")
    vals = torch.randn(256 * 256, 64, device="cuda", generator=g) * 0.02
    lib = L.lib()
    for M in (300, 129):   # two calls in a row, different sizes: the array keeps stale contents
        cfg = _cfg(M)
        q = torch.randn(M, 4, 128, device="cuda", generator=g)
        nbytes = C.c_size_t()
        L.check(lib.memlayer_pool_workspace_size(C.byref(cfg), C.byref(nbytes)), "workspace_size")
        assert nbytes.value <= 64 << 20
        ws = torch.empty(nbytes.value, dtype=torch.uint8, device="cuda")
        ref = _run("ws", cfg, q, sk, lt, vals, ws)
        got = _run("noalloc", cfg, q, sk, lt, vals)
        np.testing.assert_array_equal(got[1], ref[1])                       # slot ids
        np.testing.assert_allclose(got[2], ref[2], rtol=1e-5, atol=0)        # weights
        np.testing.assert_allclose(got[0], ref[0], rtol=1e-5, atol=1e-7)     # pool output
        assert abs(got[3] - ref[3]) <= 1e-6


def test_noalloc_rejects_too_large():
    cfg = _cfg(1 << 20)   # a million tokens needs far more than the 64 MiB array
    a = L.MemlayerPoolArgs()
    f = L.lib().memlayer_pool_forward_noalloc
    f.restype = C.c_int32
    f.argtypes = [C.POINTER(L.MemlayerConfig), C.POINTER(L.MemlayerPoolArgs), C.c_void_p]
    assert f(C.byref(cfg), C.byref(a), None) == L.ERR_WORKSPACE
