"""The JAX binding (model_b200/jax_ffi): XLA FFI handlers over the C ABI.

JAX is not installed in this image, so the handlers are neither compiled nor
run here; these checks keep the binding consistent with the C ABI: every
handler is registered under its target name, each handler's bound argument /
result / attribute counts match its C++ parameters, every attribute name is
passed by the Python wrappers, every C ABI function the handlers call is
declared in include/memlayer.h and exported by the library, and without JAX
the build skips the handlers and the registration fails loudly."""

import os
import re

import pytest

from model_b200 import _lib as L
from model_b200 import jax_ffi

SRC = open(jax_ffi.SRC).read()
PY = open(os.path.join(os.path.dirname(jax_ffi.SRC), "__init__.py")).read()


def _handlers():
    """{symbol: (function name, bind chain)} of every XLA_FFI_DEFINE_HANDLER_SYMBOL."""
    out = {}
    for m in re.finditer(r"XLA_FFI_DEFINE_HANDLER_SYMBOL\((\w+),\s*(\w+),(.*?)\);\n", SRC, flags=re.S):
        out[m.group(1)] = (m.group(2), m.group(3))
    return out


def _params(fn):
    m = re.search(r"static ffi::Error " + fn + r"\((.*?)\)\s*\{", SRC, flags=re.S)
    assert m, fn
    params, depth, cur = [], 0, ""
    for ch in m.group(1):
        if ch == "<":
            depth += 1
        elif ch == ">":
            depth -= 1
        if ch == "," and depth == 0:
            params.append(cur.strip())
            cur = ""
        else:
            cur += ch
    params.append(cur.strip())
    return params


def test_every_handler_is_registered():
    hs = _handlers()
    assert set(hs) == set(jax_ffi.HANDLERS) == set(jax_ffi.TARGETS)
    for target in jax_ffi.TARGETS.values():
        assert f'"{target}"' in PY, f"{target} is never called from Python"


@pytest.mark.parametrize("sym", ["MemlayerPoolForward", "MemlayerLayerForward", "MemlayerLayerBackward"])
def test_bindings_match_the_handler_parameters(sym):
    fn, chain = _handlers()[sym]
    ps = _params(fn)
    ctx = [p for p in ps if p.startswith(("cudaStream_t", "ffi::ScratchAllocator"))]
    args = [p for p in ps if p.startswith(("ffi::Buffer", "ffi::AnyBuffer"))]
    rets = [p for p in ps if p.startswith("ffi::Result")]
    attrs = [p for p in ps if p not in ctx + args + rets]
    assert len(ctx) == chain.count(".Ctx<")
    assert len(args) == chain.count(".Arg<")
    assert len(rets) == chain.count(".Ret<")
    names = re.findall(r'\.Attr<[\w:]+>\("(\w+)"\)', chain)
    assert len(attrs) == len(names)
    for n in names:                       # every attribute is passed by a wrapper (or by _attrs)
        assert re.search(r'\b' + n + r'\s*=|"' + n + '"|' + n + r"=", PY), f"attribute {n} never passed"


def test_called_c_abi_functions_are_declared_and_exported():
    header = open(os.path.join(jax_ffi.ROOT, "include", "memlayer.h")).read()
    lib = L.lib()
    called = set(re.findall(r"\b(memlayer_\w+)\(", SRC))
    assert {"memlayer_pool_forward", "memlayer_layer_forward", "memlayer_layer_backward"} <= called
    for f in called:
        assert re.search(r"\b" + f + r"\(", header), f"{f} not declared in memlayer.h"
        assert hasattr(lib, f), f"{f} not exported"


@pytest.mark.skipif(jax_ffi.jax_available(), reason="JAX is installed: the binding builds")
def test_without_jax_the_build_skips_and_registration_fails_loudly():
    assert jax_ffi.build() is None
    with pytest.raises(ImportError):
        jax_ffi.register()
