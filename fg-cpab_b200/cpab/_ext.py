"""Loader of _cpab_ext.so, the C++ autograd nodes of transform_grid and of
the spatial-transformer warp (csrc/torch_ext.cpp, built by
fg-cpab_b200/build.py next to this file).

They compute exactly what the Python nodes (_CPABFunction, warp._Warp)
compute -- the same C ABI calls with the same arguments -- with far less host
time per step.  The package uses them when the extension is built and
CPAB_B200_NO_EXT is not set; the Python nodes are the fallback otherwise.
"""
import importlib.machinery
import importlib.util
import os

import torch  # noqa: F401  (libtorch must be loaded before the extension)

import contextlib

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_cpab_ext.so")
_mod = None
_off = 0


@contextlib.contextmanager
def python_path():
    """Within this context transform_grid takes the Python autograd node (the
    benchmark's per-call instrumentation wraps that path's C ABI calls)."""
    global _off
    _off += 1
    try:
        yield
    finally:
        _off -= 1


def module():
    """The extension module, or None when it is not built or disabled."""
    global _mod
    if _off:
        return None
    if _mod is None:
        if os.environ.get("CPAB_B200_NO_EXT") or not os.path.exists(PATH):
            return None
        loader = importlib.machinery.ExtensionFileLoader("_cpab_ext", PATH)
        spec = importlib.util.spec_from_file_location("_cpab_ext", PATH, loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        _mod = mod
    return _mod


def call(fn, *args):
    """fn(*args) of the extension; a failed C ABI call (the node's message
    starts with the library's name) raises the same error type as the
    Python path."""
    from . import _native
    try:
        return fn(*args)
    except RuntimeError as e:
        first = str(e).split("\n", 1)[0]
        if first.startswith("libcpab_b200: "):
            raise _native.CpabNativeError(first[len("libcpab_b200: "):]) from None
        raise
