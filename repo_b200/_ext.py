"""Loader of the torch binding ``lib/_cs_torch.so`` (csrc/torch_api.cpp).

The binding calls the C ABI of ``libcubicsplat_b200.so`` once per autograd
stage (forward, backward, metric) with torch tensors, allocating from torch's
caching allocator and launching on the current torch stream.  Like the ctypes
binding it has no fallback: a missing library raises.
"""
from __future__ import annotations

import importlib.util
import os
import threading

from . import _native

EXT_PATH = os.path.join(_native.HERE, "lib", "_cs_torch.so")

_lock = threading.Lock()
_mod = None


def load():
    """The binding module (raises if it has not been built)."""
    global _mod
    if _mod is not None:
        return _mod
    with _lock:
        if _mod is None:
            _native.load()  # the C-ABI library the binding links against
            if not os.path.exists(EXT_PATH):
                raise _native.NativeError(
                    f"{EXT_PATH} is missing: build it with `python -m repo_b200.build` "
                    "(there is no CPU fallback)")
            spec = importlib.util.spec_from_file_location("repo_b200._cs_torch", EXT_PATH)
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            _mod = mod
    return _mod
