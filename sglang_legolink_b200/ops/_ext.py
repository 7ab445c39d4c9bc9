"""Locate and import the prebuilt in-tree extensions by path.

Importing never compiles: ``__graft_entry__.build()`` / ``python -m
sglang_legolink_b200.build_ext`` does.  On a CUDA tensor, every op requires
``legolink_cuda``; a missing build raises instead of falling back.
"""

from __future__ import annotations

import glob
import importlib.util
import os
import sys
import threading

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_EXT_DIR = os.path.join(_PKG, "_ext")
_lock = threading.Lock()
_mods: dict[str, object] = {}


class ExtensionMissing(RuntimeError):
    pass


def _import_so(name: str):
    with _lock:
        if name in _mods:
            return _mods[name]
        cands = sorted(glob.glob(os.path.join(_EXT_DIR, name, f"{name}*.so")))
        if not cands:
            raise ExtensionMissing(
                f"native extension '{name}' is not built; run "
                f"`python -m sglang_legolink_b200.build_ext` (expected under {_EXT_DIR}/{name})"
            )
        import torch  # noqa: F401  (loads libtorch / libc10 the .so links against)

        spec = importlib.util.spec_from_file_location(name, cands[0])
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        sys.modules[name] = mod
        _mods[name] = mod
        return mod


class _Counted:
    """Proxy over the kernel module that credits each launch to
    :mod:`sglang_legolink_b200.utils.launch_count`."""

    _KERNELS = {"gemm_small_m_splits": 0, "attn_prefill_tc_set_variant": 0, "attn_prefill_tc_trace": 0}

    def __init__(self, mod):
        self._mod = mod
        self._cache = {}

    def __getattr__(self, name):
        fn = self._cache.get(name)
        if fn is None:
            target = getattr(self._mod, name)
            from ..utils import launch_count

            k = self._KERNELS.get(name, 1)
            if name == "attn_decode":
                def fn(*a, **kw):
                    launch_count.add(2 if a[8] > 1 else 1)
                    return target(*a, **kw)
            elif k:
                def fn(*a, **kw):
                    launch_count.add(k)
                    return target(*a, **kw)
            else:
                fn = target
            self._cache[name] = fn
        return fn


_counted = None


def cuda():
    global _counted
    if _counted is None:
        _counted = _Counted(_import_so("legolink_cuda"))
    return _counted


def host():
    return _import_so("legolink_host")


def so_path(name: str) -> str:
    cands = sorted(glob.glob(os.path.join(_EXT_DIR, name, f"{name}*.so")))
    return cands[0] if cands else ""
