"""Run the reference's own hot-path tests against the drop-in (CPU, test
infrastructure).

The reference's test modules (``rfsn_v10_5`` package tests) import
``rfsn_v10_5.cache``, ``.block_manager``, ``.residency`` and ``.storage``;
here those names resolve to this repository's drop-in modules, while the
reference's own ``config``, ``layer``, ``model`` and ``attention_exact`` run
unmodified over the torch-CPU ``mlx`` shim. So the reference's model drives
the drop-in cache exactly as it drives its own, and the reference's own
assertions check the result.

Two adapters sit on the boundary, because the drop-in takes torch tensors
where the reference passes MLX arrays:
* arrays going in (``append_exact``) are unwrapped to their torch tensors;
* tensors coming out (segments, ``hot_k`` / ``hot_v``, materialized
  contexts) are wrapped as shim arrays.
The device mechanics are the CPU test double of ``tests/fake_ops.py`` (no
GPU here); RoPE and attention are the reference's.
"""

from __future__ import annotations

import importlib
import os
import sys
import types
import unittest
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
REFERENCE = Path(os.environ.get("RFSN_REFERENCE", "/root/reference"))
DROP_IN = ("block_manager", "residency", "storage")
HOT_PATH_TESTS = ("test_page_table", "test_prefetch", "test_archived_runtime", "test_runtime_spine",
                  "test_context_bounds", "test_exactness_vs_reference", "test_generation_restore_continuity",
                  "test_session_persistence", "test_archive_integrity")


def reference_available() -> bool:
    return (REFERENCE / "rfsn_v10_5" / "cache.py").exists() and (REFERENCE / "tests").is_dir()


def _facade_cache_module():
    import torch

    import mlx.core as mx
    from fake_ops import FakeDeviceOps
    from rfsn_b200 import cache as drop_in

    def wrap(x):
        return mx.array(x) if isinstance(x, torch.Tensor) else x

    def unwrap(x):
        return x._t if isinstance(x, mx.array) else x

    def wrap_segments(segs):
        return [(wrap(k), wrap(v), int(s)) for k, v, s in segs]

    def wrap_context(ctx):
        return tuple(wrap(x) for x in ctx)

    class LayerKVCache(drop_in.LayerKVCache):
        # segments are wrapped for callers outside the cache only: the drop-in's
        # own methods (materialize_*) call the segment getters on torch tensors
        _inside = 0

        def __init__(self, config, batch_size, num_heads, num_kv_heads=None, **kw):
            kw.setdefault("ops", FakeDeviceOps())
            kw.setdefault("device", "cpu")
            super().__init__(config, batch_size, num_heads, num_kv_heads, **kw)

        def _out(self, segs):
            return segs if self._inside else wrap_segments(segs)

        def _inner(self, fn, *a):
            self._inside += 1
            try:
                return fn(*a)
            finally:
                self._inside -= 1

        def append_exact(self, k, v):
            return super().append_exact(unwrap(k), unwrap(v))

        def get_attention_segments(self):
            return self._out(super().get_attention_segments())

        def get_archived_attention_segments(self):
            return self._out(super().get_archived_attention_segments())

        def get_hot_attention_segments(self):
            return self._out(super().get_hot_attention_segments())

        def get_mixed_attention_segments(self, *a):
            return self._out(super().get_mixed_attention_segments(*a))

        def materialize_exact_context(self):
            return wrap_context(self._inner(super().materialize_exact_context))

        def materialize_archived_context(self, *a):
            return wrap_context(self._inner(super().materialize_archived_context, *a))

        def materialize_mixed_context(self, *a):
            return wrap_context(self._inner(super().materialize_mixed_context, *a))

        @property
        def hot_k(self):
            return wrap(drop_in.LayerKVCache.hot_k.fget(self))

        @property
        def hot_v(self):
            return wrap(drop_in.LayerKVCache.hot_v.fget(self))

    class RFSNCache(drop_in.RFSNCache):
        def __init__(self, config, batch_size, **kw):
            kw.setdefault("device", "cpu")
            kw.setdefault("ops_factory", FakeDeviceOps)
            super().__init__(config, batch_size, **kw)
            for lc in self.layers:
                lc.__class__ = LayerKVCache

    mod = types.ModuleType("rfsn_v10_5.cache")
    mod.__dict__.update({k: getattr(drop_in, k) for k in dir(drop_in) if not k.startswith("__")})
    mod.LayerKVCache = LayerKVCache
    mod.RFSNCache = RFSNCache
    return mod


def install() -> None:
    """Make ``rfsn_v10_5`` the reference package with the drop-in's cache,
    block manager, residency and storage modules (idempotent)."""
    if getattr(sys.modules.get("rfsn_v10_5"), "__drop_in__", False):
        return
    for p in (str(REPO / "oracle" / "mlx_shim"), str(REFERENCE), str(REPO / "rfsn-mlx_b200"), str(REPO / "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    for name in list(sys.modules):
        if name == "rfsn_v10_5" or name.startswith("rfsn_v10_5.") or name == "tests" or name.startswith("tests."):
            del sys.modules[name]
    for name in DROP_IN:
        sys.modules[f"rfsn_v10_5.{name}"] = importlib.import_module(f"rfsn_b200.{name}")
    sys.modules["rfsn_v10_5.cache"] = _facade_cache_module()
    pkg = importlib.import_module("rfsn_v10_5")
    pkg.__drop_in__ = True
    for name in DROP_IN + ("cache",):
        setattr(pkg, name, sys.modules[f"rfsn_v10_5.{name}"])


def run_reference_tests(module_name: str) -> unittest.TestResult:
    """Load one of the reference's test modules (from its tests/ package) and run it."""
    install()
    if str(REFERENCE) not in sys.path:
        sys.path.insert(0, str(REFERENCE))
    mod = importlib.import_module(f"tests.{module_name}")
    suite = unittest.defaultTestLoader.loadTestsFromModule(mod)
    result = unittest.TestResult()
    cwd = os.getcwd()
    import tempfile

    with tempfile.TemporaryDirectory() as tmp:
        os.chdir(tmp)  # the reference's default disk_cache_dir is relative
        try:
            suite.run(result)
        finally:
            os.chdir(cwd)
    return result
