"""Loading of the in-tree native extensions.

`_C` holds the sm_100a kernels and the ring engine; `_sched` the C++ workload
model, schedulers and shard plans. Both are built in place by
``python setup.py build_ext --inplace`` (or ``__graft_entry__.build()``).
A missing extension raises immediately: there is no Python fallback for any
kernel.
"""
from __future__ import annotations

import importlib

_cache: dict[str, object] = {}


def _load(name: str):
    mod = _cache.get(name)
    if mod is None:
        try:
            mod = importlib.import_module(f"multi_gpu_flashattention_b200.{name}")
        except ImportError as e:  # pragma: no cover - exercised only on broken installs
            raise ImportError(
                f"native extension multi_gpu_flashattention_b200.{name} is not built; run "
                "`python setup.py build_ext --inplace` in the repository root"
            ) from e
        _cache[name] = mod
    return mod


def C():
    """The CUDA extension (kernels + ring engine)."""
    return _load("_C")


def sched():
    """The C++ scheduler / shard-plan extension."""
    return _load("_sched")
