"""Loads the in-tree native extensions.

The host runtime (``_host``) is required everywhere. The CUDA extension (``_cuda``) is required on
a GPU box: every op raises if it is missing — there is no silent PyTorch fallback.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

_EXT = Path(__file__).resolve().parent / "_ext"
_cache: dict[str, object] = {}


def _load(name: str, sub: str):
    if name in _cache:
        return _cache[name]
    path = _EXT / sub / f"{name}.so"
    if not path.exists():
        raise ImportError(
            f"vm_c_b200 native extension {name} is not built ({path} missing); "
            f"run `python -m vm_c_b200._build {sub}` or `python -c 'import __graft_entry__ as g; g.build()'`")
    if sub == "cuda":
        import torch  # noqa: F401  (libtorch / libc10 symbols must be loaded first)
    else:
        import torch  # noqa: F401
    spec = importlib.util.spec_from_file_location(name, str(path))
    mod = importlib.util.module_from_spec(spec)
    assert spec.loader is not None
    spec.loader.exec_module(mod)
    sys.modules[f"vm_c_b200.{name}"] = mod
    _cache[name] = mod
    return mod


def host():
    """The C++ host runtime module."""
    return _load("_host", "host")


def cuda():
    """The sm_100a kernel module (raises ImportError when it has not been built)."""
    return _load("_cuda", "cuda")


def cuda_available() -> bool:
    try:
        cuda()
        return True
    except ImportError:
        return False
