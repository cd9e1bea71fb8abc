"""Where the reference project's source tree lives (TEST INFRASTRUCTURE ONLY).

One place for the path: the environment variable ``RECIR_REFERENCE_ROOT`` if set, else the
conventional checkout location.  The tree is only needed to (re)build ``oracle/_ref`` and to
(re)generate the golden fixtures under ``tests/golden/``; nothing that runs on a GPU machine
reads it, and tests that want it skip when it is absent.
"""
from __future__ import annotations

import importlib.util
import os
import sys
import types
from unittest import mock

_DEFAULT = os.path.join(os.sep, "root", "reference")


def reference_root() -> str:
    return os.environ.get("RECIR_REFERENCE_ROOT", _DEFAULT)


def reference_path(*parts: str) -> str:
    return os.path.join(reference_root(), *parts)


def reference_present() -> bool:
    return os.path.isdir(reference_path("recir"))


def load_reference_module(rel_path: str, name: str, stub_modules=()):
    """Imports ONE file of the reference tree by path (the package itself cannot be imported:
    its ``__init__`` chain needs jax).  ``stub_modules`` names third-party modules that the file
    imports but does not need for the functions used here; they are replaced by mocks while the
    file executes."""
    path = reference_path(*rel_path.split("/"))
    if not os.path.exists(path):
        raise FileNotFoundError(path)
    saved = {}
    for m in stub_modules:
        saved[m] = sys.modules.get(m)
        stub = mock.MagicMock(name=m)
        stub.__spec__ = None
        sys.modules[m] = stub
    try:
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        assert isinstance(mod, types.ModuleType)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    finally:
        for m, old in saved.items():
            if old is None:
                sys.modules.pop(m, None)
            else:
                sys.modules[m] = old
    return mod
