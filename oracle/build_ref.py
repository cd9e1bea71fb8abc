"""Build the reference's own C++/ATen HSTU attention into ``oracle/_ref/``.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package may import this.

The reference implements ``hammer::triton_ragged_attention_fwd`` as the ATen
composite ``raggedAttention`` in ``recir/ops/kjt_split_per_feature.cpp:602-693``
(registration ``:780-793``).  That single translation unit compiles against
the installed torch headers, so it is built where it lies (no source is copied
into this repository) and only the resulting shared object lands in
``oracle/_ref/``.  The shared object is what travels to a GPU machine; the
reference tree itself does not.

Usage:  python oracle/build_ref.py [/path/to/reference]
(default: ``oracle.refroot.reference_root()``, i.e. ``$RECIR_REFERENCE_ROOT`` or the conventional
checkout location)
"""
from __future__ import annotations

import os
import shutil
import sys

if __package__ in (None, ""):
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from oracle import refroot  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
LIB_NAME = "recir_ref_ops"
LIB_PATH = os.path.join(OUT_DIR, LIB_NAME + ".so")
REL_SOURCE = os.path.join("recir", "ops", "kjt_split_per_feature.cpp")


def ref_available() -> bool:
    return os.path.exists(LIB_PATH)


def build(reference_root: str | None = None, verbose: bool = False) -> str | None:
    """Compile the reference op; returns the .so path or None if no source tree."""
    if reference_root is None:
        reference_root = refroot.reference_root()
    src = os.path.join(reference_root, REL_SOURCE)
    if not os.path.exists(src):
        return LIB_PATH if ref_available() else None
    if ref_available() and os.path.getmtime(LIB_PATH) >= os.path.getmtime(src):
        return LIB_PATH
    from torch.utils import cpp_extension

    os.makedirs(OUT_DIR, exist_ok=True)
    build_dir = os.path.join(OUT_DIR, "build")
    os.makedirs(build_dir, exist_ok=True)
    cpp_extension.load(
        name=LIB_NAME,
        sources=[src],
        extra_include_paths=[reference_root],
        extra_cflags=["-O2"],
        build_directory=build_dir,
        is_python_module=False,
        verbose=verbose,
    )
    shutil.copyfile(os.path.join(build_dir, LIB_NAME + ".so"), LIB_PATH)
    shutil.rmtree(build_dir, ignore_errors=True)
    return LIB_PATH


def load() -> None:
    """Load the built reference library so ``torch.ops.hammer.*`` resolves."""
    import torch

    if not ref_available():
        raise FileNotFoundError(
            f"{LIB_PATH} missing: run `python oracle/build_ref.py` where the reference tree exists"
        )
    torch.ops.load_library(LIB_PATH)


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else None
    print(build(root, verbose=True))
