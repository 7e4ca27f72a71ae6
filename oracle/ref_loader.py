"""Import the unmodified RFSN reference modules through the torch-CPU ``mlx`` shim.

TEST INFRASTRUCTURE ONLY: used by ``tests/golden/make_golden.py`` to generate
golden fixtures from the reference's own code.  The reference tree is read
only and is not present on GPU machines, so nothing on the product path, in
``bench.py`` or in the ``-m gpu`` tests calls this module.
"""
from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path

SHIM_DIR = Path(__file__).resolve().parent / "mlx_shim"


def reference_dir() -> Path:
    """The reference checkout named by RFSN_REFERENCE_DIR (there is no default location)."""
    d = os.environ.get("RFSN_REFERENCE_DIR")
    if not d:
        raise FileNotFoundError("set RFSN_REFERENCE_DIR to a checkout of the reference sources")
    return Path(d)

_MODULES = ("storage", "quantization", "attention", "cache", "rfsn_v10_mlx_ane_complete")


def reference_available(path: Path = None) -> bool:
    try:
        path = reference_dir() if path is None else path
    except FileNotFoundError:
        return False
    return (path / "quantization.py").is_file()


def load_reference(path: Path = None):
    """Return a namespace dict of the reference's modules, imported via the shim."""
    path = reference_dir() if path is None else path
    if not reference_available(path):
        raise FileNotFoundError(f"reference sources not found under {path}")
    sys.dont_write_bytecode = True  # the reference tree is read-only
    for p in (str(path), str(SHIM_DIR)):
        if p not in sys.path:
            sys.path.insert(0, p)
    mods = {}
    for name in _MODULES:
        mods[name] = importlib.import_module(name)
    return mods
