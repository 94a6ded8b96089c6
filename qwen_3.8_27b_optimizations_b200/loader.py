"""Load this package by path under the importable name ``iq4xs_b200``.

The package directory is named ``qwen_3.8_27b_optimizations_b200`` (dots are not valid in an
import statement), so callers do::

    import importlib.util, pathlib
    spec = importlib.util.spec_from_file_location("_iq4xs_loader", <repo>/qwen_3.8_27b_optimizations_b200/loader.py)
    ...
or simply use ``load()`` from a module that already imported this file.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

NAME = "iq4xs_b200"
PKG_DIR = Path(__file__).resolve().parent


def load():
    if NAME in sys.modules:
        return sys.modules[NAME]
    spec = importlib.util.spec_from_file_location(NAME, PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[NAME] = mod
    spec.loader.exec_module(mod)
    return mod
