"""Access to the reference package ``ivonar_inference``, whose decoder interface this package plugs into.

``B200Decoder`` is a subclass of the reference's ``StaticDecoder`` (as the reference's own GPU decoder
``KernelDecoder`` is), and the models it runs are the reference's ``IvonarModel`` objects built by the
reference's loader. The reference therefore has to be importable: installed in the environment, on
``PYTHONPATH``, or installed into this repository's ``baseline/_ref`` directory with
``python -m pip install --no-deps --target baseline/_ref <path to the reference>``.
"""

from __future__ import annotations

import sys
from pathlib import Path
from types import ModuleType

_BUNDLED = Path(__file__).resolve().parent.parent / "baseline" / "_ref"


def load() -> ModuleType:
    """The ``ivonar_inference`` package (from the environment first, else from ``baseline/_ref``)."""

    try:
        import ivonar_inference
    except ImportError:
        if not (_BUNDLED / "ivonar_inference").is_dir():
            raise ImportError(
                "the reference package ivonar_inference is required (install it, put it on PYTHONPATH, or "
                f"install it into {_BUNDLED} with pip --target)"
            ) from None
        if str(_BUNDLED) not in sys.path:
            sys.path.append(str(_BUNDLED))
        import ivonar_inference
    return ivonar_inference


def module(name: str) -> ModuleType:
    """A submodule of the reference package, e.g. ``module("decoder")``."""

    load()
    import importlib

    return importlib.import_module(f"ivonar_inference.{name}")
