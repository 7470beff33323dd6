"""fasth3_b200: the B200 (sm_100a) quantized DiT-block hot path of FastH3 behind FastVideo's operator surface.

The directory is named ``fasth3-gb300_b200``; it is imported as ``fasth3_b200`` through :func:`load_package` in the
repository's ``__graft_entry__.py`` (a hyphenated directory is not an importable module name).
"""
from __future__ import annotations

from . import ops  # noqa: F401
from ._lib import LIB_PATH, lib  # noqa: F401
from . import layout, model, reduction, runner, sp, weights  # noqa: F401,E402

__all__ = ["ops", "lib", "LIB_PATH", "layout", "model", "reduction", "runner", "sp", "weights"]
