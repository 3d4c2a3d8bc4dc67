"""tenzor_b200 -- sm_100a (B200) backend for the Arctic-embed-xs encoder hot path of tenzor.

The compute lives in libtenzor_cuda.so (include/tenzor_cuda.h); this package is its host-side
mirror of the reference's model and kernel API.  Importing it never falls back to CPU compute.
"""
from . import synthetic  # noqa: F401  (pure numpy, always importable)
from ._lib import EXPORTS, LIB_PATH, TenzorError, lib  # noqa: F401

__all__ = ["synthetic", "lib", "TenzorError", "LIB_PATH", "EXPORTS"]
