"""B200-native (sm_100a) grafted-MLP training library.

The compute path is the in-tree CUDA library ``libglt_b200.so`` (C ABI in
``include/glt_graft.h``); this package is its Python host binding and the
host-side mirror of the reference's graft interface.
"""
from . import _lib  # noqa: F401  (fails loudly when the CUDA library is missing)
from ._lib import GltError, check, last_error  # noqa: F401

__all__ = ["GltError", "check", "last_error"]
