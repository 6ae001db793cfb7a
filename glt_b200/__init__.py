"""B200-native (sm_100a) grafted-MLP training library.

The compute path is the in-tree CUDA library ``libglt_b200.so`` (C ABI in
``include/glt_graft.h``).  ``glt_b200.graft`` is the host-side mirror of the
reference's graft interface; importing it (or ``glt_b200._lib``) loads the
library and raises ImportError when it is missing -- there is no fallback.
``python -m glt_b200.build`` compiles the library in-tree.
"""

__all__ = ["graft"]
