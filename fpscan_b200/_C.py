"""Stand-in for the reference's compiled extension module ``fpscan._C``.

The reference loads its extension by importing a candidate module that has a
``fullscan_forward`` attribute (fpscan/ops.py:14, 29-38; bound at
csrc/main.cpp:10).  Importing this module gives it that attribute, backed by
``libfpscan_b200.so``.  ``dimwise_forward`` (csrc/main.cpp:9) is the
reference's experimental content-dependent combine, not part of its public
API, and is not provided.
"""
from .ops import fullscan_forward

__all__ = ["fullscan_forward"]
