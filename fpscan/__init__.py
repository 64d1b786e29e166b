"""Drop-in import name for the reference package.

``from fpscan import pscan, scan_forward, PScan`` (the reference's
fpscan/__init__.py:1-3) resolves here to the B200 implementation in
``fpscan_b200``, and ``fpscan._C`` -- the first candidate of the
reference's extension loader (fpscan/ops.py:14, 29-38) -- is this package's
``_C`` module, whose ``fullscan_forward`` runs on ``libfpscan_b200.so``.
A caller that keeps the reference's own ``fpscan/ops.py`` therefore binds
this library without editing it.
"""
from fpscan_b200 import PScan, pscan, scan_forward

__all__ = ["pscan", "scan_forward", "PScan"]
__version__ = "0.1.2"
