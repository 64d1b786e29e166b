"""``fpscan.ops`` (the reference's module path for the public API,
fpscan/ops.py:47-87), served by fpscan_b200."""
from fpscan_b200.ops import PScan, pscan, scan_forward

__all__ = ["pscan", "scan_forward", "PScan"]
