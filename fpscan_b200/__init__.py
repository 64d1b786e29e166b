"""fpscan_b200: B200 (sm_100a) linear-recurrence scan with fpscan's Python API.

``from fpscan_b200 import pscan, scan_forward, PScan`` is a drop-in for
``from fpscan import pscan, scan_forward, PScan`` (reference fpscan/__init__.py:1-3).
``fpscan_b200._C`` offers the reference extension's ``fullscan_forward`` so the
reference's own loader (fpscan/ops.py:14, _EXT_CANDIDATES) can bind it.
"""
from .ops import (PScan, pscan, pscan_anylen, pscan_channels_last, pscan_gated, scan_backward,
                  scan_forward, scan_forward_anylen, scan_forward_channels_last,
                  scan_forward_gated)
from ._lib import DeviceStatusError, check_device_status, set_wait_limit

__all__ = ["pscan", "scan_forward", "PScan"]
__version__ = "0.1.0"
