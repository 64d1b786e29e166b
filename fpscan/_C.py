"""``fpscan._C`` for the reference's extension loader (fpscan/ops.py:14):
``fullscan_forward(gates, tokens, out, reverse)`` with the contract of the
reference's pybind binding (csrc/main.cpp:10), backed by libfpscan_b200.so."""
from fpscan_b200._C import fullscan_forward

__all__ = ["fullscan_forward"]
