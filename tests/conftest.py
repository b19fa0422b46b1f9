"""pytest configuration: the ``gpu`` marker and import paths.

Tests marked ``gpu`` need a CUDA device (they run the sm_100a kernels through
the C-ABI library); everything else runs on the CPU.
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "rocm-qlora_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and the built sm_100a library")


def pytest_terminal_summary(terminalreporter):
    """One line per recorded parity check: the plain max-abs / RMS figure and
    the count of outputs that passed only through the ulp allowance."""
    from tests.tolerance import RECORDED
    if not RECORDED:
        return
    tr = terminalreporter
    tr.write_line("parity (max-abs/RMS, outputs over the bare 1e-2*RMS bar / outputs):")
    for label, rel, n_ulp, n in RECORDED:
        tr.write_line(f"  {label}: {rel:.2e}, {n_ulp}/{n}")
