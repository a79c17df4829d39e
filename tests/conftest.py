"""Shared pytest setup: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs everything that needs no GPU (oracle vs golden
vectors, host-side logic, C-ABI symbol checks); ``-m gpu`` runs the parity
tests of the CUDA kernels on a B200.
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")


def require_cuda():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("this test needs a CUDA device (run with -m 'not gpu' on CPU)")
    return torch.device("cuda", 0)

# The reference package (an unmodified copy installed under baseline/_ref)
# is used by a few GPU tests as a second, independent checker when present.
_REF = os.path.join(ROOT, "baseline", "_ref")
if os.path.isdir(_REF) and _REF not in sys.path:
    sys.path.append(_REF)
