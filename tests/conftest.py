"""Shared test configuration.

``-m "not gpu"``: oracle vs golden vectors, host-side logic, the C-ABI library
loading and exporting its symbols, multi-rank logic on gloo. ``-m gpu``: the
parity tests proper, through the C ABI on a B200.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
