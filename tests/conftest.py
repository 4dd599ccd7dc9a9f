"""Shared pytest setup: the ``gpu`` marker and import paths.

Tests marked ``gpu`` need a CUDA device and the built library; everything else
runs on the CPU (the oracle against the golden fixtures, host-side logic, and
loading the C-ABI library without launching anything).
"""
import os
import pathlib
import sys

ROOT = pathlib.Path(__file__).resolve().parent.parent
PKG = ROOT / "adaptive-specdec_b200"
for p in (str(PKG), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")
