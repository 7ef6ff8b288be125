"""Shared pytest setup: markers and import paths.

``gpu``-marked tests need a CUDA device and the built ``libhotcold.so``; all
other tests run on a CPU-only host.
"""
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "hot-cold-neural-split-openinfer2_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built native library")
