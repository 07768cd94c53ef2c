"""pytest configuration: the `gpu` marker (tests that need a B200; run with -m gpu) and the import paths of the
in-tree package (mac-ai-engineering_b200/macai_b200) and of the CPU oracle (oracle/, test infrastructure)."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "mac-ai-engineering_b200"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a); run with -m gpu")
