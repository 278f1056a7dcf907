"""Shared pytest setup.

* registers the ``gpu`` marker (tests that need a B200);
* puts the package directory (rmlx-serve_b200/) and the oracle on sys.path;
* builds the oracle (test infrastructure) and the product library if their
  shared objects are missing, so a fresh checkout runs as-is.
"""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "rmlx-serve_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (PKG, ORACLE, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

if not os.path.exists(os.path.join(PKG, "lib", "librmlx_kv.so")):
    subprocess.run(["make", "-s", "-j8", "-C", PKG], check=True)
if not os.path.exists(os.path.join(ORACLE, "_build", "libkv_oracle.so")):
    subprocess.run(["make", "-s", "-C", ORACLE], check=True)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
