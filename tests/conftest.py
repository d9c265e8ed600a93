"""Test configuration: import paths, the `gpu` marker, shared fixtures."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "faster-weathernext_b200"))
sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
  config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and libfwn_attn.so")


@pytest.fixture(scope="session")
def golden():
  """Fixtures written by tests/golden/make_golden.py from the reference's own NumPy code."""
  out = {name: np.load(os.path.join(GOLDEN, name + ".npz")) for name in ("tiles", "hilbert", "chunked", "attention")}
  digests = {}
  with open(os.path.join(GOLDEN, "digests.txt")) as f:
    for line in f:
      k, v = line.split()
      digests[k] = v
  out["digests"] = digests
  return out


@pytest.fixture(scope="session")
def cuda():
  import torch
  if not torch.cuda.is_available():
    pytest.fail("GPU test collected on a machine without CUDA (run with -m 'not gpu')")
  major, minor = torch.cuda.get_device_capability()
  if major != 10:
    pytest.fail(f"needs an sm_100 device, found sm_{major}{minor}")
  from faster_weathernext import _lib
  _lib.lib()
  return torch.device("cuda", 0)
