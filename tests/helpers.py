"""Shared helpers for the tests (mask recipes of the reference's tests, golden lookups)."""
import hashlib

import numpy as np
from scipy import sparse


def golden_mask(g, name):
  sh = tuple(int(x) for x in g[name + "/shape"])
  idx = g[name + "/indices"]
  return sparse.csr_matrix((np.ones(len(idx), bool), idx, g[name + "/indptr"]), shape=sh)


def golden_names(g):
  return sorted({k.split("/")[0] for k in g.files})


def digest(*arrays):
  """Same digest as tests/golden/make_golden.py."""
  h = hashlib.sha256()
  for a in arrays:
    a = np.ascontiguousarray(a)
    h.update(str(a.dtype).encode())
    h.update(np.asarray(a.shape, np.int64).tobytes())
    h.update(a.tobytes())
  return h.hexdigest()


def kernel_inputs(seed, shape, count):
  """rng.standard_normal float32 arrays, in the order the reference's tests draw them."""
  rng = np.random.default_rng(seed)
  return [rng.standard_normal(shape).astype(np.float32) for _ in range(count)]
