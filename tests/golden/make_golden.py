"""Generate the golden fixtures in tests/golden/ from the reference's own NumPy code.

Run in the build container (where the reference checkout exists), never on the GPU box:

    python tests/golden/make_golden.py --reference <path to the Faster-WeatherNext checkout>

The reference's modules import JAX at top level (absent here), so the pure NumPy/SciPy functions
are pulled out of the source files with `ast` and executed in a namespace holding numpy/scipy:

  src/faster_weathernext/pallas_attn.py   _hilbert3, hilbert_order, build_tile_mask
  src/faster_weathernext/patch.py         build_chunked_mask
  tests/test_pallas_kernel.py             _reference, _reference_grads  (float64 dense references)

Nothing of the reference is written into this repository except the outputs of those functions on
seeded inputs (and digests of the larger outputs).
"""

import argparse
import ast
import hashlib
import os
import sys

import numpy as np
from scipy import sparse

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "faster-weathernext_b200"))

from faster_weathernext import mesh  # noqa: E402


def extract(path, names):
  src = open(path).read()
  tree = ast.parse(src)
  body = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
  missing = set(names) - {n.name for n in body}
  assert not missing, missing
  ns = {"np": np, "sparse": sparse, "BLOCK_Q": 64, "BLOCK_K": 32}
  exec(compile(ast.Module(body=body, type_ignores=[]), path, "exec"), ns)
  return ns


def digest(*arrays):
  h = hashlib.sha256()
  for a in arrays:
    a = np.ascontiguousarray(a)
    h.update(str(a.dtype).encode())
    h.update(np.asarray(a.shape, np.int64).tobytes())
    h.update(a.tobytes())
  return h.hexdigest()


def random_mask(n, density, seed):
  """tests/test_masks.py:_random_mask recipe."""
  m = sparse.random(n, n, density=density, random_state=seed, format="csr").astype(bool)
  return (m + sparse.identity(n, dtype=bool, format="csr")).tocsr()


def kernel_masks():
  """The masks of tests/test_pallas_kernel.py (forward, grads sym/non-sym, transposed-list guard)."""
  fwd = (sparse.random(300, 300, density=0.1, random_state=1, format="csr").astype(bool)
         + sparse.identity(300, dtype=bool)).tocsr()
  base = sparse.random(300, 300, density=0.08, random_state=3, format="csr").astype(bool)
  sym = ((base + base.T) + sparse.identity(300, dtype=bool)).tocsr().astype(bool)
  nonsym = (base + sparse.identity(300, dtype=bool)).tocsr().astype(bool)
  guard = (sparse.random(130, 130, density=0.1, random_state=5, format="csr").astype(bool)
           + sparse.identity(130, dtype=bool)).tocsr()
  return {"k_fwd": fwd, "k_sym": sym, "k_nonsym": nonsym, "k_guard": guard}


def main():
  ap = argparse.ArgumentParser()
  ap.add_argument("--reference", required=True)
  args = ap.parse_args()
  ref = args.reference
  pa = extract(os.path.join(ref, "src/faster_weathernext/pallas_attn.py"),
               ["_hilbert3", "hilbert_order", "build_tile_mask"])
  pt = extract(os.path.join(ref, "src/faster_weathernext/patch.py"), ["build_chunked_mask"])
  tk = extract(os.path.join(ref, "tests/test_pallas_kernel.py"), ["_reference", "_reference_grads"])

  # ---- tile lists --------------------------------------------------------------------------
  tiles = {}
  masks = {f"rand{n}": random_mask(n, 0.05, 0) for n in (100, 257, 1000)}
  masks.update(kernel_masks())
  masks["k_nonsym_T"] = masks["k_nonsym"].T.tocsr()
  masks["k_guard_T"] = masks["k_guard"].T.tocsr()
  cfg_masks = {}
  for c in (1, 2, 3):
    m, lat, lon = mesh.config_mask(c)
    cfg_masks[c] = (m, lat, lon)
  masks["cfg1"] = cfg_masks[1][0]
  for name, m in masks.items():
    m = m.tocsr().astype(bool)
    m.sort_indices()
    ptr, kb, bits = pa["build_tile_mask"](m)
    tiles[f"{name}/indptr"] = m.indptr.astype(np.int32)
    tiles[f"{name}/indices"] = m.indices.astype(np.int32)
    tiles[f"{name}/shape"] = np.asarray(m.shape, np.int64)
    tiles[f"{name}/ptr"] = ptr
    tiles[f"{name}/kb"] = kb
    tiles[f"{name}/bits"] = bits
  digests = {}
  for c in (2, 3):
    m = cfg_masks[c][0]
    ptr, kb, bits = pa["build_tile_mask"](m)
    digests[f"cfg{c}/mask"] = mesh.csr_digest(m)
    digests[f"cfg{c}/tiles"] = digest(ptr, kb, bits)
    digests[f"cfg{c}/n_tiles"] = str(len(kb))
  digests["cfg1/mask"] = mesh.csr_digest(cfg_masks[1][0])
  np.savez_compressed(os.path.join(HERE, "tiles.npz"), **tiles)

  # ---- Hilbert order -----------------------------------------------------------------------
  rng = np.random.default_rng(0)
  lat, lon = rng.uniform(-90, 90, 5000), rng.uniform(0, 360, 5000)
  lat[:3] = np.nan
  hil = {"lat": lat, "lon": lon, "perm": pa["hilbert_order"](lat, lon).astype(np.int32)}
  for c in (1, 2, 3):
    _, la, lo = cfg_masks[c]
    digests[f"cfg{c}/hilbert"] = digest(pa["hilbert_order"](la, lo).astype(np.int64))
  np.savez_compressed(os.path.join(HERE, "hilbert.npz"), **hil)

  # ---- chunked (XLA-path) masks ------------------------------------------------------------
  n, chunk = 700, 64
  i, j = np.meshgrid(np.arange(n), np.arange(n), indexing="ij")
  banded = sparse.csr_matrix(np.abs(i - j) <= 40)
  ch = {}
  for name, m, c in (("banded", banded, chunk), ("cfg1", cfg_masks[1][0], 128), ("k_fwd", masks["k_fwd"], 64)):
    starts, bits, window, n_kv = pt["build_chunked_mask"](m, c)
    ch[f"{name}/starts"] = starts
    ch[f"{name}/bits"] = bits
    ch[f"{name}/window"] = np.int64(window)
    ch[f"{name}/n_kv"] = np.int64(n_kv)
    ch[f"{name}/chunk"] = np.int64(c)
  ch["banded/indptr"] = banded.indptr.astype(np.int32)
  ch["banded/indices"] = banded.indices.astype(np.int32)
  np.savez_compressed(os.path.join(HERE, "chunked.npz"), **ch)

  # ---- float64 attention references (the reference's own test functions) --------------------
  att = {}
  every = 6
  rng = np.random.default_rng(0)
  q, k, v = (rng.standard_normal((2, 300, 2, 64)).astype(np.float32) for _ in range(3))
  dense = masks["k_fwd"].toarray()
  for b in range(2):
    att[f"fwd/b{b}/out"] = tk["_reference"](q[b], k[b], v[b], dense, 64 ** -0.5)[::every].astype(np.float32)
  for sym in (True, False):
    rng = np.random.default_rng(2)
    q, k, v, do = (rng.standard_normal((1, 300, 2, 64)).astype(np.float32) for _ in range(4))
    m = masks["k_sym" if sym else "k_nonsym"].toarray()
    dq, dk, dv = tk["_reference_grads"](q[0], k[0], v[0], do[0], m, 64 ** -0.5)
    tag = "sym" if sym else "nonsym"
    for nm, x in (("dq", dq), ("dk", dk), ("dv", dv)):
      att[f"grad_{tag}/{nm}"] = x[::every].astype(np.float32)
  rng = np.random.default_rng(4)
  q, k, v, do = (rng.standard_normal((1, 130, 1, 32)).astype(np.float32) for _ in range(4))
  att["guard/dk"] = tk["_reference_grads"](q[0], k[0], v[0], do[0], masks["k_guard"].toarray(), 32 ** -0.5)[1].astype(np.float32)
  # Configuration 1: n=642 (icosphere level 3, Morton order), B1 H4 D64, Q/K/V from seed 0, dO from seed 1.
  m1 = cfg_masks[1][0].toarray()
  rng = np.random.default_rng(0)
  q, k, v = (rng.standard_normal((1, 642, 4, 64)).astype(np.float32) for _ in range(3))
  do = np.random.default_rng(1).standard_normal((1, 642, 4, 64)).astype(np.float32)
  att["cfg1/out"] = tk["_reference"](q[0], k[0], v[0], m1, 64 ** -0.5)[::every].astype(np.float32)
  dq, dk, dv = tk["_reference_grads"](q[0], k[0], v[0], do[0], m1, 64 ** -0.5)
  for nm, x in (("dq", dq), ("dk", dk), ("dv", dv)):
    att[f"cfg1/{nm}"] = x[::every].astype(np.float32)
  att["every"] = np.int64(every)
  np.savez_compressed(os.path.join(HERE, "attention.npz"), **att)

  with open(os.path.join(HERE, "digests.txt"), "w") as f:
    for key in sorted(digests):
      f.write(f"{key} {digests[key]}\n")
  print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
  main()
