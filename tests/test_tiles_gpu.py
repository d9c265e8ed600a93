"""GPU: the CUDA tile-list builder, pairing and Hilbert codes against the reference's outputs (bit-exact)."""
import numpy as np
import pytest
import torch
from scipy import sparse

from oracle import tiles as ot
from tests.helpers import digest, golden_mask, golden_names

pytestmark = pytest.mark.gpu


def _build(m, device):
  from faster_weathernext import tiled_attn as ta
  m = sparse.csr_matrix(m)
  indptr = torch.from_numpy(m.indptr.astype(np.int32)).to(device)
  indices = torch.from_numpy(m.indices.astype(np.int32)).to(device)
  return ta.build_tiles_device(indptr, indices, m.shape[0], m.shape[1])


def test_builder_bit_exact_on_reference_cases(golden, cuda):
  g = golden["tiles"]
  for name in golden_names(g):
    ptr, kb, bits = _build(golden_mask(g, name), cuda).numpy()
    np.testing.assert_array_equal(ptr, g[name + "/ptr"], err_msg=name)
    np.testing.assert_array_equal(kb, g[name + "/kb"], err_msg=name)
    np.testing.assert_array_equal(bits, g[name + "/bits"], err_msg=name)


def test_build_tile_mask_dropin_returns_reference_types(golden, cuda):
  from faster_weathernext import tiled_attn as ta
  g = golden["tiles"]
  ptr, kb, bits = ta.build_tile_mask(golden_mask(g, "rand257"))
  assert ptr.dtype == np.int32 and kb.dtype == np.int32 and bits.dtype == np.uint32 and bits.shape[1] == 64
  np.testing.assert_array_equal(bits, g["rand257/bits"])


@pytest.mark.parametrize("cfg", [2, 3])
def test_builder_config_lists_match_reference_digest(golden, cuda, cfg):
  from faster_weathernext import mesh
  m, _, _ = mesh.config_mask(cfg)
  assert mesh.csr_digest(m) == golden["digests"][f"cfg{cfg}/mask"]
  ptr, kb, bits = _build(m, cuda).numpy()
  assert digest(ptr, kb, bits) == golden["digests"][f"cfg{cfg}/tiles"]


def test_builder_unsorted_duplicate_and_empty_rows(cuda):
  """CSR with unsorted columns, duplicate entries and empty rows gives the same list as the clean mask."""
  rng = np.random.default_rng(7)
  n = 333
  m = sparse.random(n, n, density=0.03, random_state=8, format="csr").astype(bool)
  m[5] = False
  m[200:260] = False
  m.eliminate_zeros()
  ref = ot.build_tile_mask(m)
  rows = np.repeat(np.arange(n), np.diff(m.indptr))
  cols = m.indices.copy()
  dup = rng.integers(0, len(cols), 100)
  rows = np.concatenate([rows, rows[dup]])
  cols = np.concatenate([cols, cols[dup]])
  order = rng.permutation(len(rows))
  order = order[np.argsort(rows[order], kind="stable")]   # rows sorted, columns shuffled
  indptr = np.zeros(n + 1, np.int32)
  np.add.at(indptr, rows + 1, 1)
  indptr = np.cumsum(indptr).astype(np.int32)
  t = torch.from_numpy(indptr).to(cuda), torch.from_numpy(cols[order].astype(np.int32)).to(cuda)
  from faster_weathernext import tiled_attn as ta
  got = ta.build_tiles_device(t[0], t[1], n, n).numpy()
  for a, b in zip(got, ref):
    np.testing.assert_array_equal(a, b)


def test_builder_rectangular_and_empty(cuda):
  m = sparse.random(70, 1000, density=0.02, random_state=3, format="csr").astype(bool)
  for mm in (m, sparse.csr_matrix((64, 64), dtype=bool)):
    got = _build(mm, cuda).numpy()
    ref = ot.build_tile_mask(mm)
    for a, b in zip(got, ref):
      np.testing.assert_array_equal(a, b)


def test_builder_large_block_uses_global_path(cuda):
  """A query block with more tiles than fit in shared memory (dense 64 x 40,000 block)."""
  n_cols = 40000
  rows = np.repeat(np.arange(64), 700)
  rng = np.random.default_rng(1)
  cols = rng.integers(0, n_cols, len(rows))
  m = sparse.csr_matrix((np.ones(len(rows), bool), (rows, cols)), shape=(64, n_cols))
  got = _build(m, cuda).numpy()
  ref = ot.build_tile_mask(m)
  for a, b in zip(got, ref):
    np.testing.assert_array_equal(a, b)


def test_pairing_matches_oracle(golden, cuda):
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  g = golden["tiles"]
  cases = [golden_mask(g, nm) for nm in ("rand100", "rand257", "rand1000", "k_nonsym_T", "cfg1")]
  cases.append(mesh.config_mask(3)[0])
  for m in cases:
    t64 = _build(m, cuda)
    got = ta.pair_tiles(t64).numpy()
    ref = ot.pair_tiles(*ot.build_tile_mask(m))
    for a, b in zip(got, ref):
      np.testing.assert_array_equal(a, b)


def test_hilbert_order_matches_reference(golden, cuda):
  from faster_weathernext import tiled_attn as ta
  h = golden["hilbert"]
  np.testing.assert_array_equal(ta.hilbert_order(h["lat"], h["lon"]), h["perm"])


@pytest.mark.parametrize("cfg", [1, 2, 3])
def test_hilbert_order_config_digests(golden, cuda, cfg):
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  _, lat, lon = mesh.config_mask(cfg)
  assert digest(ta.hilbert_order(lat, lon).astype(np.int64)) == golden["digests"][f"cfg{cfg}/hilbert"]


def test_gather_lists_match_oracle(golden, cuda):
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  g = golden["tiles"]
  cases = [golden_mask(g, nm) for nm in ("rand100", "rand257", "rand1000", "k_nonsym_T", "cfg1")]
  cases.append(mesh.config_mask(3)[0])
  for m in cases:
    t128 = ta.pair_tiles(_build(m, cuda))
    got = ta.gather_tiles(t128).numpy()
    ref = ot.gather_tiles(*ot.pair_tiles(*ot.build_tile_mask(m)))
    for a, b in zip(got, ref):
      np.testing.assert_array_equal(a, b)
