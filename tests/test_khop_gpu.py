"""GPU: device k-hop masks (bitset reach + CSR) against the host sparse matrix power the reference uses
(`adj_mat ** attention_k_hop`, src/faster_weathernext/patch.py:209) and the BFS in `mesh.k_hop_mask`;
and tile lists built from the device CSR against the reference builder's lists (bit-exact)."""
import numpy as np
import pytest
import torch
from scipy import sparse

from oracle import tiles as ot

pytestmark = pytest.mark.gpu


def _device_csr(adj, hops, device):
  from faster_weathernext import tiled_attn as ta
  ip, ix = ta.khop_csr_device(adj, hops, device)
  n = adj.shape[0]
  return sparse.csr_matrix((np.ones(ix.numel(), bool), ix.cpu().numpy(), ip.cpu().numpy()), shape=(n, n))


def _power_pattern(adj, hops):
  """Nonzero pattern of (adj + I) ** hops (float powers as scipy's `**` on the reference's matrix)."""
  a = (sparse.csr_matrix(adj).astype(np.float64) + sparse.identity(adj.shape[0], format="csr")).tocsr()
  a.data[:] = 1.0
  r = sparse.identity(adj.shape[0], format="csr")
  for _ in range(hops):
    r = (r @ a).tocsr()
    r.data[:] = 1.0
  r = r.astype(bool).tocsr()
  r.sort_indices()
  return r


def _equal(a, b):
  a, b = a.tocsr(), b.tocsr()
  a.sort_indices()
  b.sort_indices()
  return a.shape == b.shape and np.array_equal(a.indptr, b.indptr) and np.array_equal(a.indices, b.indices)


@pytest.mark.parametrize("level,hops", [(3, 0), (3, 1), (3, 2), (3, 5), (4, 8), (3, 40)])
def test_khop_matches_matrix_power_on_mesh(cuda, level, hops):
  from faster_weathernext import mesh
  xyz, faces = mesh.icosphere(level)
  adj = mesh.adjacency(faces, xyz.shape[0])
  got = _device_csr(adj, hops, cuda)
  assert _equal(got, _power_pattern(adj, hops))
  if hops:
    assert _equal(got, mesh.k_hop_mask(adj, hops))
  if hops >= 2:
    # Without self edges the plain power (the reference's `adj_mat ** k`) has the same pattern on a mesh.
    plain = sparse.csr_matrix(adj - sparse.identity(adj.shape[0], dtype=bool, format="csr")).astype(np.float64)
    plain.eliminate_zeros()
    ref = (plain ** hops).astype(bool).tocsr()
    assert _equal(got, ref)


def test_khop_general_graph_unsorted_duplicates(cuda):
  """Non-symmetric random graph, n not a multiple of 32, duplicate and unsorted CSR entries, isolated rows."""
  n = 1001
  m = sparse.random(n, n, density=0.002, random_state=3, format="csr").astype(bool)
  m[17] = False
  m.eliminate_zeros()
  rows = np.repeat(np.arange(n), np.diff(m.indptr))
  cols = m.indices.copy()
  rng = np.random.default_rng(5)
  dup = rng.integers(0, len(cols), 200)
  rows, cols = np.concatenate([rows, rows[dup]]), np.concatenate([cols, cols[dup]])
  order = rng.permutation(len(rows))
  rows, cols = rows[order], cols[order]
  # Build a CSR whose per-row column order is the shuffled one (no sorting, duplicates kept).
  srt = np.argsort(rows, kind="stable")
  indptr = np.concatenate([[0], np.cumsum(np.bincount(rows, minlength=n))]).astype(np.int32)
  raw = sparse.csr_matrix((np.ones(len(rows), bool), cols[srt].astype(np.int32), indptr), shape=(n, n))
  for hops in (1, 3, 6):
    assert _equal(_device_csr(raw, hops, cuda), _power_pattern(m, hops)), hops


def test_khop_tiles_match_reference_builder(cuda):
  """Lists from the device k-hop CSR equal the reference builder's lists of the host mask (level 4, 6 hops)."""
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  xyz, faces = mesh.icosphere(4)
  lat, lon = mesh.latlon(xyz)
  perm = mesh.morton_order(lat, lon)
  adj = mesh.permute(mesh.adjacency(faces, xyz.shape[0]), perm)
  n = adj.shape[0]
  ip, ix = ta.khop_csr_device(adj, 6, cuda)
  ptr, kb, bits = ta.build_tiles_device(ip, ix, n, n).numpy()
  host = mesh.k_hop_mask(adj, 6)
  rptr, rkb, rbits = ot.build_tile_mask(host)
  np.testing.assert_array_equal(ptr, rptr)
  np.testing.assert_array_equal(kb, rkb)
  np.testing.assert_array_equal(bits, rbits)
  tiles = ta.AttentionTiles.from_khop(adj, 6, device=cuda)
  ref = ta.AttentionTiles.from_mask(host, device=cuda)
  for a, b in ((tiles.fwd, ref.fwd), (tiles.fwd_g, ref.fwd_g)):
    for x, y in zip(a.numpy(), b.numpy()):
      np.testing.assert_array_equal(x, y)


def test_khop_rejects_bad_arguments(cuda):
  from faster_weathernext import _lib
  lib = _lib.lib()
  with pytest.raises(ValueError):
    _lib.check(lib.fwn_khop_bitset(0, 0, 10, -1, 0, 0, 0))
  with pytest.raises(ValueError):
    _lib.check(lib.fwn_khop_bitset(0, 0, 10, 2, 0, 0, 0))
  with pytest.raises(NotImplementedError):
    _lib.check(lib.fwn_bitset_csr_count(0, 50000, 50000, 0, 0, 0, 0))
  assert lib.fwn_bitset_words(40962) == 1284 and lib.fwn_bitset_words(32) == 4


@pytest.mark.parametrize("power", [0, 1, 2, 3, 7])
def test_walk_pattern_matches_plain_matrix_power(cuda, power):
  """fwn_walk_bitset: the pattern of adj ** power itself (the reference's `adj_mat ** attention_k_hop`) for a
  directed graph with a few self edges, duplicate entries and isolated rows; and on a mesh without self edges,
  where power 1 is the bare adjacency (no diagonal) and differs from the k-hop pattern."""
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  n = 777
  a = sparse.random(n, n, density=0.004, random_state=31, format="coo")
  a = sparse.coo_matrix((np.ones(a.nnz + 5), (np.r_[a.row, [3, 3, 9, 9, 40]], np.r_[a.col, [3, 3, 9, 500, 40]])),
                        shape=(n, n)).tocsr()
  xyz, faces = mesh.icosphere(3)
  m = mesh.adjacency(faces, xyz.shape[0]).astype(np.float64)
  m.setdiag(0)
  m.eliminate_zeros()
  for adj in (a, m):
    ip, ix = ta.power_csr_device(adj, power, cuda)
    got = sparse.csr_matrix((np.ones(ix.numel(), bool), ix.cpu().numpy(), ip.cpu().numpy()), shape=adj.shape)
    plain = sparse.csr_matrix(adj, dtype=np.float64)
    plain.data[:] = 1.0
    want = sparse.identity(adj.shape[0], format="csr")
    for _ in range(power):
      want = (want @ plain).tocsr()
      want.data[:] = 1.0
    assert _equal(got, want.astype(bool))
