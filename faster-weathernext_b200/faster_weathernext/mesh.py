"""Synthetic mesh masks for the benchmark configurations.

The configurations name an icosahedral mesh refined r times (10 * 4**r + 2 unit-sphere vertices),
ordered by the Morton code of (lat, lon), with pair (i, j) allowed iff the great-circle distance is
at most a radius (self pairs included). None of this is in the reference (its masks come from the
official `weathernext.utils.icosahedral_mesh`, which is not available here), so it is defined once,
deterministically, in this module:

* icosahedron: the 12 vertices (0, +-1, +-phi) and cyclic permutations, normalised; 20 faces.
* refinement: each triangle (a, b, c) -> 4 triangles over the normalised edge midpoints; a
  midpoint gets the next vertex id the first time its edge is met (faces visited in order).
* lat = asin(z), lon = atan2(y, x) in degrees, lon wrapped to [0, 360).
* Morton order: lat -> 16-bit round((lat + 90) / 180 * 65535), lon -> 16-bit
  floor(lon / 360 * 65536) clipped to 65535; code bit 2i = lon bit i, bit 2i+1 = lat bit i;
  stable argsort of the code.
* mask: dot(x_i, x_j) >= cos(radius), each dot computed as (x*x' + y*y') + z*z' with numpy
  elementwise float64 ops (no BLAS, no FMA), so the same mask comes out on every x86 host.

`k_hop_mask` builds the real WeatherNext 2 neighbourhood (adjacency of the finest mesh plus self
edges, raised to the k-th boolean power) by breadth-first search instead of a sparse matrix power.
"""

import hashlib

import numpy as np
from scipy import sparse
from scipy.spatial import cKDTree


def icosphere(level: int):
  """Unit-sphere vertices [n, 3] float64 and faces [f, 3] int64 of the icosahedron refined `level` times."""
  phi = (1.0 + 5.0 ** 0.5) / 2.0
  verts = [(-1, phi, 0), (1, phi, 0), (-1, -phi, 0), (1, -phi, 0),
           (0, -1, phi), (0, 1, phi), (0, -1, -phi), (0, 1, -phi),
           (phi, 0, -1), (phi, 0, 1), (-phi, 0, -1), (-phi, 0, 1)]
  faces = [(0, 11, 5), (0, 5, 1), (0, 1, 7), (0, 7, 10), (0, 10, 11),
           (1, 5, 9), (5, 11, 4), (11, 10, 2), (10, 7, 6), (7, 1, 8),
           (3, 9, 4), (3, 4, 2), (3, 2, 6), (3, 6, 8), (3, 8, 9),
           (4, 9, 5), (2, 4, 11), (6, 2, 10), (8, 6, 7), (9, 8, 1)]
  v = np.asarray(verts, np.float64)
  v = v / np.sqrt((v[:, 0] * v[:, 0] + v[:, 1] * v[:, 1]) + v[:, 2] * v[:, 2])[:, None]
  pts = [tuple(p) for p in v]
  f = list(faces)
  for _ in range(level):
    mid = {}
    out = []

    def midpoint(a, b):
      key = (a, b) if a < b else (b, a)
      idx = mid.get(key)
      if idx is None:
        pa, pb = pts[a], pts[b]
        m = np.array([(pa[0] + pb[0]) * 0.5, (pa[1] + pb[1]) * 0.5, (pa[2] + pb[2]) * 0.5])
        m = m / np.sqrt((m[0] * m[0] + m[1] * m[1]) + m[2] * m[2])
        idx = len(pts)
        pts.append(tuple(m))
        mid[key] = idx
      return idx

    for a, b, c in f:
      ab, bc, ca = midpoint(a, b), midpoint(b, c), midpoint(c, a)
      out += [(a, ab, ca), (b, bc, ab), (c, ca, bc), (ab, bc, ca)]
    f = out
  return np.asarray(pts, np.float64), np.asarray(f, np.int64)


def latlon(xyz):
  """Degrees (lat, lon) with lon in [0, 360)."""
  lat = np.degrees(np.arcsin(np.clip(xyz[:, 2], -1.0, 1.0)))
  lon = np.degrees(np.arctan2(xyz[:, 1], xyz[:, 0])) % 360.0
  return lat, lon


def _spread16(x):
  x = x.astype(np.uint64) & np.uint64(0xFFFF)
  x = (x | (x << np.uint64(8))) & np.uint64(0x00FF00FF)
  x = (x | (x << np.uint64(4))) & np.uint64(0x0F0F0F0F)
  x = (x | (x << np.uint64(2))) & np.uint64(0x33333333)
  x = (x | (x << np.uint64(1))) & np.uint64(0x55555555)
  return x


def morton_order(lat_deg, lon_deg) -> np.ndarray:
  """Permutation sorting points by the Morton code of (lat, lon) (bit layout in the module docstring)."""
  lat = np.asarray(lat_deg, np.float64)
  lon = np.asarray(lon_deg, np.float64)
  iy = np.clip(np.floor((lat + 90.0) / 180.0 * 65535.0 + 0.5), 0, 65535).astype(np.uint64)
  ix = np.clip(np.floor(lon / 360.0 * 65536.0), 0, 65535).astype(np.uint64)
  code = _spread16(ix) | (_spread16(iy) << np.uint64(1))
  return np.argsort(code, kind="stable")


def great_circle_mask(xyz, radius: float) -> sparse.csr_matrix:
  """Boolean CSR [n, n]: True iff the great-circle distance is <= radius (self included)."""
  n = xyz.shape[0]
  chord = 2.0 * np.sin(radius / 2.0) * (1.0 + 1e-9) + 1e-12
  pairs = cKDTree(xyz).query_pairs(chord, output_type="ndarray")
  i, j = pairs[:, 0], pairs[:, 1]
  a, b = xyz[i], xyz[j]
  dot = (a[:, 0] * b[:, 0] + a[:, 1] * b[:, 1]) + a[:, 2] * b[:, 2]
  keep = dot >= np.cos(radius)
  i, j = i[keep], j[keep]
  rows = np.concatenate([i, j, np.arange(n)])
  cols = np.concatenate([j, i, np.arange(n)])
  m = sparse.csr_matrix((np.ones(len(rows), bool), (rows, cols)), shape=(n, n))
  m.sum_duplicates()
  m.sort_indices()
  return m


def permute(mask: sparse.spmatrix, perm) -> sparse.csr_matrix:
  """mask'[i, j] = mask[perm[i], perm[j]] with sorted indices."""
  m = mask.tocsr()[perm][:, perm].tocsr()
  m.sort_indices()
  return m


def adjacency(faces, n) -> sparse.csr_matrix:
  """Symmetric mesh adjacency from triangle faces, self edges included."""
  e = np.concatenate([faces[:, [0, 1]], faces[:, [1, 2]], faces[:, [2, 0]]])
  rows = np.concatenate([e[:, 0], e[:, 1], np.arange(n)])
  cols = np.concatenate([e[:, 1], e[:, 0], np.arange(n)])
  m = sparse.csr_matrix((np.ones(len(rows), bool), (rows, cols)), shape=(n, n))
  m.sum_duplicates()
  m.sort_indices()
  return m


def k_hop_mask(adj: sparse.csr_matrix, k: int) -> sparse.csr_matrix:
  """Boolean (adj ** k) for an adjacency that includes self edges: all nodes within k hops."""
  adj = adj.tocsr().astype(np.int32)
  n = adj.shape[0]
  reach = sparse.identity(n, dtype=np.int32, format="csr")
  frontier = reach
  for _ in range(k):
    nxt = (frontier @ adj).tocsr()
    nxt.data[:] = 1
    new = (nxt - nxt.multiply(reach)).tocsr()   # nodes first reached at this hop
    new.eliminate_zeros()
    if new.nnz == 0:
      break
    reach = (reach + new).tocsr()
    frontier = new
  reach = reach.astype(bool).tocsr()
  reach.sort_indices()
  return reach


CONFIGS = {
    # cfg: (level, radius, batch, heads, head_dim)
    1: (3, 0.25, 1, 4, 64),
    2: (5, 0.12, 2, 8, 64),
    3: (6, 0.06, 1, 8, 64),
}


def config_mask(cfg: int):
  """(mask CSR in Morton order, lat, lon in Morton order) for benchmark configuration 1, 2 or 3."""
  level, radius = CONFIGS[cfg][:2]
  xyz, _ = icosphere(level)
  lat, lon = latlon(xyz)
  perm = morton_order(lat, lon)
  mask = great_circle_mask(xyz, radius)
  return permute(mask, perm), lat[perm], lon[perm]


# The real WeatherNext 2 attention shape: finest mesh (level 6), 32-hop neighbourhood, batch 1, 6 heads x 128.
WN2 = {"level": 6, "hops": 32, "batch": 1, "heads": 6, "head_dim": 128}


def wn2_adjacency(order: str = "hilbert"):
  """(adjacency CSR with self edges, lat, lon) of the level-6 mesh in Hilbert (GPU codes) or Morton order;
  its WN2["hops"]-hop mask is the attention mask (AttentionTiles.from_khop builds it on the device)."""
  xyz, faces = icosphere(WN2["level"])
  lat, lon = latlon(xyz)
  if order == "hilbert":
    from faster_weathernext import _hilbert
    perm = _hilbert.hilbert_order(lat, lon)
  elif order == "morton":
    perm = morton_order(lat, lon)
  else:
    raise ValueError(f"unknown order {order!r}")
  return permute(adjacency(faces, xyz.shape[0]), perm), lat[perm], lon[perm]


def csr_digest(m: sparse.csr_matrix) -> str:
  """sha256 over (shape, indptr int64, indices int64) of a CSR with sorted indices."""
  m = m.tocsr()
  m.sort_indices()
  h = hashlib.sha256()
  h.update(np.asarray(m.shape, np.int64).tobytes())
  h.update(np.asarray(m.indptr, np.int64).tobytes())
  h.update(np.asarray(m.indices, np.int64).tobytes())
  return h.hexdigest()
