"""Tile lists, node orderings and chunked masks on the CPU (test infrastructure; see oracle/__init__.py).

Restates:
  build_tile_mask      — src/faster_weathernext/pallas_attn.py:85-109
  hilbert_order        — src/faster_weathernext/pallas_attn.py:41-82 (Skilling, "Programming the
                         Hilbert curve", AIP Conf. Proc. 707 (2004): axes -> transpose, Gray code)
  build_chunked_mask   — src/faster_weathernext/patch.py:106-127
"""

import numpy as np
from scipy import sparse

BLOCK_Q = 64
BLOCK_K = 32


def _coo(mask):
  m = sparse.csr_matrix(mask).astype(bool)
  m.eliminate_zeros()
  rows = np.repeat(np.arange(m.shape[0], dtype=np.int64), np.diff(m.indptr))
  return rows, m.indices.astype(np.int64), m.shape


def build_tile_mask(mask, block_q: int = BLOCK_Q, block_k: int = BLOCK_K):
  """(tile_ptr int32[nqb+1], tile_kb int32[T], tile_bits uint32[T, block_q]) of a boolean [n, m] mask.

  Same contract as pallas_attn.py:85-109: tiles of a query block are the distinct key blocks that
  hold at least one allowed pair, in ascending key-block order; bit j of tile_bits[t, r] is
  mask[qb*block_q + r, tile_kb[t]*block_k + j].
  """
  assert block_k == 32, "one uint32 word per query row per tile"
  rows, cols, (n, m) = _coo(mask)
  nqb = -(-n // block_q)
  nkb = -(-m // block_k)
  key = (rows // block_q) * nkb + cols // block_k
  order = np.argsort(key, kind="stable")
  key_s = key[order]
  first = np.ones(len(key_s), bool)
  first[1:] = key_s[1:] != key_s[:-1]
  tile_of = np.cumsum(first) - 1
  uniq = key_s[first]
  words = np.zeros(len(uniq) * block_q, np.uint32)
  np.bitwise_or.at(words, tile_of * block_q + rows[order] % block_q,
                   np.left_shift(np.uint32(1), (cols[order] % block_k).astype(np.uint32)))
  tile_qb = uniq // nkb
  ptr = np.searchsorted(tile_qb, np.arange(nqb + 1), side="left")
  return ptr.astype(np.int32), (uniq % nkb).astype(np.int32), words.reshape(len(uniq), block_q)


def pair_tiles(ptr, kb, bits):
  """Derive the 128-row list the CUDA kernels walk from a 64-row list.

  Block p covers the reference's query blocks 2p and 2p+1. Its tiles are the sorted union of their
  key blocks; rows 0-63 of a paired tile carry block 2p's mask words (0 where 2p lacks that key
  block), rows 64-127 block 2p+1's. Returns (ptr2 int32[np+1], kb2 int32[T2], bits2 uint32[T2, 128]).
  """
  ptr = np.asarray(ptr, np.int64)
  kb = np.asarray(kb, np.int64)
  bits = np.asarray(bits, np.uint32)
  nqb = len(ptr) - 1
  npb = (nqb + 1) // 2
  qb = np.repeat(np.arange(nqb), np.diff(ptr))
  big = int(kb.max()) + 1 if len(kb) else 1
  key = (qb // 2) * big + kb
  uniq, inv = np.unique(key, return_inverse=True)
  bits2 = np.zeros((len(uniq), 128), np.uint32)
  half = (qb % 2) * 64
  for r in range(64):
    bits2[inv, half + r] = bits[:, r]
  pb = uniq // big
  ptr2 = np.searchsorted(pb, np.arange(npb + 1), side="left")
  return ptr2.astype(np.int32), (uniq % big).astype(np.int32), bits2


def gather_tiles(ptr2, kb2, bits2):
  """Gathered list derived from a 128-row (paired) list: per block, the distinct columns any of its rows
  may attend to, ascending, packed into tiles of 32 slots (the last tile padded with its last column,
  whose padding slots carry no bits). Returns (ptr_g int32[np+1], cols int32[Tg, 32], bits uint32[Tg, 128]);
  bit j of bits[t, r] allows (row r of the block, column cols[t, j])."""
  ptr2 = np.asarray(ptr2, np.int64)
  kb2 = np.asarray(kb2, np.int64)
  bits2 = np.asarray(bits2, np.uint32)
  npb = len(ptr2) - 1
  colmask = np.bitwise_or.reduce(bits2, axis=1) if len(bits2) else np.zeros(0, np.uint32)
  ptr_g = np.zeros(npb + 1, np.int64)
  cols_out, bits_out = [], []
  j = np.arange(32, dtype=np.uint32)
  for p in range(npb):
    e0, e1 = ptr2[p], ptr2[p + 1]
    used = ((colmask[e0:e1, None] >> j) & 1).astype(bool)            # [tiles, 32]
    keys = (kb2[e0:e1, None] * 32 + j.astype(np.int64))[used]          # ascending
    slot_of = np.full((e1 - e0, 32), -1, np.int64)
    slot_of[used] = np.arange(len(keys))
    ng = -(-len(keys) // 32)
    cols = np.full(ng * 32, keys[-1] if len(keys) else 0, np.int64)
    cols[:len(keys)] = keys
    words = np.zeros((ng, 128), np.uint32)
    for e in range(e1 - e0):
      w = bits2[e0 + e]                                                # [128]
      hit = ((w[:, None] >> j) & 1).astype(bool)                       # [128, 32]
      rr, jj = np.nonzero(hit)
      s = slot_of[e, jj]
      np.bitwise_or.at(words, (s // 32, rr), np.left_shift(np.uint32(1), (s % 32).astype(np.uint32)))
    cols_out.append(cols.reshape(ng, 32))
    bits_out.append(words)
    ptr_g[p + 1] = ptr_g[p] + ng
  cols = np.concatenate(cols_out) if cols_out else np.zeros((0, 32), np.int64)
  bits = np.concatenate(bits_out) if bits_out else np.zeros((0, 128), np.uint32)
  return ptr_g.astype(np.int32), cols.astype(np.int32), bits


def gathered_to_dense(ptr_g, cols, bits, n_rows, n_cols, block_q=128):
  dense = np.zeros((n_rows, n_cols), bool)
  j = np.arange(32, dtype=np.uint32)
  for p in range(len(ptr_g) - 1):
    for t in range(ptr_g[p], ptr_g[p + 1]):
      hit = ((np.asarray(bits[t], np.uint32)[:, None] >> j) & 1).astype(bool)
      for r, jj in zip(*np.nonzero(hit)):
        if p * block_q + r < n_rows:
          dense[p * block_q + r, cols[t, jj]] = True
  return dense


def tiles_to_dense(ptr, kb, bits, n_rows, n_cols, block_q=BLOCK_Q, block_k=BLOCK_K):
  """Inverse of build_tile_mask: the boolean [n_rows, n_cols] mask the list describes."""
  nqb = len(ptr) - 1
  width = (int(np.max(kb)) + 1 if len(kb) else 1) * block_k
  dense = np.zeros((nqb * block_q, max(width, n_cols)), bool)
  j = np.arange(block_k, dtype=np.uint32)
  for q in range(nqb):
    for t in range(ptr[q], ptr[q + 1]):
      w = np.asarray(bits[t], np.uint32)
      dense[q * block_q:(q + 1) * block_q, kb[t] * block_k:(kb[t] + 1) * block_k] = ((w[:, None] >> j) & 1) == 1
  return dense[:n_rows, :n_cols]


def _hilbert_index(ints: np.ndarray, bits: int) -> np.ndarray:
  """Hilbert-curve index of n points with 3 coordinates in [0, 2**bits) (Skilling 2004)."""
  x = [ints[:, a].astype(np.int64) for a in range(3)]
  top = 1 << (bits - 1)
  # Axes -> transpose: undo excess work, walking the bit planes from the top.
  q = top
  while q > 1:
    low = q - 1
    for a in range(3):
      set_ = (x[a] & q) != 0
      flip = np.where(set_, low, 0)                    # invert the low bits of x[0]
      swap = np.where(set_, 0, (x[0] ^ x[a]) & low)    # or exchange low bits of x[0] and x[a]
      x[0] = x[0] ^ flip ^ swap
      x[a] = x[a] ^ swap
    q >>= 1
  # Gray encode.
  x[1] = x[1] ^ x[0]
  x[2] = x[2] ^ x[1]
  acc = np.zeros_like(x[0])
  q = top
  while q > 1:
    acc = np.where((x[2] & q) != 0, acc ^ (q - 1), acc)
    q >>= 1
  x = [c ^ acc for c in x]
  # Interleave the transposed bits, most significant plane first, axis 0 first.
  code = np.zeros_like(x[0])
  for b in range(bits - 1, -1, -1):
    for a in range(3):
      code = (code << 1) | ((x[a] >> b) & 1)
  return code


def hilbert_order(lat_deg, lon_deg, bits: int = 10) -> np.ndarray:
  """Permutation along the 3D Hilbert curve of the unit-sphere points (non-finite points last)."""
  lat = np.radians(np.asarray(lat_deg, np.float64).ravel())
  lon = np.radians(np.asarray(lon_deg, np.float64).ravel())
  xyz = np.stack([np.cos(lat) * np.cos(lon), np.cos(lat) * np.sin(lon), np.sin(lat)], axis=1)
  finite = np.isfinite(xyz).all(axis=1)
  scale = (1 << bits) - 1
  ints = np.clip(np.round((np.nan_to_num(xyz) + 1.0) / 2.0 * scale), 0, scale).astype(np.int64)
  code = np.where(finite, _hilbert_index(ints, bits), np.iinfo(np.int64).max)
  return np.argsort(code, kind="stable")


def build_chunked_mask(mask, chunk: int):
  """(starts int32[nc], packed uint8[nc, chunk, W/8], W, n_kv) — the XLA path's banded windows.

  Per chunk of `chunk` query rows: one key window of W keys (W = the largest span over all chunks,
  rounded up to 128), starting at the chunk's smallest key (clamped to n_kv - W); the mask inside
  the window bit-packed little-endian.
  """
  m = sparse.csr_matrix(mask).astype(bool).tocsr()
  m.sort_indices()
  n = m.shape[0]
  nc = -(-n // chunk)
  counts = np.diff(m.indptr)
  assert (counts > 0).all(), "every row needs at least one allowed key"
  lo = m.indices[m.indptr[:-1]]
  hi = m.indices[m.indptr[1:] - 1]
  span = 0
  for c in range(nc):
    r0, r1 = c * chunk, min((c + 1) * chunk, n)
    span = max(span, int(hi[r0:r1].max() - lo[r0:r1].min() + 1))
  window = -(-span // 128) * 128
  n_kv = max(n, window)
  starts = np.zeros(nc, np.int32)
  packed = np.zeros((nc, chunk, window // 8), np.uint8)
  for c in range(nc):
    r0, r1 = c * chunk, min((c + 1) * chunk, n)
    s = min(int(lo[r0:r1].min()), n_kv - window)
    starts[c] = s
    blk = np.zeros((r1 - r0, window), bool)
    rr = np.repeat(np.arange(r1 - r0), counts[r0:r1])
    cc = m.indices[m.indptr[r0]:m.indptr[r1]] - s
    assert (cc >= 0).all() and (cc < window).all(), f"chunk {c} window too narrow"
    blk[rr, cc] = True
    packed[c, :r1 - r0] = np.packbits(blk, axis=-1, bitorder="little")
  return starts, packed, window, n_kv
