"""Masked-softmax attention on the CPU (test infrastructure; see oracle/__init__.py).

Tensors use the reference's public layout [batch, n, heads, head_dim]; the mask is a boolean
[n, n] matrix with mask[query, key].

  ChunkedPath / chunked_attention / chunked_attention_vjp
                       — the reference's XLA attention path, patch.py:130-162 (per chunk of queries:
                         einsum over the chunk's key window * scale, where(mask, ., -1e30), softmax
                         upcast to float32, einsum with V) and its autodiff, in float32 or float64.
  sparse_attention     — the same masked softmax evaluated only on allowed pairs (masked pairs get
                         weight exp(-1e30 - max) == 0 exactly), float64, with the forward's
                         log-sum-exp lse = m + log(max(l, 1e-30)) (pallas_attn.py:138-140).
  sparse_attention_vjp — dQ, dK, dV of the masked softmax: dS = P * (dP - rowsum(dP * P))
                         (tests/test_pallas_kernel.py:58-69), float64.
  dense_attention(_vjp)— the float64 dense references of tests/test_pallas_kernel.py:15-21, 58-69.
  sampled_attention    — the same float64 forward and gradients on sampled query rows (out, lse, dq) and
                         key rows (dk, dv) of a large problem, computed block-wise with dense BLAS.
  rel_rms              — RMS(x - ref) / std(ref) (scripts/attn_bench.py:122).
"""

import numpy as np
from scipy import sparse

from oracle.tiles import build_chunked_mask

MASK_VALUE = -1e30


def rel_rms(x, ref) -> float:
  x = np.asarray(x, np.float64)
  ref = np.asarray(ref, np.float64)
  return float(np.sqrt(np.mean((x - ref) ** 2)) / ref.std())


def max_rel(x, ref) -> float:
  """max|x - ref| / max|ref| (the metric of tests/test_pallas_kernel.py:54)."""
  x = np.asarray(x, np.float64)
  ref = np.asarray(ref, np.float64)
  return float(np.abs(x - ref).max() / np.abs(ref).max())


def _softmax_lastaxis(x):
  m = x.max(-1, keepdims=True)
  e = np.exp(x - m)
  return e / e.sum(-1, keepdims=True)


class ChunkedPath:
  """The reference's XLA chunked attention path (patch.py:106-162) on the CPU, split into the layout
  step (pad to whole chunks / the key window, head-major copies; patch.py:137-142) and the per-chunk
  work (patch.py:144-152 and its autodiff), so a bounded sample of chunks can be timed."""

  def __init__(self, mask, chunk=512, dtype=np.float32):
    self.starts, self.packed, self.window, self.n_kv = build_chunked_mask(mask, chunk)
    self.chunk, self.dtype = chunk, dtype
    self.n = mask.shape[0]
    self.n_chunks = len(self.starts)

  def layout(self, q, k, v, do=None):
    b, n, h, d = q.shape
    def head_major(x, rows):
      out = np.zeros((b, h, rows, d), self.dtype)
      out[:, :, :n] = np.asarray(x, self.dtype).transpose(0, 2, 1, 3)
      return out
    rows_q = self.n_chunks * self.chunk
    t = {"q": head_major(q, rows_q), "k": head_major(k, self.n_kv), "v": head_major(v, self.n_kv)}
    if do is not None:
      t["do"] = head_major(do, rows_q)
    return t

  def _probs(self, t, c, scale, r0=0, r1=None):
    s0 = int(self.starts[c])
    rows = slice(c * self.chunk + r0, c * self.chunk + (self.chunk if r1 is None else r1))
    keys = slice(s0, s0 + self.window)
    qc, kc, vc = t["q"][:, :, rows], t["k"][:, :, keys], t["v"][:, :, keys]
    logits = np.matmul(qc, kc.transpose(0, 1, 3, 2)) * self.dtype(scale)
    m = np.unpackbits(self.packed[c], axis=-1, count=self.window, bitorder="little").astype(bool)
    m = m[r0:self.chunk if r1 is None else r1]
    logits = np.where(m[None, None], logits, self.dtype(MASK_VALUE))
    # wrap_fn_for_upcast_downcast: the softmax runs in float32 at least.
    p = _softmax_lastaxis(logits.astype(np.float32) if self.dtype != np.float64 else logits).astype(self.dtype)
    return rows, keys, p

  def forward_chunk(self, t, c, scale, out, r0=0, r1=None):
    """Chunk c (optionally only its query rows [r0, r1)): out[rows] = softmax(mask(q k^T)) v."""
    rows, keys, p = self._probs(t, c, scale, r0, r1)
    out[:, :, rows] = np.matmul(p, t["v"][:, :, keys])

  def vjp_chunk(self, t, c, scale, dq, dk, dv, r0=0, r1=None):
    """Autodiff of one chunk (or its rows [r0, r1)): dP = dO V^T, dS = P (dP - rowsum(dP P)), then dQ, dK, dV."""
    rows, keys, p = self._probs(t, c, scale, r0, r1)
    sc = self.dtype(scale)
    gc, qc = t["do"][:, :, rows], t["q"][:, :, rows]
    kc, vc = t["k"][:, :, keys], t["v"][:, :, keys]
    dp = np.matmul(gc, vc.transpose(0, 1, 3, 2))
    ds = p * (dp - (dp * p).sum(-1, keepdims=True))
    dq[:, :, rows] = np.matmul(ds, kc) * sc
    dk[:, :, keys] += np.matmul(ds.transpose(0, 1, 3, 2), qc) * sc
    dv[:, :, keys] += np.matmul(p.transpose(0, 1, 3, 2), gc)

  def back(self, x):
    return x[:, :, :self.n].transpose(0, 2, 1, 3)


def chunked_attention(q, k, v, mask, scale, chunk=512, dtype=np.float32, chunks=None):
  """The XLA chunked path's forward (patch.py:130-162). Returns [B, n, H, D] in `dtype`;
  `chunks` evaluates only those query chunks (rows of other chunks stay zero)."""
  path = ChunkedPath(mask, chunk, dtype)
  t = path.layout(q, k, v)
  out = np.zeros_like(t["q"])
  for c in (range(path.n_chunks) if chunks is None else chunks):
    path.forward_chunk(t, c, scale, out)
  return path.back(out)


def chunked_attention_vjp(q, k, v, do, mask, scale, chunk=512, dtype=np.float32, chunks=None):
  """dQ, dK, dV of the XLA chunked path (JAX autodiff of patch.py:144-159). Returns [B, n, H, D] arrays."""
  path = ChunkedPath(mask, chunk, dtype)
  t = path.layout(q, k, v, do)
  dq, dk, dv = np.zeros_like(t["q"]), np.zeros_like(t["k"]), np.zeros_like(t["v"])
  for c in (range(path.n_chunks) if chunks is None else chunks):
    path.vjp_chunk(t, c, scale, dq, dk, dv)
  return path.back(dq), path.back(dk), path.back(dv)


def _pairs(mask):
  m = sparse.csr_matrix(mask).astype(bool).tocsr()
  m.sum_duplicates()
  m.sort_indices()
  rows = np.repeat(np.arange(m.shape[0], dtype=np.int64), np.diff(m.indptr))
  return m, rows, m.indices.astype(np.int64)


def _row_blocks(indptr, max_pairs):
  """Split rows into contiguous ranges with at most ~max_pairs allowed pairs each."""
  n = len(indptr) - 1
  r0 = 0
  while r0 < n:
    target = indptr[r0] + max_pairs
    r1 = int(np.searchsorted(indptr, target, side="right")) - 1
    r1 = max(r1, r0 + 1)
    yield r0, min(r1, n)
    r0 = min(r1, n)


def sparse_attention(q, k, v, mask, scale, max_pairs=1 << 21):
  """float64 masked softmax attention on allowed pairs. Returns (out [B,n,H,D], lse [B,H,n])."""
  m, rows_all, cols_all = _pairs(mask)
  b, n, h, d = q.shape
  out = np.zeros((b, n, h, d))
  lse = np.zeros((b, h, n))
  for bi in range(b):
    for hi in range(h):
      qq = np.asarray(q[bi, :, hi], np.float64)
      kk = np.asarray(k[bi, :, hi], np.float64)
      vv = np.asarray(v[bi, :, hi], np.float64)
      for r0, r1 in _row_blocks(m.indptr, max_pairs):
        e0, e1 = m.indptr[r0], m.indptr[r1]
        if e1 == e0:
          continue
        rows, cols = rows_all[e0:e1], cols_all[e0:e1]
        s = np.einsum("ed,ed->e", qq[rows], kk[cols]) * scale
        seg = m.indptr[r0:r1] - e0
        nonempty = np.diff(m.indptr[r0:r1 + 1]) > 0
        mx = np.full(r1 - r0, -np.inf)
        mx[nonempty] = np.maximum.reduceat(s, seg[nonempty])
        p = np.exp(s - mx[rows - r0])
        l = np.zeros(r1 - r0)
        l[nonempty] = np.add.reduceat(p, seg[nonempty])
        pm = sparse.csr_matrix((p, cols, m.indptr[r0:r1 + 1] - e0), shape=(r1 - r0, n))
        out[bi, r0:r1, hi] = (pm @ vv) / np.maximum(l, 1e-30)[:, None]
        lse[bi, hi, r0:r1] = mx + np.log(np.maximum(l, 1e-30))
  return out, lse


def sparse_attention_vjp(q, k, v, do, mask, scale, max_pairs=1 << 21):
  """float64 (dq, dk, dv) of masked softmax attention, each [B, n, H, D]."""
  m, rows_all, cols_all = _pairs(mask)
  b, n, h, d = q.shape
  dq = np.zeros((b, n, h, d))
  dk = np.zeros((b, n, h, d))
  dv = np.zeros((b, n, h, d))
  for bi in range(b):
    for hi in range(h):
      qq = np.asarray(q[bi, :, hi], np.float64)
      kk = np.asarray(k[bi, :, hi], np.float64)
      vv = np.asarray(v[bi, :, hi], np.float64)
      gg = np.asarray(do[bi, :, hi], np.float64)
      for r0, r1 in _row_blocks(m.indptr, max_pairs):
        e0, e1 = m.indptr[r0], m.indptr[r1]
        if e1 == e0:
          continue
        rows, cols = rows_all[e0:e1], cols_all[e0:e1]
        s = np.einsum("ed,ed->e", qq[rows], kk[cols]) * scale
        seg = m.indptr[r0:r1] - e0
        nonempty = np.diff(m.indptr[r0:r1 + 1]) > 0
        mx = np.full(r1 - r0, -np.inf)
        mx[nonempty] = np.maximum.reduceat(s, seg[nonempty])
        p = np.exp(s - mx[rows - r0])
        l = np.zeros(r1 - r0)
        l[nonempty] = np.add.reduceat(p, seg[nonempty])
        p = p / l[rows - r0]
        dp = np.einsum("ed,ed->e", gg[rows], vv[cols])
        delta = np.zeros(r1 - r0)
        delta[nonempty] = np.add.reduceat(p * dp, seg[nonempty])
        ds = p * (dp - delta[rows - r0])
        indptr = m.indptr[r0:r1 + 1] - e0
        dsm = sparse.csr_matrix((ds, cols, indptr), shape=(r1 - r0, n))
        pm = sparse.csr_matrix((p, cols, indptr), shape=(r1 - r0, n))
        dq[bi, r0:r1, hi] = (dsm @ kk) * scale
        dk[bi, :, hi] += (dsm.T @ qq[r0:r1]) * scale
        dv[bi, :, hi] += pm.T @ gg[r0:r1]
  return dq, dk, dv


def sampled_attention(q, k, v, do, mask, scale, q_rows, k_rows, block=128):
  """float64 out, lse, dq at query rows `q_rows` and dk, dv at key rows `k_rows` of one batch element.

  q, k, v, do: [n, H, D]; mask: [n, n] CSR (mask[query, key]). The math is sparse_attention /
  sparse_attention_vjp's (P = softmax of the allowed logits, dS = P (dP - rowsum(P dP)), dQ = scale dS K,
  dK = scale dS^T Q, dV = P^T dO), evaluated only where needed: every query row that attends to a sampled key
  gets its full row statistics, so the sampled dk / dv are exact sums over all their queries. Rows are taken
  in groups of `block` (ascending), each against the dense union of its keys.
  Returns dict(out [Rq, H, D], lse [H, Rq], dq [Rq, H, D], dk [Rk, H, D], dv [Rk, H, D]) in the order given."""
  m = sparse.csr_matrix(mask).astype(bool).tocsr()
  m.sum_duplicates()
  m.sort_indices()
  n, h, d = q.shape
  q_rows = np.asarray(q_rows, np.int64)
  k_rows = np.asarray(k_rows, np.int64)
  mt = m.T.tocsr()
  users = np.unique(mt[k_rows].indices) if len(k_rows) else np.zeros(0, np.int64)
  rows = np.union1d(q_rows, users)
  k_slot = np.full(n, -1, np.int64)
  k_slot[k_rows] = np.arange(len(k_rows))
  q_slot = np.full(n, -1, np.int64)
  q_slot[q_rows] = np.arange(len(q_rows))
  f = lambda x: np.asarray(x, np.float64)
  out = np.zeros((len(q_rows), h, d))
  lse = np.zeros((h, len(q_rows)))
  dq = np.zeros((len(q_rows), h, d))
  dk = np.zeros((len(k_rows), h, d))
  dv = np.zeros((len(k_rows), h, d))
  for c0 in range(0, len(rows), block):
    rc = rows[c0:c0 + block]
    sub = m[rc]
    keys = np.unique(sub.indices)
    if keys.size == 0:
      continue
    pos = np.searchsorted(keys, sub.indices)
    allowed = np.zeros((len(rc), len(keys)), bool)
    allowed[np.repeat(np.arange(len(rc)), np.diff(sub.indptr)), pos] = True
    qh, gh = f(q[rc]).transpose(1, 0, 2), f(do[rc]).transpose(1, 0, 2)             # [H, r, D]
    kh, vh = f(k[keys]).transpose(1, 0, 2), f(v[keys]).transpose(1, 0, 2)           # [H, c, D]
    s = np.where(allowed[None], np.matmul(qh, kh.transpose(0, 2, 1)) * scale, -np.inf)
    mx = s.max(-1, keepdims=True)
    mx = np.where(np.isfinite(mx), mx, 0.0)
    p = np.exp(s - mx)
    l = p.sum(-1, keepdims=True)
    p = p / np.maximum(l, 1e-300)
    o = np.matmul(p, vh)
    dp = np.matmul(gh, vh.transpose(0, 2, 1))
    ds = p * (dp - (p * dp).sum(-1, keepdims=True))
    sel = q_slot[rc] >= 0
    if sel.any():
      dst = q_slot[rc][sel]
      out[dst] = o[:, sel].transpose(1, 0, 2)
      lse[:, dst] = (mx + np.log(np.maximum(l, 1e-300)))[:, sel, 0]
      dq[dst] = (np.matmul(ds[:, sel], kh) * scale).transpose(1, 0, 2)
    kc = k_slot[keys] >= 0
    if kc.any():
      dst = k_slot[keys][kc]
      dk[dst] += (np.matmul(ds[:, :, kc].transpose(0, 2, 1), qh) * scale).transpose(1, 0, 2)
      dv[dst] += np.matmul(p[:, :, kc].transpose(0, 2, 1), gh).transpose(1, 0, 2)
  return {"out": out, "lse": lse, "dq": dq, "dk": dk, "dv": dv}


def dense_attention(q, k, v, mask, scale):
  """float64 dense masked softmax for one batch element, q/k/v [n, H, D] (test_pallas_kernel.py:15-21)."""
  s = np.einsum("nhd,mhd->hnm", q.astype(np.float64), k.astype(np.float64)) * scale
  s = np.where(mask[None], s, -np.inf)
  p = np.exp(s - s.max(-1, keepdims=True))
  p /= p.sum(-1, keepdims=True)
  return np.einsum("hnm,mhd->nhd", p, v.astype(np.float64))


def dense_attention_vjp(q, k, v, do, mask, scale):
  """float64 dQ, dK, dV for one batch element (test_pallas_kernel.py:58-69)."""
  q, k, v, do = (x.astype(np.float64) for x in (q, k, v, do))
  s = np.where(mask[None], np.einsum("nhd,mhd->hnm", q, k) * scale, -np.inf)
  p = np.exp(s - s.max(-1, keepdims=True))
  p /= p.sum(-1, keepdims=True)
  dp = np.einsum("nhd,mhd->hnm", do, v)
  ds = p * (dp - (dp * p).sum(-1, keepdims=True))
  dq = np.einsum("hnm,mhd->nhd", ds, k) * scale
  dk = np.einsum("hnm,nhd->mhd", ds, q) * scale
  dv = np.einsum("hnm,nhd->mhd", p, do)
  return dq, dk, dv


def bf16_round(x):
  """Round float32/float64 values to bfloat16 (round to nearest even), returned as float32."""
  a = np.ascontiguousarray(np.asarray(x, np.float32))
  u = a.view(np.uint32).astype(np.uint64)
  r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
  return r.astype(np.uint32).view(np.float32).reshape(a.shape)
