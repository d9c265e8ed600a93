"""Block-sparse masked flash attention on B200, the drop-in for faster_weathernext.pallas_attn.

Public API (names and argument meanings follow src/faster_weathernext/pallas_attn.py):

  build_tile_mask(mask, block_q=64, block_k=32)  pallas_attn.py:85-109, computed by the CUDA builder;
                                                 returns NumPy (tile_ptr int32, tile_kb int32, tile_bits uint32)
  hilbert_order(lat_deg, lon_deg, bits=10)       pallas_attn.py:71-82 (host, NumPy)
  tiled_flash_attention(q, k, v, tile_ptr, tile_kb, tile_bits, *, scale, strict_fp32=False, tiles_t=None, ...)
                                                 pallas_attn.py:317-354; differentiable (torch.autograd),
                                                 the analogue of the reference's jax.custom_vjp

Device-side building blocks (torch tensors on the current CUDA device):

  build_tiles_device(indptr, indices, n_rows, n_cols)     -> TileList64 (64-row list, bit-exact with the reference)
  pair_tiles(tiles64)                                     -> TileList128 (what the kernels walk)
  AttentionTiles.from_mask(mask) / .from_lists(...)       -> forward + transposed paired lists, cached
  attention_forward(q, k, v, tiles, scale, mode, with_lse) / attention_backward(...)

Precision (pallas_attn.py:336-342): bf16 tensors run in bf16. float32 tensors follow the matmul precision in
force — `precision=` of the call, else the innermost `default_matmul_precision(...)` block, the analogue of
`jax.default_matmul_precision`: "highest" / "float32" run 3xTF32 (the reference's TF32_TF32_F32_X3), anything
else TF32 (TF32_TF32_F32, the reference's default). `strict_fp32=True` matters only under "highest", where the
reference switches to IEEE float32 dots (F32_F32_F32); those have no tensor-core form and are not built here,
so that combination raises NotImplementedError instead of silently running 3xTF32.

Head sizes: the kernels are built for head_dim 64 and 128; other sizes up to 128 are zero-padded to the next
of the two inside the op (padded q / k columns add 0 to every logit, padded v columns give 0 outputs that are
sliced off), which costs one copy of q, k, v.
"""

import contextlib
import ctypes
import dataclasses
import threading
from typing import Optional

import numpy as np
import torch
from scipy import sparse

from faster_weathernext import _lib
from faster_weathernext._hilbert import hilbert_order  # noqa: F401  (re-exported)

BLOCK_Q = 64
BLOCK_K = 32
MASK_VALUE = -1e30


def _stream() -> int:
  return torch.cuda.current_stream().cuda_stream


def _device(device=None) -> torch.device:
  if device is None:
    if not torch.cuda.is_available():
      raise RuntimeError("faster_weathernext attention needs a CUDA device (sm_100a); none is available")
    return torch.device("cuda", torch.cuda.current_device())
  return torch.device(device)


@dataclasses.dataclass
class TileList64:
  """A build_tile_mask list on the device: ptr [nqb+1], kb [T], bits [T, 64] (int32 storage of uint32)."""
  ptr: torch.Tensor
  kb: torch.Tensor
  bits: torch.Tensor
  n_rows: int
  n_cols: int

  @property
  def n_blocks(self):
    return self.ptr.numel() - 1

  @property
  def n_tiles(self):
    return self.kb.numel()

  def struct(self) -> _lib.TileList:
    return _lib.TileList(self.ptr.data_ptr(), self.kb.data_ptr() if self.n_tiles else 0,
                         self.bits.data_ptr() if self.n_tiles else 0, self.n_blocks, self.n_tiles, 64, self.n_cols, 0)

  def numpy(self):
    """(tile_ptr int32, tile_kb int32, tile_bits uint32 [T, 64]) — the reference's return types."""
    return (self.ptr.cpu().numpy(), self.kb.cpu().numpy(),
            self.bits.cpu().numpy().view(np.uint32).reshape(-1, 64))


@dataclasses.dataclass
class TileList128:
  """128-row list the attention kernels walk: paired (kb: key block of each tile) or gathered
  (cols: the column of each of a tile's 32 slots)."""
  ptr: torch.Tensor
  kb: torch.Tensor
  bits: torch.Tensor
  n_cols: int
  cols: Optional[torch.Tensor] = None

  @property
  def n_blocks(self):
    return self.ptr.numel() - 1

  @property
  def n_tiles(self):
    return self.bits.shape[0]

  def struct(self) -> _lib.TileList:
    n = self.n_tiles
    return _lib.TileList(self.ptr.data_ptr(), self.kb.data_ptr() if n and self.kb.numel() else 0,
                         self.bits.data_ptr() if n else 0, self.n_blocks, n, 128, self.n_cols,
                         self.cols.data_ptr() if (self.cols is not None and n) else 0)

  def numpy(self):
    second = self.cols.cpu().numpy().reshape(-1, 32) if self.cols is not None else self.kb.cpu().numpy()
    return (self.ptr.cpu().numpy(), second, self.bits.cpu().numpy().view(np.uint32).reshape(-1, 128))


def _read_last(ptr: torch.Tensor) -> int:
  return int(ptr[-1].item())


def build_tiles_device(indptr: torch.Tensor, indices: torch.Tensor, n_rows: int, n_cols: int,
                       block_q: int = BLOCK_Q) -> TileList64:
  """CUDA tile-list builder over a device CSR (int32 indptr [n_rows+1], indices [nnz])."""
  lib = _lib.lib()
  dev = indptr.device
  indptr = indptr.to(torch.int32).contiguous()
  indices = indices.to(torch.int32).contiguous()
  nqb = -(-n_rows // block_q)
  ws_bytes = ctypes.c_size_t(0)
  _lib.check(lib.fwn_tiles_workspace_size(n_rows, n_cols, block_q, ctypes.byref(ws_bytes)))
  ws = torch.empty(ws_bytes.value, dtype=torch.uint8, device=dev)
  ptr = torch.empty(nqb + 1, dtype=torch.int32, device=dev)
  s = _stream()
  _lib.check(lib.fwn_tiles_count(indptr.data_ptr(), indices.data_ptr() if indices.numel() else 0, n_rows, n_cols,
                                 block_q, ptr.data_ptr(), ws.data_ptr(), ws_bytes.value, s))
  n_tiles = _read_last(ptr)
  kb = torch.empty(max(n_tiles, 1), dtype=torch.int32, device=dev)[:n_tiles]
  bits = torch.empty(max(n_tiles, 1) * block_q, dtype=torch.int32, device=dev)[:n_tiles * block_q]
  if n_tiles:
    _lib.check(lib.fwn_tiles_fill(indptr.data_ptr(), indices.data_ptr(), n_rows, n_cols, block_q, ptr.data_ptr(),
                                  kb.data_ptr(), bits.data_ptr(), s))
  return TileList64(ptr, kb, bits.view(n_tiles, block_q), n_rows, n_cols)


def _bitset_csr_device(adj, steps: int, device, include_self: bool):
  lib = _lib.lib()
  dev = _device(device)
  a = sparse.csr_matrix(adj).astype(bool)
  a.eliminate_zeros()
  n = a.shape[0]
  assert a.shape == (n, n), "adjacency must be square"
  ip, ix, _ = _csr_to_device(a, dev)
  words = lib.fwn_bitset_words(n)
  reach = torch.empty(n * words, dtype=torch.int32, device=dev)
  scratch = torch.empty(n * words, dtype=torch.int32, device=dev)
  s = _stream()
  fn = lib.fwn_khop_bitset if include_self else lib.fwn_walk_bitset
  _lib.check(fn(ip.data_ptr(), ix.data_ptr() if ix.numel() else 0, n, steps, reach.data_ptr(), scratch.data_ptr(), s))
  del scratch
  indptr = torch.empty(n + 1, dtype=torch.int32, device=dev)
  ws = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
  _lib.check(lib.fwn_bitset_csr_count(reach.data_ptr(), n, n, indptr.data_ptr(), ws.data_ptr(), ws.numel() * 4, s))
  nnz = _read_last(indptr)
  indices = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)[:nnz]
  _lib.check(lib.fwn_bitset_csr_fill(reach.data_ptr(), n, n, indptr.data_ptr(), indices.data_ptr(), s))
  return indptr, indices


def khop_csr_device(adj, hops: int, device=None):
  """Device CSR (int32 indptr [n+1], indices [nnz], ascending) of every node within `hops` edges of each
  node, self included: the pattern of (adj + I) ** hops, built on the GPU (bitset k-hop kernels)."""
  return _bitset_csr_device(adj, hops, device, True)


def power_csr_device(adj, power: int, device=None):
  """Device CSR of the nonzero pattern of adj ** power (walks of exactly `power` edges; self edges only where
  adj has them): the reference's `adj_mat ** attention_k_hop` (patch.py:209), built on the GPU."""
  return _bitset_csr_device(adj, power, device, False)


def pair_tiles(t: TileList64) -> TileList128:
  """128-row list derived from a 64-row list (union of the two blocks' key tiles)."""
  lib = _lib.lib()
  dev = t.ptr.device
  npb = (t.n_blocks + 1) // 2
  st = t.struct()
  ws = torch.empty(npb * 4 + 512, dtype=torch.uint8, device=dev)
  ptr2 = torch.empty(npb + 1, dtype=torch.int32, device=dev)
  s = _stream()
  _lib.check(lib.fwn_tiles_pair_count(ctypes.byref(st), ptr2.data_ptr(), ws.data_ptr(), ws.numel(), s))
  n2 = _read_last(ptr2)
  kb2 = torch.empty(max(n2, 1), dtype=torch.int32, device=dev)[:n2]
  bits2 = torch.empty(max(n2, 1) * 128, dtype=torch.int32, device=dev)[:n2 * 128]
  if n2:
    _lib.check(lib.fwn_tiles_pair_fill(ctypes.byref(st), ptr2.data_ptr(), kb2.data_ptr(), bits2.data_ptr(), s))
  return TileList128(ptr2, kb2, bits2.view(n2, 128), t.n_cols)


def gather_tiles(t: TileList128) -> TileList128:
  """Gathered list from a paired list: each block's distinct columns packed into 32-slot tiles."""
  lib = _lib.lib()
  dev = t.ptr.device
  st = t.struct()
  ws = torch.empty(t.n_blocks * 4 + 512, dtype=torch.uint8, device=dev)
  ptr_g = torch.empty(t.n_blocks + 1, dtype=torch.int32, device=dev)
  s = _stream()
  _lib.check(lib.fwn_tiles_gather_count(ctypes.byref(st), ptr_g.data_ptr(), ws.data_ptr(), ws.numel(), s))
  ng = _read_last(ptr_g)
  max_block = int(torch.diff(t.ptr).max().item()) if t.n_blocks else 0
  cols = torch.empty(max(ng, 1) * 32, dtype=torch.int32, device=dev)[:ng * 32]
  bits = torch.empty(max(ng, 1) * 128, dtype=torch.int32, device=dev)[:ng * 128]
  if ng:
    _lib.check(lib.fwn_tiles_gather_fill(ctypes.byref(st), max_block, ptr_g.data_ptr(), cols.data_ptr(),
                                         bits.data_ptr(), s))
  empty = torch.empty(0, dtype=torch.int32, device=dev)
  return TileList128(ptr_g, empty, bits.view(ng, 128), t.n_cols, cols)


def _csr_to_device(mask, device):
  m = sparse.csr_matrix(mask)
  m.sum_duplicates()
  indptr = torch.from_numpy(np.asarray(m.indptr, np.int32)).to(device)
  indices = torch.from_numpy(np.asarray(m.indices, np.int32)).to(device)
  return indptr, indices, m.shape


def build_tile_mask(mask, block_q: int = BLOCK_Q, block_k: int = BLOCK_K, device=None):
  """Drop-in for pallas_attn.build_tile_mask: NumPy (tile_ptr, tile_kb, tile_bits) built on the GPU."""
  assert block_k == 32, "one uint32 mask word per query row per tile"
  if block_q != 64:
    raise ValueError("the reference's tile lists use 64-row query blocks")
  dev = _device(device)
  m = sparse.csr_matrix(mask).astype(bool)
  m.eliminate_zeros()
  indptr, indices, (n_rows, n_cols) = _csr_to_device(m, dev)
  return build_tiles_device(indptr, indices, n_rows, n_cols, block_q).numpy()


def _check_lists(tile_ptr, tile_kb, tile_bits, n, what):
  """Shape checks of a reference-format triple for an n-node mask (what pallas_attn.py:317-354 relies on:
  ceil(n / 64) query blocks, key blocks below ceil(n / 32), one 64-word row set per tile)."""
  ptr, kb, bits = (np.asarray(x) for x in (tile_ptr, tile_kb, tile_bits))
  nqb = -(-n // BLOCK_Q)
  if ptr.ndim != 1 or ptr.size != nqb + 1:
    raise ValueError(f"{what}: tile_ptr has {ptr.size} entries, expected ceil({n} / 64) + 1 = {nqb + 1}")
  t = int(ptr[-1]) if ptr.size else 0
  if ptr[0] != 0 or np.any(np.diff(ptr.astype(np.int64)) < 0) or kb.size != t:
    raise ValueError(f"{what}: tile_ptr is not a CSR pointer over {kb.size} tiles")
  if bits.size != t * BLOCK_Q:
    raise ValueError(f"{what}: tile_bits has {bits.size} words, expected {t} x 64")
  if t and (kb.min() < 0 or kb.max() >= -(-n // BLOCK_K)):
    raise ValueError(f"{what}: key blocks outside [0, ceil({n} / 32))")


def _tiles64_from_arrays(tile_ptr, tile_kb, tile_bits, n_cols, device) -> TileList64:
  ptr = torch.as_tensor(np.asarray(tile_ptr, np.int32), device=device)
  kb = torch.as_tensor(np.asarray(tile_kb, np.int32), device=device)
  bits = torch.as_tensor(np.ascontiguousarray(np.asarray(tile_bits, np.uint32)).view(np.int32), device=device)
  return TileList64(ptr, kb, bits.reshape(-1, 64), (ptr.numel() - 1) * 64, n_cols)


class AttentionTiles:
  """Forward and transposed 128-row lists of one mask, resident on the device (built once per mask,
  like the reference's tile constants, patch.py:208-219): paired lists (fwd, bwd) and their gathered
  forms (fwd_g, bwd_g), which the kernels use whenever q/k/v/o have a node- or head-major layout."""

  def __init__(self, fwd: TileList128, bwd: TileList128, n: int, symmetric: bool, gather: bool = True):
    self.fwd = fwd
    self.bwd = bwd
    self.n = n
    self.symmetric = symmetric
    self.fwd_g = gather_tiles(fwd) if gather else None
    self.bwd_g = (self.fwd_g if bwd is fwd else gather_tiles(bwd)) if gather else None
    # Dense: gathering the distinct keys of each block would save under a quarter of the tiles (the
    # neighbourhoods fill their 32-key tiles), or, without gathered lists, 16+ tiles per 128-row block. Dense
    # masks run the wide-chunk kernels on the 32-key tile lists.
    if self.fwd_g is not None:
      self.dense = 4 * fwd.n_tiles < 5 * max(self.fwd_g.n_tiles, 1)
    else:
      self.dense = fwd.n_tiles >= 16 * fwd.n_blocks

  @classmethod
  def from_mask(cls, mask, device=None, gather: bool = True) -> "AttentionTiles":
    dev = _device(device)
    m = sparse.csr_matrix(mask).astype(bool)
    m.eliminate_zeros()
    n = m.shape[0]
    assert m.shape == (n, n), "attention masks are square [n, n]"
    indptr, indices, _ = _csr_to_device(m, dev)
    fwd = pair_tiles(build_tiles_device(indptr, indices, n, n))
    symmetric = (m != m.T).nnz == 0
    if symmetric:
      bwd = fwd
    else:
      mt = m.T.tocsr()
      ip, ix, _ = _csr_to_device(mt, dev)
      bwd = pair_tiles(build_tiles_device(ip, ix, n, n))
    return cls(fwd, bwd, n, symmetric, gather)

  @classmethod
  def from_khop(cls, adj, hops: int, device=None, gather: bool = True) -> "AttentionTiles":
    """Lists of the k-hop mask of a symmetric adjacency, built entirely on the device (mask, CSR, lists);
    permute the adjacency first for a node order (the k-hop mask of a permuted graph is the permuted mask)."""
    dev = _device(device)
    a = sparse.csr_matrix(adj).astype(bool)
    assert (a != a.T).nnz == 0, "from_khop takes a symmetric adjacency"
    n = a.shape[0]
    indptr, indices = khop_csr_device(a, hops, dev)
    fwd = pair_tiles(build_tiles_device(indptr, indices, n, n))
    return cls(fwd, fwd, n, True, gather)

  @classmethod
  def from_adjacency(cls, adj, k_hop: int, latlon=None, reorder: bool = True, device=None,
                     gather: bool = True):
    """(tiles, perm) for the attention mask adj ** k_hop, the sequence of the reference's _transformer_init
    (patch.py:207-219) on the device:

      mask = adj ** k_hop                                   the matrix-power pattern (fwn_walk_bitset)
      perm = hilbert_order(lat, lon) if reorder and latlon  node order (None: the given order)
      mask = mask[perm][:, perm]                            (the power of the permuted adjacency: same pattern)
      lists of mask; lists of mask.T if adj is not symmetric

    latlon: (lat_deg, lon_deg) of the nodes, or None to take them from adj._fwn_latlon (the attribute the
    reference's patched _get_adjacency_matrix sets, patch.py:296-302) when present. perm: int64 [n] or None;
    node i of the permuted order is node perm[i] of adj (pass it to Processor.forward(..., perm=perm))."""
    dev = _device(device)
    if latlon is None:
      latlon = getattr(adj, "_fwn_latlon", None)
    a = sparse.csr_matrix(adj).astype(bool)
    a.eliminate_zeros()
    n = a.shape[0]
    assert a.shape == (n, n), "adjacency must be square"
    perm = None
    if reorder and latlon is not None:
      lat, lon = (np.asarray(x, np.float64).ravel() for x in latlon)
      if lat.size != n or lon.size != n:
        raise ValueError(f"latlon has {lat.size} / {lon.size} points for {n} nodes")
      perm = np.asarray(hilbert_order(lat, lon), np.int64)
      a = a[perm][:, perm].tocsr()
    symmetric = (a != a.T).nnz == 0
    indptr, indices = power_csr_device(a, k_hop, dev)
    fwd = pair_tiles(build_tiles_device(indptr, indices, n, n))
    if symmetric:
      return cls(fwd, fwd, n, True, gather), perm
    ip_t, ix_t = power_csr_device(a.T.tocsr(), k_hop, dev)
    bwd = pair_tiles(build_tiles_device(ip_t, ix_t, n, n))
    return cls(fwd, bwd, n, False, gather), perm

  @classmethod
  def from_lists(cls, tile_ptr, tile_kb, tile_bits, n: int, tiles_t=None, device=None,
                 gather: bool = True) -> "AttentionTiles":
    """From the reference's (tile_ptr, tile_kb, tile_bits) arrays (and optionally the transposed triple)."""
    dev = _device(device)
    _check_lists(tile_ptr, tile_kb, tile_bits, n, "tiles")
    if tiles_t is not None:
      _check_lists(*tiles_t, n, "tiles_t")
    fwd = pair_tiles(_tiles64_from_arrays(tile_ptr, tile_kb, tile_bits, n, dev))
    if tiles_t is None:
      return cls(fwd, fwd, n, True, gather)
    bwd = pair_tiles(_tiles64_from_arrays(*tiles_t, n, dev))
    return cls(fwd, bwd, n, False, gather)


_PRECISION = threading.local()
_HIGHEST = ("highest", "float32")
_PRECISION_NAMES = ("default", "high", "highest", "bfloat16", "tensorfloat32", "float32", "bfloat16_3x",
                    "fastest")


@contextlib.contextmanager
def default_matmul_precision(name: Optional[str]):
  """with default_matmul_precision("highest"): ...  — the matmul precision of float32 attention calls in the
  block that pass no `precision=` (jax.default_matmul_precision's role for the reference, pallas_attn.py:336).
  Thread-local; blocks nest."""
  if name is not None and name not in _PRECISION_NAMES:
    raise ValueError(f"unknown matmul precision {name!r}")
  stack = getattr(_PRECISION, "stack", None)
  if stack is None:
    stack = _PRECISION.stack = []
  stack.append(name)
  try:
    yield
  finally:
    stack.pop()


def current_matmul_precision() -> Optional[str]:
  stack = getattr(_PRECISION, "stack", None)
  return stack[-1] if stack else None


def _mode_for(dtype: torch.dtype, precision: Optional[str], strict_fp32: bool) -> int:
  """Kernel mode for q's dtype and the precision in force (pallas_attn.py:336-342)."""
  if dtype == torch.bfloat16:
    return _lib.MODE_BF16
  if dtype != torch.float32:
    raise TypeError(f"q/k/v must be bfloat16 or float32, got {dtype}")
  if precision is None:
    precision = current_matmul_precision()
  if precision is not None and precision not in _PRECISION_NAMES:
    raise ValueError(f"unknown matmul precision {precision!r}")
  if precision in _HIGHEST:
    if strict_fp32:
      raise NotImplementedError(
          "strict_fp32 under 'highest' asks for IEEE float32 dots (the reference's F32_F32_F32), which have no "
          "tensor-core form and are not built; 'highest' without strict_fp32 runs 3xTF32 (rel RMS <= 2e-5)")
    return _lib.MODE_TF32X3
  return _lib.MODE_TF32


def _desc(q: torch.Tensor, o: torch.Tensor, scale: float, mode: int, grad: torch.Tensor = None) -> _lib.AttnDesc:
  """q's strides for q, k, v; o's strides for o, d_o and, unless `grad` (a [B, n, H, D] view with the gradients'
  strides) is given, for dq, dk, dv."""
  b, n, h, d = q.shape
  sb, sn, sh, sd = q.stride()
  ob, on, oh, od = o.stride()
  if sd != 1 or od != 1:
    raise ValueError("head_dim must be contiguous")
  dt = _lib.DTYPE_BF16 if q.dtype == torch.bfloat16 else _lib.DTYPE_F32
  if grad is None:
    return _lib.AttnDesc(b, h, n, d, float(scale), dt, mode, 0, sb, sn, sh, ob, on, oh)
  gb, gn, gh, gd = grad.stride()
  if gd != 1:
    raise ValueError("head_dim of the gradients must be contiguous")
  return _lib.AttnDesc(b, h, n, d, float(scale), dt, mode, _lib.DESC_GRAD_STRIDES, sb, sn, sh, ob, on, oh, gb, gn,
                       gh)


def _gather_layout(t: torch.Tensor) -> int:
  """0: (batch, node, head) rows form one strided 2D view; 1: (batch, head, node) rows do; -1: neither."""
  b, n, h, _ = t.shape
  sb, sn, sh, _ = t.stride()
  if (h == 1 or sn == h * sh) and (b == 1 or sb == n * sn):
    return 0
  if (n == 1 or sh == n * sn) and (b == 1 or sb == h * sh):
    return 1
  return -1


def _lists(tiles: "AttentionTiles", q: torch.Tensor, o: torch.Tensor):
  """(forward list, transposed list): gathered when the layouts allow gathered row loads and the mask is
  sparse; the 32-key tile lists for dense masks (where gathering saves few tiles and the wide-chunk kernels
  apply) and for bf16 at head_dim 128."""
  if tiles.dense or (q.shape[-1] == 128 and q.dtype == torch.bfloat16):
    return tiles.fwd, tiles.bwd
  if tiles.fwd_g is not None:
    a, c = _gather_layout(q), _gather_layout(o)
    if a >= 0 and a == c:
      return tiles.fwd_g, tiles.bwd_g
  return tiles.fwd, tiles.bwd


def _same_layout(*ts):
  ref = ts[0]
  return all(t.shape == ref.shape and t.stride() == ref.stride() and t.dtype == ref.dtype for t in ts)


def _canon(*ts):
  """Make tensors share one [B, n, H, D] layout with head_dim contiguous."""
  if _same_layout(*ts) and ts[0].stride(-1) == 1:
    return ts
  return tuple(t.contiguous() for t in ts)


def attention_forward(q, k, v, tiles: AttentionTiles, scale: float, mode: int, with_lse: bool = True):
  """o [B, n, H, D] (q's dtype) and lse float32 [B, H, lse_rows] (or None)."""
  lib = _lib.lib()
  q, k, v = _canon(q, k, v)
  o = torch.empty(q.shape, dtype=q.dtype, device=q.device)
  desc = _desc(q, o, scale, mode)
  lse = None
  if with_lse:
    b, n, h, _ = q.shape
    lse = torch.empty(b, h, lib.fwn_lse_rows(n), dtype=torch.float32, device=q.device)
  st = _lists(tiles, q, o)[0].struct()
  _lib.check(lib.fwn_attn_fwd(ctypes.byref(desc), q.data_ptr(), k.data_ptr(), v.data_ptr(), ctypes.byref(st),
                              o.data_ptr(), lse.data_ptr() if lse is not None else 0, _stream()))
  return o, lse


_SIDE_STREAMS = {}


def _side_stream(device: torch.device) -> torch.cuda.Stream:
  """One extra stream per device: the dQ pass runs on it while the dK/dV pass runs on the caller's stream."""
  st = _SIDE_STREAMS.get(device.index)
  if st is None:
    st = _SIDE_STREAMS[device.index] = torch.cuda.Stream(device)
  return st


def attention_backward(q, k, v, o, lse, do, tiles: AttentionTiles, scale: float, mode: int, dqkv=None):
  """(dq, dk, dv), each [B, n, H, D] in q's dtype; with dqkv ([B, n, H, 3, D], q's dtype and device) the kernels
  write them into its slices [..., 0, :], [..., 1, :], [..., 2, :] (the gradient of a fused projection's output)
  and the slices are returned.

  delta = rowsum(o * do) first (fwn_attn_bwd_delta); then the dQ pass (over the forward list) on a side stream
  and the dK/dV pass (over the transposed list) on the current stream at the same time, joined before return:
  the two passes read the same inputs and write different outputs, and running them together overlaps their
  tails (configuration 3: 3 % of the step). The launches are fwn_attn_bwd's, one by one."""
  lib = _lib.lib()
  q, k, v = _canon(q, k, v)
  o, do = _canon(o.contiguous(), do.contiguous())
  if dqkv is not None:
    dq, dk, dv = dqkv[:, :, :, 0], dqkv[:, :, :, 1], dqkv[:, :, :, 2]
    desc = _desc(q, o, scale, mode, grad=dq)
  else:
    dq, dk, dv = (torch.empty(q.shape, dtype=q.dtype, device=q.device) for _ in range(3))
    desc = _desc(q, o, scale, mode)
  ws_bytes = ctypes.c_size_t(0)
  _lib.check(lib.fwn_attn_bwd_workspace_size(ctypes.byref(desc), ctypes.byref(ws_bytes)))
  ws = torch.empty(max(ws_bytes.value, 16), dtype=torch.uint8, device=q.device)
  lf, lb = _lists(tiles, q, o)
  sf, sb = lf.struct(), lb.struct()
  d = ctypes.byref(desc)
  main = torch.cuda.current_stream(q.device)
  side = _side_stream(q.device)
  _lib.check(lib.fwn_attn_bwd_delta(d, o.data_ptr(), do.data_ptr(), ws.data_ptr(), ws.numel(), main.cuda_stream))
  side.wait_stream(main)
  _lib.check(lib.fwn_attn_bwd_dq(d, q.data_ptr(), k.data_ptr(), v.data_ptr(), lse.data_ptr(), do.data_ptr(),
                                 ctypes.byref(sf), dq.data_ptr(), ws.data_ptr(), ws.numel(), side.cuda_stream))
  _lib.check(lib.fwn_attn_bwd_dkv(d, q.data_ptr(), k.data_ptr(), v.data_ptr(), lse.data_ptr(), do.data_ptr(),
                                  ctypes.byref(sb), dk.data_ptr(), dv.data_ptr(), ws.data_ptr(), ws.numel(),
                                  main.cuda_stream))
  main.wait_stream(side)
  return dq, dk, dv


class _TiledAttention(torch.autograd.Function):
  """custom VJP (pallas_attn.py:260-314): forward saves (q, k, v, o, lse); backward runs the dQ and
  dK/dV kernels, recomputing P from the saved log-sum-exp."""

  @staticmethod
  def forward(ctx, q, k, v, tiles, scale, mode):
    needs = any(ctx.needs_input_grad[:3])
    o, lse = attention_forward(q, k, v, tiles, scale, mode, with_lse=needs)
    if needs:
      ctx.save_for_backward(q, k, v, o, lse)
    ctx.tiles, ctx.scale, ctx.mode = tiles, scale, mode
    return o

  @staticmethod
  def backward(ctx, do):
    q, k, v, o, lse = ctx.saved_tensors
    dq, dk, dv = attention_backward(q, k, v, o, lse, do, ctx.tiles, ctx.scale, ctx.mode)
    return dq, dk, dv, None, None, None


class _TiledAttentionQKV(torch.autograd.Function):
  """The same attention over q, k, v given as one fused projection output qkv [B, n, H, 3, D] (q, k, v its slices
  along dim 3, read in place): the backward writes dq, dk, dv straight into one [B, n, H, 3, D] gradient
  (FWN_DESC_GRAD_STRIDES), where autograd would otherwise zero-fill a full-size buffer per slice, copy each slice
  gradient into it and sum the three."""

  @staticmethod
  def forward(ctx, qkv, tiles, scale, mode):
    q, k, v = qkv[:, :, :, 0], qkv[:, :, :, 1], qkv[:, :, :, 2]
    needs = ctx.needs_input_grad[0]
    o, lse = attention_forward(q, k, v, tiles, scale, mode, with_lse=needs)
    if needs:
      ctx.save_for_backward(qkv, o, lse)
    ctx.tiles, ctx.scale, ctx.mode = tiles, scale, mode
    return o

  @staticmethod
  def backward(ctx, do):
    qkv, o, lse = ctx.saved_tensors
    dqkv = torch.empty(qkv.shape, dtype=qkv.dtype, device=qkv.device)
    q, k, v = qkv[:, :, :, 0], qkv[:, :, :, 1], qkv[:, :, :, 2]
    attention_backward(q, k, v, o, lse, do, ctx.tiles, ctx.scale, ctx.mode, dqkv=dqkv)
    return dqkv, None, None, None


_BUILT_HEAD_DIMS = (64, 128)


def attention_qkv(qkv, tiles: AttentionTiles, *, scale: float, precision: Optional[str] = None,
                  strict_fp32: bool = False):
  """attention() over a fused projection output qkv [B, n, H, 3, D] (q, k, v = qkv[:, :, :, i]) -> [B, n, H, D];
  its gradient is one [B, n, H, 3, D] tensor written by the backward kernels. Head dims other than 64 and 128 take
  attention() on the slices (zero padding)."""
  if qkv.dim() != 5 or qkv.shape[3] != 3:
    raise ValueError(f"qkv has shape {tuple(qkv.shape)}, expected [B, n, H, 3, D]")
  mode = _mode_for(qkv.dtype, precision, strict_fp32)
  if qkv.shape[-1] not in _BUILT_HEAD_DIMS or qkv.stride(-1) != 1:
    return attention(qkv[:, :, :, 0], qkv[:, :, :, 1], qkv[:, :, :, 2], tiles, scale=scale, precision=precision,
                     strict_fp32=strict_fp32)
  return _TiledAttentionQKV.apply(qkv, tiles, float(scale), mode)


def attention(q, k, v, tiles: AttentionTiles, *, scale: float, precision: Optional[str] = None,
              strict_fp32: bool = False):
  """Differentiable masked attention over prepared tiles: q, k, v [B, n, H, D] -> [B, n, H, D]."""
  mode = _mode_for(q.dtype, precision, strict_fp32)
  d = q.shape[-1]
  if d in _BUILT_HEAD_DIMS:
    return _TiledAttention.apply(q, k, v, tiles, float(scale), mode)
  if d > _BUILT_HEAD_DIMS[-1] or d < 1:
    raise NotImplementedError(f"head_dim {d} not built (64 or 128; smaller sizes are zero-padded)")
  pad = next(x for x in _BUILT_HEAD_DIMS if x > d) - d
  qp, kp, vp = (torch.nn.functional.pad(x, (0, pad)) for x in (q, k, v))
  return _TiledAttention.apply(qp, kp, vp, tiles, float(scale), mode)[..., :d]


class _TileCache:
  """AttentionTiles of the last reference-format lists passed to tiled_flash_attention.

  The entry holds the argument objects themselves, so none of them can be freed and its id reused while the
  entry lives, and it is used only when every list argument is the same object as before (and n and the
  device match): rebuilt lists, or lists passed as new arrays, are converted again. As with the reference,
  whose lists become constants when the model is traced (patch.py:266), a list edited in place after its first
  use is not seen; pass new arrays instead."""

  def __init__(self):
    self._args = None
    self._tiles = None

  def get(self, args, n, device):
    hit = (self._args is not None and len(self._args) == len(args) and
           all(a is b for a, b in zip(self._args, args)))
    if hit and self._tiles.n == n and self._tiles.fwd.ptr.device == device:
      return self._tiles
    ptr, kb, bits = (_np(x) for x in args[:3])
    tiles_t = tuple(_np(x) for x in args[3:6]) if len(args) > 3 else None
    tiles = AttentionTiles.from_lists(ptr, kb, bits, n, tiles_t=tiles_t, device=device)
    self._args, self._tiles = tuple(args), tiles
    return tiles

  def clear(self):
    self._args = self._tiles = None


_TILE_CACHE = _TileCache()


def tiled_flash_attention(q, k, v, tile_ptr, tile_kb, tile_bits, *, scale, strict_fp32=False, tiles_t=None,
                          block_q=BLOCK_Q, block_k=BLOCK_K, num_warps=None, num_stages=None, bwd_num_warps=None,
                          bwd_split=None, interpret=False, precision=None):
  """Drop-in for pallas_attn.tiled_flash_attention: q, k, v [batch, n, heads, head_dim] -> same shape.

  tile lists are the reference's (build_tile_mask) 64-row lists, NumPy or torch; tiles_t is the
  transposed mask's list (None: the mask is symmetric). The Triton launch knobs (num_warps,
  num_stages, bwd_num_warps, bwd_split) have no meaning here and are accepted for compatibility;
  `interpret` (Pallas interpret mode) is refused: there is no CPU path. Precision: `precision=`, else the
  enclosing default_matmul_precision block, else TF32 for float32 inputs (see the module docstring).
  """
  if interpret:
    raise NotImplementedError("interpret mode: this implementation has no CPU path")
  if block_q != BLOCK_Q or block_k != BLOCK_K:
    raise ValueError("the tile lists use 64-row query blocks and 32-key tiles")
  if tiles_t is not None and len(tiles_t) != 3:
    raise ValueError("tiles_t is the transposed mask's (tile_ptr, tile_kb, tile_bits)")
  n = q.shape[1]
  args = (tile_ptr, tile_kb, tile_bits) + (tuple(tiles_t) if tiles_t is not None else ())
  tiles = _TILE_CACHE.get(args, n, q.device)
  return attention(q, k, v, tiles, scale=scale, precision=precision, strict_fp32=strict_fp32)


def _np(x):
  """NumPy view of a tile-list array. Tile bits are uint32 in the reference; an int32 array of rank 2 (the
  same bits in signed storage, as torch holds them) is reinterpreted, every other array is taken as is."""
  if isinstance(x, torch.Tensor):
    x = x.detach().cpu().numpy()
  x = np.asarray(x)
  return x.view(np.uint32) if x.dtype == np.int32 and x.ndim == 2 else x
