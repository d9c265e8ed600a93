"""GPU: the reference-named drop-in, case by case as the reference's own kernel tests run it.

tiled_attn.tiled_flash_attention(q, k, v, *build_tile_mask(m), scale=..., tiles_t=...) with the reference's 64-row
NumPy triples, mirroring tests/test_pallas_kernel.py:35-118 (same seeds, shapes, masks and metric: max|err| /
max|ref| against the float64 dense softmax, 1e-5 under "highest" (3xTF32), 2e-2 forward / 3e-2 gradients in
the default precision (TF32)); the precision is set the reference's way, with a default_matmul_precision block.
Then: strict_fp32 semantics, the argument checks, the list cache, patch.tiled_mha against a dense restatement
(patch.py:165-177), and patch.transformer_tiles (the mask part of _transformer_init, patch.py:207-219) against
the oracle's lists of the permuted matrix power.
"""
import numpy as np
import pytest
import torch
from scipy import sparse

from oracle import attention as oa
from oracle import tiles as ot

pytestmark = pytest.mark.gpu


def _dense_ref(q, k, v, mask, scale):
  """tests/test_pallas_kernel.py:15-22: float64 dense masked softmax of one batch element ((n, heads, d))."""
  s = np.einsum("nhd,mhd->hnm", q.astype(np.float64), k.astype(np.float64)) * scale
  s = np.where(mask[None], s, -np.inf)
  p = np.exp(s - s.max(-1, keepdims=True))
  p /= p.sum(-1, keepdims=True)
  return np.einsum("hnm,mhd->nhd", p, v.astype(np.float64))


def _dense_grads(q, k, v, do, mask, scale):
  """tests/test_pallas_kernel.py:58-69: float64 dQ, dK, dV of one batch element."""
  q, k, v, do = (x.astype(np.float64) for x in (q, k, v, do))
  s = np.where(mask[None], np.einsum("nhd,mhd->hnm", q, k) * scale, -np.inf)
  p = np.exp(s - s.max(-1, keepdims=True))
  p /= p.sum(-1, keepdims=True)
  dp = np.einsum("nhd,mhd->hnm", do, v)
  ds = p * (dp - (dp * p).sum(-1, keepdims=True))
  return (np.einsum("hnm,mhd->nhd", ds, k) * scale, np.einsum("hnm,nhd->mhd", ds, q) * scale,
          np.einsum("hnm,nhd->mhd", p, do))


def _err(got, ref):
  return np.abs(np.asarray(got, np.float64) - ref).max() / np.abs(ref).max()


def _t(x, device, grad=False):
  t = torch.from_numpy(np.ascontiguousarray(x)).to(device)
  return t.requires_grad_(True) if grad else t


@pytest.mark.parametrize("batch", [1, 2])
@pytest.mark.parametrize("precision,tol", [("highest", 1e-5), ("default", 2e-2)])
def test_dropin_matches_dense_reference(cuda, precision, tol, batch):
  """tests/test_pallas_kernel.py:35-55."""
  from faster_weathernext import tiled_attn as ta
  rng = np.random.default_rng(0)
  n, h, d = 300, 2, 64
  q, k, v = (rng.standard_normal((batch, n, h, d)).astype(np.float32) for _ in range(3))
  m = (sparse.random(n, n, density=0.1, random_state=1, format="csr").astype(bool)
       + sparse.identity(n, dtype=bool)).tocsr()
  tiles = ta.build_tile_mask(m)
  for a, b in zip(tiles, ot.build_tile_mask(m)):
    assert a.dtype == b.dtype and np.array_equal(a, b)
  with ta.default_matmul_precision(precision):
    out = ta.tiled_flash_attention(_t(q, cuda), _t(k, cuda), _t(v, cuda), *tiles, scale=d ** -0.5)
  out = out.cpu().numpy()
  for b in range(batch):
    ref = _dense_ref(q[b], k[b], v[b], m.toarray(), d ** -0.5)
    assert _err(out[b], ref) < tol, (b, _err(out[b], ref))
    if precision == "highest":
      assert oa.rel_rms(out[b], ref) < 2e-5


@pytest.mark.parametrize("split", [1, 2])
@pytest.mark.parametrize("symmetric", [True, False])
@pytest.mark.parametrize("batch", [1, 2])
@pytest.mark.parametrize("precision,tol", [("highest", 1e-5), ("default", 3e-2)])
def test_dropin_grads_match_dense_reference(cuda, precision, tol, batch, symmetric, split):
  """tests/test_pallas_kernel.py:72-99 (n = 300: padding rows; the transposed list for non-symmetric masks;
  bwd_split is a Triton launch knob, accepted and without effect here)."""
  from faster_weathernext import tiled_attn as ta
  rng = np.random.default_rng(2)
  n, h, d = 300, 2, 64
  q, k, v, do = (rng.standard_normal((batch, n, h, d)).astype(np.float32) for _ in range(4))
  m = sparse.random(n, n, density=0.08, random_state=3, format="csr").astype(bool)
  m = ((m + m.T) if symmetric else m) + sparse.identity(n, dtype=bool)
  m = m.tocsr().astype(bool)
  tiles = ta.build_tile_mask(m)
  tiles_t = None if symmetric else ta.build_tile_mask(m.T.tocsr())
  tq, tk, tv = (_t(x, cuda, grad=True) for x in (q, k, v))
  with ta.default_matmul_precision(precision):
    out = ta.tiled_flash_attention(tq, tk, tv, *tiles, tiles_t=tiles_t, scale=d ** -0.5, bwd_split=split)
    out.backward(_t(do, cuda))
  grads = [x.grad.cpu().numpy() for x in (tq, tk, tv)]
  for b in range(batch):
    for name, got, ref in zip("qkv", grads, _dense_grads(q[b], k[b], v[b], do[b], m.toarray(), d ** -0.5)):
      assert _err(got[b], ref) < tol, (name, b, _err(got[b], ref))


def test_dropin_nonsymmetric_mask_needs_transposed_tiles(cuda):
  """tests/test_pallas_kernel.py:102-118 at the reference's head_dim 32 (zero-padded to 64 inside the op):
  reusing the forward list for dK of a non-symmetric mask is wrong; with tiles_t it is right."""
  from faster_weathernext import tiled_attn as ta
  rng = np.random.default_rng(4)
  n, h, d = 130, 1, 32
  q, k, v, do = (rng.standard_normal((1, n, h, d)).astype(np.float32) for _ in range(4))
  m = (sparse.random(n, n, density=0.1, random_state=5, format="csr").astype(bool)
       + sparse.identity(n, dtype=bool)).tocsr()
  tiles = ta.build_tile_mask(m)
  ref = _dense_grads(q[0], k[0], v[0], do[0], m.toarray(), d ** -0.5)[1]
  for tiles_t, wrong in ((None, True), (ta.build_tile_mask(m.T.tocsr()), False)):
    tk = _t(k, cuda, grad=True)
    out = ta.tiled_flash_attention(_t(q, cuda), tk, _t(v, cuda), *tiles, tiles_t=tiles_t, scale=d ** -0.5)
    assert out.shape == (1, n, h, d)
    out.backward(_t(do, cuda))
    err = _err(tk.grad[0].cpu().numpy(), ref)
    assert (err > 1e-2) if wrong else (err < 3e-2), (wrong, err)


def test_dropin_strict_fp32_and_argument_checks(cuda):
  """strict_fp32 changes nothing under the default precision (the reference's TF32, pallas_attn.py:342) and
  asks for the unbuilt IEEE float32 dots under "highest"; interpret mode and other block sizes are refused."""
  from faster_weathernext import tiled_attn as ta
  rng = np.random.default_rng(7)
  n = 200
  q, k, v = (_t(rng.standard_normal((1, n, 2, 64)).astype(np.float32), cuda) for _ in range(3))
  m = (sparse.random(n, n, density=0.1, random_state=8, format="csr").astype(bool)
       + sparse.identity(n, dtype=bool)).tocsr()
  tiles = ta.build_tile_mask(m)
  a = ta.tiled_flash_attention(q, k, v, *tiles, scale=0.125)
  b = ta.tiled_flash_attention(q, k, v, *tiles, scale=0.125, strict_fp32=True)
  assert torch.equal(a, b)
  with ta.default_matmul_precision("highest"):
    with pytest.raises(NotImplementedError):
      ta.tiled_flash_attention(q, k, v, *tiles, scale=0.125, strict_fp32=True)
  with pytest.raises(NotImplementedError):
    ta.tiled_flash_attention(q, k, v, *tiles, scale=0.125, interpret=True)
  with pytest.raises(ValueError):
    ta.tiled_flash_attention(q, k, v, *tiles, scale=0.125, block_k=16)
  with pytest.raises(ValueError):
    ta.tiled_flash_attention(q[:, :100], k[:, :100], v[:, :100], *tiles, scale=0.125)


def test_dropin_list_cache_and_list_types(cuda):
  """The device lists of a triple are reused while the same arrays are passed, and rebuilt for other arrays
  (new masks, or the same lists as torch tensors, whose int32 bits are the reference's uint32 words)."""
  from faster_weathernext import tiled_attn as ta
  rng = np.random.default_rng(9)
  n = 257
  q, k, v = (_t(rng.standard_normal((1, n, 2, 64)).astype(np.float32), cuda) for _ in range(3))
  masks = [(sparse.random(n, n, density=0.06, random_state=s, format="csr").astype(bool)
            + sparse.identity(n, dtype=bool)).tocsr() for s in (10, 11)]
  triples = [ta.build_tile_mask(m) for m in masks]
  outs = []
  for m, tr in zip(masks, triples):
    o1 = ta.tiled_flash_attention(q, k, v, *tr, scale=0.125)
    cached = ta._TILE_CACHE._tiles
    o2 = ta.tiled_flash_attention(q, k, v, *tr, scale=0.125)
    assert ta._TILE_CACHE._tiles is cached and torch.equal(o1, o2)
    ref, _ = oa.sparse_attention(*(x.cpu().numpy() for x in (q, k, v)), m, 0.125)
    assert oa.rel_rms(o1.cpu().numpy(), ref) < 5e-3
    outs.append(o1)
  assert not torch.equal(outs[0], outs[1])
  as_torch = [torch.from_numpy(x.view(np.int32) if x.dtype == np.uint32 else x).to(cuda) for x in triples[0]]
  o3 = ta.tiled_flash_attention(q, k, v, *as_torch, scale=0.125)
  assert torch.equal(o3, outs[0])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_tiled_mha_matches_dense_restatement(cuda, dtype):
  """patch.tiled_mha (patch.py:165-177): fused q/k/v projection, the block-sparse attention, output projection,
  against the same computation with a float64 dense masked softmax (rel RMS <= 5e-3)."""
  from faster_weathernext import mesh, patch
  from faster_weathernext import tiled_attn as ta
  m, _, _ = mesh.config_mask(1)
  n = m.shape[0]
  heads, key_size, d = 4, 64, 128
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  g = torch.Generator(device=cuda).manual_seed(11)
  x = torch.randn(2, n, d, device=cuda, generator=g).to(dtype)
  w_qkv = (torch.randn(d, heads * 3 * key_size, device=cuda, generator=g) * d ** -0.5).to(dtype)
  w_out = (torch.randn(heads * key_size, d, device=cuda, generator=g) * (heads * key_size) ** -0.5).to(dtype)
  b_out = torch.randn(d, device=cuda, generator=g).to(dtype)
  got = patch.tiled_mha(x, w_qkv, w_out, tiles, heads, key_size, b_out=b_out)
  assert got.shape == (2, n, d) and got.dtype == dtype
  qkv = (x.double() @ w_qkv.double()).view(2, n, heads, 3, key_size)
  if dtype == torch.bfloat16:
    qkv = qkv.to(dtype).double()                      # the kernel reads the bf16 projection
  o, _ = oa.sparse_attention(*(qkv[:, :, :, i].cpu().numpy() for i in range(3)), m, key_size ** -0.5)
  ref = torch.from_numpy(o).to(cuda).reshape(2, n, -1) @ w_out.double() + b_out.double()
  assert oa.rel_rms(got.double().cpu().numpy(), ref.cpu().numpy()) < (5e-3 if dtype == torch.float32 else 1e-2)


def _tagged_mesh_adjacency(level):
  """Mesh adjacency with self edges, tagged with the nodes' (lat, lon) as the reference's patched
  _get_adjacency_matrix tags it (patch.py:296-302)."""
  from faster_weathernext import mesh
  xyz, faces = mesh.icosphere(level)
  lat, lon = mesh.latlon(xyz)
  adj = mesh.adjacency(faces, xyz.shape[0])
  adj._fwn_latlon = (lat, lon)
  return adj, lat, lon


def _host_power(adj, k):
  a = sparse.csr_matrix(adj).astype(np.float64)
  a.data[:] = 1.0
  r = sparse.identity(a.shape[0], format="csr")
  for _ in range(k):
    r = (r @ a).tocsr()
    r.data[:] = 1.0
  return r.astype(bool).tocsr()


def _expect_paired(mask):
  return ot.pair_tiles(*ot.build_tile_mask(mask))


def _same_paired(lst, expected):
  got = lst.numpy()
  return all(np.array_equal(np.asarray(a), np.asarray(b)) for a, b in zip(got, expected))


@pytest.mark.parametrize("reorder", [True, False])
def test_transformer_tiles_follow_the_reference_init(cuda, reorder):
  """enable(reorder=...) then patch.transformer_tiles(adj, k) on a level-4 mesh: the permutation is the
  reference's Hilbert order of the tagged (lat, lon) (oracle restatement, pinned to the reference's output),
  and the lists equal the oracle's lists of (adj ** k)[perm][:, perm] (patch.py:209-214), bit for bit."""
  import faster_weathernext
  from faster_weathernext import patch
  adj, lat, lon = _tagged_mesh_adjacency(4)
  try:
    faster_weathernext.enable(reorder=reorder)
    tiles, perm = patch.transformer_tiles(adj, 5, device=cuda)
  finally:
    patch.OPTIONS = patch.Options()
    faster_weathernext.disable()
  mask = _host_power(adj, 5)
  if reorder:
    expected_perm = ot.hilbert_order(lat, lon)
    assert np.array_equal(perm, expected_perm)
    mask = mask[perm][:, perm].tocsr()
  else:
    assert perm is None
  assert tiles.symmetric and tiles.bwd is tiles.fwd
  assert _same_paired(tiles.fwd, _expect_paired(mask))


@pytest.mark.parametrize("power", [1, 2, 3])
def test_from_adjacency_nonsymmetric_walk_pattern(cuda, power):
  """A directed graph without self edges: the mask is the pattern of adj ** power itself (walks of exactly
  `power` edges, as scipy's matrix power gives the reference), and the backward walks the lists of its
  transpose (patch.py:215-218)."""
  from faster_weathernext import tiled_attn as ta
  n = 700
  adj = sparse.random(n, n, density=0.004, random_state=21, format="csr").astype(bool)
  adj.setdiag(False)
  adj.eliminate_zeros()
  tiles, perm = ta.AttentionTiles.from_adjacency(adj, power, device=cuda)
  assert perm is None and not tiles.symmetric
  mask = _host_power(adj, power)
  assert _same_paired(tiles.fwd, _expect_paired(mask))
  assert _same_paired(tiles.bwd, _expect_paired(mask.T.tocsr()))
