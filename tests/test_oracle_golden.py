"""CPU: the oracle against the golden vectors made from the reference's own code."""
import numpy as np
import pytest
from scipy import sparse

from oracle import attention as oa
from oracle import tiles as ot
from tests.helpers import digest, golden_mask, golden_names, kernel_inputs


def test_build_tile_mask_matches_reference(golden):
  g = golden["tiles"]
  for name in golden_names(g):
    m = golden_mask(g, name)
    ptr, kb, bits = ot.build_tile_mask(m)
    np.testing.assert_array_equal(ptr, g[name + "/ptr"], err_msg=name)
    np.testing.assert_array_equal(kb, g[name + "/kb"], err_msg=name)
    np.testing.assert_array_equal(bits, g[name + "/bits"], err_msg=name)
    assert ptr.dtype == np.int32 and kb.dtype == np.int32 and bits.dtype == np.uint32


@pytest.mark.parametrize("cfg", [2, 3])
def test_config_tile_lists_match_reference_digest(golden, cfg):
  from faster_weathernext import mesh
  m, _, _ = mesh.config_mask(cfg)
  assert mesh.csr_digest(m) == golden["digests"][f"cfg{cfg}/mask"], "mesh/mask generation changed"
  ptr, kb, bits = ot.build_tile_mask(m)
  assert str(len(kb)) == golden["digests"][f"cfg{cfg}/n_tiles"]
  assert digest(ptr, kb, bits) == golden["digests"][f"cfg{cfg}/tiles"]


def test_tile_roundtrip_and_invariants(golden):
  """tests/test_masks.py:25-36 on the oracle: round trip, ptr bounds, distinct non-empty tiles."""
  g = golden["tiles"]
  for name in ("rand100", "rand257", "rand1000", "k_nonsym", "cfg1"):
    m = golden_mask(g, name)
    ptr, kb, bits = ot.build_tile_mask(m)
    assert ptr[0] == 0 and ptr[-1] == len(kb) == len(bits)
    np.testing.assert_array_equal(ot.tiles_to_dense(ptr, kb, bits, m.shape[0], m.shape[1]), m.toarray())
    for q in range(len(ptr) - 1):
      seg = kb[ptr[q]:ptr[q + 1]]
      assert len(np.unique(seg)) == len(seg)
      assert (np.diff(seg) > 0).all()
      assert bits[ptr[q]:ptr[q + 1]].any(axis=1).all()


def test_pairing_covers_the_same_mask(golden):
  g = golden["tiles"]
  for name in ("rand257", "rand1000", "k_fwd", "cfg1"):
    m = golden_mask(g, name)
    ptr, kb, bits = ot.build_tile_mask(m)
    p2, kb2, b2 = ot.pair_tiles(ptr, kb, bits)
    assert len(p2) - 1 == -(-m.shape[0] // 128)
    np.testing.assert_array_equal(ot.tiles_to_dense(p2, kb2, b2, m.shape[0], m.shape[1], block_q=128), m.toarray())
    for q in range(len(p2) - 1):
      seg = kb2[p2[q]:p2[q + 1]]
      assert (np.diff(seg) > 0).all()


def test_hilbert_order_matches_reference(golden):
  h = golden["hilbert"]
  np.testing.assert_array_equal(ot.hilbert_order(h["lat"], h["lon"]), h["perm"])


@pytest.mark.parametrize("cfg", [1, 2, 3])
def test_hilbert_order_config_digests(golden, cfg):
  from faster_weathernext import mesh
  _, lat, lon = mesh.config_mask(cfg)
  assert digest(ot.hilbert_order(lat, lon).astype(np.int64)) == golden["digests"][f"cfg{cfg}/hilbert"]


def test_chunked_mask_matches_reference(golden):
  c = golden["chunked"]
  from faster_weathernext import mesh
  banded = sparse.csr_matrix((np.ones(len(c["banded/indices"]), bool), c["banded/indices"], c["banded/indptr"]),
                             shape=(700, 700))
  cfg1, _, _ = mesh.config_mask(1)
  t = golden["tiles"]
  kfwd = golden_mask(t, "k_fwd")
  for name, m in (("banded", banded), ("cfg1", cfg1), ("k_fwd", kfwd)):
    starts, bits, window, n_kv = ot.build_chunked_mask(m, int(c[name + "/chunk"]))
    np.testing.assert_array_equal(starts, c[name + "/starts"])
    np.testing.assert_array_equal(bits, c[name + "/bits"])
    assert window == int(c[name + "/window"]) and n_kv == int(c[name + "/n_kv"])


def test_dense_references_match_reference_tests(golden):
  """The oracle's float64 forward/gradient equal the reference test functions' outputs."""
  a = golden["attention"]
  t = golden["tiles"]
  ev = int(a["every"])
  q, k, v = kernel_inputs(0, (2, 300, 2, 64), 3)
  dense = golden_mask(t, "k_fwd").toarray()
  for b in range(2):
    np.testing.assert_allclose(oa.dense_attention(q[b], k[b], v[b], dense, 0.125)[::ev], a[f"fwd/b{b}/out"],
                               rtol=1e-6, atol=1e-6)
  for tag in ("sym", "nonsym"):
    q, k, v, do = kernel_inputs(2, (1, 300, 2, 64), 4)
    m = golden_mask(t, "k_" + tag).toarray()
    for nm, x in zip(("dq", "dk", "dv"), oa.dense_attention_vjp(q[0], k[0], v[0], do[0], m, 0.125)):
      np.testing.assert_allclose(x[::ev], a[f"grad_{tag}/{nm}"], rtol=1e-5, atol=1e-6, err_msg=nm)


def test_sparse_and_chunked_oracles_agree_with_dense(golden):
  """The CSR-form and chunked (XLA-path) forwards, and the CSR-form VJP, against the dense float64 ones."""
  t = golden["tiles"]
  a = golden["attention"]
  ev = int(a["every"])
  m = golden_mask(t, "k_nonsym")
  q, k, v, do = kernel_inputs(2, (1, 300, 2, 64), 4)
  out, lse = oa.sparse_attention(q, k, v, m, 0.125)
  ref = oa.dense_attention(q[0], k[0], v[0], m.toarray(), 0.125)
  assert oa.max_rel(out[0], ref) < 1e-12
  ch = oa.chunked_attention(q, k, v, m, 0.125, chunk=64, dtype=np.float64)
  assert oa.max_rel(ch[0], ref) < 1e-12
  ch32 = oa.chunked_attention(q, k, v, m, 0.125, chunk=64, dtype=np.float32)
  assert oa.rel_rms(ch32[0], ref) < 1e-6
  grads = oa.sparse_attention_vjp(q, k, v, do, m, 0.125)
  for nm, x in zip(("dq", "dk", "dv"), grads):
    np.testing.assert_allclose(x[0][::ev], a[f"grad_nonsym/{nm}"], rtol=1e-5, atol=1e-6, err_msg=nm)
  # lse = log sum exp of the allowed scaled logits.
  s = np.einsum("nhd,mhd->hnm", q[0].astype(np.float64), k[0].astype(np.float64)) * 0.125
  s = np.where(m.toarray()[None], s, -np.inf)
  np.testing.assert_allclose(lse[0], np.log(np.exp(s - s.max(-1, keepdims=True)).sum(-1)) + s.max(-1), rtol=1e-12)


def test_config1_golden(golden):
  """Configuration 1 (n=642, B1 H4 D64): oracle forward and VJP against the reference's float64 functions."""
  from faster_weathernext import mesh
  a = golden["attention"]
  ev = int(a["every"])
  m, _, _ = mesh.config_mask(1)
  rng = np.random.default_rng(0)
  q, k, v = (rng.standard_normal((1, 642, 4, 64)).astype(np.float32) for _ in range(3))
  do = np.random.default_rng(1).standard_normal((1, 642, 4, 64)).astype(np.float32)
  out, _ = oa.sparse_attention(q, k, v, m, 0.125)
  np.testing.assert_allclose(out[0][::ev], a["cfg1/out"], rtol=1e-5, atol=1e-6)
  for nm, x in zip(("dq", "dk", "dv"), oa.sparse_attention_vjp(q, k, v, do, m, 0.125)):
    np.testing.assert_allclose(x[0][::ev], a[f"cfg1/{nm}"], rtol=1e-5, atol=1e-6, err_msg=nm)


def test_chunked_vjp_matches_analytic_gradient(golden):
  """The XLA-path backward restatement (autodiff of patch.py:144-159) equals the reference tests' gradient."""
  a = golden["attention"]
  ev = int(a["every"])
  m = golden_mask(golden["tiles"], "k_sym")
  q, k, v, do = kernel_inputs(2, (1, 300, 2, 64), 4)
  got = oa.chunked_attention_vjp(q, k, v, do, m, 0.125, chunk=64, dtype=np.float64)
  for nm, x in zip(("dq", "dk", "dv"), got):
    np.testing.assert_allclose(x[0][::ev], a[f"grad_sym/{nm}"], rtol=1e-5, atol=1e-6, err_msg=nm)


def test_gathered_lists_cover_the_same_mask(golden):
  g = golden["tiles"]
  for name in ("rand257", "k_nonsym", "cfg1"):
    m = golden_mask(g, name)
    p2, kb2, b2 = ot.pair_tiles(*ot.build_tile_mask(m))
    pg, cols, bits = ot.gather_tiles(p2, kb2, b2)
    np.testing.assert_array_equal(ot.gathered_to_dense(pg, cols, bits, m.shape[0], m.shape[1]), m.toarray())
    for p in range(len(pg) - 1):
      c = cols[pg[p]:pg[p + 1]].ravel()
      assert (np.diff(c) >= 0).all()                      # ascending (padding repeats the last column)
      rows = np.arange(p * 128, min(m.shape[0], p * 128 + 128))
      assert len(np.unique(c)) == len(np.unique(m[rows].indices))
