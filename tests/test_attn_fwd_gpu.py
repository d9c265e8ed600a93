"""GPU: forward kernel parity with the oracle (the reference's masked softmax) and the golden vectors.

Tolerances: rel RMS (RMS(diff) / std(ref), scripts/attn_bench.py:122) <= 5e-3 for bf16 and TF32 (the
stated bound for those modes), <= 2e-5 for 3xTF32; plus the reference test's max-abs metric
(tests/test_pallas_kernel.py:54: 2e-2 TF32). bf16 runs are compared with the oracle on the same
bf16-rounded inputs.
"""
import numpy as np
import pytest
import torch

from oracle import attention as oa
from tests.helpers import golden_mask, kernel_inputs

pytestmark = pytest.mark.gpu

TOL = {"bf16": 5e-3, "tf32": 5e-3, "tf32x3": 2e-5}


def _run(q, k, v, mask, scale, mode, device, with_lse=True, gather=True):
  from faster_weathernext import _lib
  from faster_weathernext import tiled_attn as ta
  dt = torch.bfloat16 if mode == "bf16" else torch.float32
  tiles = ta.AttentionTiles.from_mask(mask, device=device, gather=gather)
  m = {"bf16": _lib.MODE_BF16, "tf32": _lib.MODE_TF32, "tf32x3": _lib.MODE_TF32X3}[mode]
  tq, tk, tv = (torch.from_numpy(x).to(device=device, dtype=dt) for x in (q, k, v))
  o, lse = ta.attention_forward(tq, tk, tv, tiles, scale, m, with_lse=with_lse)
  torch.cuda.synchronize()
  assert _lib.device_error() == 0
  return o.float().cpu().numpy(), (lse.cpu().numpy() if lse is not None else None)


def _inputs_for(mode, arrays):
  return [oa.bf16_round(a) if mode == "bf16" else a for a in arrays]


@pytest.mark.parametrize("gather", [True, False])
@pytest.mark.parametrize("mode", ["bf16", "tf32"])
@pytest.mark.parametrize("batch", [1, 2])
def test_forward_reference_test_case(golden, cuda, mode, batch, gather):
  """tests/test_pallas_kernel.py:35-55 (n=300, h=2, d=64, density 0.1 + identity) on the GPU."""
  q, k, v = kernel_inputs(0, (2, 300, 2, 64), 3)
  q, k, v = q[:batch], k[:batch], v[:batch]
  m = golden_mask(golden["tiles"], "k_fwd")
  out, lse = _run(q, k, v, m, 64 ** -0.5, mode, cuda, gather=gather)
  qi, ki, vi = _inputs_for(mode, (q, k, v))
  ref, ref_lse = oa.sparse_attention(qi, ki, vi, m, 64 ** -0.5)
  assert oa.rel_rms(out, ref) < TOL[mode]
  assert oa.max_rel(out, ref) < 2e-2
  np.testing.assert_allclose(lse[:, :, :300], ref_lse, rtol=0, atol=2e-2 if mode == "bf16" else 5e-3)
  if mode == "tf32":
    a = golden["attention"]
    ev = int(a["every"])
    for b in range(batch):
      assert oa.max_rel(out[b][::ev], a[f"fwd/b{b}/out"]) < 2e-2


@pytest.mark.parametrize("mode", ["bf16", "tf32"])
def test_forward_config1(golden, cuda, mode):
  """Configuration 1: n=642, B1 H4 D64, 0.25 rad mask, Q/K/V from seed 0."""
  from faster_weathernext import mesh
  m, _, _ = mesh.config_mask(1)
  rng = np.random.default_rng(0)
  q, k, v = (rng.standard_normal((1, 642, 4, 64)).astype(np.float32) for _ in range(3))
  out, _ = _run(q, k, v, m, 0.125, mode, cuda)
  ref, _ = oa.sparse_attention(*_inputs_for(mode, (q, k, v)), m, 0.125)
  assert oa.rel_rms(out, ref) < TOL[mode]
  if mode == "tf32":
    a = golden["attention"]
    assert oa.max_rel(out[0][::int(a["every"])], a["cfg1/out"]) < 2e-2


@pytest.mark.parametrize("gather", [True, False])
@pytest.mark.parametrize("head_dim", [64, 128])
def test_forward_bf16_head_dims_and_odd_sizes(cuda, head_dim, gather):
  """n not a multiple of 64/128, H=3, non-symmetric random mask with empty query blocks."""
  from scipy import sparse
  n = 457
  m = sparse.random(n, n, density=0.05, random_state=11, format="csr").astype(bool)
  m = (m + sparse.identity(n, dtype=bool)).tocsr()
  q, k, v = kernel_inputs(5, (2, n, 3, head_dim), 3)
  out, lse = _run(q, k, v, m, head_dim ** -0.5, "bf16", cuda, gather=gather)
  ref, ref_lse = oa.sparse_attention(*_inputs_for("bf16", (q, k, v)), m, head_dim ** -0.5)
  assert oa.rel_rms(out, ref) < TOL["bf16"]
  np.testing.assert_allclose(lse[:, :, :n], ref_lse, rtol=0, atol=2e-2)


def test_forward_rows_without_keys_are_zero(cuda):
  """Rows with no allowed key (not produced by the reference's meshes) give O = 0 and LSE = -inf."""
  from scipy import sparse
  n = 200
  m = sparse.random(n, n, density=0.05, random_state=2, format="csr").astype(bool).tolil()
  m[10, :] = False
  m[150:180, :] = False
  m = m.tocsr()
  q, k, v = kernel_inputs(9, (1, n, 2, 64), 3)
  out, lse = _run(q, k, v, m, 0.125, "bf16", cuda)
  empty = np.diff(m.indptr) == 0
  assert np.all(out[0][empty] == 0)
  assert np.all(np.isneginf(lse[0][:, :n][:, empty]))
  ref, _ = oa.sparse_attention(*_inputs_for("bf16", (q, k, v)), m, 0.125)
  assert oa.rel_rms(out[0][~empty], ref[0][~empty]) < TOL["bf16"]


def test_forward_strided_input_layout(cuda):
  """q, k, v as views of one fused [B, n, H, 3, D] projection (strided heads, no copy)."""
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  m, _, _ = mesh.config_mask(1)
  x = torch.randn(1, 642, 4, 3, 64, device=cuda, dtype=torch.bfloat16)
  q, k, v = x[:, :, :, 0], x[:, :, :, 1], x[:, :, :, 2]
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  o = ta.attention(q, k, v, tiles, scale=0.125)
  ref, _ = oa.sparse_attention(*(t.float().cpu().numpy() for t in (q, k, v)), m, 0.125)
  assert oa.rel_rms(o.float().cpu().numpy(), ref) < TOL["bf16"]


@pytest.mark.parametrize("cfg,mode,gather", [(2, "bf16", True), (3, "bf16", True), (3, "tf32", True),
                                             (3, "bf16", False)])
def test_forward_full_size_configs(cuda, cfg, mode, gather):
  """Configurations 2 and 3 at full size (oracle on the allowed pairs only)."""
  from faster_weathernext import mesh
  m, _, _ = mesh.config_mask(cfg)
  _, _, b, h, d = mesh.CONFIGS[cfg]
  n = m.shape[0]
  rng = np.random.default_rng(0)
  q, k, v = (rng.standard_normal((b, n, h, d)).astype(np.float32) for _ in range(3))
  out, lse = _run(q, k, v, m, d ** -0.5, mode, cuda, gather=gather)
  ref, ref_lse = oa.sparse_attention(*_inputs_for(mode, (q, k, v)), m, d ** -0.5)
  assert oa.rel_rms(out, ref) < TOL[mode]
  assert np.abs(lse[:, :, :n] - ref_lse).max() < 5e-2


def test_forward_head_major_layout_gathered(cuda):
  """q, k, v as [B, n, H, D] views of head-major [B, H, n, D] storage: gathered rows use (b, h, node)."""
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  m, _, _ = mesh.config_mask(1)
  x = torch.randn(3, 2, 4, 642, 64, device=cuda, dtype=torch.bfloat16)
  q, k, v = (x[i].transpose(1, 2) for i in range(3))
  assert ta._gather_layout(q) == 1
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  o = ta.attention(q, k, v, tiles, scale=0.125)
  ref, _ = oa.sparse_attention(*(t.float().cpu().numpy() for t in (q, k, v)), m, 0.125)
  assert oa.rel_rms(o.float().cpu().numpy(), ref) < TOL["bf16"]


@pytest.mark.parametrize("gather", [True, False])
@pytest.mark.parametrize("batch", [1, 2])
def test_forward_tf32x3_reference_test_case(golden, cuda, batch, gather):
  """The fp32-equivalent mode (3xTF32, the reference's `highest`): rel RMS <= 2e-5 and the reference test's
  max|err| / max|ref| < 1e-5 (tests/test_pallas_kernel.py:36) against the float64 reference."""
  q, k, v = kernel_inputs(0, (2, 300, 2, 64), 3)
  q, k, v = q[:batch], k[:batch], v[:batch]
  m = golden_mask(golden["tiles"], "k_fwd")
  out, lse = _run(q, k, v, m, 64 ** -0.5, "tf32x3", cuda, gather=gather)
  ref, ref_lse = oa.sparse_attention(q, k, v, m, 64 ** -0.5)
  assert oa.rel_rms(out, ref) < TOL["tf32x3"]
  assert oa.max_rel(out, ref) < 1e-5
  np.testing.assert_allclose(lse[:, :, :300], ref_lse, rtol=0, atol=1e-5)
  gold = golden["attention"]
  for b in range(batch):
    assert oa.max_rel(out[b][::int(gold["every"])], gold[f"fwd/b{b}/out"]) < 1e-5


@pytest.mark.parametrize("cfg", [1, 3])
def test_forward_tf32x3_configs(cuda, cfg):
  from faster_weathernext import mesh
  m, _, _ = mesh.config_mask(cfg)
  _, _, b, h, d = mesh.CONFIGS[cfg]
  rng = np.random.default_rng(0)
  q, k, v = (rng.standard_normal((b, m.shape[0], h, d)).astype(np.float32) for _ in range(3))
  out, _ = _run(q, k, v, m, d ** -0.5, "tf32x3", cuda)
  ref, _ = oa.sparse_attention(q, k, v, m, d ** -0.5)
  assert oa.rel_rms(out, ref) < TOL["tf32x3"]


def _khop_mask(level, hops):
  from faster_weathernext import mesh
  xyz, faces = mesh.icosphere(level)
  lat, lon = mesh.latlon(xyz)
  adj = mesh.permute(mesh.adjacency(faces, xyz.shape[0]), mesh.morton_order(lat, lon))
  return mesh.k_hop_mask(adj, hops)


@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("kernel", ["wide", "narrow"])
def test_forward_dense_mask_both_kernels(cuda, head_dim, kernel):
  """Dense neighbourhood mask (level-4 mesh, 6 hops: ~127 keys per query, > 16 tiles per block): the
  wide-chunk kernel (32-key tile lists) and the narrow kernel (gathered lists through the C ABI)."""
  import ctypes
  from faster_weathernext import _lib
  from faster_weathernext import tiled_attn as ta
  m = _khop_mask(4, 6)
  n = m.shape[0]
  q, k, v = kernel_inputs(21, (2, n, 3, head_dim), 3)
  tiles = ta.AttentionTiles.from_mask(m, device=cuda, gather=True)
  assert tiles.fwd.n_tiles >= 16 * tiles.fwd.n_blocks
  tq, tk, tv = (torch.from_numpy(x).to(device=cuda, dtype=torch.bfloat16) for x in (q, k, v))
  lib = _lib.lib()
  o = torch.empty_like(tq)
  lse = torch.empty(2, 3, lib.fwn_lse_rows(n), device=cuda)
  desc = ta._desc(tq, o, head_dim ** -0.5, _lib.MODE_BF16)
  st = (tiles.fwd if kernel == "wide" else tiles.fwd_g).struct()
  _lib.check(lib.fwn_attn_fwd(ctypes.byref(desc), tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), ctypes.byref(st),
                              o.data_ptr(), lse.data_ptr(), 0))
  torch.cuda.synchronize()
  assert _lib.device_error() == 0
  ref, ref_lse = oa.sparse_attention(*_inputs_for("bf16", (q, k, v)), m, head_dim ** -0.5)
  assert oa.rel_rms(o.float().cpu().numpy(), ref) < TOL["bf16"]
  np.testing.assert_allclose(lse.cpu().numpy()[:, :, :n], ref_lse, rtol=0, atol=2e-2)


@pytest.mark.parametrize("head_dim", [64, 128])
def test_forward_dense_growing_logits_rescale(cuda, head_dim):
  """Logits that grow along the key order by several powers of two per chunk: the one-pass softmax must
  fall back to the exact two-pass update and rescale O in TMEM (wide kernel)."""
  m = _khop_mask(4, 6)
  n = m.shape[0]
  rng = np.random.default_rng(3)
  u = rng.standard_normal(head_dim).astype(np.float32)
  u /= np.linalg.norm(u)
  ramp = (np.arange(n, dtype=np.float32) / n * 4000.0)[:, None]
  q = np.broadcast_to(u * 3.0, (1, n, 2, head_dim)).copy() + 0.05 * rng.standard_normal((1, n, 2, head_dim)).astype(np.float32)
  k = (ramp * u)[None, :, None, :].repeat(2, axis=2) * head_dim ** 0.5 / 3.0 / 40.0
  v = rng.standard_normal((1, n, 2, head_dim)).astype(np.float32)
  out, lse = _run(q, k.astype(np.float32), v, m, head_dim ** -0.5, "bf16", cuda, gather=False)
  ref, ref_lse = oa.sparse_attention(*_inputs_for("bf16", (q, k.astype(np.float32), v)), m, head_dim ** -0.5)
  assert oa.rel_rms(out, ref) < TOL["bf16"]
  np.testing.assert_allclose(lse[:, :, :n], ref_lse, rtol=2e-3, atol=5e-2)
