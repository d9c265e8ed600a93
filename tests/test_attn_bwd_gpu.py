"""GPU: backward kernels (delta, dQ over the forward list, dK/dV over the transposed list) against the
oracle's analytic float64 gradient (tests/test_pallas_kernel.py:58-69) and the golden vectors.

Tolerances: rel RMS <= 5e-3 in bf16 / TF32 (the stated bound for outputs and dQ/dK/dV), and for TF32
the reference test's max-abs metric max|err| / max|ref| < 3e-2 (tests/test_pallas_kernel.py:98).
"""
import numpy as np
import pytest
import torch
from scipy import sparse

from oracle import attention as oa
from tests.helpers import golden_mask, kernel_inputs

pytestmark = pytest.mark.gpu

TOL = {"bf16": 5e-3, "tf32": 5e-3, "tf32x3": 2e-5}


def _grads(q, k, v, do, mask, scale, mode, device, tiles=None, gather=True):
  from faster_weathernext import _lib
  from faster_weathernext import tiled_attn as ta
  dt = torch.bfloat16 if mode == "bf16" else torch.float32
  if tiles is None:
    tiles = ta.AttentionTiles.from_mask(mask, device=device, gather=gather)
  m = {"bf16": _lib.MODE_BF16, "tf32": _lib.MODE_TF32, "tf32x3": _lib.MODE_TF32X3}[mode]
  tq, tk, tv, tdo = (torch.from_numpy(x).to(device=device, dtype=dt) for x in (q, k, v, do))
  o, lse = ta.attention_forward(tq, tk, tv, tiles, scale, m, with_lse=True)
  dq, dk, dv = ta.attention_backward(tq, tk, tv, o, lse, tdo, tiles, scale, m)
  torch.cuda.synchronize()
  assert _lib.device_error() == 0
  return [x.float().cpu().numpy() for x in (dq, dk, dv)]


def _rounded(mode, arrays):
  return [oa.bf16_round(a) if mode == "bf16" else a for a in arrays]


@pytest.mark.parametrize("gather", [True, False])
@pytest.mark.parametrize("mode", ["bf16", "tf32"])
@pytest.mark.parametrize("symmetric", [True, False])
@pytest.mark.parametrize("batch", [1, 2])
def test_grads_reference_test_case(golden, cuda, mode, symmetric, batch, gather):
  """tests/test_pallas_kernel.py:72-99: n=300 (padding rows), h=2, d=64, density 0.08, sym / non-sym."""
  q, k, v, do = kernel_inputs(2, (1, 300, 2, 64), 4)
  if batch == 2:
    q2, k2, v2, do2 = kernel_inputs(12, (1, 300, 2, 64), 4)
    q, k, v, do = (np.concatenate([a, b]) for a, b in zip((q, k, v, do), (q2, k2, v2, do2)))
  m = golden_mask(golden["tiles"], "k_sym" if symmetric else "k_nonsym")
  got = _grads(q, k, v, do, m, 0.125, mode, cuda, gather=gather)
  ref = oa.sparse_attention_vjp(*_rounded(mode, (q, k, v, do)), m, 0.125)
  for name, a, r in zip(("dq", "dk", "dv"), got, ref):
    assert oa.rel_rms(a, r) < TOL[mode], (name, oa.rel_rms(a, r))
    assert oa.max_rel(a, r) < 3e-2, (name, oa.max_rel(a, r))
  if mode == "tf32":
    gold = golden["attention"]
    ev = int(gold["every"])
    tag = "sym" if symmetric else "nonsym"
    for name, a in zip(("dq", "dk", "dv"), got):
      assert oa.max_rel(a[0][::ev], gold[f"grad_{tag}/{name}"]) < 3e-2, name


def test_nonsymmetric_mask_needs_transposed_tiles(golden, cuda):
  """tests/test_pallas_kernel.py:102-118: reusing the forward list for dK/dV of a non-symmetric mask is wrong."""
  from faster_weathernext import tiled_attn as ta
  q, k, v, do = kernel_inputs(4, (1, 130, 1, 32), 4)
  # head_dim 32 is not built: pad the head dimension with zeros (identical logits and outputs).
  pad = lambda x: np.concatenate([x, np.zeros(x.shape[:-1] + (32,), np.float32)], -1)
  q, k, v, do = (pad(x) for x in (q, k, v, do))
  m = golden_mask(golden["tiles"], "k_guard")
  scale = 32 ** -0.5
  good = ta.AttentionTiles.from_mask(m, device=cuda, gather=False)
  wrong = ta.AttentionTiles(good.fwd, good.fwd, 130, True, gather=False)
  ref_dk = golden["attention"]["guard/dk"]
  _, dk_good, _ = _grads(q, k, v, do, m, scale, "tf32", cuda, tiles=good)
  _, dk_bad, _ = _grads(q, k, v, do, m, scale, "tf32", cuda, tiles=wrong)
  assert oa.max_rel(dk_good[0][..., :32], ref_dk) < 3e-2
  assert oa.max_rel(dk_bad[0][..., :32], ref_dk) > 1e-2


@pytest.mark.parametrize("mode", ["bf16", "tf32"])
def test_grads_config1(golden, cuda, mode):
  """Configuration 1 VJP (upstream gradient from seed 1) against the reference's float64 gradient."""
  from faster_weathernext import mesh
  m, _, _ = mesh.config_mask(1)
  rng = np.random.default_rng(0)
  q, k, v = (rng.standard_normal((1, 642, 4, 64)).astype(np.float32) for _ in range(3))
  do = np.random.default_rng(1).standard_normal((1, 642, 4, 64)).astype(np.float32)
  got = _grads(q, k, v, do, m, 0.125, mode, cuda)
  ref = oa.sparse_attention_vjp(*_rounded(mode, (q, k, v, do)), m, 0.125)
  for name, a, r in zip(("dq", "dk", "dv"), got, ref):
    assert oa.rel_rms(a, r) < TOL[mode], (name, oa.rel_rms(a, r))
  if mode == "tf32":
    gold = golden["attention"]
    for name, a in zip(("dq", "dk", "dv"), got):
      assert oa.max_rel(a[0][::int(gold["every"])], gold[f"cfg1/{name}"]) < 3e-2, name


@pytest.mark.parametrize("gather", [True, False])
@pytest.mark.parametrize("head_dim", [64, 128])
def test_grads_bf16_odd_sizes_nonsymmetric(cuda, head_dim, gather):
  n = 457
  m = sparse.random(n, n, density=0.05, random_state=11, format="csr").astype(bool)
  m = (m + sparse.identity(n, dtype=bool)).tocsr()
  q, k, v, do = kernel_inputs(6, (2, n, 3, head_dim), 4)
  got = _grads(q, k, v, do, m, head_dim ** -0.5, "bf16", cuda, gather=gather)
  ref = oa.sparse_attention_vjp(*_rounded("bf16", (q, k, v, do)), m, head_dim ** -0.5)
  for name, a, r in zip(("dq", "dk", "dv"), got, ref):
    assert oa.rel_rms(a, r) < TOL["bf16"], (name, oa.rel_rms(a, r))


@pytest.mark.parametrize("mode,gather", [("bf16", True), ("tf32", True), ("bf16", False)])
def test_grads_full_size_config3(cuda, mode, gather):
  from faster_weathernext import mesh
  m, _, _ = mesh.config_mask(3)
  n = m.shape[0]
  rng = np.random.default_rng(0)
  q, k, v = (rng.standard_normal((1, n, 8, 64)).astype(np.float32) for _ in range(3))
  do = np.random.default_rng(1).standard_normal((1, n, 8, 64)).astype(np.float32)
  got = _grads(q, k, v, do, m, 0.125, mode, cuda, gather=gather)
  ref = oa.sparse_attention_vjp(*_rounded(mode, (q, k, v, do)), m, 0.125)
  for name, a, r in zip(("dq", "dk", "dv"), got, ref):
    assert oa.rel_rms(a, r) < TOL[mode], (name, oa.rel_rms(a, r))


def test_autograd_matches_explicit_backward(cuda):
  """torch.autograd through attention() (the custom-VJP analogue) gives the kernels' gradients."""
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  m, _, _ = mesh.config_mask(1)
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  g = torch.Generator(device=cuda).manual_seed(0)
  q, k, v, do = (torch.randn(1, 642, 4, 64, device=cuda, generator=g, dtype=torch.bfloat16) for _ in range(4))
  qq, kk, vv = (x.clone().requires_grad_(True) for x in (q, k, v))
  out = ta.attention(qq, kk, vv, tiles, scale=0.125)
  out.backward(do)
  ref = oa.sparse_attention_vjp(*(x.float().cpu().numpy() for x in (q, k, v, do)), m, 0.125)
  for t, r in zip((qq.grad, kk.grad, vv.grad), ref):
    assert oa.rel_rms(t.float().cpu().numpy(), r) < TOL["bf16"]


@pytest.mark.parametrize("gather", [True, False])
@pytest.mark.parametrize("symmetric", [True, False])
@pytest.mark.parametrize("batch", [1, 2])
def test_grads_tf32x3_reference_test_case(golden, cuda, symmetric, batch, gather):
  """fp32-equivalent backward (3xTF32: delta, dQ, then dV and dK as separate passes): rel RMS <= 2e-5 against
  the float64 VJP on the reference test's case (tests/test_pallas_kernel.py:72-99), max|err| / max|ref| < 1e-4."""
  q, k, v, do = kernel_inputs(2, (1, 300, 2, 64), 4)
  if batch == 2:
    q2, k2, v2, do2 = kernel_inputs(12, (1, 300, 2, 64), 4)
    q, k, v, do = (np.concatenate([a, b]) for a, b in zip((q, k, v, do), (q2, k2, v2, do2)))
  m = golden_mask(golden["tiles"], "k_sym" if symmetric else "k_nonsym")
  got = _grads(q, k, v, do, m, 0.125, "tf32x3", cuda, gather=gather)
  ref = oa.sparse_attention_vjp(q, k, v, do, m, 0.125)
  for name, a, r in zip(("dq", "dk", "dv"), got, ref):
    assert oa.rel_rms(a, r) < TOL["tf32x3"], (name, oa.rel_rms(a, r))
    assert oa.max_rel(a, r) < 1e-4, (name, oa.max_rel(a, r))
  gold = golden["attention"]
  tag = "sym" if symmetric else "nonsym"
  for name, a in zip(("dq", "dk", "dv"), got):
    assert oa.max_rel(a[0][::int(gold["every"])], gold[f"grad_{tag}/{name}"]) < 1e-4, name


@pytest.mark.parametrize("cfg", [1, 3])
def test_grads_tf32x3_configs(cuda, cfg):
  """Configurations 1 and 3 (full size) in the fp32-equivalent mode: rel RMS <= 2e-5 per gradient."""
  from faster_weathernext import mesh
  m, _, _ = mesh.config_mask(cfg)
  _, _, b, h, d = mesh.CONFIGS[cfg]
  n = m.shape[0]
  rng = np.random.default_rng(0)
  q, k, v = (rng.standard_normal((b, n, h, d)).astype(np.float32) for _ in range(3))
  do = np.random.default_rng(1).standard_normal((b, n, h, d)).astype(np.float32)
  got = _grads(q, k, v, do, m, d ** -0.5, "tf32x3", cuda)
  ref = oa.sparse_attention_vjp(q, k, v, do, m, d ** -0.5)
  for name, a, r in zip(("dq", "dk", "dv"), got, ref):
    assert oa.rel_rms(a, r) < TOL["tf32x3"], (name, oa.rel_rms(a, r))


def _khop_mask(level, hops):
  from faster_weathernext import mesh
  xyz, faces = mesh.icosphere(level)
  lat, lon = mesh.latlon(xyz)
  adj = mesh.permute(mesh.adjacency(faces, xyz.shape[0]), mesh.morton_order(lat, lon))
  return mesh.k_hop_mask(adj, hops)


@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("mask_kind", ["khop", "random_nonsym"])
def test_grads_dense_masks_wide_passes(cuda, head_dim, mask_kind):
  """Dense masks (> 16 tiles per 128-row block): the wide-chunk dQ / dV / dK passes, batch 2, H 3, ragged n."""
  if mask_kind == "khop":
    m = _khop_mask(4, 6)
  else:
    n = 700
    m = sparse.random(n, n, density=0.3, random_state=5, format="csr").astype(bool)
    m = (m + sparse.identity(n, dtype=bool)).tocsr()
  n = m.shape[0]
  q, k, v, do = kernel_inputs(31, (2, n, 3, head_dim), 4)
  got = _grads(q, k, v, do, m, head_dim ** -0.5, "bf16", cuda, gather=False)
  ref = oa.sparse_attention_vjp(*_rounded("bf16", (q, k, v, do)), m, head_dim ** -0.5)
  for name, a, r in zip(("dq", "dk", "dv"), got, ref):
    assert oa.rel_rms(a, r) < TOL["bf16"], (name, oa.rel_rms(a, r))


@pytest.mark.parametrize("mask_kind", ["ref_sym", "ref_nonsym", "khop"])
def test_tf32_head_dim_128(golden, cuda, mask_kind):
  """TF32 at head_dim 128 (the WeatherNext 2 head size in the reference's default precision): forward and
  gradients within 5e-3 rel RMS and the reference test's max-abs bounds (2e-2 output, 3e-2 gradients)."""
  from faster_weathernext import _lib
  from faster_weathernext import tiled_attn as ta
  if mask_kind == "khop":
    m = _khop_mask(4, 6)
  else:
    m = golden_mask(golden["tiles"], "k_sym" if mask_kind == "ref_sym" else "k_nonsym")
  n = m.shape[0]
  q, k, v, do = kernel_inputs(41, (2, n, 2, 128), 4)
  scale = 128 ** -0.5
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  tq, tk, tv, tdo = (torch.from_numpy(x).to(cuda) for x in (q, k, v, do))
  o, lse = ta.attention_forward(tq, tk, tv, tiles, scale, _lib.MODE_TF32, with_lse=True)
  dq, dk, dv = ta.attention_backward(tq, tk, tv, o, lse, tdo, tiles, scale, _lib.MODE_TF32)
  torch.cuda.synchronize()
  assert _lib.device_error() == 0
  ref_o, _ = oa.sparse_attention(q, k, v, m, scale)
  assert oa.rel_rms(o.cpu().numpy(), ref_o) < TOL["tf32"]
  assert oa.max_rel(o.cpu().numpy(), ref_o) < 2e-2
  ref = oa.sparse_attention_vjp(q, k, v, do, m, scale)
  for name, a, r in zip(("dq", "dk", "dv"), (dq, dk, dv), ref):
    a = a.cpu().numpy()
    assert oa.rel_rms(a, r) < TOL["tf32"], (name, oa.rel_rms(a, r))
    assert oa.max_rel(a, r) < 3e-2, (name, oa.max_rel(a, r))


@pytest.mark.parametrize("mask_kind", ["khop", "ref_nonsym"])
@pytest.mark.parametrize("gather", [True, False])
def test_tf32x3_head_dim_128(golden, cuda, mask_kind, gather):
  """3xTF32 at head_dim 128 (the WeatherNext 2 head size in the fp32-equivalent mode; Q / the first row operand in
  TMEM as hi and lo copies): forward and gradients within 2e-5 rel RMS of the float64 reference, and the reference
  test's max-abs bounds (1e-5 output, 1e-4 gradients, tests/test_pallas_kernel.py:36, 98)."""
  from faster_weathernext import _lib
  from faster_weathernext import tiled_attn as ta
  if mask_kind == "khop":
    m = _khop_mask(4, 6)
  else:
    m = golden_mask(golden["tiles"], "k_nonsym")
  n = m.shape[0]
  q, k, v, do = kernel_inputs(43, (2, n, 2, 128), 4)
  scale = 128 ** -0.5
  tiles = ta.AttentionTiles.from_mask(m, device=cuda, gather=gather)
  tq, tk, tv, tdo = (torch.from_numpy(x).to(cuda) for x in (q, k, v, do))
  o, lse = ta.attention_forward(tq, tk, tv, tiles, scale, _lib.MODE_TF32X3, with_lse=True)
  dq, dk, dv = ta.attention_backward(tq, tk, tv, o, lse, tdo, tiles, scale, _lib.MODE_TF32X3)
  torch.cuda.synchronize()
  assert _lib.device_error() == 0
  ref_o, _ = oa.sparse_attention(q, k, v, m, scale)
  assert oa.rel_rms(o.cpu().numpy(), ref_o) < TOL["tf32x3"]
  assert oa.max_rel(o.cpu().numpy(), ref_o) < 1e-5
  ref = oa.sparse_attention_vjp(q, k, v, do, m, scale)
  for name, a, r in zip(("dq", "dk", "dv"), (dq, dk, dv), ref):
    a = a.cpu().numpy()
    assert oa.rel_rms(a, r) < TOL["tf32x3"], (name, oa.rel_rms(a, r))
    assert oa.max_rel(a, r) < 1e-4, (name, oa.max_rel(a, r))


@pytest.mark.parametrize("head_dim", [64, 128])
def test_autograd_fused_qkv_layout_dense_mask(cuda, head_dim):
  """Gradients through the public API (tiled_attn.attention + autograd) with q, k, v as strided views of one
  fused [B, n, H, 3, D] projection (the processor's layout) on a dense k-hop mask: the wide dQ and one-pass dK / dV
  kernels read the strided rows and write the gradients into the fused tensor's gradient."""
  from faster_weathernext import tiled_attn as ta
  m = _khop_mask(4, 6)
  n = m.shape[0]
  g = torch.Generator(device=cuda).manual_seed(11)
  x = torch.randn(2, n, 2, 3, head_dim, device=cuda, generator=g).to(torch.bfloat16).requires_grad_(True)
  do = torch.randn(2, n, 2, head_dim, device=cuda, generator=g).to(torch.bfloat16)
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  o = ta.attention(x[:, :, :, 0], x[:, :, :, 1], x[:, :, :, 2], tiles, scale=head_dim ** -0.5)
  (gx,) = torch.autograd.grad(o, x, do)
  torch.cuda.synchronize()
  q, k, v = (x[:, :, :, i].detach().float().cpu().numpy() for i in range(3))
  ref = oa.sparse_attention_vjp(q, k, v, do.float().cpu().numpy(), m, head_dim ** -0.5)
  got = gx.float().cpu().numpy()
  for i, name in enumerate(("dq", "dk", "dv")):
    assert oa.rel_rms(got[:, :, :, i], ref[i]) < TOL["bf16"], (name, oa.rel_rms(got[:, :, :, i], ref[i]))


@pytest.mark.parametrize("mode", ["bf16", "tf32"])
@pytest.mark.parametrize("mask_kind", ["ref_nonsym", "khop"])
@pytest.mark.parametrize("head_dim", [64, 128])
def test_attention_qkv_writes_the_fused_gradient_in_place(golden, cuda, mode, mask_kind, head_dim):
  """tiled_attn.attention_qkv (the backward writes dq, dk, dv into one [B, n, H, 3, D] gradient through
  FWN_DESC_GRAD_STRIDES) gives bit-identical outputs and gradients to attention() on the three slices (the same
  kernels, whose per-slice gradients autograd assembles), and the gradient matches the oracle's VJP."""
  from faster_weathernext import _lib
  from faster_weathernext import tiled_attn as ta
  if mask_kind == "khop":
    m = _khop_mask(4, 6)
  else:
    m = golden_mask(golden["tiles"], "k_nonsym")
  n = m.shape[0]
  dt = torch.bfloat16 if mode == "bf16" else torch.float32
  g = torch.Generator(device=cuda).manual_seed(21)
  x = torch.randn(2, n, 2, 3, head_dim, device=cuda, generator=g).to(dt)
  do = torch.randn(2, n, 2, head_dim, device=cuda, generator=g).to(dt)
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  scale = head_dim ** -0.5
  xa = x.clone().requires_grad_(True)
  oa_ = ta.attention_qkv(xa, tiles, scale=scale)
  (ga,) = torch.autograd.grad(oa_, xa, do)
  xb = x.clone().requires_grad_(True)
  ob = ta.attention(xb[:, :, :, 0], xb[:, :, :, 1], xb[:, :, :, 2], tiles, scale=scale)
  (gb,) = torch.autograd.grad(ob, xb, do)
  torch.cuda.synchronize()
  assert _lib.device_error() == 0
  assert torch.equal(oa_, ob)
  assert torch.equal(ga, gb)
  q, k, v = (x[:, :, :, i].float().cpu().numpy() for i in range(3))
  ref = oa.sparse_attention_vjp(q, k, v, do.float().cpu().numpy(), m, scale)
  got = ga.float().cpu().numpy()
  for i, name in enumerate(("dq", "dk", "dv")):
    assert oa.rel_rms(got[:, :, :, i], ref[i]) < TOL[mode], (name, oa.rel_rms(got[:, :, :, i], ref[i]))
