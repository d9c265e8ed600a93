"""GPU: the processor (configurations 4-5 structure) and the fine-tune step with the B200 attention, against
the same processor whose attention is a dense float32 masked softmax in torch (test-only subclass).
Tolerances: the processor computes in bf16 (projections, attention), so rel RMS <= 2e-2 for outputs and
<= 5e-2 for the global relative L2 error of all parameter gradients."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _small():
  from faster_weathernext.processor import ProcessorConfig
  return ProcessorConfig(layers=2, d_model=128, heads=2, head_dim=64, mlp_hidden=256, cond_dim=8)


def _dense_processor_class(mask_dense):
  from faster_weathernext.processor import Processor

  class DenseProcessor(Processor):
    def _mha(self, h, w_qkv, w_out, tiles):
      """patch.tiled_mha restated with a dense float32 masked softmax (patch.py:165-177)."""
      cfg = self.cfg
      b, n, _ = h.shape
      qkv = (h @ w_qkv).view(b, n, cfg.heads, 3, cfg.head_dim)
      qf, kf, vf = (qkv[:, :, :, i].float().permute(0, 2, 1, 3) for i in range(3))   # [B, H, n, D]
      s = (qf @ kf.transpose(-1, -2)) * cfg.head_dim ** -0.5
      s = s.masked_fill(~mask_dense, float("-inf"))
      o = (torch.softmax(s, -1) @ vf).permute(0, 2, 1, 3).to(h.dtype)
      return o.reshape(b, n, -1) @ w_out
  return DenseProcessor


def _rel(a, b):
  a, b = a.double(), b.double()
  return float(torch.sqrt(torch.mean((a - b) ** 2)) / b.std())


def test_processor_forward_and_gradients_match_dense_reference(cuda):
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  from faster_weathernext.processor import Processor
  m, _, _ = mesh.config_mask(1)
  n = m.shape[0]
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  mask_dense = torch.from_numpy(m.toarray()).to(cuda)
  cfg = _small()
  ours = Processor(cfg, seed=3, device=cuda)
  ref = _dense_processor_class(mask_dense)(cfg, seed=3, device=cuda)
  g = torch.Generator(device=cuda).manual_seed(5)
  x = torch.randn(2, n, cfg.d_model, device=cuda, generator=g)
  c = torch.randn(2, cfg.cond_dim, device=cuda, generator=g)
  t = torch.randn(2, n, cfg.d_model, device=cuda, generator=g)
  ya, yb = ours(x, c, tiles), ref(x, c, tiles)
  assert _rel(ya, yb) < 2e-2
  torch.nn.functional.mse_loss(ya, t).backward()
  torch.nn.functional.mse_loss(yb, t).backward()
  ga = torch.cat([p.grad.reshape(-1) for p in ours.parameters()])
  gb = torch.cat([p.grad.reshape(-1) for p in ref.parameters()])
  assert float((ga - gb).norm() / gb.norm()) < 5e-2


def test_finetune_step_runs_and_lowers_the_loss(cuda):
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  from faster_weathernext.finetune import DataParallelStep
  from faster_weathernext.processor import Processor
  m, _, _ = mesh.config_mask(1)
  n = m.shape[0]
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  cfg = _small()
  model = Processor(cfg, seed=0, device=cuda)
  step = DataParallelStep(model, members=2, lr=1e-3)
  g = torch.Generator(device=cuda).manual_seed(1)
  xs = [torch.randn(1, n, cfg.d_model, device=cuda, generator=g) for _ in range(2)]
  cs = [torch.randn(1, cfg.cond_dim, device=cuda, generator=g) for _ in range(2)]
  ts = [torch.randn(1, n, cfg.d_model, device=cuda, generator=g) for _ in range(2)]
  losses = [float(step.step(xs, cs, ts, forward=lambda x, c: model(x, c, tiles))) for _ in range(4)]
  assert all(np.isfinite(losses)) and losses[-1] < losses[0]


def test_processor_fused_inference_matches_autograd_path(cuda):
  """The inference path (fused conditioned LayerNorm kernel, GEMM-epilogue bias + GELU, in-place residual) gives
  the autograd path's output within bf16 rounding (rel RMS <= 1e-2), at the configurations' width."""
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  from faster_weathernext.processor import Processor, ProcessorConfig
  m, _, _ = mesh.config_mask(1)
  n = m.shape[0]
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  cfg = ProcessorConfig(layers=3)
  model = Processor(cfg, seed=4, device=cuda)
  g = torch.Generator(device=cuda).manual_seed(6)
  x = torch.randn(2, n, cfg.d_model, device=cuda, generator=g)
  c = torch.randn(2, cfg.cond_dim, device=cuda, generator=g)
  y_grad = model(x, c, tiles)
  with torch.no_grad():
    y_fused = model(x, c, tiles)
  assert _rel(y_fused, y_grad.detach()) < 1e-2


def test_cond_layernorm_kernel_matches_torch(cuda):
  """fwn_cond_layernorm against torch: LayerNorm (eps 1e-5) * (1 + scale) + offset per sample, bf16 and fp32."""
  from faster_weathernext import _lib
  lib = _lib.lib()
  g = torch.Generator(device=cuda).manual_seed(0)
  for d in (128, 512, 1024):
    b, n = 3, 257
    x = torch.randn(b * n, d, device=cuda, generator=g) * 3 + 1
    so = torch.randn(b, 2 * d, device=cuda, generator=g) * 0.2
    ref = torch.nn.functional.layer_norm(x.view(b, n, d), (d,))
    ref = (ref * (1 + so[:, None, :d]) + so[:, None, d:]).view(b * n, d)
    for dt, tol in ((_lib.DTYPE_F32, 1e-5), (_lib.DTYPE_BF16, 1e-2)):
      out = torch.empty(b * n, d, device=cuda, dtype=torch.float32 if dt == _lib.DTYPE_F32 else torch.bfloat16)
      _lib.check(lib.fwn_cond_layernorm(x.data_ptr(), b * n, d, n, so.data_ptr(), 1e-5, out.data_ptr(), dt, 0))
      torch.cuda.synchronize()
      assert float((out.float() - ref).abs().max() / ref.abs().max()) < tol, (d, dt)


def test_cond_layernorm_scatter_kernel(cuda):
  """fwn_cond_layernorm_scatter: the conditioned norm with row i of each sample stored at row out_node[i]
  (the un-permutation after the final norm, patch.py:291-292), bit-equal to the plain kernel followed by the
  scatter; an out-of-range entry drops its row."""
  from faster_weathernext import _lib
  lib = _lib.lib()
  g = torch.Generator(device=cuda).manual_seed(2)
  b, n, d = 2, 300, 512
  x = torch.randn(b * n, d, device=cuda, generator=g)
  so = torch.randn(b, 2 * d, device=cuda, generator=g) * 0.2
  perm = torch.randperm(n, device=cuda, generator=g).to(torch.int32)
  plain = torch.empty(b * n, d, device=cuda)
  _lib.check(lib.fwn_cond_layernorm(x.data_ptr(), b * n, d, n, so.data_ptr(), 1e-5, plain.data_ptr(),
                                    _lib.DTYPE_F32, 0))
  out = torch.full((b * n, d), 7.0, device=cuda)
  _lib.check(lib.fwn_cond_layernorm_scatter(x.data_ptr(), b * n, d, n, perm.data_ptr(), so.data_ptr(), 1e-5,
                                            out.data_ptr(), _lib.DTYPE_F32, 0))
  expected = torch.empty_like(plain).view(b, n, d)
  expected[:, perm.long()] = plain.view(b, n, d)
  torch.cuda.synchronize()
  assert torch.equal(out.view(b, n, d), expected)
  # An entry outside [0, n) drops its row; the row it would have replaced keeps its old content.
  bad = perm.clone()
  victim = int(bad[5])
  bad[5] = n + 3
  out2 = torch.full((b * n, d), 7.0, device=cuda)
  _lib.check(lib.fwn_cond_layernorm_scatter(x.data_ptr(), b * n, d, n, bad.data_ptr(), so.data_ptr(), 1e-5,
                                            out2.data_ptr(), _lib.DTYPE_F32, 0))
  torch.cuda.synchronize()
  assert torch.all(out2.view(b, n, d)[:, victim] == 7.0)
  assert _lib.lib().fwn_cond_layernorm_scatter(x.data_ptr(), b * n, d, n, None, so.data_ptr(), 1e-5,
                                               out2.data_ptr(), _lib.DTYPE_F32, 0) != 0


def test_processor_node_permutation(cuda):
  """forward(x, perm=perm) = forward(x[:, perm])[:, argsort(perm)] (patch.py:275-276, 291-292): bit-equal on the
  inference path (gather as the residual copy, un-permutation fused into the final norm), and the autograd
  path agrees within bf16 rounding."""
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  from faster_weathernext.processor import Processor, ProcessorConfig
  m, _, _ = mesh.config_mask(1)
  n = m.shape[0]
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  cfg = ProcessorConfig(layers=2)
  model = Processor(cfg, seed=7, device=cuda)
  g = torch.Generator(device=cuda).manual_seed(8)
  x = torch.randn(2, n, cfg.d_model, device=cuda, generator=g)
  c = torch.randn(2, cfg.cond_dim, device=cuda, generator=g)
  perm = torch.randperm(n, device=cuda, generator=g)
  inv = torch.argsort(perm)
  with torch.no_grad():
    y_perm = model(x, c, tiles, perm=perm)
    y_ref = model(x[:, perm], c, tiles)[:, inv]
  assert torch.equal(y_perm, y_ref)
  y_grad = model(x, c, tiles, perm=perm)
  assert _rel(y_grad.detach(), y_ref) < 1e-2
  with pytest.raises(ValueError):
    model(x, c, tiles, perm=perm[:-1])


def test_processor_fused_weight_cache_follows_updates(cuda):
  """The inference path casts each weight to bf16 once and reuses the copy across calls; an in-place update of
  a parameter (as an optimizer step makes) must be seen by the next call."""
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  from faster_weathernext.processor import Processor, ProcessorConfig
  m, _, _ = mesh.config_mask(1)
  n = m.shape[0]
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  cfg = ProcessorConfig(layers=2)
  model = Processor(cfg, seed=5, device=cuda)
  g = torch.Generator(device=cuda).manual_seed(7)
  x = torch.randn(1, n, cfg.d_model, device=cuda, generator=g)
  c = torch.randn(1, cfg.cond_dim, device=cuda, generator=g)
  with torch.no_grad():
    y0 = model(x, c, tiles)
    assert torch.equal(model(x, c, tiles), y0)                    # cached copies: same result
    model.blocks[1].w2.mul_(-2.0)
    model.blocks[0].b1.add_(0.5)
    y1 = model(x, c, tiles)
  y_ref = model(x, c, tiles)                                       # autograd path, no cache
  assert not torch.equal(y1, y0)
  assert _rel(y1, y_ref.detach()) < 1e-2


def test_processor_input_checks(cuda):
  """The fused inference path runs only on float32 residual streams (it reads and writes float32 rows); other
  dtypes take the autograd-path blocks. A [1, cond_dim] conditioning vector broadcasts over the batch on both
  paths; a cond batch that is neither 1 nor B, and a perm that is not a permutation, raise ValueError."""
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  from faster_weathernext.processor import Processor, ProcessorConfig
  m, _, _ = mesh.config_mask(1)
  n = m.shape[0]
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  cfg = ProcessorConfig(layers=1)
  model = Processor(cfg, seed=9, device=cuda)
  g = torch.Generator(device=cuda).manual_seed(9)
  x = torch.randn(2, n, cfg.d_model, device=cuda, generator=g)
  c1 = torch.randn(1, cfg.cond_dim, device=cuda, generator=g)
  with torch.no_grad():
    y_b = model(x, c1.expand(2, -1).contiguous(), tiles)
    y_1 = model(x, c1, tiles)
    assert torch.equal(y_1, y_b)
    y_bf = model(x.to(torch.bfloat16), c1, tiles)              # not float32: no fused kernel on it
    assert y_bf.dtype == torch.bfloat16 and _rel(y_bf.float(), y_b) < 2e-2
    with pytest.raises(ValueError):
      model(x, torch.randn(3, cfg.cond_dim, device=cuda), tiles)
    bad = torch.arange(n, device=cuda)
    bad[3] = 4
    with pytest.raises(ValueError):
      model(x, c1, tiles, perm=bad)
    bad[3] = n
    with pytest.raises(ValueError):
      model(x, c1, tiles, perm=bad)


def test_processor_remat_gives_the_same_gradients(cuda):
  """patch.OPTIONS.remat recomputes each block in the backward (activation checkpointing); the gradients are the
  stored-activation ones (same kernels on the same inputs; relative L2 difference <= 1e-6)."""
  from faster_weathernext import mesh, patch
  from faster_weathernext import tiled_attn as ta
  from faster_weathernext.processor import Processor
  m, _, _ = mesh.config_mask(1)
  n = m.shape[0]
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  cfg = _small()
  model = Processor(cfg, seed=2, device=cuda)
  g = torch.Generator(device=cuda).manual_seed(3)
  x = torch.randn(1, n, cfg.d_model, device=cuda, generator=g)
  c = torch.randn(1, cfg.cond_dim, device=cuda, generator=g)
  grads = []
  for remat in (False, True):
    patch.OPTIONS.remat = remat
    try:
      model.zero_grad(set_to_none=True)
      model(x, c, tiles).square().mean().backward()
    finally:
      patch.OPTIONS.remat = False
    grads.append(torch.cat([p.grad.reshape(-1) for p in model.parameters()]))
  assert float((grads[1] - grads[0]).norm() / grads[0].norm()) <= 1e-6


def test_cond_layernorm_residual_kernel(cuda):
  """fwn_cond_layernorm_residual: x += residual (bf16) in place, then the conditioned norm of the sum, bit-equal to a
  float32 add followed by fwn_cond_layernorm (and, with an output node map, fwn_cond_layernorm_scatter)."""
  from faster_weathernext import _lib
  lib = _lib.lib()
  g = torch.Generator(device=cuda).manual_seed(4)
  for d in (128, 512, 1024):
    b, n = 2, 301
    x = torch.randn(b * n, d, device=cuda, generator=g)
    r = torch.randn(b * n, d, device=cuda, generator=g).to(torch.bfloat16)
    so = torch.randn(b, 2 * d, device=cuda, generator=g) * 0.2
    perm = torch.randperm(n, device=cuda, generator=g).to(torch.int32)
    for out_node in (None, perm):
      x_ref = x + r.float()
      ref = torch.empty(b * n, d, device=cuda, dtype=torch.bfloat16)
      if out_node is None:
        _lib.check(lib.fwn_cond_layernorm(x_ref.data_ptr(), b * n, d, n, so.data_ptr(), 1e-5, ref.data_ptr(),
                                          _lib.DTYPE_BF16, 0))
      else:
        _lib.check(lib.fwn_cond_layernorm_scatter(x_ref.data_ptr(), b * n, d, n, out_node.data_ptr(), so.data_ptr(),
                                                  1e-5, ref.data_ptr(), _lib.DTYPE_BF16, 0))
      x_got = x.clone()
      got = torch.empty_like(ref)
      _lib.check(lib.fwn_cond_layernorm_residual(x_got.data_ptr(), r.data_ptr(), b * n, d, n,
                                                 out_node.data_ptr() if out_node is not None else None,
                                                 so.data_ptr(), 1e-5, got.data_ptr(), _lib.DTYPE_BF16, 0))
      torch.cuda.synchronize()
      assert torch.equal(x_got, x_ref), d
      assert torch.equal(got, ref), d
  assert lib.fwn_cond_layernorm_residual(x.data_ptr(), None, 4, 128, 2, None, so.data_ptr(), 1e-5, x.data_ptr(),
                                         _lib.DTYPE_F32, 0) == _lib.FWN_ERR_INVALID_ARGUMENT


def _cond_norm_torch(x, a, so, n):
  """Composed float32 torch form of the conditioned norm: xn = x (+ a), y = LN(xn) (1 + scale) + offset."""
  b = so.shape[0]
  d = x.shape[1]
  xn = x + a.float() if a is not None else x
  y = torch.nn.functional.layer_norm(xn.view(b, n, d), (d,), eps=1e-5)
  scale, offset = so.unsqueeze(1).chunk(2, dim=-1)
  return xn, (y * (1 + scale) + offset).view(b * n, d)


def test_cond_layernorm_backward_matches_torch_autograd(cuda):
  """fwn_cond_layernorm_bwd through the processor's autograd Function against torch autograd of the composed
  float32 form, for d in {128, 256, 512}, 301 rows per sample (ragged against the kernel's 128-row CTAs), with and
  without a residual input, bf16 and float32 output: dx and d(scale, offset) within 1e-4 of the gradient's scale
  (float32, different summation orders), d(residual) the bf16 rounding of dx exactly; two calls give identical
  scale / offset gradients (fixed reduction order)."""
  from faster_weathernext.processor import _CondNorm
  g = torch.Generator(device=cuda).manual_seed(11)
  b, n = 3, 301
  for d in (128, 256, 512):
    for with_a in (False, True):
      for out_dtype in (torch.bfloat16, torch.float32):
        x = torch.randn(b * n, d, device=cuda, generator=g) * 2 + 0.5
        a = (torch.randn(b * n, d, device=cuda, generator=g)).to(torch.bfloat16) if with_a else None
        so = torch.randn(b, 2 * d, device=cuda, generator=g) * 0.3
        dy = torch.randn(b * n, d, device=cuda, generator=g).to(out_dtype)
        dxn = torch.randn(b * n, d, device=cuda, generator=g) if with_a else None
        # ours
        xo = x.clone().requires_grad_()
        ao = a.clone().requires_grad_() if with_a else None
        soo = so.clone().requires_grad_()
        out = _CondNorm.apply(xo, ao, soo, n, out_dtype)
        if with_a:
          xn_o, h_o = out
          torch.autograd.backward([xn_o, h_o], [dxn, dy])
        else:
          h_o = out
          h_o.backward(dy)
        # torch
        xr = x.clone().requires_grad_()
        ar = a.float().clone().requires_grad_() if with_a else None
        sor = so.clone().requires_grad_()
        xn_r, h_r = _cond_norm_torch(xr, ar, sor, n)
        if with_a:
          torch.autograd.backward([xn_r, h_r], [dxn, dy.float()])
        else:
          h_r.backward(dy.float())
        torch.testing.assert_close(h_o.float(), h_r.detach().to(out_dtype).float(), atol=1e-2 if out_dtype ==
                                   torch.bfloat16 else 1e-5, rtol=1e-2 if out_dtype == torch.bfloat16 else 1e-5)
        scale_dx = float(xr.grad.abs().max())
        assert float((xo.grad - xr.grad).abs().max()) <= 1e-4 * scale_dx, (d, with_a, out_dtype)
        scale_ds = float(sor.grad.abs().max())
        assert float((soo.grad - sor.grad).abs().max()) <= 1e-4 * scale_ds, (d, with_a, out_dtype)
        if with_a:
          assert ao.grad.dtype == torch.bfloat16
          assert torch.equal(ao.grad, xo.grad.to(torch.bfloat16))
        first = soo.grad.clone()
        soo.grad = None
        out = _CondNorm.apply(xo, ao, soo, n, out_dtype)
        (out[1] if with_a else out).backward(dy)
        assert torch.equal(soo.grad, first)


def test_cond_layernorm_backward_abi_checks(cuda):
  """fwn_cond_layernorm_bwd rejects an unbuilt width, a short workspace and rows that are not whole samples."""
  from faster_weathernext import _lib
  lib = _lib.lib()
  x = torch.zeros(8, 1024, device=cuda)
  so = torch.zeros(2, 2048, device=cuda)
  dy, dx, dso = torch.zeros_like(x), torch.empty_like(x), torch.empty_like(so)
  ws = torch.zeros(1 << 16, dtype=torch.uint8, device=cuda)
  args = lambda d, rps, nbytes: (x.data_ptr(), 8, d, rps, so.data_ptr(), 1e-5, dy.data_ptr(), _lib.DTYPE_F32, None,
                                 dx.data_ptr(), None, dso.data_ptr(), ws.data_ptr(), nbytes, 0)
  assert lib.fwn_cond_layernorm_bwd(*args(1024, 4, ws.numel())) == _lib.FWN_ERR_UNSUPPORTED
  assert lib.fwn_cond_layernorm_bwd(*args(512, 3, ws.numel())) == _lib.FWN_ERR_INVALID_ARGUMENT
  need = lib.fwn_cond_layernorm_bwd_workspace(8, 512, 4)
  assert need == 2 * 1 * 2 * 512 * 4
  assert lib.fwn_cond_layernorm_bwd(*args(512, 4, need - 4)) == _lib.FWN_ERR_INVALID_ARGUMENT
  assert lib.fwn_cond_layernorm_bwd(*args(512, 4, need)) == _lib.FWN_OK
  torch.cuda.synchronize()
  assert not bool(dso.view(-1)[:2 * 1024].any())


def test_processor_fused_training_matches_composed_path(cuda):
  """The autograd path on the fused norms (fused_training, the default) against the composed torch form of the same
  blocks (fused_training = False): outputs within rel RMS 1e-2 and all parameter and input gradients within 3e-2
  global relative L2 (bf16 compute; the fused path computes the conditioning's scale / offset in float32, the
  composed one in bf16)."""
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  from faster_weathernext.processor import Processor
  m, _, _ = mesh.config_mask(1)
  n = m.shape[0]
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  cfg = _small()
  model = Processor(cfg, seed=6, device=cuda)
  g = torch.Generator(device=cuda).manual_seed(8)
  x = torch.randn(2, n, cfg.d_model, device=cuda, generator=g)
  c = torch.randn(2, cfg.cond_dim, device=cuda, generator=g)
  t = torch.randn(2, n, cfg.d_model, device=cuda, generator=g)
  ys, grads = [], []
  for fused in (True, False):
    model.fused_training = fused
    model.zero_grad(set_to_none=True)
    xi = x.clone().requires_grad_()
    ci = c.clone().requires_grad_()
    y = model(xi, ci, tiles)
    torch.nn.functional.mse_loss(y, t).backward()
    ys.append(y.detach())
    grads.append(torch.cat([p.grad.reshape(-1) for p in model.parameters()] + [xi.grad.reshape(-1),
                                                                                ci.grad.reshape(-1)]))
  model.fused_training = True
  assert _rel(ys[0], ys[1]) < 1e-2
  assert float((grads[0] - grads[1]).norm() / grads[1].norm()) < 3e-2
