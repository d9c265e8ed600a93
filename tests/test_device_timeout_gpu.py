"""GPU: failure detection of the kernels' bounded waits, without a fault.

fwn_test_attn_fwd_timeout runs the narrow forward with one K / V load left out (the producer of CTA 0 skips
the first load of its first work item; no copy is issued for it), and every wait bounded at 1 ms: the MMA
warp's wait on that load expires, the CTA's roles leave their loops, the producer drains the copies it did
issue, the CTA frees its tensor memory and returns. The host reads FWN_ERR_DEVICE_TIMEOUT through
fwn_device_error, the context stays usable, and the same forward launched normally afterwards (its persistent
CTAs allocate tensor memory on every SM, so memory left allocated would show) is bit-identical to one made
before the timeout.
"""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_reports_and_leaves_the_context_usable(cuda):
  from faster_weathernext import _lib, mesh
  from faster_weathernext import tiled_attn as ta
  lib = _lib.lib()
  m, _, _ = mesh.config_mask(1)
  n = m.shape[0]
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  g = torch.Generator(device=cuda).manual_seed(0)
  q, k, v = (torch.randn(1, n, 4, 64, device=cuda, dtype=torch.bfloat16, generator=g) for _ in range(3))
  mode = _lib.MODE_BF16
  o_before, lse_before = ta.attention_forward(q, k, v, tiles, 0.125, mode)
  torch.cuda.synchronize()
  assert _lib.device_error() == 0

  o = torch.zeros_like(q)
  lse = torch.zeros(1, 4, lib.fwn_lse_rows(n), device=cuda)
  desc = ta._desc(q, o, 0.125, mode)
  st = ta._lists(tiles, q, o)[0].struct()
  stream = torch.cuda.current_stream().cuda_stream
  t0 = time.monotonic()
  _lib.check(lib.fwn_test_attn_fwd_timeout(ctypes.byref(desc), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                           ctypes.byref(st), o.data_ptr(), lse.data_ptr(), 1_000_000, stream))
  code = _lib.device_error(stream)            # synchronises the stream
  elapsed = time.monotonic() - t0
  assert code == _lib.FWN_ERR_DEVICE_TIMEOUT
  assert elapsed < 1.0, elapsed                # the 1 ms bound, not the default 2 s
  assert _lib.device_error(stream) == 0        # reading clears the word

  for _ in range(2):
    o_after, lse_after = ta.attention_forward(q, k, v, tiles, 0.125, mode)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.equal(o_after, o_before) and torch.equal(lse_after, lse_before)
  # The backward (other kernels, their own tensor memory) runs normally too.
  qq, kk, vv = (x.clone().requires_grad_(True) for x in (q, k, v))
  ta.attention(qq, kk, vv, tiles, scale=0.125).backward(torch.ones_like(q))
  torch.cuda.synchronize()
  assert _lib.device_error() == 0 and torch.isfinite(qq.grad.float()).all()


def test_timeout_entry_point_refuses_other_kernels(cuda):
  """Only the narrow bf16 head_dim-64 forward takes a fault-injected launch; bounds on the wait limit."""
  from faster_weathernext import _lib
  from faster_weathernext import tiled_attn as ta
  from scipy import sparse
  lib = _lib.lib()
  n = 300
  m = (sparse.random(n, n, density=0.05, random_state=0, format="csr").astype(bool)
       + sparse.identity(n, dtype=bool)).tocsr()
  tiles = ta.AttentionTiles.from_mask(m, device=cuda)
  q = torch.zeros(1, n, 2, 64, device=cuda, dtype=torch.float32)
  desc = ta._desc(q, q, 0.125, _lib.MODE_TF32)
  st = tiles.fwd.struct()
  s = lib.fwn_test_attn_fwd_timeout(ctypes.byref(desc), q.data_ptr(), q.data_ptr(), q.data_ptr(), ctypes.byref(st),
                                    q.data_ptr(), None, 1_000_000, 0)
  assert s == _lib.FWN_ERR_UNSUPPORTED
  qb = q.to(torch.bfloat16)
  desc = ta._desc(qb, qb, 0.125, _lib.MODE_BF16)
  s = lib.fwn_test_attn_fwd_timeout(ctypes.byref(desc), qb.data_ptr(), qb.data_ptr(), qb.data_ptr(), ctypes.byref(st),
                                    qb.data_ptr(), None, 10, 0)
  assert s == _lib.FWN_ERR_INVALID_ARGUMENT
  torch.cuda.synchronize()
  assert _lib.device_error() == 0
