"""GPU: fwn_attn_bwd_noalloc, the backward entry point that allocates nothing.

Some callers cannot allocate device memory where they call the backward (an XLA custom-call handler
whose buffers all belong to XLA, or a loop that must not take cudaMalloc's implicit synchronisation),
so this entry point keeps the per-row delta in a fixed array inside the library instead of a caller
workspace. The test calls it through the C ABI and checks dq, dk, dv against fwn_attn_bwd (with a
workspace) on two calls in a row with different problems, so the second call also shows that a call
does not depend on what the previous one left in the shared array. Both entry points launch the same
deterministic kernels (no atomics) on the same inputs, with delta at a different address, so the outputs
must be bit-identical: any stale delta row left by the previous call would show. This file is collected
last on purpose.
"""
import ctypes

import pytest
import torch
from scipy import sparse

pytestmark = pytest.mark.gpu


def _problem(mask, heads, seed, device):
  from faster_weathernext import tiled_attn as ta
  n = mask.shape[0]
  g = torch.Generator(device=device).manual_seed(seed)
  q, k, v, do = (torch.randn(1, n, heads, 64, device=device, dtype=torch.bfloat16, generator=g) for _ in range(4))
  tiles = ta.AttentionTiles.from_mask(mask, device=device)
  return q, k, v, do, tiles


def _both(q, k, v, do, tiles):
  """dq, dk, dv from fwn_attn_bwd (caller workspace) and from fwn_attn_bwd_noalloc."""
  from faster_weathernext import _lib
  from faster_weathernext import tiled_attn as ta
  lib = _lib.lib()
  scale = 0.125
  o, lse = ta.attention_forward(q, k, v, tiles, scale, _lib.MODE_BF16)
  desc = ta._desc(q, o, scale, _lib.MODE_BF16)
  lf, lb = ta._lists(tiles, q, o)
  sf, sb = lf.struct(), lb.struct()
  stream = torch.cuda.current_stream().cuda_stream
  ws_bytes = ctypes.c_size_t(0)
  _lib.check(lib.fwn_attn_bwd_workspace_size(ctypes.byref(desc), ctypes.byref(ws_bytes)))
  ws = torch.empty(ws_bytes.value, dtype=torch.uint8, device=q.device)
  ref = [torch.empty_like(o) for _ in range(3)]
  got = [torch.empty_like(o) for _ in range(3)]
  _lib.check(lib.fwn_attn_bwd(ctypes.byref(desc), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                              do.data_ptr(), ctypes.byref(sf), ctypes.byref(sb), ref[0].data_ptr(), ref[1].data_ptr(),
                              ref[2].data_ptr(), ws.data_ptr(), ws_bytes.value, stream))
  _lib.check(lib.fwn_attn_bwd_noalloc(ctypes.byref(desc), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                      lse.data_ptr(), do.data_ptr(), ctypes.byref(sf), ctypes.byref(sb),
                                      got[0].data_ptr(), got[1].data_ptr(), got[2].data_ptr(), stream))
  torch.cuda.synchronize()
  assert _lib.device_error(stream) == 0
  return ref, got


def test_noalloc_backward_matches_workspace_backward_twice(cuda):
  from faster_weathernext import mesh
  # Call 1: configuration 1 (symmetric 0.25 rad mask, 642 nodes, 4 heads).
  m1, _, _ = mesh.config_mask(1)
  ref, got = _both(*_problem(m1, 4, 0, cuda))
  for a, b in zip(got, ref):
    assert torch.equal(a, b)
  # Call 2: a different, non-symmetric problem (457 nodes, 3 heads, transposed list for dK/dV).
  m2 = sparse.random(457, 457, density=0.05, random_state=11, format="csr").astype(bool)
  m2 = (m2 + sparse.identity(457, dtype=bool)).tocsr()
  ref, got = _both(*_problem(m2, 3, 1, cuda))
  for a, b in zip(got, ref):
    assert torch.equal(a, b)


def test_noalloc_backward_rejects_problems_beyond_its_capacity(cuda):
  """batch * heads * lse_rows above FWN_NOALLOC_DELTA_ROWS is refused before anything is launched."""
  from faster_weathernext import _lib
  lib = _lib.lib()
  n = 40962
  heads, batch = 8, 4  # 4 * 8 * 41,088 rows > 2^20
  desc = _lib.AttnDesc(batch, heads, n, 64, 0.125, _lib.DTYPE_BF16, _lib.MODE_BF16, 0, n * heads * 64, heads * 64, 64,
                       n * heads * 64, heads * 64, 64)
  status = lib.fwn_attn_bwd_noalloc(ctypes.byref(desc), 16, 16, 16, 16, 16, 16, None, None, 16, 16, 16, 0)
  assert status == _lib.FWN_ERR_WORKSPACE
  assert b"capacity" in lib.fwn_last_error_string()
