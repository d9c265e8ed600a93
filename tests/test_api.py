"""CPU: the drop-in API (enable / disable / options, Options fields) behaves as the reference's."""
import dataclasses

import pytest


def test_enable_rejects_unknown_options_and_keeps_reference_fields():
  import faster_weathernext
  from faster_weathernext import patch
  names = {f.name for f in dataclasses.fields(patch.Options)}
  # The reference's Options fields (src/faster_weathernext/patch.py:50-82).
  assert names == {"attention", "replace_attention", "reorder", "strict_fp32", "attn_chunk", "grid_chunk",
                   "edge_chunk", "layer_loop", "remat", "sequential_samples"}
  with pytest.raises(TypeError):
    faster_weathernext.enable(not_an_option=1)
  with pytest.warns(UserWarning, match="attn_chunk"):
    opts = faster_weathernext.enable(force=True, reorder=False, attn_chunk=256)
  assert opts is faster_weathernext.options() and opts.reorder is False and opts.attn_chunk == 256
  assert patch.is_enabled()
  faster_weathernext.disable()
  assert not patch.is_enabled()
  patch.OPTIONS.reorder, patch.OPTIONS.attn_chunk = True, 512


def test_attention_impl_refuses_other_backends():
  from faster_weathernext import patch
  patch.OPTIONS.attention = "xla"
  try:
    with pytest.raises(ValueError):
      patch.attention_impl()
  finally:
    patch.OPTIONS.attention = "auto"


def test_processor_bf16_weight_cache_on_host():
  """The inference path's bf16 weight copies: reused while a parameter is unchanged, recast after an in-place
  update (the version counter moves) or a new storage (.data replaced)."""
  import torch
  from faster_weathernext.processor import Processor, ProcessorConfig
  model = Processor(ProcessorConfig(layers=1, d_model=64, heads=2, head_dim=32, mlp_hidden=128, cond_dim=8),
                    seed=1, device="cpu")
  w = model.blocks[0].w1
  a = model._bf16(w)
  assert a.dtype == torch.bfloat16 and torch.equal(a, w.detach().to(torch.bfloat16))
  assert model._bf16(w) is a
  with torch.no_grad():
    w.mul_(2.0)
  b = model._bf16(w)
  assert b is not a and torch.equal(b, w.detach().to(torch.bfloat16))
  w.data = torch.zeros_like(w)
  c = model._bf16(w)
  assert c is not b and not c.any()


def test_layout_helpers_on_host():
  """Host-side layout logic of the op: which strided views gathered row loads accept, the descriptor's strides,
  and the refusal of a non-contiguous head_dim."""
  import torch
  from faster_weathernext import tiled_attn as ta
  x = torch.zeros(2, 50, 4, 64)
  assert ta._gather_layout(x) == 0                                   # [B, n, H, D] contiguous
  fused = torch.zeros(2, 50, 4, 3, 64)
  assert ta._gather_layout(fused[:, :, :, 1]) == 0                   # fused q/k/v: one 2D view, rows 3 D apart
  assert ta._gather_layout(x[:, :, :2]) == -1                        # a head slice: rows are not evenly spaced
  head_major = torch.zeros(2, 4, 50, 64).transpose(1, 2)
  assert ta._gather_layout(head_major) == 1
  d = ta._desc(fused[:, :, :, 0], x, 0.125, 0)
  assert (d.batch, d.heads, d.n, d.head_dim) == (2, 4, 50, 64)
  assert (d.stride_b, d.stride_n, d.stride_h) == (50 * 4 * 3 * 64, 4 * 3 * 64, 3 * 64)
  assert (d.out_stride_b, d.out_stride_n, d.out_stride_h) == (50 * 4 * 64, 4 * 64, 64)
  with pytest.raises(ValueError):
    ta._desc(torch.zeros(2, 50, 4, 64).transpose(2, 3).transpose(2, 3)[..., ::2], x, 0.125, 0)
  a, b = ta._canon(head_major, x)
  assert a.stride() == b.stride() == x.stride()


def test_options_without_effect_warn_and_acted_on_options_do_not():
  """Options that configure parts of the reference outside this build warn when set away from their defaults;
  reorder, strict_fp32, remat, edge_chunk and attention are acted on and do not."""
  import warnings
  import faster_weathernext
  from faster_weathernext import patch
  try:
    with warnings.catch_warnings():
      warnings.simplefilter("error")
      faster_weathernext.enable(force=True, reorder=False, strict_fp32=True, remat=True, attention="tiled",
                                grid_chunk=32768, edge_chunk=1024)
    for name, value in (("grid_chunk", 1024), ("layer_loop", False), ("sequential_samples", True),
                        ("replace_attention", False)):
      with pytest.warns(UserWarning, match=name):
        faster_weathernext.enable(force=True, **{name: value})
  finally:
    patch.OPTIONS = patch.Options()
    faster_weathernext.disable()


def test_matmul_precision_selects_the_reference_modes():
  """pallas_attn.py:336-342: float32 runs TF32 by default and 3xTF32 under "highest"; strict_fp32 only matters
  under "highest", where the IEEE float32 dots it asks for are not built (NotImplementedError); bf16 is bf16."""
  import torch
  from faster_weathernext import _lib
  from faster_weathernext import tiled_attn as ta
  f32, bf = torch.float32, torch.bfloat16
  assert ta._mode_for(f32, None, False) == _lib.MODE_TF32
  assert ta._mode_for(f32, None, True) == _lib.MODE_TF32
  assert ta._mode_for(f32, "highest", False) == _lib.MODE_TF32X3
  assert ta._mode_for(f32, "float32", False) == _lib.MODE_TF32X3
  assert ta._mode_for(bf, "highest", True) == _lib.MODE_BF16
  with pytest.raises(NotImplementedError):
    ta._mode_for(f32, "highest", True)
  with ta.default_matmul_precision("highest"):
    assert ta._mode_for(f32, None, False) == _lib.MODE_TF32X3
    with ta.default_matmul_precision("default"):
      assert ta._mode_for(f32, None, False) == _lib.MODE_TF32
    assert ta._mode_for(f32, "default", False) == _lib.MODE_TF32
  assert ta.current_matmul_precision() is None
  with pytest.raises(ValueError):
    with ta.default_matmul_precision("fp64"):
      pass
  with pytest.raises(TypeError):
    ta._mode_for(torch.float16, None, False)


def test_reference_list_checks():
  """tiled_flash_attention's lists are checked against n before anything reaches the device."""
  import numpy as np
  from faster_weathernext import tiled_attn as ta
  ptr = np.array([0, 1, 2], np.int32)
  kb = np.array([0, 3], np.int32)
  bits = np.ones((2, 64), np.uint32)
  ta._check_lists(ptr, kb, bits, 100, "tiles")                      # 2 blocks of 64 rows, 4 key blocks
  with pytest.raises(ValueError, match="tile_ptr"):
    ta._check_lists(ptr, kb, bits, 200, "tiles")
  with pytest.raises(ValueError, match="key blocks"):
    ta._check_lists(ptr, np.array([0, 4], np.int32), bits, 100, "tiles")
  with pytest.raises(ValueError, match="tile_bits"):
    ta._check_lists(ptr, kb, bits[:1], 100, "tiles")
  with pytest.raises(ValueError, match="CSR"):
    ta._check_lists(np.array([0, 2, 1], np.int32), kb, bits, 100, "tiles")
