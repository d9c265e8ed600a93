"""CPU: the C-ABI library loads and exports every symbol include/fwn_attn.h declares (no GPU calls)."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
  with open(os.path.join(ROOT, "include", "fwn_attn.h")) as f:
    text = f.read()
  return sorted(set(re.findall(r"FWN_API\s+[\w\s\*]*?\b(fwn_\w+)\s*\(", text)))


def test_header_declares_the_entry_points():
  names = _declared()
  for must in ("fwn_tiles_count", "fwn_tiles_fill", "fwn_attn_fwd", "fwn_attn_bwd", "fwn_hilbert_codes"):
    assert must in names


def test_library_loads_and_exports_every_declared_symbol():
  from faster_weathernext import _build, _lib
  path = _build.build()
  lib = ctypes.CDLL(path)
  for name in _declared():
    assert hasattr(lib, name), name
  assert set(_declared()) <= set(_lib.SYMBOLS)


def test_host_only_entry_points_need_no_gpu():
  from faster_weathernext import _lib
  lib = _lib.lib()
  assert lib.fwn_version().startswith(b"fwn_attn")
  assert lib.fwn_lse_rows(300) == 384 and lib.fwn_lse_rows(40962) == 41088
  # Argument checks fail before any CUDA call.
  desc = _lib.AttnDesc(1, 2, 300, 96, 0.125, _lib.DTYPE_BF16, _lib.MODE_BF16, 0, 600 * 96, 2 * 96, 96,
                       600 * 96, 2 * 96, 96)
  size = ctypes.c_size_t(0)
  assert lib.fwn_attn_bwd_workspace_size(ctypes.byref(desc), ctypes.byref(size)) == _lib.FWN_ERR_UNSUPPORTED
  assert b"head_dim" in lib.fwn_last_error_string()
  desc.head_dim = 64
  desc.mode = _lib.MODE_TF32  # TF32 needs float32 tensors
  assert lib.fwn_attn_bwd_workspace_size(ctypes.byref(desc), ctypes.byref(size)) == _lib.FWN_ERR_INVALID_ARGUMENT


def test_desc_flags_are_checked_before_any_cuda_call():
  """fwn_attn_desc.flags: unknown bits are refused; FWN_DESC_GRAD_STRIDES makes the gradient strides checked (16-byte
  multiples, rows not overlapping); flags = 0 never reads them."""
  from faster_weathernext import _lib
  lib = _lib.lib()
  size = ctypes.c_size_t(0)
  desc = _lib.AttnDesc(1, 2, 300, 64, 0.125, _lib.DTYPE_BF16, _lib.MODE_BF16, 0, 600 * 64, 2 * 64, 64,
                       600 * 64, 2 * 64, 64, 1, 1, 1)   # bad gradient strides, ignored without the flag
  assert lib.fwn_attn_bwd_workspace_size(ctypes.byref(desc), ctypes.byref(size)) == _lib.FWN_OK
  desc.flags = 4
  assert lib.fwn_attn_bwd_workspace_size(ctypes.byref(desc), ctypes.byref(size)) == _lib.FWN_ERR_INVALID_ARGUMENT
  assert b"flags" in lib.fwn_last_error_string()
  desc.flags = _lib.DESC_GRAD_STRIDES
  assert lib.fwn_attn_bwd_workspace_size(ctypes.byref(desc), ctypes.byref(size)) == _lib.FWN_ERR_INVALID_ARGUMENT
  desc.grad_stride_b, desc.grad_stride_n, desc.grad_stride_h = 300 * 2 * 3 * 64, 2 * 3 * 64, 3 * 64
  assert lib.fwn_attn_bwd_workspace_size(ctypes.byref(desc), ctypes.byref(size)) == _lib.FWN_OK
