"""ctypes binding of libfwn_attn.so (include/fwn_attn.h).

The library is the only implementation of the attention path: if it is missing or cannot be loaded
the import of the op fails loudly (there is no CPU or framework fallback).
"""

import ctypes
import os

from faster_weathernext import _build

FWN_OK = 0
FWN_ERR_INVALID_ARGUMENT = 1
FWN_ERR_UNSUPPORTED = 2
FWN_ERR_WORKSPACE = 3
FWN_ERR_LAUNCH = 4
FWN_ERR_DEVICE_TIMEOUT = 5
FWN_ERR_NO_DEVICE = 6

DTYPE_BF16 = 0
DTYPE_F32 = 1
MODE_BF16 = 0
MODE_TF32 = 1
MODE_TF32X3 = 2
DESC_GRAD_STRIDES = 1
ACT_NONE = 0
ACT_GELU_TANH = 1
ACT_SWISH = 2
ACT_GELU_TANH_AUX = 3
ACT_GELU_TANH_GRAD = 4

# Every symbol include/fwn_attn.h declares.
SYMBOLS = ("fwn_version", "fwn_last_error_string", "fwn_device_error", "fwn_lse_rows",
           "fwn_tiles_workspace_size", "fwn_tiles_count", "fwn_tiles_fill", "fwn_tiles_pair_count",
           "fwn_tiles_pair_fill", "fwn_tiles_gather_count", "fwn_tiles_gather_fill", "fwn_hilbert_codes", "fwn_attn_fwd", "fwn_attn_bwd_workspace_size", "fwn_attn_bwd",
           "fwn_attn_bwd_delta", "fwn_attn_bwd_dq", "fwn_attn_bwd_dkv", "fwn_attn_bwd_noalloc",
           "fwn_bitset_words", "fwn_khop_bitset", "fwn_walk_bitset", "fwn_bitset_csr_count", "fwn_bitset_csr_fill",
           "fwn_cond_layernorm", "fwn_cond_layernorm_scatter", "fwn_cond_layernorm_residual",
           "fwn_cond_layernorm_add", "fwn_cond_layernorm_bwd_workspace", "fwn_cond_layernorm_bwd",
           "fwn_gemm_bf16", "fwn_gemm_bf16_aux", "fwn_gemm_bf16_gather", "fwn_gnn_gather_add_act", "fwn_gnn_ln_segment_sum", "fwn_test_attn_fwd_timeout")


class AttnDesc(ctypes.Structure):
  _fields_ = [("batch", ctypes.c_int32), ("heads", ctypes.c_int32), ("n", ctypes.c_int32),
              ("head_dim", ctypes.c_int32), ("scale", ctypes.c_float), ("dtype", ctypes.c_int32),
              ("mode", ctypes.c_int32), ("flags", ctypes.c_int32), ("stride_b", ctypes.c_int64),
              ("stride_n", ctypes.c_int64), ("stride_h", ctypes.c_int64), ("out_stride_b", ctypes.c_int64),
              ("out_stride_n", ctypes.c_int64), ("out_stride_h", ctypes.c_int64), ("grad_stride_b", ctypes.c_int64),
              ("grad_stride_n", ctypes.c_int64), ("grad_stride_h", ctypes.c_int64)]


class TileList(ctypes.Structure):
  _fields_ = [("ptr", ctypes.c_void_p), ("kb", ctypes.c_void_p), ("bits", ctypes.c_void_p),
              ("n_blocks", ctypes.c_int32), ("n_tiles", ctypes.c_int32), ("block_rows", ctypes.c_int32),
              ("n_cols", ctypes.c_int32), ("cols", ctypes.c_void_p)]


class FwnError(RuntimeError):
  def __init__(self, status, message):
    super().__init__(f"fwn status {status}: {message}")
    self.status = status


_P = ctypes.c_void_p
_I = ctypes.c_int32
_SZ = ctypes.c_size_t


def _declare(lib):
  lib.fwn_version.restype = ctypes.c_char_p
  lib.fwn_last_error_string.restype = ctypes.c_char_p
  lib.fwn_lse_rows.argtypes = [_I]
  lib.fwn_lse_rows.restype = _I
  lib.fwn_bitset_words.argtypes = [_I]
  lib.fwn_bitset_words.restype = _I
  lib.fwn_cond_layernorm_bwd_workspace.argtypes = [ctypes.c_int64, _I, _I]
  lib.fwn_cond_layernorm_bwd_workspace.restype = _SZ
  sigs = {
      "fwn_device_error": [_P, ctypes.POINTER(_I)],
      "fwn_tiles_workspace_size": [_I, _I, _I, ctypes.POINTER(_SZ)],
      "fwn_tiles_count": [_P, _P, _I, _I, _I, _P, _P, _SZ, _P],
      "fwn_tiles_fill": [_P, _P, _I, _I, _I, _P, _P, _P, _P],
      "fwn_tiles_pair_count": [ctypes.POINTER(TileList), _P, _P, _SZ, _P],
      "fwn_tiles_pair_fill": [ctypes.POINTER(TileList), _P, _P, _P, _P],
      "fwn_tiles_gather_count": [ctypes.POINTER(TileList), _P, _P, _SZ, _P],
      "fwn_tiles_gather_fill": [ctypes.POINTER(TileList), _I, _P, _P, _P, _P],
      "fwn_hilbert_codes": [_P, _P, _I, _I, _P, _P],
      "fwn_khop_bitset": [_P, _P, _I, _I, _P, _P, _P],
      "fwn_walk_bitset": [_P, _P, _I, _I, _P, _P, _P],
      "fwn_cond_layernorm": [_P, ctypes.c_int64, _I, _I, _P, ctypes.c_float, _P, _I, _P],
      "fwn_cond_layernorm_scatter": [_P, ctypes.c_int64, _I, _I, _P, _P, ctypes.c_float, _P, _I, _P],
      "fwn_cond_layernorm_residual": [_P, _P, ctypes.c_int64, _I, _I, _P, _P, ctypes.c_float, _P, _I, _P],
      "fwn_cond_layernorm_add": [_P, _P, _P, ctypes.c_int64, _I, _I, _P, ctypes.c_float, _P, _I, _P],
      "fwn_cond_layernorm_bwd": [_P, ctypes.c_int64, _I, _I, _P, ctypes.c_float, _P, _I, _P, _P, _P, _P, _P,
                                 ctypes.c_size_t, _P],
      "fwn_gemm_bf16": [_P, _P, _P, _P, ctypes.c_int64, _I, _I, _I, _P],
      "fwn_gemm_bf16_aux": [_P, _P, _P, _P, _P, ctypes.c_int64, _I, _I, _I, _P],
      "fwn_gemm_bf16_gather": [_P, _P, _P, _P, _P, _P, ctypes.c_int64, _P, _P, ctypes.c_int64, ctypes.c_int64, _I, _I,
                               _I, _P],
      "fwn_gnn_gather_add_act": [_P, _P, _P, _P, _P, _P, ctypes.c_int64, _I, _I, _P, _P],
      "fwn_gnn_ln_segment_sum": [_P, _P, ctypes.c_int64, _I, _P, _P, ctypes.c_float, ctypes.c_float, _P, _P, _I, _P],
      "fwn_bitset_csr_count": [_P, _I, _I, _P, _P, _SZ, _P],
      "fwn_bitset_csr_fill": [_P, _I, _I, _P, _P, _P],
      "fwn_attn_fwd": [ctypes.POINTER(AttnDesc), _P, _P, _P, ctypes.POINTER(TileList), _P, _P, _P],
      "fwn_attn_bwd_workspace_size": [ctypes.POINTER(AttnDesc), ctypes.POINTER(_SZ)],
      "fwn_test_attn_fwd_timeout": [ctypes.POINTER(AttnDesc), _P, _P, _P, ctypes.POINTER(TileList), _P, _P,
                                    ctypes.c_uint64, _P],
      "fwn_attn_bwd": [ctypes.POINTER(AttnDesc), _P, _P, _P, _P, _P, _P, ctypes.POINTER(TileList),
                       ctypes.POINTER(TileList), _P, _P, _P, _P, _SZ, _P],
      "fwn_attn_bwd_noalloc": [ctypes.POINTER(AttnDesc), _P, _P, _P, _P, _P, _P, ctypes.POINTER(TileList),
                               ctypes.POINTER(TileList), _P, _P, _P, _P],
      "fwn_attn_bwd_delta": [ctypes.POINTER(AttnDesc), _P, _P, _P, _SZ, _P],
      "fwn_attn_bwd_dq": [ctypes.POINTER(AttnDesc), _P, _P, _P, _P, _P, ctypes.POINTER(TileList), _P, _P, _SZ, _P],
      "fwn_attn_bwd_dkv": [ctypes.POINTER(AttnDesc), _P, _P, _P, _P, _P, ctypes.POINTER(TileList), _P, _P, _P, _SZ,
                           _P],
  }
  for name, args in sigs.items():
    fn = getattr(lib, name)
    fn.argtypes = args
    fn.restype = ctypes.c_int


_LIB = None


def lib():
  """The loaded library (built in-tree on first use if the sources are newer)."""
  global _LIB
  if _LIB is None:
    path = _build.LIB
    if not os.path.exists(path) or not _build.up_to_date():
      path = _build.build()
    _LIB = ctypes.CDLL(path)
    _declare(_LIB)
  return _LIB


def check(status: int):
  if status == FWN_OK:
    return
  msg = lib().fwn_last_error_string().decode()
  if status == FWN_ERR_INVALID_ARGUMENT or status == FWN_ERR_WORKSPACE:
    raise ValueError(f"fwn status {status}: {msg}")
  if status == FWN_ERR_UNSUPPORTED:
    raise NotImplementedError(f"fwn status {status}: {msg}")
  raise FwnError(status, msg)


def device_error(stream_handle: int = 0) -> int:
  code = ctypes.c_int32(0)
  check(lib().fwn_device_error(stream_handle, ctypes.byref(code)))
  return code.value
