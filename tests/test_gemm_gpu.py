"""GPU: fwn_gemm_bf16, the projections' GEMM with a fused bias / GELU epilogue, against a float64 torch reference of
the same bf16 inputs. Bound: rel RMS <= 5e-3 (bf16 output rounding and float32 accumulation order; GELU's tanh is
the hardware approximation), with row counts that are not multiples of the 128-row tile."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, bt, bias, act):
  y = a.double() @ bt.double().T
  if bias is not None:
    y = y + bias.double()
  if act:
    y = 0.5 * y * (1.0 + torch.tanh((2.0 / torch.pi) ** 0.5 * (y + 0.044715 * y ** 3)))
  return y


def _rel(x, ref):
  x = x.double()
  return float(torch.sqrt(torch.mean((x - ref) ** 2)) / ref.std())


@pytest.mark.parametrize("m,n,k,bias,act", [(1000, 256, 64, True, 1), (1000, 512, 512, False, 0),
                                           (40_962 + 77, 2048, 512, True, 1), (5_003, 1536, 512, False, 0),
                                           (7_777, 512, 2048, True, 0)])
def test_gemm_matches_reference(cuda, m, n, k, bias, act):
  from faster_weathernext import _lib
  lib = _lib.lib()
  g = torch.Generator(device=cuda).manual_seed(m + n + k)
  a = torch.randn(m, k, device=cuda, generator=g).to(torch.bfloat16)
  bt = (torch.randn(n, k, device=cuda, generator=g) * k ** -0.5).to(torch.bfloat16)
  b = (torch.randn(n, device=cuda, generator=g) * 0.5).to(torch.bfloat16) if bias else None
  c = torch.full((m, n), float("nan"), device=cuda, dtype=torch.bfloat16)
  _lib.check(lib.fwn_gemm_bf16(a.data_ptr(), bt.data_ptr(), b.data_ptr() if b is not None else None, c.data_ptr(),
                               m, n, k, act, torch.cuda.current_stream().cuda_stream))
  torch.cuda.synchronize()
  assert _lib.device_error() == 0
  assert torch.isfinite(c.float()).all()
  assert _rel(c, _ref(a, bt, b, act)) <= 5e-3


def test_gemm_argument_checks(cuda):
  from faster_weathernext import _lib
  lib = _lib.lib()
  x = torch.zeros(256, 256, device=cuda, dtype=torch.bfloat16)
  assert lib.fwn_gemm_bf16(x.data_ptr(), x.data_ptr(), None, x.data_ptr(), 256, 200, 256, 0, 0) == _lib.FWN_ERR_UNSUPPORTED
  assert lib.fwn_gemm_bf16(x.data_ptr(), x.data_ptr(), None, x.data_ptr(), 256, 256, 100, 0, 0) == _lib.FWN_ERR_UNSUPPORTED
  assert lib.fwn_gemm_bf16(x.data_ptr(), x.data_ptr(), None, x.data_ptr(), 256, 256, 256, 7, 0) == _lib.FWN_ERR_INVALID_ARGUMENT
  assert lib.fwn_gemm_bf16(x.data_ptr() + 2, x.data_ptr(), None, x.data_ptr(), 256, 256, 256, 0, 0) == \
      _lib.FWN_ERR_INVALID_ARGUMENT
