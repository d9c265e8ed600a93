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


def _gelu_grad(x):
  u = (2.0 / torch.pi) ** 0.5 * (x + 0.044715 * x ** 3)
  t = torch.tanh(u)
  return 0.5 * (1.0 + t) + 0.5 * x * (1.0 - t * t) * (2.0 / torch.pi) ** 0.5 * (1.0 + 3 * 0.044715 * x * x)


@pytest.mark.parametrize("m", [1000, 40_962 + 77])
def test_gemm_aux_gelu_forward_and_backward(cuda, m):
  """fwn_gemm_bf16_aux (the training MLP): FWN_ACT_GELU_TANH_AUX gives c = GELU(x) and aux = x for x = a bt^T + bias
  (rel RMS <= 5e-3 each against float64); FWN_ACT_GELU_TANH_GRAD gives c = (a bt^T) GELU'(aux) for a bf16 aux (rel RMS
  <= 5e-3 against float64 on the same bf16 aux). Rows past m are not written (a guard row after the output)."""
  from faster_weathernext import _lib
  lib = _lib.lib()
  n, k = 2048, 512
  g = torch.Generator(device=cuda).manual_seed(m)
  a = torch.randn(m, k, device=cuda, generator=g).to(torch.bfloat16)
  bt = (torch.randn(n, k, device=cuda, generator=g) * k ** -0.5).to(torch.bfloat16)
  b = (torch.randn(n, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
  st = torch.cuda.current_stream().cuda_stream
  c = torch.full((m + 1, n), 7.0, device=cuda, dtype=torch.bfloat16)
  aux = torch.full((m + 1, n), 7.0, device=cuda, dtype=torch.bfloat16)
  _lib.check(lib.fwn_gemm_bf16_aux(a.data_ptr(), bt.data_ptr(), b.data_ptr(), c.data_ptr(), aux.data_ptr(), m, n, k,
                                   _lib.ACT_GELU_TANH_AUX, st))
  torch.cuda.synchronize()
  assert _lib.device_error() == 0
  assert bool((c[m] == 7.0).all()) and bool((aux[m] == 7.0).all())
  assert _rel(aux[:m], _ref(a, bt, b, 0)) <= 5e-3
  assert _rel(c[:m], _ref(a, bt, b, 1)) <= 5e-3
  # Backward: gradient of the activation (a bt^T) times GELU' of the stored pre-activation.
  pre = aux[:m].contiguous()
  d = torch.full((m + 1, n), 7.0, device=cuda, dtype=torch.bfloat16)
  _lib.check(lib.fwn_gemm_bf16_aux(a.data_ptr(), bt.data_ptr(), None, d.data_ptr(), pre.data_ptr(), m, n, k,
                                   _lib.ACT_GELU_TANH_GRAD, st))
  torch.cuda.synchronize()
  assert _lib.device_error() == 0
  assert bool((d[m] == 7.0).all())
  assert _rel(d[:m], _ref(a, bt, None, 0) * _gelu_grad(pre.double())) <= 5e-3
  # Argument checks: the aux modes need aux; fwn_gemm_bf16 takes neither mode.
  assert lib.fwn_gemm_bf16_aux(a.data_ptr(), bt.data_ptr(), None, d.data_ptr(), None, m, n, k,
                               _lib.ACT_GELU_TANH_GRAD, st) == _lib.FWN_ERR_INVALID_ARGUMENT
  assert lib.fwn_gemm_bf16(a.data_ptr(), bt.data_ptr(), None, d.data_ptr(), m, n, k, _lib.ACT_GELU_TANH_AUX,
                           st) == _lib.FWN_ERR_INVALID_ARGUMENT


def test_gelu_mlp_function_matches_torch_autograd(cuda):
  """processor._GeluMLP (forward and backward through the aux GEMM epilogues) against torch autograd of the composed
  bf16 MLP at the processor's width: output and every gradient within rel RMS 1e-2 (bf16 rounding of the
  activations on both sides)."""
  from faster_weathernext.processor import _GeluMLP
  import torch.nn.functional as F
  g = torch.Generator(device=cuda).manual_seed(2)
  m, d, hid = 3001, 512, 2048
  h = torch.randn(m, d, device=cuda, generator=g).to(torch.bfloat16)
  params = [torch.randn(d, hid, device=cuda, generator=g) * d ** -0.5, torch.randn(hid, device=cuda, generator=g) * 0.1,
            torch.randn(hid, d, device=cuda, generator=g) * hid ** -0.5, torch.randn(d, device=cuda, generator=g) * 0.1]
  dy = torch.randn(m, d, device=cuda, generator=g).to(torch.bfloat16)
  ha = h.clone().requires_grad_()
  pa = [p.clone().requires_grad_() for p in params]
  ya = _GeluMLP.apply(ha, *pa)
  ya.backward(dy)
  hb = h.clone().requires_grad_()
  pb = [p.clone().requires_grad_() for p in params]
  bf = torch.bfloat16
  yb = torch.addmm(pb[3].to(bf), F.gelu(torch.addmm(pb[1].to(bf), hb, pb[0].to(bf)), approximate="tanh"), pb[2].to(bf))
  yb.backward(dy)
  torch.cuda.synchronize()
  assert _rel(ya, yb.double()) <= 1e-2
  assert _rel(ha.grad, hb.grad.double()) <= 1e-2
  for x, y in zip(pa, pb):
    assert x.grad.dtype == torch.float32
    assert _rel(x.grad, y.grad.double()) <= 1e-2


@pytest.mark.parametrize("m,n,k,idx", [(3001, 512, 512, True), (40_962 + 77, 256, 512, False)])
def test_gemm_gather_add_swish(cuda, m, n, k, idx):
  """fwn_gemm_bf16_gather: c = swish(a bt^T + bias + add0[idx0] + add1[idx1]) against float64 on the same bf16
  operands (rel RMS <= 5e-3), gathered indices (the interaction network's edge MLP) or the rows themselves (its node
  MLP); an index out of range is reported as FWN_ERR_INVALID_ARGUMENT by fwn_device_error, in bounds."""
  from faster_weathernext import _lib
  lib = _lib.lib()
  g = torch.Generator(device=cuda).manual_seed(m)
  a = torch.randn(m, k, device=cuda, generator=g).to(torch.bfloat16)
  bt = (torch.randn(n, k, device=cuda, generator=g) * k ** -0.5).to(torch.bfloat16)
  b = (torch.randn(n, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
  r0, r1 = (97, 2 * m) if idx else (m, m)
  add0 = torch.randn(r0, n, device=cuda, generator=g).to(torch.bfloat16)
  add1 = torch.randn(r1, n, device=cuda, generator=g).to(torch.bfloat16)
  i0 = torch.randint(0, r0, (m,), device=cuda, generator=g, dtype=torch.int32) if idx else None
  i1 = torch.randint(0, r1, (m,), device=cuda, generator=g, dtype=torch.int32) if idx else None
  c = torch.full((m, n), float("nan"), device=cuda, dtype=torch.bfloat16)
  st = torch.cuda.current_stream().cuda_stream
  ptr = lambda t: t.data_ptr() if t is not None else None
  _lib.check(lib.fwn_gemm_bf16_gather(a.data_ptr(), bt.data_ptr(), b.data_ptr(), c.data_ptr(), add0.data_ptr(), ptr(i0),
                                      r0, add1.data_ptr(), ptr(i1), r1, m, n, k, _lib.ACT_SWISH, st))
  torch.cuda.synchronize()
  assert _lib.device_error() == 0
  g0 = add0.double()[i0.long()] if idx else add0.double()
  g1 = add1.double()[i1.long()] if idx else add1.double()
  x = _ref(a, bt, b, 0) + g0 + g1
  assert _rel(c, x * torch.sigmoid(x)) <= 5e-3
  if idx:
    bad = i0.clone()
    bad[m // 2] = r0                                  # one past the last row
    _lib.check(lib.fwn_gemm_bf16_gather(a.data_ptr(), bt.data_ptr(), b.data_ptr(), c.data_ptr(), add0.data_ptr(),
                                        bad.data_ptr(), r0, add1.data_ptr(), i1.data_ptr(), r1, m, n, k, _lib.ACT_SWISH,
                                        st))
    code = ctypes.c_int32(0)
    _lib.check(lib.fwn_device_error(st, ctypes.byref(code)))
    assert code.value == _lib.FWN_ERR_INVALID_ARGUMENT
  assert lib.fwn_gemm_bf16_gather(a.data_ptr(), bt.data_ptr(), b.data_ptr(), c.data_ptr(), add0.data_ptr(), None,
                                  m - 1, None, None, 0, m, n, k, _lib.ACT_SWISH, st) == _lib.FWN_ERR_INVALID_ARGUMENT
