"""GPU: the grid <-> mesh interaction-network step (faster_weathernext.gnn, patch.py:347-509's structure) against the
float64 oracle (oracle/gnn.py) on the same bf16-rounded inputs and weights, for the decoder's shape (every receiver
has exactly k in-edges, mesh -> points) and the encoder's (variable in-degree, receivers with no edges, points ->
mesh); edge blocks (Options.edge_chunk) against one pass. Bound: rel RMS <= 2e-2 of the node updates (bf16
matmul operands and bf16 hidden / message rows, float32 accumulation; the same bound as the processor's tests).
The kernels on their own: the gather-add-swish pass and the LayerNorm segment-sum against torch."""
import numpy as np
import pytest
import torch

from oracle import attention as oa
from oracle import gnn as og

pytestmark = pytest.mark.gpu


def _graph(kind, ns, nr, seed):
  rng = np.random.default_rng(seed)
  if kind == "fixed_k":
    k = 3
    rcv = np.repeat(np.arange(nr), k)
    snd = rng.integers(0, ns, size=nr * k)
  else:
    deg = rng.integers(0, 9, size=nr)
    deg[rng.choice(nr, size=nr // 10, replace=False)] = 0
    rcv = np.repeat(np.arange(nr), deg)
    snd = rng.integers(0, ns, size=rcv.size)
  return snd, rcv


def _bf(x):
  return oa.bf16_round(np.asarray(x, np.float32)).astype(np.float64)


@pytest.mark.parametrize("kind,f", [("fixed_k", 512), ("variable", 512), ("variable", 256)])
def test_interaction_network_matches_oracle(cuda, kind, f):
  from faster_weathernext.gnn import GNNConfig, InteractionNetwork
  ns, nr = 777, 1_203
  snd, rcv = _graph(kind, ns, nr, 5)
  cfg = GNNConfig(latent=f, hidden=512, aggregate_normalization=4.0)
  net = InteractionNetwork(cfg, seed=3, device=cuda)
  with torch.no_grad():
    for prm in (net.b1, net.b2, net.c1, net.c2, net.d1, net.d2, net.ln_e_b, net.ln_r_b, net.ln_s_b):
      prm.normal_(0, 0.1)
    for prm in (net.ln_e_g, net.ln_r_g, net.ln_s_g):
      prm.uniform_(0.5, 1.5)
  g = torch.Generator(device=cuda).manual_seed(9)
  sx = torch.randn(ns, f, device=cuda, generator=g)
  rx = torch.randn(nr, f, device=cuda, generator=g)
  ex = torch.randn(snd.size, f, device=cuda, generator=g)
  new_s, new_r = net(sx, rx, ex, torch.from_numpy(snd), torch.from_numpy(rcv), edge_chunk=0)
  torch.cuda.synchronize()
  params = {k: _bf(v.detach().cpu().numpy()) for k, v in net.named_parameters()}
  ref_s, ref_r = og.interaction_network(params, _bf(sx.cpu()), _bf(rx.cpu()), _bf(ex.cpu()), snd, rcv,
                                        eps=cfg.eps, norm=1.0 / cfg.aggregate_normalization)
  # The updates (outputs minus the residual inputs) carry the network's error.
  for got, ref, x in ((new_r, ref_r, rx), (new_s, ref_s, sx)):
    assert oa.rel_rms(got.cpu().numpy() - x.cpu().numpy(), ref - _bf(x.cpu())) <= 2e-2
  # Blocks of 500 edges (a receiver's run split across blocks) give the same result up to summation order.
  new_s2, new_r2 = net(sx, rx, ex, torch.from_numpy(snd), torch.from_numpy(rcv), edge_chunk=500)
  assert torch.equal(new_s2, new_s)
  assert float((new_r2 - new_r).abs().max()) <= 1e-4 * float(new_r.abs().max())


def test_gnn_kernels_against_torch(cuda):
  """fwn_gnn_gather_add_act and fwn_gnn_ln_segment_sum on their own (bf16 inputs, float32 math)."""
  from faster_weathernext import _lib
  from faster_weathernext.gnn import segment_offsets
  lib = _lib.lib()
  g = torch.Generator(device=cuda).manual_seed(2)
  e, ns, nr, h = 3_001, 400, 700, 512
  snd = torch.randint(0, ns, (e,), device=cuda, generator=g).to(torch.int32)
  rcv = torch.sort(torch.randint(0, nr, (e,), device=cuda, generator=g)).values.to(torch.int32)
  ep, sp, rp = (torch.randn(n, h, device=cuda, generator=g).to(torch.bfloat16) for n in (e, ns, nr))
  b = torch.randn(h, device=cuda, generator=g).to(torch.bfloat16)
  out = torch.empty(e, h, device=cuda, dtype=torch.bfloat16)
  _lib.check(lib.fwn_gnn_gather_add_act(ep.data_ptr(), sp.data_ptr(), snd.data_ptr(), rp.data_ptr(), rcv.data_ptr(),
                                        b.data_ptr(), e, h, _lib.ACT_SWISH, out.data_ptr(), 0))
  x = ep.float() + sp.float()[snd.long()] + rp.float()[rcv.long()] + b.float()
  ref = x * torch.sigmoid(x)
  torch.cuda.synchronize()
  assert float(((out.float() - ref) ** 2).mean().sqrt() / ref.std()) <= 5e-3
  seg = segment_offsets(rcv, nr)
  gm = torch.rand(h, device=cuda, generator=g).to(torch.bfloat16)
  bt = torch.randn(h, device=cuda, generator=g).to(torch.bfloat16)
  res = torch.randn(nr, h, device=cuda, generator=g)
  agg = torch.empty(nr, h, device=cuda)
  _lib.check(lib.fwn_gnn_ln_segment_sum(out.data_ptr(), seg.data_ptr(), nr, h, gm.data_ptr(), bt.data_ptr(), 1e-5, 0.5,
                                        res.data_ptr(), agg.data_ptr(), _lib.DTYPE_F32, 0))
  ln = torch.nn.functional.layer_norm(out.float(), (h,), gm.float(), bt.float(), 1e-5)
  ref = torch.zeros(nr, h, device=cuda).index_add_(0, rcv.long(), ln) * 0.5 + res
  torch.cuda.synchronize()
  assert float((agg - ref).abs().max()) <= 1e-3 * float(ref.abs().max())
  empty = torch.diff(seg) == 0
  assert bool(empty.any()) and torch.allclose(agg[empty], res[empty])
  with pytest.raises(ValueError):
    segment_offsets(rcv.flip(0), nr)
