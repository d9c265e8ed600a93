"""Grid <-> mesh interaction networks of the encoder / decoder on B200 (src/faster_weathernext/patch.py:347-509).

The reference's ChunkedDeepGNN runs the official one-step InteractionNetwork block by block so that the per-edge
tensors (3.1 M mesh -> grid edges x 768 features) never exist whole: the first layer of the edge MLP is applied per
node before the gather (pre_gather_{senders,receivers,edges}_for_edges_fn), the messages of a block of edges are
summed into their receivers with a sorted segment_sum, and the nodes are updated by a node MLP with a residual. The
MLPs themselves are the third-party `weathernext` package's, which is not available here; this module restates
the structure with the conventional interaction-network MLPs (one hidden layer, swish, LayerNorm on the output):

    m_e   = LN_e(swish(e_e W_e + s[snd_e] W_s + r[rcv_e] W_r + b1) W2 + b2)
    agg_i = norm * sum over the edges e into receiver i of m_e                      (edges sorted by receiver)
    r_i'  = r_i + LN_r(swish(r_i U_r + agg_i U_a + c1) U2 + c2)
    s_j'  = s_j + LN_s(swish(s_j V_s + d1) V2 + d2)                                  (senders: no messages)

Kernels: the matmuls on fwn_gemm_bf16 (this package's tcgen05 GEMM; cuBLAS where a width does not fit its tiles);
the MLPs' input layers as fwn_gemm_bf16_gather, whose epilogue adds the gathered pre-projected sender / receiver
rows (edge MLP) or the aggregate's projection (receiver MLP) and the bias, then swish, so that the layer's own
product never goes to memory (fwn_gnn_gather_add_act does the same adds after a plain GEMM where the widths do not
fit the tiles); and the message LayerNorm with the sorted segment-sum in one pass, one warp per receiver, no atomics
(fwn_gnn_ln_segment_sum). Edges are processed in blocks of patch.OPTIONS.edge_chunk (0: all at once): a block's
receivers are a contiguous id range, and their running sums accumulate in float32. Features [n, F] for one sample
(the reference's [n, batch, F] is a loop over the batch here), bf16 matmuls with float32 accumulation, float32
node outputs.
"""

import dataclasses
import math
from typing import Optional

import numpy as np
import torch

from faster_weathernext import _lib
from faster_weathernext import patch


@dataclasses.dataclass
class GNNConfig:
  latent: int = 512        # node and edge feature width F
  hidden: int = 512        # MLP hidden width H
  aggregate_normalization: Optional[float] = None  # agg / this (the reference's _aggregate_normalization)
  eps: float = 1e-5


def _glorot(gen, fan_in, fan_out, device):
  bound = math.sqrt(6.0 / (fan_in + fan_out))
  w = torch.empty(fan_in, fan_out, device=device)
  w.uniform_(-bound, bound, generator=gen)
  return torch.nn.Parameter(w)


def segment_offsets(receivers: torch.Tensor, n_receivers: int) -> torch.Tensor:
  """CSR offsets [n_receivers + 1] (int32) of edges sorted by receiver; raises if they are not sorted."""
  r = receivers.to(torch.int64)
  if r.numel() and bool((r[1:] < r[:-1]).any()):
    raise ValueError("edges must be sorted by receiver (the reference's indices_are_sorted=True)")
  counts = torch.bincount(r, minlength=n_receivers) if r.numel() else torch.zeros(n_receivers, dtype=torch.int64,
                                                                                  device=receivers.device)
  seg = torch.zeros(n_receivers + 1, dtype=torch.int64, device=receivers.device)
  seg[1:] = torch.cumsum(counts, 0)
  return seg.to(torch.int32)


class InteractionNetwork(torch.nn.Module):
  """One message-passing step from sender nodes to receiver nodes over edges sorted by receiver (inference)."""

  def __init__(self, cfg: GNNConfig = GNNConfig(), seed: int = 0, device=None):
    super().__init__()
    self.cfg = cfg
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(seed)
    f, h = cfg.latent, cfg.hidden
    mk = lambda a, b: _glorot(g, a, b, dev)
    zeros = lambda n: torch.nn.Parameter(torch.zeros(n, device=dev))
    ones = lambda n: torch.nn.Parameter(torch.ones(n, device=dev))
    # edge MLP (first layer split over its three inputs), receiver MLP (split over node and aggregate), sender MLP
    self.w_e, self.w_s, self.w_r, self.b1, self.w2, self.b2 = mk(f, h), mk(f, h), mk(f, h), zeros(h), mk(h, f), zeros(f)
    self.ln_e_g, self.ln_e_b = ones(f), zeros(f)
    self.u_r, self.u_a, self.c1, self.u2, self.c2 = mk(f, h), mk(f, h), zeros(h), mk(h, f), zeros(f)
    self.ln_r_g, self.ln_r_b = ones(f), zeros(f)
    self.v_s, self.d1, self.v2, self.d2 = mk(f, h), zeros(h), mk(h, f), zeros(f)
    self.ln_s_g, self.ln_s_b = ones(f), zeros(f)
    self._cache = {}

  # bf16 copies of the parameters (transposed for the GEMM's K-major weight operand), recast when a parameter changes
  def _bf(self, p, transpose=False):
    key = (id(p), transpose)
    hit = self._cache.get(key)
    if hit is not None and hit[0] == p._version and hit[1] == p.data_ptr():
      return hit[2]
    w = (p.detach().t() if transpose else p.detach()).contiguous().to(torch.bfloat16)
    self._cache[key] = (p._version, p.data_ptr(), w)
    return w

  def _mm(self, x, w, bias=None, act=_lib.ACT_NONE):
    """bf16 x [m, k] @ w [k, n] (+ bias, act) on fwn_gemm_bf16 where the widths fit its tiles, else cuBLAS."""
    m, k = x.shape
    n = w.shape[1]
    if n % 256 == 0 and k % 64 == 0 and m > 0:
      out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
      _lib.check(_lib.lib().fwn_gemm_bf16(x.data_ptr(), self._bf(w, True).data_ptr(),
                                          self._bf(bias).data_ptr() if bias is not None else None, out.data_ptr(),
                                          m, n, k, act, torch.cuda.current_stream().cuda_stream))
      return out
    y = x @ self._bf(w) + (self._bf(bias) if bias is not None else 0)
    if act == _lib.ACT_GELU_TANH:
      y = torch.nn.functional.gelu(y, approximate="tanh")
    return y

  def _mm_add_act(self, x, w, bias, add0=None, idx0=None, add1=None, idx1=None):
    """swish(x w + bias + add0[idx0] + add1[idx1]) in bf16: fwn_gemm_bf16_gather (the adds and swish in the GEMM's
    epilogue, one pass) where the widths fit its tiles; else the GEMM, then fwn_gnn_gather_add_act. idx None: the
    row itself."""
    m, k = x.shape
    n = w.shape[1]
    if n % 256 == 0 and k % 64 == 0 and m > 0:
      out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
      ptr = lambda t: t.data_ptr() if t is not None else None
      rows = lambda t: t.shape[0] if t is not None else 0
      _lib.check(_lib.lib().fwn_gemm_bf16_gather(
          x.data_ptr(), self._bf(w, True).data_ptr(), self._bf(bias).data_ptr(), out.data_ptr(), ptr(add0), ptr(idx0),
          rows(add0), ptr(add1), ptr(idx1), rows(add1), m, n, k, _lib.ACT_SWISH, torch.cuda.current_stream().cuda_stream))
      return out
    return self._gather_act(m, n, e_proj=self._mm(x, w), s_proj=add0, snd=idx0, r_proj=add1, rcv=idx1,
                            bias=self._bf(bias))

  def _gather_act(self, rows, h, e_proj=None, s_proj=None, snd=None, r_proj=None, rcv=None, bias=None, act=True):
    out = torch.empty(rows, h, dtype=torch.bfloat16, device=self.b1.device)
    p = lambda t: t.data_ptr() if t is not None else None
    _lib.check(_lib.lib().fwn_gnn_gather_add_act(p(e_proj), p(s_proj), p(snd), p(r_proj), p(rcv), p(bias), rows, h,
                                                 _lib.ACT_SWISH if act else _lib.ACT_NONE, out.data_ptr(),
                                                 torch.cuda.current_stream().cuda_stream))
    return out

  def _ln_sum(self, m, seg, n_out, gamma, beta, norm=1.0, residual=None, out=None):
    f = m.shape[1]
    if out is None:
      out = torch.empty(n_out, f, dtype=torch.float32, device=m.device)
    _lib.check(_lib.lib().fwn_gnn_ln_segment_sum(m.data_ptr(), seg.data_ptr() if seg is not None else None, n_out, f,
                                                 self._bf(gamma).data_ptr(), self._bf(beta).data_ptr(),
                                                 self.cfg.eps, norm, residual.data_ptr() if residual is not None else None,
                                                 out.data_ptr(), _lib.DTYPE_F32, torch.cuda.current_stream().cuda_stream))
    return out

  def _node_mlp(self, x32, x16, w_in, b_in, w_out, b_out, ln_g, ln_b, agg16=None, w_agg=None):
    """x + LN(swish(x w_in (+ agg w_agg) + b_in) w_out + b_out), x float32 [n, F] (x16 its bf16 copy)."""
    n = x32.shape[0]
    ha = self._mm(agg16, w_agg) if agg16 is not None else None
    hid = self._mm_add_act(x16, w_in, b_in, add0=ha)
    y = self._mm(hid, w_out, b_out)
    return self._ln_sum(y, None, n, ln_g, ln_b, residual=x32)

  @torch.no_grad()
  def forward(self, senders_x, receivers_x, edges_x, senders, receivers, edge_chunk: Optional[int] = None):
    """senders_x [Ns, F], receivers_x [Nr, F], edges_x [E, F] (float32 or bf16); senders / receivers int [E], edges
    sorted by receiver. Returns (senders_x', receivers_x') float32. edge_chunk: edges per block (default
    patch.OPTIONS.edge_chunk; 0 or None: all edges at once)."""
    cfg = self.cfg
    if edge_chunk is None:
      edge_chunk = patch.OPTIONS.edge_chunk
    ns, nr, ne = senders_x.shape[0], receivers_x.shape[0], edges_x.shape[0]
    dev = senders_x.device
    snd = senders.to(device=dev, dtype=torch.int32).contiguous()
    rcv = receivers.to(device=dev, dtype=torch.int32).contiguous()
    if ne and (int(snd.min()) < 0 or int(snd.max()) >= ns or int(rcv.min()) < 0 or int(rcv.max()) >= nr):
      raise ValueError("sender / receiver index out of range")
    seg = segment_offsets(rcv, nr)
    s16, r16 = senders_x.to(torch.bfloat16).contiguous(), receivers_x.to(torch.bfloat16).contiguous()
    e16 = edges_x.to(torch.bfloat16).contiguous()
    # Pre-gather projections: the edge MLP's first layer on each node once.
    s_proj = self._mm(s16, self.w_s)
    r_proj = self._mm(r16, self.w_r)
    norm = 1.0 / cfg.aggregate_normalization if cfg.aggregate_normalization else 1.0
    agg = torch.zeros(nr, cfg.latent, dtype=torch.float32, device=dev)
    block = ne if not edge_chunk or edge_chunk <= 0 else int(edge_chunk)
    plan = []
    if block < ne:
      # Each block's receivers are a contiguous id range; their runs clipped to the block, all blocks' offsets
      # computed on the host and uploaded once (no copy, and no wait, inside the loop).
      seg_host = seg.cpu().numpy().astype(np.int64)
      parts, off = [], 0
      for e0 in range(0, ne, block):
        e1 = min(ne, e0 + block)
        r_lo = int(np.searchsorted(seg_host, e0, side="right")) - 1
        r_hi = int(np.searchsorted(seg_host, e1, side="left"))
        parts.append(np.clip(seg_host[r_lo:r_hi + 1], e0, e1) - e0)
        plan.append((e0, e1, r_lo, r_hi, off))
        off += r_hi - r_lo + 1
      subs = torch.from_numpy(np.concatenate(parts).astype(np.int32)).to(dev)
    else:
      plan.append((0, ne, 0, nr, None))
    for e0, e1, r_lo, r_hi, off in plan:
      if e1 <= e0:
        continue
      hid = self._mm_add_act(e16[e0:e1], self.w_e, self.b1, add0=s_proj, idx0=snd[e0:e1], add1=r_proj,
                             idx1=rcv[e0:e1])
      msg = self._mm(hid, self.w2, self.b2)
      if off is None:
        self._ln_sum(msg, seg, nr, self.ln_e_g, self.ln_e_b, norm=norm, out=agg)
      else:
        part = agg[r_lo:r_hi]
        self._ln_sum(msg, subs[off:off + r_hi - r_lo + 1], r_hi - r_lo, self.ln_e_g, self.ln_e_b, norm=norm,
                     residual=part, out=part)
    agg16 = agg.to(torch.bfloat16)
    new_r = self._node_mlp(receivers_x.float().contiguous(), r16, self.u_r, self.c1, self.u2, self.c2, self.ln_r_g,
                           self.ln_r_b, agg16=agg16, w_agg=self.u_a)
    new_s = self._node_mlp(senders_x.float().contiguous(), s16, self.v_s, self.d1, self.v2, self.d2, self.ln_s_g,
                           self.ln_s_b)
    return new_s, new_r

  def flops(self, ns, nr, ne):
    """Matmul FLOPs of one forward (the edge MLP's two layers over the edges dominate)."""
    f, h = self.cfg.latent, self.cfg.hidden
    return 2.0 * (ns * f * h + nr * f * h + ne * f * h + ne * h * f + nr * 2 * f * h + nr * h * f + ns * f * h + ns * h * f)
