"""Mesh-transformer processor around the B200 attention op (configurations 4 and 5).

Structure of the reference's patched processor (src/faster_weathernext/patch.py:229-293): pre-LN blocks

    h = cond(LN(x));  x = x + mha_final(attention(q(h), k(h), v(h)))      (patch.py:238-246, tiled_mha :165-177)
    x = x + ffw(cond(LN(x)))                                               (patch.py:250-252)

with LayerNorm without scale / offset, a norm conditioning (per-sample scale and offset from the
conditioning vector, as the official LinearNormConditioning), a final LN + conditioning (patch.py:288-290),
q/k/v/out projections and a GELU MLP. The official modules (`weathernext.utils.sparse_transformer`,
`dense.LinearNormConditioning`) are third-party and not available here, so this is a synthetic processor of
the configurations' shape (24 blocks, width 512, 8 x 64 heads, MLP 2048, GELU in the tanh form that is
jax.nn.gelu's default; Glorot-uniform weights from a seed), not a numerical copy of the official one. The
q/k/v, output and down projections run as cuBLAS GEMMs; the attention block is patch.tiled_mha (the B200 kernel;
q, k, v are strided views of one fused projection, no copies, and its backward writes their gradients into one
tensor). Without autograd (inference), each norm is one fused kernel that also adds the previous sub-block's output
into the residual stream, and the MLP up-projection runs on this package's tcgen05 GEMM with bias + GELU in its
epilogue (faster than cuBLASLt's GELU epilogue at these shapes). With autograd in bf16 (training), the norms are a
differentiable fused kernel pair (_CondNorm: residual add + norm forward, one-pass backward) and the MLP's GELU and its
backward live in the same GEMM's epilogues (_GeluMLP). With patch.OPTIONS.remat, each block's activations are
recomputed in the backward instead of stored (the reference's per-layer rematerialisation, patch.py:69-73).

Node order: the reference's transformer gathers the latents into the mask's node order with `perm` before the
first block and takes them back with argsort(perm) after the final norm (patch.py:275-276, 291-292). `forward`
does the same when given `perm`; on the inference path the gather is the residual stream's initial copy and the
un-permutation is fused into the final norm's store (fwn_cond_layernorm_scatter).
"""

import dataclasses
import math

import torch
import torch.nn.functional as F
import torch.utils.checkpoint

from faster_weathernext import _lib
from faster_weathernext import patch
from faster_weathernext import tiled_attn


@dataclasses.dataclass
class ProcessorConfig:
  layers: int = 24
  d_model: int = 512
  heads: int = 8
  head_dim: int = 64
  mlp_hidden: int = 2048
  cond_dim: int = 32


def _glorot(gen, fan_in, fan_out, device):
  bound = math.sqrt(6.0 / (fan_in + fan_out))
  w = torch.empty(fan_in, fan_out, device=device)
  w.uniform_(-bound, bound, generator=gen)
  return torch.nn.Parameter(w)


class _CondNorm(torch.autograd.Function):
  """Differentiable fused conditioned norm of the training path: h = cond_norm(x) or, with a sub-block output a,
  (x + a, cond_norm(x + a)). x float32 [M, d] (M = samples x rows_per_sample), a bf16 [M, d] or None, so float32
  [samples, 2 d] (per-sample scale, offset). Forward: one pass (fwn_cond_layernorm / fwn_cond_layernorm_add);
  backward: one pass for dx (plus the incoming gradient of x + a, plus the bf16 gradient of a) and one small
  deterministic reduction for the scale / offset gradient (fwn_cond_layernorm_bwd). Replaces the add, LayerNorm,
  multiply-add, casts and their backward kernels of the composed torch form, _cond_norm."""

  @staticmethod
  def forward(ctx, x, a, so, rows_per_sample, out_dtype):
    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    m, d = x.shape
    h = torch.empty(m, d, dtype=out_dtype, device=x.device)
    code = _lib.DTYPE_BF16 if out_dtype == torch.bfloat16 else _lib.DTYPE_F32
    ctx.rows_per_sample = rows_per_sample
    ctx.has_a = a is not None
    ctx.set_materialize_grads(False)
    if a is None:
      _lib.check(lib.fwn_cond_layernorm(x.data_ptr(), m, d, rows_per_sample, so.data_ptr(), _EPS, h.data_ptr(), code,
                                        stream))
      ctx.save_for_backward(x, so)
      return h
    xn = torch.empty_like(x)
    _lib.check(lib.fwn_cond_layernorm_add(x.data_ptr(), a.data_ptr(), xn.data_ptr(), m, d, rows_per_sample,
                                          so.data_ptr(), _EPS, h.data_ptr(), code, stream))
    ctx.save_for_backward(xn, so)
    return xn, h

  @staticmethod
  def backward(ctx, *grads):
    xn, so = ctx.saved_tensors
    g_xn, g_h = (grads[0], grads[1]) if ctx.has_a else (None, grads[0])
    m, d = xn.shape
    if g_h is None:
      g_h = torch.zeros(m, d, dtype=torch.float32, device=xn.device)
    if g_h.dtype not in (torch.bfloat16, torch.float32):
      g_h = g_h.float()
    g_h = g_h.contiguous()
    if g_xn is not None:
      g_xn = g_xn.float().contiguous()
    lib = _lib.lib()
    dx = torch.empty_like(xn)
    da = torch.empty(m, d, dtype=torch.bfloat16, device=xn.device) if ctx.has_a else None
    dso = torch.empty_like(so)
    nbytes = lib.fwn_cond_layernorm_bwd_workspace(m, d, ctx.rows_per_sample)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=xn.device)
    _lib.check(lib.fwn_cond_layernorm_bwd(
        xn.data_ptr(), m, d, ctx.rows_per_sample, so.data_ptr(), _EPS, g_h.data_ptr(),
        _lib.DTYPE_BF16 if g_h.dtype == torch.bfloat16 else _lib.DTYPE_F32,
        g_xn.data_ptr() if g_xn is not None else None, dx.data_ptr(), da.data_ptr() if da is not None else None,
        dso.data_ptr(), ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream))
    return dx, da, dso, None, None


_EPS = 1e-5


class _GeluMLP(torch.autograd.Function):
  """The training path's MLP, GELU(h w1 + b1) w2 + b2 in bf16 (h bf16 [M, d]; w1 [d, hidden], b1, w2 [hidden, d],
  b2 float32 parameters), with the GELU in the epilogues of this package's GEMM: forward fwn_gemm_bf16_aux with
  FWN_ACT_GELU_TANH_AUX (the activation, and the pre-activation kept for the backward, in one pass); backward
  d_pre = (d_out w2^T) GELU'(pre) by the same GEMM with FWN_ACT_GELU_TANH_GRAD (w2 as stored is its K-major
  operand). The down-projection and the weight / input gradients are cuBLAS GEMMs; the bias gradients are float32
  column sums. Replaces torch's bias + GELU forward and GELU backward passes over the [M, hidden] activations.
  Requires hidden % 256 == 0 and d % 64 == 0."""

  @staticmethod
  def forward(ctx, h, w1, b1, w2, b2):
    bf = torch.bfloat16
    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    m, d = h.shape
    hidden = w1.shape[1]
    w1t = w1.detach().t().contiguous().to(bf)           # [hidden, d]: K-major operand of the up-projection
    w2h = w2.detach().to(bf)                            # [hidden, d]
    pre = torch.empty(m, hidden, dtype=bf, device=h.device)
    act = torch.empty(m, hidden, dtype=bf, device=h.device)
    _lib.check(lib.fwn_gemm_bf16_aux(h.data_ptr(), w1t.data_ptr(), b1.detach().to(bf).data_ptr(), act.data_ptr(),
                                     pre.data_ptr(), m, hidden, d, _lib.ACT_GELU_TANH_AUX, stream))
    out = torch.addmm(b2.detach().to(bf), act, w2h)
    ctx.save_for_backward(h, pre, act, w1t, w2h)
    return out

  @staticmethod
  def backward(ctx, d_out):
    h, pre, act, w1t, w2h = ctx.saved_tensors
    lib = _lib.lib()
    m, hidden = pre.shape
    d = h.shape[1]
    d_out = d_out.to(torch.bfloat16).contiguous()
    d_pre = torch.empty_like(pre)
    _lib.check(lib.fwn_gemm_bf16_aux(d_out.data_ptr(), w2h.data_ptr(), None, d_pre.data_ptr(), pre.data_ptr(), m,
                                     hidden, d, _lib.ACT_GELU_TANH_GRAD, torch.cuda.current_stream().cuda_stream))
    d_b2 = torch.sum(d_out, 0, dtype=torch.float32)
    d_w2 = torch.mm(act.t(), d_out).float()
    d_b1 = torch.sum(d_pre, 0, dtype=torch.float32)
    d_w1 = torch.mm(h.t(), d_pre).float()
    d_h = torch.mm(d_pre, w1t)
    return d_h, d_w1, d_b1, d_w2, d_b2


class Processor(torch.nn.Module):
  """Random-init processor; parameters float32, compute in `dtype` (bf16 by default)."""

  def __init__(self, cfg: ProcessorConfig = ProcessorConfig(), seed: int = 0, device=None):
    super().__init__()
    self.cfg = cfg
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev).manual_seed(seed)
    d, hd = cfg.d_model, cfg.heads * cfg.head_dim
    self.blocks = torch.nn.ModuleList()
    for _ in range(cfg.layers):
      blk = torch.nn.Module()
      # Fused q/k/v projection; output columns ordered [head, (q, k, v), head_dim] so that q, k, v are
      # strided [B, n, H, D] views of one tensor.
      blk.w_qkv = _glorot(gen, d, 3 * hd, dev)
      blk.w_out = _glorot(gen, hd, d, dev)
      blk.w1 = _glorot(gen, d, cfg.mlp_hidden, dev)
      blk.b1 = torch.nn.Parameter(torch.zeros(cfg.mlp_hidden, device=dev))
      blk.w2 = _glorot(gen, cfg.mlp_hidden, d, dev)
      blk.b2 = torch.nn.Parameter(torch.zeros(d, device=dev))
      blk.cond1 = _glorot(gen, cfg.cond_dim, 2 * d, dev)
      blk.cond2 = _glorot(gen, cfg.cond_dim, 2 * d, dev)
      self.blocks.append(blk)
    self.cond_final = _glorot(gen, cfg.cond_dim, 2 * d, dev)
    self._bf16_cache = {}
    # With autograd and bf16 compute: the fused differentiable norms (_forward_train); False selects the composed
    # torch form of the same blocks (_block), which other dtypes and widths take.
    self.fused_training = True

  def _bf16_t(self, p: torch.Tensor) -> torch.Tensor:
    """bf16 copy of p's transpose (contiguous), the K-major weight operand of fwn_gemm_bf16; cached as _bf16."""
    key = ("t", id(p))
    hit = self._bf16_cache.get(key)
    if hit is not None and hit[0] == p._version and hit[1] == p.data_ptr():
      return hit[2]
    w = p.detach().t().contiguous().to(torch.bfloat16)
    self._bf16_cache[key] = (p._version, p.data_ptr(), w)
    return w

  def _mlp_up(self, h: torch.Tensor, blk) -> torch.Tensor:
    """GELU(h @ w1 + b1) in bf16 for the inference path: fwn_gemm_bf16 with bias and GELU in its epilogue where the
    shapes fit its tiles (hidden a multiple of 256, width of 64), cuBLASLt's bias + GELU epilogue otherwise."""
    m, d = h.shape
    hidden = blk.w1.shape[1]
    if hidden % 256 or d % 64:
      return torch._addmm_activation(self._bf16(blk.b1), h, self._bf16(blk.w1), use_gelu=True)
    lib = _lib.lib()
    out = torch.empty(m, hidden, dtype=torch.bfloat16, device=h.device)
    _lib.check(lib.fwn_gemm_bf16(h.data_ptr(), self._bf16_t(blk.w1).data_ptr(), self._bf16(blk.b1).data_ptr(),
                                 out.data_ptr(), m, hidden, d, _lib.ACT_GELU_TANH,
                                 torch.cuda.current_stream().cuda_stream))
    return out

  def _bf16(self, p: torch.Tensor) -> torch.Tensor:
    """bf16 copy of parameter p for the inference path, cast again only when p has changed: the cache entry
    holds p's storage address and in-place version counter, which optimizer steps, load_state_dict and .to()
    change. The 16 forwards of a processor step therefore cast each weight once, not once per forward."""
    hit = self._bf16_cache.get(id(p))
    if hit is not None and hit[0] == p._version and hit[1] == p.data_ptr():
      return hit[2]
    w = p.detach().to(torch.bfloat16)
    self._bf16_cache[id(p)] = (p._version, p.data_ptr(), w)
    return w

  def _mha(self, h, w_qkv, w_out, tiles):
    """The attention block: patch.tiled_mha over the fused projection (h [B, n, d] in the compute dtype)."""
    cfg = self.cfg
    return patch.tiled_mha(h, w_qkv, w_out, tiles, cfg.heads, cfg.head_dim)

  @staticmethod
  def _cond_norm(x, cond, w):
    """LayerNorm without scale / offset, then x * (1 + scale) + offset from the conditioning vector."""
    y = F.layer_norm(x, x.shape[-1:])
    so = (cond @ w.to(cond.dtype)).unsqueeze(1)          # [B, 1, 2d]
    scale, offset = so.chunk(2, dim=-1)
    return y * (1 + scale) + offset

  def forward(self, x: torch.Tensor, cond: torch.Tensor, tiles: "tiled_attn.AttentionTiles",
              dtype=torch.bfloat16, perm: torch.Tensor = None) -> torch.Tensor:
    """x [B, n, d_model] (float32 residual stream), cond [B, cond_dim] -> [B, n, d_model]. `perm` (int, [n],
    a permutation of the nodes; optional): `tiles` is built in the permuted order, node i of the blocks is node
    perm[i] of x, and the output is returned in x's order."""
    b, n, d = x.shape
    if cond.dim() != 2 or cond.shape[0] not in (1, b):
      raise ValueError(f"cond has shape {tuple(cond.shape)}, expected ({b}, cond_dim) or (1, cond_dim)")
    if perm is not None:
      perm = torch.as_tensor(perm, device=x.device).to(torch.int64)
      if perm.shape != (n,):
        raise ValueError(f"perm has shape {tuple(perm.shape)}, expected ({n},)")
      if n and (int(perm.min()) < 0 or int(perm.max()) >= n or
                not bool((torch.bincount(perm, minlength=n) == 1).all())):
        raise ValueError("perm is not a permutation of the nodes")
    fused_ok = x.dtype == torch.float32 and d in (128, 256, 512, 1024)
    if not torch.is_grad_enabled() and dtype == torch.bfloat16 and fused_ok:
      return self._forward_fused(x, cond.expand(b, -1), tiles, perm)
    if dtype == torch.bfloat16 and fused_ok and d <= 512 and self.fused_training:
      return self._forward_train(x, cond.expand(b, -1), tiles, perm)
    c = cond.to(dtype)
    if perm is not None:
      x = x.index_select(1, perm)
    remat = patch.OPTIONS.remat and torch.is_grad_enabled()
    for blk in self.blocks:
      if remat:
        x = torch.utils.checkpoint.checkpoint(self._block, x, c, blk, tiles, dtype, use_reentrant=False)
      else:
        x = self._block(x, c, blk, tiles, dtype)
    y = self._cond_norm(x, c, self.cond_final).to(x.dtype)
    if perm is not None:
      y = y.index_select(1, torch.argsort(perm))
    return y

  def _block(self, x, c, blk, tiles, dtype):
    """One pre-LN block (patch.py:238-252): attention then MLP, each on a conditioned norm, residual adds."""
    h = self._cond_norm(x, c, blk.cond1).to(dtype)
    x = x + self._mha(h, blk.w_qkv.to(dtype), blk.w_out.to(dtype), tiles).to(x.dtype)
    h = self._cond_norm(x, c, blk.cond2).to(dtype)
    m = F.gelu(h @ blk.w1.to(dtype) + blk.b1.to(dtype), approximate="tanh")
    return x + (m @ blk.w2.to(dtype) + blk.b2.to(dtype)).to(x.dtype)

  def _forward_train(self, x, cond, tiles, perm=None):
    """The autograd path with the fused differentiable norms (_CondNorm): each norm also adds the previous
    sub-block's bf16 output into the float32 residual stream, and its backward is one pass plus a per-sample
    reduction. The MLP is _GeluMLP (GELU and its backward in this package's GEMM epilogues) where its shapes fit the
    GEMM's tiles, the other projections are cuBLAS GEMMs, the attention is patch.tiled_mha; the conditioning's
    scale / offset are computed in float32. x float32 [B, n, d]; cond [B, cond_dim]."""
    b, n, d = x.shape
    if perm is not None:
      x = x.index_select(1, perm)
    xs = x.reshape(b * n, d).contiguous()
    cf = cond.float()
    remat = patch.OPTIONS.remat
    pending = None
    for blk in self.blocks:
      so1 = cf @ blk.cond1.float()
      so2 = cf @ blk.cond2.float()
      if remat:
        xs, pending = torch.utils.checkpoint.checkpoint(self._block_train, xs, pending, so1, so2, blk, tiles, b, n,
                                                        use_reentrant=False)
      else:
        xs, pending = self._block_train(xs, pending, so1, so2, blk, tiles, b, n)
    so = cf @ self.cond_final.float()
    y = _CondNorm.apply(xs, pending, so, n, torch.float32)[1] if pending is not None else \
        _CondNorm.apply(xs, None, so, n, torch.float32)
    y = y.view(b, n, d)
    if perm is not None:
      y = y.index_select(1, torch.argsort(perm))
    return y

  def _block_train(self, xs, pending, so1, so2, blk, tiles, b, n):
    """One pre-LN block on the fused norms: returns the residual stream after the attention's add and the MLP's
    bf16 output, which the next norm adds (xs float32 [b n, d]; pending bf16 [b n, d] or None)."""
    bf = torch.bfloat16
    d = xs.shape[1]
    if pending is None:
      h = _CondNorm.apply(xs, None, so1, n, bf)
    else:
      xs, h = _CondNorm.apply(xs, pending, so1, n, bf)
    a = self._mha(h.view(b, n, d), blk.w_qkv.to(bf), blk.w_out.to(bf), tiles).reshape(b * n, d)
    xs, h = _CondNorm.apply(xs, a, so2, n, bf)
    if blk.w1.shape[1] % 256 == 0 and d % 64 == 0 and h.shape[0] > 0:
      return xs, _GeluMLP.apply(h, blk.w1, blk.b1, blk.w2, blk.b2)
    mlp = F.gelu(torch.addmm(blk.b1.to(bf), h, blk.w1.to(bf)), approximate="tanh")
    return xs, torch.addmm(blk.b2.to(bf), mlp, blk.w2.to(bf))

  def _forward_fused(self, x, cond, tiles, perm=None):
    """Inference: the same blocks with the LayerNorm, conditioning and cast in one kernel per norm, which also adds
    the previous sub-block's bf16 output into the float32 residual stream in place (fwn_cond_layernorm_residual: one
    pass instead of an add and a norm), the MLP up-projection with bias and GELU in the epilogue of this package's
    GEMM (fwn_gemm_bf16), the other projections on cuBLAS. x float32 [B, n, d]; cond [B, cond_dim]; perm checked by
    forward."""
    b, n, d = x.shape
    m_rows = b * n
    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    bf = torch.bfloat16
    # The residual stream: a copy of x, gathered into the blocks' node order when permuted.
    xs = x.index_select(1, perm).contiguous() if perm is not None else x.contiguous().clone()
    x2 = xs.view(m_rows, d)
    h = torch.empty(m_rows, d, dtype=bf, device=x.device)
    cf = cond.float()

    def norm(w, out, out_dtype, residual=None, out_node=None):
      """out = cond_norm(x) (x += residual first, in the same pass; rows to out_node[row] when given)."""
      so = (cf @ w.float()).contiguous()                    # [B, 2d]: per-sample scale, offset
      if residual is None and out_node is None:
        _lib.check(lib.fwn_cond_layernorm(x2.data_ptr(), m_rows, d, n, so.data_ptr(), 1e-5, out.data_ptr(),
                                          out_dtype, stream))
      elif residual is None:
        _lib.check(lib.fwn_cond_layernorm_scatter(x2.data_ptr(), m_rows, d, n, out_node.data_ptr(), so.data_ptr(),
                                                  1e-5, out.data_ptr(), out_dtype, stream))
      else:
        _lib.check(lib.fwn_cond_layernorm_residual(x2.data_ptr(), residual.data_ptr(), m_rows, d, n,
                                                   out_node.data_ptr() if out_node is not None else None,
                                                   so.data_ptr(), 1e-5, out.data_ptr(), out_dtype, stream))

    # Each sub-block's output (bf16) is added into the residual stream by the norm that follows it.
    pending = None
    for blk in self.blocks:
      norm(blk.cond1, h, _lib.DTYPE_BF16, residual=pending)
      pending = self._mha(h.view(b, n, d), self._bf16(blk.w_qkv), self._bf16(blk.w_out), tiles).view(m_rows, d)
      norm(blk.cond2, h, _lib.DTYPE_BF16, residual=pending)
      mlp = self._mlp_up(h, blk)
      pending = torch.addmm(self._bf16(blk.b2), mlp, self._bf16(blk.w2))
    out = torch.empty_like(xs)
    # Final norm; with perm, the un-permutation is fused into its store: row i of each sample goes to row perm[i].
    out_node = perm.to(torch.int32).contiguous() if perm is not None else None
    norm(self.cond_final, out.view(m_rows, d), _lib.DTYPE_F32, residual=pending, out_node=out_node)
    return out

  def gemm_flops_per_forward(self, n: int) -> float:
    """Projection + MLP GEMM FLOPs of one member's forward (2 n (4 d^2 + 2 d m) per block)."""
    cfg = self.cfg
    hd = cfg.heads * cfg.head_dim
    per = 2 * n * (cfg.d_model * 3 * hd + hd * cfg.d_model + 2 * cfg.d_model * cfg.mlp_hidden)
    return float(cfg.layers * per)
