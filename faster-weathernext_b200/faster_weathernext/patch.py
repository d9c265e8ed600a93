"""Options and the attention call of the patched processor (src/faster_weathernext/patch.py:50-99, 165-226).

`Options` keeps the reference's fields (read when a model is built / traced). This package acts on:
  attention     only "auto" / "tiled" select an implementation (the B200 kernels); "pallas" and "xla" name the
                reference's backends, which are not part of this build (ValueError);
  reorder       Hilbert order of the mesh nodes in transformer_tiles (patch.py:210-213);
  strict_fp32   passed to the attention as the reference's tiled_mha does (patch.py:173-174): it matters only
                under default_matmul_precision("highest"), where IEEE float32 dots are asked for (not built);
  remat         the processor recomputes each block's activations in the backward (patch.py:69-73);
  edge_chunk    edges per block of the grid <-> mesh interaction network (faster_weathernext.gnn).
The others configure parts of the reference this build does not include (its XLA attention fallback's chunk, the
node blocking of the GNNs, encoder and decoder, Haiku's layer loop, sequential samples in training); they are
accepted so that option sets written for the reference keep working, and setting one to a non-default value
warns that it has no effect here.

install() / uninstall() mark the patch active. The official `weathernext` (JAX / Haiku) package is not part of
this build: transformer_tiles is the mask part of the reference's _transformer_init and tiled_mha its
attention call, for the torch processor in faster_weathernext.processor.
"""

import dataclasses
import warnings

import torch

from faster_weathernext import tiled_attn


@dataclasses.dataclass
class Options:
  """Execution options (same names and defaults as the reference's, patch.py:50-82)."""
  attention: str = "auto"
  replace_attention: bool = True
  reorder: bool = True
  strict_fp32: bool = False
  attn_chunk: int = 512
  grid_chunk: int = 32768
  edge_chunk: int = 65536
  layer_loop: bool = True
  remat: bool = False
  sequential_samples: bool = False


OPTIONS = Options()
_enabled = False

# Options that configure parts of the reference this build does not include, and what they configure.
NO_EFFECT = {
    "replace_attention": "which attention types of the official configs are routed to the fused kernel "
                         "(every attention here is the fused kernel)",
    "attn_chunk": "the query chunk of the reference's XLA attention fallback (not built: no fallback)",
    "grid_chunk": "the node blocking of the grid / mesh GNNs, encoder and decoder (the interaction network here "
                  "processes all nodes at once; edge_chunk blocks its edges)",
    "layer_loop": "Haiku's scan over the transformer layers (the torch processor runs its layers eagerly)",
    "sequential_samples": "the reference's training loop over samples (DataParallelStep's micro_batch sets "
                          "how many members run together)",
}


def warn_no_effect(changed):
  """Warn once per call for options in `changed` that have no effect in this build."""
  defaults = Options()
  names = [k for k in changed if k in NO_EFFECT and getattr(OPTIONS, k) != getattr(defaults, k)]
  for k in names:
    warnings.warn(f"faster_weathernext option {k}={getattr(OPTIONS, k)!r} has no effect in this build: it "
                  f"configures {NO_EFFECT[k]}", UserWarning, stacklevel=3)
  return names


def attention_impl() -> str:
  """The attention implementation in use: "tiled" (the sm_100a kernels). Unlike the reference
  (patch.py:86-99) there is no fallback: anything but an sm_100 device is an error."""
  if OPTIONS.attention not in ("auto", "tiled"):
    raise ValueError(f"attention={OPTIONS.attention!r}: this build has one implementation, 'tiled' (B200)")
  if not torch.cuda.is_available():
    raise RuntimeError("faster_weathernext needs a CUDA device (sm_100a)")
  major, _ = torch.cuda.get_device_capability()
  if major != 10:
    raise RuntimeError(f"faster_weathernext's kernels are built for sm_100a; found sm_{major}x")
  return "tiled"


def install(force: bool = False):
  """Activate the patch (idempotent). Checks the device unless force=True."""
  global _enabled
  if not force:
    attention_impl()
  _enabled = True


def uninstall():
  global _enabled
  _enabled = False


def is_enabled() -> bool:
  return _enabled


def transformer_tiles(adj_mat, attention_k_hop: int, latlon=None, device=None):
  """The mask part of the reference's patched Transformer.__init__ (_transformer_init, patch.py:207-219) under
  OPTIONS: tile lists of adj_mat ** attention_k_hop, in Hilbert order when OPTIONS.reorder and the nodes'
  (lat, lon) are known (argument, or adj_mat._fwn_latlon as the reference's patched _get_adjacency_matrix sets
  it), with the transposed mask's lists when adj_mat is not symmetric. Returns (AttentionTiles, perm or None);
  perm goes to the processor's forward as the reference's num_padding_nodes slot carries it to its blocks
  (patch.py:219, 275-276)."""
  attention_impl()
  return tiled_attn.AttentionTiles.from_adjacency(adj_mat, attention_k_hop, latlon=latlon,
                                                  reorder=OPTIONS.reorder, device=device)


def tiled_mha(x, w_qkv, w_out, tiles: "tiled_attn.AttentionTiles", heads: int, key_size: int, b_out=None):
  """patch.tiled_mha (patch.py:165-177) for torch: q / k / v projections, the block-sparse attention with scale
  key_size ** -0.5 and strict_fp32=OPTIONS.strict_fp32 (precision from the enclosing
  tiled_attn.default_matmul_precision block), then the output projection.

  x [B, n, d]; w_qkv [d, heads * 3 * key_size], output columns ordered [head, (q, k, v), key_size] so that q, k, v
  are strided [B, n, heads, key_size] views of one GEMM's output (the kernels read them in place, no copies, and
  the backward writes their gradients into one [B, n, heads, 3, key_size] tensor, tiled_attn.attention_qkv);
  w_out [heads * key_size, d_out]; b_out [d_out] or None. Returns [B, n, d_out] in x's dtype."""
  b, n, _ = x.shape
  qkv = (x @ w_qkv).view(b, n, heads, 3, key_size)
  out = tiled_attn.attention_qkv(qkv, tiles, scale=key_size ** -0.5, strict_fp32=OPTIONS.strict_fp32)
  out = out.reshape(b, n, heads * key_size)
  return out @ w_out if b_out is None else torch.addmm(b_out, out.view(b * n, -1), w_out).view(b, n, -1)
