"""Options and the attention call of the patched processor (src/faster_weathernext/patch.py:50-99, 165-177).

`Options` keeps the reference's fields (read when a model is built / traced). Of them, this package acts on
`attention` (only "auto" / "tiled" select an implementation: the B200 kernel; "pallas" and "xla" name the
reference's backends, which are not part of this build), `reorder` (Hilbert order of the mesh nodes) and
`strict_fp32` (fp32-level accuracy: 3xTF32); the memory-blocking options of the GNN / encoder / decoder
(grid_chunk, edge_chunk, ...) belong to parts of the reference outside the attention path and are kept only
so that option dictionaries written for the reference are accepted.

install() / uninstall() mark the patch active. The official `weathernext` (JAX/Haiku) package is not part of
this build; a JAX model reaches the kernels through the jax.ffi custom calls described in INTEGRATION.md.
"""

import dataclasses

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


def tiled_mha(x, w_q, w_k, w_v, w_out, tiles: "tiled_attn.AttentionTiles", heads: int, key_size: int):
  """patch.tiled_mha (patch.py:165-177) for torch: q/k/v projections, block-sparse attention with
  scale key_size ** -0.5, output projection. x [B, n, d]; w_q/w_k/w_v [d, heads * key_size]."""
  b, n, _ = x.shape
  q, k, v = ((x @ w).view(b, n, heads, key_size) for w in (w_q, w_k, w_v))
  precision = "highest" if OPTIONS.strict_fp32 else None
  out = tiled_attn.attention(q, k, v, tiles, scale=key_size ** -0.5, precision=precision)
  return out.reshape(b, n, heads * key_size) @ w_out
