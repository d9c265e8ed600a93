"""GPU: full-size parity at the real WeatherNext 2 attention shape (level-6 mesh in Hilbert order, 32-hop mask,
127,019,682 allowed pairs = 3,101 keys per query, batch 1, 6 heads x 128), the shape of the reference's
published attention numbers (scripts/attn_bench.py:26-33; docs/results/attn_bwd/attn_bwd_default_rtx5090.txt).

The mask and lists are built on the device (k-hop bitsets -> CSR -> tile lists), as the benchmark builds them;
the test copies the CSR back and checks sampled rows of it against a host breadth-first search. The public
autograd API runs the forward and backward at full size; a float64 oracle (oracle.attention.sampled_attention)
evaluates out, lse and dQ on 1,024 query rows (8 blocks of 128 spread over the mesh) and dK, dV on 512 key rows
(two pairs of adjacent 128-key blocks), with every query of a sampled key in its sums. Bound: rel RMS <= 5e-3
(the north star's bf16 / TF32 bound) for out, dQ, dK, dV; lse within 2e-2 absolute. bf16 runs the wide-chunk
kernels on the 32-key tile lists, TF32 the narrow kernels on the same lists.
"""
import numpy as np
import pytest
import torch
from scipy import sparse
from scipy.sparse import csgraph

from oracle import attention as oa

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def wn2(cuda):
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  adj, _, _ = mesh.wn2_adjacency("hilbert")
  n = adj.shape[0]
  indptr, indices = ta.khop_csr_device(adj, mesh.WN2["hops"], cuda)
  fwd = ta.pair_tiles(ta.build_tiles_device(indptr, indices, n, n))
  tiles = ta.AttentionTiles(fwd, fwd, n, True)
  host = sparse.csr_matrix((np.ones(indices.numel(), bool), indices.cpu().numpy(), indptr.cpu().numpy()),
                           shape=(n, n))
  del indptr, indices
  return adj, tiles, host


def _blocks(starts, n):
  return np.concatenate([np.arange(b * 128, min(b * 128 + 128, n)) for b in starts])


def test_wn2_mask_rows_match_host_bfs(wn2):
  """The device 32-hop CSR at 16 sampled rows equals a host breadth-first search of the mesh to depth 32."""
  from faster_weathernext import mesh
  adj, tiles, host = wn2
  n = adj.shape[0]
  assert host.nnz == 127_019_682
  assert tiles.dense and tiles.fwd.n_blocks == (n + 127) // 128
  rows = np.linspace(0, n - 1, 16).astype(np.int64)
  dist = csgraph.dijkstra(adj.astype(np.float64), directed=False, indices=rows, unweighted=True,
                          limit=mesh.WN2["hops"] + 0.5)
  for i, r in enumerate(rows):
    want = np.flatnonzero(np.isfinite(dist[i]))
    assert np.array_equal(host.indices[host.indptr[r]:host.indptr[r + 1]], want), r


@pytest.mark.parametrize("mode", ["bf16", "tf32"])
def test_wn2_forward_backward_sampled_parity(cuda, wn2, mode):
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  adj, tiles, host = wn2
  n = adj.shape[0]
  h, d = mesh.WN2["heads"], mesh.WN2["head_dim"]
  scale = d ** -0.5
  rng = np.random.default_rng(42)
  arrays = [rng.standard_normal((1, n, h, d)).astype(np.float32) for _ in range(4)]
  if mode == "bf16":
    arrays = [oa.bf16_round(a) for a in arrays]
  dt = torch.bfloat16 if mode == "bf16" else torch.float32
  q, k, v, do = (torch.from_numpy(a).to(cuda, dt) for a in arrays)
  qq, kk, vv = (x.clone().requires_grad_(True) for x in (q, k, v))
  o = ta.attention(qq, kk, vv, tiles, scale=scale)
  o.backward(do)
  _, lse = ta.attention_forward(q, k, v, tiles, scale, ta._mode_for(dt, None, False))
  torch.cuda.synchronize()
  from faster_weathernext import _lib
  assert _lib.device_error() == 0
  nb = (n + 127) // 128
  q_rows = _blocks(np.linspace(0, nb - 1, 8).astype(int), n)
  k_rows = _blocks([nb // 5, nb // 5 + 1, (3 * nb) // 5, (3 * nb) // 5 + 1], n)
  ref = oa.sampled_attention(*(a[0] for a in arrays), host, scale, q_rows, k_rows)
  qi, ki = torch.from_numpy(q_rows).to(cuda), torch.from_numpy(k_rows).to(cuda)
  got = {"out": o.detach()[0, qi], "dq": qq.grad[0, qi], "dk": kk.grad[0, ki], "dv": vv.grad[0, ki]}
  errs = {name: oa.rel_rms(t.float().cpu().numpy(), ref[name]) for name, t in got.items()}
  assert all(e <= 5e-3 for e in errs.values()), errs
  lse_got = lse[0][:, qi].cpu().numpy()
  assert np.abs(lse_got - ref["lse"]).max() < 2e-2
