"""Interaction-network step on the CPU (test infrastructure; see oracle/__init__.py), float64.

Restates the structure of the reference's blocked grid <-> mesh GNN step (src/faster_weathernext/patch.py:347-509,
ChunkedDeepGNN._mesh_to_points / _points_to_mesh): an edge MLP over (edge, sender, receiver) features whose first
layer is applied per node before the gather, a sorted segment-sum of the messages into the receivers (optionally
normalised), a receiver node MLP on (node, aggregate) with a residual, and a sender node MLP without messages. The
MLPs' own definition lives in the third-party `weathernext` package (absent); the conventional form is used here:
one hidden layer, swish, LayerNorm (scale, offset) on the output. Parity of this structure with the official MLPs is
therefore not pinned.
"""

import numpy as np


def _swish(x):
  return x / (1.0 + np.exp(-x))


def _ln(x, g, b, eps):
  mu = x.mean(-1, keepdims=True)
  var = ((x - mu) ** 2).mean(-1, keepdims=True)
  return (x - mu) / np.sqrt(var + eps) * g + b


def interaction_network(params, senders_x, receivers_x, edges_x, senders, receivers, eps=1e-5, norm=1.0):
  """params: dict of float arrays named as faster_weathernext.gnn.InteractionNetwork's parameters. Returns
  (senders_x', receivers_x') float64."""
  p = {k: np.asarray(v, np.float64) for k, v in params.items()}
  s, r, e = (np.asarray(x, np.float64) for x in (senders_x, receivers_x, edges_x))
  snd, rcv = np.asarray(senders, np.int64), np.asarray(receivers, np.int64)
  hid = _swish(e @ p["w_e"] + (s @ p["w_s"])[snd] + (r @ p["w_r"])[rcv] + p["b1"])
  msg = _ln(hid @ p["w2"] + p["b2"], p["ln_e_g"], p["ln_e_b"], eps)
  agg = np.zeros_like(r)
  np.add.at(agg, rcv, msg)
  agg *= norm
  new_r = r + _ln(_swish(r @ p["u_r"] + agg @ p["u_a"] + p["c1"]) @ p["u2"] + p["c2"], p["ln_r_g"], p["ln_r_b"], eps)
  new_s = s + _ln(_swish(s @ p["v_s"] + p["d1"]) @ p["v2"] + p["d2"], p["ln_s_g"], p["ln_s_b"], eps)
  return new_s, new_r
