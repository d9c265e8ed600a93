#!/usr/bin/env python
"""Benchmark of the block-sparse masked flash attention (forward + custom-VJP backward) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--mode bf16|tf32]

Metric: block-sparse attention useful TFLOP/s, forward + backward. Workload:
configuration 3 — icosahedral mesh refined 6 times (40,962 nodes) in Morton order, great-circle mask
<= 0.06 rad, batch 1 x 8 heads x head_dim 64 per GPU (one ensemble member per GPU: weak scaling,
no inter-GPU communication). Useful FLOPs per step = 14 * B * H * nnz * D (forward 4, backward 10).

One step = fwn_attn_fwd (with LSE) + fwn_attn_bwd (delta, dQ, dK/dV) over inputs already in HBM; three
rotating input sets of 168 MB each keep every step's inputs out of the 126 MB L2. Under torchrun
(N > 1) every rank runs its own member; the step time is the max over ranks.

--impl reference times the reference's CPU path for this op — its XLA chunked attention
(patch.py:106-162) with its autodiff backward, as the NumPy restatement in oracle/ (JAX is not
installed) — on the host cores, each step a bounded sample of query chunks of the same workload.
"""

import argparse
import datetime
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "faster-weathernext_b200"), ROOT]

import numpy as np  # noqa: E402

METRIC = "block-sparse attn useful TFLOP/s fwd+bwd"
UNIT = "TFLOP/s"
CFG = 3
# Kernel FLOP counts per allowed (query, key) pair per head and head_dim element: forward S and P V (4);
# dQ kernel S, dP, dQ (6); dK/dV kernel S, dP, dV, dK (8). Useful FLOPs count S and dP once: 4 + 10.
USEFUL_PER_PAIR = 14
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch from one ncu capture of each workload on the
# current kernels (summaries under profiles/): configuration 3 bf16 and the WN2 shape bf16.
NCU_TRAFFIC = {("attention", "bf16", "gathered"): {"attn_fwd": 151_399_936, "attn_bwd_dq": 198_163_712,
                                                   "attn_bwd_dkv": 228_230_400},
               ("wn2", "bf16", "paired"): {"attn_fwd": 372_274_688, "attn_bwd_dq": 469_790_720,
                                           "attn_bwd_dkv": 537_186_560}}


def peaks():
  path = os.path.join(ROOT, "MEASURED_PEAKS.json")
  if os.path.exists(path):
    with open(path) as f:
      p = json.load(f)
    return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
  return 6650.0, 1590.0, "fallback"


class ClockSampler:
  """nvidia-smi clocks and throttle reasons sampled every 100 ms while running."""

  FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
            "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
            "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

  def __init__(self, gpu_index):
    self.gpu = gpu_index
    self.proc = None
    self.lines = []
    self.t0 = self.t1 = None

  def start(self):
    try:
      self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                    "-lms", "100", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                   stderr=subprocess.DEVNULL, text=True)
      threading.Thread(target=self._read, daemon=True).start()
    except OSError:
      self.proc = None

  def _read(self):
    for line in self.proc.stdout:
      self.lines.append((time.time(), line.strip()))

  def mark(self, which):
    setattr(self, which, time.time())

  def stop(self):
    if self.proc is not None:
      time.sleep(0.25)
      self.proc.terminate()
      try:
        self.proc.wait(timeout=5)
      except subprocess.TimeoutExpired:
        self.proc.kill()

  def summary(self):
    rows = []
    for t, line in self.lines:
      parts = [x.strip() for x in line.split(",")]
      if len(parts) < 9:
        continue
      try:
        rows.append((t, float(parts[1]), float(parts[2]), parts[4:9]))
      except ValueError:
        continue
    if not rows:
      return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"], "samples": 0}
    inside = [r for r in rows if self.t0 and self.t1 and self.t0 - 0.15 <= r[0] <= self.t1 + 0.15] or rows
    names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    reasons = sorted({names[i] for r in inside for i in range(1, 5) if r[3][i].strip() == "Active"})
    return {"sm_mhz": float(np.median([r[1] for r in inside])), "sm_max_mhz": max(r[2] for r in inside),
            "reasons": reasons, "samples": len(inside)}


class MaskInfo:
  """n, nnz and (on demand) the host CSR of a workload's mask."""

  def __init__(self, n, nnz, host=None, device_csr=None):
    self.n, self.nnz, self._host, self._dev = n, nnz, host, device_csr

  def host(self):
    if self._host is None:
      from scipy import sparse
      ip, ix = (x.cpu().numpy() for x in self._dev)
      self._host = sparse.csr_matrix((np.ones(ix.size, bool), ix, ip), shape=(self.n, self.n))
    return self._host


def workload(device, seed, mode, name="attention"):
  """(mask info, device tile lists, 3 input sets of [1, n, H, D] q/k/v/dO, heads, head_dim)."""
  import torch
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  if name == "wn2":
    # The real WeatherNext 2 shape: level-6 mesh in Hilbert order, 32-hop mask built on the device.
    adj, _, _ = mesh.wn2_adjacency("hilbert")
    n = adj.shape[0]
    indptr, indices = ta.khop_csr_device(adj, mesh.WN2["hops"], device)
    fwd = ta.pair_tiles(ta.build_tiles_device(indptr, indices, n, n))
    tiles = ta.AttentionTiles(fwd, fwd, n, True)
    info = MaskInfo(n, int(indices.numel()), device_csr=(indptr, indices))
    heads, head_dim = mesh.WN2["heads"], mesh.WN2["head_dim"]
  else:
    mask, _, _ = mesh.config_mask(CFG)
    _, _, _, heads, head_dim = mesh.CONFIGS[CFG]
    n = mask.shape[0]
    tiles = ta.AttentionTiles.from_mask(mask, device=device)
    info = MaskInfo(n, mask.nnz, host=mask)
  dt = torch.bfloat16 if mode == "bf16" else torch.float32
  g = torch.Generator(device=device).manual_seed(seed)
  sets = [[torch.randn(1, n, heads, head_dim, device=device, dtype=dt, generator=g) for _ in range(4)]
          for _ in range(3)]
  return info, tiles, sets, heads, head_dim


def kernel_costs(nnz, n, heads, head_dim, es, lf, lb):
  """Algorithmic FLOPs and DRAM bytes per launch (one batch element); lf / lb the lists walked."""
  t = heads * n * head_dim * es                 # one [1, n, H, D] tensor
  vec = heads * ((n + 127) // 128 * 128) * 4     # one lse / delta vector set
  size = lambda l: 4 * (l.n_blocks + 1) + (128 if l.cols is not None else 4) * l.n_tiles + 512 * l.n_tiles
  fwd_list, bwd_list = size(lf), size(lb)
  pair = heads * nnz * head_dim
  return {
      "attn_fwd": (4 * pair, 3 * t + t + vec + fwd_list),
      "attn_bwd_delta": (2 * heads * n * head_dim, 2 * t + vec),
      "attn_bwd_dq": (6 * pair, 4 * t + 2 * vec + t + fwd_list),
      "attn_bwd_dkv": (8 * pair, 4 * t + 2 * vec + 2 * t + bwd_list),
  }


class Ranks:
  """One process per GPU (torchrun env) or a single process: device, barrier and max over ranks."""

  def __init__(self, timeout_s=120):
    import torch
    import torch.distributed as dist
    self.world = int(os.environ.get("WORLD_SIZE", "1"))
    self.rank = int(os.environ.get("RANK", "0"))
    self.local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(self.local)
    self.device = torch.device("cuda", self.local)
    if self.world > 1:
      dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s), device_id=self.device)

  def barrier(self):
    import torch
    import torch.distributed as dist
    torch.cuda.synchronize()
    if self.world > 1:
      dist.barrier()

  def max(self, x):
    import torch
    import torch.distributed as dist
    if self.world == 1:
      return x
    t = torch.tensor([x], dtype=torch.float64, device=self.device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())

  def close(self):
    import torch.distributed as dist
    if self.world > 1:
      dist.barrier()
      dist.destroy_process_group()


def _sample_rows(n, q_blocks, k_blocks):
  """Query rows (q_blocks blocks of 128 spread over the nodes) and key rows (k_blocks adjacent blocks)."""
  nb = (n + 127) // 128
  rows = lambda starts: np.concatenate([np.arange(b * 128, min(b * 128 + 128, n)) for b in starts])
  qb = np.linspace(0, nb - 1, q_blocks).astype(int)
  kb = nb // 3 + np.arange(k_blocks)
  return rows(qb), rows(np.minimum(kb, nb - 1))


def sampled_parity(mask_host, arrays, outs, scale, q_blocks, k_blocks):
  """rel RMS of o, dq, dk, dv (and max |lse error|) at sampled rows against the float64 oracle."""
  from oracle import attention as oa
  _all_host_threads()
  n = mask_host.shape[0]
  q_rows, k_rows = _sample_rows(n, q_blocks, k_blocks)
  t0 = time.perf_counter()
  ref = oa.sampled_attention(*(a[0] for a in arrays), mask_host, scale, q_rows, k_rows)
  got = {"out": outs["o"][0][q_rows], "dq": outs["dq"][0][q_rows], "dk": outs["dk"][0][k_rows],
         "dv": outs["dv"][0][k_rows]}
  res = {name: float(f"{oa.rel_rms(got[name], ref[name]):.3e}") for name in got}
  res["lse_max_abs"] = float(f"{np.abs(outs['lse'][0][:, q_rows] - ref['lse']).max():.3e}")
  res["sample"] = f"{len(q_rows)} query rows, {len(k_rows)} key rows; float64 oracle {time.perf_counter() - t0:.1f} s"
  return res


def attention_block(args, ranks, workload_name, mode_name, steps, warmup, e2e=False, parity=False, clocks=None):
  """Time `steps` steps (fwd + delta + dQ + dK/dV) of one workload / mode on resident inputs; per-kernel times,
  roofline of the dominant kernel, issued-tile rate; optionally e2e through the public API and sampled parity."""
  import ctypes
  import torch
  from faster_weathernext import _lib
  from faster_weathernext import tiled_attn as ta

  device = ranks.device
  mode = {"bf16": _lib.MODE_BF16, "tf32": _lib.MODE_TF32, "tf32x3": _lib.MODE_TF32X3}[mode_name]
  mask, tiles, sets, heads, head_dim = workload(device, 1000 + ranks.rank, mode_name, workload_name)
  n, nnz = mask.n, mask.nnz
  scale = head_dim ** -0.5
  es = 2 if mode_name == "bf16" else 4
  useful = USEFUL_PER_PAIR * heads * nnz * head_dim
  stream = torch.cuda.current_stream()
  lib = _lib.lib()

  q0 = sets[0][0]
  o_like = torch.empty_like(q0)
  desc = ta._desc(q0, o_like, scale, mode)
  lse_rows = lib.fwn_lse_rows(n)
  outs = [dict(o=torch.empty_like(q0), lse=torch.empty(1, heads, lse_rows, device=device),
               dq=torch.empty_like(q0), dk=torch.empty_like(q0), dv=torch.empty_like(q0)) for _ in sets]
  ws_bytes = heads * lse_rows * 4
  ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
  if args.lists == "auto":
    lf, lb = ta._lists(tiles, q0, o_like)   # what the public API walks for this mask and layout
  else:
    lf, lb = (tiles.fwd_g, tiles.bwd_g) if args.lists == "gathered" else (tiles.fwd, tiles.bwd)
  lists_used = "gathered" if lf.cols is not None else "paired"
  sf, sb = lf.struct(), lb.struct()
  dref = ctypes.byref(desc)

  side = torch.cuda.Stream(device)

  def launch(i, events=None):
    """One step: forward, delta, then (timed loop) the dQ pass on a side stream concurrent with the dK/dV pass on
    the main stream, as tiled_attn.attention_backward runs them; with `events`, the four launches one after
    another, each between events on the main stream."""
    q, k, v, do = sets[i % 3]
    ob = outs[i % 3]
    s = stream.cuda_stream
    s_dq = s if events is not None else side.cuda_stream
    calls = (
        ("attn_fwd", lambda: lib.fwn_attn_fwd(dref, q.data_ptr(), k.data_ptr(), v.data_ptr(), ctypes.byref(sf),
                                              ob["o"].data_ptr(), ob["lse"].data_ptr(), s)),
        ("attn_bwd_delta", lambda: lib.fwn_attn_bwd_delta(dref, ob["o"].data_ptr(), do.data_ptr(), ws.data_ptr(),
                                                          ws_bytes, s)),
        ("attn_bwd_dq", lambda: lib.fwn_attn_bwd_dq(dref, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                    ob["lse"].data_ptr(), do.data_ptr(), ctypes.byref(sf),
                                                    ob["dq"].data_ptr(), ws.data_ptr(), ws_bytes, s_dq)),
        ("attn_bwd_dkv", lambda: lib.fwn_attn_bwd_dkv(dref, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                      ob["lse"].data_ptr(), do.data_ptr(), ctypes.byref(sb),
                                                      ob["dk"].data_ptr(), ob["dv"].data_ptr(), ws.data_ptr(),
                                                      ws_bytes, s)),
    )
    for name, fn in calls:
      if events is not None:
        e0 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
      elif name == "attn_bwd_dq":
        side.wait_stream(stream)
      _lib.check(fn())
      if events is not None:
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record(stream)
        events.setdefault(name, []).append((e0, e1))
    if events is None:
      stream.wait_stream(side)
    return len(calls)

  for i in range(warmup):
    launch(i)
  ranks.barrier()
  if _lib.device_error(stream.cuda_stream):
    raise RuntimeError("device timeout during warm-up")
  start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  if clocks is not None:
    clocks.mark("t0")
  start.record(stream)
  launches = 0
  for i in range(steps):
    launches += launch(i)
  end.record(stream)
  ranks.barrier()
  if clocks is not None:
    clocks.mark("t1")
  ms = ranks.max(start.elapsed_time(end)) / steps
  if _lib.device_error(stream.cuda_stream):
    raise RuntimeError("device timeout in the timed steps")
  value = ranks.world * useful / (ms * 1e-3) / 1e12

  # Per-kernel durations (events on the launching stream around each C-ABI call), outside the timed region.
  events = {}
  ranks.barrier()
  for i in range(min(steps, 200)):
    launch(i, events)
  ranks.barrier()
  kernel_ms = {k: float(np.mean([a.elapsed_time(b) for a, b in v])) for k, v in events.items()}
  costs = kernel_costs(nnz, n, heads, head_dim, es, lf, lb)
  hbm, tc, peak_kind = peaks()
  kernels = {}
  for k, ms_k in kernel_ms.items():
    flops, nbytes = costs[k]
    kernels[k] = {"ms": round(ms_k, 5), "useful_tflops": round(flops / (ms_k * 1e-3) / 1e12, 2),
                  "algorithmic_gbs": round(nbytes / (ms_k * 1e-3) / 1e9, 1),
                  "bound": "tensor" if flops / (tc * 1e12) > nbytes / (hbm * 1e9) else "hbm"}
  dom = max(kernel_ms, key=kernel_ms.get)
  traffic = NCU_TRAFFIC.get((workload_name, mode_name, lists_used), {})
  flops, nbytes = costs[dom]
  bound = kernels[dom]["bound"]
  if bound == "hbm":
    achieved = nbytes / (kernel_ms[dom] * 1e-3) / 1e9
    roof = {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(achieved / hbm, 4), "peak_source": peak_kind,
            "algorithmic_bytes": nbytes, "traffic": traffic.get(dom)}
  else:
    achieved = flops / (kernel_ms[dom] * 1e-3) / 1e12
    roof = {"bound": "tensor", "kernel": dom, "achieved": round(achieved, 2), "peak": tc, "unit": "TFLOP/s",
            "frac": round(achieved / tc, 4), "peak_source": peak_kind,
            "algorithmic_flops": flops, "traffic": traffic.get(dom)}
  if mode_name != "bf16":
    # The mode's own peak as well: dense TF32 runs at half the bf16 rate on B200 (1.1 vs 2.25 PFLOP/s nominal);
    # only the bf16 rate is measured, so the TF32 peak is taken as half of it. 3xTF32 counts useful FLOPs
    # once against the same TF32 peak.
    mode_tflops = flops / (kernel_ms[dom] * 1e-3) / 1e12
    roof["mode_peak"] = round(tc / 2, 1)
    roof["mode_frac"] = round(mode_tflops / (tc / 2), 4)
    roof["mode_peak_source"] = "half the " + peak_kind + " bf16 rate"
  # Tensor-core work actually issued on 128 x 32 tiles: forward 2 MMAs, dQ 3, dK/dV 4 per tile in one pass, 5
  # where dK/dV runs as a dV-only (S, dV) and a dK-only (S, dP, dK) pass (3xTF32, and TF32 at head_dim 128).
  # 3xTF32 issues three products per MMA.
  split = mode_name == "tf32x3" or (mode_name == "tf32" and head_dim == 128)
  issued = (2 * heads * head_dim * 128 * 32 * (5 * lf.n_tiles + (5 if split else 4) * lb.n_tiles) *
            (3 if mode_name == "tf32x3" else 1))

  block = {"workload": workload_name, "mode": mode_name, "nodes": n, "pairs": nnz, "heads": heads,
           "head_dim": head_dim, "tile_lists": lists_used, "steps": steps, "warmup": warmup,
           "ms_per_step": round(ms, 5), "value": round(value, 3), "unit": UNIT, "kernels": kernels,
           "roofline": roof, "issued_tile_tflops": round(issued / (ms * 1e-3) / 1e12, 2), "gpu_launches": launches,
           "l2": f"inputs larger than L2: 3 rotating input sets of "
                 f"{4 * q0.numel() * q0.element_size() / 1e6:.0f} MB"}

  if parity and ranks.rank == 0:
    torch.cuda.synchronize()
    arrays = [x.float().cpu().numpy() for x in sets[0]]
    host_outs = {k: v.float().cpu().numpy() for k, v in outs[0].items()}
    qb, kb = (4, 2) if workload_name == "wn2" else (8, 8)
    block["parity"] = sampled_parity(mask.host(), arrays, host_outs, scale, qb, kb)
    bound_ = 5e-3 if mode_name in ("bf16", "tf32") else 2e-5
    block["parity"]["bound_rel_rms"] = bound_
    block["parity"]["ok"] = all(block["parity"][k] <= bound_ for k in ("out", "dq", "dk", "dv"))

  if e2e:
    # End to end through the public API: every step copies its q, k, v, dO from pinned host memory, runs
    # tiled_attn.attention + torch.autograd.grad, and copies o, dq, dk, dv back to pinned host memory. As in a
    # training loop, the copies run on their own streams (two buffer slots), so that step i's upload, step
    # i-1's compute and step i-2's download overlap; all of them lie inside the timed region.
    dt = torch.bfloat16 if mode_name == "bf16" else torch.float32
    host_in = [[x.cpu().pin_memory() for x in s_] for s_ in sets[:2]]
    host_out = [[torch.empty(q0.shape, dtype=dt).pin_memory() for _ in range(4)] for _ in range(2)]
    dev_in = [[torch.empty_like(x) for x in sets[0]] for _ in range(2)]
    s_h2d, s_d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_cmp = [torch.cuda.Event() for _ in range(2)]
    e2e_steps = min(steps, 50)
    precision = "highest" if mode_name == "tf32x3" else None

    def e2e_step(i):
      sl = i % 2
      if i >= 2:
        s_h2d.wait_event(ev_cmp[sl])  # step i-2 has finished reading this slot
      with torch.cuda.stream(s_h2d):
        for d, h in zip(dev_in[sl], host_in[i % 2]):
          d.copy_(h, non_blocking=True)
      ev_in[sl].record(s_h2d)
      stream.wait_event(ev_in[sl])
      q, k, v = (x.detach().requires_grad_(True) for x in dev_in[sl][:3])
      o = ta.attention(q, k, v, tiles, scale=scale, precision=precision)
      dq, dk, dv = torch.autograd.grad(o, (q, k, v), dev_in[sl][3])
      ev_cmp[sl].record(stream)
      s_d2h.wait_event(ev_cmp[sl])
      with torch.cuda.stream(s_d2h):
        for dst, src in zip(host_out[sl], (o, dq, dk, dv)):
          dst.copy_(src.detach(), non_blocking=True)
          src.record_stream(s_d2h)

    for i in range(3):
      e2e_step(i)
    ranks.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    s_h2d.wait_event(a)
    for i in range(e2e_steps):
      e2e_step(i)
    stream.wait_stream(s_d2h)
    b.record(stream)
    ranks.barrier()
    e2e_ms = ranks.max(a.elapsed_time(b)) / e2e_steps
    tb = q0.numel() * q0.element_size()
    block["e2e"] = {"value": round(ranks.world * useful / (e2e_ms * 1e-3) / 1e12, 3), "unit": UNIT,
                    "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": 4 * tb, "d2h_bytes_per_step": 4 * tb,
                    "overlap": "H2D, compute and D2H on three streams, two buffer slots"}
  block["_mask"] = mask
  del sets, outs, ws
  return block


def finetune_block(args, ranks, steps, warmup):
  """Configuration 5 (fine-tune step: 8 members split over the ranks, forward + backward through the custom-VJP
  attention, gradient all-reduce, Adam) with the all-reduce overlapped with the backward (bucketed, issued from
  gradient hooks) and without it (one all-reduce after the backward); plus the gradient all-reduce alone."""
  import torch
  import torch.distributed as dist
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  from faster_weathernext.finetune import DataParallelStep, RankWatchdog
  from faster_weathernext.processor import Processor, ProcessorConfig

  device = ranks.device
  mask, _, _ = mesh.config_mask(CFG)
  n = mask.shape[0]
  tiles = ta.AttentionTiles.from_mask(mask, device=device)
  cfg = ProcessorConfig()
  members = 8
  local_m = members // ranks.world
  g = torch.Generator(device=device).manual_seed(100 + ranks.rank)
  xs = [torch.randn(1, n, cfg.d_model, device=device, generator=g) for _ in range(local_m)]
  cs = [torch.randn(1, cfg.cond_dim, device=device, generator=g) for _ in range(local_m)]
  ts = [torch.randn(1, n, cfg.d_model, device=device, generator=g) for _ in range(local_m)]
  dog = None
  if ranks.world > 1:
    from torch.distributed import distributed_c10d as c10d
    dog = RankWatchdog(c10d._get_default_store(), ranks.rank, ranks.world, timeout=60.0).start()
  out = {"workload": "cfg5: 8 members, MSE, fwd + bwd + gradient all-reduce + Adam, level-6 mesh 0.06 rad",
         "members_per_gpu": local_m, "micro_batch": args.micro_batch, "steps": steps, "warmup": warmup}
  stream = torch.cuda.current_stream()
  for overlap in (True, False):
    model = Processor(cfg, seed=0, device=device)
    trainer = DataParallelStep(model, members, lr=1e-5, overlap=overlap, watchdog=dog)

    def step():
      return trainer.step(xs, cs, ts, forward=lambda x, c: model(x, c, tiles), micro_batch=args.micro_batch)
    for _ in range(warmup):
      step()
    ranks.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
      loss = step()
    b.record(stream)
    ranks.barrier()
    ms = ranks.max(a.elapsed_time(b)) / steps
    key = "overlapped" if overlap else "not_overlapped"
    out[key] = {"ms_per_step": round(ms, 3), "buckets": len(trainer.buckets) if overlap else 1,
                "loss": round(float(loss), 6)}
    out["grad_bytes"] = trainer.numel * 4
    del model, trainer
    torch.cuda.empty_cache()
  out["peak_memory_gb"] = round(torch.cuda.max_memory_allocated(device) / 1e9, 1)
  if ranks.world > 1:
    # The gradient all-reduce alone: one float32 buffer of the model's gradient size, NCCL over NVLink.
    buf = torch.ones(out["grad_bytes"] // 4, dtype=torch.float32, device=device)
    for _ in range(3):
      dist.all_reduce(buf)
    ranks.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    a.record(stream)
    for _ in range(reps):
      dist.all_reduce(buf)
    b.record(stream)
    ranks.barrier()
    ar_ms = ranks.max(a.elapsed_time(b)) / reps
    busbw = out["grad_bytes"] * 2 * (ranks.world - 1) / ranks.world / (ar_ms * 1e-3) / 1e9
    out["allreduce"] = {"ms": round(ar_ms, 3), "bytes": out["grad_bytes"], "busbw_gbs": round(busbw, 1),
                        "reference_busbw_gbs": 725.0,
                        "note": "NCCL all-reduce of the float32 gradient buffer; busbw = 2 (N-1) / N x bytes / time"}
    del buf
    dog.stop()
  else:
    out["allreduce"] = None
  return out


def processor_block(args, ranks, steps, warmup):
  """Configuration 4 (processor inference: 8 members x 2 noise samples = 16 forwards of the 24-block processor, split
  over the ranks, no communication): ms per step, max over ranks."""
  import torch
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  from faster_weathernext.processor import Processor, ProcessorConfig

  device = ranks.device
  mask, _, _ = mesh.config_mask(CFG)
  n = mask.shape[0]
  tiles = ta.AttentionTiles.from_mask(mask, device=device)
  cfg = ProcessorConfig()
  model = Processor(cfg, seed=0, device=device)
  forwards = 16
  local_f = forwards // ranks.world
  g = torch.Generator(device=device).manual_seed(200 + ranks.rank)
  x = torch.randn(local_f, n, cfg.d_model, device=device, generator=g)
  c = torch.randn(local_f, cfg.cond_dim, device=device, generator=g)
  stream = torch.cuda.current_stream()

  def step():
    with torch.no_grad():
      return model(x, c, tiles)
  for _ in range(warmup):
    step()
  ranks.barrier()
  a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  a.record(stream)
  for _ in range(steps):
    y = step()
  b.record(stream)
  ranks.barrier()
  ms = ranks.max(a.elapsed_time(b)) / steps
  gemm = model.gemm_flops_per_forward(n) * local_f
  hbm, tc, peak_kind = peaks()
  out = {"workload": "cfg4: 24 pre-LN blocks d512 8x64 MLP2048 GELU, 16 forwards (8 members x 2 samples) split over "
                     "the ranks, no communication, level-6 mesh 0.06 rad",
         "forwards_per_gpu": local_f, "steps": steps, "warmup": warmup, "ms_per_step": round(ms, 3),
         "forwards_per_s": round(forwards / (ms * 1e-3), 2),
         "gemm_tflops_per_gpu": round(gemm / (ms * 1e-3) / 1e12, 1), "gemm_frac_of_peak": round(gemm / (ms * 1e-3) / 1e12 / tc, 4),
         "output_finite": bool(torch.isfinite(y).all())}
  del model, x, c, y
  torch.cuda.empty_cache()
  return out


def gnn_block(args, ranks, steps, warmup):
  """The decoder's grid <-> mesh interaction network at the WeatherNext 2 shape (patch.py:347-509): 40,962 mesh
  nodes send to the 1,038,240 points of the 0.25-degree grid, each point receiving from its 3 nearest mesh nodes
  (3,114,720 edges sorted by receiver), latent and hidden width 512; edges in one pass and in the reference's blocks of
  Options.edge_chunk. ms per step and matmul TFLOP/s."""
  import torch
  from scipy.spatial import cKDTree
  from faster_weathernext import mesh, patch
  from faster_weathernext.gnn import GNNConfig, InteractionNetwork

  device = ranks.device
  xyz, _ = mesh.icosphere(6)
  lat = np.deg2rad(np.linspace(-90.0, 90.0, 721))
  lon = np.deg2rad(np.arange(1440) * 0.25)
  la, lo = np.meshgrid(lat, lon, indexing="ij")
  pts = np.stack([np.cos(la) * np.cos(lo), np.cos(la) * np.sin(lo), np.sin(la)], -1).reshape(-1, 3)
  t0 = time.perf_counter()
  _, nn = cKDTree(xyz).query(pts, k=3)
  build_s = time.perf_counter() - t0
  ns, nr = xyz.shape[0], pts.shape[0]
  senders = torch.from_numpy(nn.reshape(-1).astype(np.int32))
  receivers = torch.from_numpy(np.repeat(np.arange(nr, dtype=np.int32), 3))
  cfg = GNNConfig(latent=512, hidden=512)
  net = InteractionNetwork(cfg, seed=0, device=device)
  g = torch.Generator(device=device).manual_seed(300 + ranks.rank)
  sx = torch.randn(ns, cfg.latent, device=device, generator=g)
  rx = torch.randn(nr, cfg.latent, device=device, generator=g)
  ex = torch.randn(senders.numel(), cfg.latent, device=device, generator=g)
  stream = torch.cuda.current_stream()
  out = {"workload": "decoder interaction network: 40,962 mesh nodes -> 1,038,240 grid points (0.25 deg), 3 nearest "
                     "mesh nodes per point, 3,114,720 edges sorted by receiver, latent / hidden 512",
         "graph_build_s": round(build_s, 2), "steps": steps, "warmup": warmup,
         "matmul_gflop": round(net.flops(ns, nr, senders.numel()) / 1e9, 1)}
  for name, chunk in (("one_pass", 0), ("edge_chunk_default", patch.Options().edge_chunk)):
    def step():
      return net(sx, rx, ex, senders, receivers, edge_chunk=chunk)
    for _ in range(warmup):
      step()
    ranks.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
      ys, yr = step()
    b.record(stream)
    ranks.barrier()
    ms = ranks.max(a.elapsed_time(b)) / steps
    out[name] = {"edge_chunk": chunk, "ms_per_step": round(ms, 3),
                 "matmul_tflops": round(net.flops(ns, nr, senders.numel()) / (ms * 1e-3) / 1e12, 1),
                 "output_finite": bool(torch.isfinite(yr).all() and torch.isfinite(ys).all())}
  del net, sx, rx, ex
  torch.cuda.empty_cache()
  return out


def run_ours(args):
  import torch

  ranks = Ranks()
  clocks = ClockSampler(ranks.local)
  clocks.start()
  head = attention_block(args, ranks, args.workload, args.mode, args.steps, args.warmup, e2e=not args.no_e2e,
                         parity=False, clocks=clocks)
  clocks.stop()
  mask = head.pop("_mask")
  cpu = None
  if ranks.rank == 0 and ranks.world == 1 and not args.no_cpu:
    cpu = cpu_baseline(mask.host(), head["heads"], head["head_dim"], seconds=args.cpu_seconds, name=args.workload)
  del mask
  torch.cuda.empty_cache()

  # Other modes and shapes in the same run (default run at N = 1 only: at N > 1 they would be the same replicas):
  # config 3 in the reference's own precision (TF32) and its `highest` (3xTF32), and the real WN2 shape in bf16;
  # each with sampled-row parity against the oracle.
  modes = {}
  if not args.no_blocks and args.workload == "attention" and args.mode == "bf16" and ranks.world == 1:
    blk_steps, blk_warmup = min(args.steps, 20), max(3, min(args.warmup, 5))
    for wl, md in (("attention", "tf32"), ("attention", "tf32x3"), ("wn2", "bf16")):
      blk = attention_block(args, ranks, wl, md, blk_steps, blk_warmup, parity=True)
      blk.pop("_mask")
      modes[("cfg3" if wl == "attention" else wl) + "_" + md] = blk
      torch.cuda.empty_cache()
    modes["gnn_decoder"] = gnn_block(args, ranks, steps=min(args.steps, 5), warmup=3)
  finetune = processor = None
  if not args.no_finetune and args.workload == "attention" and args.mode == "bf16":
    processor = processor_block(args, ranks, steps=min(args.steps, 5), warmup=3)
    finetune = finetune_block(args, ranks, steps=min(args.steps, 5), warmup=3)

  if ranks.rank == 0:
    world, n, nnz = ranks.world, head["nodes"], head["pairs"]
    heads, head_dim = head["heads"], head["head_dim"]
    if args.workload == "wn2":
      desc_w = (f"WN2 real shape fwd+bwd: 40,962 nodes (level-6 mesh, Hilbert order), 32-hop mask ({nnz} pairs, "
                f"built on the device), B1 H{heads} D{head_dim} per GPU")
      data = "synthetic: Q/K/V/dO ~ N(0,1) seeded per rank; icosphere level-6 32-hop mask built on the GPU"
    else:
      desc_w = (f"cfg3 fwd+bwd: 40,962 nodes (Morton), mask <= 0.06 rad ({nnz} pairs), "
                f"B1 H{heads} D{head_dim} per GPU")
      data = "synthetic: Q/K/V/dO ~ N(0,1) seeded per rank; icosphere level-6 great-circle mask built on the host"
    line = {
        "metric": METRIC, "value": head["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": published_ratio(args, head["value"], nnz, heads, head_dim),
        "dtype": {"bf16": "bf16", "tf32": "tf32", "tf32x3": "3xtf32"}[args.mode], "data": data,
        "config": {"workload": desc_w, "global_batch": world, "nodes": n,
                   "heads": heads, "head_dim": head_dim, "parallelism": f"replicas x{world} (no communication)",
                   "l2": head["l2"], "tile_lists": head["tile_lists"]},
        "roofline": head["roofline"], "cpu_baseline": cpu, "e2e": head.get("e2e"), "gpu_launches": head["gpu_launches"],
        "clocks": clocks.summary(), "kernels": head["kernels"], "issued_tile_tflops": head["issued_tile_tflops"],
        "modes": modes or None, "processor": processor, "finetune": finetune,
    }
    print(json.dumps(line), flush=True)
  ranks.close()


# The reference's published fwd+bwd times at the WN2 shape (RTX 5090, one layer, 6 x 128 heads, 32-hop mask,
# 3,101 keys per query): TF32 42.2 ms, 3xTF32 115.4 ms (docs/results/attn_bwd/attn_bwd_{default,highest}_rtx5090.txt:6).
PUBLISHED_WN2_MS = {"tf32": 42.2, "tf32x3": 115.4}
PUBLISHED_WN2_NNZ = 40_962 * 3_101


def published_ratio(args, value, nnz, heads, head_dim):
  """value / the reference's published useful TFLOP/s for the same metric, shape and precision (else None)."""
  ms = PUBLISHED_WN2_MS.get(args.mode) if args.workload == "wn2" else None
  if ms is None:
    return None
  ref = USEFUL_PER_PAIR * heads * PUBLISHED_WN2_NNZ * head_dim / (ms * 1e-3) / 1e12
  return round(value / ref, 3)


def run_model_workload(args):
  """Configurations 4 (processor: 8 members x 2 noise samples = 16 forwards, split over the ranks, no
  communication) and 5 (fine-tune: 8 members split over the ranks, forward + backward through the
  custom-VJP attention, one NCCL all-reduce of the float32 gradients, Adam). Metric: ms per step (max over
  ranks); GEMM FLOPs against the bf16 tensor-core peak as the roofline."""
  import torch
  import torch.distributed as dist
  from faster_weathernext import mesh
  from faster_weathernext import tiled_attn as ta
  from faster_weathernext.finetune import DataParallelStep
  from faster_weathernext.processor import Processor, ProcessorConfig

  world = int(os.environ.get("WORLD_SIZE", "1"))
  rank = int(os.environ.get("RANK", "0"))
  local = int(os.environ.get("LOCAL_RANK", "0"))
  torch.cuda.set_device(local)
  device = torch.device("cuda", local)
  if world > 1:
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
  mask, _, _ = mesh.config_mask(CFG)
  n = mask.shape[0]
  tiles = ta.AttentionTiles.from_mask(mask, device=device)
  cfg = ProcessorConfig()
  model = Processor(cfg, seed=0, device=device)
  finetune = args.workload == "finetune"
  members = 8 if finetune else 16
  if members % world:
    raise SystemExit(f"{members} members do not split over {world} GPUs")
  local_m = members // world
  g = torch.Generator(device=device).manual_seed(100 + rank)
  if finetune:
    xs = [torch.randn(1, n, cfg.d_model, device=device, generator=g) for _ in range(local_m)]
    cs = [torch.randn(1, cfg.cond_dim, device=device, generator=g) for _ in range(local_m)]
    ts = [torch.randn(1, n, cfg.d_model, device=device, generator=g) for _ in range(local_m)]
    trainer = DataParallelStep(model, members, lr=1e-5)

    def step():
      return trainer.step(xs, cs, ts, forward=lambda x, c: model(x, c, tiles), micro_batch=args.micro_batch)
  else:
    x = torch.randn(local_m, n, cfg.d_model, device=device, generator=g)
    c = torch.randn(local_m, cfg.cond_dim, device=device, generator=g)

    def step():
      with torch.no_grad():
        return model(x, c, tiles)

  def barrier():
    torch.cuda.synchronize()
    if world > 1:
      dist.barrier()

  clocks = ClockSampler(local)
  clocks.start()
  for _ in range(args.warmup):
    step()
  barrier()
  stream = torch.cuda.current_stream()
  a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  clocks.mark("t0")
  a.record(stream)
  for _ in range(args.steps):
    step()
  b.record(stream)
  barrier()
  clocks.mark("t1")
  clocks.stop()
  ms = a.elapsed_time(b)
  if world > 1:
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
  ms /= args.steps
  gemm = model.gemm_flops_per_forward(n) * local_m * (3 if finetune else 1)
  attn = (USEFUL_PER_PAIR if finetune else 4) * cfg.heads * mask.nnz * cfg.head_dim * cfg.layers * local_m
  hbm, tc, peak_kind = peaks()
  achieved = gemm / (ms * 1e-3) / 1e12
  if world > 1:
    dist.barrier()
  if rank == 0:
    name = "fine-tune step ms (cfg5)" if finetune else "processor step ms (cfg4)"
    print(json.dumps({
        "metric": name, "value": round(ms, 3), "unit": "ms", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic: latents / targets ~ N(0,1), Glorot-uniform weights",
        "config": {"workload": ("cfg5: 8 members, MSE, fwd + bwd + NCCL all-reduce + Adam" if finetune else
                                "cfg4: 24 pre-LN blocks d512 8x64 MLP2048 GELU, 16 forwards") +
                               f", level-6 mesh 0.06 rad", "members": members, "members_per_gpu": local_m,
                   "parallelism": f"{'dp' if finetune else 'replicas'}{world}"},
        "roofline": {"bound": "tensor", "kernel": "processor GEMMs (cuBLAS and fwn_gemm_bf16, bf16) per GPU", "achieved": round(achieved, 1),
                     "peak": tc, "unit": "TFLOP/s", "frac": round(achieved / tc, 4), "peak_source": peak_kind,
                     "traffic": None},
        "attention_useful_gflop_per_gpu": round(attn / 1e9, 1), "gemm_gflop_per_gpu": round(gemm / 1e9, 1),
        "peak_memory_gb": round(torch.cuda.max_memory_allocated(device) / 1e9, 1),
        "micro_batch": args.micro_batch if finetune else None,
        "cpu_baseline": None, "e2e": None, "clocks": clocks.summary(),
        "gpu_launches": None,
    }), flush=True)
  if world > 1:
    dist.destroy_process_group()


def _all_host_threads():
  """Raise the BLAS / OpenMP pools to every host core (torchrun sets OMP_NUM_THREADS=1 for its ranks) and
  return the thread count now in use."""
  n = os.cpu_count() or 1
  try:
    from threadpoolctl import threadpool_info, threadpool_limits
    threadpool_limits(limits=n)
    return max([p.get("num_threads", 1) for p in threadpool_info()] or [n])
  except Exception:
    return n


def cpu_baseline(mask, heads, head_dim, seconds=15.0, steps=None, name="attention"):
  """The reference's CPU path (XLA chunked attention fwd + autodiff bwd, float32, NumPy/BLAS on all
  host cores) timed on a bounded sample of query chunks; returned in useful TFLOP/s."""
  from oracle import attention as oa
  cores = _all_host_threads()
  n = mask.shape[0]
  rng = np.random.default_rng(0)
  q, k, v, do = (rng.standard_normal((1, n, heads, head_dim)).astype(np.float32) for _ in range(4))
  path = oa.ChunkedPath(mask, 512, np.float32)
  t = path.layout(q, k, v, do)
  out = np.zeros_like(t["q"])
  dq, dk, dv = np.zeros_like(t["q"]), np.zeros_like(t["k"]), np.zeros_like(t["v"])
  rows_nnz = np.diff(mask.indptr)
  order = [(7 * i + 3) % path.n_chunks for i in range(path.n_chunks)]
  path.forward_chunk(t, order[0], head_dim ** -0.5, out)   # warm-up
  done, flops, t0 = 0, 0, time.perf_counter()
  while True:
    c = order[done % len(order)]
    path.forward_chunk(t, c, head_dim ** -0.5, out)
    path.vjp_chunk(t, c, head_dim ** -0.5, dq, dk, dv)
    flops += USEFUL_PER_PAIR * heads * head_dim * int(rows_nnz[c * 512:(c + 1) * 512].sum())
    done += 1
    el = time.perf_counter() - t0
    if (steps is None and el > seconds) or (steps is not None and done >= steps):
      break
  return {"value": round(flops / el / 1e12, 6), "unit": UNIT, "cores": cores, "kind": "port",
          "sample": f"{done} of {path.n_chunks} query chunks (512 queries, key window {path.window}) of "
                    f"{'the WN2 shape' if name == 'wn2' else 'cfg3'}, "
                    f"fwd + bwd, float32, {el:.1f} s"}


def run_reference(args):
  """CPU reference arm: rank 0 only, the oracle's restatement of the reference XLA path on the host."""
  rank = int(os.environ.get("RANK", "0"))
  if rank != 0:
    return
  from faster_weathernext import mesh
  from oracle import attention as oa
  cores = _all_host_threads()
  if args.workload == "wn2":
    # The WN2 shape built on the host: Hilbert order (the reference's permutation, restated in the oracle) and
    # the 32-hop neighbourhood as a sparse matrix power (patch.py:209), about a minute on the host.
    from oracle import tiles as ot
    xyz, faces = mesh.icosphere(mesh.WN2["level"])
    lat, lon = mesh.latlon(xyz)
    adj = mesh.permute(mesh.adjacency(faces, xyz.shape[0]), ot.hilbert_order(lat, lon))
    mask = mesh.k_hop_mask(adj, mesh.WN2["hops"])
    heads, head_dim = mesh.WN2["heads"], mesh.WN2["head_dim"]
    label = "the WN2 shape"
    desc_w = (f"WN2 real shape fwd+bwd: 40,962 nodes (level-6 mesh, Hilbert order), 32-hop mask ({mask.nnz} pairs), "
              f"B1 H{heads} D{head_dim}")
    data = "synthetic: Q/K/V/dO ~ N(0,1); icosphere level-6 32-hop mask built on the host"
  else:
    mask, _, _ = mesh.config_mask(CFG)
    _, _, _, heads, head_dim = mesh.CONFIGS[CFG]
    label = "cfg3"
    desc_w = f"cfg3 fwd+bwd: 40,962 nodes (Morton), mask <= 0.06 rad ({mask.nnz} pairs), B1 H{heads} D{head_dim}"
    data = "synthetic: Q/K/V/dO ~ N(0,1); icosphere level-6 great-circle mask"
  n = mask.shape[0]
  rng = np.random.default_rng(0)
  q, k, v, do = (rng.standard_normal((1, n, heads, head_dim)).astype(np.float32) for _ in range(4))
  path = oa.ChunkedPath(mask, 512, np.float32)
  t = path.layout(q, k, v, do)
  out = np.zeros_like(t["q"])
  dq, dk, dv = np.zeros_like(t["q"]), np.zeros_like(t["k"]), np.zeros_like(t["v"])
  rows_nnz = np.diff(mask.indptr)
  scale = head_dim ** -0.5

  # Each step is one query chunk, or a slice of its rows with the same key window, sized so that the
  # whole --warmup W --steps K run takes about --ref-seconds (a minute and a half by default).
  chunk_s = time.perf_counter()
  path.forward_chunk(t, 3, scale, out)
  path.vjp_chunk(t, 3, scale, dq, dk, dv)
  chunk_s = time.perf_counter() - chunk_s
  rows = int(np.clip(512 * args.ref_seconds / max(args.steps + args.warmup, 1) / chunk_s, 8, 512)) // 8 * 8

  def step(i):
    c = (7 * i + 3) % path.n_chunks
    path.forward_chunk(t, c, scale, out, 0, rows)
    path.vjp_chunk(t, c, scale, dq, dk, dv, 0, rows)
    return USEFUL_PER_PAIR * heads * head_dim * int(rows_nnz[c * 512:min(c * 512 + rows, n)].sum())

  for i in range(args.warmup):
    step(i)
  t0 = time.perf_counter()
  flops = sum(step(args.warmup + i) for i in range(args.steps))
  el = time.perf_counter() - t0
  value = flops / el / 1e12
  sample = (f"per step {rows} query rows of one of the {path.n_chunks} query chunks (key window {path.window}) "
            f"of {label}, fwd + autodiff bwd, float32 NumPy/BLAS restatement of the XLA path (JAX absent)")
  print(json.dumps({
      "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": UNIT, "n_gpus": args.gpus,
      "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
      "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
      "data": data,
      "config": {"workload": desc_w, "nodes": n, "heads": heads, "head_dim": head_dim, "parallelism": "host CPU"},
      "cpu_baseline": {"value": round(value, 6), "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
      "e2e": {"value": round(value, 6), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
  }), flush=True)


def main():
  ap = argparse.ArgumentParser()
  ap.add_argument("--gpus", type=int, default=1)
  ap.add_argument("--steps", type=int, default=2000)
  ap.add_argument("--warmup", type=int, default=20)
  ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
  ap.add_argument("--mode", choices=["bf16", "tf32", "tf32x3"], default="bf16",
                  help="bf16 MMAs, TF32 (the reference's default precision) or 3xTF32 (its `highest`)")
  ap.add_argument("--workload", choices=["attention", "wn2", "processor", "finetune"], default="attention",
                  help="attention: configuration 3 (the headline); wn2: the real WeatherNext 2 shape (32-hop mask, "
                       "6 x 128 heads); processor / finetune: configurations 4 / 5")
  ap.add_argument("--lists", choices=["auto", "gathered", "paired"], default="auto",
                  help="tile lists the kernels walk: gathered (distinct keys per block), paired 32-key tiles, or "
                       "auto (the public API's choice: gathered for sparse masks, paired for dense ones / D 128)")
  ap.add_argument("--micro-batch", type=int, default=4,
                  help="fine-tune: members per forward / backward on a rank (activations ~29 GB per member)")
  ap.add_argument("--no-e2e", action="store_true")
  ap.add_argument("--no-cpu", action="store_true")
  ap.add_argument("--no-blocks", action="store_true",
                  help="default run: skip the TF32 / 3xTF32 / WN2 blocks")
  ap.add_argument("--no-finetune", action="store_true",
                  help="default run: skip the configuration-4 (processor) and configuration-5 (fine-tune) blocks")
  ap.add_argument("--cpu-seconds", type=float, default=15.0)
  ap.add_argument("--ref-seconds", type=float, default=90.0,
                  help="--impl reference: host seconds the warm-up and timed steps take together")
  args = ap.parse_args()
  if args.warmup < 3:
    ap.error("--warmup must be >= 3")
  if args.impl == "reference":
    if args.workload not in ("attention", "wn2"):
      print(json.dumps({"impl": "reference", "unavailable": "the reference's processor runs in JAX, which is not "
                        "installed on this image"}))
      return
    run_reference(args)
  elif args.workload in ("attention", "wn2"):
    run_ours(args)
  else:
    run_model_workload(args)


if __name__ == "__main__":
  main()
