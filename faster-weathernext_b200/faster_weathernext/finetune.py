"""Data-parallel fine-tuning step on the processor (configuration 5).

One step over a batch of ensemble members split across ranks: each rank runs forward + backward (the
attention's custom-VJP kernels included) for its members, accumulating gradients; the float32 gradients are
summed across ranks with NCCL all-reduces over NVLink, and Adam updates the parameters identically on every
rank. The loss is the mean-squared error to the targets. The reference's fine-tuning library
(src/faster_weathernext/finetune.py:136-150: value_and_grad, optax update, single device) has no collective;
the all-reduce is what sharding members across GPUs adds.

Gradient buckets: every parameter's .grad is a view into one flat float32 buffer laid out in reverse parameter
order (the order the backward produces gradients: last block first), cut into buckets of about `bucket_mb`.
During the last micro-batch's backward, a bucket is all-reduced (asynchronously, on the communicator's stream)
as soon as all of its gradients are accumulated, while the backward of earlier layers continues; buckets are
issued in bucket order on every rank, so all ranks take the same collective steps. `overlap=False` runs one
all-reduce of the whole buffer after the backward instead (the baseline the overlap is measured against).

Rank failures (RankWatchdog): each rank publishes a heartbeat counter in the process group's key-value store
from a host thread; a rank that leaves marks itself in the store. Before every step the others check the
marks and heartbeats and raise RankFailure before any launch of that step, so no collective is entered with a
missing peer; a rank that dies without warning is caught by its stale heartbeat or, inside a collective, by
the process group's own timeout. abort_group() then tears the communicator down.
"""

import threading
import time

import torch
import torch.distributed as dist


class RankFailure(RuntimeError):
  """A peer rank left or stopped answering; the step was not started."""

  def __init__(self, rank, why):
    super().__init__(f"rank {rank} {why}")
    self.rank = rank


class RankWatchdog:
  """Host-side liveness of the ranks of a process group through its key-value store.

  Heartbeats are counters (no clocks are compared across hosts): a peer whose counter has not moved for
  `timeout` seconds of this rank's monotonic clock is taken as failed. `leave()` marks this rank as gone
  (call it between steps, with no kernel or collective of this rank in flight)."""

  def __init__(self, store, rank: int, world: int, interval: float = 0.2, timeout: float = 5.0,
               prefix: str = "fwn_watchdog"):
    self.store, self.rank, self.world = store, rank, world
    self.interval, self.timeout, self.prefix = interval, timeout, prefix
    self._beats = 0
    self._seen = {}
    self._stop = threading.Event()
    self._thread = None

  def _key(self, rank, what):
    return f"{self.prefix}/{rank}/{what}"

  def start(self):
    self.store.set(self._key(self.rank, "beat"), "0")
    self._thread = threading.Thread(target=self._run, daemon=True, name=f"fwn-watchdog-{self.rank}")
    self._thread.start()
    return self

  def _run(self):
    while not self._stop.wait(self.interval):
      self._beats += 1
      try:
        self.store.set(self._key(self.rank, "beat"), str(self._beats))
      except Exception:  # the store is gone (its host rank died): check() reports it
        return

  def leave(self):
    """Mark this rank as gone and stop its heartbeat."""
    self._stop.set()
    try:
      self.store.set(self._key(self.rank, "left"), "1")
    except Exception:
      pass

  def stop(self):
    self._stop.set()

  def check(self):
    """Raise RankFailure if a peer left or its heartbeat stalled for longer than `timeout`."""
    now = time.monotonic()
    for r in range(self.world):
      if r == self.rank:
        continue
      try:
        if self.store.check([self._key(r, "left")]):
          raise RankFailure(r, "left the job")
        beat = self.store.get(self._key(r, "beat")) if self.store.check([self._key(r, "beat")]) else b"-1"
      except RankFailure:
        raise
      except Exception as e:  # the store itself does not answer
        raise RankFailure(r, f"is unreachable (store error: {e})") from e
      last = self._seen.get(r)
      if last is None or last[0] != beat:
        self._seen[r] = (beat, now)
      elif now - last[1] > self.timeout:
        raise RankFailure(r, f"sent no heartbeat for {now - last[1]:.1f} s")


def abort_group(group=None):
  """Tear down a process group after a rank failure without waiting on the missing peer (NCCL communicators are
  aborted, not finalised); falls back to destroy_process_group where no abort is available."""
  from torch.distributed import distributed_c10d as c10d
  abort = getattr(c10d, "_abort_process_group", None)
  if abort is not None:
    try:
      abort(group)
      return
    except Exception:
      pass
  dist.destroy_process_group(group)


class DataParallelStep:
  """loss = mean over members of MSE(model(x_m, cond_m), target_m); grads all-reduced; Adam.

  `model(x, cond) -> y` is any torch module taking one member batch; `members` is the global number of
  members per step (split evenly across ranks: each rank takes members // world of them).
  """

  def __init__(self, model: torch.nn.Module, members: int, lr: float = 1e-4, group=None, bucket_mb: float = 25.0,
               overlap: bool = True, watchdog: RankWatchdog = None):
    self.model = model
    self.group = group
    self.world = dist.get_world_size(group) if dist.is_initialized() else 1
    self.rank = dist.get_rank(group) if dist.is_initialized() else 0
    if members % self.world:
      raise ValueError(f"{members} members do not split over {self.world} ranks")
    self.members = members
    self.local = members // self.world
    self.overlap = overlap
    self.watchdog = watchdog
    self.params = [p for p in model.parameters() if p.requires_grad]
    self.numel = sum(p.numel() for p in self.params)
    dev = self.params[0].device
    self.flat = torch.zeros(self.numel, dtype=torch.float32, device=dev)
    # Reverse parameter order: the backward produces the last block's gradients first.
    limit = max(1, int(bucket_mb * 2 ** 20 / 4))
    self.buckets = []            # (start, end, [params])
    off, start, members_of = 0, 0, []
    for p in reversed(self.params):
      k = p.numel()
      p.grad = self.flat[off:off + k].view_as(p)
      members_of.append(p)
      off += k
      if off - start >= limit:
        self.buckets.append((start, off, members_of))
        start, members_of = off, []
    if members_of:
      self.buckets.append((start, off, members_of))
    self._bucket_of = {id(p): i for i, (_, _, ps) in enumerate(self.buckets) for p in ps}
    self._pending = [0] * len(self.buckets)
    self._issued = 0
    self._works = []
    self._final = False
    if self.world > 1 and overlap:
      for p in self.params:
        p.register_post_accumulate_grad_hook(self._grad_ready)
    self.opt = torch.optim.Adam(self.params, lr=lr)

  def my_members(self):
    """Global indices of the members this rank processes."""
    return range(self.rank * self.local, (self.rank + 1) * self.local)

  def _grad_ready(self, p):
    if not self._final:
      return
    i = self._bucket_of[id(p)]
    self._pending[i] -= 1
    # Issue every complete bucket in bucket order (the same order on every rank).
    while self._issued < len(self.buckets) and self._pending[self._issued] == 0:
      self._issue(self._issued)
      self._issued += 1

  def _issue(self, i):
    s, e, _ = self.buckets[i]
    self._works.append(dist.all_reduce(self.flat[s:e], group=self.group, async_op=True))

  def _check_grad_views(self):
    for p in self.params:
      if p.grad is None or p.grad.data_ptr() < self.flat.data_ptr() or \
         p.grad.data_ptr() >= self.flat.data_ptr() + self.flat.numel() * 4:
        raise RuntimeError("a parameter's .grad was replaced; DataParallelStep keeps gradients in its buckets")

  def step(self, inputs, conds, targets, forward=None, micro_batch: int = 4) -> torch.Tensor:
    """inputs / conds / targets: sequences of this rank's member tensors (batch 1 each).

    micro_batch: members run together in one forward and backward (larger GEMMs, the attention's batch
    dimension); the gradient is the same sum of per-member terms. Activations for the backward take ~29 GB
    per member at configuration 5 (24 blocks over 40,962 nodes) without patch.OPTIONS.remat, which bounds it
    on one GPU. Returns the global mean loss (float32 scalar tensor on the device, identical on every rank)."""
    if self.watchdog is not None:
      self.watchdog.check()
    fwd = forward or (lambda x, c: self.model(x, c))
    self.flat.zero_()
    self._check_grad_views()
    loss_sum = torch.zeros((), dtype=torch.float32, device=self.flat.device)
    mb = max(1, micro_batch)
    starts = list(range(0, len(inputs), mb))
    self._pending = [len(ps) for _, _, ps in self.buckets]
    self._issued, self._works = 0, []
    for j, i in enumerate(starts):
      x, c, t = (torch.cat(list(v[i:i + mb])) for v in (inputs, conds, targets))
      y = fwd(x, c)
      # mean over a member's elements, summed over the micro-batch's members, over the global member count
      loss = torch.nn.functional.mse_loss(y.float(), t.float(), reduction="sum") / (y[0].numel() * self.members)
      self._final = self.world > 1 and self.overlap and j == len(starts) - 1
      try:
        loss.backward()
      finally:
        self._final = False
      loss_sum += loss.detach()
    if self.world > 1:
      if self.overlap:
        # Buckets whose parameters received no gradient in this backward (unused parameters) go now.
        while self._issued < len(self.buckets):
          self._issue(self._issued)
          self._issued += 1
      else:
        self._works.append(dist.all_reduce(self.flat, group=self.group, async_op=True))
      self._works.append(dist.all_reduce(loss_sum, group=self.group, async_op=True))
      for w in self._works:
        w.wait()
      self._works = []
    self.opt.step()
    return loss_sum
