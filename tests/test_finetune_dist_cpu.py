"""CPU: the data-parallel fine-tune step on 2 gloo ranks equals the single-process step; rank failures are
detected on the host.

The product step (faster_weathernext.finetune.DataParallelStep) is generic over the model; here it runs a
small test-only model on the CPU (no attention kernel involved) to check the distributed logic: member
split, gradient accumulation, the bucketed all-reduce issued from gradient hooks during the backward (and the
one-buffer all-reduce after it), identical Adam updates on every rank, and the RankWatchdog: a rank that
leaves between steps, or dies without a word, makes the others raise instead of waiting in a collective.
"""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


class TinyModel(torch.nn.Module):
  def __init__(self):
    super().__init__()
    g = torch.Generator().manual_seed(0)
    self.w = torch.nn.Parameter(torch.randn(8, 8, generator=g) * 0.3)
    self.c = torch.nn.Parameter(torch.randn(4, 8, generator=g) * 0.3)

  def forward(self, x, cond):
    return torch.tanh(x @ self.w + (cond @ self.c).unsqueeze(1))


def _data(members):
  g = torch.Generator().manual_seed(1)
  xs = [torch.randn(1, 16, 8, generator=g) for _ in range(members)]
  cs = [torch.randn(1, 4, generator=g) for _ in range(members)]
  ts = [torch.randn(1, 16, 8, generator=g) for _ in range(members)]
  return xs, cs, ts


def _worker(rank, world, port, members, out, overlap, bucket_mb):
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
  dist.init_process_group("gloo", rank=rank, world_size=world)
  from faster_weathernext.finetune import DataParallelStep
  model = TinyModel()
  step = DataParallelStep(model, members, lr=1e-2, overlap=overlap, bucket_mb=bucket_mb)
  xs, cs, ts = _data(members)
  idx = list(step.my_members())
  for _ in range(2):
    loss = step.step([xs[i] for i in idx], [cs[i] for i in idx], [ts[i] for i in idx], micro_batch=1)
  out[rank] = (torch.cat([p.detach().reshape(-1) for p in model.parameters()]), float(loss), len(step.buckets))
  dist.destroy_process_group()


def _free_port():
  with socket.socket() as s:
    s.bind(("127.0.0.1", 0))
    return s.getsockname()[1]


@pytest.mark.timeout(120)
@pytest.mark.parametrize("overlap,bucket_mb", [(True, 1e-4), (True, 25.0), (False, 25.0)])
def test_two_rank_step_matches_single_process(overlap, bucket_mb):
  """Two ranks (two members each, one per micro-batch) equal one process with all four members: buckets
  of one parameter each issued from the backward's hooks, one bucket, or one all-reduce after the backward."""
  from faster_weathernext.finetune import DataParallelStep
  members = 4
  model = TinyModel()
  step = DataParallelStep(model, members, lr=1e-2)
  xs, cs, ts = _data(members)
  for _ in range(2):
    loss1 = step.step(xs, cs, ts)
  ref = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
  with mp.Manager() as m:
    out = m.dict()
    mp.start_processes(_worker, args=(2, _free_port(), members, out, overlap, bucket_mb), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
      params, loss, n_buckets = out[r]
      torch.testing.assert_close(params, ref, rtol=1e-5, atol=1e-6)
      assert abs(loss - float(loss1)) < 1e-5
      assert n_buckets == (2 if bucket_mb < 1 else 1)


def _failing_worker(rank, world, port, how, out):
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
  dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
  from torch.distributed import distributed_c10d as c10d
  from faster_weathernext.finetune import DataParallelStep, RankFailure, RankWatchdog, abort_group
  store = c10d._get_default_store()
  dog = RankWatchdog(store, rank, world, interval=0.1, timeout=1.0).start()
  model = TinyModel()
  step = DataParallelStep(model, 4, lr=1e-2, watchdog=dog, bucket_mb=1e-4)
  xs, cs, ts = _data(4)
  idx = list(step.my_members())
  args = ([xs[i] for i in idx], [cs[i] for i in idx], [ts[i] for i in idx])
  step.step(*args)
  if rank == 1:
    # Between steps, with nothing of this rank in flight: leave politely, or vanish.
    if how == "leave":
      dog.leave()
    store.set("test/rank1_gone", "1")
    os._exit(0)
  store.wait(["test/rank1_gone"])
  if how == "vanish":
    time.sleep(1.5)                 # longer than the heartbeat timeout
  t0 = time.monotonic()
  try:
    step.step(*args)
    out[rank] = ("no error", time.monotonic() - t0)
  except RankFailure as e:
    out[rank] = ("RankFailure", time.monotonic() - t0, e.rank)
  except RuntimeError as e:       # the collective itself failed (the peer's connection closed)
    out[rank] = ("RuntimeError", time.monotonic() - t0)
  dog.stop()
  abort_group()


@pytest.mark.timeout(120)
@pytest.mark.parametrize("how", ["leave", "vanish"])
def test_rank_failure_between_steps_raises_instead_of_hanging(how):
  """A rank that leaves between steps is seen in the store before the next step's first launch (RankFailure
  naming it, at once); one that exits without a word is seen by its stalled heartbeat, or at the latest by
  the next collective failing, well inside the process group's 20 s timeout."""
  with mp.Manager() as m:
    out = m.dict()
    mp.start_processes(_failing_worker, args=(2, _free_port(), how, out), nprocs=2, join=True,
                       start_method="spawn")
    res = out[0]
  if how == "leave":
    assert res[0] == "RankFailure" and res[2] == 1 and res[1] < 1.0, res
  else:
    assert res[0] in ("RankFailure", "RuntimeError") and res[1] < 10.0, res


def test_batched_step_equals_member_loop():
  """Micro-batches of 1, 2 or 3 members give the same gradient and loss (CPU, tiny model)."""
  import torch
  from faster_weathernext.finetune import DataParallelStep

  class Tiny(torch.nn.Module):
    def __init__(self):
      super().__init__()
      self.w = torch.nn.Parameter(torch.linspace(-1, 1, 12).reshape(3, 4))

    def forward(self, x, c):
      return torch.tanh(x @ self.w) * (1 + c[:, None, :1])

  g = torch.Generator().manual_seed(0)
  xs = [torch.randn(1, 5, 3, generator=g) for _ in range(3)]
  cs = [torch.randn(1, 2, generator=g) for _ in range(3)]
  ts = [torch.randn(1, 5, 4, generator=g) for _ in range(3)]
  grads, losses = [], []
  for mb in (1, 2, 3):
    model = Tiny()
    step = DataParallelStep(model, members=3, lr=0.0)
    losses.append(float(step.step(xs, cs, ts, micro_batch=mb)))
    grads.append(model.w.grad.clone())
  for loss, grad in zip(losses[1:], grads[1:]):
    assert abs(losses[0] - loss) < 1e-6
    assert torch.allclose(grads[0], grad, atol=1e-6)
