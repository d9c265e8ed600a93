"""CPU: the data-parallel fine-tune step on 2 gloo ranks equals the single-process step.

The product step (faster_weathernext.finetune.DataParallelStep) is generic over the model; here it runs a
small test-only model on the CPU (no attention kernel involved) to check the distributed logic: member
split, gradient accumulation, the flat-bucket all-reduce and identical Adam updates on every rank.
"""
import os
import socket

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


def _worker(rank, world, port, members, out):
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
  dist.init_process_group("gloo", rank=rank, world_size=world)
  from faster_weathernext.finetune import DataParallelStep
  model = TinyModel()
  step = DataParallelStep(model, members, lr=1e-2)
  xs, cs, ts = _data(members)
  idx = list(step.my_members())
  for _ in range(2):
    loss = step.step([xs[i] for i in idx], [cs[i] for i in idx], [ts[i] for i in idx])
  out[rank] = (torch.cat([p.detach().reshape(-1) for p in model.parameters()]), float(loss))
  dist.destroy_process_group()


def _free_port():
  with socket.socket() as s:
    s.bind(("127.0.0.1", 0))
    return s.getsockname()[1]


@pytest.mark.timeout(120)
def test_two_rank_step_matches_single_process():
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
    mp.start_processes(_worker, args=(2, _free_port(), members, out), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
      params, loss = out[r]
      torch.testing.assert_close(params, ref, rtol=1e-5, atol=1e-6)
      assert abs(loss - float(loss1)) < 1e-5


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
