"""Data-parallel fine-tuning step on the processor (configuration 5).

One step over a batch of ensemble members split across ranks: each rank runs forward + backward (the
attention's custom-VJP kernels included) for its members, accumulating gradients; the float32 gradients
are summed across ranks with one NCCL all-reduce over NVLink (one flat bucket), averaged, and Adam
updates the parameters identically on every rank. The loss is the mean-squared error to the targets.
The reference's fine-tuning library (src/faster_weathernext/finetune.py:136-150: value_and_grad, optax
update, single device) has no collective; the all-reduce is what sharding members across GPUs adds.
"""

import torch
import torch.distributed as dist


class DataParallelStep:
  """loss = mean over members of MSE(model(x_m, cond_m), target_m); grads all-reduced; Adam.

  `model(x, cond) -> y` is any torch module taking one member batch; `members` is the global number of
  members per step (split evenly across ranks: each rank takes members // world of them).
  """

  def __init__(self, model: torch.nn.Module, members: int, lr: float = 1e-4, group=None):
    self.model = model
    self.group = group
    self.world = dist.get_world_size(group) if dist.is_initialized() else 1
    self.rank = dist.get_rank(group) if dist.is_initialized() else 0
    if members % self.world:
      raise ValueError(f"{members} members do not split over {self.world} ranks")
    self.members = members
    self.local = members // self.world
    self.params = [p for p in model.parameters() if p.requires_grad]
    self.numel = sum(p.numel() for p in self.params)
    dev = self.params[0].device
    self.flat = torch.empty(self.numel, dtype=torch.float32, device=dev)
    self.opt = torch.optim.Adam(self.params, lr=lr)

  def my_members(self):
    """Global indices of the members this rank processes."""
    return range(self.rank * self.local, (self.rank + 1) * self.local)

  def step(self, inputs, conds, targets, forward=None, micro_batch: int = 4) -> torch.Tensor:
    """inputs / conds / targets: sequences of this rank's member tensors (batch 1 each).

    micro_batch: members run together in one forward and backward (larger GEMMs, the attention's batch
    dimension); the gradient is the same sum of per-member terms. Activations for the backward take ~29 GB
    per member at configuration 5 (24 blocks over 40,962 nodes), which bounds it on one GPU.
    Returns the global mean loss (float32 scalar tensor on the device, identical on every rank)."""
    fwd = forward or (lambda x, c: self.model(x, c))
    self.opt.zero_grad(set_to_none=False)
    loss_sum = torch.zeros((), dtype=torch.float32, device=self.flat.device)
    mb = max(1, micro_batch)
    for i in range(0, len(inputs), mb):
      x, c, t = (torch.cat(list(v[i:i + mb])) for v in (inputs, conds, targets))
      y = fwd(x, c)
      # mean over a member's elements, summed over the micro-batch's members, over the global member count
      loss = torch.nn.functional.mse_loss(y.float(), t.float(), reduction="sum") / (y[0].numel() * self.members)
      loss.backward()
      loss_sum += loss.detach()
    # One flat float32 bucket: gather, all-reduce (sum over ranks of per-member-mean contributions), scatter.
    off = 0
    for p in self.params:
      k = p.numel()
      self.flat[off:off + k].copy_(p.grad.reshape(-1))
      off += k
    if self.world > 1:
      dist.all_reduce(self.flat, group=self.group)
      dist.all_reduce(loss_sum, group=self.group)
    off = 0
    for p in self.params:
      k = p.numel()
      p.grad.copy_(self.flat[off:off + k].view_as(p.grad))
      off += k
    self.opt.step()
    return loss_sum
