"""Data-parallel gradient exchange of the filtered-QKV parameters.

Training shards the batch across ranks (one process per GPU); the scan and the projection need
no communication. The one exchange step is the gradient reduction of the parameters the path
touches — c.weight, logit_bias and init_param of every filtered layer — which the reference
performs inside DistMuonAdamW (nanochat/optim.py:367-403: all_reduce for small tensors,
reduce_scatter for the stacked matrices). Here those gradients are flattened into one bucket
(grouped by dtype) and reduced with a single all_reduce, over NCCL/NVLink on GPUs (gloo on CPU).
"""

from __future__ import annotations

from typing import Iterable, List, Optional

import torch
import torch.distributed as dist


def filter_parameters(modules: Iterable[torch.nn.Module]) -> List[torch.nn.Parameter]:
    """c.weight, logit_bias and init_param of every filter found in `modules` (in order)."""
    out: List[torch.nn.Parameter] = []
    seen = set()
    for m in modules:
        for sub in m.modules():
            for name in ("c", "logit_bias", "init_param"):
                p = getattr(sub, name, None)
                if name == "c" and p is not None:
                    p = getattr(p, "weight", None)
                if isinstance(p, torch.nn.Parameter) and hasattr(sub, "num_alpha_groups") and id(p) not in seen:
                    seen.add(id(p))
                    out.append(p)
    return out


class PendingReduce:
    """An all_reduce of a GradBucket in flight (`GradBucket.start`)."""

    def __init__(self, bucket: "GradBucket", slot: int, works, world: int, average: bool):
        self.bucket, self.slot, self.works, self.world, self.average = bucket, slot, works, world, average

    def wait(self, copy_back: bool = True) -> None:
        """Orders the current stream after the reduction; averages, and writes the results back into
        the parameters' .grad unless `copy_back` is False (the flat buffers then hold them)."""
        for w in self.works:
            w.wait()
        for dt, ps in self.bucket.groups.items():
            buf = self.bucket.buffers[self.slot][dt]
            if self.average and self.world > 1:
                buf.div_(self.world)
            if copy_back:
                self.bucket._scatter(ps, buf)


class GradBucket:
    """Flat buffers per dtype holding the gradients of a fixed parameter list.

    Buffers are allocated once (two sets, so that one reduction can be in flight while the next
    step's gradients are copied in); `reduce()` copies the gradients in, issues one all_reduce per
    dtype (average over the group) and copies the results back. `start()` is the same split in
    two: the all_reduce runs asynchronously (overlapping whatever the stream does next) until the
    returned handle's `wait()`.
    """

    def __init__(self, params: List[torch.nn.Parameter]):
        self.params = list(params)
        self.groups = {}
        for p in self.params:
            self.groups.setdefault(p.dtype, []).append(p)
        self.buffers = [{
            dt: torch.empty(sum(p.numel() for p in ps), dtype=dt, device=ps[0].device)
            for dt, ps in self.groups.items()
        } for _ in range(2)]
        self._next = 0

    def _gather(self, ps, buf) -> None:
        off = 0
        for p in ps:
            n = p.numel()
            if p.grad is None:
                buf[off:off + n].zero_()
            else:
                buf[off:off + n].copy_(p.grad.reshape(-1))
            off += n

    def _scatter(self, ps, buf) -> None:
        off = 0
        for p in ps:
            n = p.numel()
            if p.grad is None:
                p.grad = buf[off:off + n].view_as(p).clone()
            else:
                p.grad.copy_(buf[off:off + n].view_as(p))
            off += n

    def start(self, group: Optional[dist.ProcessGroup] = None, average: bool = True) -> PendingReduce:
        slot = self._next
        self._next ^= 1
        works = []
        for dt, ps in self.groups.items():
            buf = self.buffers[slot][dt]
            self._gather(ps, buf)
            works.append(dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group, async_op=True))
        return PendingReduce(self, slot, works, dist.get_world_size(group), average)

    def reduce(self, group: Optional[dist.ProcessGroup] = None, average: bool = True) -> None:
        self.start(group, average).wait(copy_back=True)


def sync_filter_grads(modules: Iterable[torch.nn.Module], group: Optional[dist.ProcessGroup] = None,
                      average: bool = True) -> None:
    """One-shot helper: average the filter gradients of `modules` across the process group."""
    GradBucket(filter_parameters(modules)).reduce(group, average)
