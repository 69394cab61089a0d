"""Data-parallel gradient exchange of the filtered-QKV parameters.

Training shards the batch across ranks (one process per GPU); the scan and the projection need
no communication. The one exchange step is the gradient reduction of the parameters the path
touches — c.weight, logit_bias and init_param of every filtered layer — which the reference
performs inside DistMuonAdamW (nanochat/optim.py:367-403: all_reduce for small tensors,
reduce_scatter for the stacked matrices). Here those gradients are flattened into buckets
(grouped by dtype) and reduced with all_reduce, over NCCL/NVLink on GPUs (gloo on CPU): one bucket
for all layers (GradBucket, sync_filter_grads), or one per layer started from backward hooks as soon
as the layer's gradients are final (LayerGradSync), overlapping the rest of the backward.
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


def filter_modules(modules: Iterable[torch.nn.Module]) -> List[torch.nn.Module]:
    """The filters (modules holding c.weight, logit_bias and init_param) found in `modules`, in order."""
    out: List[torch.nn.Module] = []
    seen = set()
    for m in modules:
        for sub in m.modules():
            if hasattr(sub, "num_alpha_groups") and isinstance(getattr(sub, "logit_bias", None), torch.nn.Parameter) \
                    and id(sub) not in seen:
                seen.add(id(sub))
                out.append(sub)
    return out


class LayerGradSync:
    """One gradient bucket per filter layer, reduced as soon as that layer's gradients are final.

    The reference reduces every filter gradient in its optimizer step, after the whole backward
    (nanochat/optim.py:367-403). Here each layer's c.weight, logit_bias and init_param get a
    post-accumulate-grad hook; when the last of a layer's parameters has its gradient for this
    backward, the layer's bucket starts its all_reduce asynchronously, so the exchange of the later
    layers (whose backward runs first) overlaps the backward of the earlier ones. `wait()` ends the
    step: every started reduction is waited for and the averaged gradients are written back into the
    parameters' .grad. Layers whose gradients never arrived (unused in this step) are reduced in
    `wait()` with zero gradients, so every rank issues the same collectives in the same order.

    Gradient accumulation: with `sync = False` (e.g. inside `no_sync()`) the hooks do nothing and
    gradients accumulate locally; the backward of the step's last micro-batch runs with
    sync = True. Call `remove()` to detach the hooks.
    """

    def __init__(self, modules: Iterable[torch.nn.Module], group: Optional[dist.ProcessGroup] = None,
                 average: bool = True):
        self.group, self.average = group, average
        self.layers = [filter_parameters([m]) for m in filter_modules(modules)]
        self.buckets = [GradBucket(ps) for ps in self.layers]
        self.pending: List[Optional[PendingReduce]] = [None] * len(self.layers)
        self.arrived = [set() for _ in self.layers]
        self.started_order: List[int] = []  # layer indices in the order their reductions started
        self.sync = True
        self.handles = []
        for li, ps in enumerate(self.layers):
            for p in ps:
                self.handles.append(p.register_post_accumulate_grad_hook(self._hook(li)))

    def _hook(self, li: int):
        def hook(p: torch.nn.Parameter) -> None:
            if not self.sync or self.pending[li] is not None:
                return
            self.arrived[li].add(id(p))
            if len(self.arrived[li]) == len(self.layers[li]):
                self.pending[li] = self.buckets[li].start(self.group, self.average)
                self.started_order.append(li)
        return hook

    class _NoSync:
        def __init__(self, owner):
            self.owner = owner

        def __enter__(self):
            self.prev, self.owner.sync = self.owner.sync, False
            return self.owner

        def __exit__(self, *exc):
            self.owner.sync = self.prev
            return False

    def no_sync(self):
        """Context manager: backward passes inside it accumulate gradients without reducing them."""
        return LayerGradSync._NoSync(self)

    def wait(self) -> None:
        # in layer order on every rank: reductions not started by hooks are started here
        for li in range(len(self.layers)):
            if self.pending[li] is None:
                self.pending[li] = self.buckets[li].start(self.group, self.average)
                self.started_order.append(li)
        for li in range(len(self.layers)):
            self.pending[li].wait(copy_back=True)
            self.pending[li] = None
            self.arrived[li].clear()

    def remove(self) -> None:
        for h in self.handles:
            h.remove()
        self.handles = []


def sync_filter_grads(modules: Iterable[torch.nn.Module], group: Optional[dist.ProcessGroup] = None,
                      average: bool = True) -> None:
    """One-shot helper: average the filter gradients of `modules` across the process group."""
    GradBucket(filter_parameters(modules)).reduce(group, average)
