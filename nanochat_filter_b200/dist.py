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


class GradBucket:
    """Flat buffer per dtype holding the gradients of a fixed parameter list.

    The buffer is allocated once; `reduce()` copies the gradients in, issues one all_reduce per
    dtype (average over the group) and copies the results back.
    """

    def __init__(self, params: List[torch.nn.Parameter]):
        self.params = list(params)
        self.groups = {}
        for p in self.params:
            self.groups.setdefault(p.dtype, []).append(p)
        self.buffers = {
            dt: torch.empty(sum(p.numel() for p in ps), dtype=dt, device=ps[0].device)
            for dt, ps in self.groups.items()
        }

    def reduce(self, group: Optional[dist.ProcessGroup] = None, average: bool = True) -> None:
        world = dist.get_world_size(group)
        for dt, ps in self.groups.items():
            buf = self.buffers[dt]
            off = 0
            for p in ps:
                n = p.numel()
                if p.grad is None:
                    buf[off:off + n].zero_()
                else:
                    buf[off:off + n].copy_(p.grad.reshape(-1))
                off += n
            dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
            if average and world > 1:
                buf.div_(world)
            off = 0
            for p in ps:
                n = p.numel()
                if p.grad is None:
                    p.grad = buf[off:off + n].view_as(p).clone()
                else:
                    p.grad.copy_(buf[off:off + n].view_as(p))
                off += n


def sync_filter_grads(modules: Iterable[torch.nn.Module], group: Optional[dist.ProcessGroup] = None,
                      average: bool = True) -> None:
    """One-shot helper: average the filter gradients of `modules` across the process group."""
    GradBucket(filter_parameters(modules)).reduce(group, average)
