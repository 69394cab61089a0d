"""Multi-rank gradient exchange on CPU (gloo, world size 2).

Each rank holds one batch shard, computes the filtered-QKV gradients of its shard with the CPU
oracle (standing in for the GPU kernels, which these CPU ranks cannot run), stores them as the
parameters' .grad and calls the package's bucketed all_reduce. After the exchange every rank
must hold the full-batch gradient average — the data-parallel contract of the training configs.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(seed=0, B=4, T=16, NH=1, NKVH=1, D=8, r=4):
    rng = np.random.default_rng(seed)
    H, Da = NH + 2 * NKVH, D // r
    C = NH * D
    F = H * (D + Da)
    x = rng.standard_normal((B, T, C)).astype(np.float32)
    w = (rng.standard_normal((F, C)) / np.sqrt(C)).astype(np.float32)
    init = (0.5 * rng.standard_normal((H, D))).astype(np.float32)
    bias = rng.standard_normal((H, Da)).astype(np.float32)
    gq = rng.standard_normal((B, NH, T, D)).astype(np.float32)
    gk = rng.standard_normal((B, NKVH, T, D)).astype(np.float32)
    gv = rng.standard_normal((B, NKVH, T, D)).astype(np.float32)
    return dict(x=x, w=w, init=init, bias=bias, gq=gq, gk=gk, gv=gv, NH=NH, NKVH=NKVH, Da=Da, r=r)


def _grads(p, sl):
    import sys
    sys.path.insert(0, ROOT)
    from oracle import oracle as O

    B = p["x"][sl].shape[0]
    res = O.layer_fwd_bwd(p["x"][sl], p["w"], np.repeat(p["init"][None], B, 0), p["bias"], p["gq"][sl], p["gk"][sl],
                          p["gv"][sl], p["NH"], p["NKVH"], p["Da"], p["r"], bf16=False)
    # parameter gradients of the shard's mean loss contribution (scaled by the shard size)
    return res["grad_w"], res["grad_logit_bias"], res["grad_inits"].sum(0)


def _worker(rank, world, port, out_q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from nanochat_filter_b200 import LtvCombinedHeadMajorQkvFilter
        from nanochat_filter_b200.dist import sync_filter_grads

        p = _problem()
        B = p["x"].shape[0]
        shard = slice(rank * B // world, (rank + 1) * B // world)
        f = LtvCombinedHeadMajorQkvFilter(p["NH"], p["NKVH"], p["Da"] * p["r"], p["r"])
        gw, gb, gi = _grads(p, shard)
        f.c.weight.grad = torch.from_numpy(gw)
        f.logit_bias.grad = torch.from_numpy(gb)
        f.init_param.grad = torch.from_numpy(gi)
        sync_filter_grads([f])
        out_q.put((rank, f.c.weight.grad.numpy().copy(), f.logit_bias.grad.numpy().copy(),
                   f.init_param.grad.numpy().copy()))
    finally:
        dist.destroy_process_group()


def test_two_rank_gradient_average_matches_full_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    results = [q.get(timeout=240) for _ in range(2)]
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    p = _problem()
    gw, gb, gi = _grads(p, slice(None))
    for _, rw, rb, ri in results:
        # the average over 2 equal shards is half the full-batch sum
        np.testing.assert_allclose(rw, gw / 2, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(rb, gb / 2, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(ri, gi / 2, rtol=1e-5, atol=1e-6)


def _worker_async(rank, world, port, out_q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from nanochat_filter_b200 import LtvCombinedHeadMajorQkvFilter
        from nanochat_filter_b200.dist import GradBucket, filter_parameters

        p = _problem()
        B = p["x"].shape[0]
        shard = slice(rank * B // world, (rank + 1) * B // world)
        f = LtvCombinedHeadMajorQkvFilter(p["NH"], p["NKVH"], p["Da"] * p["r"], p["r"])
        bucket = GradBucket(filter_parameters([f]))
        gw, gb, gi = _grads(p, shard)
        # step 1's gradients go out, then step 2 overwrites .grad before step 1's reduction is awaited
        f.c.weight.grad, f.logit_bias.grad, f.init_param.grad = (torch.from_numpy(a) for a in (gw, gb, gi))
        h1 = bucket.start()
        f.c.weight.grad, f.logit_bias.grad, f.init_param.grad = (torch.from_numpy(2 * a) for a in (gw, gb, gi))
        h2 = bucket.start()
        h1.wait(copy_back=False)
        flat1 = bucket.buffers[h1.slot][torch.float32].numpy().copy()
        h2.wait(copy_back=True)
        out_q.put((rank, flat1, f.c.weight.grad.numpy().copy(), f.logit_bias.grad.numpy().copy(),
                   f.init_param.grad.numpy().copy()))
    finally:
        dist.destroy_process_group()


def test_two_rank_overlapped_reductions_keep_their_own_gradients():
    """Two reductions in flight (GradBucket.start): each averages the gradients it was started with."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_async, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    results = [q.get(timeout=240) for _ in range(2)]
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    p = _problem()
    gw, gb, gi = _grads(p, slice(None))
    flat_expect = np.concatenate([gw.reshape(-1), gb.reshape(-1), gi.reshape(-1)]) / 2
    for _, flat1, rw, rb, ri in results:
        np.testing.assert_allclose(flat1, flat_expect, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(rw, gw, rtol=1e-5, atol=1e-6)   # average of 2x the shard sums
        np.testing.assert_allclose(rb, gb, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(ri, gi, rtol=1e-5, atol=1e-6)


class _CpuFilter(torch.nn.Module):
    """A CPU stand-in with a filter's parameters (c.weight, logit_bias, init_param) and a plain
    differentiable forward, so the hook-driven exchange can be exercised on gloo ranks."""

    def __init__(self, C, H, D, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.num_alpha_groups = 1
        self.c = torch.nn.Linear(C, H * (D + 1), bias=False)
        with torch.no_grad():
            self.c.weight.copy_(torch.randn(H * (D + 1), C, generator=g) / C ** 0.5)
        self.logit_bias = torch.nn.Parameter(torch.randn(H, 1, generator=g))
        self.init_param = torch.nn.Parameter(torch.randn(H, D, generator=g))
        self.H, self.D, self.C = H, D, C

    def forward(self, x):
        y = torch.tanh(x @ self.c.weight.t())[..., : self.C]
        return y + (self.logit_bias.sum() + self.init_param.mean()) * 0.1


def _layered_grads(model, x):
    model.zero_grad(set_to_none=True)
    h = x
    for layer in model:
        h = layer(h)
    (h * h).sum().backward()
    return [[p.grad.detach().clone() for p in (l.c.weight, l.logit_bias, l.init_param)] for l in model]


def _worker_layers(rank, world, port, out_q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from nanochat_filter_b200.dist import LayerGradSync

        model = torch.nn.ModuleList([_CpuFilter(8, 2, 4, seed=10 + i) for i in range(3)])
        x = torch.randn(4, 5, 8, generator=torch.Generator().manual_seed(7))
        shard = x[rank * 2:(rank + 1) * 2]
        sync = LayerGradSync(model)
        # two micro-batches of the shard: the first accumulates locally, the second reduces
        with sync.no_sync():
            _layered_grads(model, shard[:1])
        started_no_sync = list(sync.started_order)
        h = shard[1:]
        for layer in model:
            h = layer(h)
        (h * h).sum().backward()
        started_in_backward = list(sync.started_order)
        sync.wait()
        out_q.put((rank, started_no_sync, started_in_backward,
                   [[p.grad.numpy().copy() for p in (l.c.weight, l.logit_bias, l.init_param)] for l in model]))
        sync.remove()
    finally:
        dist.destroy_process_group()


def test_two_rank_layer_buckets_reduced_from_backward_hooks():
    """LayerGradSync: each layer's reduction starts from its parameters' post-accumulate-grad hooks
    during the backward (last layer first), nothing is reduced inside no_sync, and after wait() every
    rank holds the average over ranks of its accumulated gradients."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_layers, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    results = [q.get(timeout=240) for _ in range(2)]
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    model = torch.nn.ModuleList([_CpuFilter(8, 2, 4, seed=10 + i) for i in range(3)])
    x = torch.randn(4, 5, 8, generator=torch.Generator().manual_seed(7))
    per_micro = [_layered_grads(model, x[i:i + 1]) for i in range(4)]
    expect = [[sum(per_micro[i][li][pi] for i in range(4)).numpy() / 2 for pi in range(3)] for li in range(3)]
    for _, started_no_sync, started_in_backward, grads in results:
        assert started_no_sync == []
        assert started_in_backward == [2, 1, 0]  # started by hooks during the backward, last layer first
        for li in range(3):
            for pi in range(3):
                np.testing.assert_allclose(grads[li][pi], expect[li][pi], rtol=1e-5, atol=1e-6)
