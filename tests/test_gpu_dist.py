"""Data-parallel exchange on two GPUs over NCCL (skipped where fewer than two GPUs are visible).

Two ranks each run the fp32 filter forward and backward on their half of the batch; the layer's
c.weight, logit_bias and init_param gradients are averaged by LayerGradSync, whose all_reduce is
started from the parameters' post-accumulate-grad hooks during the backward. After wait() every
rank must hold the full-batch oracle gradients divided by two (each rank's loss sums its own
shard), elementwise within the fp32 bound 1e-5 (floor 1% of max|e|).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT, max_rel_err

pytestmark = pytest.mark.gpu

NH, NKVH, D, r, B, T = 2, 1, 128, 64, 4, 96


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    g = torch.Generator().manual_seed(5)
    C = NH * D
    x = torch.randn(B, T, C, generator=g)
    grads = [torch.randn(B, T, n, D, generator=g) for n in (NH, NKVH, NKVH)]
    return x, grads


def _worker(rank, world, port, out_q):
    import sys
    from datetime import timedelta

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from nanochat_filter_b200 import LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter, LtvInitValues
        from nanochat_filter_b200.dist import LayerGradSync

        torch.manual_seed(0)
        f = LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter(NH, NKVH, D, r)
        f.init_weights(alpha_mlp_bias_init=-1.0, weight_s=0.05, bias_s=0.5, init_s=0.5)
        f = f.to(dev)
        sync = LayerGradSync([f])
        x, grads = _problem()
        sl = slice(rank * B // world, (rank + 1) * B // world)
        q, k, v = f(x[sl].to(dev), LtvInitValues())
        torch.autograd.backward([q, k, v], [g[sl].to(dev) for g in grads])
        started = list(sync.started_order)
        sync.wait()
        torch.cuda.synchronize()
        out_q.put((rank, started, f.c.weight.detach().cpu().numpy(), f.logit_bias.detach().cpu().numpy(),
                   f.init_param.detach().cpu().numpy(), f.c.weight.grad.cpu().numpy(),
                   f.logit_bias.grad.cpu().numpy(), f.init_param.grad.cpu().numpy()))
        sync.remove()
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


def test_two_gpu_hook_reduced_gradients_equal_full_batch_oracle():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(rk, 2, port, q)) for rk in range(2)]
    for pr in procs:
        pr.start()
    results = [q.get(timeout=300) for _ in range(2)]
    for pr in procs:
        pr.join(timeout=120)
        assert pr.exitcode == 0
    import sys
    sys.path.insert(0, ROOT)
    from oracle import oracle as O

    x, grads = _problem()
    _, _, w, bias, init, _, _, _ = results[0]
    ref = O.layer_fwd_bwd(x.numpy(), w, np.repeat(init[None], B, 0), bias,
                          *[g.transpose(1, 2).contiguous().numpy() for g in grads], NH, NKVH, D // r, r, bf16=False)
    for _, started, _, _, _, gw, gb, gi in results:
        assert started == [0]  # the layer's reduction was started by its hooks, inside the backward
        assert max_rel_err(gw, ref["grad_w"] / 2, 1e-2) <= 1e-5
        assert max_rel_err(gb, ref["grad_logit_bias"] / 2, 1e-2) <= 1e-5
        assert max_rel_err(gi, ref["grad_inits"].sum(0) / 2, 1e-2) <= 1e-5
