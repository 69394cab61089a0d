#!/usr/bin/env python
"""Filtered-QKV hot-path benchmark: one layer's forward + backward, tokens/s.

`python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config config2]`
Under torchrun each rank drives one GPU on its own batch shard (weak scaling) and the step
ends with the all-reduce of the filter gradients (the path's one exchange step).

A step is the reference's layer composition: projection (x[B,T,C] x W^T -> [B,F,T]), scan,
scan backward, projection backward (dx and dW), [all-reduce of dW, d logit_bias, d init].
`value`: device-resident inputs, timed with CUDA events, max over ranks.
`e2e`: the same step through the public module API (filter forward + autograd backward),
with the step's inputs (x and the upstream q/k/v gradients) copied from pinned host memory
and the step's result (the layer's parameter gradients: dW, d logit_bias, d init) read back,
inside the timed region.
Prints one JSON line (rank 0).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "filtered-QKV fwd+bwd tokens/s"
UNIT = "tokens/s"

CONFIGS = {
    # Benchmark configs 1-3 mapped onto the reference parameterisation (head_dim 128, r = 128 ->
    # one decay logit per head per token; F = (NH + 2 NKVH) * 129).
    "config2": dict(B=32, T=1024, C=768, NH=6, NKVH=6, D=128, r=128, dtype="bf16", bias=0.0,
                    desc="d=12 training shape: B=32/rank, T=1024, C=768, 6+6+6 heads x 128, r=128, bf16"),
    # config 3's decay a = 1 - alpha ~ 0.95 (reference gate alpha = sigmoid(logit)): the decay
    # pre-activation ~ N(3, 1) as logit rows ~ N(0, 1/sqrt(C)) (pre-activation std 1) and bias -3
    "config3": dict(B=4, T=16384, C=1024, NH=8, NKVH=8, D=128, r=128, dtype="bf16", bias=-3.0, logit_std="1/sqrt(C)",
                    desc="long sequence: B=4/rank, T=16384, C=1024, 8+8+8 heads x 128, r=128, bf16, a~0.95"),
    "config1": dict(B=2, T=256, C=768, NH=6, NKVH=6, D=128, r=128, dtype="f32", bias=0.0,
                    desc="CPU-runnable shape in fp32: B=2/rank, T=256, C=768, 6+6+6 heads x 128"),
}

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(kernel: str, config: str):
    """DRAM bytes per launch recorded from an ncu capture in profiles/<kernel>_<config>.md
    (line `dram_bytes_per_launch: N`), or None."""
    p = os.path.join(ROOT, "profiles", f"{kernel}_{config}.md")
    try:
        with open(p) as f:
            for line in f:
                if line.strip().startswith("dram_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].strip().split()[0])
    except OSError:
        pass
    return None


# ------------------------------------------------------------------------------------------
# Clock sampling during the timed region
# ------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def gpu_id_for(dev_index: int) -> str:
    import torch

    try:
        props = torch.cuda.get_device_properties(dev_index)
        bus = getattr(props, "pci_bus_id", None)
        dom = getattr(props, "pci_domain_id", None)
        devid = getattr(props, "pci_device_id", None)
        if bus is not None and dom is not None and devid is not None:
            return f"{dom:08X}:{bus:02X}:{devid:02X}.0"
    except Exception:
        pass
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        return vis.split(",")[dev_index]
    return str(dev_index)


# ------------------------------------------------------------------------------------------
# Workload
# ------------------------------------------------------------------------------------------
def _logit_std(cfg):
    return 1.0 / math.sqrt(cfg["C"]) if cfg.get("logit_std") == "1/sqrt(C)" else 0.02


def make_inputs(cfg, device, seed):
    import torch

    g = torch.Generator(device="cpu").manual_seed(seed)
    B, T, C, NH, NKVH, D, r = (cfg[k] for k in ("B", "T", "C", "NH", "NKVH", "D", "r"))
    H, Da = NH + 2 * NKVH, D // r
    F = H * (D + Da)
    dt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float32
    x = torch.randn(B, T, C, generator=g).to(dt)
    wv = torch.randn(H, D, C, generator=g) / math.sqrt(C)      # value rows ~ N(0, 1/sqrt(C))
    wl = torch.randn(H, Da, C, generator=g) * _logit_std(cfg)  # decay-logit rows ~ N(0, 0.02) (config 3: 1/sqrt(C))
    W = torch.cat([wv, wl], dim=1).reshape(F, C)              # head-major interleaved, fp32 master
    bias = torch.full((H, Da), float(cfg["bias"]))
    init = torch.zeros(H, D)
    gq = torch.randn(B, NH, T, D, generator=g).to(dt)
    gk = torch.randn(B, NKVH, T, D, generator=g).to(dt)
    gv = torch.randn(B, NKVH, T, D, generator=g).to(dt)
    host = dict(x=x, W=W, bias=bias, init=init, gq=gq, gk=gk, gv=gv)
    dev = {k: v.to(device) for k, v in host.items()}
    return host, dev, dict(B=B, T=T, C=C, NH=NH, NKVH=NKVH, D=D, r=r, H=H, Da=Da, F=F, dt=dt)


def _graph_us(fn, device, reps=20):
    """Average device time (us) of `fn` replayed as one CUDA graph, timed with CUDA events."""
    import torch

    cs = torch.cuda.Stream(device)
    cs.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cs):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(cs)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=cs):
        fn()
    for _ in range(3):
        g.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    del g
    return us


def prologue_timing(cfg, d, W, bias, init, s, device):
    """The layer step followed by the reference attention's prologue on q and k (rotary embedding then
    RMS norm, nanochat/gpt.py:224-230) and its backward, three ways on the bench's inputs: without the
    prologue, with it as separate kernels after the filter (ltv_rotary_qk_norm and its backward), and
    folded into the filter's kernels (ltv_proj_scan_rope_norm_cuda_op, the raw q/k replayed from the
    checkpoints in the backward). Only on the one-kernel shapes (where the fused form exists)."""
    import torch

    import nanochat_filter_b200 as nf

    ops = torch.ops.nanochat_cuda
    B, T, NH, NKVH, D, r, H, Da, dt = (s[k] for k in ("B", "T", "NH", "NKVH", "D", "r", "H", "Da", "dt"))
    if len(nf.ops._ckpt_shape(d["x"], NH, NKVH, Da, r)) != 4:
        return None
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, dtype=torch.float32, device=device) / D))
    fr = torch.outer(torch.arange(T, dtype=torch.float32, device=device), inv)
    cos, sin = fr.cos().to(dt)[None, :, None, :], fr.sin().to(dt)[None, :, None, :]
    a = (NH, NKVH, Da, r)
    Wg = torch.zeros_like(W)

    def tail(comb, inits, ckpt, dq, dk):
        combined = comb.transpose(1, 2)
        gc = torch.empty_like(combined)
        gi, gb = torch.empty(H, D, device=device), torch.empty_like(bias)
        ops.ltv_scan_ckpt_backward_kernel(combined, inits, bias, ckpt, dq, dk, d["gv"], gc, gi, gb, *a, True)
        ops.fused_linear_transpose_backward_kernel(d["x"], W.to(dt), gc.transpose(1, 2), torch.empty_like(d["x"]), Wg)

    def plain():
        inits = init.to(dt)
        comb, q, k, v, ckpt = ops.ltv_proj_scan_cuda_op(d["x"], W.to(dt), inits, bias, *a, True)
        tail(comb, inits, ckpt, d["gq"], d["gk"])

    def separate():
        inits = init.to(dt)
        comb, q, k, v, ckpt = ops.ltv_proj_scan_cuda_op(d["x"], W.to(dt), inits, bias, *a, True)
        ops.ltv_rotary_qk_norm(q.transpose(1, 2), k.transpose(1, 2), cos, sin)
        dq, dk = ops.ltv_rotary_qk_norm_backward(q.transpose(1, 2), k.transpose(1, 2), cos, sin,
                                                 d["gq"].transpose(1, 2), d["gk"].transpose(1, 2))
        tail(comb, inits, ckpt, dq.transpose(1, 2), dk.transpose(1, 2))

    def fused():
        inits = init.to(dt)
        comb, qn, kn, v, ckpt = ops.ltv_proj_scan_rope_norm_cuda_op(d["x"], W.to(dt), inits, bias, cos, sin, *a, True)
        dq, dk = ops.ltv_rotary_qk_norm_ckpt_backward(comb.transpose(1, 2), inits, bias, ckpt, cos, sin, d["gq"],
                                                      d["gk"], *a, True)
        tail(comb, inits, ckpt, dq, dk)

    out = {k: round(_graph_us(fn, device), 1) for k, fn in (("step_us", plain), ("separate_us", separate),
                                                            ("fused_us", fused))}
    out["what"] = ("layer step (fwd + bwd) followed by the attention's q/k prologue (rotary + RMS norm) and its "
                   "backward: without it, as separate kernels after the filter, folded into the filter's kernels; "
                   "each replayed as one CUDA graph, CUDA-event timing")
    return out


def run_ours(args, cfg):
    import torch
    import torch.distributed as dist

    import nanochat_filter_b200 as nf
    from nanochat_filter_b200 import _lib
    from nanochat_filter_b200.dist import GradBucket, LayerGradSync

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta

        torch.cuda.set_device(local)
        # The filter-grad all-reduce (7 MB) runs concurrently with the next step's persistent
        # kernels; capping NCCL at 4 channels (4 CTAs) leaves them more SMs and still finishes the
        # reduction well inside one step (2 GPUs: 124.1M -> 128.3M tokens/s). On NVSwitch NCCL picks
        # NVLS for this size, whose channel count the first cap does not bound (24 CTAs at 8 GPUs),
        # so from 4 GPUs up it is capped too (8 GPUs: 494.5M -> 518.3M tokens/s; NVLS off, ring:
        # 356.8M); 2 GPUs measured no better with it (130.8M against 141.9M without, other boxes).
        # Overridable.
        os.environ.setdefault("NCCL_MAX_NCHANNELS", "4")
        if world >= 4:
            os.environ.setdefault("NCCL_NVLS_NCHANNELS", "4")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    _lib.load()

    host, d, s = make_inputs(cfg, device, seed=1234 + rank)
    B, T, C, NH, NKVH, D, r, H, Da, F, dt = (s[k] for k in ("B", "T", "C", "NH", "NKVH", "D", "r", "H", "Da", "F",
                                                           "dt"))
    ops = torch.ops.nanochat_cuda
    scan_args = (NH, NKVH, Da, r)
    W = d["W"]
    Wg = torch.zeros_like(W)
    bias = d["bias"]
    init = d["init"]
    bucket_params = [torch.nn.Parameter(W), torch.nn.Parameter(bias), torch.nn.Parameter(init)]
    bucket = GradBucket(bucket_params) if world > 1 else None

    ev = None

    def step(record):
        # one layer fwd + bwd with the same operators the filter's autograd graph runs
        w_c = W.to(dt)                                              # weight cast (autocast's job)
        inits = init.to(dt)                 # one initial state [H, D] for every sequence (training)
        if record is not None:
            record[0].record()
        # projection + scan forward in one call (equal to fused_linear_transpose_cuda_op followed
        # by the scan op on comb^T, the filter's composition); ckpt: the scan states at the 32-token
        # chunk starts, from which the scan backward replays q/k/v instead of reading them
        comb, q, k, v, ckpt = ops.ltv_proj_scan_cuda_op(d["x"], w_c, inits, bias, *scan_args, True)  # comb [B, F, T]
        if record is not None:
            record[1].record()
            record[2].record()
        combined = comb.transpose(1, 2)
        gc = torch.empty_like(combined)
        if ckpt.numel():
            # the initial state's gradient summed over the batch and the logit-bias gradient are
            # written (not accumulated) by the kernel
            gi = torch.empty(H, D, device=device)
            gb = torch.empty_like(bias)
            if record is not None:
                record[3].record()
            ops.ltv_scan_ckpt_backward_kernel(combined, inits, bias, ckpt, d["gq"], d["gk"], d["gv"], gc, gi, gb,
                                              *scan_args, True)
        else:
            # shapes without the one-kernel forward: the per-sequence form, summed over the batch
            ib = inits.unsqueeze(0).expand(B, -1, -1).contiguous()
            gib = torch.empty_like(ib)
            gb = torch.zeros_like(bias)
            if record is not None:
                record[3].record()
            ops.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_backward_kernel(
                combined, ib, bias, q, k, v, d["gq"], d["gk"], d["gv"], gc, gib, gb, *scan_args, 32, 2, 8, True)
            gi = gib.float().sum(0)
        if record is not None:
            record[4].record()
        gx = torch.empty_like(d["x"])
        if record is not None:
            record[5].record()
        ops.fused_linear_transpose_backward_kernel(d["x"], w_c, gc.transpose(1, 2), gx, Wg)
        if record is not None:
            record[6].record()
        return gb, gi

    def reduce_grads(gb, gi_sum):
        # the data-parallel exchange: one all-reduce of the filter grads (outside any graph)
        if bucket is not None:
            bucket_params[0].grad = Wg
            bucket_params[1].grad = gb
            bucket_params[2].grad = gi_sum
            bucket.reduce()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(max(args.warmup, 3)):
        reduce_grads(*step(None))
    torch.cuda.synchronize()
    assert _lib.all_workspace_errors() == 0, "a device-side wait timed out during warm-up"

    # ---------------- per-phase CUDA-event timing (eager launches) ----------------
    KP = max(3, min(args.steps, 10))
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(7)] for _ in range(KP)]
    for i in range(KP):
        reduce_grads(*step(events[i]))
    torch.cuda.synchronize()
    phases = {"proj_scan_fwd": (0, 2), "scan_bwd": (3, 4), "gemm_bwd": (5, 6)}
    phase_ms = {n: statistics.mean(events[i][a].elapsed_time(events[i][b]) for i in range(KP))
                for n, (a, b) in phases.items()}

    # ---------------- the step's launches captured once as a CUDA graph ----------------
    # Same kernels, same work per step; replaying removes the host launch gaps between them. The
    # gradient all-reduce stays outside the graph (eager NCCL after each replay).
    graph, graph_note, graph_out = None, "captured", None
    try:
        cs = torch.cuda.Stream(device)
        cs.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cs):
            for _ in range(2):
                step(None)   # the capture stream's workspace exists before capture
        torch.cuda.current_stream().wait_stream(cs)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cs):
            graph_out = step(None)
        graph = g
    except Exception as exc:  # capture unsupported here: time the eager launches instead
        graph, graph_note = None, f"eager ({type(exc).__name__})"
        torch.cuda.synchronize()

    # With N > 1 each step's filter-grad all-reduce runs asynchronously and overlaps the next
    # step's kernels (as it would overlap the backward of the other layers in a model); the last
    # one is waited for inside the timed region.
    pending = [None]

    def timed_step():
        if graph is not None:
            graph.replay()
            gb_, gi_ = graph_out
        else:
            gb_, gi_ = step(None)
        if bucket is not None:
            if pending[0] is not None:
                pending[0].wait(copy_back=False)
            bucket_params[0].grad = Wg
            bucket_params[1].grad = gb_
            bucket_params[2].grad = gi_
            pending[0] = bucket.start()

    def drain():
        if pending[0] is not None:
            pending[0].wait(copy_back=False)
            pending[0] = None

    for _ in range(2):
        timed_step()
    drain()
    torch.cuda.synchronize()

    # ---------------- timed region (device-resident inputs) ----------------
    K = args.steps
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(gpu_id_for(local))
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    wall0 = time.time()
    start.record()
    for i in range(K):
        timed_step()
    drain()
    end.record()
    torch.cuda.synchronize()
    wall = time.time() - wall0
    barrier()
    clocks = sampler.stop()
    elapsed_ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([elapsed_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ms_per_step = elapsed_ms / K
    value = world * B * T / (ms_per_step / 1e3)
    assert _lib.all_workspace_errors() == 0, "a device-side wait timed out during the timed region"

    # ---------------- e2e through the public module API ----------------
    filt = nf.LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter(NH, NKVH, D, r).to(device)
    with torch.no_grad():
        filt.c.weight.copy_(W)
        filt.logit_bias.copy_(bias)
        filt.init_param.copy_(init)
    # the model-side exchange: the layer's all_reduce is started by its parameters' post-accumulate-grad
    # hooks inside the backward (LayerGradSync) and waited for at the end of the step
    e2e_sync = LayerGradSync([filt]) if world > 1 else None
    pin = {k: host[k].pin_memory() for k in ("x", "gq", "gk", "gv")}
    # two device copies of the step's inputs: the host->device copy of step i+1 (its own stream)
    # overlaps the compute of step i, as a prefetching data loader does; every step's copy is
    # still issued and completed inside the timed region
    dev_in = [{k: torch.empty_like(d[k]) for k in pin} for _ in range(2)]
    copy_stream = torch.cuda.Stream(device)
    copied = [torch.cuda.Event() for _ in range(2)]     # slot's inputs are on the device
    consumed = [torch.cuda.Event() for _ in range(2)]   # slot's previous step is done with them
    # the step's result read back: the layer's parameter gradients (dW fp32 [F, C], d logit_bias,
    # d init_param), what an optimizer step consumes; dx stays on the device for the layer below
    out_host = [torch.empty(p.shape, dtype=torch.float32).pin_memory()
                for p in (filt.c.weight, filt.logit_bias, filt.init_param)]
    h2d_bytes = sum(t.numel() * t.element_size() for t in pin.values())
    d2h_bytes = sum(t.numel() * t.element_size() for t in out_host)

    def issue_copy(slot):
        copy_stream.wait_event(consumed[slot])
        with torch.cuda.stream(copy_stream):
            for k2, src in pin.items():
                dev_in[slot][k2].copy_(src, non_blocking=True)
            copied[slot].record(copy_stream)

    def e2e_step(i, last):
        slot = i % 2
        if not last:
            issue_copy(1 - slot)  # the next step's inputs
        torch.cuda.current_stream(device).wait_event(copied[slot])
        dv = dev_in[slot]
        filt.zero_grad(set_to_none=True)
        xin = dv["x"].detach().requires_grad_(True)
        q, k, v = filt(xin, nf.LtvInitValues())
        torch.autograd.backward([q, k, v], [dv["gq"].transpose(1, 2), dv["gk"].transpose(1, 2),
                                            dv["gv"].transpose(1, 2)])
        if e2e_sync is not None:
            e2e_sync.wait()
        for dst, p in zip(out_host, (filt.c.weight, filt.logit_bias, filt.init_param)):
            dst.copy_(p.grad, non_blocking=True)  # the step's result, read back
        consumed[slot].record(torch.cuda.current_stream(device))

    def e2e_run(n):
        for slot in range(2):  # nothing in flight yet
            consumed[slot].record(torch.cuda.current_stream(device))
        issue_copy(0)
        for i in range(n):
            e2e_step(i, i == n - 1)

    e2e_run(max(args.warmup, 3))
    torch.cuda.synchronize()
    K2 = max(3, min(K, 20))
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    s2.record()
    e2e_run(K2)
    e2.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = s2.elapsed_time(e2)
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * B * T / (e2e_ms / K2 / 1e3)

    # ---------------- roofline of the dominant kernel and of the step ----------------
    peaks, peaks_src = load_peaks()
    sustained = elapsed_ms >= 1000.0
    tc_peak = peaks["bf16_tflops_sustained"] if sustained else peaks["bf16_tflops"]
    gemm_bwd_flops = 4.0 * B * T * C * F
    achieved = gemm_bwd_flops / (phase_ms["gemm_bwd"] / 1e3) / 1e12
    traffic = profile_traffic("gemm_bwd", args.config)
    step_flops = 6.0 * B * T * C * F
    esz = 2 if dt == torch.bfloat16 else 4
    step_bytes = float(B * T * (6 * C + 6 * H * D) * esz + F * C * esz)
    t_tc = step_flops / (tc_peak * 1e12)
    t_hbm = step_bytes / (peaks["hbm_gbs"] * 1e9)
    # per rank (weak scaling: every rank's step does the same work)
    step_frac = max(t_tc, t_hbm) / (ms_per_step / 1e3)

    result = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": UNIT,
        "n_gpus": world,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": cfg["dtype"],
        "data": "synthetic (seeded N(0,1) activations and upstream grads; value rows N(0,1/sqrt(C)), "
                f"decay rows N(0,{cfg.get('logit_std', 0.02)}), bias {cfg['bias']}; random-init weights)",
        "config": {
            "workload": f"{args.config}: {cfg['desc']}",
            "tokens_per_rank_per_step": B * T,
            "parallelism": f"dp{world} (batch-sharded; all_reduce of filter grads)" if world > 1 else "single GPU",
            "l2": "working set per step > 126 MB L2 (inputs larger than L2; no flush)",
            "launch": ("step replayed as one CUDA graph (same kernels; with N > 1 the filter-grad "
                       "all-reduce runs asynchronously after each replay, overlapping the next step); "
                       "phases_ms from eager launches with per-phase CUDA events"
                       if graph is not None else f"eager launches ({graph_note})"),
        },
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d_bytes,
                "d2h_bytes_per_step": d2h_bytes, "steps": K2,
                "path": "LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter forward + autograd backward",
                "h2d": "pinned host -> device on a copy stream, one step ahead (overlaps the previous step's "
                       "compute; every step's copy is inside the timed region)"},
        "gpu_launches": 4 * K,  # logit pre-pass, projection+scan, scan backward, projection backward
        "roofline": {"bound": "tensor", "kernel": "gemm_pair_kernel (projection backward: dW + dx, CTA pairs)",
                     "achieved": round(achieved, 1), "peak": tc_peak, "unit": "TFLOP/s",
                     "frac": round(achieved / tc_peak, 4),
                     "traffic": traffic,
                     "peak_source": f"{peaks_src} ({'sustained' if sustained else 'burst'})",
                     "algorithmic_flops_per_launch": gemm_bwd_flops},
        "step_roofline": {"frac": None if step_frac is None else round(step_frac, 4),
                          "bound": "tensor" if t_tc >= t_hbm else "hbm",
                          "t_tensor_us": round(t_tc * 1e6, 1), "t_hbm_us": round(t_hbm * 1e6, 1),
                          "flops_per_step": step_flops, "bytes_per_step": step_bytes},
        "phases_ms": {k: round(v, 4) for k, v in phase_ms.items()},
        "clocks": clocks,
        "wall_s_timed": round(wall, 3),
    }
    if world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(cfg, args.cpu_seconds)
    del graph, graph_out
    if world == 1:
        result["prologue"] = prologue_timing(cfg, d, W, bias, init, s, device)  # release the graph (and its memory pool) before the process group goes
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


# ------------------------------------------------------------------------------------------
# CPU baseline / reference arm: the reference's own CPU code for the path when its offline install
# (baseline/_ref) is present, else the oracle port of the same algorithm
# ------------------------------------------------------------------------------------------
REF_OPS = os.path.join(ROOT, "baseline", "_ref", "nanochat", "ops", "ltv_reference_ops.py")


def _oracle_sample(cfg, seqs, seed=7, T=None):
    import numpy as np

    rng = np.random.default_rng(seed)
    C, NH, NKVH, D, r = (cfg[k] for k in ("C", "NH", "NKVH", "D", "r"))
    T = cfg["T"] if T is None else T
    H, Da = NH + 2 * NKVH, D // r
    F = H * (D + Da)
    x = rng.standard_normal((seqs, T, C)).astype(np.float32)
    w = np.concatenate([rng.standard_normal((H, D, C)) / np.sqrt(C), rng.standard_normal((H, Da, C)) * _logit_std(cfg)],
                       axis=1).reshape(F, C).astype(np.float32)
    init = np.zeros((seqs, H, D), np.float32)
    bias = np.full((H, Da), float(cfg["bias"]), np.float32)
    gq = rng.standard_normal((seqs, NH, T, D)).astype(np.float32)
    gk = rng.standard_normal((seqs, NKVH, T, D)).astype(np.float32)
    gv = rng.standard_normal((seqs, NKVH, T, D)).astype(np.float32)
    return x, w, init, bias, gq, gk, gv, NH, NKVH, Da, r


def _reference_ops():
    """The reference's CPU implementation of the path, `nanochat/ops/ltv_reference_ops.py` of the
    offline install in baseline/_ref (it imports only torch), loaded by file path so that the
    package's other modules (GPU extensions, Metal, Triton) are not imported. None when absent."""
    if not os.path.exists(REF_OPS):
        return None
    import importlib.util

    spec = importlib.util.spec_from_file_location("_nanochat_ltv_reference_ops", REF_OPS)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class _RefLayer:
    """One layer step through the reference's own CPU code: `fused_linear_transpose_reference`
    (x @ W^T -> [B, F, T]), `ltv_fused_concat_head_major_register_cast_blelloch_scan_reference` on
    its [B, T, F] view (the per-token QuantizedStateUpdate loop), then autograd back to x, the fp32
    master W, logit_bias and the initial state — the composition the reference filter runs
    (nanochat/ltv_cuda_fused_concat_head_major_register_cast_blelloch_scan_qkv_filter.py:24-73)."""

    def __init__(self, R, cfg, tokens):
        import torch

        self.R, self.torch = R, torch
        x, w, init, bias, gq, gk, gv, NH, NKVH, Da, r = _oracle_sample(cfg, 1, T=tokens)
        dt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float32
        self.dt, self.meta = dt, (NH, NKVH, Da, r)
        self.x = torch.from_numpy(x).to(dt)
        self.w = torch.from_numpy(w)
        self.init, self.bias = torch.from_numpy(init), torch.from_numpy(bias)
        self.grads = [torch.from_numpy(g).to(dt) for g in (gq, gk, gv)]
        self.tokens = tokens

    def step(self):
        torch, R = self.torch, self.R
        NH, NKVH, Da, r = self.meta
        x = self.x.detach().requires_grad_()
        w = self.w.detach().requires_grad_()
        init = self.init.detach().requires_grad_()
        bias = self.bias.detach().requires_grad_()
        combined = R.fused_linear_transpose_reference(x, w.to(self.dt))
        q, k, v = R.ltv_fused_concat_head_major_register_cast_blelloch_scan_reference(
            combined.transpose(1, 2), init.to(self.dt), bias, NH, NKVH, Da, r, 8, 8, 4, 32, 2, 8, True)
        torch.autograd.backward([q, k, v], self.grads)
        return w.grad


def _ref_tokens_for(R, cfg, seconds_per_step):
    """Tokens of one sequence per step so that a step of the reference's code takes at most about
    `seconds_per_step`: from 64 tokens, doubled while the next size's estimated time fits (at most
    the config's T). Its backward costs more per token as the sequence grows (each token's output
    is an in-place slice write whose backward passes the whole gradient buffer), so the estimate
    for the next size is 2.6x the measured time and a shorter sample favours the reference."""
    tokens = 64
    layer = _RefLayer(R, cfg, tokens)
    layer.step()  # first call: allocator and thread-pool warm-up
    while True:
        t0 = time.perf_counter()
        layer.step()
        dt = time.perf_counter() - t0
        if 2 * tokens > cfg["T"] or 2.6 * dt > seconds_per_step:
            return tokens
        tokens *= 2
        layer = _RefLayer(R, cfg, tokens)


def _ref_sample_desc(tokens, cfg, runs):
    return (f"1 sequence x {tokens} tokens per run of {cfg['desc']}; the reference's own CPU code: "
            "nanochat/ops/ltv_reference_ops.py from the offline install in baseline/_ref "
            "(fused_linear_transpose_reference, the blelloch_scan_reference token loop, autograd "
            f"backward through QuantizedStateUpdate), median of {runs} runs")


def _port_seconds(cfg, seqs, runs_max, seconds):
    from oracle import oracle as O

    O.build()
    cores = O.set_threads(os.cpu_count() or 1)  # every host core, whatever the launcher set
    sample = _oracle_sample(cfg, seqs)
    bf16 = cfg["dtype"] == "bf16"
    O.layer_fwd_bwd(*sample, bf16=bf16)  # warm-up (thread pool, page faults)
    times = []
    t_all = time.perf_counter()
    while len(times) < runs_max and (time.perf_counter() - t_all < seconds or len(times) < 1):
        t0 = time.perf_counter()
        O.layer_fwd_bwd(*sample, bf16=bf16)
        times.append(time.perf_counter() - t0)
    return times, cores


def cpu_baseline(cfg, seconds=10.0, seqs=1):
    """The path on the host cores, over a bounded sample: the reference's own CPU code when
    baseline/_ref holds it (kind "reference"), else the oracle port (C, OpenMP over all host
    cores; kind "port"). The port's rate is reported beside the reference's as `port_value`."""
    times, cores = _port_seconds(cfg, seqs, 8, seconds)
    port_value = round(seqs * cfg["T"] / statistics.median(times), 2)
    port_desc = (f"{seqs} sequence(s) x {cfg['T']} tokens of {cfg['desc']}; oracle port of the "
                 f"reference's CPU algorithm (oracle/ltv_oracle.c scan, float64 BLAS GEMMs), "
                 f"median of {len(times)} runs")
    R = _reference_ops()
    if R is None:
        return {"value": port_value, "unit": UNIT, "cores": cores, "kind": "port", "sample": port_desc}
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    tokens = _ref_tokens_for(R, cfg, seconds / 3)
    layer = _RefLayer(R, cfg, tokens)
    rt = []
    for _ in range(3):
        t0 = time.perf_counter()
        layer.step()
        rt.append(time.perf_counter() - t0)
    return {"value": round(tokens / statistics.median(rt), 2), "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "reference", "sample": _ref_sample_desc(tokens, cfg, len(rt)),
            "port_value": port_value, "port_sample": port_desc}


def run_reference(args, cfg):
    """`--impl reference`: the reference's own CPU code for the path (baseline/_ref), each step one
    sequence of a bounded token count, so that K steps end within a few minutes; rank 0 only.
    Without the install, the oracle port of the same algorithm, one full sequence per step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    n = int(os.environ.get("WORLD_SIZE", "1"))
    R = _reference_ops()
    if R is not None:
        import torch

        torch.set_num_threads(os.cpu_count() or 1)  # all host threads (torchrun sets OMP_NUM_THREADS=1)
        cores = torch.get_num_threads()
        tokens = _ref_tokens_for(R, cfg, min(6.0, 120.0 / max(1, args.steps)))
        layer = _RefLayer(R, cfg, tokens)
        for _ in range(max(1, min(args.warmup, 1))):
            layer.step()
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            layer.step()
            times.append(time.perf_counter() - t0)
        kind, sample_desc = "reference", _ref_sample_desc(tokens, cfg, args.steps).replace(
            f", median of {args.steps} runs", f", {args.steps} timed steps")
    else:
        from oracle import oracle as O

        O.build()
        cores = O.set_threads(os.cpu_count() or 1)
        tokens = cfg["T"]
        sample = _oracle_sample(cfg, 1)
        bf16 = cfg["dtype"] == "bf16"
        for _ in range(max(1, min(args.warmup, 2))):
            O.layer_fwd_bwd(*sample, bf16=bf16)
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            O.layer_fwd_bwd(*sample, bf16=bf16)
            times.append(time.perf_counter() - t0)
        kind = "port"
        sample_desc = (f"1 sequence x {tokens} tokens per step of {cfg['desc']}; oracle port of the "
                       "reference's CPU algorithm (C scan, float64 BLAS GEMMs): the reference's install "
                       "(baseline/_ref) is absent")
    total = sum(times)
    value = args.steps * tokens / total
    print(json.dumps({
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": n, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 * total / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": cfg["dtype"], "data": "synthetic",
        "config": {"workload": f"{args.config}: {cfg['desc']}", "tokens_per_step": tokens},
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": sample_desc},
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_decode(args):
    """Benchmark config 4, kernel level: the filter-state decode update of a d=12 model (12 layers,
    C=768, 6+6+6 heads x 128, batch 64, bf16) for 256 token steps — one `ltv_decode_step` launch
    per layer-step (projection of the new token, gate, recurrence step), replayed as a CUDA graph
    per token step, updating the cache's states in place. Attention, MLP and the prompt prefill
    are outside the path; the layer inputs
    are synthetic N(0, 1) activations, weights N(0, 0.02)."""
    import torch

    import nanochat_filter_b200 as nf
    from nanochat_filter_b200 import _lib

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    _lib.load()
    L, Bd, C, NH, NKVH, D, r, steps = 12, 64, 768, 6, 6, 128, 128, 256
    H, Da = NH + 2 * NKVH, D // r
    F = H * (D + Da)
    g = torch.Generator(device="cpu").manual_seed(4)
    W = [(torch.randn(F, C, generator=g) * 0.02).to(device, torch.bfloat16) for _ in range(L)]
    bias = [torch.zeros(H, Da, device=device) for _ in range(L)]
    init = [torch.zeros(H, D, device=device, dtype=torch.bfloat16) for _ in range(L)]
    xs = (torch.randn(L, Bd, C, generator=g)).to(device, torch.bfloat16)
    state = [[torch.zeros(Bd, n, D, device=device, dtype=torch.bfloat16) for n in (NH, NKVH, NKVH)] for _ in range(L)]

    op = torch.ops.nanochat_cuda.ltv_decode_step_

    def token_step():
        for l in range(L):  # the cache's states updated in place: one launch per layer-step
            op(xs[l], W[l], bias[l], state[l][0], state[l][1], state[l][2], NH, NKVH, Da, r, True)

    for _ in range(3):
        token_step()
    torch.cuda.synchronize()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side), torch.cuda.graph(graph, stream=side):
        token_step()
    torch.cuda.current_stream(device).wait_stream(side)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    us_layer_step = ms * 1e3 / (steps * L)
    peaks, src = load_peaks()
    layer_bytes = F * C * 2 + Bd * H * D * 2 * 2 + Bd * C * 2  # weights, state read + write, token
    achieved = layer_bytes / (us_layer_step * 1e-6) / 1e9
    print(json.dumps({
        "metric": "filter decode update tokens/s", "value": round(Bd * steps / (ms / 1e3), 1), "unit": "tokens/s",
        "n_gpus": 1, "steps": steps, "warmup": 3, "ms_per_step": round(ms / steps, 4), "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic (N(0,1) layer inputs, N(0,0.02) weights)",
        "config": {"workload": "config4 (kernel level): d=12, 12 layers, C=768, 6+6+6 heads x 128, batch 64, "
                               "256 token steps of the filter-state update", "launch": "one CUDA graph per token step"},
        "us_per_layer_step": round(us_layer_step, 3),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "bytes_per_layer_step": layer_bytes,
                     "peak_source": src,
                     "note": "the 12 layers' weights (43 MB) stay in L2 across token steps"},
        "gpu_launches": steps * L,
    }))
    del graph


def run_lookback(args):
    """The look-back (chunk-restarting) scan, forward + backward, kernel level (f1): config 2's
    shape (B=32, T=1024, 6+6+6 heads x 128, r=128, bf16) with the reference's chunking
    (P, Q, K) = (128, 112, 17) — the first 128 tokens as one chunk, then 112-token chunks each
    restarted 16 tokens back. The scan's input `combined` is the projection buffer's [B, T, F]
    view, as the look-back filter passes it. Replayed as one CUDA graph per step."""
    import torch

    from nanochat_filter_b200 import _lib

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    _lib.load()
    B, T, NH, NKVH, D, r, P, Q, K = 32, 1024, 6, 6, 128, 128, 128, 112, 17
    H, Da = NH + 2 * NKVH, D // r
    F = H * (D + Da)
    g = torch.Generator(device="cpu").manual_seed(5)
    comb = torch.randn(B, F, T, generator=g).to(device, torch.bfloat16)
    combined = comb.transpose(1, 2)
    inits = torch.zeros(B, H, D, device=device, dtype=torch.bfloat16)
    bias = torch.zeros(H, Da, device=device)
    grads = [torch.randn(B, n, T, D, generator=g).to(device, torch.bfloat16) for n in (NH, NKVH, NKVH)]
    outs = [torch.empty(B, n, T, D, device=device, dtype=torch.bfloat16) for n in (NH, NKVH, NKVH)]
    gc = torch.empty_like(combined)
    gi = torch.empty_like(inits)
    gb = torch.empty_like(bias)
    name = "ltv_look_back_fused_concat_head_major_register_cast_blelloch_scan_cuda_{}"
    fwd = getattr(torch.ops.nanochat_cuda, name.format("forward_kernel"))
    bwd = getattr(torch.ops.nanochat_cuda, name.format("backward_kernel"))

    def step():
        fwd(combined, inits, bias, *outs, B, T, NH, NKVH, Da, r, P, Q, K, 8, 8, 4, True)
        gb.zero_()
        bwd(combined, inits, bias, *outs, *grads, gc, gi, gb, NH, NKVH, Da, r, P, Q, K, 32, 2, 8, True)

    def fwd_only():
        fwd(combined, inits, bias, *outs, B, T, NH, NKVH, Da, r, P, Q, K, 8, 8, 4, True)

    steps = max(1, args.steps)
    us = _graph_us(step, device, reps=steps)
    fwd_us = _graph_us(fwd_only, device, reps=steps)
    nch = 1 + (T - P + Q - 1) // Q
    # bytes per step: forward reads combined and writes q/k/v; backward reads combined, the outputs
    # and their gradients, and writes grad_combined (the warm-up prefixes re-read combined from L2)
    step_bytes = 2 * (B * T * F) * 2 + 3 * (B * T * H * D) * 2 + B * T * F * 2
    peaks, src = load_peaks()
    achieved = step_bytes / (us * 1e-6) / 1e9
    print(json.dumps({
        "metric": "look-back scan fwd+bwd tokens/s", "value": round(B * T / (us * 1e-6), 1), "unit": "tokens/s",
        "n_gpus": 1, "steps": steps, "warmup": 3, "ms_per_step": round(us / 1e3, 4), "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic (N(0,1) projection buffer and upstream gradients)",
        "config": {"workload": f"look-back scan (kernel level): B={B}, T={T}, 6+6+6 heads x 128, r=128, "
                               f"(P, Q, K) = ({P}, {Q}, {K}): {nch} chunks per row",
                   "launch": "one CUDA graph per step: forward kernel, bias-gradient zero fill, chunk-parallel "
                             "backward kernel, overlap fix-up kernel, logit-bias reduction"},
        "forward_us": round(fwd_us, 1), "backward_us": round(us - fwd_us, 1),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "bytes_per_step": step_bytes,
                     "peak_source": src},
        "gpu_launches": 4 * steps,
    }))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS) + ["decode", "lookback"], default="config2",
                    help="config2 (default), config1/config3, decode (config 4, kernel level) or lookback "
                         "(the look-back scan at config 2's shape, kernel level)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--batch", type=int, default=0,
                    help="override the config's sequences per rank (small profiling cases; not a bench line)")
    args = ap.parse_args()
    if args.config == "decode":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "config 4 is measured at kernel level only "
                              "(the reference's decode runs inside its GPT model, which is outside the path)"}))
            return
        run_decode(args)
        return
    if args.config == "lookback":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the look-back scan is measured at kernel level only "
                              "(the reference's CPU code for it is the same token loop as the main path's)"}))
            return
        run_lookback(args)
        return
    cfg = dict(CONFIGS[args.config])
    if args.batch:
        cfg["B"] = args.batch
        cfg["desc"] += f" [B overridden to {args.batch}: a profiling case, not the benchmark config]"
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
