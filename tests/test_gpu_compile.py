"""torch.compile(fullgraph=True) of the filter, forward and backward.

The reference compiles its model with torch.compile (scripts/base_train.py:468-470), which traces
the filter's operators through their fake (meta) kernels (nanochat/ops/ltv_cuda_meta.py:155-258)
and AOTAutograd traces their registered backward formulas. Here the filter's forward and backward
are compiled with fullgraph=True (any graph break raises) on the one-kernel shape (projection +
scan with state checkpoints, checkpoint backward, batch-shared initial state) and on a shape that
takes the two-operator path, and the compiled results must equal eager's (same kernels, so equal
to the bit). The same holds for the forward with the attention's q / k prologue folded in
(`forward_rotary_norm`, nanochat/gpt.py:224-230).
"""

from __future__ import annotations

import pytest
import torch

from nanochat_filter_b200 import LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter, LtvInitValues

pytestmark = pytest.mark.gpu


def _run(fn, f, x, grads):
    q, k, v = fn(x)
    torch.autograd.backward([q, k, v], list(grads))
    return [t.detach().clone() for t in (q, k, v, x.grad, f.c.weight.grad, f.logit_bias.grad, f.init_param.grad)]


@pytest.mark.parametrize("rope", [False, True])
@pytest.mark.parametrize("backend", ["aot_eager", "inductor"])
@pytest.mark.parametrize("B,T,C", [(32, 64, 128), (2, 96, 256)])
def test_filter_compiles_fullgraph_and_matches_eager(cuda_device, backend, B, T, C, rope):
    dev = cuda_device
    NH, NKVH, D, r = 6, 6, 128, 128
    torch.manual_seed(0)
    f = LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter(NH, NKVH, D, r)
    f.c = torch.nn.Linear(C, f.c.out_features, bias=False)  # model width C
    f.init_weights(alpha_mlp_bias_init=-1.0, weight_s=0.05, bias_s=0.5, init_s=0.5)
    f = f.to(dev)
    g = torch.Generator(device=dev).manual_seed(1)
    x0 = torch.randn(B, T, C, device=dev, generator=g).to(torch.bfloat16)
    grads = [torch.randn(B, T, n, D, device=dev, generator=g).to(torch.bfloat16) for n in (NH, NKVH, NKVH)]

    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, dtype=torch.float32, device=dev) / D))
    fr = torch.outer(torch.arange(T, dtype=torch.float32, device=dev), inv)
    cs = (fr.cos().bfloat16()[None, :, None, :], fr.sin().bfloat16()[None, :, None, :])

    def fn(x):
        return f.forward_rotary_norm(x, LtvInitValues(), cs) if rope else f(x, LtvInitValues())

    x = x0.clone().requires_grad_(True)
    eager = _run(fn, f, x, grads)
    f.zero_grad(set_to_none=True)

    torch._dynamo.reset()
    cfn = torch.compile(fn, fullgraph=True, backend=backend)
    xc = x0.clone().requires_grad_(True)
    comp = _run(cfn, f, xc, grads)
    torch.cuda.synchronize()
    names = ("q", "k", "v", "dx", "dW", "dbias", "dinit")
    for n, a, e in zip(names, comp, eager):
        assert a.shape == e.shape and a.dtype == e.dtype, n
        assert torch.equal(a, e), f"{n}: compiled differs from eager (max {(a.float() - e.float()).abs().max()})"
