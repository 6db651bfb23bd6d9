"""Stream ordering of the device-pointer path.

The staging, range-fixup and attention kernels are launched as programmatic
dependents: each may start while the kernel before it on the stream is
finishing, and every thread waits (griddepcontrol.wait) before its first
global-memory access. Chained calls on one stream, each reading the previous
call's output -- directly or through a torch kernel in between -- must
therefore give exactly what the same calls give with a device synchronise
between them.
"""
from __future__ import annotations

import math

import pytest

pytestmark = pytest.mark.gpu


def _inputs(cuda_device, B, S, Hq, Hk, D, dtype, seed):
    import torch

    g = torch.Generator(device=cuda_device).manual_seed(seed)
    q = torch.randn((B, S, Hq, D), generator=g, device=cuda_device).to(dtype)
    k = torch.randn((B, S, Hk, D), generator=g, device=cuda_device).to(dtype)
    v = torch.randn((B, S, Hk, D), generator=g, device=cuda_device).to(dtype)
    return q, k, v


@pytest.mark.parametrize("dtype_name,theta,D", [("bfloat16", 1e4, 128), ("float16", None, 128), ("float16", 1e4, 64)])
def test_chained_calls_without_sync(fa, cuda_device, dtype_name, theta, D):
    import torch

    dtype = getattr(torch, dtype_name)
    B, S, Hq, Hk = 2, 1000, 4, 2
    q, k, v = _inputs(cuda_device, B, S, Hq, Hk, D, dtype, seed=31)
    kw = dict(softmax_scale=1 / math.sqrt(D), is_causal=True, rope_theta=theta)

    def chain(sync):
        x = q
        outs = []
        for i in range(4):
            o = fa.forward(x, k, v, **kw)        # output in Q's dtype and shape
            if sync:
                torch.cuda.synchronize()
            outs.append(o)
            # the next call reads this output, directly or through a torch kernel
            x = o if i % 2 == 0 else (o * 3.0 + 0.25).to(dtype)
            if sync:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        fa.check_status()
        return outs

    ref = chain(sync=True)
    got = chain(sync=False)
    for i, (a, b) in enumerate(zip(ref, got)):
        assert torch.equal(a, b), f"call {i} differs without synchronisation"


def test_output_overwritten_by_next_call(fa, cuda_device):
    """A call whose output buffer the previous call's output was read from:
    the second call must not write O before the torch kernel reading the
    first result has finished."""
    import torch

    B, S, Hq, Hk, D = 1, 2048, 8, 2, 128
    q, k, v = _inputs(cuda_device, B, S, Hq, Hk, D, torch.bfloat16, seed=32)
    kw = dict(softmax_scale=1 / math.sqrt(D), is_causal=True, rope_theta=5e5)
    out = torch.empty_like(q)
    fa.forward(q, k, v, out=out, **kw)
    first = out.float().sum(dim=(1, 3))      # torch kernels reading `out` ...
    fa.forward(k.repeat_interleave(4, dim=2), k, v, out=out, **kw)  # ... then the next call overwrites it
    torch.cuda.synchronize()
    fa.check_status()
    out_ref = torch.empty_like(q)
    fa.forward(q, k, v, out=out_ref, **kw)
    torch.cuda.synchronize()
    assert torch.equal(first, out_ref.float().sum(dim=(1, 3)))
