"""One process driving two GPUs: every tcgen05 kernel runs on the second device as well.

Kernel function attributes (the dynamic shared-memory limit above 48 KB) belong to each device's
context, so a library that set them only on the first device it saw would fail its first
large-shared-memory launch on any other device of the same process.  Each op here runs through
the C ABI on device 0 and then on device 1 with the same inputs, and the outputs must be bit for
bit equal (same kernels, same arithmetic).  Skipped with fewer than two visible GPUs."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ops(lc, torch, dev):
    """Runs the op set on `dev` with seeded inputs; returns the outputs as host arrays."""
    L = lc.lib
    p = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    g = torch.Generator(device="cpu").manual_seed(11)
    outs = {}
    with torch.cuda.device(dev):
        sp = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        # bf16 attention: causal (one-tile kernel) and non-causal head_dim 128 (two-tile kernel).
        q, k, v = (torch.randn((4, 384, 128), generator=g).to(torch.bfloat16).to(dev) for _ in range(3))
        for causal in (1, 0):
            o = torch.empty_like(q)
            lc.check(L.lcAttentionForward(p(q), p(k), p(v), p(o), 4, 384, 128, causal, lc.BF16, None, sp), "attn")
            outs[f"attn_bf16_{causal}"] = o
        # bf16 GEMMs: 2048^3 (2-SM kernel, 64 tiles of 256x256) and 512^3 (1-SM kernel).
        for n in (2048, 512):
            a = ((torch.rand((n, n), generator=g) * 2 - 1) / n ** 0.5).to(torch.bfloat16).to(dev)
            b = (torch.rand((n, n), generator=g) * 2 - 1).to(torch.bfloat16).to(dev)
            c = torch.empty((n, n), dtype=torch.bfloat16, device=dev)
            lc.check(L.lcMatMul(p(a), p(b), p(c), n, n, n, lc.BF16, None, sp), "gemm bf16")
            outs[f"gemm_bf16_{n}"] = c
        # fp32 GEMM 1024^3 (3xTF32 on CTA pairs) and fp32 attention head_dim 64 (3xTF32 kernel).
        a = torch.rand((1024, 1024), generator=g).to(dev) * 2 - 1
        b = torch.rand((1024, 1024), generator=g).to(dev) * 2 - 1
        c = torch.empty_like(a)
        lc.check(L.lcMatMul(p(a), p(b), p(c), 1024, 1024, 1024, lc.F32, None, sp), "gemm f32")
        outs["gemm_f32"] = c
        q, k, v = (torch.randn((2, 500, 64), generator=g).to(dev) for _ in range(3))
        o = torch.empty_like(q)
        lc.check(L.lcAttentionForward(p(q), p(k), p(v), p(o), 2, 500, 64, 0, lc.F32, None, sp), "attn f32")
        outs["attn_f32"] = o
        # fp32 conv 3x3 large enough for the implicit tensor-core conv.
        x = torch.randn((4, 64, 56, 56), generator=g).to(dev)
        w = ((torch.rand((192, 64, 3, 3), generator=g) * 2 - 1) * 0.06).to(dev)
        bias = torch.zeros(192, device=dev)
        y = torch.empty((4, 192, 56, 56), device=dev)
        lc.check(L.lcConv2dNchw(p(x), p(w), p(bias), p(y), 4, 64, 56, 56, 192, 3, 3, 1, 1, 1, 1, 1, None, sp),
                 "conv")
        outs["conv"] = y
        torch.cuda.synchronize(dev)
        err = C.c_uint(0)
        lc.check(L.lcGetDeviceErrorWord(C.byref(err)), "error word")
        assert err.value == 0
    return {name: t.float().cpu().numpy() for name, t in outs.items()}


def test_every_tc_kernel_runs_on_a_second_device(gpu):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two visible GPUs")
    first = _ops(gpu, torch, 0)
    second = _ops(gpu, torch, 1)
    for name, want in first.items():
        got = second[name]
        assert np.isfinite(got).all(), name
        assert np.array_equal(want, got), name
