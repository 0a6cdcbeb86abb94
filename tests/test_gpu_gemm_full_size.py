"""The persistent GEMMs at the sizes the benchmark times, checked against the oracle.

Every tcgen05 GEMM is persistent: one CTA (or CTA pair) walks many output tiles, switching TMEM
accumulator buffers and mbarrier phases per tile and walking the grouped tile order.  These tests
give each CTA several tiles -- BASELINE config 4's bf16 sizes (4096^3, 8192^3, 16384^3 and
16384x4096x1024) and the fp32 3xTF32 sizes 2048^3 and 4096x1024x4096 -- through the default
dispatch and forced onto every tensor-core kernel that takes the shape.

Checks (the oracle protocol for large shapes: whole row blocks against the reference CPU loop):
  * three 128-row blocks (first, middle, last) against the oracle matmul of the same bf16-rounded
    inputs (reference src/ops/matmul_cpu.cpp:49-60), bf16 tolerance 2e-3 + 2e-2|ref|;
  * the whole output against a float32 matmul of the same inputs computed on the device (every
    tile of every CTA), same tolerance.
fp32: sampled rows at |err| <= 1e-4 + 1e-4|ref| against the oracle.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import close_enough
from oracle import oracle as O

pytestmark = pytest.mark.gpu
P = O.port()
BF16_TOL = (2e-3, 2e-2)
F32_TOL = (1e-4, 1e-4)


def _blocks(m, rows=128):
    mid = (m // 2) // rows * rows
    return [(0, rows), (mid, mid + rows), (m - rows, m)]


def _run(gpu, torch, a, b, c, m, k, n, dtype):
    gpu.check(gpu.lib.lcMatMul(C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()), C.c_void_p(c.data_ptr()), m, k,
                               n, dtype, None, None), "lcMatMul")
    torch.cuda.synchronize()


@pytest.mark.parametrize("kernel", ["default", "tcgen05_128x256", "tcgen05_2sm_256x256"])
@pytest.mark.parametrize("m,k,n", [(8192, 8192, 8192), (4096, 4096, 4096), (16384, 1024, 4096),
                                   (16384, 16384, 16384)])
def test_matmul_bf16_config4(gpu, kernel, m, k, n):
    import torch

    if m == 16384 and k == 16384 and kernel == "tcgen05_128x256":
        pytest.skip("16384^3 runs the 2-SM kernel by default; the 1-SM kernel is covered at the other sizes")
    g = torch.Generator(device="cuda").manual_seed(3)
    a = ((torch.rand((m, k), generator=g, device="cuda") * 2 - 1) / k ** 0.5).to(torch.bfloat16)
    b = ((torch.rand((k, n), generator=g, device="cuda") * 2 - 1) / k ** 0.5).to(torch.bfloat16)
    c = torch.full((m, n), float("nan"), device="cuda", dtype=torch.bfloat16)
    if kernel != "default":
        gpu.tune_cache_set(gpu.TUNE_MATMUL, m, k, n, kernel, gpu.BF16)
    try:
        _run(gpu, torch, a, b, c, m, k, n, gpu.BF16)
    finally:
        gpu.tune_cache_reset()
    # every tile: against a float32 product of the same bf16 inputs on the device, in row slabs
    slab = 2048
    bf = b.float()
    for r0 in range(0, m, slab):
        ref = a[r0:r0 + slab].float() @ bf
        err = (c[r0:r0 + slab].float() - ref).abs()
        bad = err > BF16_TOL[0] + BF16_TOL[1] * ref.abs()
        assert not bool(bad.any()), f"rows {r0}+: {int(bad.sum())} bad, max err {float(err.max()):.3g}"
    del bf
    # sampled row blocks: against the oracle (the reference CPU loop) on the host
    bh = b.float().cpu().numpy()
    for r0, r1 in _blocks(m):
        ah = np.ascontiguousarray(a[r0:r1].float().cpu().numpy())
        close_enough(P.matmul(ah, bh, threads=8), c[r0:r1].float().cpu().numpy(), *BF16_TOL)


@pytest.mark.parametrize("kernel", ["default", "tcgen05_3xtf32"])
@pytest.mark.parametrize("m,k,n", [(2048, 2048, 2048), (4096, 1024, 4096)])
def test_matmul_f32_multi_tile(gpu, kernel, m, k, n):
    """Strict fp32 at sizes that give each persistent 3xTF32 CTA three or more tiles."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(1)
    a = torch.rand((m, k), generator=g, device="cuda") * 2 - 1
    b = torch.rand((k, n), generator=g, device="cuda") * 2 - 1
    c = torch.full((m, n), float("nan"), device="cuda")
    if kernel != "default":
        gpu.tune_cache_set(gpu.TUNE_MATMUL, m, k, n, kernel, gpu.F32)
    try:
        _run(gpu, torch, a, b, c, m, k, n, gpu.F32)
    finally:
        gpu.tune_cache_reset()
    assert bool(torch.isfinite(c).all())
    bh = b.cpu().numpy()
    rows = np.unique(np.concatenate([np.arange(0, 64), np.linspace(0, m - 1, 192).astype(int),
                                     np.arange(m - 64, m)]))
    ah = np.ascontiguousarray(a.cpu().numpy()[rows])
    close_enough(P.matmul(ah, bh, threads=8), c.cpu().numpy()[rows], *F32_TOL)


def test_conv_attention_config5_all_images(gpu):
    """Config 5 at its full 32 images (the batch the benchmark times: ~10 conv tiles per CTA),
    images 0, 15 and 31 checked against the reference-batch oracle."""
    import torch

    rng = np.random.default_rng(4)
    x = rng.standard_normal((32, 64, 56, 56)).astype(np.float32)
    w = rng.uniform(-np.sqrt(6 / 576), np.sqrt(6 / 576), (192, 64, 3, 3)).astype(np.float32)
    bias = np.zeros(192, np.float32)
    pw = np.random.default_rng(5).uniform(-np.sqrt(6 / 64), np.sqrt(6 / 64), (64, 64)).astype(np.float32)
    dx, dw, db, dp = (torch.from_numpy(t).cuda() for t in (x, w, bias, pw))
    out = torch.full((32, 3136, 64), float("nan"), device="cuda")
    ptr = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    gpu.check(gpu.lib.lcConvAttentionNchw(ptr(dx), ptr(dw), ptr(db), ptr(dp), ptr(out), 32, 64, 56, 56, 192, 3, 3,
                                          1, 1, 1, 1, 3136, 64, 64, 1, None, None), "lcConvAttentionNchw")
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    pick = [0, 15, 31]
    ref = P.conv_attention_images(np.ascontiguousarray(x[pick]), w, bias, pw, 3136, 64, threads=3)
    close_enough(ref, got[pick], *F32_TOL)


@pytest.mark.parametrize("m,k,n", [(512, 4096, 512), (512, 1188, 520), (300, 2052, 260)])
def test_matmul_f32_split_k(gpu, m, k, n):
    """Shapes whose 256x64 pair tiles fill under half of the SM pairs, so K is split across pairs
    (uneven last split, ragged M and N edges): the split partial sums are added by whichever split
    finishes last, in split order.  Every row against the oracle at 1e-4 + 1e-4|ref|."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(11)
    a = torch.rand((m, k), generator=g, device="cuda") * 2 - 1
    b = torch.rand((k, n), generator=g, device="cuda") * 2 - 1
    c = torch.full((m, n), float("nan"), device="cuda")
    outs = []
    for _ in range(2):  # the same bits on a repeat: the split order fixes the summation order
        _run(gpu, torch, a, b, c, m, k, n, gpu.F32)
        outs.append(c.cpu().numpy().copy())
    assert np.array_equal(outs[0], outs[1])
    close_enough(P.matmul(a.cpu().numpy(), b.cpu().numpy(), threads=8), outs[0], *F32_TOL)
