"""CUDA path vs the oracle: every op through the C ABI (liblc_b200.so), on a B200.

Tolerances (north star): fp32 paths |err| <= 1e-4 + 1e-4|ref|; bf16 paths 2e-2 relative (plus a
small absolute floor for values near zero, stated per test)."""
import ctypes as C

import numpy as np
import pytest

from conftest import close_enough, golden
from oracle import oracle as O

pytestmark = pytest.mark.gpu
F32_TOL = (1e-4, 1e-4)
P = O.port()


def bf(lc, x):
    return lc.to_bf16(x)


# ---------------------------------------------------------------- attention fp32
def test_attention_kats(gpu):
    g = golden("kat_attn")
    out = gpu.attention2d(g["q"], g["k"], g["v"])
    close_enough([[6.6976, 6.6048], [3.3024, 13.3952]], out, 0.05, 0)
    close_enough(g["out"], out, *F32_TOL)
    g = golden("kat_attn_post")
    pol = gpu.default_attention_policy()
    pol.output_scale, pol.output_bias, pol.output_relu = 0.5, -2.0, 1
    close_enough(g["out"], gpu.attention2d(g["q"], g["k"], g["v"], policy=pol), *F32_TOL)


@pytest.mark.parametrize("name", ["parity_attention", "cfg1_attention_256x64"])
def test_attention_golden(gpu, name):
    g = golden(name)
    close_enough(g["out"], gpu.attention2d(g["q"], g["k"], g["v"]), *F32_TOL)


@pytest.mark.parametrize("s,d,causal", [(1, 8, 0), (17, 64, 1), (63, 32, 0), (65, 128, 1), (200, 100, 1),
                                        (129, 256, 0), (300, 64, 1), (1000, 128, 0)])
def test_attention_f32_shapes(gpu, s, d, causal):
    rng = np.random.default_rng(s * 1000 + d)
    q, k, v = (rng.standard_normal((s, d)).astype(np.float32) for _ in range(3))
    close_enough(P.attention(q, k, v, causal), gpu.attention2d(q, k, v, causal=bool(causal)), *F32_TOL)


def test_attention_f32_batched_units(gpu):
    rng = np.random.default_rng(5)
    q, k, v = (rng.standard_normal((6, 130, 64)).astype(np.float32) for _ in range(3))
    for causal in (False, True):
        close_enough(P.attention_units(q, k, v, causal), gpu.attention_batched(q, k, v, causal), *F32_TOL)


# ---------------------------------------------------------------- attention bf16
def test_attention_bf16_golden(gpu):
    g = golden("cfg3_causal_bf16in_2x200x128")
    out = gpu.attention_batched(bf(gpu, g["q"]), bf(gpu, g["k"]), bf(gpu, g["v"]), True, gpu.BF16)
    close_enough(g["out"], gpu.from_bf16(out), 2e-2, 2e-2)


@pytest.mark.parametrize("units,s,d,causal", [(3, 128, 128, 1), (2, 257, 128, 1), (2, 300, 64, 0), (1, 77, 64, 1),
                                              (2, 1024, 128, 1), (2, 96, 48, 0)])
def test_attention_bf16_shapes(gpu, units, s, d, causal):
    rng = np.random.default_rng(units + s + d)
    q, k, v = (P.bf16_round(rng.standard_normal((units, s, d)).astype(np.float32)) for _ in range(3))
    ref = P.attention_units(q, k, v, causal)
    out = gpu.attention_batched(bf(gpu, q), bf(gpu, k), bf(gpu, v), bool(causal), gpu.BF16)
    close_enough(ref, gpu.from_bf16(out), 2e-2, 2e-2)


@pytest.mark.parametrize("kernel", ["tcgen05_1q", "tcgen05_1qp", "tcgen05_2q"])
@pytest.mark.parametrize("units,s,causal", [(1, 256, 0), (1, 256, 1), (2, 100, 1), (3, 777, 0), (2, 1000, 1),
                                            (1, 300, 0), (1, 4100, 0), (40, 1024, 1)])
def test_attention_bf16_each_tc_kernel(gpu, kernel, units, s, causal):
    """Every bf16 tensor-core attention kernel for head_dim 128 (one Q tile per CTA with 64-key
    tiles; the same with persistent CTAs walking several Q tiles each; two Q tiles per CTA with
    128-key tiles), pinned through the tune cache, on ragged and short sequences (a second Q tile
    wholly past the end included) and on a shape with more Q tiles than resident CTAs."""
    rng = np.random.default_rng(units * 31 + s + causal)
    q, k, v = (P.bf16_round(rng.standard_normal((units, s, 128)).astype(np.float32)) for _ in range(3))
    gpu.tune_cache_set(gpu.TUNE_ATTENTION, s, 128, causal, kernel, gpu.BF16)
    try:
        out = gpu.attention_batched(bf(gpu, q), bf(gpu, k), bf(gpu, v), bool(causal), gpu.BF16)
    finally:
        gpu.tune_cache_reset(gpu.TUNE_ATTENTION)
    units_checked = range(units) if s <= 1000 and units <= 3 else [0, units - 1]
    for u in units_checked:
        rows = slice(0, s) if s <= 1000 else slice(s - 300, s)
        ref = P.attention_rows(q[u], k[u], v[u], bool(causal), rows.start, rows.stop)
        close_enough(ref, gpu.from_bf16(out)[u, rows], 2e-2, 2e-2)


def test_attention_bf16_config3_sampled(gpu):
    """Config 3 at full size ([8,16,2048,128] causal), checked on sampled heads and rows."""
    rng = np.random.default_rng(2)
    shape = (128, 2048, 128)
    q, k, v = (rng.standard_normal(shape, dtype=np.float32) for _ in range(3))
    qb, kb, vb = bf(gpu, q), bf(gpu, k), bf(gpu, v)
    out = gpu.from_bf16(gpu.attention_batched(qb, kb, vb, True, gpu.BF16))
    q, k, v = gpu.from_bf16(qb), gpu.from_bf16(kb), gpu.from_bf16(vb)
    for h in (0, 77, 127):
        for r0 in (0, 1000, 1984):
            ref = P.attention_rows(q[h], k[h], v[h], True, r0, r0 + 64)
            close_enough(ref, out[h, r0:r0 + 64], 2e-2, 2e-2)
    assert np.isfinite(out).all()


# ---------------------------------------------------------------- matmul fp32
def test_matmul_kats(gpu):
    g = golden("kat_matmul")
    np.testing.assert_allclose(gpu.matmul2d(g["a"], g["b"]), [[58, 64], [139, 154]], atol=1e-4)
    for name in ("parity_matmul", "cfg2_matmul_128x256x96"):
        g = golden(name)
        close_enough(g["out"], gpu.matmul2d(g["a"], g["b"]), *F32_TOL)


@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (17, 33, 65), (257, 129, 63), (256, 256, 256), (512, 512, 512),
                                   (1024, 1024, 1024), (130, 2048, 7)])
def test_matmul_f32_shapes(gpu, m, k, n):
    rng = np.random.default_rng(m + k + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    close_enough(P.matmul(a, b, threads=8), gpu.matmul2d(a, b), *F32_TOL)


@pytest.mark.parametrize("kernel", ["tcgen05_3xtf32", "simt128x128"])
@pytest.mark.parametrize("m,k,n", [(1024, 1024, 1024), (300, 516, 260), (1000, 36, 1004), (129, 4100, 388)])
def test_matmul_f32_each_kernel(gpu, kernel, m, k, n):
    """Strict fp32 matmul on the 3xTF32 tensor-core kernel and on the SIMT kernel, forced through
    the tune cache, within the 1e-4 contract of the reference CPU loop (tails in M, N and K)."""
    rng = np.random.default_rng(m + 7 * k + 11 * n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    gpu.tune_cache_set(gpu.TUNE_MATMUL, m, k, n, kernel, gpu.F32)
    try:
        out = gpu.matmul2d(a, b)
    finally:
        gpu.tune_cache_reset()
    rows = np.unique(np.linspace(0, m - 1, min(m, 64)).astype(int))
    close_enough(P.matmul(np.ascontiguousarray(a[rows]), b, threads=8), out[rows], *F32_TOL)


# ---------------------------------------------------------------- matmul bf16
def test_matmul_bf16_golden(gpu):
    g = golden("cfg4_gemm_bf16in_192x256x264")
    out = gpu.from_bf16(gpu.matmul2d(bf(gpu, g["a"]), bf(gpu, g["b"]), dtype=gpu.BF16))
    close_enough(g["out"], out, 2e-4, 2e-2)


@pytest.mark.parametrize("m,k,n", [(128, 64, 256), (300, 72, 136), (1, 8, 8), (129, 520, 264), (2048, 2048, 2048),
                                   (64, 100, 30), (4096, 1024, 512)])
def test_matmul_bf16_shapes(gpu, m, k, n):
    rng = np.random.default_rng(m * 7 + k * 3 + n)
    a = P.bf16_round((rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32))
    b = P.bf16_round(rng.uniform(-1, 1, (k, n)).astype(np.float32))
    out = gpu.from_bf16(gpu.matmul2d(bf(gpu, a), bf(gpu, b), dtype=gpu.BF16))
    rows = np.unique(np.linspace(0, m - 1, min(m, 96)).astype(int))
    ref = P.matmul(np.ascontiguousarray(a[rows]), b, threads=8)
    close_enough(ref, out[rows], 2e-3, 2e-2)


@pytest.mark.parametrize("kernel", ["tcgen05_128x256", "tcgen05_2sm_256x256"])
@pytest.mark.parametrize("m,k,n", [(256, 64, 256), (300, 72, 264), (2176, 520, 1288), (1000, 1000, 1000)])
def test_matmul_bf16_each_tc_kernel(gpu, kernel, m, k, n):
    """Both tcgen05 GEMMs (1-SM 128x256 and the 2-SM cluster-pair 256x256 tile), forced through the
    tune cache, on shapes with M/N/K tails and fewer tiles than SM pairs."""
    rng = np.random.default_rng(m + 3 * k + 5 * n)
    a = P.bf16_round((rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32))
    b = P.bf16_round(rng.uniform(-1, 1, (k, n)).astype(np.float32))
    gpu.tune_cache_set(gpu.TUNE_MATMUL, m, k, n, kernel, gpu.BF16)
    try:
        out = gpu.from_bf16(gpu.matmul2d(bf(gpu, a), bf(gpu, b), dtype=gpu.BF16))
    finally:
        gpu.tune_cache_reset()
    rows = np.unique(np.linspace(0, m - 1, min(m, 96)).astype(int))
    ref = P.matmul(np.ascontiguousarray(a[rows]), b, threads=8)
    close_enough(ref, out[rows], 2e-3, 2e-2)


@pytest.mark.parametrize("kernel", ["tcgen05_3xtf32", "simt"])
@pytest.mark.parametrize("units,seq,causal", [(1, 256, 0), (3, 777, 1), (2, 100, 0)])
def test_attention_f32_each_kernel(gpu, kernel, units, seq, causal):
    """Strict fp32 attention (head_dim 64) on the 3xTF32 tensor-core kernel (the default) and on
    the SIMT kernel (pinned through the tune cache), both within 1e-4 of the reference loop."""
    rng = np.random.default_rng(units * 100 + seq)
    q, k, v = (rng.standard_normal((units, seq, 64)).astype(np.float32) for _ in range(3))
    if kernel == "simt":
        gpu.tune_cache_set(gpu.TUNE_ATTENTION, seq, 64, causal, "simt", gpu.F32)
    try:
        out = gpu.attention_batched(q, k, v, causal=bool(causal), dtype=gpu.F32)
    finally:
        gpu.tune_cache_reset(gpu.TUNE_ATTENTION)
    for u in range(units):
        close_enough(P.attention(q[u], k[u], v[u], bool(causal)), out[u], *F32_TOL)


# ---------------------------------------------------------------- pipelined host staging
def test_attention_host_pipelined_bf16(gpu):
    """Host inputs + host output above 24 MB take the chunked path (uploads, kernels and
    downloads overlapped); results must match the oracle like the single-shot path."""
    rng = np.random.default_rng(31)
    units, seq, d = 16, 2048, 128  # 4 x 8 MB of transfers
    q, k, v = (P.bf16_round(rng.standard_normal((units, seq, d)).astype(np.float32)) for _ in range(3))
    out = gpu.from_bf16(gpu.attention_batched(bf(gpu, q), bf(gpu, k), bf(gpu, v), causal=True, dtype=gpu.BF16))
    for u in (0, 7, 15):
        rows = (0, 1023, 2047)
        for r in rows:
            ref = P.attention_rows(q[u], k[u], v[u], True, r, r + 1)
            close_enough(ref, out[u, r:r + 1], 2e-2, 2e-2)


def test_attention_host_pipelined_f32(gpu):
    rng = np.random.default_rng(32)
    units, seq, d = 12, 2048, 64  # 4 x 6 MB
    q, k, v = (rng.standard_normal((units, seq, d)).astype(np.float32) for _ in range(3))
    out = gpu.attention_batched(q, k, v, causal=True, dtype=gpu.F32)
    for u in (0, 5, 11):
        ref = P.attention_rows(q[u], k[u], v[u], True, 1900, 1910)
        close_enough(ref, out[u, 1900:1910], *F32_TOL)


def test_matmul_host_pipelined_bf16(gpu):
    rng = np.random.default_rng(33)
    m = k = n = 2048  # 3 x 8 MB
    a = P.bf16_round((rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32))
    b = P.bf16_round(rng.uniform(-1, 1, (k, n)).astype(np.float32))
    out = gpu.from_bf16(gpu.matmul2d(bf(gpu, a), bf(gpu, b), dtype=gpu.BF16))
    rows = np.array([0, 255, 256, 1023, 1024, 1535, 2047])
    close_enough(P.matmul(np.ascontiguousarray(a[rows]), b, threads=8), out[rows], 2e-3, 2e-2)


# ---------------------------------------------------------------- graph fused nodes
@pytest.mark.parametrize("units,seq,d,cols,causal", [(1, 256, 64, 64, 0), (3, 100, 64, 48, 0), (2, 130, 64, 160, 1),
                                                     (1, 77, 32, 8, 0)])
def test_attention_proj_f32(gpu, units, seq, d, cols, causal):
    """attention_proj_v1: attention then @ proj_w, fused in one kernel for d, cols <= 128 and
    attention + GEMM otherwise (cols = 160)."""
    rng = np.random.default_rng(units * 1000 + seq + cols)
    q, k, v = (rng.standard_normal((units, seq, d)).astype(np.float32) for _ in range(3))
    w = (rng.uniform(-1, 1, (d, cols)) * np.sqrt(6.0 / d)).astype(np.float32)
    out = gpu.attention_proj(q, k, v, w, causal=bool(causal))
    for u in range(units):
        ref = P.matmul(P.attention(q[u], k[u], v[u], causal=bool(causal)), w)
        close_enough(ref, out[u], *F32_TOL)


def test_attention_proj_bf16(gpu):
    rng = np.random.default_rng(21)
    units, seq, d, cols = 4, 384, 128, 128
    q, k, v = (P.bf16_round(rng.standard_normal((units, seq, d)).astype(np.float32)) for _ in range(3))
    w = P.bf16_round((rng.uniform(-1, 1, (d, cols)) / np.sqrt(d)).astype(np.float32))
    out = gpu.from_bf16(gpu.attention_proj(bf(gpu, q), bf(gpu, k), bf(gpu, v), bf(gpu, w), causal=True,
                                           dtype=gpu.BF16))
    for u in range(units):
        attn = P.bf16_round(P.attention(q[u], k[u], v[u], causal=True))
        close_enough(P.matmul(attn, w), out[u], 2e-2, 3e-2)


@pytest.mark.parametrize("have_factor", [3.0, 1.4, 0.3])
def test_attention_qkv_proj(gpu, have_factor):
    """attention_qkv_proj_v1 with a packed input of 3x, 1.4x and 0.3x seq*d floats (the short
    ones take the pack node's cyclic repeat)."""
    seq, d, cols = 196, 64, 64
    rng = np.random.default_rng(int(have_factor * 10))
    flat = rng.standard_normal(int(have_factor * seq * d)).astype(np.float32)
    w = (rng.uniform(-1, 1, (d, cols)) * np.sqrt(6.0 / d)).astype(np.float32)
    out = gpu.attention_qkv_proj(flat, w, seq, d)
    q, k, v = (x.reshape(seq, d) for x in O.qkv_pack_repeat(flat, seq * d))
    ref = P.matmul(P.attention(q, k, v, causal=False), w)
    close_enough(ref, out, *F32_TOL)


# ---------------------------------------------------------------- conv + integrated pipeline
@pytest.mark.parametrize("name,stride,pad,relu", [("parity_conv", (1, 1), (1, 1), False),
                                                  ("conv_stride2_pad0", (2, 1), (0, 1), True)])
def test_conv_golden(gpu, name, stride, pad, relu):
    g = golden(name)
    out = gpu.conv2d_nchw(g["x"], g["w"], g["bias"], stride[0], stride[1], pad[0], pad[1], apply_relu=relu)
    close_enough(g["out"], out, *F32_TOL)


def test_conv_config5_shape(gpu):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2, 64, 56, 56)).astype(np.float32)
    w = rng.uniform(-np.sqrt(6 / 576), np.sqrt(6 / 576), (192, 64, 3, 3)).astype(np.float32)
    bias = rng.standard_normal(192).astype(np.float32)
    out = gpu.conv2d_nchw(x, w, bias, 1, 1, 1, 1, apply_relu=True)
    close_enough(P.conv2d(x, w, bias, (1, 1), (1, 1), True), out, *F32_TOL)


def test_conv_attention_golden(gpu):
    g = golden("cfg5_conv_attention_2x8x12x12")
    out = gpu.lightning_conv_attention_torchstrong_nchw(g["x"], g["w"], g["bias"], 144, 16, pad_h=1, pad_w=1,
                                                         proj_w=g["proj_w"], per_image=True)
    close_enough(g["out"], out, *F32_TOL)
    out = gpu.lightning_conv_attention_torchstrong_nchw(g["x"], g["w"], g["bias"], 144, 16, pad_h=1, pad_w=1,
                                                         per_image=True)
    close_enough(g["out_noproj"], out, *F32_TOL)
    # reference batch semantics: one attention over the first 3*seq*d floats of the flat conv
    # output of the whole batch (here image 0's 24 channels then image 1's)
    out = gpu.lightning_conv_attention_torchstrong_nchw(g["x"], g["w"], g["bias"], 144, 16, pad_h=1, pad_w=1)
    flat = P.conv2d(g["x"], g["w"], g["bias"], (1, 1), (1, 1), True).reshape(-1)
    need = 144 * 16
    q, k, v = (np.ascontiguousarray(flat[i * need:(i + 1) * need].reshape(144, 16)) for i in range(3))
    close_enough(P.attention(q, k, v).reshape(-1), out, *F32_TOL)


def test_conv_attention_repeat(gpu):
    g = golden("conv_attention_repeat")
    out = gpu.lightning_conv_attention_torchstrong_nchw(g["x"], g["w"], None, 40, 4, pad_h=1, pad_w=1)
    close_enough(g["out"].reshape(-1), out, *F32_TOL)


def test_conv_attention_config5_sampled_images(gpu):
    """Config 5 pipeline shape on 3 images: conv 64->192 3x3 p1 + ReLU, attention S=3136 d=64, proj 64x64."""
    rng = np.random.default_rng(4)
    x = rng.standard_normal((3, 64, 56, 56)).astype(np.float32)
    w = rng.uniform(-np.sqrt(6 / 576), np.sqrt(6 / 576), (192, 64, 3, 3)).astype(np.float32)
    bias = np.zeros(192, np.float32)
    pw = np.random.default_rng(5).uniform(-np.sqrt(6 / 64), np.sqrt(6 / 64), (64, 64)).astype(np.float32)
    out = gpu.lightning_conv_attention_torchstrong_nchw(x, w, bias, 3136, 64, pad_h=1, pad_w=1, proj_w=pw,
                                                         per_image=True)
    ref = P.conv_attention_images(x, w, bias, pw, 3136, 64, threads=3)
    close_enough(ref, out, *F32_TOL)


# ---------------------------------------------------------------- elementwise
def test_vector_add(gpu):
    g = golden("parity_vector_add")
    close_enough(g["out"], gpu.vector_add(g["a"], g["b"]), 1e-4, 1e-4)
    rng = np.random.default_rng(9)
    for n in (1, 3, 1025, 1 << 20, (1 << 22) + 7):
        a = rng.uniform(-1, 1, n).astype(np.float32)
        b = rng.uniform(-1, 1, n).astype(np.float32)
        np.testing.assert_array_equal(gpu.vector_add(a, b), P.vector_add(a, b))
    a = rng.uniform(-1, 1, 1001)
    np.testing.assert_array_equal(gpu.vector_add(a, a[::-1].copy()), a + a[::-1])
    # unaligned views take the scalar kernel
    big = rng.uniform(-1, 1, 4099).astype(np.float32)
    np.testing.assert_array_equal(gpu.vector_add(big[1:], big[:-1]), big[1:] + big[:-1])


@pytest.mark.parametrize("rows,cols", [(1024, 1024), (37, 100), (5, 5000), (2048, 1024)])
def test_layer_norm(gpu, rows, cols):
    x = np.random.default_rng(rows).standard_normal((rows, cols)).astype(np.float32)
    close_enough(P.layer_norm(x), gpu.layer_norm(x), 1e-4, 1e-4)


@pytest.mark.parametrize("name", ["ln_readme_16x1024", "ln_readme_5x333"])
def test_layer_norm_readme_golden(gpu, name):
    """lcLayerNorm against the reference's own numpy helper (README.md:2267-2270) output."""
    g = golden(name)
    close_enough(g["out"], gpu.layer_norm(g["x"]), 1e-4, 1e-4)


# ---------------------------------------------------------------- runtime on the device
def test_device_runtime(gpu):
    L = gpu.lib
    n = C.c_int()
    assert L.lcGetDeviceCount(C.byref(n)) == 0 and n.value >= 1
    assert L.lcBackendName().decode() == "cuda"
    buf = gpu.DeviceBuffer.from_array(np.arange(10, dtype=np.float32))
    np.testing.assert_array_equal(buf.download(10, np.float32), np.arange(10, dtype=np.float32))
    assert L.lcDeviceSynchronize() == 0
    code = C.c_uint(123)
    assert L.lcGetDeviceErrorWord(C.byref(code)) == 0 and code.value == 0


@pytest.mark.parametrize("units,s,d,causal", [(128, 2048, 128, 1), (40, 2048, 128, 0), (300, 256, 128, 1),
                                              (7, 3333, 128, 1), (128, 2048, 64, 1), (16, 4096, 128, 1)])
def test_attention_bf16_stress_vs_torch_fp32(gpu, units, s, d, causal):
    """Many-CTA shapes (every TMEM/P-buffer hand-off exercised thousands of times) against a float32
    reference computed on the device from the same bf16 inputs; all heads, all rows."""
    import torch

    torch.manual_seed(units + s)
    q, k, v = (torch.randn((units, s, d), device="cuda").to(torch.bfloat16) for _ in range(3))
    o = torch.zeros_like(q)
    gpu.check(gpu.lib.lcAttentionForward(C.c_void_p(q.data_ptr()), C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()),
                                         C.c_void_p(o.data_ptr()), units, s, d, causal, gpu.BF16, None, None))
    torch.cuda.synchronize()
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=bool(causal))
    err = (o.float() - ref).abs()
    assert bool((err <= 2e-2 + 2e-2 * ref.abs()).all()), float(err.max())


def test_matrix_sub_div(gpu):
    # tests/test_backend_parity.cpp:113-155 inputs and tolerances (sub exact; div 2e-4, as the
    # reference's -ffast-math build divides approximately while the GPU divides in IEEE)
    g = golden("parity_matrix_ops")
    np.testing.assert_array_equal(gpu.matrix_sub(g["a"], g["b"], 9, 13), g["sub"])
    close_enough(g["div"], gpu.matrix_div(g["a"], g["b"], 9, 13), 2e-4, 2e-4)
    rng = np.random.default_rng(12)
    for rows, cols in ((1, 1), (3, 1027), (1024, 1024)):
        a = rng.uniform(-1, 1, (rows, cols)).astype(np.float32)
        b = rng.uniform(0.5, 2, (rows, cols)).astype(np.float32)
        np.testing.assert_array_equal(gpu.matrix_sub(a, b, rows, cols), a - b)
        np.testing.assert_array_equal(gpu.matrix_div(a, b, rows, cols), a / b)
    a = rng.uniform(-1, 1, 999)
    b = rng.uniform(0.5, 2, 999)
    np.testing.assert_array_equal(gpu.matrix_div(a, b, 9, 111), a / b)


def test_reference_c_example_runs(gpu):
    """The reference's unchanged C example, built against include/lc_b200.h and linked to
    liblc_b200.so: lcMalloc / lcMemcpy both ways / lcDeviceSynchronize on the GPU, data round trip."""
    import os
    import subprocess

    from conftest import ROOT

    exe = os.path.join(ROOT, "oracle", "_ref", "c_api_example")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/c_api_example not built")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "Lightning Core C API example: OK" in r.stdout
    assert "backend=cuda" in r.stdout and "cuda=1" in r.stdout


def test_reference_cpp_ops_route_kcuda_here(gpu):
    """The reference's own C++ operator templates (lightning_core::ops::vectorAdd, matMulWithPolicy
    at 256^3 and 1024^3, matrixSubWithPolicy, matrixDivWithPolicy) called with Device::kCUDA, whose
    hooks lightining-core_b200/integration/reference_cuda_hooks.cpp serves from liblc_b200.so:
    each result matches the same call with Device::kCPU (the reference's CPU loops), and every
    kCUDA call was completed by liblc_b200.so rather than by the reference's CPU fallback."""
    import os
    import subprocess

    from conftest import ROOT

    exe = os.path.join(ROOT, "oracle", "_ref", "reference_ops_on_cuda")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/reference_ops_on_cuda not built (needs the reference sources)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "kCUDA calls 5, served by liblc_b200.so 5" in r.stdout, r.stdout


@pytest.mark.parametrize("units,s,d,causal,post", [(37, 1000, 64, 1, 0), (37, 1000, 64, 1, 1), (300, 256, 128, 1, 1),
                                                   (5, 333, 128, 0, 0), (128, 2048, 128, 1, 0)])
def test_attention_bf16_persistent_matches_one_cta_per_tile(gpu, units, s, d, causal, post):
    """The persistent one-tile kernel (tcgen05_1qp) runs the same per-tile arithmetic as the
    one-CTA-per-tile kernel (tcgen05_1q), so their outputs agree bit for bit -- with the
    postprocess, at head_dim 64 and 128, and with many Q tiles per resident CTA."""
    import torch

    torch.manual_seed(units * 7 + s)
    q, k, v = (torch.randn((units, s, d), device="cuda").to(torch.bfloat16) for _ in range(3))
    pol = gpu.default_attention_policy()
    pol.upload_q = pol.upload_k = pol.upload_v = pol.upload_target = 0
    pol.download_out = pol.download_v = 0
    if post:
        pol.output_scale, pol.output_bias, pol.output_relu = 0.5, -0.25, 1
    outs = {}
    for kern in ("tcgen05_1q", "tcgen05_1qp"):
        o = torch.full_like(q, float("nan"))
        gpu.tune_cache_set(gpu.TUNE_ATTENTION, s, d, causal, kern, gpu.BF16)
        try:
            gpu.check(gpu.lib.lcAttentionForward(C.c_void_p(q.data_ptr()), C.c_void_p(k.data_ptr()),
                                                 C.c_void_p(v.data_ptr()), C.c_void_p(o.data_ptr()), units, s, d,
                                                 causal, gpu.BF16, C.byref(pol), None))
            torch.cuda.synchronize()
        finally:
            gpu.tune_cache_reset(gpu.TUNE_ATTENTION)
        outs[kern] = o
    assert torch.equal(outs["tcgen05_1q"], outs["tcgen05_1qp"])
    assert bool(torch.isfinite(outs["tcgen05_1qp"].float()).all())
