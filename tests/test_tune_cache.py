"""Auto-tune cache file format and behaviour (CPU), after the reference's
tests/test_python_tune_cache_format_smoke.py: `#lc_tune_cache,<kind>,2` header, a `#columns,`
line, version-1 files accepted, unknown headers rejected without touching the current rows."""
import numpy as np
import pytest

from conftest import close_enough


@pytest.fixture(autouse=True)
def _clean(lc):
    for kind in (lc.TUNE_MATMUL, lc.TUNE_ATTENTION, lc.TUNE_CONV):
        lc.lib.lcTuneCacheReset(kind)
    yield
    for kind in (lc.TUNE_MATMUL, lc.TUNE_ATTENTION, lc.TUNE_CONV):
        lc.lib.lcTuneCacheReset(kind)


def test_roundtrip_v2(lc, tmp_path):
    lc.tune_cache_set(lc.TUNE_MATMUL, 1024, 1024, 1024, "simt64x64")
    lc.tune_cache_set(lc.TUNE_MATMUL, 8192, 8192, 8192, "tcgen05_128x256", lc.BF16)
    lc.tune_cache_set(lc.TUNE_ATTENTION, 2048, 128, 1, "tcgen05", lc.BF16)
    f = tmp_path / "mm.csv"
    assert lc.lib.lcTuneCacheSave(lc.TUNE_MATMUL, str(f).encode()) == 0
    lines = f.read_text().splitlines()
    assert lines[0] == "#lc_tune_cache,matmul,2"
    assert lines[1].startswith("#columns,")
    assert "1024,1024,1024,f32,simt64x64" in lines
    assert "8192,8192,8192,bf16,tcgen05_128x256" in lines
    lc.lib.lcTuneCacheReset(lc.TUNE_MATMUL)
    assert lc.lib.lcTuneCacheSize(lc.TUNE_MATMUL) == 0
    assert lc.lib.lcTuneCacheLoad(lc.TUNE_MATMUL, str(f).encode()) == 0
    assert lc.tune_cache_get(lc.TUNE_MATMUL, 1024, 1024, 1024) == "simt64x64"
    assert lc.tune_cache_get(lc.TUNE_MATMUL, 8192, 8192, 8192, lc.BF16) == "tcgen05_128x256"
    assert lc.tune_cache_get(lc.TUNE_MATMUL, 8192, 8192, 8192) is None  # dtype is part of the key
    assert lc.tune_cache_get(lc.TUNE_ATTENTION, 2048, 128, 1, lc.BF16) == "tcgen05"


def test_v1_rows_load_as_f32(lc, tmp_path):
    f = tmp_path / "v1.csv"
    f.write_text("#lc_tune_cache,matmul,1\n#columns,m,k,n,config\n256,256,256,simt128x64\n")
    assert lc.lib.lcTuneCacheLoad(lc.TUNE_MATMUL, str(f).encode()) == 0
    assert lc.tune_cache_get(lc.TUNE_MATMUL, 256, 256, 256) == "simt128x64"


def test_crlf_and_padded_rows_load(lc, tmp_path):
    f = tmp_path / "crlf.csv"
    f.write_bytes(b"#lc_tune_cache,matmul,2\r\n#columns,m,k,n,dtype,config\r\n"
                  b"512,512,512,f32,simt64x64\r\n 64 , 32 , 16 , bf16 , tcgen05_128x256 \r\n\r\n")
    assert lc.lib.lcTuneCacheLoad(lc.TUNE_MATMUL, str(f).encode()) == 0
    assert lc.tune_cache_get(lc.TUNE_MATMUL, 512, 512, 512) == "simt64x64"
    assert lc.tune_cache_get(lc.TUNE_MATMUL, 64, 32, 16, lc.BF16) == "tcgen05_128x256"
    assert lc.lib.lcTuneCacheSize(lc.TUNE_MATMUL) == 2


@pytest.mark.parametrize("header", ["#lc_tune_cache,matmul,9", "#lc_tune_cache,attention,2", "m,k,n", ""])
def test_unknown_header_rejected(lc, tmp_path, header):
    lc.tune_cache_set(lc.TUNE_MATMUL, 1, 2, 3, "simt64x64")
    f = tmp_path / "bad.csv"
    f.write_text(header + "\n4,5,6,f32,simt128x128\n")
    assert lc.lib.lcTuneCacheLoad(lc.TUNE_MATMUL, str(f).encode()) == lc.LC_NOT_SUPPORTED
    assert lc.tune_cache_get(lc.TUNE_MATMUL, 1, 2, 3) == "simt64x64"
    assert lc.tune_cache_get(lc.TUNE_MATMUL, 4, 5, 6) is None


def test_bad_arguments(lc):
    assert lc.lib.lcTuneCacheSet(lc.TUNE_MATMUL, 1, 1, 1, 0, b"a,b") == lc.LC_INVALID_VALUE
    assert lc.lib.lcTuneCacheSet(7, 1, 1, 1, 0, b"x") == lc.LC_INVALID_VALUE
    assert lc.lib.lcTuneCacheLoad(lc.TUNE_MATMUL, b"/nonexistent/file.csv") == lc.LC_NOT_SUPPORTED


@pytest.mark.gpu
@pytest.mark.parametrize("cfg", ["simt128x128", "simt128x64", "simt64x64"])
def test_every_f32_tile_config_parity(gpu, cfg):
    from oracle import oracle as O

    m, k, n = 200, 136, 72
    rng = np.random.default_rng(1)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    gpu.tune_cache_set(gpu.TUNE_MATMUL, m, k, n, cfg)
    close_enough(O.port().matmul(a, b), gpu.matmul2d(a, b), 1e-4, 1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_autotune_records_and_is_used(gpu, dtype, tmp_path, monkeypatch):
    from oracle import oracle as O

    n = 1024
    rng = np.random.default_rng(3)
    a = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    b = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    dt = gpu.F32 if dtype == "f32" else gpu.BF16
    if dt == gpu.BF16:
        a, b = O.port().bf16_round(a / 32), O.port().bf16_round(b)
        ha, hb = gpu.to_bf16(a), gpu.to_bf16(b)
    else:
        ha, hb = a, b
    da, db = gpu.DeviceBuffer.from_array(ha), gpu.DeviceBuffer.from_array(hb)
    dc = gpu.DeviceBuffer(n * n * (4 if dt == gpu.F32 else 2))
    best = gpu.matmul_autotune(da, db, dc, n, n, n, dt)
    assert gpu.tune_cache_get(gpu.TUNE_MATMUL, n, n, n, dt) == best
    out = gpu.matmul2d(ha, hb, dtype=dt)
    got = out if dt == gpu.F32 else gpu.from_bf16(out)
    ref = O.port().matmul(a[:64], b, threads=8)
    close_enough(ref, got[:64], *((1e-4, 1e-4) if dt == gpu.F32 else (2e-3, 2e-2)))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,d,causal", [("bf16", 128, 0), ("bf16", 128, 1), ("bf16", 64, 1), ("f32", 64, 0)])
def test_attention_autotune_records_and_is_used(gpu, dtype, d, causal):
    """lcAttentionAutotune times the kernels that can take the shape, stores the fastest under
    (seq, head_dim, causal, dtype), and the next call through the dispatch uses it correctly."""
    from oracle import oracle as O

    units, seq = 4, 384
    dt = gpu.F32 if dtype == "f32" else gpu.BF16
    rng = np.random.default_rng(d + causal)
    q, k, v = (rng.standard_normal((units, seq, d)).astype(np.float32) for _ in range(3))
    if dt == gpu.BF16:
        q, k, v = (O.port().bf16_round(x) for x in (q, k, v))
        hq, hk, hv = (gpu.to_bf16(x) for x in (q, k, v))
    else:
        hq, hk, hv = q, k, v
    dq, dk, dv = (gpu.DeviceBuffer.from_array(x) for x in (hq, hk, hv))
    dout = gpu.DeviceBuffer(units * seq * d * (4 if dt == gpu.F32 else 2))
    try:
        best = gpu.attention_autotune(dq, dk, dv, dout, units, seq, d, bool(causal), dt)
        allowed = {"simt", "tcgen05_3xtf32"} if dt == gpu.F32 else {"simt", "tcgen05_1q", "tcgen05_1qp", "tcgen05_2q"}
        assert best in allowed
        assert best != "tcgen05_2q" or d == 128
        assert gpu.tune_cache_get(gpu.TUNE_ATTENTION, seq, d, causal, dt) == best
        out = gpu.attention_batched(hq, hk, hv, bool(causal), dt)
    finally:
        gpu.tune_cache_reset(gpu.TUNE_ATTENTION)
    got = out if dt == gpu.F32 else gpu.from_bf16(out)
    tol = (1e-4, 1e-4) if dt == gpu.F32 else (2e-2, 2e-2)
    for u in range(units):
        close_enough(O.port().attention(q[u], k[u], v[u], bool(causal)), got[u], *tol)


def test_conv_cache_roundtrip(lc, tmp_path):
    """The conv kind uses the same file format: `#lc_tune_cache,conv,2` with packed shape keys."""
    key = lc.conv_tune_key(32, 64, 56, 56, 192, 3, 3, 1, 1, 1, 1)
    lc.tune_cache_set(lc.TUNE_CONV, *key, "tcgen05_3xtf32", lc.F32)
    path = str(tmp_path / "conv.csv")
    assert lc.lib.lcTuneCacheSave(lc.TUNE_CONV, path.encode()) == lc.LC_SUCCESS
    lines = open(path).read().splitlines()
    assert lines[0] == "#lc_tune_cache,conv,2" and lines[1].startswith("#columns,")
    lc.lib.lcTuneCacheReset(lc.TUNE_CONV)
    assert lc.lib.lcTuneCacheLoad(lc.TUNE_CONV, path.encode()) == lc.LC_SUCCESS
    assert lc.tune_cache_get(lc.TUNE_CONV, *key, lc.F32) == "tcgen05_3xtf32"


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("m,k,n", [(1, 1024, 1024), (2, 4096, 777), (1, 3, 5), (2, 8192, 8), (1, 50000, 96)])
def test_small_m_gemv(gpu, dtype, m, k, n):
    """m <= 2 runs the GEMV (the reference's small-M path, src/ops/matmul_metal.mm:795-863), by
    default and pinned; against the oracle; the autotune offers it and its result is used."""
    from oracle import oracle as O

    P = O.port()
    rng = np.random.default_rng(m * 7 + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
    dt = gpu.F32 if dtype == "f32" else gpu.BF16
    if dt == gpu.BF16:
        a, b = P.bf16_round(a), P.bf16_round(b)
    ref = P.matmul(a, b)
    tol = (1e-4, 1e-4) if dt == gpu.F32 else (2e-3, 2e-2)
    conv = (lambda x: x) if dt == gpu.F32 else gpu.from_bf16
    ha, hb = (a, b) if dt == gpu.F32 else (gpu.to_bf16(a), gpu.to_bf16(b))
    close_enough(ref, conv(gpu.matmul2d(ha, hb, dtype=dt)), *tol)
    gpu.tune_cache_set(gpu.TUNE_MATMUL, m, k, n, "gemv", dt)
    close_enough(ref, conv(gpu.matmul2d(ha, hb, dtype=dt)), *tol)
    gpu.lib.lcTuneCacheReset(gpu.TUNE_MATMUL)
    da, db = gpu.DeviceBuffer.from_array(ha), gpu.DeviceBuffer.from_array(hb)
    dc = gpu.DeviceBuffer(m * n * (4 if dt == gpu.F32 else 2))
    best = gpu.matmul_autotune(da, db, dc, m, k, n, dt)
    assert gpu.tune_cache_get(gpu.TUNE_MATMUL, m, k, n, dt) == best
    close_enough(ref, conv(gpu.matmul2d(ha, hb, dtype=dt)), *tol)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(2, 64, 56, 56, 192, 1, 1, 3), (3, 8, 12, 12, 24, 1, 1, 3),
                                   (1, 32, 30, 30, 64, 2, 0, 3), (2, 32, 17, 23, 48, 1, 2, 5),
                                   (3, 96, 9, 9, 256, 1, 1, 3), (1, 64, 7, 7, 16, 1, 0, 1)])
def test_conv_modes_and_autotune(gpu, shape):
    """The conv kernel-mode cache (the reference's chooseModeWithAutotune,
    src/ops/conv2d_metal.mm:577-672): every mode pinned through LC_TUNE_CONV matches the oracle, and
    lcConvAutotune stores a mode that is then used."""
    import ctypes as C

    from oracle import oracle as O

    P = O.port()
    n, c, h, w_, oc, st, pd, ks = shape
    rng = np.random.default_rng(n + c + oc)
    x = rng.standard_normal((n, c, h, w_)).astype(np.float32)
    w = rng.uniform(-0.2, 0.2, (oc, c, ks, ks)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, oc).astype(np.float32)
    ref = P.conv2d(x, w, bias, (st, st), (pd, pd), True)
    key = gpu.conv_tune_key(n, c, h, w_, oc, ks, ks, st, st, pd, pd)
    modes = ["simt"] + (["tcgen05_3xtf32"] if oc >= 32 else [])
    modes += ["tcgen05_implicit"] if c % 32 == 0 and oc % 16 == 0 and 16 <= oc <= 256 else []
    for mode in modes:
        gpu.tune_cache_set(gpu.TUNE_CONV, *key, mode, gpu.F32)
        close_enough(ref, gpu.conv2d_nchw(x, w, bias, st, st, pd, pd, apply_relu=True), 1e-4, 1e-4)
    gpu.lib.lcTuneCacheReset(gpu.TUNE_CONV)
    dx, dw, db = (gpu.DeviceBuffer.from_array(t) for t in (x, w, bias))
    dout = gpu.DeviceBuffer(ref.size * 4)
    best = C.create_string_buffer(64)
    gpu.check(gpu.lib.lcConvAutotune(dx.ptr, dw.ptr, db.ptr, dout.ptr, n, c, h, w_, oc, ks, ks, st, st, pd, pd, 1,
                                     None, best, 64), "lcConvAutotune")
    assert best.value.decode() in modes
    assert gpu.tune_cache_get(gpu.TUNE_CONV, *key, gpu.F32) == best.value.decode()
    close_enough(ref, dout.download(ref.shape, np.float32), 1e-4, 1e-4)
    close_enough(ref, gpu.conv2d_nchw(x, w, bias, st, st, pd, pd, apply_relu=True), 1e-4, 1e-4)
