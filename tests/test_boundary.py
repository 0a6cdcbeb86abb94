"""The drop-in boundary on CPU: liblc_b200.so loads, exports every symbol include/*.h declares,
keeps the reference's frozen runtime ABI (tests/test_c_api_abi_freeze.cpp of the reference) and
rejects bad arguments before touching a GPU.  No compute calls here."""
import ctypes as C
import glob
import os
import re

import numpy as np
import pytest

from conftest import ROOT

# Frozen struct sizes of the reference ABI on x86-64 (lcGetStructSize of the reference built here).
FROZEN_SIZES = {1: 40, 2: 16, 3: 24, 4: 24, 5: 32, 6: 144}


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(lc[A-Z]\w*)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


def test_exports_every_declared_symbol(lc):
    syms = declared_symbols()
    assert len(syms) > 40
    missing = [s for s in syms if not hasattr(lc.lib, s)]
    assert not missing, missing


def test_only_lc_symbols_exported():
    so = os.path.join(ROOT, "lightining-core_b200", "liblc_b200.so")
    out = os.popen(f"nm -D --defined-only {so}").read().split("\n")
    text = [l.split()[-1] for l in out if " T " in l]
    assert text and all(t.startswith("lc") for t in text), [t for t in text if not t.startswith("lc")][:5]


def test_version_and_struct_freeze(lc):
    a, b, c = C.c_int(), C.c_int(), C.c_int()
    assert lc.lib.lcGetApiVersion(C.byref(a), C.byref(b), C.byref(c)) == lc.LC_SUCCESS
    assert (a.value, b.value, c.value) == (0, 6, 0)
    assert lc.api_version() == "0.6.0-rc0"
    for sid, size in FROZEN_SIZES.items():
        assert lc.lib.lcGetStructSize(sid) == size
        assert lc.lib.lcCheckStructSize(sid, size) == 1
        assert lc.lib.lcCheckStructSize(sid, size + 8) == 0
    assert lc.lib.lcGetStructSize(99) == 0
    assert lc.lib.lcGetApiVersion(None, None, None) == lc.LC_INVALID_VALUE


def test_struct_sizes_match_reference_build(lc):
    from oracle import oracle as O
    if not O.ref_available():
        pytest.skip("reference not built here")
    R = C.CDLL(O.REF_SO)
    R.lcGetStructSize.restype = C.c_size_t
    for sid in FROZEN_SIZES:
        assert R.lcGetStructSize(sid) == lc.lib.lcGetStructSize(sid)


def test_error_strings_and_names(lc):
    # src/runtime.cpp:762-781 strings of the reference
    want = ["success", "not initialized", "invalid value", "out of memory", "not supported", "driver error",
            "unknown error"]
    assert [lc.lib.lcGetErrorString(i).decode() for i in range(7)] == want
    assert lc.lib.lcGetMemoryModel() == 0
    assert lc.lib.lcGetMemoryModelName(0).decode() == "native-device"
    assert lc.lib.lcIsMetalAvailable() == 0


def test_invalid_arguments_rejected_before_gpu(lc):
    L = lc.lib
    p = C.c_void_p()
    assert L.lcMalloc(None, 16) == lc.LC_INVALID_VALUE
    assert L.lcMalloc(C.byref(p), 0) == lc.LC_INVALID_VALUE
    assert L.lcMemcpy(None, None, 4, lc.H2D) == lc.LC_INVALID_VALUE
    assert L.lcFree(None) == lc.LC_SUCCESS
    x = np.zeros(16, np.float32).ctypes.data_as(C.c_void_p)
    # null pointers / zero sizes -> invalid value (src/attention.cpp:145-148; ops.hpp:366-369)
    assert L.lcAttentionForward(None, x, x, x, 1, 4, 4, 0, lc.F32, None, None) == lc.LC_INVALID_VALUE
    assert L.lcAttentionForward(x, x, x, x, 1, 0, 4, 0, lc.F32, None, None) == lc.LC_INVALID_VALUE
    assert L.lcAttentionForward(x, x, x, x, 1, 4, 4, 0, 7, None, None) == lc.LC_NOT_SUPPORTED
    assert L.lcAttentionForward(x, x, x, x, 1, 4, 512, 0, lc.F32, None, None) == lc.LC_NOT_SUPPORTED
    assert L.lcMatMul(x, None, x, 2, 2, 2, lc.F32, None, None) == lc.LC_INVALID_VALUE
    assert L.lcMatMul(x, x, x, 2, 0, 2, lc.F32, None, None) == lc.LC_INVALID_VALUE
    assert L.lcConv2dNchw(x, x, None, x, 1, 1, 2, 2, 1, 3, 3, 1, 1, 0, 0, 0, None, None) == lc.LC_INVALID_VALUE
    assert L.lcConv2dNchw(x, x, None, x, 1, 1, 2, 2, 1, 1, 1, 0, 1, 0, 0, 0, None, None) == lc.LC_INVALID_VALUE
    assert L.lcVectorAdd(x, x, None, 4, lc.F32, None, None) == lc.LC_INVALID_VALUE
    assert L.lcVectorAdd(x, x, x, 4, lc.BF16, None, None) == lc.LC_NOT_SUPPORTED
    assert L.lcLayerNorm(x, x, 0, 4, 1e-5, None) == lc.LC_INVALID_VALUE
    # graph fused nodes: missing projection / zero columns / non-neutral postprocess
    assert L.lcAttentionProjForward(x, x, x, None, x, 1, 4, 4, 4, 0, lc.F32, None, None) == lc.LC_INVALID_VALUE
    assert L.lcAttentionProjForward(x, x, x, x, x, 1, 4, 4, 0, 0, lc.F32, None, None) == lc.LC_INVALID_VALUE
    pol = lc.default_attention_policy()
    pol.output_relu = 1
    assert L.lcAttentionProjForward(x, x, x, x, x, 1, 4, 4, 4, 0, lc.F32, C.byref(pol), None) == lc.LC_NOT_SUPPORTED
    assert L.lcAttentionQkvProjForward(x, 0, x, x, 4, 4, 4, None, None) == lc.LC_INVALID_VALUE
    # attention autotune: null buffers / zero sizes / unsupported dtype or size, before any launch
    buf = C.create_string_buffer(64)
    assert L.lcAttentionAutotune(None, x, x, x, 1, 4, 4, 0, lc.F32, None, buf, 64) == lc.LC_INVALID_VALUE
    assert L.lcAttentionAutotune(x, x, x, x, 1, 0, 4, 0, lc.F32, None, buf, 64) == lc.LC_INVALID_VALUE
    assert L.lcAttentionAutotune(x, x, x, x, 1, 4, 4, 0, 7, None, buf, 64) == lc.LC_NOT_SUPPORTED
    assert L.lcAttentionAutotune(x, x, x, x, 1, 4, 512, 0, lc.F32, None, buf, 64) == lc.LC_NOT_SUPPORTED


def test_policy_defaults_and_loop_presets(lc):
    p = lc.default_attention_policy()
    assert (p.upload_q, p.upload_k, p.upload_v, p.download_out, p.synchronize) == (1, 1, 1, 1, 1)
    assert (p.output_scale, p.output_bias, p.output_relu, p.loss_every) == (1.0, 0.0, 0, 1)
    # include/lightning_core/core/ops/policy.hpp:37-71 of the reference
    table = {lc.LOOP_START: (1, 1, 0, 0), lc.LOOP_RUN: (0, 0, 0, 0), lc.LOOP_FINISH: (0, 0, 1, 1),
             lc.LOOP_SYNC: (0, 0, 0, 1)}
    for stage, want in table.items():
        q = lc.matmul_policy_for_stage(stage)
        assert (q.upload_a, q.upload_b, q.download_out, q.synchronize) == want
        for fn in (lc.lib.lcVectorPolicyForStage, lc.lib.lcElemwisePolicyForStage):
            v = lc.VectorAddIoPolicy()
            fn(stage, C.byref(v))
            assert (v.upload_a, v.upload_b, v.download_out, v.synchronize) == want


def test_attention_loop_presets(lc):
    """makeAttentionPolicyForLoop (include/lightning_core/core/model_customization.hpp:146-185): the
    transfer/sync flags per stage; loss_every and the postprocess are left as the caller set them."""
    flags = ("upload_q", "upload_k", "upload_v", "upload_target", "download_out", "download_v", "synchronize")
    table = {lc.LOOP_START: (1, 1, 1, 1, 0, 0, 0), lc.LOOP_RUN: (0,) * 7, lc.LOOP_SYNC: (0,) * 6 + (1,)}
    for training in (0, 1):
        table[lc.LOOP_FINISH] = (0, 0, 0, 0, 1, training, 1)
        for stage, want in table.items():
            p = lc.default_attention_policy()
            p.loss_every, p.output_scale, p.output_bias, p.output_relu = 8, 0.5, -1.0, 1
            lc.lib.lcAttentionPolicyForStage(stage, training, C.byref(p))
            assert tuple(getattr(p, f) for f in flags) == want, (stage, training)
            assert (p.loss_every, p.output_scale, p.output_bias, p.output_relu) == (8, 0.5, -1.0, 1)


def test_conv_tune_key_packing(lc):
    d = lc.conv_tune_key(32, 64, 56, 56, 192, 3, 3, 1, 1, 1, 1)
    assert d == ((64 << 32) | 192, (56 << 32) | 56, (32 << 32) | (3 << 24) | (3 << 16) | (1 << 12) | (1 << 8) | (1 << 4) | 1)
    with pytest.raises(lc.LightningError):
        lc.conv_tune_key(1, 3, 8, 8, 4, 3, 3, 16, 1, 0, 0)  # stride does not fit the key


def test_trace_ring(lc):
    L = lc.lib
    assert L.lcRuntimeTraceCapacity() == 4096
    L.lcRuntimeTraceClear()
    L.lcRuntimeTraceSetEnabled(1)
    p = C.c_void_p()
    L.lcMalloc(C.byref(p), 0)  # traced even when rejected
    L.lcRuntimeTraceSetEnabled(0)
    assert L.lcRuntimeTraceCount() == 1
    ev = lc.RuntimeTraceEvent()
    assert L.lcRuntimeTraceGet(0, C.byref(ev)) == lc.LC_SUCCESS
    assert (ev.type, ev.status) == (0, lc.LC_INVALID_VALUE)
    assert L.lcRuntimeTraceGet(5, C.byref(ev)) == lc.LC_INVALID_VALUE


def test_python_api_shape_errors(lc):
    with pytest.raises(ValueError):
        lc.attention2d(np.zeros((4, 4)), np.zeros((4, 5)), np.zeros((4, 4)))
    with pytest.raises(ValueError):
        lc.matmul2d(np.zeros((2, 3)), np.zeros((4, 2)))
    with pytest.raises(ValueError):
        lc.conv2d_nchw(np.zeros((1, 2, 4, 4)), np.zeros((3, 1, 3, 3)))
    with pytest.raises(ValueError):
        lc.attention2d(np.zeros((4, 4)), np.zeros((4, 4)), np.zeros((4, 4)), device="cpu")


def test_bf16_helpers(lc):
    x = np.random.default_rng(0).standard_normal(1000).astype(np.float32)
    from oracle import oracle as O
    np.testing.assert_array_equal(lc.from_bf16(lc.to_bf16(x)), O.port().bf16_round(x))


def test_reference_c_example_links_against_this_library():
    """The reference's own C example (examples/lightning_core_c_api.c), compiled unchanged against
    include/lc_b200.h by `make -C oracle example`, resolves its lc* symbols from liblc_b200.so."""
    exe = os.path.join(ROOT, "oracle", "_ref", "c_api_example")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/c_api_example not built (needs the reference sources)")
    out = os.popen(f"ldd {exe}").read()
    assert "liblc_b200.so" in out and "not found" not in out, out


def test_reference_kcuda_route_fails_loudly_without_a_gpu(lc):
    """The reference's C++ ops called with Device::kCUDA through the integration hooks
    (tests/native/reference_ops_on_cuda.cpp): on a machine without a visible GPU every kCUDA call
    comes back as an error (kNotInitialized = 1) instead of kNotSupported, which would send the
    reference's dispatcher into its silent CPU fallback; the driver exits non-zero."""
    import subprocess

    exe = os.path.join(ROOT, "oracle", "_ref", "reference_ops_on_cuda")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/reference_ops_on_cuda not built (needs the reference sources)")
    if lc.cuda_available():
        pytest.skip("a GPU is visible: the GPU test runs this driver for real")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode != 0
    lines = [ln for ln in r.stdout.splitlines() if "cpu=" in ln]
    assert len(lines) == 5, r.stdout
    assert all("cpu=0 cuda=1 " in ln for ln in lines), r.stdout
    assert "served by liblc_b200.so 0" in r.stdout


def test_conv_sizes_beyond_int_rejected_before_gpu(lc):
    """The conv launchers work in int: a reduction length in_channels*kh*kw, a padded extent or any
    size argument beyond INT_MAX is LC_NOT_SUPPORTED before anything touches the GPU, in every conv
    entry point (lcConv2dNchw, lcConvAttentionNchw, lcConvAttentionNchwNoAlloc, lcConvAutotune)."""
    L = lc.lib
    x = np.zeros(16, np.float32).ctypes.data_as(C.c_void_p)
    big_c = 1 << 30  # 2^30 channels x 3 x 3 > INT_MAX
    assert L.lcConv2dNchw(x, x, None, x, 1, big_c, 4, 4, 4, 3, 3, 1, 1, 1, 1, 0, None, None) == lc.LC_NOT_SUPPORTED
    assert L.lcConvAttentionNchw(x, x, None, None, x, 1, big_c, 4, 4, 4, 3, 3, 1, 1, 1, 1, 4, 4, 0, 1, None,
                                 None) == lc.LC_NOT_SUPPORTED
    assert L.lcConvAttentionNchwNoAlloc(x, x, None, None, x, 1, big_c, 4, 4, 4, 3, 3, 1, 1, 1, 1, 4, 4, 0, 1,
                                        None) == lc.LC_NOT_SUPPORTED
    huge_pad = 1 << 31
    assert L.lcConv2dNchw(x, x, None, x, 1, 4, 4, 4, 4, 3, 3, 1, 1, huge_pad, 1, 0, None, None) == lc.LC_NOT_SUPPORTED
    buf = C.create_string_buffer(64)
    assert L.lcConvAutotune(x, x, None, x, 1, big_c, 4, 4, 4, 3, 3, 1, 1, 1, 1, 0, None, buf, 64) == \
        lc.LC_NOT_SUPPORTED
