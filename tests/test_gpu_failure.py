"""Failure paths on the GPU, in the forms this pool allows (no fault, trap or hang):

* a bounded device wait that runs out: lcTestStallNextGemm makes one CTA of the 1-SM tcgen05
  GEMM leave a k-block unloaded, so its MMA warp's 2 s mbarrier wait gives up; the kernel records
  the site in the device error word, drains and exits, the call returns LC_DRIVER_ERROR, and after
  lcClearDeviceErrorWord the next call is correct again (the reference's status contract:
  include/lightning_core/core/runtime.hpp:24-32 -- errors are returned, never thrown);
* allocation failure on the host side: lcTestFailAllocations makes the library's next device
  allocations fail; the ops return LC_OUT_OF_MEMORY, hold nothing afterwards, and work on the
  next call;
* the strict-fp32 tensor-core paths take their workspace per call on the caller's stream, so two
  streams run side by side (no library lock or cross-stream event orders them)."""
import ctypes as C
import time

import numpy as np
import pytest

from conftest import close_enough
from oracle import oracle as O

pytestmark = pytest.mark.gpu
P = O.port()
ERR_GEMM_SITES = (0x101, 0x102, 0x103)  # producer / MMA / epilogue waits of the GEMM: whichever gives up first


def _p(t):
    return C.c_void_p(t.data_ptr())


def test_bounded_wait_timeout_reports_driver_error(gpu):
    import torch

    L = gpu.lib
    m, k, n = 256, 128, 256  # two 128x256 tiles, two k-blocks each
    rng = np.random.default_rng(3)
    a_h = P.bf16_round((rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32))
    b_h = P.bf16_round(rng.uniform(-1, 1, (k, n)).astype(np.float32))
    a = torch.from_numpy(a_h).to(torch.bfloat16).cuda()
    b = torch.from_numpy(b_h).to(torch.bfloat16).cuda()
    c = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
    pol = gpu.MatMulIoPolicy(0, 0, 0, 1)  # device pointers, synchronize
    gpu.tune_cache_set(gpu.TUNE_MATMUL, m, k, n, "tcgen05_128x256", gpu.BF16)
    try:
        assert L.lcClearDeviceErrorWord() == gpu.LC_SUCCESS
        L.lcTestStallNextGemm(1)
        t0 = time.time()
        rc = L.lcMatMul(_p(a), _p(b), _p(c), m, k, n, gpu.BF16, C.byref(pol), None)
        took = time.time() - t0
        assert rc == gpu.LC_DRIVER_ERROR, rc
        assert 1.5 < took < 30, took  # the wait limit is 2 s
        code = C.c_uint()
        assert L.lcGetDeviceErrorWord(C.byref(code)) == gpu.LC_DRIVER_ERROR
        assert code.value in ERR_GEMM_SITES, hex(code.value)
        # the context is still usable: clear, rerun, correct
        assert L.lcClearDeviceErrorWord() == gpu.LC_SUCCESS
        assert L.lcGetDeviceErrorWord(C.byref(code)) == gpu.LC_SUCCESS and code.value == 0
        rc = L.lcMatMul(_p(a), _p(b), _p(c), m, k, n, gpu.BF16, C.byref(pol), None)
        assert rc == gpu.LC_SUCCESS
    finally:
        L.lcTestStallNextGemm(-1)
        L.lcClearDeviceErrorWord()  # never leave the word set for later tests
        gpu.tune_cache_reset()
    close_enough(P.matmul(a_h, b_h), c.float().cpu().numpy(), 2e-3, 2e-2)


def test_allocation_failure_returns_oom_without_leak(gpu):
    import torch

    L = gpu.lib
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    # session: the third of its four buffers fails; the first two must be released
    h = C.c_void_p()
    L.lcTestFailAllocations(2, 1)
    try:
        rc = L.lcAttentionSessionCreate(C.byref(h), 4, 4096, 128, 1, gpu.BF16)
    finally:
        L.lcTestFailAllocations(0, 0)
    assert rc == gpu.LC_OUT_OF_MEMORY and not h.value
    assert torch.cuda.mem_get_info()[0] == free0
    assert L.lcAttentionSessionCreate(C.byref(h), 4, 4096, 128, 1, gpu.BF16) == gpu.LC_SUCCESS
    assert L.lcAttentionSessionDestroy(h) == gpu.LC_SUCCESS
    # host-pointer matmul whose staging buffer must grow (larger than any earlier call): OOM, fine
    rng = np.random.default_rng(4)
    big = np.zeros((8192, 6144), np.float32)  # 201 MB: more than any staging slot holds yet
    bb = np.zeros((6144, 8), np.float32)
    L.lcTestFailAllocations(0, 1)
    try:
        with pytest.raises(gpu.LightningError) as ei:
            gpu.matmul2d(big, bb)
        assert ei.value.code == gpu.LC_OUT_OF_MEMORY
    finally:
        L.lcTestFailAllocations(0, 0)
    del big
    a = rng.uniform(-1, 1, (700, 300)).astype(np.float32)
    b = rng.uniform(-1, 1, (300, 500)).astype(np.float32)
    close_enough(P.matmul(a, b), gpu.matmul2d(a, b), 1e-4, 1e-4)
    # the 3xTF32 workspace (stream-ordered pool): OOM, then fine
    ta = torch.from_numpy(rng.uniform(-1, 1, (1024, 1024)).astype(np.float32)).cuda()
    tb = torch.from_numpy(rng.uniform(-1, 1, (1024, 1024)).astype(np.float32)).cuda()
    tc = torch.zeros_like(ta)
    L.lcTestFailAllocations(0, 1)
    try:
        rc = L.lcMatMul(_p(ta), _p(tb), _p(tc), 1024, 1024, 1024, gpu.F32, None, None)
    finally:
        L.lcTestFailAllocations(0, 0)
    assert rc == gpu.LC_OUT_OF_MEMORY
    assert L.lcMatMul(_p(ta), _p(tb), _p(tc), 1024, 1024, 1024, gpu.F32, None, None) == gpu.LC_SUCCESS
    torch.cuda.synchronize()
    rows = [0, 511, 1023]
    close_enough(P.matmul(np.ascontiguousarray(ta.cpu().numpy()[rows]), tb.cpu().numpy()),
                 tc.cpu().numpy()[rows], 1e-4, 1e-4)


def test_fp32_tensor_core_calls_overlap_across_streams(gpu):
    """Two strict-fp32 attention calls (3xTF32 kernel, few CTAs each) on two streams: their device
    intervals overlap, i.e. nothing in the library serialises them."""
    import torch

    L = gpu.lib
    units, seq, d = 2, 2048, 64
    g = torch.Generator(device="cuda").manual_seed(5)
    qs = [torch.randn((units, seq, d), generator=g, device="cuda") for _ in range(6)]
    outs = [torch.empty((units, seq, d), device="cuda") for _ in range(2)]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]

    def call(i):
        q, k, v = qs[3 * i:3 * i + 3]
        return L.lcAttentionForward(_p(q), _p(k), _p(v), _p(outs[i]), units, seq, d, 0, gpu.F32, None,
                                    C.c_void_p(streams[i].cuda_stream))

    for i in range(2):
        assert call(i) == gpu.LC_SUCCESS
    torch.cuda.synchronize()
    overlapped = False
    for _ in range(5):
        base = torch.cuda.Event(enable_timing=True)
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(2)]
        base.record()
        torch.cuda.synchronize()
        for i in range(2):
            ev[i][0].record(streams[i])
            assert call(i) == gpu.LC_SUCCESS
            ev[i][1].record(streams[i])
        torch.cuda.synchronize()
        (s0, e0), (s1, e1) = ((base.elapsed_time(a), base.elapsed_time(b)) for a, b in ev)
        if s1 < e0 and s0 < e1:
            overlapped = True
            break
    assert overlapped, (s0, e0, s1, e1)
    for i in range(2):
        q, k, v = (t.cpu().numpy() for t in qs[3 * i:3 * i + 3])
        close_enough(P.attention(q[0], k[0], v[0]), outs[i][0].cpu().numpy(), 1e-4, 1e-4)


def test_async_host_input_calls_on_two_streams_keep_their_inputs(gpu):
    """Two asynchronous calls with host inputs (upload set, no download, no synchronize) on two
    streams from one thread: both go through this thread's staging buffers, so the second call's
    uploads must wait until the first call's kernel has read them.  Each output must equal the
    output of the same call made alone and synchronously (same kernel, bit for bit)."""
    import torch

    L = gpu.lib
    units, seq, d = 48, 2048, 128
    g = torch.Generator().manual_seed(9)
    host = [torch.randn((units, seq, d), generator=g).to(torch.bfloat16).pin_memory() for _ in range(6)]
    outs = [torch.empty((units, seq, d), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    want = [torch.empty_like(outs[0]) for _ in range(2)]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    pol = gpu.default_attention_policy()
    pol.upload_q = pol.upload_k = pol.upload_v = 1
    pol.download_out = 0
    pol.synchronize = 0

    def call(i, out, stream):
        q, k, v = host[3 * i:3 * i + 3]
        return L.lcAttentionForward(_p(q), _p(k), _p(v), _p(out), units, seq, d, 1, gpu.BF16, C.byref(pol),
                                    C.c_void_p(stream.cuda_stream))

    for i in range(2):  # alone, one at a time
        assert call(i, want[i], streams[0]) == gpu.LC_SUCCESS
        torch.cuda.synchronize()
    for _ in range(3):  # back to back on two streams, nothing synchronised in between
        for o in outs:
            o.zero_()
        torch.cuda.synchronize()
        assert call(0, outs[0], streams[0]) == gpu.LC_SUCCESS
        assert call(1, outs[1], streams[1]) == gpu.LC_SUCCESS
        torch.cuda.synchronize()
        for i in range(2):
            assert torch.equal(outs[i], want[i]), i
