"""Device-resident sessions (AttentionSession / MatMulMetalResidentSession of the reference):
the resident loop start -> run* -> finish, buffer reuse without uploads, thread sharing
(tests/test_attention.cpp:170-221 of the reference runs 4 threads on one session)."""
import ctypes as C
import threading

import numpy as np
import pytest

from conftest import close_enough
from oracle import oracle as O


def test_session_argument_errors(lc):
    h = C.c_void_p()
    assert lc.lib.lcAttentionSessionCreate(None, 1, 4, 4, 0, lc.F32) == lc.LC_INVALID_VALUE
    assert lc.lib.lcAttentionSessionCreate(C.byref(h), 1, 0, 4, 0, lc.F32) == lc.LC_INVALID_VALUE
    assert lc.lib.lcAttentionSessionCreate(C.byref(h), 1, 4, 4, 0, 9) == lc.LC_NOT_SUPPORTED
    assert lc.lib.lcMatMulSessionCreate(C.byref(h), 0, 4, 4, lc.F32) == lc.LC_INVALID_VALUE
    assert lc.lib.lcAttentionSessionDestroy(None) == lc.LC_INVALID_VALUE
    assert lc.lib.lcMatMulSessionRun(None, None, None, None, None, None) == lc.LC_INVALID_VALUE


@pytest.mark.gpu
def test_attention_session_forward_and_resident_reuse(gpu):
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((130, 64)).astype(np.float32) for _ in range(3))
    P = O.port()
    ref = P.attention(q, k, v, True)
    sess = gpu.AttentionSession(130, 64, causal=True)
    close_enough(ref, sess.forward(q, k, v), 1e-4, 1e-4)
    # resident call: nothing uploaded, inputs reused from the session buffers
    pol = gpu.default_attention_policy()
    pol.upload_q = pol.upload_k = pol.upload_v = 0
    pol.synchronize = 1
    out = np.empty_like(q)
    sess.forward_with_policy(None, None, None, out, pol)
    close_enough(ref, out, 1e-4, 1e-4)
    # postprocess through the session policy
    pol.output_scale, pol.output_bias, pol.output_relu = 0.5, -0.1, 1
    sess.forward_with_policy(None, None, None, out, pol)
    close_enough(np.maximum(ref * 0.5 - 0.1, 0), out, 1e-4, 1e-4)
    sess.close()


@pytest.mark.gpu
def test_matmul_resident_loop(gpu):
    rng = np.random.default_rng(1)
    a = rng.uniform(-1, 1, (96, 200)).astype(np.float32)
    b = rng.uniform(-1, 1, (200, 72)).astype(np.float32)
    ref = O.port().matmul(a, b)
    s = gpu.MatMulResidentSession(96, 200, 72)
    s.start(a, b)
    for _ in range(3):
        s.run()
    s.sync()
    close_enough(ref, s.finish(), 1e-4, 1e-4)
    close_enough(ref, s.run_batch_sync(None, None, 5), 1e-4, 1e-4)  # cached inputs
    a2 = rng.uniform(-1, 1, (96, 200)).astype(np.float32)
    close_enough(O.port().matmul(a2, b), s.run_batch_sync(a2, None, 2), 1e-4, 1e-4)
    s.close()


@pytest.mark.gpu
def test_attention_session_shared_by_four_threads(gpu):
    rng = np.random.default_rng(2)
    s_len, d = 64, 32
    sess = gpu.AttentionSession(s_len, d)
    inputs = [tuple(rng.standard_normal((s_len, d)).astype(np.float32) for _ in range(3)) for _ in range(4)]
    P = O.port()
    refs = [P.attention(*x) for x in inputs]
    errors = []

    def worker(i):
        try:
            for _ in range(20):
                close_enough(refs[i], sess.forward(*inputs[i]), 1e-4, 1e-4)
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    th = [threading.Thread(target=worker, args=(i,)) for i in range(4)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    assert not errors, errors[0]
