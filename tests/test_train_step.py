"""Attention train step on the GPU (dV-only SGD with MSE loss, src/attention_cpu.cpp:114-163)
against the reference's own outputs (golden) and the oracle; loss cadence of
AttentionSession::trainStepWithPolicy (src/attention.cpp:301-343)."""
import ctypes as C

import numpy as np
import pytest

from conftest import close_enough, golden
from oracle import oracle as O

F32_TOL = (1e-4, 1e-4)


def test_train_step_rejects_bad_arguments(lc):
    x = np.zeros(16, np.float32).ctypes.data_as(C.c_void_p)
    L = lc.lib
    assert L.lcAttentionTrainStep(x, x, x, x, x, 0.0, 1, 4, 4, 0, None, None, None) == lc.LC_INVALID_VALUE
    assert L.lcAttentionTrainStep(x, x, x, None, x, 0.1, 1, 4, 4, 0, None, None, None) == lc.LC_INVALID_VALUE
    assert L.lcAttentionTrainStep(x, x, x, x, x, 0.1, 1, 4, 256, 0, None, None, None) == lc.LC_NOT_SUPPORTED


@pytest.mark.gpu
@pytest.mark.parametrize("causal", [0, 1])
def test_train_step_golden(gpu, causal):
    g = golden(f"train_step_64x32_c{causal}")
    out, v_new, loss = gpu.attention_train_step(g["q"], g["k"], g["v"], g["target"], float(g["lr"]), bool(causal))
    close_enough(g["out"], out, *F32_TOL)
    close_enough(g["v_new"], v_new, *F32_TOL)
    assert abs(loss - float(g["loss"])) <= 1e-4 * abs(float(g["loss"])) + 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("units,s,d,causal", [(3, 130, 64, 1), (2, 256, 128, 0), (1, 77, 40, 1)])
def test_train_step_batched_vs_oracle(gpu, units, s, d, causal):
    rng = np.random.default_rng(units + s)
    q, k, v, t = (rng.standard_normal((units, s, d)).astype(np.float32) for _ in range(4))
    out, v_new, loss = gpu.attention_train_step(q, k, v, t, 0.05, bool(causal))
    P = O.port()
    for u in range(units):
        o_ref, v_ref, l_ref = P.attention_train_step(q[u], k[u], v[u], t[u], 0.05, bool(causal))
        close_enough(o_ref, out[u], *F32_TOL)
        close_enough(v_ref, v_new[u], *F32_TOL)
        assert abs(loss[u] - l_ref) <= 1e-4 * abs(l_ref) + 1e-6


@pytest.mark.gpu
def test_session_training_reduces_loss_and_samples_it(gpu):
    # tests/test_attention.cpp of the reference: repeated train steps must lower the loss.
    rng = np.random.default_rng(3)
    q, k, v, t = (rng.standard_normal((256, 64)).astype(np.float32) for _ in range(4))
    sess = gpu.AttentionSession(256, 64)
    pol = gpu.default_attention_policy()
    pol.loss_every = 3
    _, first = sess.train_step(q, k, v, t, 0.5, pol)
    pol.upload_q = pol.upload_k = pol.upload_v = pol.upload_target = 0  # train the resident v
    pol.download_v = 0
    losses = [first]
    for _ in range(8):
        losses.append(sess.train_step(None, None, None, None, 0.5, pol)[1])
    # sampled every 3rd step; in between the last sampled value is repeated
    assert losses[1] == losses[0] and losses[2] == losses[0]
    assert losses[3] < losses[0] and losses[6] < losses[3]
    # the oracle run of the same 9 steps gives the same sampled losses
    P = O.port()
    vv = v.copy()
    ref = []
    for _ in range(9):
        _, vv, l = P.attention_train_step(q, k, vv, t, 0.5)
        ref.append(l)
    for i in (0, 3, 6):
        assert abs(losses[i] - ref[i]) <= 1e-4 * abs(ref[i])
