"""The oracle (oracle/lc_oracle.c) against the reference's own known answers and against the
golden fixtures produced by the reference itself (tests/golden/make_golden.py)."""
import numpy as np
import pytest

from conftest import close_enough, golden
from oracle import oracle as O


@pytest.fixture(scope="module")
def P():
    return O.port()


def test_attention_kat(P):
    # tests/test_attention.cpp:49-68 of the reference, tolerance 0.05
    g = golden("kat_attn")
    out = P.attention(g["q"], g["k"], g["v"])
    close_enough([[6.6976, 6.6048], [3.3024, 13.3952]], out, 0.05, 0)
    close_enough(g["out"], out, 1e-6, 1e-6)


def test_attention_postprocess_kat(P):
    # tests/test_attention.cpp:70-92: scale 0.5, bias -2, ReLU
    g = golden("kat_attn_post")
    out = P.attention(g["q"], g["k"], g["v"], scale=0.5, bias=-2.0, relu=True)
    close_enough(g["out"], out, 1e-6, 1e-6)
    assert out.min() >= 0.0


def test_matmul_kat(P):
    g = golden("kat_matmul")
    out = P.matmul(g["a"], g["b"])
    np.testing.assert_array_equal(out, [[58, 64], [139, 154]])
    np.testing.assert_array_equal(out, g["out"])


@pytest.mark.parametrize("name,atol,rtol", [("parity_matmul", 1e-6, 1e-6), ("cfg2_matmul_128x256x96", 1e-5, 1e-5),
                                            ("cfg4_gemm_bf16in_192x256x264", 1e-6, 1e-5)])
def test_matmul_golden(P, name, atol, rtol):
    g = golden(name)
    close_enough(g["out"], P.matmul(g["a"], g["b"]), atol, rtol)


@pytest.mark.parametrize("name", ["parity_attention", "cfg1_attention_256x64"])
def test_attention_golden(P, name):
    g = golden(name)
    close_enough(g["out"], P.attention(g["q"], g["k"], g["v"]), 1e-5, 1e-5)


def test_attention_causal_units_golden(P):
    g = golden("cfg3_causal_bf16in_2x200x128")
    full = P.attention_units(g["q"], g["k"], g["v"], causal=True, threads=2)
    close_enough(g["out"], full, 1e-5, 1e-5)
    # row sampling is the same arithmetic as the full head
    rows = P.attention_rows(g["q"][1], g["k"][1], g["v"][1], True, 50, 120)
    np.testing.assert_array_equal(full[1][50:120], rows)


def test_vector_add_golden(P):
    g = golden("parity_vector_add")
    np.testing.assert_array_equal(P.vector_add(g["a"], g["b"]), g["out"])


@pytest.mark.parametrize("name,stride,pad,relu", [("parity_conv", (1, 1), (1, 1), False),
                                                  ("conv_stride2_pad0", (2, 1), (0, 1), True)])
def test_conv_golden(P, name, stride, pad, relu):
    g = golden(name)
    close_enough(g["out"], P.conv2d(g["x"], g["w"], g["bias"], stride, pad, relu), 1e-6, 1e-6)


def test_conv_attention_golden(P):
    g = golden("cfg5_conv_attention_2x8x12x12")
    out = P.conv_attention_images(g["x"], g["w"], g["bias"], g["proj_w"], 144, 16, threads=2)
    close_enough(g["out"], out, 1e-5, 1e-5)
    out = P.conv_attention_images(g["x"], g["w"], g["bias"], None, 144, 16, threads=2)
    close_enough(g["out_noproj"], out, 1e-5, 1e-5)


def test_conv_attention_repeat_golden(P):
    g = golden("conv_attention_repeat")
    close_enough(g["out"], P.conv_attention_images(g["x"], g["w"], None, None, 40, 4, threads=1), 1e-5, 1e-5)


def test_layer_norm_formula(P):
    # README.md:2267-2270 (numpy formula) restated in float64
    x = np.random.default_rng(7).standard_normal((33, 100)).astype(np.float32)
    x64 = x.astype(np.float64)
    ref = (x64 - x64.mean(-1, keepdims=True)) / np.sqrt(x64.var(-1, keepdims=True) + 1e-5)
    close_enough(ref, P.layer_norm(x), 1e-5, 1e-5)


@pytest.mark.parametrize("name", ["ln_readme_16x1024", "ln_readme_5x333"])
def test_layer_norm_readme_golden(P, name):
    # Fixtures from the reference's own `_layer_norm_np` (README.md:2267-2270), run by
    # tests/golden/make_golden.py on np.random.rand-style inputs; numpy reduces in float32.
    g = golden(name)
    close_enough(g["out"], P.layer_norm(g["x"]), 2e-5, 2e-5)


def test_bf16_round(P):
    x = np.array([1.0, 1.00390625, 1.01171875, -3.14159, 65504.0, 1e-30], np.float32)
    r = P.bf16_round(x)
    u = r.view(np.uint32)
    assert np.all((u & 0xFFFF) == 0)
    assert r[1] == 1.0  # tie -> even
    assert r[2] == np.float32(1.015625)


@pytest.mark.skipif(not O.ref_available(), reason="reference not built here")
def test_port_matches_reference_random(P):
    R = O.ref()
    rng = np.random.default_rng(11)
    for s, d, c in [(1, 8, 0), (77, 32, 1), (130, 128, 1)]:
        q, k, v = (rng.standard_normal((s, d)).astype(np.float32) for _ in range(3))
        close_enough(R.attention(q, k, v, c), P.attention(q, k, v, c), 1e-5, 1e-5)
    a = rng.uniform(-1, 1, (33, 70)).astype(np.float32)
    b = rng.uniform(-1, 1, (70, 19)).astype(np.float32)
    np.testing.assert_array_equal(R.matmul(a, b), P.matmul(a, b))


@pytest.mark.parametrize("causal", [0, 1])
def test_train_step_golden(P, causal):
    g = golden(f"train_step_64x32_c{causal}")
    out, v_new, loss = P.attention_train_step(g["q"], g["k"], g["v"], g["target"], float(g["lr"]), bool(causal))
    close_enough(g["out"], out, 1e-5, 1e-5)
    close_enough(g["v_new"], v_new, 1e-5, 1e-5)
    assert abs(loss - float(g["loss"])) <= 1e-5 * abs(float(g["loss"])) + 1e-6


def test_matrix_ops_golden(P):
    g = golden("parity_matrix_ops")
    np.testing.assert_array_equal(P.matrix_op("sub", g["a"], g["b"]), g["sub"])
    # the reference build (-ffast-math) divides approximately; its own parity tolerance is 2e-4
    close_enough(g["div"], P.matrix_op("div", g["a"], g["b"]), 2e-4, 2e-4)


def test_qkv_pack_repeat_matches_reference_loop():
    """oracle.qkv_pack_repeat against a literal restatement of the pack node's doubling copy
    (reference include/lightning_core/core/graph.hpp:3168-3185)."""
    rng = np.random.default_rng(11)
    for have, need in [(5, 4), (12, 4), (100, 7), (3, 50), (600, 100)]:
        flat = rng.standard_normal(have).astype(np.float32)
        total = 3 * need
        packed = np.zeros(total, np.float32)
        copied = min(have, total)
        packed[:copied] = flat[:copied]
        while copied < total:
            chunk = min(copied, total - copied)
            packed[copied:copied + chunk] = packed[:chunk]
            copied += chunk
        q, k, v = O.qkv_pack_repeat(flat, need)
        assert np.array_equal(np.concatenate([q, k, v]), packed)
