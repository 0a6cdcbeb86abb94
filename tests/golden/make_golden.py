"""Generates tests/golden/*.npz from the reference itself.

Runs the reference's own CPU path -- compiled in place from the reference sources by
`make -C oracle ref` into oracle/_ref/liblc_ref.so -- on the inputs of the reference's own tests
(tests/test_attention.cpp:49-92, tests/test_matmul.cpp:20-40, tests/test_backend_parity.cpp:12-249)
and on small seeded inputs shaped like the benchmark configs, and stores inputs and outputs.
The fixtures pin both the C restatement in oracle/ and the CUDA path; they are committed so
that machines without the reference sources (the GPU box) can still check against them.

    python tests/golden/make_golden.py      # needs oracle/_ref/liblc_ref.so
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))
from oracle import oracle as O  # noqa: E402


def make_value(i, scale=1.0):
    # tests/test_backend_parity.cpp:12-15
    return np.float32(np.int64((i * 37 + 11) % 97) - 48) * np.float32(scale)


def make_vec(n, scale=0.01, bias=0.0):
    # tests/test_backend_parity.cpp:17-23
    i = np.arange(n, dtype=np.int64)
    return (((i * 37 + 11) % 97 - 48).astype(np.float32) * np.float32(scale) + np.float32(bias)).astype(np.float32)


def bf16r(x):
    return O.port().bf16_round(np.ascontiguousarray(x, np.float32))


REF_ROOT = os.environ.get("LC_REF_ROOT", os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(HERE))),
                                                       "reference"))


def readme_layer_norm():
    """The reference's LN helper is Python inside its README's benchmark script
    (README.md:2267-2270, `_layer_norm_np`, used at :3779-3818): the function's own lines are
    taken from the README and executed as they stand, so the fixture comes from the reference's
    code, not from a restatement."""
    lines = open(os.path.join(REF_ROOT, "README.md"), encoding="utf-8").read().splitlines()
    start = next(i for i, ln in enumerate(lines) if ln.startswith("def _layer_norm_np("))
    end = start + 1
    while end < len(lines) and (lines[end].startswith(("\t", " ")) or not lines[end].strip()):
        end += 1
    ns = {"np": np}
    exec("\n".join(lines[start:end]), ns)  # noqa: S102 - the reference's own helper
    return ns["_layer_norm_np"]


def main():
    R = O.ref()
    out = {}
    # LN helper: README shapes are [1024|2048, 1024] of np.random.rand; smaller row counts here.
    ln = readme_layer_norm()
    rng = np.random.default_rng(8)
    for rows, cols in ((16, 1024), (5, 333)):
        x = rng.random((rows, cols)).astype(np.float32)
        out[f"ln_readme_{rows}x{cols}"] = dict(x=x, out=ln(x.copy()))

    # --- reference known-answer tests ----------------------------------------------------
    q = np.array([[1, 0], [0, 1]], np.float32)
    v = np.array([[10, 0], [0, 20]], np.float32)
    out["kat_attn"] = dict(q=q, k=q, v=v, out=R.attention(q, q, v))
    out["kat_attn_post"] = dict(q=q, k=q, v=v, out=R.attention(q, q, v, scale=0.5, bias=-2.0, relu=True))
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    b = np.array([[7, 8], [9, 10], [11, 12]], np.float32)
    out["kat_matmul"] = dict(a=a, b=b, out=R.matmul(a, b))

    # --- test_backend_parity.cpp generator cases -------------------------------------------
    a = make_vec(4 * 7, 0.02).reshape(4, 7)
    b = make_vec(7 * 5, 0.015, 0.01).reshape(7, 5)
    out["parity_matmul"] = dict(a=a, b=b, out=R.matmul(a, b))
    a = make_vec(257, 0.005, 0.2)
    b = make_vec(257, 0.003, -0.1)
    out["parity_vector_add"] = dict(a=a, b=b, out=R.vector_add(a, b))
    # tests/test_backend_parity.cpp:113-155 (b pushed away from zero as there)
    a = make_vec(9 * 13, 0.01, 0.7).reshape(9, 13)
    b = make_vec(9 * 13, 0.008, 0.5).reshape(9, 13)
    b = np.where(np.abs(b) < 0.1, np.where(b < 0, -0.1, 0.1), b).astype(np.float32)
    out["parity_matrix_ops"] = dict(a=a, b=b, sub=R.matrix_op("sub", a, b), div=R.matrix_op("div", a, b))
    q = make_vec(16 * 32, 0.01).reshape(16, 32)
    k = make_vec(16 * 32, 0.009, 0.02).reshape(16, 32)
    v = make_vec(16 * 32, 0.008, -0.01).reshape(16, 32)
    out["parity_attention"] = dict(q=q, k=k, v=v, out=R.attention(q, k, v))
    x = make_vec(1 * 3 * 8 * 8, 0.01, 0.05).reshape(1, 3, 8, 8)
    w = make_vec(8 * 3 * 3 * 3, 0.01, -0.03).reshape(8, 3, 3, 3)
    bias = make_vec(8, 0.01, 0.02)
    out["parity_conv"] = dict(x=x, w=w, bias=bias, out=R.conv2d(x, w, bias, (1, 1), (1, 1), False))

    # --- seeded cases shaped like the benchmark configs ------------------------------------
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((256, 64)).astype(np.float32) for _ in range(3))
    out["cfg1_attention_256x64"] = dict(q=q, k=k, v=v, out=R.attention(q, k, v))
    rng = np.random.default_rng(1)
    a = rng.uniform(-1, 1, (128, 256)).astype(np.float32)
    b = rng.uniform(-1, 1, (256, 96)).astype(np.float32)
    out["cfg2_matmul_128x256x96"] = dict(a=a, b=b, out=R.matmul(a, b))
    rng = np.random.default_rng(2)
    q, k, v = (bf16r(rng.standard_normal((2, 200, 128))) for _ in range(3))
    out["cfg3_causal_bf16in_2x200x128"] = dict(q=q, k=k, v=v, out=R.attention_units(q, k, v, causal=True))
    rng = np.random.default_rng(3)
    a = bf16r(rng.uniform(-1, 1, (192, 256)) / 16.0)
    b = bf16r(rng.uniform(-1, 1, (256, 264)) / 16.0)
    out["cfg4_gemm_bf16in_192x256x264"] = dict(a=a, b=b, out=R.matmul(a, b))
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2, 8, 12, 12)).astype(np.float32)
    bound = np.sqrt(6.0 / (8 * 9))
    w = rng.uniform(-bound, bound, (24, 8, 3, 3)).astype(np.float32)
    bias = np.zeros(24, np.float32)
    pw = rng.uniform(-np.sqrt(6.0 / 16), np.sqrt(6.0 / 16), (16, 16)).astype(np.float32)
    out["cfg5_conv_attention_2x8x12x12"] = dict(
        x=x, w=w, bias=bias, proj_w=pw,
        out=R.conv_attention_images(x, w, bias, pw, seq=144, d=16, pad=(1, 1)),
        out_noproj=R.conv_attention_images(x, w, bias, None, seq=144, d=16, pad=(1, 1)))
    # short conv output -> cyclic repeat (bind_integrated.cpp:718-728)
    x = rng.standard_normal((1, 3, 5, 5)).astype(np.float32)
    w = rng.standard_normal((4, 3, 3, 3)).astype(np.float32)
    out["conv_attention_repeat"] = dict(
        x=x, w=w, out=R.conv_attention_images(x, w, None, None, seq=40, d=4, pad=(1, 1)))
    # strided / unpadded conv
    x = rng.standard_normal((2, 5, 9, 11)).astype(np.float32)
    w = rng.standard_normal((7, 5, 3, 2)).astype(np.float32)
    bias = rng.standard_normal(7).astype(np.float32)
    out["conv_stride2_pad0"] = dict(x=x, w=w, bias=bias, out=R.conv2d(x, w, bias, (2, 1), (0, 1), True))

    # train step (src/attention_cpu.cpp:114-163)
    rng = np.random.default_rng(6)
    q, k, v, t = (rng.standard_normal((64, 32)).astype(np.float32) for _ in range(4))
    for causal in (0, 1):
        o2, v2, loss = R.attention_train_step(q, k, v, t, 0.1, causal=bool(causal))
        out[f"train_step_64x32_c{causal}"] = dict(q=q, k=k, v=v, target=t, lr=np.float32(0.1), out=o2, v_new=v2,
                                                  loss=np.float32(loss))

    for name, d in out.items():
        np.savez(os.path.join(HERE, f"{name}.npz"), **d)
    print(f"wrote {len(out)} fixtures to {HERE}")


if __name__ == "__main__":
    main()
