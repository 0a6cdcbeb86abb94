"""Test infrastructure only -- NOT the product path.

ctypes face over the two CPU checkers built by oracle/Makefile:

* ``port()``  -> liblc_oracle.so: our plain-C restatement of the reference CPU path.
* ``ref()``   -> _ref/liblc_ref.so: the reference's own CPU sources compiled in place, behind
  oracle/ref_shim.cpp.  Present wherever it was built (it travels with the repo snapshot).

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs import this module.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "liblc_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "liblc_ref.so")

_f = C.POINTER(C.c_float)
_sz = C.c_size_t


def _p(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(_f)


class _Lib:
    def __init__(self, path: str, prefix: str):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (run `make -C oracle {'ref' if prefix == 'ref' else 'oracle'}`)")
        self.lib = C.CDLL(path)
        self.prefix = prefix
        L, pfx = self.lib, prefix
        sig = {
            "attention_forward": [_f, _f, _f, _f, _sz, _sz, C.c_int, C.c_float, C.c_float, C.c_int],
            "matmul": [_f, _f, _f, _sz, _sz, _sz],
            "matmul_threads": [_f, _f, _f, _sz, _sz, _sz, C.c_int],
            "conv2d_nchw": [_f, _f, _f, _f] + [_sz] * 11 + [C.c_int],
            "vector_add": [_f, _f, _f, _sz],
            "attention_train_step": [_f, _f, _f, _f, _f, C.c_float, _sz, _sz, C.c_int, _f],
        }
        if pfx == "ref":
            sig["matrix_sub"] = [_f, _f, _f, _sz, _sz]
            sig["matrix_div"] = [_f, _f, _f, _sz, _sz]
            sig["attention_forward_units"] = [_f, _f, _f, _f, _sz, _sz, _sz, C.c_int, C.c_int]
            sig["conv_attention_images"] = [_f, _f, _f, _f, _f] + [_sz] * 14 + [C.c_int]
        else:
            sig["attention_units"] = [_f, _f, _f, _f, _sz, _sz, _sz, C.c_int, C.c_int]
            sig["attention_rows"] = [_f, _f, _f, _f, _sz, _sz, C.c_int, _sz, _sz]
            sig["conv_attention_images"] = [_f, _f, _f, _f, _f] + [_sz] * 14 + [C.c_int]
            sig["layer_norm"] = [_f, _f, _sz, _sz, C.c_float]
            sig["bf16_round_array"] = [_f, _f, _sz]
            sig["matrix_sub"] = [_f, _f, _f, _sz]
            sig["matrix_div"] = [_f, _f, _f, _sz]
        for name, args in sig.items():
            fn = getattr(L, f"{pfx}_{name}")
            fn.argtypes = args
            fn.restype = C.c_int if name not in ("vector_add", "layer_norm", "bf16_round_array", "matrix_sub",
                                                 "matrix_div") or pfx == "ref" else None

    def _call(self, name, *args):
        return getattr(self.lib, f"{self.prefix}_{name}")(*args)

    # -- attention -----------------------------------------------------------------------
    def attention(self, q, k, v, causal=False, scale=1.0, bias=0.0, relu=False):
        s, d = q.shape
        out = np.zeros((s, d), np.float32)
        rc = self._call("attention_forward", _p(q), _p(k), _p(v), _p(out), s, d, int(causal), scale, bias, int(relu))
        if rc:
            raise RuntimeError(f"attention rc={rc}")
        return out

    def attention_units(self, q, k, v, causal=False, threads=None):
        """q,k,v: [units, seq, d] fp32 -> out [units, seq, d]."""
        u, s, d = q.shape
        out = np.zeros_like(q)
        fn = "attention_forward_units" if self.prefix == "ref" else "attention_units"
        rc = self._call(fn, _p(q), _p(k), _p(v), _p(out), u, s, d, int(causal), threads or os.cpu_count())
        if rc:
            raise RuntimeError(f"attention_units rc={rc}")
        return out

    def attention_rows(self, q, k, v, causal, row0, row1):
        s, d = q.shape
        out = np.zeros((row1 - row0, d), np.float32)
        rc = self._call("attention_rows", _p(q), _p(k), _p(v), _p(out), s, d, int(causal), row0, row1)
        if rc:
            raise RuntimeError(f"attention_rows rc={rc}")
        return out

    def attention_train_step(self, q, k, v, target, lr, causal=False):
        s, d = q.shape
        v = v.copy()
        out = np.zeros((s, d), np.float32)
        loss = np.zeros(1, np.float32)
        rc = self._call("attention_train_step", _p(q), _p(k), _p(v), _p(target), _p(out), lr, s, d, int(causal),
                        _p(loss))
        if rc:
            raise RuntimeError(f"train rc={rc}")
        return out, v, float(loss[0])

    # -- matmul --------------------------------------------------------------------------
    def matmul(self, a, b, threads=1):
        m, k = a.shape
        k2, n = b.shape
        assert k == k2
        out = np.zeros((m, n), np.float32)
        if threads > 1:
            rc = self._call("matmul_threads", _p(a), _p(b), _p(out), m, k, n, threads)
        else:
            rc = self._call("matmul", _p(a), _p(b), _p(out), m, k, n)
        if rc:
            raise RuntimeError(f"matmul rc={rc}")
        return out

    # -- conv ----------------------------------------------------------------------------
    def conv2d(self, x, w, bias, stride=(1, 1), pad=(0, 0), relu=False):
        n, c, h, wd = x.shape
        oc, c2, kh, kw = w.shape
        assert c == c2
        oh = (h + 2 * pad[0] - kh) // stride[0] + 1
        ow = (wd + 2 * pad[1] - kw) // stride[1] + 1
        out = np.zeros((n, oc, oh, ow), np.float32)
        rc = self._call("conv2d_nchw", _p(x), _p(w), _p(bias), _p(out), n, c, h, wd, oc, kh, kw, stride[0],
                        stride[1], pad[0], pad[1], int(relu))
        if rc:
            raise RuntimeError(f"conv rc={rc}")
        return out

    def conv_attention_images(self, x, w, bias, proj_w, seq, d, stride=(1, 1), pad=(1, 1), threads=None):
        n, c, h, wd = x.shape
        oc, _, kh, kw = w.shape
        cols = proj_w.shape[1] if proj_w is not None else d
        out = np.zeros((n, seq, cols), np.float32)
        rc = self._call("conv_attention_images", _p(x), _p(w), _p(bias), _p(proj_w), _p(out), n, c, h, wd, oc, kh,
                        kw, stride[0], stride[1], pad[0], pad[1], seq, d, cols, threads or os.cpu_count())
        if rc:
            raise RuntimeError(f"conv_attention rc={rc}")
        return out

    # -- elementwise ----------------------------------------------------------------------
    def vector_add(self, a, b):
        out = np.zeros_like(a)
        self._call("vector_add", _p(a), _p(b), _p(out), a.size)
        return out

    def matrix_op(self, op, a, b):
        out = np.zeros_like(a)
        if self.prefix == "ref":
            rc = self._call(f"matrix_{op}", _p(a), _p(b), _p(out), a.shape[0], a.size // a.shape[0])
            if rc:
                raise RuntimeError(f"matrix_{op} rc={rc}")
        else:
            self._call(f"matrix_{op}", _p(a), _p(b), _p(out), a.size)
        return out

    def layer_norm(self, x, eps=1e-5):
        out = np.zeros_like(x)
        self._call("layer_norm", _p(x), _p(out), x.shape[0], x.shape[1], eps)
        return out

    def bf16_round(self, x):
        out = np.zeros_like(x)
        self._call("bf16_round_array", _p(x), _p(out), x.size)
        return out


_cache: dict = {}


def qkv_pack_repeat(flat, need):
    """The graph's kQkvPackRepeat node (reference include/lightning_core/core/graph.hpp:3138-3185):
    the first 3*need floats of `flat`, repeated cyclically when shorter, split into Q, K, V."""
    flat = np.asarray(flat, np.float32).reshape(-1)
    total = 3 * need
    reps = -(-total // flat.size)
    packed = np.tile(flat, reps)[:total]
    return packed[:need], packed[need:2 * need], packed[2 * need:]


def port() -> _Lib:
    if "port" not in _cache:
        _cache["port"] = _Lib(PORT_SO, "orc")
    return _cache["port"]


def ref() -> _Lib:
    if "ref" not in _cache:
        _cache["ref"] = _Lib(REF_SO, "ref")
    return _cache["ref"]


def ref_available() -> bool:
    return os.path.exists(REF_SO)
