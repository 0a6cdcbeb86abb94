"""Python face of liblc_b200.so -- the B200 build of Lightning Core's attention / matmul2d /
conv->attention hot path.

Mirrors the reference's pybind surface for that path (python/bindings/bind_attention.cpp:298-366,
bind_ops.cpp:728-760 and 1164-1210, bind_integrated.cpp:958-1140): same function names, argument
meaning and errors (ValueError for bad shapes, RuntimeError carrying lcGetErrorString for a
failed status).  The only device is "cuda"; there is no CPU compute path, so "cpu"/"metal"
raise ValueError.  The library must be built (``make -C lightining-core_b200``); importing this
module without it raises ImportError -- nothing falls back to NumPy.

bf16 tensors are passed as ``numpy.uint16`` arrays holding the bf16 bit patterns
(see :func:`to_bf16` / :func:`from_bf16`).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_PKG_ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
LIB_PATH = os.environ.get("LC_B200_LIB") or os.path.join(_PKG_ROOT, "liblc_b200.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is not built; run `make -C {_PKG_ROOT}`")

lib = C.CDLL(LIB_PATH)

# ---- enums (include/lc_b200.h) ---------------------------------------------------------------
LC_SUCCESS, LC_NOT_INITIALIZED, LC_INVALID_VALUE, LC_OUT_OF_MEMORY, LC_NOT_SUPPORTED, LC_DRIVER_ERROR, LC_UNKNOWN = range(7)
H2H, H2D, D2H, D2D = range(4)
F32, BF16, F64 = 0, 1, 2
LOOP_START, LOOP_RUN, LOOP_FINISH, LOOP_SYNC = range(4)
TUNE_MATMUL, TUNE_ATTENTION, TUNE_CONV = 0, 1, 2


class AttentionIoPolicy(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("upload_q", "upload_k", "upload_v", "upload_target", "download_out",
                                       "download_v", "synchronize", "loss_every")] + [
        ("output_scale", C.c_float), ("output_bias", C.c_float), ("output_relu", C.c_int)]


class MatMulIoPolicy(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("upload_a", "upload_b", "download_out", "synchronize")]


class VectorAddIoPolicy(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("upload_a", "upload_b", "download_out", "synchronize")]


class Conv2dIoPolicy(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("upload_x", "upload_w", "upload_bias", "download_out", "synchronize")]


class RuntimeTraceEvent(C.Structure):
    _fields_ = [("type", C.c_int), ("status", C.c_int), ("timestamp_ns", C.c_uint64), ("size_bytes", C.c_size_t),
                ("detail0", C.c_int), ("detail1", C.c_int)]


_vp, _sz, _i, _f = C.c_void_p, C.c_size_t, C.c_int, C.c_float
_SIGS = {
    "lcMalloc": (_i, [C.POINTER(_vp), _sz]),
    "lcFree": (_i, [_vp]),
    "lcMemcpy": (_i, [_vp, _vp, _sz, _i]),
    "lcDeviceSynchronize": (_i, []),
    "lcGetDeviceCount": (_i, [C.POINTER(_i)]),
    "lcIsCudaAvailable": (_i, []),
    "lcIsMetalAvailable": (_i, []),
    "lcGetApiVersionString": (C.c_char_p, []),
    "lcGetApiVersion": (_i, [C.POINTER(_i)] * 3),
    "lcGetErrorString": (C.c_char_p, [_i]),
    "lcBackendName": (C.c_char_p, []),
    "lcGetStructSize": (_sz, [_i]),
    "lcCheckStructSize": (_i, [_i, _sz]),
    "lcGetMemoryModel": (_i, []),
    "lcGetMemoryModelName": (C.c_char_p, [_i]),
    "lcAttentionIoPolicyDefault": (None, [C.POINTER(AttentionIoPolicy)]),
    "lcMatMulIoPolicyDefault": (None, [C.POINTER(MatMulIoPolicy)]),
    "lcConv2dIoPolicyDefault": (None, [C.POINTER(Conv2dIoPolicy)]),
    "lcVectorAddIoPolicyDefault": (None, [C.POINTER(VectorAddIoPolicy)]),
    "lcMatMulPolicyForStage": (None, [_i, C.POINTER(MatMulIoPolicy)]),
    "lcVectorPolicyForStage": (None, [_i, C.POINTER(VectorAddIoPolicy)]),
    "lcElemwisePolicyForStage": (None, [_i, C.POINTER(VectorAddIoPolicy)]),
    "lcAttentionPolicyForStage": (None, [_i, _i, C.POINTER(AttentionIoPolicy)]),
    "lcAttentionForward": (_i, [_vp, _vp, _vp, _vp, _sz, _sz, _sz, _i, _i, C.POINTER(AttentionIoPolicy), _vp]),
    "lcMatMul": (_i, [_vp, _vp, _vp, _sz, _sz, _sz, _i, C.POINTER(MatMulIoPolicy), _vp]),
    "lcConv2dNchw": (_i, [_vp, _vp, _vp, _vp] + [_sz] * 11 + [_i, C.POINTER(Conv2dIoPolicy), _vp]),
    "lcConvAttentionNchw": (_i, [_vp] * 5 + [_sz] * 14 + [_i, C.POINTER(Conv2dIoPolicy), _vp]),
    "lcAttentionProjForward": (_i, [_vp] * 5 + [_sz] * 4 + [_i, _i, C.POINTER(AttentionIoPolicy), _vp]),
    "lcAttentionQkvProjForward": (_i, [_vp, _sz, _vp, _vp, _sz, _sz, _sz, C.POINTER(AttentionIoPolicy), _vp]),
    "lcVectorAdd": (_i, [_vp, _vp, _vp, _sz, _i, C.POINTER(VectorAddIoPolicy), _vp]),
    "lcLayerNorm": (_i, [_vp, _vp, _sz, _sz, _f, _vp]),
    "lcGetDeviceErrorWord": (_i, [C.POINTER(C.c_uint)]),
    "lcClearDeviceErrorWord": (_i, []),
    "lcRuntimeTraceSetEnabled": (None, [_i]),
    "lcRuntimeTraceIsEnabled": (_i, []),
    "lcRuntimeTraceClear": (None, []),
    "lcRuntimeTraceCount": (_sz, []),
    "lcRuntimeTraceCapacity": (_sz, []),
    "lcRuntimeTraceGet": (_i, [_sz, C.POINTER(RuntimeTraceEvent)]),
    "lcMatrixSub": (_i, [_vp, _vp, _vp, _sz, _sz, _i, C.POINTER(VectorAddIoPolicy), _vp]),
    "lcMatrixDiv": (_i, [_vp, _vp, _vp, _sz, _sz, _i, C.POINTER(VectorAddIoPolicy), _vp]),
    "lcTuneCacheLoad": (_i, [_i, C.c_char_p]),
    "lcTuneCacheSave": (_i, [_i, C.c_char_p]),
    "lcTuneCacheReset": (_i, [_i]),
    "lcTuneCacheSize": (_sz, [_i]),
    "lcTuneCacheGet": (_i, [_i, _sz, _sz, _sz, _i, C.c_char_p, _sz]),
    "lcTuneCacheSet": (_i, [_i, _sz, _sz, _sz, _i, C.c_char_p]),
    "lcMatMulAutotune": (_i, [_vp, _vp, _vp, _sz, _sz, _sz, _i, _vp, C.c_char_p, _sz]),
    "lcAttentionAutotune": (_i, [_vp, _vp, _vp, _vp, _sz, _sz, _sz, _i, _i, _vp, C.c_char_p, _sz]),
    "lcConvAttentionNchwNoAlloc": (_i, [_vp] * 5 + [_sz] * 14 + [_i, _vp]),
    "lcAttentionSessionCreate": (_i, [C.POINTER(_vp), _sz, _sz, _sz, _i, _i]),
    "lcAttentionSessionDestroy": (_i, [_vp]),
    "lcAttentionSessionSetDefaultPolicy": (_i, [_vp, C.POINTER(AttentionIoPolicy)]),
    "lcAttentionSessionBuffer": (_i, [_vp, _i, C.POINTER(_vp)]),
    "lcAttentionSessionForward": (_i, [_vp, _vp, _vp, _vp, _vp, C.POINTER(AttentionIoPolicy), _vp]),
    "lcMatMulSessionCreate": (_i, [C.POINTER(_vp), _sz, _sz, _sz, _i]),
    "lcMatMulSessionDestroy": (_i, [_vp]),
    "lcMatMulSessionBuffer": (_i, [_vp, _i, C.POINTER(_vp)]),
    "lcMatMulSessionRun": (_i, [_vp, _vp, _vp, _vp, C.POINTER(MatMulIoPolicy), _vp]),
    "lcMatMulSessionRunBatch": (_i, [_vp, _vp, _vp, _vp, _sz, _vp]),
    "lcAttentionTrainStep": (_i, [_vp] * 5 + [_f, _sz, _sz, _sz, _i, _vp, C.POINTER(AttentionIoPolicy), _vp]),
    "lcAttentionSessionTrainStep": (_i, [_vp] * 6 + [_f, _vp, C.POINTER(AttentionIoPolicy), _vp]),
    "lcTestFailAllocations": (None, [_i, _i]),
    "lcTestStallNextGemm": (None, [_i]),
    "lcConvTuneKey": (_i, [_sz] * 11 + [C.POINTER(_sz)] * 3),
    "lcConvAutotune": (_i, [_vp] * 4 + [_sz] * 11 + [_i, _vp, C.c_char_p, _sz]),
    "lcCommAvailable": (_i, []),
    "lcCommGetUniqueId": (_i, [_vp]),
    "lcCommInitRank": (_i, [C.POINTER(_vp), _i, _vp, _i]),
    "lcCommDestroy": (_i, [_vp]),
    "lcCommAbort": (_i, [_vp]),
    "lcCommRankInfo": (_i, [_vp, C.POINTER(_i), C.POINTER(_i)]),
    "lcShardRange": (_i, [_sz, _i, _i, C.POINTER(_sz), C.POINTER(_sz)]),
    "lcCommAllGatherRows": (_i, [_vp, _vp, _sz, _sz, _vp]),
    "lcAttentionForwardSharded": (_i, [_vp] * 5 + [_sz, _sz, _sz, _i, _i, C.POINTER(AttentionIoPolicy), _vp]),
    "lcMatMulSharded": (_i, [_vp] * 4 + [_sz, _sz, _sz, _i, C.POINTER(MatMulIoPolicy), _vp]),
    "lcConvAttentionNchwSharded": (_i, [_vp] * 6 + [_sz] * 14 + [C.POINTER(Conv2dIoPolicy), _vp]),
}
for _name, (_res, _args) in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


class LightningError(RuntimeError):
    def __init__(self, code: int, what: str = ""):
        self.code = code
        msg = lib.lcGetErrorString(code).decode()
        super().__init__(f"{what}: {msg}" if what else msg)


def check(code: int, what: str = "") -> None:
    if code != LC_SUCCESS:
        raise LightningError(code, what)


def cuda_available() -> bool:
    return bool(lib.lcIsCudaAvailable())


def api_version() -> str:
    return lib.lcGetApiVersionString().decode()


# ---- bf16 helpers ---------------------------------------------------------------------------
def to_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7F800000) == 0x7F800000
    nan &= (u & 0x007FFFFF) != 0
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def from_bf16(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---- device memory --------------------------------------------------------------------------
class DeviceBuffer:
    """A cudaMalloc'd buffer owned from Python (lcMalloc / lcFree)."""

    def __init__(self, nbytes: int):
        self.nbytes = int(nbytes)
        self.ptr = C.c_void_p()
        check(lib.lcMalloc(C.byref(self.ptr), max(1, self.nbytes)), "lcMalloc")

    @classmethod
    def from_array(cls, a: np.ndarray) -> "DeviceBuffer":
        a = np.ascontiguousarray(a)
        buf = cls(a.nbytes)
        buf.upload(a)
        return buf

    @property
    def value(self) -> int:
        return self.ptr.value

    def upload(self, a: np.ndarray) -> None:
        a = np.ascontiguousarray(a)
        assert a.nbytes <= self.nbytes
        check(lib.lcMemcpy(self.ptr, a.ctypes.data_as(C.c_void_p), a.nbytes, H2D), "lcMemcpy H2D")

    def download(self, shape, dtype) -> np.ndarray:
        out = np.empty(shape, dtype=dtype)
        check(lib.lcMemcpy(out.ctypes.data_as(C.c_void_p), self.ptr, out.nbytes, D2H), "lcMemcpy D2H")
        return out

    def free(self) -> None:
        if self.ptr is not None and self.ptr.value:
            lib.lcFree(self.ptr)
        self.ptr = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


# ---- reference-mirroring ops ------------------------------------------------------------------
def _parse_device(device: str) -> None:
    if device not in ("cuda", "gpu"):
        raise ValueError(f"device '{device}' is not served by the B200 build (only 'cuda'; no CPU path)")


def _f32(a, name):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a


def _vp(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _require_2d(a, name):
    if a.ndim != 2:
        raise ValueError(f"{name} must be a 2D float32 array shaped [seq_len, head_dim]")
    return a.shape


def attention2d_into(q, k, v, out, causal: bool = False, device: str = "cuda", policy: AttentionIoPolicy = None):
    """bind_attention.cpp:329-366: out[seq, d] = softmax(q k^T / sqrt(d)) v (host arrays)."""
    _parse_device(device)
    q, k, v = _f32(q, "q"), _f32(k, "k"), _f32(v, "v")
    s, d = _require_2d(q, "q")
    if _require_2d(k, "k") != (s, d) or _require_2d(v, "v") != (s, d):
        raise ValueError("q/k/v must have identical 2D shape [seq_len, head_dim]")
    if out.dtype != np.float32 or out.shape != (s, d) or not out.flags["C_CONTIGUOUS"]:
        raise ValueError("out must be a 2D float32 array shaped [seq_len, head_dim]")
    pol = policy or default_attention_policy()
    check(lib.lcAttentionForward(_vp(q), _vp(k), _vp(v), _vp(out), 1, s, d, int(causal), F32, C.byref(pol), None),
          "attention2d")
    return out


def attention2d(q, k, v, causal: bool = False, device: str = "cuda", policy: AttentionIoPolicy = None):
    """bind_attention.cpp:298-327."""
    q = _f32(q, "q")
    if q.ndim != 2:
        raise ValueError("q must be a 2D float32 array shaped [seq_len, head_dim]")
    out = np.empty(q.shape, np.float32)
    return attention2d_into(q, k, v, out, causal, device, policy)


def attention_batched(q, k, v, causal: bool = False, dtype: int = F32):
    """Host [units, seq, d] arrays (float32, or uint16 bf16 bits with dtype=BF16)."""
    q = np.ascontiguousarray(q)
    units, s, d = q.shape
    out = np.empty_like(q)
    pol = default_attention_policy()
    check(lib.lcAttentionForward(_vp(q), _vp(np.ascontiguousarray(k)), _vp(np.ascontiguousarray(v)), _vp(out),
                                 units, s, d, int(causal), dtype, C.byref(pol), None), "attention")
    return out


def attention_proj(q, k, v, proj_w, causal: bool = False, dtype: int = F32):
    """Graph fused node attention_proj_v1 (graph.hpp:3454-3555): attention(q, k, v) @ proj_w.

    q, k, v: host [seq, d] or [units, seq, d]; proj_w [d, cols]; float32, or uint16 bf16 bits with
    dtype=BF16.  Returns [.., seq, cols]."""
    q = np.ascontiguousarray(q)
    squeeze = q.ndim == 2
    q3 = q[None] if squeeze else q
    units, s, d = q3.shape
    proj_w = np.ascontiguousarray(proj_w)
    if proj_w.ndim != 2 or proj_w.shape[0] != d:
        raise ValueError("proj_w must be [head_dim, cols]")
    cols = proj_w.shape[1]
    out = np.empty((units, s, cols), dtype=q.dtype)
    pol = default_attention_policy()
    check(lib.lcAttentionProjForward(_vp(q3), _vp(np.ascontiguousarray(k)), _vp(np.ascontiguousarray(v)),
                                     _vp(proj_w), _vp(out), units, s, d, cols, int(causal), dtype, C.byref(pol),
                                     None), "attention_proj")
    return out[0] if squeeze else out


def attention_qkv_proj(packed, proj_w, seq_len: int, head_dim: int):
    """Graph fused node attention_qkv_proj_v1 (graph.hpp:3138-3185, 3556-3584): Q, K, V are the
    consecutive [seq, d] slices of the flat `packed` float32 input (repeated cyclically when
    short), then attention and the projection.  Returns [seq, cols] float32."""
    packed = np.ascontiguousarray(packed, dtype=np.float32).reshape(-1)
    proj_w = np.ascontiguousarray(proj_w, dtype=np.float32)
    if proj_w.ndim != 2 or proj_w.shape[0] != head_dim:
        raise ValueError("proj_w must be [head_dim, cols]")
    out = np.empty((seq_len, proj_w.shape[1]), np.float32)
    pol = default_attention_policy()
    check(lib.lcAttentionQkvProjForward(_vp(packed), packed.size, _vp(proj_w), _vp(out), seq_len, head_dim,
                                        proj_w.shape[1], C.byref(pol), None), "attention_qkv_proj")
    return out


def default_attention_policy() -> AttentionIoPolicy:
    p = AttentionIoPolicy()
    lib.lcAttentionIoPolicyDefault(C.byref(p))
    return p


def default_matmul_policy() -> MatMulIoPolicy:
    p = MatMulIoPolicy()
    lib.lcMatMulIoPolicyDefault(C.byref(p))
    return p


def matmul_policy_for_stage(stage: int) -> MatMulIoPolicy:
    p = MatMulIoPolicy()
    lib.lcMatMulPolicyForStage(stage, C.byref(p))
    return p


def matmul2d_into(a, b, out, device: str = "cuda", dtype: int = F32):
    """bind_ops.cpp:1187-1210."""
    _parse_device(device)
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    if a.ndim != 2 or b.ndim != 2:
        raise ValueError("matmul2d expects 2D arrays")
    m, kk = a.shape
    if b.shape[0] != kk:
        raise ValueError("matmul2d_into shape mismatch: a.shape[1] must equal b.shape[0]")
    n = b.shape[1]
    if out.size != m * n or not out.flags["C_CONTIGUOUS"]:
        raise ValueError("out must be [m, n] or flat m*n")
    pol = default_matmul_policy()
    check(lib.lcMatMul(_vp(a), _vp(b), _vp(out), m, kk, n, dtype, C.byref(pol), None), "matmul2d")
    return out


def matmul2d(a, b, device: str = "cuda", dtype: int = F32):
    """bind_ops.cpp:1164-1185 (float32), or bf16 bits (uint16) with dtype=BF16."""
    if dtype == F32:
        a = _f32(a, "a")
        b = _f32(b, "b")
    if np.ndim(a) != 2 or np.ndim(b) != 2:
        raise ValueError("matmul2d expects 2D arrays")
    if a.shape[1] != b.shape[0]:
        raise ValueError("matmul2d shape mismatch: a.shape[1] must equal b.shape[0]")
    out = np.empty((a.shape[0], b.shape[1]), np.float32 if dtype == F32 else np.uint16)
    return matmul2d_into(a, b, out, device, dtype)


def _conv_dims(x, w, stride_h, stride_w, pad_h, pad_w):
    if x.ndim != 4 or w.ndim != 4:
        raise ValueError("x and w must be 4D arrays (NCHW and OIHW)")
    n, c, h, wd = x.shape
    oc, wc, kh, kw = w.shape
    if c != wc:
        raise ValueError("x channels and w in_channels mismatch")
    if stride_h == 0 or stride_w == 0:
        raise ValueError("stride must be > 0")
    if h + 2 * pad_h < kh or wd + 2 * pad_w < kw:
        raise ValueError("invalid padding/kernel for input size")
    return n, c, h, wd, oc, kh, kw, (h + 2 * pad_h - kh) // stride_h + 1, (wd + 2 * pad_w - kw) // stride_w + 1


def conv2d_nchw(x, w, bias=None, stride_h=1, stride_w=1, pad_h=0, pad_w=0, device="cuda", apply_relu=False):
    """bind_ops.cpp:728-800 (+ the apply_relu flag of ops::conv2dNchw)."""
    _parse_device(device)
    x, w = _f32(x, "x"), _f32(w, "w")
    n, c, h, wd, oc, kh, kw, oh, ow = _conv_dims(x, w, stride_h, stride_w, pad_h, pad_w)
    if bias is not None:
        bias = _f32(bias, "bias")
        if bias.size != oc:
            raise ValueError("bias shape mismatch")
    out = np.empty((n, oc, oh, ow), np.float32)
    pol = Conv2dIoPolicy()
    lib.lcConv2dIoPolicyDefault(C.byref(pol))
    check(lib.lcConv2dNchw(_vp(x), _vp(w), _vp(bias), _vp(out), n, c, h, wd, oc, kh, kw, stride_h, stride_w, pad_h,
                           pad_w, int(apply_relu), C.byref(pol), None), "conv2d_nchw")
    return out


def lightning_conv_attention_torchstrong_nchw_into(x, w, bias, out, seq_len, head_dim, stride_h=1, stride_w=1,
                                                   pad_h=0, pad_w=0, device="cuda", execution_mode="eager",
                                                   proj_w=None, per_image=False):
    """bind_integrated.cpp:614-730 (+ optional projection, graph.hpp:3529-3547).

    per_image=False keeps the reference's batch semantics (one attention over the first
    3*seq*d floats of the flat conv output); per_image=True runs them on each image."""
    _parse_device(device)
    if execution_mode not in ("eager", "graph"):
        raise ValueError("execution_mode must be 'eager' or 'graph'")
    x, w = _f32(x, "x"), _f32(w, "w")
    n, c, h, wd, oc, kh, kw, oh, ow = _conv_dims(x, w, stride_h, stride_w, pad_h, pad_w)
    if bias is not None:
        bias = _f32(bias, "bias")
        if bias.size != oc:
            raise ValueError("bias shape mismatch")
    cols = head_dim
    if proj_w is not None:
        proj_w = _f32(proj_w, "proj_w")
        if proj_w.ndim != 2 or proj_w.shape[0] != head_dim:
            raise ValueError("proj_w must be [head_dim, out_cols]")
        cols = proj_w.shape[1]
    units = n if per_image else 1
    if out.dtype != np.float32 or out.size != units * seq_len * cols or not out.flags["C_CONTIGUOUS"]:
        raise ValueError("out size mismatch")
    pol = Conv2dIoPolicy()
    lib.lcConv2dIoPolicyDefault(C.byref(pol))
    check(lib.lcConvAttentionNchw(_vp(x), _vp(w), _vp(bias), _vp(proj_w), _vp(out), n, c, h, wd, oc, kh, kw,
                                  stride_h, stride_w, pad_h, pad_w, seq_len, head_dim, cols, int(per_image),
                                  C.byref(pol), None), "conv_attention")
    return out


def lightning_conv_attention_torchstrong_nchw(x, w, bias, seq_len, head_dim, stride_h=1, stride_w=1, pad_h=0,
                                              pad_w=0, device="cuda", execution_mode="eager", proj_w=None,
                                              per_image=False):
    """bind_integrated.cpp:958-1140: returns the flat [seq*cols] (or [batch, seq, cols]) result."""
    cols = head_dim if proj_w is None else np.shape(proj_w)[1]
    units = np.shape(x)[0] if per_image else 1
    out = np.empty(units * seq_len * cols, np.float32)
    lightning_conv_attention_torchstrong_nchw_into(x, w, bias, out, seq_len, head_dim, stride_h, stride_w, pad_h,
                                                   pad_w, device, execution_mode, proj_w, per_image)
    return out.reshape(units, seq_len, cols) if per_image else out


def vector_add(a, b, device="cuda"):
    """bind_ops.cpp:1098-1125 (float32 or float64)."""
    _parse_device(device)
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    if a.shape != b.shape or a.dtype != b.dtype or a.dtype not in (np.float32, np.float64):
        raise ValueError("vector_add expects two same-shape float32/float64 arrays")
    out = np.empty_like(a)
    pol = VectorAddIoPolicy()
    lib.lcVectorAddIoPolicyDefault(C.byref(pol))
    check(lib.lcVectorAdd(_vp(a), _vp(b), _vp(out), a.size, F32 if a.dtype == np.float32 else F64, C.byref(pol),
                          None), "vector_add")
    return out


def _matrix_op(fn, name, a, b, rows, cols, device):
    _parse_device(device)
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    if a.size != rows * cols or b.size != rows * cols or a.dtype != b.dtype or a.dtype not in (np.float32,
                                                                                            np.float64):
        raise ValueError(f"{name}: a and b must be float32/float64 arrays of rows*cols elements")
    out = np.empty_like(a)
    pol = VectorAddIoPolicy()
    lib.lcVectorAddIoPolicyDefault(C.byref(pol))
    check(fn(_vp(a), _vp(b), _vp(out), rows, cols, F32 if a.dtype == np.float32 else F64, C.byref(pol), None), name)
    return out


def matrix_sub(a, b, rows, cols, device="cuda"):
    """bind_ops.cpp:1126-1160: out = a - b over rows x cols."""
    return _matrix_op(lib.lcMatrixSub, "matrix_sub", a, b, rows, cols, device)


def matrix_div(a, b, rows, cols, device="cuda"):
    """out = a / b over rows x cols (IEEE division)."""
    return _matrix_op(lib.lcMatrixDiv, "matrix_div", a, b, rows, cols, device)


def layer_norm(x, eps=1e-5):
    """The reference benchmark's LN (README.md:2267-2270) over the last axis, on the GPU."""
    x = _f32(x, "x")
    rows, cols = x.reshape(-1, x.shape[-1]).shape
    dx = DeviceBuffer.from_array(x)
    dy = DeviceBuffer(x.nbytes)
    check(lib.lcLayerNorm(dx.ptr, dy.ptr, rows, cols, eps, None), "layer_norm")
    check(lib.lcDeviceSynchronize(), "sync")
    return dy.download(x.shape, np.float32)


# ---- auto-tune cache ------------------------------------------------------------------------
def tune_cache_get(kind: int, d0: int, d1: int, d2: int, dtype: int = F32):
    buf = C.create_string_buffer(64)
    rc = lib.lcTuneCacheGet(kind, d0, d1, d2, dtype, buf, 64)
    return buf.value.decode() if rc == LC_SUCCESS else None


def tune_cache_set(kind: int, d0: int, d1: int, d2: int, config: str, dtype: int = F32) -> None:
    check(lib.lcTuneCacheSet(kind, d0, d1, d2, dtype, config.encode()), "tune_cache_set")


def tune_cache_reset(kind: int = TUNE_MATMUL) -> None:
    """Drops every entry of one cache (the reference's matMulMetalResetTuning)."""
    check(lib.lcTuneCacheReset(kind), "tune_cache_reset")


def matmul_autotune(a: "DeviceBuffer", b: "DeviceBuffer", out: "DeviceBuffer", m: int, k: int, n: int,
                    dtype: int = F32) -> str:
    buf = C.create_string_buffer(64)
    check(lib.lcMatMulAutotune(a.ptr, b.ptr, out.ptr, m, k, n, dtype, None, buf, 64), "matmul_autotune")
    return buf.value.decode()


def attention_autotune(q: "DeviceBuffer", k: "DeviceBuffer", v: "DeviceBuffer", out: "DeviceBuffer", units: int,
                       seq: int, head_dim: int, causal: bool = False, dtype: int = F32) -> str:
    """Times every attention kernel that can take the shape on device [units, seq, head_dim]
    buffers, stores the fastest in the attention tune cache and returns its name."""
    buf = C.create_string_buffer(64)
    check(lib.lcAttentionAutotune(q.ptr, k.ptr, v.ptr, out.ptr, units, seq, head_dim, int(causal), dtype, None, buf,
                                  64), "attention_autotune")
    return buf.value.decode()


# ---- sessions (AttentionSession / MatMulMetalResidentSession of the reference) ---------------
class AttentionSession:
    """attention.hpp:86-129: a shape-bound handle with device-resident q/k/v/out buffers."""

    def __init__(self, seq_len: int, head_dim: int, causal: bool = False, units: int = 1, dtype: int = F32):
        self.shape = (units, seq_len, head_dim) if units > 1 else (seq_len, head_dim)
        self.np_dtype = np.float32 if dtype == F32 else np.uint16
        self.h = C.c_void_p()
        check(lib.lcAttentionSessionCreate(C.byref(self.h), units, seq_len, head_dim, int(causal), dtype),
              "AttentionSession")

    def set_default_policy(self, policy: AttentionIoPolicy) -> None:
        check(lib.lcAttentionSessionSetDefaultPolicy(self.h, C.byref(policy)))

    def forward_with_policy(self, q, k, v, out, policy: AttentionIoPolicy):
        arrs = [None if x is None else np.ascontiguousarray(x, dtype=self.np_dtype) for x in (q, k, v)]
        check(lib.lcAttentionSessionForward(self.h, *[_vp(x) for x in arrs], _vp(out), C.byref(policy), None),
              "AttentionSession.forward")
        return out

    def forward(self, q, k, v):
        out = np.empty(self.shape, self.np_dtype)
        check(lib.lcAttentionSessionForward(self.h, *[_vp(np.ascontiguousarray(x, dtype=self.np_dtype))
                                                      for x in (q, k, v)], _vp(out), None, None),
              "AttentionSession.forward")
        lib.lcDeviceSynchronize()
        return out

    def train_step(self, q, k, v, target, learning_rate: float, policy: AttentionIoPolicy = None):
        """AttentionSession::trainStep (src/attention.cpp:285-343): returns (out, loss).  With the
        default policy q/k/v/target are uploaded each call; pass a policy with upload_v = 0 to keep
        training the session's resident v."""
        out = np.empty(self.shape, np.float32)
        loss = np.zeros(max(1, self.shape[0] if len(self.shape) == 3 else 1), np.float32)
        arrs = [None if x is None else np.ascontiguousarray(x, dtype=np.float32) for x in (q, k, v, target)]
        pol = policy if policy is not None else default_attention_policy()
        check(lib.lcAttentionSessionTrainStep(self.h, *[_vp(x) for x in arrs], _vp(out), learning_rate,
                                              _vp(loss), C.byref(pol), None), "train_step")
        return out, (float(loss[0]) if loss.size == 1 else loss)

    def buffer(self, which: int) -> int:
        p = C.c_void_p()
        check(lib.lcAttentionSessionBuffer(self.h, which, C.byref(p)))
        return p.value

    def close(self) -> None:
        if self.h and self.h.value:
            lib.lcAttentionSessionDestroy(self.h)
        self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class MatMulResidentSession:
    """ops.hpp:1339-1379 (MatMulMetalResidentSession): start / run / finish / sync / run_batch_sync."""

    def __init__(self, m: int, k: int, n: int, dtype: int = F32):
        self.m, self.k, self.n = m, k, n
        self.np_dtype = np.float32 if dtype == F32 else np.uint16
        self.h = C.c_void_p()
        check(lib.lcMatMulSessionCreate(C.byref(self.h), m, k, n, dtype), "MatMulResidentSession")

    def _stage(self, stage, a, b, out):
        pol = matmul_policy_for_stage(stage)
        pa = None if a is None else np.ascontiguousarray(a, dtype=self.np_dtype)
        pb = None if b is None else np.ascontiguousarray(b, dtype=self.np_dtype)
        check(lib.lcMatMulSessionRun(self.h, _vp(pa), _vp(pb), _vp(out), C.byref(pol), None), "matmul session")
        return out

    def start(self, a, b):
        return self._stage(LOOP_START, a, b, None)

    def run(self):
        return self._stage(LOOP_RUN, None, None, None)

    def finish(self):
        out = np.empty((self.m, self.n), self.np_dtype)
        return self._stage(LOOP_FINISH, None, None, out)

    def sync(self):
        return self._stage(LOOP_SYNC, None, None, None)

    def run_batch_sync(self, a, b, repeat: int, download: bool = True):
        out = np.empty((self.m, self.n), self.np_dtype) if download else None
        pa = None if a is None else np.ascontiguousarray(a, dtype=self.np_dtype)
        pb = None if b is None else np.ascontiguousarray(b, dtype=self.np_dtype)
        check(lib.lcMatMulSessionRunBatch(self.h, _vp(pa), _vp(pb), _vp(out), repeat, None), "run_batch_sync")
        return out

    def buffer(self, which: int) -> int:
        p = C.c_void_p()
        check(lib.lcMatMulSessionBuffer(self.h, which, C.byref(p)))
        return p.value

    def close(self) -> None:
        if self.h and self.h.value:
            lib.lcMatMulSessionDestroy(self.h)
        self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def attention_train_step(q, k, v, target, learning_rate: float, causal: bool = False):
    """attentionTrainStep (src/attention.cpp:203-214) on the GPU: returns (out, updated v, loss).
    q/k/v/target: [seq, d] or [units, seq, d] float32; loss per unit for batched input."""
    q, k, t = (np.ascontiguousarray(x, dtype=np.float32) for x in (q, k, target))
    v = np.array(v, dtype=np.float32, copy=True, order="C")
    shape = q.shape
    units = shape[0] if q.ndim == 3 else 1
    seq, d = shape[-2], shape[-1]
    out = np.empty_like(q)
    loss = np.zeros(units, np.float32)
    pol = default_attention_policy()
    check(lib.lcAttentionTrainStep(_vp(q), _vp(k), _vp(v), _vp(t), _vp(out), learning_rate, units, seq, d,
                                   int(causal), _vp(loss), C.byref(pol), None), "attention_train_step")
    return out, v, (float(loss[0]) if q.ndim == 2 else loss)


# ---- multi-GPU (one process per GPU) -----------------------------------------------------------
class Comm:
    """A communicator of liblc_b200.so (NCCL underneath) for this process's current device.

    `exchange(bytes) -> bytes` hands rank 0's 128-byte unique id to every rank over whatever host
    channel the caller already has (e.g. a torch.distributed broadcast); it is called on every rank
    with rank 0's id (other ranks pass zeros) and must return rank 0's bytes."""

    def __init__(self, rank: int, nranks: int, exchange):
        if not lib.lcCommAvailable():
            raise RuntimeError("NCCL (libnccl.so.2) could not be loaded")
        uid = (C.c_char * 128)()
        if rank == 0:
            check(lib.lcCommGetUniqueId(uid), "lcCommGetUniqueId")
        got = exchange(bytes(uid))
        if len(got) != 128:
            raise ValueError("unique id must be 128 bytes")
        uid = (C.c_char * 128).from_buffer_copy(got)
        self.handle = C.c_void_p()
        check(lib.lcCommInitRank(C.byref(self.handle), nranks, uid, rank), "lcCommInitRank")
        self.rank, self.nranks = rank, nranks

    def close(self, abort: bool = False) -> None:
        if self.handle:
            fn = lib.lcCommAbort if abort else lib.lcCommDestroy
            check(fn(self.handle), "lcCommAbort" if abort else "lcCommDestroy")
            self.handle = C.c_void_p()


def shard_range(total: int, rank: int, nranks: int) -> tuple[int, int]:
    """[lo, hi) of `total` units owned by `rank` (the library's balanced contiguous split)."""
    lo, hi = C.c_size_t(), C.c_size_t()
    if lib.lcShardRange(total, rank, nranks, C.byref(lo), C.byref(hi)) != LC_SUCCESS:
        raise ValueError("bad shard request")
    return lo.value, hi.value


def conv_tune_key(batch, in_c, in_h, in_w, out_c, kh, kw, sh=1, sw=1, ph=0, pw=0):
    """The LC_TUNE_CONV cache key (d0, d1, d2) of a conv shape (lcConvTuneKey)."""
    d = [C.c_size_t() for _ in range(3)]
    check(lib.lcConvTuneKey(batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, *(C.byref(x) for x in d)),
          "conv_tune_key")
    return tuple(x.value for x in d)
