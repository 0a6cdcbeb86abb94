"""The library's multi-GPU layer (lcComm*, lc*Sharded) on real GPUs, one process per GPU.

Each rank computes its shard of attention heads / matmul rows / conv->attention images and the
full output is assembled on every rank by the library's NCCL all-gather.  Checked against the
oracle on sampled units and rows (bf16 2e-2 relative, fp32 1e-4 + 1e-4|ref|), with device
buffers (full output on every rank) and with host buffers (each rank downloads its own rows; the
matmul's B is uploaded as 1/N slices and all-gathered over NVLink).  A one-rank communicator runs
on a single GPU; the two-rank case needs two GPUs and is skipped otherwise."""
import os
import socket

import numpy as np
import pytest

from conftest import ROOT, close_enough  # noqa: F401  (sets sys.path)

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(11)
    units, seq, d = 6, 300, 128
    q, k, v = (rng.standard_normal((units, seq, d)).astype(np.float32) for _ in range(3))
    m, kk, n = 1000, 512, 264
    a = (rng.uniform(-1, 1, (m, kk)) / np.sqrt(kk)).astype(np.float32)
    b = rng.uniform(-1, 1, (kk, n)).astype(np.float32)
    x = rng.standard_normal((3, 8, 12, 12)).astype(np.float32)
    w = rng.uniform(-0.3, 0.3, (24, 8, 3, 3)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, 24).astype(np.float32)
    pw = rng.uniform(-0.5, 0.5, (16, 16)).astype(np.float32)
    return dict(q=q, k=k, v=v, a=a, b=b, x=x, w=w, bias=bias, pw=pw)


def _worker(rank, world, port, out_dir):
    import ctypes as C

    import torch
    import torch.distributed as dist

    import lightning_core_b200 as lc
    from oracle import oracle as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        P = O.port()
        inp = _inputs()

        def exchange(uid):
            obj = [uid]
            dist.broadcast_object_list(obj, 0)
            return obj[0]

        comm = lc.Comm(rank, world, exchange)
        L = lc.lib
        ptr = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
        res = {}
        # -- attention bf16, device buffers: full output on every rank
        q, k, v = (torch.from_numpy(P.bf16_round(inp[n])).to(torch.bfloat16).cuda() for n in "qkv")
        units, seq, d = q.shape
        out = torch.zeros_like(q)
        lc.check(L.lcAttentionForwardSharded(comm.handle, ptr(q), ptr(k), ptr(v), ptr(out), units, seq, d, 1,
                                             lc.BF16, None, None))
        torch.cuda.synchronize()
        res["attn_dev"] = out.float().cpu().numpy()
        # -- matmul bf16, device buffers
        a = torch.from_numpy(P.bf16_round(inp["a"])).to(torch.bfloat16).cuda()
        b = torch.from_numpy(P.bf16_round(inp["b"])).to(torch.bfloat16).cuda()
        m, kk = a.shape
        n = b.shape[1]
        c = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
        lc.check(L.lcMatMulSharded(comm.handle, ptr(a), ptr(b), ptr(c), m, kk, n, lc.BF16, None, None))
        torch.cuda.synchronize()
        res["mm_dev"] = c.float().cpu().numpy()
        # -- matmul f32, host buffers (reference default policy): own rows downloaded, B by slices
        ha, hb = inp["a"].copy(), inp["b"].copy()
        hc = np.zeros((m, n), np.float32)
        pol = lc.default_matmul_policy()
        lc.check(L.lcMatMulSharded(comm.handle, ha.ctypes.data_as(C.c_void_p), hb.ctypes.data_as(C.c_void_p),
                                   hc.ctypes.data_as(C.c_void_p), m, kk, n, lc.F32, C.byref(pol), None))
        res["mm_host"] = hc
        # -- conv -> attention -> projection per image, device buffers
        x, w, bias, pw = (torch.from_numpy(inp[n]).cuda() for n in ("x", "w", "bias", "pw"))
        co = torch.zeros((3, 144, 16), device="cuda")
        lc.check(L.lcConvAttentionNchwSharded(comm.handle, ptr(x), ptr(w), ptr(bias), ptr(pw), ptr(co), 3, 8, 12, 12,
                                              24, 3, 3, 1, 1, 1, 1, 144, 16, 16, None, None))
        torch.cuda.synchronize()
        res["conv_dev"] = co.cpu().numpy()
        comm.close()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)
    finally:
        dist.destroy_process_group()


def _check(out_dir, world):
    import lightning_core_b200 as lc
    from oracle import oracle as O

    P = O.port()
    inp = _inputs()
    q, k, v = (P.bf16_round(inp[n]) for n in "qkv")
    a, b = P.bf16_round(inp["a"]), P.bf16_round(inp["b"])
    want_attn = P.attention_units(q, k, v, True)
    want_mm = P.matmul(a, b, threads=8)
    want_mm32 = P.matmul(inp["a"], inp["b"], threads=8)
    want_conv = P.conv_attention_images(inp["x"], inp["w"], inp["bias"], inp["pw"], 144, 16, threads=3)
    for r in range(world):
        got = np.load(os.path.join(out_dir, f"rank{r}.npz"))
        close_enough(want_attn, got["attn_dev"], 2e-2, 2e-2)
        close_enough(want_mm, got["mm_dev"], 2e-3, 2e-2)
        close_enough(want_conv, got["conv_dev"], 1e-4, 1e-4)
        lo, hi = lc.shard_range(a.shape[0], r, world)
        close_enough(want_mm32[lo:hi], got["mm_host"][lo:hi], 1e-4, 1e-4)


def test_sharded_one_rank(gpu, tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(1, _free_port(), str(tmp_path)), nprocs=1, join=True, start_method="spawn")
    _check(str(tmp_path), 1)


def test_sharded_two_ranks(gpu, tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    _check(str(tmp_path), 2)
