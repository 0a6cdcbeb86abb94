// Multi-GPU half of the C ABI: one process per GPU, an NCCL communicator per process, and
// sharded entry points for the hot path's three partitionable workloads.
//
// The reference runs on one device and has no collective anywhere; what is sharded here are its
// independent units: attention heads ([units, seq, d] -> units split across ranks), matmul rows
// (A row blocks, B replicated) and conv->attention images.  Each rank computes its contiguous,
// balanced shard with the single-GPU kernels and the full output is assembled on every rank with
// one in-place all-gather over NVLink (grouped broadcasts when the shards are uneven).  With host
// buffers the transfers are sharded too: each rank uploads only its shard of the inputs, the
// replicated matmul B is uploaded as 1/N row slices and all-gathered over NVLink instead of being
// pushed N times over PCIe, and each rank downloads only its own output rows.
//
// NCCL is opened with dlopen("libnccl.so.2") on the first communicator call, so a process that
// already loaded NCCL (PyTorch does) shares that copy, and the library does not need NCCL to
// load.  Calls on one communicator are serialised by a lock held while they enqueue work (NCCL
// requires that); the GPU work itself is asynchronous on the caller's stream.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <climits>
#include <cstring>
#include <mutex>

#include "lc_host.hpp"
#include "lc_internal.hpp"

namespace lcb {
namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*GetVersion)(int*) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

std::once_flag g_nccl_once;
NcclApi g_nccl;

const NcclApi& nccl() {
  std::call_once(g_nccl_once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    auto sym = [&](auto& fp, const char* name) {
      fp = reinterpret_cast<std::remove_reference_t<decltype(fp)>>(dlsym(h, name));
      return fp != nullptr;
    };
    g_nccl.ok = sym(g_nccl.GetUniqueId, "ncclGetUniqueId") && sym(g_nccl.CommInitRank, "ncclCommInitRank") &&
                sym(g_nccl.CommDestroy, "ncclCommDestroy") && sym(g_nccl.CommAbort, "ncclCommAbort") &&
                sym(g_nccl.CommGetAsyncError, "ncclCommGetAsyncError") && sym(g_nccl.AllGather, "ncclAllGather") &&
                sym(g_nccl.Broadcast, "ncclBroadcast") && sym(g_nccl.GroupStart, "ncclGroupStart") &&
                sym(g_nccl.GroupEnd, "ncclGroupEnd") && sym(g_nccl.GetVersion, "ncclGetVersion") &&
                sym(g_nccl.GetErrorString, "ncclGetErrorString");
  });
  return g_nccl;
}

lcError_t from_nccl(ncclResult_t r) {
  switch (r) {
    case ncclSuccess: return LC_SUCCESS;
    case ncclInvalidArgument:
    case ncclInvalidUsage: return LC_INVALID_VALUE;
    case ncclInProgress: return LC_SUCCESS;
    default: return LC_DRIVER_ERROR;
  }
}

}  // namespace
}  // namespace lcb

struct lcComm {
  ncclComm_t nccl = nullptr;
  int rank = 0, nranks = 1, device = 0;
  std::mutex mu;
  void* b_stage = nullptr;  // device copy of the replicated matmul B for host-B calls (grow-only)
  size_t b_bytes = 0;
};

using namespace lcb;

namespace {

#define LC_TRY_CUDA(expr)                              \
  do {                                                 \
    cudaError_t e_ = (expr);                           \
    if (e_ != cudaSuccess) return from_cuda(e_);       \
  } while (0)
#define LC_TRY_LC(expr)                                \
  do {                                                 \
    lcError_t s_ = (expr);                             \
    if (s_ != LC_SUCCESS) return s_;                   \
  } while (0)

void shard(size_t total, int rank, int nranks, size_t* lo, size_t* hi) {
  const size_t base = total / nranks, extra = total % nranks;
  const size_t r = static_cast<size_t>(rank);
  *lo = r * base + (r < extra ? r : extra);
  *hi = *lo + base + (r < extra ? 1 : 0);
}

// In-place all-gather of `total` rows of `row_bytes` each: rank r's rows [lo_r, hi_r) are already
// in place in `buf`.  Equal shards: one ncclAllGather (send buffer = this rank's slice of the
// receive buffer, NCCL's in-place form).  Uneven shards: one broadcast per rank, grouped.
lcError_t gather_rows(lcComm* c, void* buf, size_t total, size_t row_bytes, cudaStream_t s) {
  if (c->nranks == 1) return LC_SUCCESS;
  const NcclApi& n = nccl();
  char* b = static_cast<char*>(buf);
  if (total % c->nranks == 0) {
    const size_t count = total / c->nranks * row_bytes;
    return from_nccl(n.AllGather(b + static_cast<size_t>(c->rank) * count, b, count, ncclUint8, c->nccl, s));
  }
  LC_TRY_LC(from_nccl(n.GroupStart()));
  lcError_t st = LC_SUCCESS;
  for (int r = 0; r < c->nranks && st == LC_SUCCESS; ++r) {
    size_t lo, hi;
    shard(total, r, c->nranks, &lo, &hi);
    if (hi > lo)
      st = from_nccl(n.Broadcast(b + lo * row_bytes, b + lo * row_bytes, (hi - lo) * row_bytes, ncclUint8, r,
                                 c->nccl, s));
  }
  const lcError_t st2 = from_nccl(n.GroupEnd());
  return st != LC_SUCCESS ? st : st2;
}

lcError_t comm_ok(lcComm* c) {
  if (!c || !c->nccl) return LC_INVALID_VALUE;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return LC_DRIVER_ERROR;
  return dev == c->device ? LC_SUCCESS : LC_INVALID_VALUE;  // calls must run with the comm's device current
}

lcError_t finish(lcComm* c, cudaStream_t s, bool sync) {
  if (!sync) return LC_SUCCESS;
  LC_TRY_CUDA(cudaStreamSynchronize(s));
  ncclResult_t async = ncclSuccess;
  if (nccl().CommGetAsyncError(c->nccl, &async) != ncclSuccess || async != ncclSuccess) return LC_DRIVER_ERROR;
  unsigned code = 0;
  return lcGetDeviceErrorWord(&code);
}

}  // namespace

extern "C" {

int lcCommAvailable(void) { return nccl().ok ? 1 : 0; }

lcError_t lcCommGetUniqueId(lcCommUniqueId* id) {
  if (!id) return LC_INVALID_VALUE;
  static_assert(sizeof(lcCommUniqueId) == sizeof(ncclUniqueId), "unique id size");
  if (!nccl().ok) return LC_NOT_SUPPORTED;
  ncclUniqueId u;
  const lcError_t st = from_nccl(nccl().GetUniqueId(&u));
  if (st == LC_SUCCESS) std::memcpy(id->internal, u.internal, sizeof(u.internal));
  return st;
}

lcError_t lcCommInitRank(lcComm_t* comm, int nranks, const lcCommUniqueId* id, int rank) {
  if (!comm || !id || nranks < 1 || rank < 0 || rank >= nranks) return LC_INVALID_VALUE;
  *comm = nullptr;
  if (!nccl().ok) return LC_NOT_SUPPORTED;
  lcComm* c = new lcComm();
  c->rank = rank;
  c->nranks = nranks;
  if (cudaGetDevice(&c->device) != cudaSuccess) {
    delete c;
    return LC_DRIVER_ERROR;
  }
  ncclUniqueId u;
  std::memcpy(u.internal, id->internal, sizeof(u.internal));
  const lcError_t st = from_nccl(nccl().CommInitRank(&c->nccl, nranks, u, rank));
  if (st != LC_SUCCESS) {
    delete c;
    return st;
  }
  *comm = c;
  return LC_SUCCESS;
}

lcError_t lcCommDestroy(lcComm_t comm) {
  if (!comm) return LC_SUCCESS;
  lcError_t st = LC_SUCCESS;
  if (comm->nccl) st = from_nccl(nccl().CommDestroy(comm->nccl));
  if (comm->b_stage) cudaFree(comm->b_stage);
  delete comm;
  return st;
}

lcError_t lcCommAbort(lcComm_t comm) {
  if (!comm) return LC_SUCCESS;
  lcError_t st = LC_SUCCESS;
  if (comm->nccl) st = from_nccl(nccl().CommAbort(comm->nccl));
  comm->nccl = nullptr;
  if (comm->b_stage) cudaFree(comm->b_stage);
  delete comm;
  return st;
}

lcError_t lcCommRankInfo(lcComm_t comm, int* rank, int* nranks) {
  if (!comm || !rank || !nranks) return LC_INVALID_VALUE;
  *rank = comm->rank;
  *nranks = comm->nranks;
  return LC_SUCCESS;
}

lcError_t lcShardRange(size_t total, int rank, int nranks, size_t* lo, size_t* hi) {
  if (!lo || !hi || nranks < 1 || rank < 0 || rank >= nranks) return LC_INVALID_VALUE;
  shard(total, rank, nranks, lo, hi);
  return LC_SUCCESS;
}

lcError_t lcCommAllGatherRows(lcComm_t comm, void* buf, size_t total_rows, size_t row_bytes, lcStream_t stream) {
  if (!buf || row_bytes == 0) return LC_INVALID_VALUE;
  LC_TRY_LC(comm_ok(comm));
  std::lock_guard<std::mutex> lk(comm->mu);
  return gather_rows(comm, buf, total_rows, row_bytes, static_cast<cudaStream_t>(stream));
}

lcError_t lcAttentionForwardSharded(lcComm_t comm, const void* q, const void* k, const void* v, void* out,
                                    size_t units, size_t seq, size_t head_dim, int causal, lcDataType dtype,
                                    const lcAttentionIoPolicy* policy, lcStream_t stream) {
  if (!q || !k || !v || !out || units == 0 || seq == 0 || head_dim == 0) return LC_INVALID_VALUE;
  if (dtype != LC_DTYPE_F32 && dtype != LC_DTYPE_BF16) return LC_NOT_SUPPORTED;
  LC_TRY_LC(comm_ok(comm));
  std::lock_guard<std::mutex> lk(comm->mu);
  lcAttentionIoPolicy pol;
  if (policy) {
    pol = *policy;
  } else {
    lcAttentionIoPolicyDefault(&pol);
    pol.upload_q = pol.upload_k = pol.upload_v = pol.download_out = pol.synchronize = 0;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  size_t lo, hi;
  shard(units, comm->rank, comm->nranks, &lo, &hi);
  const size_t ub = seq * head_dim * (dtype == LC_DTYPE_BF16 ? 2 : 4);
  if (hi > lo) {
    lcAttentionIoPolicy inner = pol;
    inner.synchronize = 0;  // the gather follows on the same stream; one sync at the end
    LC_TRY_LC(lcAttentionForward(static_cast<const char*>(q) + lo * ub, static_cast<const char*>(k) + lo * ub,
                                 static_cast<const char*>(v) + lo * ub, static_cast<char*>(out) + lo * ub, hi - lo,
                                 seq, head_dim, causal, dtype, &inner, stream));
  }
  if (!pol.download_out) LC_TRY_LC(gather_rows(comm, out, units, ub, s));
  return finish(comm, s, pol.synchronize || pol.download_out);
}

lcError_t lcMatMulSharded(lcComm_t comm, const void* a, const void* b, void* out, size_t m, size_t k, size_t n,
                          lcDataType dtype, const lcMatMulIoPolicy* policy, lcStream_t stream) {
  if (!a || !b || !out || m == 0 || k == 0 || n == 0) return LC_INVALID_VALUE;
  if (dtype != LC_DTYPE_F32 && dtype != LC_DTYPE_BF16) return LC_NOT_SUPPORTED;
  LC_TRY_LC(comm_ok(comm));
  std::lock_guard<std::mutex> lk(comm->mu);
  lcMatMulIoPolicy pol = {0, 0, 0, 0};
  if (policy) pol = *policy;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t es = dtype == LC_DTYPE_BF16 ? 2 : 4;
  const void* db = b;
  if (pol.upload_b) {
    // B is needed whole on every rank: each rank uploads its 1/N row slice over PCIe into the
    // communicator's B buffer, and the slices are all-gathered over NVLink.
    const size_t bytes = k * n * es;
    if (comm->b_bytes < bytes) {
      if (comm->b_stage) LC_TRY_CUDA(cudaStreamSynchronize(s));  // an earlier call may still read it
      if (comm->b_stage) cudaFree(comm->b_stage);
      comm->b_stage = nullptr;
      comm->b_bytes = 0;
      LC_TRY_CUDA(device_malloc(&comm->b_stage, bytes));
      comm->b_bytes = bytes;
    }
    size_t klo, khi;
    shard(k, comm->rank, comm->nranks, &klo, &khi);
    if (khi > klo)
      LC_TRY_CUDA(cudaMemcpyAsync(static_cast<char*>(comm->b_stage) + klo * n * es,
                                  static_cast<const char*>(b) + klo * n * es, (khi - klo) * n * es,
                                  cudaMemcpyHostToDevice, s));
    LC_TRY_LC(gather_rows(comm, comm->b_stage, k, n * es, s));
    db = comm->b_stage;
  }
  size_t lo, hi;
  shard(m, comm->rank, comm->nranks, &lo, &hi);
  if (hi > lo) {
    lcMatMulIoPolicy inner = pol;
    inner.upload_b = 0;
    inner.synchronize = 0;
    LC_TRY_LC(lcMatMul(static_cast<const char*>(a) + lo * k * es, db, static_cast<char*>(out) + lo * n * es, hi - lo,
                       k, n, dtype, &inner, stream));
  }
  if (!pol.download_out) LC_TRY_LC(gather_rows(comm, out, m, n * es, s));
  return finish(comm, s, pol.synchronize || pol.download_out);
}

lcError_t lcConvAttentionNchwSharded(lcComm_t comm, const float* x, const float* w, const float* bias,
                                     const float* proj_w, float* out, size_t batch, size_t in_channels, size_t in_h,
                                     size_t in_w, size_t out_channels, size_t kernel_h, size_t kernel_w,
                                     size_t stride_h, size_t stride_w, size_t pad_h, size_t pad_w, size_t seq,
                                     size_t head_dim, size_t proj_cols, const lcConv2dIoPolicy* policy,
                                     lcStream_t stream) {
  if (!x || !w || !out || batch == 0 || seq == 0 || head_dim == 0 || (proj_w && proj_cols == 0))
    return LC_INVALID_VALUE;
  LC_TRY_LC(comm_ok(comm));
  std::lock_guard<std::mutex> lk(comm->mu);
  lcConv2dIoPolicy pol = {0, 0, 0, 0, 0};
  if (policy) pol = *policy;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  size_t lo, hi;
  shard(batch, comm->rank, comm->nranks, &lo, &hi);
  const size_t cols = proj_w ? proj_cols : head_dim;
  const size_t xb = in_channels * in_h * in_w, ob = seq * cols;
  if (hi > lo) {
    lcConv2dIoPolicy inner = pol;
    inner.synchronize = 0;
    LC_TRY_LC(lcConvAttentionNchw(x + lo * xb, w, bias, proj_w, out + lo * ob, hi - lo, in_channels, in_h, in_w,
                                  out_channels, kernel_h, kernel_w, stride_h, stride_w, pad_h, pad_w, seq, head_dim,
                                  proj_cols, 1, &inner, stream));
  }
  if (!pol.download_out) LC_TRY_LC(gather_rows(comm, out, batch, ob * 4, s));
  return finish(comm, s, pol.synchronize || pol.download_out);
}

}  // extern "C"
