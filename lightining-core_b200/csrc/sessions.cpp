// Shape-bound sessions that own device-resident buffers.
//
// Mirror the reference's AttentionSession (include/lightning_core/core/attention.hpp:86-129,
// src/attention.cpp:247-343) and MatMulMetalResidentSession (include/lightning_core/core/ops.hpp:
// 1339-1379): a session is created for one shape, keeps its inputs and output in device memory
// between calls, and each call's IO policy decides what moves: upload_* set copies that host
// pointer into the session's buffer; clear reuses what the buffer already holds (the pointer may
// be NULL); download_out set copies the result back to host memory; synchronize waits on the
// stream.  The loop-stage presets (start / run / finish / sync) of ops/policy.hpp:37-71 drive a
// resident loop.  A mutex per session makes concurrent calls from several threads safe (they
// serialise on the session, as the reference's shared sessions do).
#include <cuda_runtime.h>

#include <mutex>
#include <new>
#include <vector>

#include "lc_host.hpp"
#include "lc_internal.hpp"

namespace {

size_t esize(lcDataType t) { return t == LC_DTYPE_BF16 ? 2 : 4; }

struct Buf {
  void* p = nullptr;
  size_t bytes = 0;
};

lcError_t alloc_all(Buf* bufs, int n) {
  for (int i = 0; i < n; ++i) {
    if (lcb::device_malloc(&bufs[i].p, bufs[i].bytes) != cudaSuccess) {
      for (int j = 0; j < i; ++j) cudaFree(bufs[j].p);
      return LC_OUT_OF_MEMORY;
    }
  }
  return LC_SUCCESS;
}

lcError_t upload(const Buf& b, const void* host, bool flag, cudaStream_t s) {
  if (!flag) return LC_SUCCESS;
  if (!host) return LC_INVALID_VALUE;
  return lcb::from_cuda(cudaMemcpyAsync(b.p, host, b.bytes, cudaMemcpyHostToDevice, s));
}

lcError_t finish(const Buf& out, void* host, bool download, bool sync, cudaStream_t s) {
  if (download) {
    if (!host) return LC_INVALID_VALUE;
    cudaError_t e = cudaMemcpyAsync(host, out.p, out.bytes, cudaMemcpyDeviceToHost, s);
    if (e != cudaSuccess) return lcb::from_cuda(e);
  }
  if (download || sync) return lcb::from_cuda(cudaStreamSynchronize(s));
  return LC_SUCCESS;
}

}  // namespace

struct lcAttentionSession {
  size_t units, seq, head_dim;
  int causal;
  lcDataType dtype;
  int device;
  Buf b[4];       // q, k, v, out
  Buf target;     // allocated by the first train step
  size_t train_steps = 0;
  std::vector<float> last_loss;
  bool has_last_loss = false;
  lcAttentionIoPolicy def;
  std::mutex mu;
};

struct lcMatMulSession {
  size_t m, k, n;
  lcDataType dtype;
  int device;
  Buf b[3];  // a, b, out
  std::mutex mu;
};

extern "C" {

lcError_t lcAttentionSessionCreate(lcAttentionSession_t* out, size_t units, size_t seq, size_t head_dim, int causal,
                                   lcDataType dtype) {
  if (!out || units == 0 || seq == 0 || head_dim == 0) return LC_INVALID_VALUE;
  if (dtype != LC_DTYPE_F32 && dtype != LC_DTYPE_BF16) return LC_NOT_SUPPORTED;
  auto* s = new (std::nothrow) lcAttentionSession();
  if (!s) return LC_OUT_OF_MEMORY;
  s->units = units;
  s->seq = seq;
  s->head_dim = head_dim;
  s->causal = causal ? 1 : 0;
  s->dtype = dtype;
  cudaGetDevice(&s->device);
  for (auto& x : s->b) x.bytes = units * seq * head_dim * esize(dtype);
  lcAttentionIoPolicyDefault(&s->def);
  s->def.synchronize = 0;  // the reference's session default (src/attention.cpp:247-254)
  const lcError_t e = alloc_all(s->b, 4);
  if (e != LC_SUCCESS) {
    delete s;
    return e;
  }
  *out = s;
  return LC_SUCCESS;
}

lcError_t lcAttentionSessionDestroy(lcAttentionSession_t s) {
  if (!s) return LC_INVALID_VALUE;
  for (auto& x : s->b) cudaFree(x.p);
  if (s->target.p) cudaFree(s->target.p);
  delete s;
  return LC_SUCCESS;
}

lcError_t lcAttentionSessionSetDefaultPolicy(lcAttentionSession_t s, const lcAttentionIoPolicy* policy) {
  if (!s || !policy) return LC_INVALID_VALUE;
  std::lock_guard<std::mutex> lk(s->mu);
  s->def = *policy;
  return LC_SUCCESS;
}

lcError_t lcAttentionSessionBuffer(lcAttentionSession_t s, int which, void** dev_ptr) {
  if (!s || !dev_ptr || which < 0 || which > 3) return LC_INVALID_VALUE;
  *dev_ptr = s->b[which].p;
  return LC_SUCCESS;
}

lcError_t lcAttentionSessionForward(lcAttentionSession_t s, const void* q, const void* k, const void* v, void* out,
                                    const lcAttentionIoPolicy* policy, lcStream_t stream) {
  if (!s) return LC_INVALID_VALUE;
  std::lock_guard<std::mutex> lk(s->mu);
  const lcAttentionIoPolicy pol = policy ? *policy : s->def;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  lcError_t e;
  if ((e = upload(s->b[0], q, pol.upload_q, st)) != LC_SUCCESS) return e;
  if ((e = upload(s->b[1], k, pol.upload_k, st)) != LC_SUCCESS) return e;
  if ((e = upload(s->b[2], v, pol.upload_v, st)) != LC_SUCCESS) return e;
  lcAttentionIoPolicy dev = pol;  // the kernel call itself sees device buffers only
  dev.upload_q = dev.upload_k = dev.upload_v = dev.download_out = dev.synchronize = 0;
  e = lcAttentionForward(s->b[0].p, s->b[1].p, s->b[2].p, s->b[3].p, s->units, s->seq, s->head_dim, s->causal,
                         s->dtype, &dev, stream);
  if (e != LC_SUCCESS) return e;
  return finish(s->b[3], out, pol.download_out, pol.synchronize, st);
}

// src/attention.cpp:12-38: the loss cadence when the policy leaves loss_every = 0.
static int auto_loss_every(size_t seq, size_t d) {
  if (seq == 256 && d == 64) return 32;
  if (seq == 256 && d == 128) return 16;
  if ((seq == 512 || seq == 1024) && (d == 64 || d == 128)) return 8;
  return 4;
}

lcError_t lcAttentionSessionTrainStep(lcAttentionSession_t s, const float* q, const float* k, float* v,
                                      const float* target, float* out, float learning_rate, float* loss_out,
                                      const lcAttentionIoPolicy* policy, lcStream_t stream) {
  if (!s || !(learning_rate > 0.0f)) return LC_INVALID_VALUE;
  if (s->dtype != LC_DTYPE_F32) return LC_NOT_SUPPORTED;
  std::lock_guard<std::mutex> lk(s->mu);
  const lcAttentionIoPolicy pol = policy ? *policy : s->def;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!s->target.p) {
    s->target.bytes = s->b[0].bytes;
    if (lcb::device_malloc(&s->target.p, s->target.bytes) != cudaSuccess) {
      s->target.p = nullptr;
      return LC_OUT_OF_MEMORY;
    }
  }
  lcError_t e;
  if ((e = upload(s->b[0], q, pol.upload_q, st)) != LC_SUCCESS) return e;
  if ((e = upload(s->b[1], k, pol.upload_k, st)) != LC_SUCCESS) return e;
  if ((e = upload(s->b[2], v, pol.upload_v, st)) != LC_SUCCESS) return e;
  if ((e = upload(s->target, target, pol.upload_target, st)) != LC_SUCCESS) return e;
  bool take_loss = false;
  if (loss_out) {
    const int every = pol.loss_every == 0 ? auto_loss_every(s->seq, s->head_dim) : (pol.loss_every < 1 ? 1 : pol.loss_every);
    take_loss = (s->train_steps % static_cast<size_t>(every)) == 0;
  }
  std::vector<float> loss(s->units);
  lcAttentionIoPolicy dev;
  lcAttentionIoPolicyDefault(&dev);
  dev.upload_q = dev.upload_k = dev.upload_v = dev.upload_target = 0;
  dev.download_out = dev.download_v = dev.synchronize = 0;
  e = lcAttentionTrainStep(static_cast<const float*>(s->b[0].p), static_cast<const float*>(s->b[1].p),
                           static_cast<float*>(s->b[2].p), static_cast<const float*>(s->target.p),
                           static_cast<float*>(s->b[3].p), learning_rate, s->units, s->seq, s->head_dim, s->causal,
                           take_loss ? loss.data() : nullptr, &dev, stream);
  if (e != LC_SUCCESS) return e;
  if (pol.download_v) {
    if (!v) return LC_INVALID_VALUE;
    if (cudaMemcpyAsync(v, s->b[2].p, s->b[2].bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess) return LC_DRIVER_ERROR;
  }
  if ((e = finish(s->b[3], out, pol.download_out, pol.synchronize || pol.download_v, st)) != LC_SUCCESS) return e;
  if (loss_out) {
    if (take_loss) {
      s->last_loss = loss;
      s->has_last_loss = true;
    }
    for (size_t u = 0; u < s->units; ++u) loss_out[u] = s->has_last_loss ? s->last_loss[u] : 0.0f;
  }
  ++s->train_steps;
  return LC_SUCCESS;
}

lcError_t lcMatMulSessionCreate(lcMatMulSession_t* out, size_t m, size_t k, size_t n, lcDataType dtype) {
  if (!out || m == 0 || k == 0 || n == 0) return LC_INVALID_VALUE;
  if (dtype != LC_DTYPE_F32 && dtype != LC_DTYPE_BF16) return LC_NOT_SUPPORTED;
  auto* s = new (std::nothrow) lcMatMulSession();
  if (!s) return LC_OUT_OF_MEMORY;
  s->m = m;
  s->k = k;
  s->n = n;
  s->dtype = dtype;
  cudaGetDevice(&s->device);
  s->b[0].bytes = m * k * esize(dtype);
  s->b[1].bytes = k * n * esize(dtype);
  s->b[2].bytes = m * n * esize(dtype);
  const lcError_t e = alloc_all(s->b, 3);
  if (e != LC_SUCCESS) {
    delete s;
    return e;
  }
  *out = s;
  return LC_SUCCESS;
}

lcError_t lcMatMulSessionDestroy(lcMatMulSession_t s) {
  if (!s) return LC_INVALID_VALUE;
  for (auto& x : s->b) cudaFree(x.p);
  delete s;
  return LC_SUCCESS;
}

lcError_t lcMatMulSessionBuffer(lcMatMulSession_t s, int which, void** dev_ptr) {
  if (!s || !dev_ptr || which < 0 || which > 2) return LC_INVALID_VALUE;
  *dev_ptr = s->b[which].p;
  return LC_SUCCESS;
}

lcError_t lcMatMulSessionRun(lcMatMulSession_t s, const void* a, const void* b, void* out,
                             const lcMatMulIoPolicy* policy, lcStream_t stream) {
  if (!s) return LC_INVALID_VALUE;
  std::lock_guard<std::mutex> lk(s->mu);
  lcMatMulIoPolicy pol;
  if (policy) {
    pol = *policy;
  } else {
    lcMatMulIoPolicyDefault(&pol);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  lcError_t e;
  if ((e = upload(s->b[0], a, pol.upload_a, st)) != LC_SUCCESS) return e;
  if ((e = upload(s->b[1], b, pol.upload_b, st)) != LC_SUCCESS) return e;
  e = lcMatMul(s->b[0].p, s->b[1].p, s->b[2].p, s->m, s->k, s->n, s->dtype, nullptr, stream);
  if (e != LC_SUCCESS) return e;
  return finish(s->b[2], out, pol.download_out, pol.synchronize, st);
}

// runBatchSync / runBatchSyncNoDownload (ops.hpp:251-352): `repeat` launches on the resident
// buffers (inputs uploaded first when given), then one synchronize, downloading when out != NULL.
lcError_t lcMatMulSessionRunBatch(lcMatMulSession_t s, const void* a, const void* b, void* out, size_t repeat,
                                  lcStream_t stream) {
  if (!s || repeat == 0) return LC_INVALID_VALUE;
  std::lock_guard<std::mutex> lk(s->mu);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  lcError_t e;
  if ((e = upload(s->b[0], a, a != nullptr, st)) != LC_SUCCESS) return e;
  if ((e = upload(s->b[1], b, b != nullptr, st)) != LC_SUCCESS) return e;
  for (size_t r = 0; r < repeat; ++r) {
    e = lcMatMul(s->b[0].p, s->b[1].p, s->b[2].p, s->m, s->k, s->n, s->dtype, nullptr, stream);
    if (e != LC_SUCCESS) return e;
  }
  return finish(s->b[2], out, out != nullptr, true, st);
}

}  // extern "C"
