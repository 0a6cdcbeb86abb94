// Op half of the C ABI: attention / matmul2d / conv2d / integrated conv->attention / vector add /
// layer norm entry points with the reference's IO-policy semantics mapped onto explicit device
// memory (see include/lc_b200.h for the pointer conventions).  No CPU compute path exists here:
// every op runs on the GPU or returns an error.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <climits>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "lc_host.hpp"
#include "lc_internal.hpp"

namespace lcb {
namespace {

// Per-thread, per-device staging buffers for host-pointer (upload/download) calls; they grow
// by 1.5x like the reference's Metal buffers (src/attention_metal.mm:1082) and are reused.  A call
// that returns before its work is done (no synchronize, no download) may leave a slot in use on
// its stream; each slot therefore carries an event recorded after the last call that used it, and
// a later call on another stream waits for that event before touching the slot (calls on the
// same stream are ordered by the stream itself).
struct Staging {
  struct Slot {
    void* ptr = nullptr;
    size_t bytes = 0;
    cudaEvent_t done = nullptr;   // recorded on `stream` after the last call that used the slot
    cudaStream_t stream = nullptr;
  };
  std::vector<Slot> slots[64];
  ~Staging() {
    // Buffers are released with the thread; contexts may already be gone at process exit.
  }
  cudaError_t get(int dev, int slot, size_t bytes, cudaStream_t s, void** out) {
    auto& v = slots[dev];
    if (static_cast<int>(v.size()) <= slot) v.resize(slot + 1);
    Slot& sl = v[slot];
    if (sl.bytes < bytes) {
      if (sl.ptr) cudaFree(sl.ptr);  // synchronizes the device: no earlier use is still running
      sl.ptr = nullptr;
      sl.bytes = 0;
      const size_t want = bytes + bytes / 2;
      cudaError_t e = device_malloc(&sl.ptr, want);
      if (e != cudaSuccess) return e;
      sl.bytes = want;
    } else if (sl.done && sl.stream != s) {
      cudaError_t e = cudaStreamWaitEvent(s, sl.done, 0);
      if (e != cudaSuccess) return e;
    }
    *out = sl.ptr;
    return cudaSuccess;
  }
  // After a call: slots [0, n) of device `dev` were used by work enqueued on stream s.
  void release(int dev, int n, cudaStream_t s) {
    auto& v = slots[dev];
    for (int i = 0; i < n && i < static_cast<int>(v.size()); ++i) {
      Slot& sl = v[i];
      if (!sl.done && cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming) != cudaSuccess) {
        sl.done = nullptr;
        continue;
      }
      if (cudaEventRecord(sl.done, s) == cudaSuccess) sl.stream = s;
    }
  }
};
thread_local Staging t_staging;

// One call's host<->device plumbing.
class Io {
 public:
  explicit Io(cudaStream_t s) : s_(s) { cudaGetDevice(&dev_); }
  ~Io() {
    if (slot_ > 0) t_staging.release(dev_, slot_, s_);
  }
  Io(const Io&) = delete;
  Io& operator=(const Io&) = delete;
  // Input: host pointer -> copied into staging slot; device pointer -> used directly.
  cudaError_t in(const void* p, size_t bytes, bool host, const void** dev) {
    if (!host) {
      *dev = p;
      return cudaSuccess;
    }
    void* d = nullptr;
    cudaError_t e = t_staging.get(dev_, slot_++, bytes, s_, &d);
    if (e != cudaSuccess) return e;
    e = cudaMemcpyAsync(d, p, bytes, cudaMemcpyHostToDevice, s_);
    *dev = d;
    return e;
  }
  // Output: host pointer -> a staging slot receives the result; device pointer -> direct.
  cudaError_t out(void* p, size_t bytes, bool host, void** dev) {
    if (!host) {
      *dev = p;
      return cudaSuccess;
    }
    return t_staging.get(dev_, slot_++, bytes, s_, dev);
  }
  cudaError_t scratch(size_t bytes, void** dev) { return t_staging.get(dev_, slot_++, bytes, s_, dev); }
  cudaError_t finish(void* host_out, const void* dev_out, size_t bytes, bool download, bool sync) {
    cudaError_t e = cudaSuccess;
    if (download) e = cudaMemcpyAsync(host_out, dev_out, bytes, cudaMemcpyDeviceToHost, s_);
    if (e != cudaSuccess) return e;
    if (sync || download) e = cudaStreamSynchronize(s_);
    return e;
  }
  cudaStream_t stream() const { return s_; }
  int device() const { return dev_; }

 private:
  cudaStream_t s_;
  int dev_ = 0;
  int slot_ = 0;
};

// ---- pipelined staging ----------------------------------------------------------------------
// A large call with host inputs and a host output is cut into chunks along its independent
// dimension (attention units, GEMM rows): chunk c's uploads run on a helper stream, its kernel on
// the caller's stream, its download on a second helper stream, so copies in both PCIe directions
// overlap each other and the kernels.  Same results, same policy contract (the call returns with
// the output in host memory).  Helper streams and events are per thread and device.
struct PipeRes {
  cudaStream_t in[64] = {}, out[64] = {};
  std::vector<cudaEvent_t> ev[64];
  cudaError_t streams(int dev, cudaStream_t* i, cudaStream_t* o) {
    if (!in[dev]) {
      cudaError_t e = cudaStreamCreateWithFlags(&in[dev], cudaStreamNonBlocking);
      if (e != cudaSuccess) return e;
      e = cudaStreamCreateWithFlags(&out[dev], cudaStreamNonBlocking);
      if (e != cudaSuccess) return e;
    }
    *i = in[dev];
    *o = out[dev];
    return cudaSuccess;
  }
  cudaError_t event(int dev, size_t idx, cudaEvent_t* e) {
    auto& v = ev[dev];
    while (v.size() <= idx) {
      cudaEvent_t x;
      cudaError_t r = cudaEventCreateWithFlags(&x, cudaEventDisableTiming);
      if (r != cudaSuccess) return r;
      v.push_back(x);
    }
    *e = v[idx];
    return cudaSuccess;
  }
};
thread_local PipeRes t_pipe;
constexpr size_t kPipeMinBytes = size_t(24) << 20;  // smaller calls gain nothing from chunking

// One chunked host<->device transfer: element u of the chunked dimension is unit_bytes long.
struct PipeBuf {
  const void* host_in;   // host source (nullptr: device-resident, nothing to upload)
  void* host_out;        // host destination (outputs)
  void* dev;
  size_t unit_bytes;
};

// Runs launch(u0, n) for n-unit chunks of [0, units) with `ins` uploaded and `out_buf`
// downloaded chunk by chunk; `prefix` inputs are uploaded whole before the first chunk.  Chunks
// are multiples of `align` units.  Returns with everything complete on the caller's stream
// (the caller synchronizes).
template <class Launch>
cudaError_t run_pipelined(Io& io, size_t units, size_t align, const std::vector<PipeBuf>& prefix,
                          const std::vector<PipeBuf>& ins, const PipeBuf& out_buf, Launch launch) {
  const int dev = io.device();
  cudaStream_t s = io.stream(), si, so;
  cudaError_t e = t_pipe.streams(dev, &si, &so);
  if (e != cudaSuccess) return e;
  size_t per_unit = out_buf.unit_bytes;
  for (const auto& b : ins) per_unit += b.host_in ? b.unit_bytes : 0;
  const size_t total = per_unit * units;
  size_t nchunks = total / (size_t(16) << 20);
  nchunks = nchunks < 2 ? 2 : nchunks > 8 ? 8 : nchunks;
  size_t chunk = (units + nchunks - 1) / nchunks;
  chunk = (chunk + align - 1) / align * align;
  cudaEvent_t start;
  if ((e = t_pipe.event(dev, 0, &start)) != cudaSuccess) return e;
  // Prior work on the caller's stream (e.g. kernels still reading the staging buffers) first.
  if ((e = cudaEventRecord(start, s)) != cudaSuccess || (e = cudaStreamWaitEvent(si, start, 0)) != cudaSuccess ||
      (e = cudaStreamWaitEvent(so, start, 0)) != cudaSuccess)
    return e;
  for (const auto& b : prefix)
    if (b.host_in && (e = cudaMemcpyAsync(b.dev, b.host_in, b.unit_bytes, cudaMemcpyHostToDevice, si)) != cudaSuccess)
      return e;
  size_t idx = 1;
  cudaEvent_t last = nullptr;
  for (size_t u0 = 0; u0 < units; u0 += chunk) {
    const size_t n = units - u0 < chunk ? units - u0 : chunk;
    cudaEvent_t ein, ek, eout;
    if ((e = t_pipe.event(dev, idx++, &ein)) != cudaSuccess || (e = t_pipe.event(dev, idx++, &ek)) != cudaSuccess ||
        (e = t_pipe.event(dev, idx++, &eout)) != cudaSuccess)
      return e;
    for (const auto& b : ins)
      if (b.host_in &&
          (e = cudaMemcpyAsync(static_cast<char*>(b.dev) + u0 * b.unit_bytes,
                               static_cast<const char*>(b.host_in) + u0 * b.unit_bytes, n * b.unit_bytes,
                               cudaMemcpyHostToDevice, si)) != cudaSuccess)
        return e;
    if ((e = cudaEventRecord(ein, si)) != cudaSuccess || (e = cudaStreamWaitEvent(s, ein, 0)) != cudaSuccess) return e;
    if ((e = launch(u0, n)) != cudaSuccess) return e;
    if ((e = cudaEventRecord(ek, s)) != cudaSuccess || (e = cudaStreamWaitEvent(so, ek, 0)) != cudaSuccess) return e;
    if ((e = cudaMemcpyAsync(static_cast<char*>(out_buf.host_out) + u0 * out_buf.unit_bytes,
                             static_cast<const char*>(out_buf.dev) + u0 * out_buf.unit_bytes, n * out_buf.unit_bytes,
                             cudaMemcpyDeviceToHost, so)) != cudaSuccess ||
        (e = cudaEventRecord(eout, so)) != cudaSuccess)
      return e;
    last = eout;
  }
  return last ? cudaStreamWaitEvent(s, last, 0) : cudaSuccess;
}

// After a synchronizing call, a kernel that gave up a bounded wait shows in the error word.
lcError_t check_error_word(bool synced) {
  if (!synced) return LC_SUCCESS;
  DeviceCtx* c = device_ctx();
  if (!c) return LC_NOT_INITIALIZED;
  unsigned w = 0;
  if (cudaMemcpy(&w, c->err_word, sizeof(w), cudaMemcpyDeviceToHost) != cudaSuccess) return LC_DRIVER_ERROR;
  return w ? LC_DRIVER_ERROR : LC_SUCCESS;
}

#define LC_TRY(expr)                                   \
  do {                                                 \
    cudaError_t e_ = (expr);                           \
    if (e_ != cudaSuccess) return from_cuda(e_);       \
  } while (0)

size_t elem_size(lcDataType t) { return t == LC_DTYPE_BF16 ? 2 : t == LC_DTYPE_F64 ? 8 : 4; }

}  // namespace
}  // namespace lcb

using namespace lcb;

extern "C" {

void lcAttentionIoPolicyDefault(lcAttentionIoPolicy* p) {
  if (!p) return;
  p->upload_q = p->upload_k = p->upload_v = p->upload_target = 1;
  p->download_out = p->download_v = p->synchronize = 1;
  p->loss_every = 1;
  p->output_scale = 1.0f;
  p->output_bias = 0.0f;
  p->output_relu = 0;
}
void lcMatMulIoPolicyDefault(lcMatMulIoPolicy* p) {
  if (p) p->upload_a = p->upload_b = p->download_out = p->synchronize = 1;
}
void lcConv2dIoPolicyDefault(lcConv2dIoPolicy* p) {
  if (p) p->upload_x = p->upload_w = p->upload_bias = p->download_out = p->synchronize = 1;
}
void lcVectorAddIoPolicyDefault(lcVectorAddIoPolicy* p) {
  if (p) p->upload_a = p->upload_b = p->download_out = p->synchronize = 1;
}

void lcMatMulPolicyForStage(lcLoopStage stage, lcMatMulIoPolicy* p) {
  if (!p) return;
  const int start = stage == LC_LOOP_START;
  p->upload_a = start;
  p->upload_b = start;
  p->download_out = stage == LC_LOOP_FINISH;
  p->synchronize = stage == LC_LOOP_FINISH || stage == LC_LOOP_SYNC;
}

void lcVectorPolicyForStage(lcLoopStage stage, lcVectorAddIoPolicy* p) {
  if (!p) return;
  p->upload_a = p->upload_b = stage == LC_LOOP_START;
  p->download_out = stage == LC_LOOP_FINISH;
  p->synchronize = stage == LC_LOOP_FINISH || stage == LC_LOOP_SYNC;
}

void lcElemwisePolicyForStage(lcLoopStage stage, lcVectorAddIoPolicy* p) { lcVectorPolicyForStage(stage, p); }

void lcAttentionPolicyForStage(lcLoopStage stage, int training, lcAttentionIoPolicy* p) {
  if (!p) return;
  const int start = stage == LC_LOOP_START, finish = stage == LC_LOOP_FINISH;
  p->upload_q = p->upload_k = p->upload_v = p->upload_target = start;
  p->download_out = finish;
  p->download_v = finish && training;
  p->synchronize = finish || stage == LC_LOOP_SYNC;
}

lcError_t lcAttentionForward(const void* q, const void* k, const void* v, void* out, size_t units, size_t seq,
                             size_t head_dim, int causal, lcDataType dtype, const lcAttentionIoPolicy* policy,
                             lcStream_t stream) {
  if (!q || !k || !v || !out || units == 0 || seq == 0 || head_dim == 0) return LC_INVALID_VALUE;
  if (dtype != LC_DTYPE_F32 && dtype != LC_DTYPE_BF16) return LC_NOT_SUPPORTED;
  if (seq > (size_t)INT_MAX || head_dim > 256 || units > (size_t)INT_MAX) return LC_NOT_SUPPORTED;
  lcAttentionIoPolicy pol;
  if (policy) {
    pol = *policy;
  } else {
    lcAttentionIoPolicyDefault(&pol);
    pol.upload_q = pol.upload_k = pol.upload_v = pol.download_out = pol.synchronize = 0;
  }
  Io io(static_cast<cudaStream_t>(stream));
  const size_t es = elem_size(dtype);
  const size_t bytes = units * seq * head_dim * es;
  auto attn_args = [&](const void* dq, const void* dk, const void* dv, void* dout, size_t u0, size_t n) {
    const long long ustride = static_cast<long long>(seq * head_dim);
    AttnArgs a{};
    a.q = static_cast<const char*>(dq) + u0 * ustride * es;
    a.k = static_cast<const char*>(dk) + u0 * ustride * es;
    a.v = static_cast<const char*>(dv) + u0 * ustride * es;
    a.out = static_cast<char*>(dout) + u0 * ustride * es;
    a.q_unit_stride = a.k_unit_stride = a.v_unit_stride = a.out_unit_stride = ustride;
    a.units = static_cast<int>(n);
    a.seq = static_cast<int>(seq);
    a.d = static_cast<int>(head_dim);
    a.causal = causal ? 1 : 0;
    a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    a.post_scale = pol.output_scale;
    a.post_bias = pol.output_bias;
    a.post_relu = pol.output_relu ? 1 : 0;
    return a;
  };
  const bool any_upload = pol.upload_q || pol.upload_k || pol.upload_v;
  if (pol.download_out && any_upload && units >= 2 && 4 * bytes >= kPipeMinBytes) {
    // Host in, host out, large: chunked over units with overlapped copies.
    void *dq, *dk, *dv, *dout;
    LC_TRY(pol.upload_q ? io.scratch(bytes, &dq) : (dq = const_cast<void*>(q), cudaSuccess));
    LC_TRY(pol.upload_k ? io.scratch(bytes, &dk) : (dk = const_cast<void*>(k), cudaSuccess));
    LC_TRY(pol.upload_v ? io.scratch(bytes, &dv) : (dv = const_cast<void*>(v), cudaSuccess));
    LC_TRY(io.scratch(bytes, &dout));
    trace_op(kOpAttention, units * seq * seq * head_dim);
    const size_t ub = seq * head_dim * es;
    std::vector<PipeBuf> ins = {{pol.upload_q ? q : nullptr, nullptr, dq, ub},
                                {pol.upload_k ? k : nullptr, nullptr, dk, ub},
                                {pol.upload_v ? v : nullptr, nullptr, dv, ub}};
    PipeBuf ob = {nullptr, out, dout, ub};
    LC_TRY(run_pipelined(io, units, 1, {}, ins, ob, [&](size_t u0, size_t n) -> cudaError_t {
      for (size_t c0 = 0; c0 < n; c0 += 65535) {
        const AttnArgs a = attn_args(dq, dk, dv, dout, u0 + c0, n - c0 < 65535 ? n - c0 : 65535);
        cudaError_t e = dtype == LC_DTYPE_F32 ? attention_f32(a, io.stream()) : attention_bf16(a, io.stream());
        if (e != cudaSuccess) return e;
      }
      return cudaSuccess;
    }));
    LC_TRY(cudaStreamSynchronize(io.stream()));
    return check_error_word(true);
  }
  const void *dq, *dk, *dv;
  void* dout;
  LC_TRY(io.in(q, bytes, pol.upload_q, &dq));
  LC_TRY(io.in(k, bytes, pol.upload_k, &dk));
  LC_TRY(io.in(v, bytes, pol.upload_v, &dv));
  LC_TRY(io.out(out, bytes, pol.download_out, &dout));
  trace_op(kOpAttention, units * seq * seq * head_dim);

  const long long ustride = static_cast<long long>(seq * head_dim);
  for (size_t u0 = 0; u0 < units; u0 += 65535) {
    const size_t n = units - u0 < 65535 ? units - u0 : 65535;
    AttnArgs a{};
    a.q = static_cast<const char*>(dq) + u0 * ustride * es;
    a.k = static_cast<const char*>(dk) + u0 * ustride * es;
    a.v = static_cast<const char*>(dv) + u0 * ustride * es;
    a.out = static_cast<char*>(dout) + u0 * ustride * es;
    a.q_unit_stride = a.k_unit_stride = a.v_unit_stride = a.out_unit_stride = ustride;
    a.units = static_cast<int>(n);
    a.seq = static_cast<int>(seq);
    a.d = static_cast<int>(head_dim);
    a.causal = causal ? 1 : 0;
    a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    a.post_scale = pol.output_scale;
    a.post_bias = pol.output_bias;
    a.post_relu = pol.output_relu ? 1 : 0;
    LC_TRY(dtype == LC_DTYPE_F32 ? attention_f32(a, io.stream()) : attention_bf16(a, io.stream()));
  }
  LC_TRY(io.finish(out, dout, bytes, pol.download_out, pol.synchronize));
  return check_error_word(pol.synchronize || pol.download_out);
}

// Attention of `units` heads followed by the projection out[u] = attn[u] @ proj_w.  q/k/v of unit u
// start u * unit_stride elements in; out is [units, seq, cols].  f32 with head_dim, cols <= 128
// runs as one kernel (projection in the attention epilogue); otherwise attention into a scratch
// buffer, then one GEMM over all units' rows.
static lcError_t attention_proj_device(const void* dq, const void* dk, const void* dv, long long unit_stride,
                                       const void* dp, void* dout, size_t units, size_t seq, size_t head_dim,
                                       size_t cols, int causal, lcDataType dtype, Io& io) {
  const size_t es = elem_size(dtype);
  const bool fused = dtype == LC_DTYPE_F32 && head_dim <= 128 && cols <= 128;
  void* attn = nullptr;
  if (!fused) LC_TRY(io.scratch(units * seq * head_dim * es, &attn));
  trace_op(kOpAttention, units * seq * seq * head_dim);
  for (size_t u0 = 0; u0 < units; u0 += 65535) {
    const size_t n = units - u0 < 65535 ? units - u0 : 65535;
    AttnArgs a{};
    a.q = static_cast<const char*>(dq) + u0 * unit_stride * es;
    a.k = static_cast<const char*>(dk) + u0 * unit_stride * es;
    a.v = static_cast<const char*>(dv) + u0 * unit_stride * es;
    a.q_unit_stride = a.k_unit_stride = a.v_unit_stride = unit_stride;
    a.units = static_cast<int>(n);
    a.seq = static_cast<int>(seq);
    a.d = static_cast<int>(head_dim);
    a.causal = causal ? 1 : 0;
    a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    a.post_scale = 1.0f;
    a.post_bias = 0.0f;
    a.post_relu = 0;
    if (fused) {
      a.out = static_cast<char*>(dout) + u0 * seq * cols * es;
      a.out_unit_stride = static_cast<long long>(seq * cols);
      a.proj_w = static_cast<const float*>(dp);
      a.proj_cols = static_cast<int>(cols);
      LC_TRY(attention_f32(a, io.stream()));
    } else {
      a.out = static_cast<char*>(attn) + u0 * seq * head_dim * es;
      a.out_unit_stride = static_cast<long long>(seq * head_dim);
      LC_TRY(dtype == LC_DTYPE_F32 ? attention_f32(a, io.stream()) : attention_bf16(a, io.stream()));
    }
  }
  if (!fused) {
    const size_t rows = units * seq;
    if (rows > (size_t)INT_MAX) return LC_NOT_SUPPORTED;
    trace_op(kOpMatMul, rows * head_dim * cols);
    LC_TRY(dtype == LC_DTYPE_F32
               ? gemm_f32(static_cast<const float*>(attn), static_cast<const float*>(dp), static_cast<float*>(dout),
                          (int)rows, (int)head_dim, (int)cols, io.stream())
               : gemm_bf16(static_cast<const __nv_bfloat16*>(attn), static_cast<const __nv_bfloat16*>(dp),
                           static_cast<__nv_bfloat16*>(dout), (int)rows, (int)head_dim, (int)cols, io.stream()));
  }
  return LC_SUCCESS;
}

static bool neutral_postprocess(const lcAttentionIoPolicy& p) {
  return p.output_scale == 1.0f && p.output_bias == 0.0f && !p.output_relu;
}

lcError_t lcAttentionProjForward(const void* q, const void* k, const void* v, const void* proj_w, void* out,
                                 size_t units, size_t seq, size_t head_dim, size_t proj_cols, int causal,
                                 lcDataType dtype, const lcAttentionIoPolicy* policy, lcStream_t stream) {
  if (!q || !k || !v || !proj_w || !out || units == 0 || seq == 0 || head_dim == 0 || proj_cols == 0)
    return LC_INVALID_VALUE;
  if (dtype != LC_DTYPE_F32 && dtype != LC_DTYPE_BF16) return LC_NOT_SUPPORTED;
  if (seq > (size_t)INT_MAX || head_dim > 256 || units > (size_t)INT_MAX || proj_cols > (size_t)INT_MAX)
    return LC_NOT_SUPPORTED;
  lcAttentionIoPolicy pol;
  if (policy) {
    pol = *policy;
  } else {
    lcAttentionIoPolicyDefault(&pol);
    pol.upload_q = pol.upload_k = pol.upload_v = pol.download_out = pol.synchronize = 0;
  }
  if (!neutral_postprocess(pol)) return LC_NOT_SUPPORTED;
  Io io(static_cast<cudaStream_t>(stream));
  const size_t es = elem_size(dtype);
  const size_t in_bytes = units * seq * head_dim * es, out_bytes = units * seq * proj_cols * es;
  const void *dq, *dk, *dv, *dp;
  void* dout;
  LC_TRY(io.in(q, in_bytes, pol.upload_q, &dq));
  LC_TRY(io.in(k, in_bytes, pol.upload_k, &dk));
  LC_TRY(io.in(v, in_bytes, pol.upload_v, &dv));
  LC_TRY(io.in(proj_w, head_dim * proj_cols * es, pol.upload_q, &dp));
  LC_TRY(io.out(out, out_bytes, pol.download_out, &dout));
  const lcError_t st = attention_proj_device(dq, dk, dv, static_cast<long long>(seq * head_dim), dp, dout, units, seq,
                                             head_dim, proj_cols, causal, dtype, io);
  if (st != LC_SUCCESS) return st;
  LC_TRY(io.finish(out, dout, out_bytes, pol.download_out, pol.synchronize));
  return check_error_word(pol.synchronize || pol.download_out);
}

lcError_t lcAttentionQkvProjForward(const float* packed, size_t packed_len, const float* proj_w, float* out,
                                    size_t seq, size_t head_dim, size_t proj_cols,
                                    const lcAttentionIoPolicy* policy, lcStream_t stream) {
  if (!packed || packed_len == 0 || !proj_w || !out || seq == 0 || head_dim == 0 || proj_cols == 0)
    return LC_INVALID_VALUE;
  if (seq > (size_t)INT_MAX || head_dim > 256 || proj_cols > (size_t)INT_MAX) return LC_NOT_SUPPORTED;
  lcAttentionIoPolicy pol;
  if (policy) {
    pol = *policy;
  } else {
    lcAttentionIoPolicyDefault(&pol);
    pol.upload_q = pol.upload_k = pol.upload_v = pol.download_out = pol.synchronize = 0;
  }
  if (!neutral_postprocess(pol)) return LC_NOT_SUPPORTED;
  Io io(static_cast<cudaStream_t>(stream));
  const size_t need = seq * head_dim;
  const size_t out_bytes = seq * proj_cols * 4;
  const size_t used = packed_len < 3 * need ? packed_len : 3 * need;  // only the first 3*need floats matter
  const void *dsrc, *dp;
  void* dout;
  LC_TRY(io.in(packed, used * 4, pol.upload_q, &dsrc));
  LC_TRY(io.in(proj_w, head_dim * proj_cols * 4, pol.upload_q, &dp));
  LC_TRY(io.out(out, out_bytes, pol.download_out, &dout));
  const float* qkv = static_cast<const float*>(dsrc);
  if (used < 3 * need) {
    // The pack node repeats a short input cyclically up to 3*need floats (graph.hpp:3170-3180).
    void* full;
    LC_TRY(io.scratch(3 * need * 4, &full));
    LC_TRY(repeat_fill_f32(qkv, used, static_cast<float*>(full), 3 * need, io.stream()));
    qkv = static_cast<const float*>(full);
  }
  const lcError_t st = attention_proj_device(qkv, qkv + need, qkv + 2 * need, static_cast<long long>(3 * need), dp,
                                             dout, 1, seq, head_dim, proj_cols, 0, LC_DTYPE_F32, io);
  if (st != LC_SUCCESS) return st;
  LC_TRY(io.finish(out, dout, out_bytes, pol.download_out, pol.synchronize));
  return check_error_word(pol.synchronize || pol.download_out);
}

lcError_t lcMatMul(const void* a, const void* b, void* out, size_t m, size_t k, size_t n, lcDataType dtype,
                   const lcMatMulIoPolicy* policy, lcStream_t stream) {
  if (!a || !b || !out || m == 0 || k == 0 || n == 0) return LC_INVALID_VALUE;
  if (dtype != LC_DTYPE_F32 && dtype != LC_DTYPE_BF16) return LC_NOT_SUPPORTED;
  if (m > (size_t)INT_MAX || k > (size_t)INT_MAX || n > (size_t)INT_MAX) return LC_NOT_SUPPORTED;
  lcMatMulIoPolicy pol = {0, 0, 0, 0};
  if (policy) pol = *policy;
  Io io(static_cast<cudaStream_t>(stream));
  const size_t es = elem_size(dtype);
  if (dtype == LC_DTYPE_BF16 && pol.download_out && (pol.upload_a || pol.upload_b) && m >= 512 &&
      (m * k + k * n + m * n) * es >= kPipeMinBytes) {
    // Host in, host out, large: B uploaded whole, then A / C row blocks (multiples of 256 rows)
    // with overlapped copies.
    void *da, *db, *dc;
    LC_TRY(pol.upload_a ? io.scratch(m * k * es, &da) : (da = const_cast<void*>(a), cudaSuccess));
    LC_TRY(pol.upload_b ? io.scratch(k * n * es, &db) : (db = const_cast<void*>(b), cudaSuccess));
    LC_TRY(io.scratch(m * n * es, &dc));
    trace_op(kOpMatMul, m * k * n);
    std::vector<PipeBuf> prefix = {{pol.upload_b ? b : nullptr, nullptr, db, k * n * es}};
    std::vector<PipeBuf> ins = {{pol.upload_a ? a : nullptr, nullptr, da, k * es}};
    PipeBuf ob = {nullptr, out, dc, n * es};
    LC_TRY(run_pipelined(io, m, 256, prefix, ins, ob, [&](size_t r0, size_t rows) -> cudaError_t {
      return gemm_bf16(static_cast<const __nv_bfloat16*>(da) + r0 * k, static_cast<const __nv_bfloat16*>(db),
                       static_cast<__nv_bfloat16*>(dc) + r0 * n, (int)rows, (int)k, (int)n, io.stream());
    }));
    LC_TRY(cudaStreamSynchronize(io.stream()));
    return check_error_word(true);
  }
  const void *da, *db;
  void* dc;
  LC_TRY(io.in(a, m * k * es, pol.upload_a, &da));
  LC_TRY(io.in(b, k * n * es, pol.upload_b, &db));
  LC_TRY(io.out(out, m * n * es, pol.download_out, &dc));
  trace_op(kOpMatMul, m * k * n);
  if (dtype == LC_DTYPE_F32) {
    LC_TRY(gemm_f32(static_cast<const float*>(da), static_cast<const float*>(db), static_cast<float*>(dc), (int)m,
                    (int)k, (int)n, io.stream()));
  } else {
    LC_TRY(gemm_bf16(static_cast<const __nv_bfloat16*>(da), static_cast<const __nv_bfloat16*>(db),
                     static_cast<__nv_bfloat16*>(dc), (int)m, (int)k, (int)n, io.stream()));
  }
  LC_TRY(io.finish(out, dc, m * n * es, pol.download_out, pol.synchronize));
  return check_error_word(pol.synchronize || pol.download_out);
}

// Validation of include/lightning_core/core/ops.hpp:874-884.
static bool conv_shape_ok(const void* x, const void* w, const void* out, size_t batch, size_t in_c, size_t in_h,
                          size_t in_w, size_t out_c, size_t kh, size_t kw, size_t sh, size_t sw, size_t ph,
                          size_t pw) {
  if (!x || !w || !out || batch == 0 || in_c == 0 || in_h == 0 || in_w == 0 || out_c == 0 || kh == 0 || kw == 0 ||
      sh == 0 || sw == 0)
    return false;
  return in_h + 2 * ph >= kh && in_w + 2 * pw >= kw;
}

lcError_t lcConv2dNchw(const float* x, const float* w, const float* bias, float* out, size_t batch,
                       size_t in_channels, size_t in_h, size_t in_w, size_t out_channels, size_t kernel_h,
                       size_t kernel_w, size_t stride_h, size_t stride_w, size_t pad_h, size_t pad_w, int apply_relu,
                       const lcConv2dIoPolicy* policy, lcStream_t stream) {
  if (!conv_shape_ok(x, w, out, batch, in_channels, in_h, in_w, out_channels, kernel_h, kernel_w, stride_h, stride_w,
                     pad_h, pad_w))
    return LC_INVALID_VALUE;
  const size_t oh = (in_h + 2 * pad_h - kernel_h) / stride_h + 1;
  const size_t ow = (in_w + 2 * pad_w - kernel_w) / stride_w + 1;
  if (!conv_dims_fit_int(in_channels, in_h, in_w, out_channels, kernel_h, kernel_w, stride_h, stride_w, pad_h, pad_w) ||
      batch * oh * ow > (size_t)INT_MAX)
    return LC_NOT_SUPPORTED;
  lcConv2dIoPolicy pol = {0, 0, 0, 0, 0};
  if (policy) pol = *policy;
  Io io(static_cast<cudaStream_t>(stream));
  const void *dx, *dw, *db = nullptr;
  void* dout;
  const size_t out_bytes = batch * out_channels * oh * ow * 4;
  LC_TRY(io.in(x, batch * in_channels * in_h * in_w * 4, pol.upload_x, &dx));
  LC_TRY(io.in(w, out_channels * in_channels * kernel_h * kernel_w * 4, pol.upload_w, &dw));
  if (bias) LC_TRY(io.in(bias, out_channels * 4, pol.upload_bias, &db));
  LC_TRY(io.out(out, out_bytes, pol.download_out, &dout));
  trace_op(kOpConv2dNchw, batch * oh * ow * out_channels * in_channels * kernel_h * kernel_w);
  LC_TRY(conv2d_nchw_f32(static_cast<const float*>(dx), static_cast<const float*>(dw),
                         static_cast<const float*>(db), static_cast<float*>(dout), (int)batch, (int)in_channels,
                         (int)in_h, (int)in_w, (int)out_channels, (int)kernel_h, (int)kernel_w, (int)stride_h,
                         (int)stride_w, (int)pad_h, (int)pad_w, apply_relu ? 1 : 0, io.stream()));
  LC_TRY(io.finish(out, dout, out_bytes, pol.download_out, pol.synchronize));
  return check_error_word(pol.synchronize || pol.download_out);
}

lcError_t lcConvAttentionNchw(const float* x, const float* w, const float* bias, const float* proj_w, float* out,
                              size_t batch, size_t in_channels, size_t in_h, size_t in_w, size_t out_channels,
                              size_t kernel_h, size_t kernel_w, size_t stride_h, size_t stride_w, size_t pad_h,
                              size_t pad_w, size_t seq, size_t head_dim, size_t proj_cols, int per_image,
                              const lcConv2dIoPolicy* policy, lcStream_t stream) {
  if (!conv_shape_ok(x, w, out, batch, in_channels, in_h, in_w, out_channels, kernel_h, kernel_w, stride_h, stride_w,
                     pad_h, pad_w) ||
      seq == 0 || head_dim == 0 || (proj_w && proj_cols == 0))
    return LC_INVALID_VALUE;
  if (head_dim > 256 || (proj_w && (head_dim > 128 || proj_cols > 128)) || seq > (size_t)INT_MAX)
    return LC_NOT_SUPPORTED;
  if (!conv_dims_fit_int(in_channels, in_h, in_w, out_channels, kernel_h, kernel_w, stride_h, stride_w, pad_h, pad_w))
    return LC_NOT_SUPPORTED;
  const size_t oh = (in_h + 2 * pad_h - kernel_h) / stride_h + 1;
  const size_t ow = (in_w + 2 * pad_w - kernel_w) / stride_w + 1;
  if (batch * oh * ow > (size_t)INT_MAX) return LC_NOT_SUPPORTED;
  lcConv2dIoPolicy pol = {0, 0, 0, 0, 0};
  if (policy) pol = *policy;
  Io io(static_cast<cudaStream_t>(stream));
  const size_t img = out_channels * oh * ow;  // conv floats per image
  const size_t need = seq * head_dim;
  const size_t cols = proj_w ? proj_cols : head_dim;
  const size_t units = per_image ? batch : 1;
  const size_t out_bytes = units * seq * cols * 4;
  const void *dx, *dw, *db = nullptr, *dp = nullptr;
  void *dout, *conv;
  LC_TRY(io.in(x, batch * in_channels * in_h * in_w * 4, pol.upload_x, &dx));
  LC_TRY(io.in(w, out_channels * in_channels * kernel_h * kernel_w * 4, pol.upload_w, &dw));
  if (bias) LC_TRY(io.in(bias, out_channels * 4, pol.upload_bias, &db));
  if (proj_w) LC_TRY(io.in(proj_w, head_dim * proj_cols * 4, pol.upload_w, &dp));
  LC_TRY(io.out(out, out_bytes, pol.download_out, &dout));
  LC_TRY(io.scratch(batch * img * 4, &conv));
  cudaStream_t s = io.stream();
  trace_op(kOpConv2dNchw, batch * oh * ow * out_channels * in_channels * kernel_h * kernel_w);
  {
    // Fused route (per-image semantics, conv output long enough, head_dim 64, strict-fp32 tensor-core
    // attention, cluster-pair conv): the conv epilogue writes the attention's Q / K tf32 hi-lo
    // planes and the unsplit V directly, so the QKV tensor never exists as a separate NCHW buffer
    // and no split pass runs over Q and K.  Skipped when a tune-cache entry pins another kernel.
    const size_t avail_img = img;
    AttnArgs a{};
    a.units = static_cast<int>(units);
    a.seq = static_cast<int>(seq);
    a.d = static_cast<int>(head_dim);
    a.causal = 0;
    a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    a.post_scale = 1.0f;
    a.post_bias = 0.0f;
    a.post_relu = 0;
    a.proj_w = static_cast<const float*>(dp);
    a.proj_cols = static_cast<int>(proj_cols);
    a.out = dout;
    a.out_unit_stride = static_cast<long long>(seq * cols);
    std::string cfg;
    size_t k0, k1, k2;
    const bool conv_pinned =
        conv_tune_key(batch, in_channels, in_h, in_w, out_channels, kernel_h, kernel_w, stride_h, stride_w, pad_h,
                      pad_w, &k0, &k1, &k2) &&
        tune_lookup(LC_TUNE_CONV, k0, k1, k2, LC_DTYPE_F32, &cfg) && cfg != kConvImplicitName;
    const bool attn_pinned = tune_lookup(LC_TUNE_ATTENTION, seq, head_dim, 0, LC_DTYPE_F32, &cfg) && cfg == "simt";
    const long long macs = static_cast<long long>(batch * oh * ow) * out_channels * in_channels * kernel_h * kernel_w;
    if ((per_image || batch == 1) && avail_img >= 3 * need && need % (16 * oh * ow) == 0 && need <= (size_t)INT_MAX &&
        head_dim == 64 && units <= 65535 && !conv_pinned &&
        !attn_pinned && macs >= (1LL << 26) &&
        conv_qkv_split_supported((int)batch, (int)in_channels, (int)in_h, (int)in_w, (int)out_channels,
                                 (int)kernel_h, (int)kernel_w, (int)stride_h, (int)stride_w, (int)pad_h,
                                 (int)pad_w)) {
      a.q_unit_stride = a.k_unit_stride = a.v_unit_stride = static_cast<long long>(need);
      // Plane layout of the attention: [Q_hi | Q_lo | K_hi | K_lo | V^T_hi | V^T_lo], then the raw V.
      const size_t nqk = units * need;
      a.q = a.k = nullptr;  // read from the planes
      if (attention_f32_tc_supported(a)) {
        DeviceCtx* ctx = device_ctx();
        if (!ctx) return LC_NOT_INITIALIZED;
        const size_t ws_floats = attention_f32_tc_ws_floats((int)units, (int)seq) + nqk;
        float* ws = nullptr;
        LC_TRY(workspace_alloc(ctx, reinterpret_cast<void**>(&ws), ws_floats * 4, s));
        float* vraw = ws + attention_f32_tc_ws_floats((int)units, (int)seq);
        const QkvSplitOut qkv{ws, ws + nqk, ws + 2 * nqk, ws + 3 * nqk, vraw, static_cast<long long>(need)};
        a.v = vraw;
        cudaError_t e = conv2d_nchw_f32_implicit_qkv(
            static_cast<const float*>(dx), static_cast<const float*>(dw), static_cast<const float*>(db), (int)batch,
            (int)in_channels, (int)in_h, (int)in_w, (int)out_channels, (int)kernel_h, (int)kernel_w, (int)stride_h,
            (int)stride_w, (int)pad_h, (int)pad_w, 1, qkv, s);
        if (e == cudaSuccess) {
          trace_op(kOpAttention, units * seq * seq * head_dim);
          e = attention_f32_tc_presplit_qk(a, ws, s);
        }
        const cudaError_t ef = workspace_free(ws, s);
        LC_TRY(e);
        LC_TRY(ef);
        LC_TRY(io.finish(out, dout, out_bytes, pol.download_out, pol.synchronize));
        return check_error_word(pol.synchronize || pol.download_out);
      }
    }
  }
  // Conv + bias + ReLU; its NCHW output already is the QKV arrangement (raw channel-block slices).
  LC_TRY(conv2d_nchw_f32(static_cast<const float*>(dx), static_cast<const float*>(dw), static_cast<const float*>(db),
                         static_cast<float*>(conv), (int)batch, (int)in_channels, (int)in_h, (int)in_w,
                         (int)out_channels, (int)kernel_h, (int)kernel_w, (int)stride_h, (int)stride_w, (int)pad_h,
                         (int)pad_w, 1, s));
  const float* qkv = static_cast<const float*>(conv);
  long long unit_stride = static_cast<long long>(img);
  const size_t avail = per_image ? img : batch * img;
  if (avail < 3 * need) {
    // Short conv output: the reference repeats the flat buffer cyclically up to 3*need floats
    // (python/bindings/bind_integrated.cpp:718-728).  Only this rare case pays a packing pass.
    void* packed;
    LC_TRY(io.scratch(units * 3 * need * 4, &packed));
    for (size_t u = 0; u < units; ++u)
      LC_TRY(repeat_fill_f32(qkv + u * img, avail, static_cast<float*>(packed) + u * 3 * need, 3 * need, s));
    qkv = static_cast<const float*>(packed);
    unit_stride = static_cast<long long>(3 * need);
  }
  trace_op(kOpAttention, units * seq * seq * head_dim);
  for (size_t u0 = 0; u0 < units; u0 += 65535) {
    const size_t n = units - u0 < 65535 ? units - u0 : 65535;
    AttnArgs a{};
    a.q = qkv + u0 * unit_stride;
    a.k = qkv + u0 * unit_stride + need;
    a.v = qkv + u0 * unit_stride + 2 * need;
    a.out = static_cast<float*>(dout) + u0 * seq * cols;
    a.q_unit_stride = a.k_unit_stride = a.v_unit_stride = unit_stride;
    a.out_unit_stride = static_cast<long long>(seq * cols);
    a.units = static_cast<int>(n);
    a.seq = static_cast<int>(seq);
    a.d = static_cast<int>(head_dim);
    a.causal = 0;
    a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    a.post_scale = 1.0f;
    a.post_bias = 0.0f;
    a.post_relu = 0;
    a.proj_w = static_cast<const float*>(dp);
    a.proj_cols = static_cast<int>(proj_cols);
    LC_TRY(attention_f32(a, s));
  }
  LC_TRY(io.finish(out, dout, out_bytes, pol.download_out, pol.synchronize));
  return check_error_word(pol.synchronize || pol.download_out);
}

lcError_t lcVectorAdd(const void* a, const void* b, void* out, size_t n, lcDataType dtype,
                      const lcVectorAddIoPolicy* policy, lcStream_t stream) {
  if (!a || !b || !out || n == 0) return LC_INVALID_VALUE;
  if (dtype != LC_DTYPE_F32 && dtype != LC_DTYPE_F64) return LC_NOT_SUPPORTED;
  lcVectorAddIoPolicy pol = {0, 0, 0, 0};
  if (policy) pol = *policy;
  Io io(static_cast<cudaStream_t>(stream));
  const size_t bytes = n * elem_size(dtype);
  const void *da, *db;
  void* dc;
  LC_TRY(io.in(a, bytes, pol.upload_a, &da));
  LC_TRY(io.in(b, bytes, pol.upload_b, &db));
  LC_TRY(io.out(out, bytes, pol.download_out, &dc));
  trace_op(kOpVectorAdd, n);
  if (dtype == LC_DTYPE_F32)
    LC_TRY(vector_add_f32(static_cast<const float*>(da), static_cast<const float*>(db), static_cast<float*>(dc), n,
                          io.stream()));
  else
    LC_TRY(vector_add_f64(static_cast<const double*>(da), static_cast<const double*>(db), static_cast<double*>(dc), n,
                          io.stream()));
  LC_TRY(io.finish(out, dc, bytes, pol.download_out, pol.synchronize));
  return check_error_word(pol.synchronize || pol.download_out);
}

lcError_t lcLayerNorm(const float* x, float* out, size_t rows, size_t cols, float eps, lcStream_t stream) {
  if (!x || !out || rows == 0 || cols == 0) return LC_INVALID_VALUE;
  LC_TRY(layer_norm_f32(x, out, rows, cols, eps, static_cast<cudaStream_t>(stream)));
  return LC_SUCCESS;
}

}  // extern "C"

// attentionTrainStepWithPolicy (src/attention.cpp:216-242) + attentionTrainStepCpu
// (src/attention_cpu.cpp:114-163): forward, MSE against target, dV = P^T dO, v -= lr * dV.
// Batched over `units` heads; loss_out (optional, host) receives one loss per unit.
extern "C" lcError_t lcAttentionTrainStep(const float* q, const float* k, float* v, const float* target, float* out,
                                          float learning_rate, size_t units, size_t seq, size_t head_dim, int causal,
                                          float* loss_out, const lcAttentionIoPolicy* policy, lcStream_t stream) {
  if (!q || !k || !v || !target || !out || units == 0 || seq == 0 || head_dim == 0 || !(learning_rate > 0.0f))
    return LC_INVALID_VALUE;
  if (head_dim > 128 || seq > (size_t)INT_MAX || units > 65535) return LC_NOT_SUPPORTED;
  lcAttentionIoPolicy pol;
  if (policy) {
    pol = *policy;
  } else {
    lcAttentionIoPolicyDefault(&pol);
    pol.upload_q = pol.upload_k = pol.upload_v = pol.upload_target = 0;
    pol.download_out = pol.download_v = pol.synchronize = 0;
  }
  Io io(static_cast<cudaStream_t>(stream));
  cudaStream_t s = io.stream();
  const size_t n = units * seq * head_dim, bytes = n * 4;
  const void *dq, *dk, *dt;
  void *dvv, *dout, *lse, *grad, *sse;
  LC_TRY(io.in(q, bytes, pol.upload_q, &dq));
  LC_TRY(io.in(k, bytes, pol.upload_k, &dk));
  LC_TRY(io.in(target, bytes, pol.upload_target, &dt));
  {
    const void* vin;
    LC_TRY(io.in(v, bytes, pol.upload_v, &vin));  // staged copy when v is host memory
    dvv = const_cast<void*>(vin);
  }
  LC_TRY(io.out(out, bytes, pol.download_out, &dout));
  LC_TRY(io.scratch(units * seq * 4, &lse));
  LC_TRY(io.scratch(bytes, &grad));
  LC_TRY(io.scratch(units * sizeof(double), &sse));
  trace_op(kOpAttention, units * seq * seq * head_dim);
  AttnArgs a{};
  a.q = dq;
  a.k = dk;
  a.v = dvv;
  a.out = dout;
  a.q_unit_stride = a.k_unit_stride = a.v_unit_stride = a.out_unit_stride = static_cast<long long>(seq * head_dim);
  a.units = static_cast<int>(units);
  a.seq = static_cast<int>(seq);
  a.d = static_cast<int>(head_dim);
  a.causal = causal ? 1 : 0;
  a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
  a.post_scale = 1.0f;
  a.lse = static_cast<float*>(lse);
  LC_TRY(attention_f32(a, s));
  LC_TRY(attention_train_grad_out(static_cast<const float*>(dout), static_cast<const float*>(dt),
                                  static_cast<float*>(grad), static_cast<double*>(sse), (int)units,
                                  static_cast<long long>(seq * head_dim), s));
  LC_TRY(attention_train_dv_update(static_cast<const float*>(dq), static_cast<const float*>(dk),
                                   static_cast<float*>(dvv), static_cast<const float*>(grad),
                                   static_cast<const float*>(lse), (int)units, (int)seq, (int)head_dim, a.causal,
                                   a.scale, learning_rate, s));
  if (pol.download_v) LC_TRY(cudaMemcpyAsync(v, dvv, bytes, cudaMemcpyDeviceToHost, s));
  if (pol.download_out) LC_TRY(cudaMemcpyAsync(out, dout, bytes, cudaMemcpyDeviceToHost, s));
  if (loss_out) {
    std::vector<double> h(units);
    LC_TRY(cudaMemcpyAsync(h.data(), sse, units * sizeof(double), cudaMemcpyDeviceToHost, s));
    LC_TRY(cudaStreamSynchronize(s));
    const float norm = 1.0f / static_cast<float>(seq * head_dim);
    for (size_t u = 0; u < units; ++u) loss_out[u] = static_cast<float>(h[u]) * norm;
  }
  const bool synced = pol.synchronize || pol.download_out || pol.download_v || loss_out;
  if (synced) LC_TRY(cudaStreamSynchronize(s));
  return check_error_word(synced);
}

// ops::matrixSubWithPolicy / matrixDivWithPolicy (include/lightning_core/core/ops.hpp:31-49;
// CPU src/ops/matrix_elemwise.cpp:8-29): out = a - b / a / b over rows x cols.
static lcError_t matrix_op(int op, const void* a, const void* b, void* out, size_t rows, size_t cols,
                           lcDataType dtype, const lcVectorAddIoPolicy* policy, lcStream_t stream) {
  if (!a || !b || !out || rows == 0 || cols == 0) return LC_INVALID_VALUE;
  if (dtype != LC_DTYPE_F32 && dtype != LC_DTYPE_F64) return LC_NOT_SUPPORTED;
  lcVectorAddIoPolicy pol = {0, 0, 0, 0};
  if (policy) pol = *policy;
  Io io(static_cast<cudaStream_t>(stream));
  const size_t n = rows * cols, bytes = n * elem_size(dtype);
  const void *da, *db;
  void* dc;
  LC_TRY(io.in(a, bytes, pol.upload_a, &da));
  LC_TRY(io.in(b, bytes, pol.upload_b, &db));
  LC_TRY(io.out(out, bytes, pol.download_out, &dc));
  trace_op(op == 0 ? kOpMatrixSub : kOpMatrixDiv, n);
  LC_TRY(matrix_binary(op, dtype == LC_DTYPE_F64, da, db, dc, n, io.stream()));
  LC_TRY(io.finish(out, dc, bytes, pol.download_out, pol.synchronize));
  return check_error_word(pol.synchronize || pol.download_out);
}

extern "C" lcError_t lcMatrixSub(const void* a, const void* b, void* out, size_t rows, size_t cols, lcDataType dtype,
                                 const lcVectorAddIoPolicy* policy, lcStream_t stream) {
  return matrix_op(0, a, b, out, rows, cols, dtype, policy, stream);
}

extern "C" lcError_t lcMatrixDiv(const void* a, const void* b, void* out, size_t rows, size_t cols, lcDataType dtype,
                                 const lcVectorAddIoPolicy* policy, lcStream_t stream) {
  return matrix_op(1, a, b, out, rows, cols, dtype, policy, stream);
}
