// lcConvAttentionNchwNoAlloc: the integrated conv -> ReLU -> QKV -> attention (-> projection)
// pipeline for callers that must not allocate GPU memory.
//
// Who needs it: code that runs where cudaMalloc is off limits -- inside a host callback or a
// real-time loop that may not block on the allocator, under an external memory manager or
// budget that owns every device allocation, or in a plugin whose host process forbids its
// libraries from allocating.  lcConvAttentionNchw takes its conv intermediate from a staging
// buffer that grows with cudaMalloc; this variant takes it from a fixed array compiled into the
// library instead and allocates nothing.
//
// The scratch is one file-scope __device__ array of LC_NOALLOC_SCRATCH_FLOATS floats (64 MiB).
// Every GPU that loads the library holds it until the process exits.  All calls on a device
// share it and it keeps the last call's contents; each call overwrites every element it reads
// (the conv writes the whole intermediate, the repeat pass writes the whole packed Q/K/V), so
// nothing needs clearing.  Calls whose work overlaps on the GPU (two streams, or two threads)
// race on the array: serialise them on one stream.
#include <cuda_runtime.h>

#include <climits>
#include <cmath>
#include <mutex>

#include "lc_host.hpp"
#include "lc_internal.hpp"

#define LC_NOALLOC_SCRATCH_FLOATS (16u * 1024u * 1024u)

namespace lcb {
namespace {

static __device__ __align__(256) float g_noalloc_scratch[LC_NOALLOC_SCRATCH_FLOATS];

// Device address of g_noalloc_scratch, looked up once per device with that device current.
// In host code the symbol itself is only a host-side stand-in and must never reach a kernel.
std::mutex g_scratch_mu;
float* g_scratch_ptr[64] = {};

cudaError_t scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace lcb

using namespace lcb;

extern "C" lcError_t lcConvAttentionNchwNoAlloc(const float* x, const float* w, const float* bias,
                                                const float* proj_w, float* out, size_t batch, size_t in_channels,
                                                size_t in_h, size_t in_w, size_t out_channels, size_t kernel_h,
                                                size_t kernel_w, size_t stride_h, size_t stride_w, size_t pad_h,
                                                size_t pad_w, size_t seq, size_t head_dim, size_t proj_cols,
                                                int per_image, lcStream_t stream) {
  if (!x || !w || !out || batch == 0 || in_channels == 0 || in_h == 0 || in_w == 0 || out_channels == 0 ||
      kernel_h == 0 || kernel_w == 0 || stride_h == 0 || stride_w == 0 || seq == 0 || head_dim == 0 ||
      (proj_w && proj_cols == 0) || in_h + 2 * pad_h < kernel_h || in_w + 2 * pad_w < kernel_w)
    return LC_INVALID_VALUE;
  if (head_dim > 256 || (proj_w && (head_dim > 128 || proj_cols > 128)) || seq > (size_t)INT_MAX)
    return LC_NOT_SUPPORTED;
  if (!conv_dims_fit_int(in_channels, in_h, in_w, out_channels, kernel_h, kernel_w, stride_h, stride_w, pad_h, pad_w))
    return LC_NOT_SUPPORTED;
  const size_t oh = (in_h + 2 * pad_h - kernel_h) / stride_h + 1;
  const size_t ow = (in_w + 2 * pad_w - kernel_w) / stride_w + 1;
  if (batch * oh * ow > (size_t)INT_MAX) return LC_NOT_SUPPORTED;
  const size_t img = out_channels * oh * ow;
  const size_t need = seq * head_dim;
  const size_t units = per_image ? batch : 1;
  const size_t avail = per_image ? img : batch * img;
  const bool short_conv = avail < 3 * need;
  // Scratch demand: the whole conv output, plus the packed Q/K/V when it must be repeated.
  const size_t demand = batch * img + (short_conv ? units * 3 * need : 0);
  if (demand > LC_NOALLOC_SCRATCH_FLOATS) return LC_INVALID_VALUE;  // over the fixed scratch size

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess) return from_cuda(e);
  float* conv = scratch;
  // The SIMT conv sizes its tile from cudaDeviceGetAttribute; it never creates the per-device
  // library context (whose error word is allocated), so this path allocates nothing even as the
  // first library call on a device.
  e = conv2d_nchw_f32_simt(x, w, bias, conv, (int)batch, (int)in_channels, (int)in_h, (int)in_w, (int)out_channels,
                      (int)kernel_h, (int)kernel_w, (int)stride_h, (int)stride_w, (int)pad_h, (int)pad_w, 1, s);
  if (e != cudaSuccess) return from_cuda(e);
  const float* qkv = conv;
  long long unit_stride = static_cast<long long>(img);
  if (short_conv) {
    float* packed = scratch + batch * img;
    for (size_t u = 0; u < units; ++u) {
      e = repeat_fill_f32(conv + u * img, avail, packed + u * 3 * need, 3 * need, s);
      if (e != cudaSuccess) return from_cuda(e);
    }
    qkv = packed;
    unit_stride = static_cast<long long>(3 * need);
  }
  const size_t cols = proj_w ? proj_cols : head_dim;
  for (size_t u0 = 0; u0 < units; u0 += 65535) {
    const size_t n = units - u0 < 65535 ? units - u0 : 65535;
    AttnArgs a{};
    a.q = qkv + u0 * unit_stride;
    a.k = qkv + u0 * unit_stride + need;
    a.v = qkv + u0 * unit_stride + 2 * need;
    a.out = out + u0 * seq * cols;
    a.q_unit_stride = a.k_unit_stride = a.v_unit_stride = unit_stride;
    a.out_unit_stride = static_cast<long long>(seq * cols);
    a.units = static_cast<int>(n);
    a.seq = static_cast<int>(seq);
    a.d = static_cast<int>(head_dim);
    a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    a.post_scale = 1.0f;
    a.proj_w = proj_w;
    a.proj_cols = static_cast<int>(proj_cols);
    e = attention_f32_simt(a, s);  // the tensor-core path would allocate its split planes
    if (e != cudaSuccess) return from_cuda(e);
  }
  return LC_SUCCESS;
}
