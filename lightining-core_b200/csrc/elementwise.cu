// HBM-bound elementwise kernels.
//
// vector_add replaces src/ops/vector_add_cuda.cu:12-86 of the reference (a scalar grid-stride
// add followed by cudaDeviceSynchronize): 128-bit loads/stores, 4 independent vectors in flight
// per thread, grid sized to a multiple of the SM count, stream-ordered with no device sync.
// matrix_sub / matrix_div (src/ops/matrix_elemwise.cpp:8-29) are the same kernel with another
// operator (IEEE subtraction and division).
// layer_norm restates the reference's LN formula (README.md:2267-2270): per row of the last
// axis, (x - mean) / sqrt(var + eps), population variance, no affine; one warp per row, two
// passes over the row held in registers (mean first, then centred variance).
#include <math.h>

#include "lc_internal.hpp"

namespace lcb {
namespace {

struct OpAdd {
  template <typename S>
  __device__ __forceinline__ S operator()(S x, S y) const { return x + y; }
};
struct OpSub {
  template <typename S>
  __device__ __forceinline__ S operator()(S x, S y) const { return x - y; }
};
struct OpDiv {
  template <typename S>
  __device__ __forceinline__ S operator()(S x, S y) const { return x / y; }
};

template <typename V, typename S, int PER, class Op = OpAdd>
__global__ void __launch_bounds__(256) vadd_kernel(const S* __restrict__ a, const S* __restrict__ b,
                                                   S* __restrict__ out, size_t n) {
  const Op op;
  constexpr int L = sizeof(V) / sizeof(S);
  const size_t nv = n / L;
  const V* av = reinterpret_cast<const V*>(a);
  const V* bv = reinterpret_cast<const V*>(b);
  V* ov = reinterpret_cast<V*>(out);
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  for (; i + (PER - 1) * stride < nv; i += PER * stride) {
    V x[PER], y[PER];
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      x[u] = __ldcs(av + i + u * stride);
      y[u] = __ldcs(bv + i + u * stride);
    }
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      V z;
      const S* xs = reinterpret_cast<const S*>(&x[u]);
      const S* ys = reinterpret_cast<const S*>(&y[u]);
      S* zs = reinterpret_cast<S*>(&z);
#pragma unroll
      for (int e = 0; e < L; ++e) zs[e] = op(xs[e], ys[e]);
      __stcs(ov + i + u * stride, z);
    }
  }
  for (; i < nv; i += stride) {
    V x = av[i], y = bv[i], z;
    const S* xs = reinterpret_cast<const S*>(&x);
    const S* ys = reinterpret_cast<const S*>(&y);
    S* zs = reinterpret_cast<S*>(&z);
#pragma unroll
    for (int e = 0; e < L; ++e) zs[e] = op(xs[e], ys[e]);
    ov[i] = z;
  }
  // Scalar tail (n not a multiple of the vector width), handled by the first threads.
  const size_t tail0 = nv * L;
  const size_t t = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (tail0 + t < n) out[tail0 + t] = op(a[tail0 + t], b[tail0 + t]);
}

template <typename S, class Op = OpAdd>
__global__ void vadd_scalar_kernel(const S* a, const S* b, S* out, size_t n) {
  const Op op;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = op(a[i], b[i]);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename V, typename S, class Op = OpAdd>
cudaError_t vadd(const S* a, const S* b, S* out, size_t n, cudaStream_t s) {
  const int sms = device_ctx() ? device_ctx()->sm_count : 148;
  if (n == 0) return cudaSuccess;
  if (aligned16(a) && aligned16(b) && aligned16(out)) {
    constexpr int L = sizeof(V) / sizeof(S);
    const size_t nv = n / L;
    size_t blocks = (nv + 255) / 256;
    const size_t cap = static_cast<size_t>(sms) * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    vadd_kernel<V, S, 4, Op><<<static_cast<unsigned>(blocks), 256, 0, s>>>(a, b, out, n);
  } else {
    vadd_scalar_kernel<S, Op><<<sms * 8, 256, 0, s>>>(a, b, out, n);
  }
  return cudaGetLastError();
}

// One warp per row.  COLS_PER_LANE values per lane are kept in registers when the row fits
// (cols <= 32*MAXV), otherwise the row is streamed twice from global memory (L2-resident).
template <int MAXV>
__global__ void __launch_bounds__(256) layer_norm_kernel(const float* __restrict__ x, float* __restrict__ out,
                                                         size_t rows, size_t cols, float eps) {
  const size_t warp = (blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float* xr = x + warp * cols;
  float* orow = out + warp * cols;
  const bool vec = (cols % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) &&
                   ((reinterpret_cast<uintptr_t>(out) & 15u) == 0);
  if (vec && cols <= 32u * MAXV) {
    float4 r[MAXV / 4];
    float sum = 0.0f;
#pragma unroll
    for (int u = 0; u < MAXV / 4; ++u) {
      const size_t c = (static_cast<size_t>(u) * 32 + lane) * 4;
      r[u] = c < cols ? __ldg(reinterpret_cast<const float4*>(xr + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
      sum += (r[u].x + r[u].y) + (r[u].z + r[u].w);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const float mean = sum / static_cast<float>(cols);
    float var = 0.0f;
#pragma unroll
    for (int u = 0; u < MAXV / 4; ++u) {
      const size_t c = (static_cast<size_t>(u) * 32 + lane) * 4;
      if (c < cols) {
        const float a0 = r[u].x - mean, a1 = r[u].y - mean, a2 = r[u].z - mean, a3 = r[u].w - mean;
        var += (a0 * a0 + a1 * a1) + (a2 * a2 + a3 * a3);
      }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) var += __shfl_xor_sync(0xffffffffu, var, off);
    const float inv = 1.0f / sqrtf(var / static_cast<float>(cols) + eps);
#pragma unroll
    for (int u = 0; u < MAXV / 4; ++u) {
      const size_t c = (static_cast<size_t>(u) * 32 + lane) * 4;
      if (c < cols)
        __stcs(reinterpret_cast<float4*>(orow + c),
               make_float4((r[u].x - mean) * inv, (r[u].y - mean) * inv, (r[u].z - mean) * inv,
                           (r[u].w - mean) * inv));
    }
    return;
  }
  float sum = 0.0f;
  for (size_t c = lane; c < cols; c += 32) sum += xr[c];
#pragma unroll
  for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  const float mean = sum / static_cast<float>(cols);
  float var = 0.0f;
  for (size_t c = lane; c < cols; c += 32) {
    const float d = xr[c] - mean;
    var += d * d;
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) var += __shfl_xor_sync(0xffffffffu, var, off);
  const float inv = 1.0f / sqrtf(var / static_cast<float>(cols) + eps);
  for (size_t c = lane; c < cols; c += 32) orow[c] = (xr[c] - mean) * inv;
}

}  // namespace

cudaError_t vector_add_f32(const float* a, const float* b, float* out, size_t n, cudaStream_t s) {
  return vadd<float4, float>(a, b, out, n, s);
}
cudaError_t vector_add_f64(const double* a, const double* b, double* out, size_t n, cudaStream_t s) {
  return vadd<double2, double>(a, b, out, n, s);
}

cudaError_t matrix_binary(int op, int f64, const void* a, const void* b, void* out, size_t n, cudaStream_t s) {
  if (f64) {
    const double *x = static_cast<const double*>(a), *y = static_cast<const double*>(b);
    double* z = static_cast<double*>(out);
    return op == 0 ? vadd<double2, double, OpSub>(x, y, z, n, s) : vadd<double2, double, OpDiv>(x, y, z, n, s);
  }
  const float *x = static_cast<const float*>(a), *y = static_cast<const float*>(b);
  float* z = static_cast<float*>(out);
  return op == 0 ? vadd<float4, float, OpSub>(x, y, z, n, s) : vadd<float4, float, OpDiv>(x, y, z, n, s);
}

cudaError_t layer_norm_f32(const float* x, float* out, size_t rows, size_t cols, float eps, cudaStream_t s) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  const size_t blocks = (rows * 32 + 255) / 256;
  layer_norm_kernel<32><<<static_cast<unsigned>(blocks), 256, 0, s>>>(x, out, rows, cols, eps);
  return cudaGetLastError();
}

}  // namespace lcb
