// Small-M matmul (m <= 2): C[m,n] = A[m,k] B[k,n], row-major, as a bandwidth-bound GEMV over B.
// Replaces the reference's dedicated small-M Metal path (src/ops/matmul_metal.mm:795-863 kernels,
// :1893-1912 dispatch) for the same shapes; the arithmetic contract is the matmul's
// (src/ops/matmul_cpu.cpp:49-60): fp32 accumulation, f32 or bf16 in/out.
//
// The work is reading B once (k*n elements); A's one or two rows are tiny.  A block of 256 threads
// covers 128 columns: 32 column groups of 4 consecutive columns (a warp reads 512 contiguous bytes
// of a B row in f32) times 8 k-lanes that stride through the block's k range; the 8 partial sums
// are folded in shared memory.  When 128-column blocks alone cannot fill the GPU, k is split
// across blockIdx.y and the per-split partial rows are summed by a second small kernel (partials in
// a stream-ordered workspace).  Each B element is read once, so the kernel runs at HBM bandwidth.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "lc_internal.hpp"

namespace lcb {
namespace {

constexpr int kCols = 128;   // columns per block
constexpr int kLanesK = 8;   // k-lanes per block
constexpr int kThreads = 256;

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
template <class T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Four consecutive elements of a B row starting at column c (bounds- and alignment-checked).
template <class T>
__device__ __forceinline__ void load4(const T* row, int c, int n, bool vec, float (&v)[4]) {
  if (vec && c + 3 < n) {
    if constexpr (sizeof(T) == 4) {
      const float4 x = *reinterpret_cast<const float4*>(row + c);
      v[0] = x.x, v[1] = x.y, v[2] = x.z, v[3] = x.w;
    } else {
      const uint2 x = *reinterpret_cast<const uint2*>(row + c);
      v[0] = __uint_as_float(x.x << 16), v[1] = __uint_as_float(x.x & 0xffff0000u);
      v[2] = __uint_as_float(x.y << 16), v[3] = __uint_as_float(x.y & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = c + j < n ? to_f(row[c + j]) : 0.0f;
  }
}

template <class T, int MR>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                                        T* __restrict__ c, float* __restrict__ part, int k, int n,
                                                        int kchunk, bool vec) {
  __shared__ float red[kLanesK][MR][kCols];
  const int cg = threadIdx.x & 31, kl = threadIdx.x >> 5;
  const int col0 = blockIdx.x * kCols + cg * 4;
  const int k0 = blockIdx.y * kchunk;
  const int k1 = min(k, k0 + kchunk);
  float acc[MR][4] = {};
  int kk = k0 + kl;
  // Four B rows per iteration: their loads are independent, so four are in flight per thread.
  for (; kk + 3 * kLanesK < k1; kk += 4 * kLanesK) {
    float bv[4][4];
#pragma unroll
    for (int u = 0; u < 4; ++u) load4(b + static_cast<long long>(kk + u * kLanesK) * n, col0, n, vec, bv[u]);
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        const float av = to_f(a[static_cast<long long>(r) * k + kk + u * kLanesK]);
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[r][j] = fmaf(av, bv[u][j], acc[r][j]);
      }
  }
  for (; kk < k1; kk += kLanesK) {
    float bv[4];
    load4(b + static_cast<long long>(kk) * n, col0, n, vec, bv);
#pragma unroll
    for (int r = 0; r < MR; ++r) {
      const float av = to_f(a[static_cast<long long>(r) * k + kk]);
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[r][j] = fmaf(av, bv[j], acc[r][j]);
    }
  }
#pragma unroll
  for (int r = 0; r < MR; ++r)
#pragma unroll
    for (int j = 0; j < 4; ++j) red[kl][r][cg * 4 + j] = acc[r][j];
  __syncthreads();
  for (int i = threadIdx.x; i < MR * kCols; i += kThreads) {
    const int r = i / kCols, cc = i % kCols, col = blockIdx.x * kCols + cc;
    float s = 0.0f;
#pragma unroll
    for (int l = 0; l < kLanesK; ++l) s += red[l][r][cc];
    if (col < n) {
      if (gridDim.y == 1)
        c[static_cast<long long>(r) * n + col] = from_f<T>(s);
      else
        part[(static_cast<long long>(blockIdx.y) * MR + r) * n + col] = s;
    }
  }
}

template <class T>
__global__ void gemv_reduce_kernel(const float* __restrict__ part, T* __restrict__ c, int splits, int rows, int n) {
  const long long total = static_cast<long long>(rows) * n;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float s = 0.0f;
    for (int sp = 0; sp < splits; ++sp) s += part[sp * total + i];
    c[i] = from_f<T>(s);
  }
}

template <class T>
cudaError_t gemv(const T* a, const T* b, T* c, int m, int k, int n, cudaStream_t s) {
  if (m < 1 || m > 2) return cudaErrorInvalidValue;
  DeviceCtx* ctx = device_ctx();
  if (!ctx) return cudaErrorNoDevice;
  const int cblocks = (n + kCols - 1) / kCols;
  const int want = ctx->sm_count * 8;  // blocks to keep every SM's loads in flight
  int splits = cblocks >= want ? 1 : (want + cblocks - 1) / cblocks;
  const int max_splits = (k + 63) / 64;  // at least 64 k-rows per split
  if (splits > max_splits) splits = max_splits;
  if (splits > 65535) splits = 65535;
  if (splits < 1) splits = 1;
  int kchunk = (k + splits - 1) / splits;
  kchunk = (kchunk + kLanesK - 1) / kLanesK * kLanesK;
  splits = (k + kchunk - 1) / kchunk;
  const bool vec = (n % 4 == 0) && (reinterpret_cast<uintptr_t>(b) % (4 * sizeof(T)) == 0);
  float* part = nullptr;
  cudaError_t e = cudaSuccess;
  if (splits > 1 &&
      (e = workspace_alloc(ctx, reinterpret_cast<void**>(&part),
                           static_cast<size_t>(splits) * m * n * sizeof(float), s)) != cudaSuccess)
    return e;
  const dim3 grid(cblocks, splits);
  if (m == 1)
    gemv_kernel<T, 1><<<grid, kThreads, 0, s>>>(a, b, c, part, k, n, kchunk, vec);
  else
    gemv_kernel<T, 2><<<grid, kThreads, 0, s>>>(a, b, c, part, k, n, kchunk, vec);
  e = cudaGetLastError();
  if (e == cudaSuccess && splits > 1) {
    const long long total = static_cast<long long>(m) * n;
    const int blocks = static_cast<int>(total / 256 + 1 < 4096 ? total / 256 + 1 : 4096);
    gemv_reduce_kernel<T><<<blocks, 256, 0, s>>>(part, c, splits, m, n);
    e = cudaGetLastError();
  }
  if (part) {
    const cudaError_t ef = workspace_free(part, s);
    if (e == cudaSuccess) e = ef;
  }
  return e;
}

}  // namespace

cudaError_t gemv_f32(const float* a, const float* b, float* c, int m, int k, int n, cudaStream_t s) {
  return gemv<float>(a, b, c, m, k, n, s);
}
cudaError_t gemv_bf16(const __nv_bfloat16* a, const __nv_bfloat16* b, __nv_bfloat16* c, int m, int k, int n,
                      cudaStream_t s) {
  return gemv<__nv_bfloat16>(a, b, c, m, k, n, s);
}

}  // namespace lcb
