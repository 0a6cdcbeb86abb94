// Strict-fp32 SIMT GEMM and implicit-GEMM conv for sm_100a.
//
// The reference's fp32 contract (src/ops/matmul_cpu.cpp:49-60, max abs/rel error 1e-4 against
// it) rules out plain TF32 tensor cores, so these kernels accumulate with fp32 FFMA in k order,
// exactly the reduction order of the reference's i-p-j loop for each output element.
//
// Tiling: three CTA tiles (128x128 with 8x8 per thread, 128x64 with 8x8, both with BK = 8; 64x64
// with 4x4 and BK = 32), double-buffered shared memory; thread tiles are split into 4-wide strips so every
// shared-memory read is a conflict-free float4.  The tile comes from the auto-tune cache when it
// has an entry for the shape, else the largest tile that still gives every SM a CTA.
// The operands come from loader functors: dense row-major for matmul, an on-the-fly im2col
// gather (B side) for conv (the im2col matrix is never materialised); the epilogue functor writes
// row-major for matmul or NCHW (+bias, ReLU) for conv.
#include <cuda_bf16.h>

#include <cstring>

#include "lc_internal.hpp"

namespace lcb {
namespace {


template <typename T>
__device__ __forceinline__ float to_f(T v) { return static_cast<float>(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// Dense row-major A[m,k].
template <typename T>
struct DenseA {
  const T* a;
  int m, k;
  __device__ __forceinline__ float operator()(int r, int c) const {
    return (r < m && c < k) ? to_f(a[static_cast<long long>(r) * k + c]) : 0.0f;
  }
};
// Dense row-major B[k,n].
template <typename T>
struct DenseB {
  const T* b;
  int k, n;
  __device__ __forceinline__ float operator()(int r, int c) const {
    return (r < k && c < n) ? to_f(b[static_cast<long long>(r) * n + c]) : 0.0f;
  }
};
// Transposed im2col view of NCHW x: B[k = (c, ky, kx), col = (img, oy, ox)].  The k order is
// the reference's im2col column order (include/lightning_core/core/ops.hpp:1082-1084);
// out-of-image taps read as zero.  Conv runs as out^T[oc, pix] = W[oc, k] * im2col^T[k, pix] so
// that consecutive threads own consecutive pixels and the NCHW stores coalesce.
struct Im2colB {
  const float* x;
  int cols, kdim, in_c, in_h, in_w, kh, kw, sh, sw, ph, pw, oh, ow;
  __device__ __forceinline__ float operator()(int c, int r) const {
    if (r >= cols || c >= kdim) return 0.0f;
    const int hw = oh * ow;
    const int img = r / hw, pix = r - img * hw;
    const int oy = pix / ow, ox = pix - oy * ow;
    const int khw = kh * kw;
    const int ch = c / khw, rem = c - ch * khw;
    const int ky = rem / kw, kx = rem - ky * kw;
    const int y = oy * sh + ky - ph, xx = ox * sw + kx - pw;
    if (y < 0 || y >= in_h || xx < 0 || xx >= in_w) return 0.0f;
    return __ldg(x + ((static_cast<long long>(img) * in_c + ch) * in_h + y) * in_w + xx);
  }
};

template <typename T>
__device__ __forceinline__ void store_val(T* p, float v) { *p = static_cast<T>(v); }
template <>
__device__ __forceinline__ void store_val<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

template <typename T>
struct RowMajorEpi {
  T* c;
  int m, n;
  __device__ __forceinline__ void operator()(int r, int col, float v) const {
    if (r < m && col < n) store_val(c + static_cast<long long>(r) * n + col, v);
  }
};
// NCHW store of out^T[oc, pix] with bias + optional ReLU (ops.hpp:1196-1210).
struct NchwEpi {
  float* out;
  const float* bias;
  int rows, out_c, hw, relu;
  __device__ __forceinline__ void operator()(int oc, int r, float v) const {
    if (r >= rows || oc >= out_c) return;
    v += bias ? __ldg(bias + oc) : 0.0f;
    if (relu && v < 0.0f) v = 0.0f;
    const int img = r / hw, pix = r - img * hw;
    out[(static_cast<long long>(img) * out_c + oc) * hw + pix] = v;
  }
};

// Tile BM x BN per CTA, thread tile TM x TN (multiples of 4, split into 4-wide strips spaced
// BM/(TM/4) rows and BN/(TN/4) columns so every shared-memory read is a conflict-free float4).
// BK: k depth of a shared-memory stage.  The 64x64 tile is the one small problems get (few CTAs,
// bound by the latency of each stage's loads), so it takes 32-deep stages: a quarter of the
// load round trips per k; the larger tiles keep 8 (32-deep stages would not fit the 48 KB of
// static shared memory).
// The multiply-adds of every output still run in k order, so the results do not depend on BK.
template <int BM, int BN, int TM, int TN, int BK, class LA, class LB, class Epi>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
    simt_gemm_kernel(LA la, LB lb, Epi epi, int M, int N, int K) {
  constexpr int TX = BN / TN, TY = BM / TM, NT = TX * TY;
  constexpr int RS = BM / (TM / 4), CS = BN / (TN / 4);  // strip spacing
  constexpr int AE = BM * BK / NT, BE = BK * BN / NT;    // elements each thread stages
  static_assert(TM % 4 == 0 && TN % 4 == 0 && BK % AE == 0 && BN % BE == 0 && AE >= 1 && BE >= 1, "tile");
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];
  const int tid = threadIdx.x;
  const int tx = tid % TX, ty = tid / TX;
  const int row0 = blockIdx.y * BM, col0 = blockIdx.x * BN;
  const int a_r = tid / (BK / AE), a_k = (tid % (BK / AE)) * AE;   // AE consecutive k of one A row
  const int b_k = tid / (BN / BE), b_c = (tid % (BN / BE)) * BE;   // BE consecutive cols of one B row

  float ra[AE], rb[BE];
  auto gload = [&](int k0) {
#pragma unroll
    for (int i = 0; i < AE; ++i) ra[i] = la(row0 + a_r, k0 + a_k + i);
#pragma unroll
    for (int i = 0; i < BE; ++i) rb[i] = lb(k0 + b_k, col0 + b_c + i);
  };
  auto sstore = [&](int buf) {
#pragma unroll
    for (int i = 0; i < AE; ++i) As[buf][a_k + i][a_r] = ra[i];
#pragma unroll
    for (int i = 0; i < BE; ++i) Bs[buf][b_k][b_c + i] = rb[i];
  };

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

  const int ktiles = (K + BK - 1) / BK;
  gload(0);
  sstore(0);
  __syncthreads();
  for (int kt = 0; kt < ktiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ktiles) gload((kt + 1) * BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float av[TM], bv[TN];
#pragma unroll
      for (int g = 0; g < TM / 4; ++g) {
        const float4 a4 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4 + g * RS]);
        av[g * 4 + 0] = a4.x; av[g * 4 + 1] = a4.y; av[g * 4 + 2] = a4.z; av[g * 4 + 3] = a4.w;
      }
#pragma unroll
      for (int g = 0; g < TN / 4; ++g) {
        const float4 b4 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4 + g * CS]);
        bv[g * 4 + 0] = b4.x; bv[g * 4 + 1] = b4.y; bv[g * 4 + 2] = b4.z; bv[g * 4 + 3] = b4.w;
      }
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (kt + 1 < ktiles) {
      sstore(buf ^ 1);
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int r = row0 + ty * 4 + (i & 3) + (i >> 2) * RS;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int c = col0 + tx * 4 + (j & 3) + (j >> 2) * CS;
      epi(r, c, acc[i][j]);
    }
  }
}

template <int BM, int BN, int TM, int TN, int BK, class LA, class LB, class Epi>
cudaError_t run_tile(LA la, LB lb, Epi epi, int M, int N, int K, cudaStream_t s) {
  dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
  if (grid.y > 65535u) return cudaErrorInvalidConfiguration;
  simt_gemm_kernel<BM, BN, TM, TN, BK><<<grid, (BM / TM) * (BN / TN), 0, s>>>(la, lb, epi, M, N, K);
  return cudaGetLastError();
}

// Tile configurations (the names are the values stored in the auto-tune cache).
enum SimtTile { kSimt128x128 = 0, kSimt128x64, kSimt64x64, kSimtTileCount };
const char* const kSimtTileNames[kSimtTileCount] = {"simt128x128", "simt128x64", "simt64x64"};

// Without a cache entry: the largest tile that still gives every SM a CTA.
// Reads the SM count straight from the runtime (no DeviceCtx): the no-alloc pipeline runs this
// conv and must not create the per-device context, whose error word is a cudaMalloc.
int default_simt_tile(int M, int N) {
  int dev = 0, sm_count = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sm_count <= 0)
    sm_count = 148;
  const long long sms = sm_count;
  const long long big = static_cast<long long>((M + 127) / 128) * ((N + 127) / 128);
  if (big >= sms) return kSimt128x128;
  const long long mid = static_cast<long long>((M + 127) / 128) * ((N + 63) / 64);
  if (mid >= sms) return kSimt128x64;
  return kSimt64x64;
}

template <class LA, class LB, class Epi>
cudaError_t run(LA la, LB lb, Epi epi, int M, int N, int K, cudaStream_t s, int tile = -1) {
  if (tile < 0) tile = default_simt_tile(M, N);
  switch (tile) {
    case kSimt128x64: return run_tile<128, 64, 8, 8, 8>(la, lb, epi, M, N, K, s);
    case kSimt64x64: return run_tile<64, 64, 4, 4, 32>(la, lb, epi, M, N, K, s);
    default: return run_tile<128, 128, 8, 8, 8>(la, lb, epi, M, N, K, s);
  }
}

__global__ void repeat_fill_kernel(const float* src, size_t have, float* dst, size_t total) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = src[i % have];
}

}  // namespace

cudaError_t gemm_f32_tile(const float* a, const float* b, float* c, int m, int k, int n, int tile, cudaStream_t s) {
  return run(DenseA<float>{a, m, k}, DenseB<float>{b, k, n}, RowMajorEpi<float>{c, m, n}, m, n, k, s, tile);
}

int simt_tile_count() { return kSimtTileCount; }
const char* simt_tile_name(int t) { return (t >= 0 && t < kSimtTileCount) ? kSimtTileNames[t] : "?"; }
int simt_tile_from_name(const char* name) {
  for (int t = 0; t < kSimtTileCount; ++t)
    if (std::strcmp(name, kSimtTileNames[t]) == 0) return t;
  return -1;
}

cudaError_t gemm_bf16_simt(const __nv_bfloat16* a, const __nv_bfloat16* b, __nv_bfloat16* c, int m, int k, int n,
                           cudaStream_t s) {
  return run(DenseA<__nv_bfloat16>{a, m, k}, DenseB<__nv_bfloat16>{b, k, n}, RowMajorEpi<__nv_bfloat16>{c, m, n}, m,
             n, k, s);
}

cudaError_t conv2d_nchw_f32_simt(const float* x, const float* w, const float* bias, float* out, int batch, int in_c,
                                 int in_h, int in_w, int out_c, int kh, int kw, int sh, int sw, int ph, int pw,
                                 int relu, cudaStream_t s) {
  const int oh = (in_h + 2 * ph - kh) / sh + 1;
  const int ow = (in_w + 2 * pw - kw) / sw + 1;
  const int rows = batch * oh * ow;
  const int kdim = in_c * kh * kw;
  DenseA<float> la{w, out_c, kdim};  // OIHW is already W[oc, k] row-major
  Im2colB lb{x, rows, kdim, in_c, in_h, in_w, kh, kw, sh, sw, ph, pw, oh, ow};
  NchwEpi epi{out, bias, rows, out_c, oh * ow, relu};
  return run(la, lb, epi, out_c, rows, kdim, s);
}

cudaError_t repeat_fill_f32(const float* src, size_t have, float* dst, size_t total, cudaStream_t s) {
  if (have == 0) return cudaErrorInvalidValue;
  repeat_fill_kernel<<<592, 256, 0, s>>>(src, have, dst, total);
  return cudaGetLastError();
}

}  // namespace lcb
