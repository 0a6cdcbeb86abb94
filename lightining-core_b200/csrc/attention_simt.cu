// Flash-style attention forward on CUDA cores, strict fp32 arithmetic.
//
// Restates src/attention_cpu.cpp:38-101 of the reference without the S x S buffers: per query
// row, scores s_j = (q_i . k_j) * (1/sqrt(d)) with j > i masked when causal, softmax with the
// running row maximum, and out_i = sum_j p_j v_j -- computed tile by tile with the usual
// online-softmax rescaling, so memory is O(S) and nothing but Q, K, V and O touches HBM.
// The postprocess of src/attention.cpp:41-60 (out*scale + bias, optional ReLU) and, for the
// integrated conv->attention pipeline, the projection attn_out[S, d] @ W[d, P]
// (include/lightning_core/core/graph.hpp:3529-3547) run in the epilogue.
//
// This is the kernel for the fp32 contract (|err| <= 1e-4 + 1e-4|ref|), which plain TF32 tensor
// cores cannot meet, and the fallback for bf16 head dims the tcgen05 kernel does not take.
//
// CTA = 256 threads, 64 query rows x 64-key tiles.  Thread t owns rows (t>>4)*4 .. +3; its 16
// lanes t&15 of that row group split the 64 score columns (4 each) and the output columns, so
// row max / sum reductions are 4 xor-shuffles inside a half warp.  Q^T and K^T are staged
// transposed so every shared-memory read in the two inner products is a float4.
#include <cuda_bf16.h>
#include <math.h>

#include <string>

#include "../../include/lc_b200.h"
#include "lc_internal.hpp"

namespace lcb {
namespace {

constexpr int TQ = 64, TK = 64, NT = 256;

template <typename T>
__device__ __forceinline__ float ld_f(const T* p) { return static_cast<float>(*p); }
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <typename T>
__device__ __forceinline__ void st_f(T* p, float v) { *p = static_cast<T>(v); }
template <>
__device__ __forceinline__ void st_f<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

// DP: padded head dim (64, 128 or 256); columns >= d are zero in Q/K/V staging.
template <int DP, typename T>
__global__ void __launch_bounds__(NT) attn_simt_kernel(AttnArgs a) {
  extern __shared__ __align__(16) float smem[];
  float* Qt = smem;              // [DP][TQ]
  float* Kt = Qt + DP * TQ;      // [DP][TK]
  float* Vs = Kt + DP * TK;      // [TK][DP]
  float* Pt = Vs + TK * DP;      // [TK][TQ]
  float* Ws = Pt + TK * TQ;      // [d][P] (projection only)

  const int tid = threadIdx.x;
  const int rg = tid >> 4, cg = tid & 15;
  const int unit = blockIdx.y;
  const int q0 = blockIdx.x * TQ;
  const int S = a.seq, D = a.d;
  const T* q = static_cast<const T*>(a.q) + unit * a.q_unit_stride;
  const T* k = static_cast<const T*>(a.k) + unit * a.k_unit_stride;
  const T* v = static_cast<const T*>(a.v) + unit * a.v_unit_stride;

  // Stage Q^T: element (r, c) -> Qt[c][r]; r fastest across threads (conflict-free stores).
  for (int idx = tid; idx < TQ * DP; idx += NT) {
    const int r = idx % TQ, c = idx / TQ;
    const int gr = q0 + r;
    Qt[c * TQ + r] = (gr < S && c < D) ? ld_f(q + static_cast<long long>(gr) * D + c) : 0.0f;
  }

  constexpr int DC = DP / 16;  // output columns per thread: (g*16 + cg)*4 + e, g < DP/64
  float o[4][DC];
  float m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.0f;
#pragma unroll
    for (int j = 0; j < DC; ++j) o[i][j] = 0.0f;
  }

  int kv_end = S;
  if (a.causal) kv_end = min(S, q0 + TQ);
  const int ntiles = (kv_end + TK - 1) / TK;
  for (int t = 0; t < ntiles; ++t) {
    const int k0 = t * TK;
    __syncthreads();  // previous tile's Kt/Vs/Pt fully consumed
    for (int idx = tid; idx < TK * DP; idx += NT) {
      const int j = idx % TK, c = idx / TK;
      const int gj = k0 + j;
      Kt[c * TK + j] = (gj < S && c < D) ? ld_f(k + static_cast<long long>(gj) * D + c) : 0.0f;
    }
    for (int idx = tid; idx < TK * DP; idx += NT) {
      const int c = idx % DP, j = idx / DP;
      const int gj = k0 + j;
      Vs[j * DP + c] = (gj < S && c < D) ? ld_f(v + static_cast<long long>(gj) * D + c) : 0.0f;
    }
    __syncthreads();

    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
#pragma unroll 8
    for (int c = 0; c < DP; ++c) {
      const float4 qa = *reinterpret_cast<const float4*>(Qt + c * TQ + rg * 4);
      const float4 kb = *reinterpret_cast<const float4*>(Kt + c * TK + cg * 4);
      const float qv[4] = {qa.x, qa.y, qa.z, qa.w};
      const float kv[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
    }

    // Scale, mask, online softmax (row statistics over the 16 lanes of this row group).
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int gi = q0 + rg * 4 + i;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int gj = k0 + cg * 4 + j;
        float x = s[i][j] * a.scale;
        if (gj >= S || (a.causal && gj > gi)) x = -INFINITY;
        s[i][j] = x;
        mx = fmaxf(mx, x);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m[i], mx);
      // A fully masked row so far keeps m = -inf; use 0 as the reference point then.
      const float m_use = (m_new == -INFINITY) ? 0.0f : m_new;
      const float corr = expf(m[i] - m_use);
      float sum = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = expf(s[i][j] - m_use);
        s[i][j] = p;
        sum += p;
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      l[i] = l[i] * corr + sum;
      m[i] = m_new;
#pragma unroll
      for (int j = 0; j < DC; ++j) o[i][j] *= corr;
    }
    // P^T to shared memory: Pt[j][row].
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<float4*>(Pt + (cg * 4 + j) * TQ + rg * 4) = make_float4(s[0][j], s[1][j], s[2][j], s[3][j]);
    __syncthreads();

    const int jmax = min(TK, kv_end - k0);
#pragma unroll 4
    for (int j = 0; j < jmax; ++j) {
      const float4 pa = *reinterpret_cast<const float4*>(Pt + j * TQ + rg * 4);
      const float pv[4] = {pa.x, pa.y, pa.z, pa.w};
#pragma unroll
      for (int g = 0; g < DP / 64; ++g) {
        const float4 vb = *reinterpret_cast<const float4*>(Vs + j * DP + (g * 16 + cg) * 4);
        const float vv[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int e = 0; e < 4; ++e) o[i][g * 4 + e] = fmaf(pv[i], vv[e], o[i][g * 4 + e]);
      }
    }
  }

  // Row log-sum-exp (natural log, scaled-score units) for the train step's dV recomputation.
  if (a.lse != nullptr && cg == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int gi = q0 + rg * 4 + i;
      if (gi < S) a.lse[static_cast<long long>(unit) * S + gi] = m[i] + logf(l[i]);
    }
  }

  // Normalise, postprocess.
  const bool post = !(a.post_scale == 1.0f && a.post_bias == 0.0f && !a.post_relu);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float inv = 1.0f / l[i];
#pragma unroll
    for (int j = 0; j < DC; ++j) {
      float x = o[i][j] * inv;
      if (post) {
        x = x * a.post_scale + a.post_bias;
        if (a.post_relu && x < 0.0f) x = 0.0f;
      }
      o[i][j] = x;
    }
  }

  if (a.proj_w == nullptr) {
    T* out = static_cast<T*>(a.out) + unit * a.out_unit_stride;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int gi = q0 + rg * 4 + i;
      if (gi >= S) continue;
#pragma unroll
      for (int g = 0; g < DP / 64; ++g)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = (g * 16 + cg) * 4 + e;
          if (c < D) st_f(out + static_cast<long long>(gi) * D + c, o[i][g * 4 + e]);
        }
    }
    return;
  }

  // Fused projection: out[i, :] = attn[i, :] @ W, sequential over the d inner index.
  const int P = a.proj_cols;
  __syncthreads();
  float* Os = Qt;  // reuse: [TQ][DP]
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int g = 0; g < DP / 64; ++g)
#pragma unroll
      for (int e = 0; e < 4; ++e) Os[(rg * 4 + i) * DP + (g * 16 + cg) * 4 + e] = o[i][g * 4 + e];
  for (int idx = tid; idx < D * P; idx += NT) Ws[idx] = __ldg(a.proj_w + idx);
  __syncthreads();
  float* out = static_cast<float*>(a.out) + unit * a.out_unit_stride;
  for (int col = cg; col < P; col += 16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = rg * 4 + i;
      float acc = 0.0f;
      for (int c = 0; c < D; ++c) acc = fmaf(Os[r * DP + c], Ws[c * P + col], acc);
      const int gi = q0 + r;
      if (gi < S) out[static_cast<long long>(gi) * P + col] = acc;
    }
  }
}

template <int DP, typename T>
cudaError_t launch(const AttnArgs& a, cudaStream_t s) {
  size_t smem = sizeof(float) * (3 * DP * 64 + 64 * 64);
  if (a.proj_w) smem += sizeof(float) * a.d * a.proj_cols;
  cudaError_t e = cudaFuncSetAttribute(attn_simt_kernel<DP, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  dim3 grid((a.seq + TQ - 1) / TQ, a.units);
  if (grid.y > 65535u) return cudaErrorInvalidConfiguration;
  attn_simt_kernel<DP, T><<<grid, NT, smem, s>>>(a);
  return cudaGetLastError();
}

template <typename T>
cudaError_t dispatch(const AttnArgs& a, cudaStream_t s) {
  if (a.proj_w && (a.d > 128 || a.proj_cols > 128 || sizeof(T) != 4)) return cudaErrorNotSupported;
  if (a.d <= 64) return launch<64, T>(a, s);
  if (a.d <= 128) return launch<128, T>(a, s);
  if (a.d <= 256) return launch<256, T>(a, s);
  return cudaErrorNotSupported;
}

// ---- train step (src/attention_cpu.cpp:114-163) ------------------------------------------------

// dO = 2 (O - T) / (seq*d); sse[u] += sum (O - T)^2 over unit u (double accumulation).
__global__ void train_grad_out_kernel(const float* __restrict__ out, const float* __restrict__ target,
                                      float* __restrict__ dout, double* __restrict__ sse, long long per_unit) {
  const int unit = blockIdx.y;
  const float norm = 1.0f / static_cast<float>(per_unit);
  const long long base = static_cast<long long>(unit) * per_unit;
  double acc = 0.0;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < per_unit;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float diff = out[base + i] - target[base + i];
    acc += static_cast<double>(diff) * diff;
    dout[base + i] = 2.0f * diff * norm;
  }
  for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  __shared__ double part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += part[w];
    atomicAdd(sse + unit, t);
  }
}

// dV for a tile of 64 keys, recomputing P^T = exp(K Q^T * scale - lse) tile by tile (no S x S
// buffer), accumulating dV[j] = sum_i P[i][j] dO[i] over query rows i in increasing order (the
// reference's loop order), then v[j] -= lr * dV[j] in place (dV never reads v).
// Same thread layout as attn_simt_kernel: thread t owns keys (t>>4)*4 .. +3 of the tile.
template <int DP>
__global__ void __launch_bounds__(NT) attn_dv_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                     float* __restrict__ v, const float* __restrict__ dout,
                                                     const float* __restrict__ lse, int S, int D, int causal,
                                                     float scale, float lr) {
  extern __shared__ __align__(16) float smem[];
  float* Kt = smem;              // [DP][TK]  keys of this block (the "rows" here)
  float* Qt = Kt + DP * TK;      // [DP][TQ]  query rows of the current tile
  float* Gs = Qt + DP * TQ;      // [TQ][DP]  dO rows of the current tile
  float* Pt = Gs + TQ * DP;      // [TQ][TK]  P^T tile: Pt[i][j]
  float* Ls = Pt + TQ * TK;      // [TQ]      lse of the current query rows
  const int tid = threadIdx.x;
  const int rg = tid >> 4, cg = tid & 15;
  const int unit = blockIdx.y;
  const int k0 = blockIdx.x * TK;
  const long long ub = static_cast<long long>(unit) * S * D;
  for (int idx = tid; idx < TK * DP; idx += NT) {
    const int j = idx % TK, c = idx / TK;
    const int gj = k0 + j;
    Kt[c * TK + j] = (gj < S && c < D) ? k[ub + static_cast<long long>(gj) * D + c] : 0.0f;
  }
  constexpr int DC = DP / 16;
  float dv[4][DC];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < DC; ++j) dv[i][j] = 0.0f;

  // Causal: query rows i < k0 see none of these keys.
  const int qt0 = causal ? k0 / TQ : 0;
  const int nqt = (S + TQ - 1) / TQ;
  for (int t = qt0; t < nqt; ++t) {
    const int i0 = t * TQ;
    __syncthreads();
    for (int idx = tid; idx < TQ * DP; idx += NT) {
      const int r = idx % TQ, c = idx / TQ;
      const int gi = i0 + r;
      Qt[c * TQ + r] = (gi < S && c < D) ? q[ub + static_cast<long long>(gi) * D + c] : 0.0f;
    }
    for (int idx = tid; idx < TQ * DP; idx += NT) {
      const int c = idx % DP, r = idx / DP;
      const int gi = i0 + r;
      Gs[r * DP + c] = (gi < S && c < D) ? dout[ub + static_cast<long long>(gi) * D + c] : 0.0f;
    }
    for (int r = tid; r < TQ; r += NT) Ls[r] = (i0 + r < S) ? lse[static_cast<long long>(unit) * S + i0 + r] : 0.0f;
    __syncthreads();
    // S^T[j][i] for this thread's 4 keys x 4 query rows (cols cg*4..).
    float st[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) st[a][b] = 0.0f;
#pragma unroll 8
    for (int c = 0; c < DP; ++c) {
      const float4 ka = *reinterpret_cast<const float4*>(Kt + c * TK + rg * 4);
      const float4 qb = *reinterpret_cast<const float4*>(Qt + c * TQ + cg * 4);
      const float kv[4] = {ka.x, ka.y, ka.z, ka.w};
      const float qv[4] = {qb.x, qb.y, qb.z, qb.w};
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) st[a][b] = fmaf(kv[a], qv[b], st[a][b]);
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int gj = k0 + rg * 4 + a;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int li = cg * 4 + b, gi = i0 + li;
        float pv = expf(st[a][b] * scale - Ls[li]);
        if (gi >= S || gj >= S || (causal && gj > gi)) pv = 0.0f;
        Pt[li * TK + rg * 4 + a] = pv;
      }
    }
    __syncthreads();
    const int imax = min(TQ, S - i0);
#pragma unroll 4
    for (int i = 0; i < imax; ++i) {
      const float4 pa = *reinterpret_cast<const float4*>(Pt + i * TK + rg * 4);
      const float pv[4] = {pa.x, pa.y, pa.z, pa.w};
#pragma unroll
      for (int g = 0; g < DP / 64; ++g) {
        const float4 gb = *reinterpret_cast<const float4*>(Gs + i * DP + (g * 16 + cg) * 4);
        const float gv[4] = {gb.x, gb.y, gb.z, gb.w};
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int e = 0; e < 4; ++e) dv[a][g * 4 + e] = fmaf(pv[a], gv[e], dv[a][g * 4 + e]);
      }
    }
  }
  // SGD on V (src/attention_cpu.cpp:157-159).
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int gj = k0 + rg * 4 + a;
    if (gj >= S) continue;
#pragma unroll
    for (int g = 0; g < DP / 64; ++g)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c = (g * 16 + cg) * 4 + e;
        if (c < D) v[ub + static_cast<long long>(gj) * D + c] -= lr * dv[a][g * 4 + e];
      }
  }
}

template <int DP>
cudaError_t launch_dv(const float* q, const float* k, float* v, const float* dout, const float* lse, int units, int S,
                      int D, int causal, float scale, float lr, cudaStream_t s) {
  const size_t smem = sizeof(float) * (DP * TK + DP * TQ + TQ * DP + TQ * TK + TQ);
  cudaError_t e = cudaFuncSetAttribute(attn_dv_kernel<DP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  dim3 grid((S + TK - 1) / TK, units);
  if (grid.y > 65535u) return cudaErrorInvalidConfiguration;
  attn_dv_kernel<DP><<<grid, NT, smem, s>>>(q, k, v, dout, lse, S, D, causal, scale, lr);
  return cudaGetLastError();
}

}  // namespace

cudaError_t attention_train_grad_out(const float* out, const float* target, float* dout, double* sse, int units,
                                     long long per_unit, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(sse, 0, sizeof(double) * units, s);
  if (e != cudaSuccess) return e;
  long long blocks = (per_unit + 255) / 256;
  if (blocks > 64) blocks = 64;
  if (units > 65535) return cudaErrorInvalidConfiguration;
  train_grad_out_kernel<<<dim3(static_cast<unsigned>(blocks), units), 256, 0, s>>>(out, target, dout, sse, per_unit);
  return cudaGetLastError();
}

cudaError_t attention_train_dv_update(const float* q, const float* k, float* v, const float* dout, const float* lse,
                                      int units, int seq, int d, int causal, float scale, float lr, cudaStream_t s) {
  if (d <= 64) return launch_dv<64>(q, k, v, dout, lse, units, seq, d, causal, scale, lr, s);
  if (d <= 128) return launch_dv<128>(q, k, v, dout, lse, units, seq, d, causal, scale, lr, s);
  return cudaErrorNotSupported;
}

cudaError_t attention_f32_simt(const AttnArgs& a, cudaStream_t s) { return dispatch<float>(a, s); }

// fp32 attention: the 3xTF32 tensor-core kernel where it applies (head_dim 64, no LSE output),
// unless the tune cache pins the SIMT kernel for the shape.
cudaError_t attention_f32(const AttnArgs& a, cudaStream_t s) {
  std::string cfg;
  const bool pinned_simt = tune_lookup(LC_TUNE_ATTENTION, a.seq, a.d, a.causal, LC_DTYPE_F32, &cfg) && cfg == "simt";
  if (!pinned_simt && attention_f32_tc_supported(a)) return attention_f32_tc(a, s);
  return attention_f32_simt(a, s);
}
cudaError_t attention_bf16_simt(const AttnArgs& a, cudaStream_t s) { return dispatch<__nv_bfloat16>(a, s); }

}  // namespace lcb
