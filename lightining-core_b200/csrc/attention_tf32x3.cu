// Strict-fp32 attention on the 5th-generation tensor cores, head_dim 64 (configs 1 and 5: the
// reference's fp32 attentionForward, src/attention_cpu.cpp:38-101, and the integrated
// conv->attention->projection pipeline, python/bindings/bind_integrated.cpp:614-730 with
// graph.hpp:3529-3547).  fp32 accuracy by the 3xTF32 split of every product:
//   x = x_hi + x_lo, x_hi = x rounded to tf32, x_lo = x - x_hi (exact in fp32);
//   x.y ~= x_hi.y_hi + x_hi.y_lo + x_lo.y_hi   (the dropped x_lo.y_lo is ~2^-22 |x y|).
// A pre-pass writes hi/lo planes of Q and K ([units, S, 64]) and of V transposed ([units, 64, Sp],
// Sp = S rounded up to 4), so every MMA operand is K-major in shared memory.
//
// One CTA = one 128-row Q tile, one CTA per SM (192 KB of shared memory), 352 threads:
//   warp 0      TMA: Q hi/lo once, K hi/lo tiles (64 keys) into a 2-stage ring freed by S_j;
//               warp 6: V^T hi/lo tiles into a 2-stage ring freed by P.V_j.
//   warp 1      MMA: S_j = Q K_j^T (3 x 8 tcgen05.mma.kind::tf32, M=128 N=64 K=8) into one of two
//               TMEM score buffers; O_j = P_j V_j (3 x 8 MMAs with P read from TMEM) into one of
//               two TMEM buffers, a fresh partial per tile.
//   warps 2..5, 7..10  softmax, two warps per query row (32 score/output columns each, row maxima
//               and sums swapped through shared memory): scores into registers, running max m (lazy:
//               rescale only when it grows by more than 2^8), p = 2^(s*scale*log2e - m), l += p,
//               P_hi over S_j's own columns and P_lo into its own buffer; then the previous
//               tile's O partial is folded into 32 per-thread fp32 registers, O = O*alpha + O_tile
//               (round-to-nearest adds: the tensor core's long fp32 accumulations drift).  The
//               epilogue divides by l, applies the optional projection out = O @ W (W [64, cols])
//               and the postprocess, and writes fp32 rows.
// Every mbarrier wait is bounded (common.cuh).
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>
#include <mutex>

#include "../../include/lc_b200.h"
#include "common.cuh"
#include "lc_internal.hpp"

namespace lcb {

void* tensor_map_encoder();

namespace {

constexpr int D = 64;
constexpr int TILE = 128;
constexpr int TK = 64;
constexpr int NUM_THREADS = 352;
constexpr int QCH = TILE * 128;       // one [128 rows x 32 fp32] swizzled chunk = 16 KB
constexpr int KCH = TK * 128;         // [64 keys x 32 fp32] = 8 KB
constexpr int VCH = D * 128;          // [64 d-rows x 32 keys] = 8 KB
constexpr int Q_PLANE = 2 * QCH;      // 32 KB (64 d)
constexpr int K_PLANE = 2 * KCH;      // 16 KB
constexpr int V_PLANE = 2 * VCH;      // 16 KB (64 keys)
constexpr int Q_OFF = 0;              // Q_hi, Q_lo
constexpr int K_OFF = 2 * Q_PLANE;    // 2 stages x (K_hi, K_lo)
constexpr int V_OFF = K_OFF + 2 * 2 * K_PLANE;
constexpr int TAIL_OFF = V_OFF + 2 * 2 * V_PLANE;
constexpr uint32_t S_COL = 0, PL_COL = 128, O_COL = 256, TMEM_COLS = 512;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_THRESHOLD = 8.0f;
constexpr uint32_t IDESC = idesc_tf32_f32(TILE, 64, 0, 0);  // S (N = 64 keys) and O (N = D = 64)

struct Tail {
  uint64_t q_full;
  uint64_t k_full[2], v_full[2];
  uint64_t s_full[2];   // S_j in TMEM (the S group's only commit)
  uint64_t p_full[2];   // P_hi/P_lo of tile j in TMEM (8 warp arrivals)
  uint64_t o_full[2];   // the O partial of tile j in TMEM (the P.V group's only commit)
  uint64_t o_free[2];   // the softmax warps have folded that partial (8 arrivals)
  uint64_t drain;
  // Row statistics exchanged between the two column halves of the softmax warps, tagged with
  // the tile index: [tile & 1][half][row] running maxima, and [half][row] final sums.
  unsigned long long xmax[2][2][TILE];
  unsigned long long xsum[2][TILE];
  uint32_t tmem_base;
  int abort_flag;
};
constexpr size_t SMEM_BYTES = 1024 + TAIL_OFF + sizeof(Tail);

struct Params {
  float* out;
  long long out_unit_stride;
  int units, seq, nq;
  int causal;
  float scale_log2;
  float post_scale, post_bias;
  int post_relu, post;
  const float* proj_w;
  int cols;  // output columns: D, or proj_cols with a projection
  unsigned* err_word;
};

__device__ __forceinline__ float tf32_round(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & 0xffffe000u;
  return __uint_as_float(u);
}

// 2^x, MUFU ex2 without flush-to-zero (relative error ~2^-22).
__device__ __forceinline__ float exp2_acc(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- pre-pass -----------------------------------------------------------------------------------
// Rows of 64 floats (unit u at src + u*unit_stride) -> contiguous hi/lo planes [units, S, 64],
// by `nblk` blocks of 256 threads (block `bx`), four floats per thread when the unit start is
// 16-byte aligned.
__device__ __forceinline__ void split_rows(const float* __restrict__ src, long long unit_stride, float* __restrict__ hi,
                                           float* __restrict__ lo, int seq, int u, int bx, int nblk) {
  const float* su = src + static_cast<long long>(u) * unit_stride;
  float* hu = hi + static_cast<long long>(u) * seq * D;
  float* lu = lo + static_cast<long long>(u) * seq * D;
  const int n = seq * D;
  if ((reinterpret_cast<uintptr_t>(su) & 15u) == 0) {
    for (int i = (bx * 256 + static_cast<int>(threadIdx.x)) * 4; i < n; i += nblk * 256 * 4) {
      const float4 v = *reinterpret_cast<const float4*>(su + i);
      const float4 h = make_float4(tf32_round(v.x), tf32_round(v.y), tf32_round(v.z), tf32_round(v.w));
      *reinterpret_cast<float4*>(hu + i) = h;
      *reinterpret_cast<float4*>(lu + i) = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
    }
  } else {
    for (int i = bx * 256 + static_cast<int>(threadIdx.x); i < n; i += nblk * 256) {
      const float v = su[i], h = tf32_round(v);
      hu[i] = h;
      lu[i] = v - h;
    }
  }
}
// One 32-key x 32-d tile of V [units][S][64] (unit stride) -> hi/lo planes of V^T [units][64][Sp],
// zero for keys >= S, through shared memory (coalesced both ways).
__device__ __forceinline__ void split_vt_tile(const float* __restrict__ v, long long unit_stride,
                                              float* __restrict__ hi_t, float* __restrict__ lo_t, int seq, int sp,
                                              int u, int k0, int d0, float (&tile)[32][33]) {
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const float* vu = v + static_cast<long long>(u) * unit_stride;
  for (int r = ty; r < 32; r += 8) {
    const int k = k0 + r;
    tile[r][tx] = k < seq ? vu[static_cast<long long>(k) * D + d0 + tx] : 0.0f;
  }
  __syncthreads();
  float* hu = hi_t + static_cast<long long>(u) * D * sp;
  float* lu = lo_t + static_cast<long long>(u) * D * sp;
  for (int r = ty; r < 32; r += 8) {
    const int d = d0 + r, k = k0 + tx;
    if (k < sp) {
      const float x = tile[tx][r];
      const float h = tf32_round(x);
      hu[static_cast<long long>(d) * sp + k] = h;
      lu[static_cast<long long>(d) * sp + k] = x - h;
    }
  }
}
// The whole pre-pass in one launch (blockIdx.y = unit): blocks [0, nrb) split Q's rows, [nrb,
// 2 nrb) K's rows (nrb = 0 when the caller supplies Q and K planes), the rest one V^T tile each.
__global__ void __launch_bounds__(256) split_qkv_kernel(const float* __restrict__ q, long long q_stride,
                                                        const float* __restrict__ k, long long k_stride,
                                                        const float* __restrict__ v, long long v_stride,
                                                        float* __restrict__ qh, float* __restrict__ ql,
                                                        float* __restrict__ kh, float* __restrict__ kl,
                                                        float* __restrict__ vh, float* __restrict__ vl, int seq,
                                                        int sp, int nrb) {
  griddep_launch_dependents();  // the attention may take its SMs now; it waits for these planes itself
  __shared__ float tile[32][33];
  const int u = blockIdx.y, bx = blockIdx.x;
  if (bx < nrb) {
    split_rows(q, q_stride, qh, ql, seq, u, bx, nrb);
  } else if (bx < 2 * nrb) {
    split_rows(k, k_stride, kh, kl, seq, u, bx - nrb, nrb);
  } else {
    const int t = bx - 2 * nrb;
    split_vt_tile(v, v_stride, vh, vl, seq, sp, u, (t >> 1) * 32, (t & 1) * 32, tile);
  }
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    fa_f32_tc_kernel(const __grid_constant__ CUtensorMap map_qh, const __grid_constant__ CUtensorMap map_ql,
                     const __grid_constant__ CUtensorMap map_kh, const __grid_constant__ CUtensorMap map_kl,
                     const __grid_constant__ CUtensorMap map_vh, const __grid_constant__ CUtensorMap map_vl,
                     const Params p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Tail* st = reinterpret_cast<Tail*>(smem + TAIL_OFF);
  uint8_t* sQh = smem + Q_OFF;
  uint8_t* sQl = sQh + Q_PLANE;
  auto sK = [&](int stage, int lo) { return smem + K_OFF + (stage * 2 + lo) * K_PLANE; };
  auto sV = [&](int stage, int lo) { return smem + V_OFF + (stage * 2 + lo) * V_PLANE; };

  griddep_wait();  // Q/K/V planes come from the split pre-pass (or the conv epilogue)
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qt = p.nq - 1 - static_cast<int>(blockIdx.x) % p.nq;
  const int unit = static_cast<int>(blockIdx.x) / p.nq;
  const int q0 = qt * TILE;
  const int kv_all = (p.seq + TK - 1) / TK;
  const int n_kv = p.causal ? min(kv_all, (q0 + TILE - 1) / TK + 1) : kv_all;

  if (threadIdx.x == 0) {
    mbar_init(&st->q_full, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&st->k_full[b], 1);
      mbar_init(&st->v_full[b], 1);
      mbar_init(&st->s_full[b], 1);
      mbar_init(&st->p_full[b], 8);
      mbar_init(&st->o_full[b], 1);
      mbar_init(&st->o_free[b], 8);
    }
    mbar_init(&st->drain, 1);
    st->abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&map_kh);
    tma_prefetch_desc(&map_kl);
    tma_prefetch_desc(&map_vh);
    tma_prefetch_desc(&map_vl);
    mbar_arrive_expect_tx(&st->q_full, 2 * Q_PLANE);
    for (int c = 0; c < 2; ++c) {
      tma_load_3d(sQh + c * QCH, &map_qh, c * 32, q0, unit, &st->q_full);
      tma_load_3d(sQl + c * QCH, &map_ql, c * 32, q0, unit, &st->q_full);
    }
  }
  for (int i = threadIdx.x; i < 2 * 2 * TILE; i += NUM_THREADS) (&st->xmax[0][0][0])[i] = ~0ull;
  for (int i = threadIdx.x; i < 2 * TILE; i += NUM_THREADS) (&st->xsum[0][0])[i] = ~0ull;
  if (warp == 0) {
    tmem_alloc(&st->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = st->tmem_base;
  volatile int* abort_flag = &st->abort_flag;
  auto drain = [](uint64_t* bar, uint32_t ph) {
    const uint64_t t1 = globaltimer_ns();
    while (!mbar_try_wait(bar, ph) && globaltimer_ns() - t1 < 100000000ull) {
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------ K loads
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        if (j + 2 < n_kv)  // warm L2 for the K tile that will take this slot next
          for (int c = 0; c < 2; ++c) {
            tma_prefetch_l2_3d(&map_kh, c * 32, (j + 2) * TK, unit);
            tma_prefetch_l2_3d(&map_kl, c * 32, (j + 2) * TK, unit);
          }
        // Slot s last held K_{j-2}; S_{j-2} (single commit: s_full[j&1]) must be done.  S_j needs
        // the load issued here, so the parity wait is unambiguous.
        if (j >= 2 && !mbar_wait_bounded(&st->s_full[s], ((j - 2) >> 1) & 1, abort_flag, p.err_word, kErrAttnLoadWait)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&st->k_full[s], 2 * K_PLANE);
        for (int c = 0; c < 2; ++c) {
          tma_load_3d(sK(s, 0) + c * KCH, &map_kh, c * 32, j * TK, unit, &st->k_full[s]);
          tma_load_3d(sK(s, 1) + c * KCH, &map_kl, c * 32, j * TK, unit, &st->k_full[s]);
        }
        ++issued;
      }
      if (!ok) {
        drain(&st->q_full, 0);
        for (int j = issued > 2 ? issued - 2 : 0; j < issued; ++j) drain(&st->k_full[j & 1], (j >> 1) & 1);
      }
    }
  } else if (warp == 6) {
    // ------------------------------------------------------------ V^T loads
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        if (j + 2 < n_kv)
          for (int c = 0; c < 2; ++c) {
            tma_prefetch_l2_3d(&map_vh, (j + 2) * TK + c * 32, 0, unit);
            tma_prefetch_l2_3d(&map_vl, (j + 2) * TK + c * 32, 0, unit);
          }
        // Slot s last held V_{j-2}; P.V_{j-2} (single commit: o_full[j&1]) must be done.
        if (j >= 2 && !mbar_wait_bounded(&st->o_full[s], ((j - 2) >> 1) & 1, abort_flag, p.err_word, kErrAttnLoadWait)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&st->v_full[s], 2 * V_PLANE);
        for (int c = 0; c < 2; ++c) {
          tma_load_3d(sV(s, 0) + c * VCH, &map_vh, j * TK + c * 32, 0, unit, &st->v_full[s]);
          tma_load_3d(sV(s, 1) + c * VCH, &map_vl, j * TK + c * 32, 0, unit, &st->v_full[s]);
        }
        ++issued;
      }
      if (!ok)
        for (int j = issued > 2 ? issued - 2 : 0; j < issued; ++j) drain(&st->v_full[j & 1], (j >> 1) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue (whole warp, elected lane)
    {
      bool ok = warp_wait_poll(&st->q_full, 0, abort_flag, p.err_word, kErrAttnMmaWait);
      bool issued = false;
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!warp_wait_poll(&st->k_full[s], (j >> 1) & 1, abort_flag, p.err_word, kErrAttnMmaWait)) return false;
        tc_fence_after();
        const uint32_t d = tmem + S_COL + static_cast<uint32_t>(s * TK);
        // Descriptors built once per tile and advanced by constant adds (address field: bytes / 16).
        const uint64_t qh = smem_desc_sw128(smem_u32(sQh), 16, 1024), ql = smem_desc_sw128(smem_u32(sQl), 16, 1024);
        const uint64_t kh = smem_desc_sw128(smem_u32(sK(s, 0)), 16, 1024);
        const uint64_t kl = smem_desc_sw128(smem_u32(sK(s, 1)), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 8; ++kk) {
          const uint32_t qo = ((kk >> 2) * QCH + (kk & 3) * 32) >> 4, ko = ((kk >> 2) * KCH + (kk & 3) * 32) >> 4;
          umma_tf32_ss_w(d, ql + qo, kh + ko, IDESC, kk > 0 ? 1u : 0u);
          umma_tf32_ss_w(d, qh + qo, kl + ko, IDESC, 1u);
          umma_tf32_ss_w(d, qh + qo, kh + ko, IDESC, 1u);
        }
        issued = true;
        umma_commit_w(&st->s_full[s]);  // the only commit of this group
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j & 1;
        if (j + 1 < n_kv && !issue_s(j + 1)) {
          ok = false;
          break;
        }
        // p_full[s] next completes for P_{j+2}, which needs S_{j+2} (issued after this wait);
        // v_full[s] next completes after this P.V; o_free[s] next completes for the fold of
        // tile j, which needs this P.V.
        if (!warp_wait_poll(&st->p_full[s], (j >> 1) & 1, abort_flag, p.err_word, kErrAttnMmaWait) ||
            !warp_wait_poll(&st->v_full[s], (j >> 1) & 1, abort_flag, p.err_word, kErrAttnMmaWait) ||
            (j >= 2 &&
             !warp_wait_poll(&st->o_free[s], ((j - 2) >> 1) & 1, abort_flag, p.err_word, kErrAttnMmaWait))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t o = tmem + O_COL + static_cast<uint32_t>(s * D);
        const uint32_t ph = tmem + S_COL + static_cast<uint32_t>(s * TK);   // P_hi over S_j
        const uint32_t pl = tmem + PL_COL + static_cast<uint32_t>(s * TK);  // P_lo
        const uint64_t vh = smem_desc_sw128(smem_u32(sV(s, 0)), 16, 1024);
        const uint64_t vl = smem_desc_sw128(smem_u32(sV(s, 1)), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < TK / 8; ++kk) {
          const uint32_t vo = ((kk >> 2) * VCH + (kk & 3) * 32) >> 4;
          umma_tf32_ts_w(o, pl + kk * 8, vh + vo, IDESC, kk > 0 ? 1u : 0u);
          umma_tf32_ts_w(o, ph + kk * 8, vl + vo, IDESC, 1u);
          umma_tf32_ts_w(o, ph + kk * 8, vh + vo, IDESC, 1u);
        }
        umma_commit_w(&st->o_full[s]);  // the only commit of this group
      }
      if (!ok && issued) {
        umma_commit_w(&st->drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&st->drain, 0) && globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else if ((warp >= 2 && warp <= 5) || warp >= 7) {
    // ------------------------------------------------------------ softmax, fold, epilogue
    // Two warps per TMEM lane quarter: half 0 (warps 2..5) owns score and output columns 0..31,
    // half 1 (warps 7..10) columns 32..63 of the same rows.  The halves swap row maxima per tile
    // (and sums at the end) through tagged shared-memory words.
    const int quarter = warp & 3;
    const int half = warp >= 7 ? 1 : 0;
    const int row = quarter * 32 + lane;
    const int qrow = q0 + row;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t hc = static_cast<uint32_t>(half * 32);
    const int kmax = p.causal ? min(qrow, p.seq - 1) : p.seq - 1;
    float m = -INFINITY, l = 0.0f, alpha_prev = 1.0f;
    float o_acc[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) o_acc[e] = 0.0f;
    bool ok = true;
    // Publishes v under `tag` in `mine` and returns the partner's value under the same tag.
    auto swap = [&](unsigned long long* mine, unsigned long long* theirs, uint32_t tag, float v, float* out) -> bool {
      const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
      *reinterpret_cast<volatile unsigned long long*>(mine) = w;
      volatile unsigned long long* t = theirs;
      unsigned long long x = *t;
      if (static_cast<uint32_t>(x >> 32) != tag) {
        const uint64_t t0 = globaltimer_ns();
        uint32_t spins = 0;
        while (static_cast<uint32_t>((x = *t) >> 32) != tag) {
          if (*abort_flag) return false;
          if ((++spins & 63u) == 0 && globaltimer_ns() - t0 > LC_WAIT_TIMEOUT_NS) {
            *abort_flag = 1;
            atomicCAS(p.err_word, 0u, static_cast<unsigned>(kErrAttnSoftmaxWait));
            return false;
          }
        }
      }
      *out = __uint_as_float(static_cast<uint32_t>(x));
      return true;
    };
    // Folds this half of the O partial of tile t (buffer t&1) into registers: o = o * alpha + O_t.
    auto fold = [&](int t, float alpha) -> bool {
      // o_full[t&1] next completes for P.V_{t+2}, which needs this fold's o_free first.
      if (!warp_wait_poll(&st->o_full[t & 1], (t >> 1) & 1, abort_flag, p.err_word, kErrAttnCorrectionWait)) return false;
      tc_fence_after();
      uint32_t r[32];
      tmem_ld32(tmem + lane_base + O_COL + static_cast<uint32_t>((t & 1) * D) + hc, r);
#pragma unroll
      for (int e = 0; e < 32; ++e) o_acc[e] = __fmaf_rn(o_acc[e], alpha, __uint_as_float(r[e]));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&st->o_free[t & 1]);
      return true;
    };
    for (int j = 0; j < n_kv; ++j) {
      const int s = j & 1;
      // s_full[s] next completes for S_{j+2}, which needs P_j from these warps first.
      if (!warp_wait_poll(&st->s_full[s], (j >> 1) & 1, abort_flag, p.err_word, kErrAttnSoftmaxWait)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sb = tmem + lane_base + S_COL + static_cast<uint32_t>(s * TK) + hc;
      uint32_t r[32];
      tmem_ld32(sb, r);
      const int kv0 = j * TK + half * 32;
      if (kv0 + 31 > kmax) {
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (kv0 + e > kmax) r[e] = __float_as_uint(-INFINITY);
      }
      float mx4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) mx4[i] = __uint_as_float(r[i]);
#pragma unroll
      for (int e = 4; e < 32; ++e) mx4[e & 3] = fmaxf(mx4[e & 3], __uint_as_float(r[e]));
      float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])), mo;
      // Slot [j&1] is rewritten for tile j+2 only after the partner published tile j+1, which it
      // does after reading this one.
      // The verdict is made warp-uniform: the tcgen05 loads and waits below are warp-collective.
      if (!__all_sync(0xffffffffu,
                      swap(&st->xmax[s][half][row], &st->xmax[s][half ^ 1][row], static_cast<uint32_t>(j), mx, &mo))) {
        ok = false;
        break;
      }
      mx = fmaxf(mx, mo) * p.scale_log2;
      float alpha = 1.0f;
      if (mx > m + RESCALE_THRESHOLD) {
        alpha = (m == -INFINITY) ? 0.0f : exp2f(m - mx);
        l *= alpha;
        m = mx;
      }
      // P_j: p = 2^(s*scale*log2e - m) in fp32 (finite, <= 2^8); P_hi over S_j's columns, P_lo
      // into its buffer.  The last reader of both buffers before this was P.V_{j-2}, issued
      // before S_j.
      float ls4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        uint32_t wh[16], wl[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float pv = exp2_acc(__fmaf_rn(__uint_as_float(r[g * 16 + i]), p.scale_log2, -m));
          const float ph = __uint_as_float((__float_as_uint(pv) + 0x1000u) & 0xffffe000u);
          ls4[i & 3] += pv;
          wh[i] = __float_as_uint(ph);
          wl[i] = __float_as_uint(pv - ph);
        }
        tmem_st16(sb + g * 16, wh);
        tmem_st16(tmem + lane_base + PL_COL + static_cast<uint32_t>(s * TK) + hc + g * 16, wl);
      }
      l += (ls4[0] + ls4[1]) + (ls4[2] + ls4[3]);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&st->p_full[s]);
      // Fold the previous tile's partial (computed with the previous max), then remember this
      // tile's rescale factor for its own fold.
      if (j > 0 && !fold(j - 1, alpha_prev)) {
        ok = false;
        break;
      }
      alpha_prev = alpha;
    }
    float lo_other = 0.0f;
    const bool fin = ok && fold(n_kv - 1, alpha_prev) &&
                     swap(&st->xsum[half][row], &st->xsum[half ^ 1][row], static_cast<uint32_t>(n_kv), l, &lo_other);
    const float inv = 1.0f / (half == 0 ? l + lo_other : lo_other + l);
    if (p.proj_w) {
      // Both halves stage their normalised outputs in the (now idle) Q buffers, rows padded to
      // 65 floats, and half of W ([64, cols], cols <= 128) each into this lane quarter's copy in
      // the (now idle) K/V rings; once both halves of all 32 rows of the quarter are there, each
      // of the two warps projects 16 of those rows with the lanes over output columns (W rows
      // and output lines contiguous).  out[r][c] = sum_e O[r][e] W[e][c] in e order.
      float* ep_base = reinterpret_cast<float*>(sQh);
      float* wsm = reinterpret_cast<float*>(smem + K_OFF) + quarter * (D * p.cols);
      for (int e = half * 32; e < half * 32 + 32; ++e)
        for (int c = lane; c < p.cols; c += 32) wsm[e * p.cols + c] = __ldg(p.proj_w + e * p.cols + c);
      __threadfence_block();
      bool rdy = true;
      if (fin && qrow < p.seq) {
        float* ep = ep_base + row * 65;
#pragma unroll
        for (int e = 0; e < 32; ++e) ep[half * 32 + e] = o_acc[e] * inv;
        __threadfence_block();
        // The ready flag reuses the max slots of tile n_kv, free by the same argument as a tile's.
        float dummy;
        const int fs = n_kv & 1;
        rdy = swap(&st->xmax[fs][half][row], &st->xmax[fs][half ^ 1][row], static_cast<uint32_t>(n_kv), 0.0f, &dummy);
      }
      if (__all_sync(0xffffffffu, fin && rdy)) {
        __threadfence_block();
        // All 16 rows at once: each W element read from shared memory feeds 32 independent
        // accumulator chains (16 rows x 2 columns per lane); every chain still sums e in order.
        constexpr int RB = 16;
        for (int rr = 0; rr < 16; rr += RB) {
          const int r0 = quarter * 32 + half * 16 + rr;
          if (q0 + r0 >= p.seq) break;
          const float* ep0 = ep_base + r0 * 65;
          for (int c0 = 0; c0 < p.cols; c0 += 64) {
            const int ca = c0 + lane, cb = c0 + 32 + lane;
            const bool va = ca < p.cols, vb = cb < p.cols;
            const int cal = va ? ca : 0, cbl = vb ? cb : 0;  // clamped reads; results masked on store
            float acc[RB][2];
#pragma unroll
            for (int i = 0; i < RB; ++i) acc[i][0] = acc[i][1] = 0.0f;
#pragma unroll 4
            for (int e = 0; e < D; ++e) {
              const float* wr = wsm + e * p.cols;
              const float wa = wr[cal], wb = wr[cbl];
#pragma unroll
              for (int i = 0; i < RB; ++i) {
                const float o = ep0[i * 65 + e];
                acc[i][0] = __fmaf_rn(o, wa, acc[i][0]);
                acc[i][1] = __fmaf_rn(o, wb, acc[i][1]);
              }
            }
#pragma unroll
            for (int i = 0; i < RB; ++i) {
              if (q0 + r0 + i >= p.seq) break;
              float* orow_r =
                  p.out + static_cast<long long>(unit) * p.out_unit_stride + static_cast<long long>(q0 + r0 + i) * p.cols;
              if (va) orow_r[ca] = acc[i][0];
              if (vb) orow_r[cb] = acc[i][1];
            }
          }
        }
      }
    } else if (fin && qrow < p.seq) {
      float* orow = p.out + static_cast<long long>(unit) * p.out_unit_stride + static_cast<long long>(qrow) * p.cols;
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        float y[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float v = o_acc[e + i] * inv;
          if (p.post) {
            v = v * p.post_scale + p.post_bias;
            if (p.post_relu && v < 0.0f) v = 0.0f;
          }
          y[i] = v;
        }
        reinterpret_cast<float4*>(orow + half * 32)[e / 4] = make_float4(y[0], y[1], y[2], y[3]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// fp32 [units, rows, cols] (contiguous), box [1, box_rows, 32], 128-byte swizzle, zero fill.
bool make_tmap_f32_3d(CUtensorMap* map, const void* base, int units, int rows, int cols, int box_rows) {
  auto enc = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!enc) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(units)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols) * 4, static_cast<cuuint64_t>(rows) * cols * 4};
  cuuint32_t box[3] = {32, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool attention_f32_tc_supported(const AttnArgs& a) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const int cols = a.proj_w ? a.proj_cols : a.d;
  // With a projection the epilogue stages W per lane quarter in the 128 KB of K/V rings: cols <= 128.
  return a.d == D && a.lse == nullptr && a.seq >= 1 && a.seq <= (1 << 24) && cols >= 1 &&
         cols <= (a.proj_w ? 128 : 256) && al(a.out) &&
         (a.out_unit_stride % 4) == 0 && (cols % 4 == 0 || a.proj_w != nullptr) &&
         !(a.proj_w && a.post_relu) && tensor_map_encoder() != nullptr;
}

cudaError_t attention_f32_tc_planes(const AttnArgs& a, float* ws, size_t nqk, size_t nv, int sp, DeviceCtx* ctx,
                                    cudaStream_t s, bool qk_ready);

size_t attention_f32_tc_ws_floats(int units, int seq) {
  const int sp = (seq + 3) & ~3;
  return 4 * static_cast<size_t>(units) * seq * D + 2 * static_cast<size_t>(units) * D * sp;
}

cudaError_t attention_f32_tc_presplit_qk(const AttnArgs& a, float* ws, cudaStream_t s) {
  DeviceCtx* ctx = device_ctx();
  if (!ctx) return cudaErrorNoDevice;
  const int sp = (a.seq + 3) & ~3;
  const size_t nqk = static_cast<size_t>(a.units) * a.seq * D, nv = static_cast<size_t>(a.units) * D * sp;
  return attention_f32_tc_planes(a, ws, nqk, nv, sp, ctx, s, true);
}

cudaError_t attention_f32_tc(const AttnArgs& a, cudaStream_t s) {
  DeviceCtx* ctx = device_ctx();
  if (!ctx) return cudaErrorNoDevice;
  const int sp = (a.seq + 3) & ~3;
  const size_t nqk = static_cast<size_t>(a.units) * a.seq * D, nv = static_cast<size_t>(a.units) * D * sp;
  const size_t bytes = (4 * nqk + 2 * nv) * sizeof(float);
  // Split planes in a stream-ordered workspace: allocated and freed on `s` around the kernels, so
  // calls on different streams run side by side.
  float* ws = nullptr;
  cudaError_t e = workspace_alloc(ctx, reinterpret_cast<void**>(&ws), bytes, s);
  if (e != cudaSuccess) return e;
  e = attention_f32_tc_planes(a, ws, nqk, nv, sp, ctx, s, false);
  const cudaError_t ef = workspace_free(ws, s);
  return e != cudaSuccess ? e : ef;
}

cudaError_t attention_f32_tc_planes(const AttnArgs& a, float* ws, size_t nqk, size_t nv, int sp, DeviceCtx* ctx,
                                    cudaStream_t s, bool qk_ready) {
  cudaError_t e = cudaSuccess;
  float* qh = ws;
  float* ql = qh + nqk;
  float* kh = ql + nqk;
  float* kl = kh + nqk;
  float* vh = kl + nqk;
  float* vl = vh + nv;
  CUtensorMap mqh, mql, mkh, mkl, mvh, mvl;
  if (!make_tmap_f32_3d(&mqh, qh, a.units, a.seq, D, TILE) || !make_tmap_f32_3d(&mql, ql, a.units, a.seq, D, TILE) ||
      !make_tmap_f32_3d(&mkh, kh, a.units, a.seq, D, TK) || !make_tmap_f32_3d(&mkl, kl, a.units, a.seq, D, TK) ||
      !make_tmap_f32_3d(&mvh, vh, a.units, D, sp, D) || !make_tmap_f32_3d(&mvl, vl, a.units, D, sp, D))
    return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> attr_done{0};  // devices with the attributes set
  {
    const cudaError_t ea = once_per_device(attr_done, [&]() -> cudaError_t {
      if ((e = cudaFuncSetAttribute(fa_f32_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(SMEM_BYTES))) != cudaSuccess)
        return e;
      return cudaSuccess;
    });
    if (ea != cudaSuccess) return ea;
  }
  // One pre-pass launch: Q and K row splits (unless the caller wrote those planes) and V^T tiles.
  const int nrb = qk_ready ? 0
                           : static_cast<int>(std::min<long long>((static_cast<long long>(a.seq) * D / 4 + 255) / 256, 64));
  const int nvt = ((sp + 31) / 32) * (D / 32);
  split_qkv_kernel<<<dim3(static_cast<unsigned>(2 * nrb + nvt), static_cast<unsigned>(a.units)), 256, 0, s>>>(
      static_cast<const float*>(a.q), a.q_unit_stride, static_cast<const float*>(a.k), a.k_unit_stride,
      static_cast<const float*>(a.v), a.v_unit_stride, qh, ql, kh, kl, vh, vl, a.seq, sp, nrb);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  Params p;
  p.out = static_cast<float*>(a.out);
  p.out_unit_stride = a.out_unit_stride;
  p.units = a.units;
  p.seq = a.seq;
  p.nq = (a.seq + TILE - 1) / TILE;
  p.causal = a.causal;
  p.scale_log2 = a.scale * LOG2E;
  p.post_scale = a.post_scale;
  p.post_bias = a.post_bias;
  p.post_relu = a.post_relu;
  p.post = !(a.post_scale == 1.0f && a.post_bias == 0.0f && !a.post_relu);
  p.proj_w = a.proj_w;
  p.cols = a.proj_w ? a.proj_cols : D;
  p.err_word = ctx->err_word;
  const long long grid = static_cast<long long>(p.nq) * a.units;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  return launch_pdl(fa_f32_tc_kernel, dim3(static_cast<unsigned>(grid)), dim3(NUM_THREADS), SMEM_BYTES, s, mqh, mql,
                    mkh, mkl, mvh, mvl, p);
}

}  // namespace lcb
