// Strict-fp32 GEMM on the 5th-generation tensor cores by the 3xTF32 split:
//   a = a_hi + a_lo with a_hi = a rounded to tf32 and a_lo = a - a_hi (exact in fp32), likewise b,
//   C = a_hi b_hi + a_hi b_lo + a_lo b_hi  (the dropped a_lo b_lo term is ~2^-22 |a b|),
// accumulated in fp32 in TMEM.  Products and sums keep fp32-level accuracy, inside the 1e-4
// contract of the reference's fp32 matMul (src/ops/matmul_cpu.cpp:49-60, ops.hpp:354-459), at
// tensor-core rates.
//
// A pre-pass splits A [M,K] (row-major, as the reference) into hi/lo planes and B [K,N] into
// hi/lo planes of B^T [N,K], so both operands are K-major in shared memory.  The GEMM is
// persistent, one CTA per SM, 192 threads: warp 0 TMA (A planes 128x32, B^T planes 128x32,
// 128-byte swizzle, 3-stage ring of 64 KB), warp 1 one thread issuing tcgen05.mma.kind::tf32
// (M=128, N=128, K=8) three times per K step, warps 2..5 the epilogue.  The matmul runs the
// cluster-pair variant (M=256 per CTA pair, 4-stage ring); the im2col conv the one-CTA kernel.
// Accuracy: the tensor core's fp32 accumulation over thousands of terms drifts by up to ~1e-3
// (it does not round like a sequential fp32 sum), so the MMAs only accumulate 128-deep K chunks,
// each into one of four rotating 128-column TMEM buffers, and the epilogue warps add the chunks
// into per-row fp32 registers with round-to-nearest adds (one row of 128 columns per thread).
// Every mbarrier wait is bounded (common.cuh).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include <mutex>

#include "../../include/lc_b200.h"
#include "common.cuh"
#include "lc_internal.hpp"

namespace lcb {

void* tensor_map_encoder();

namespace {

constexpr int BM = 128, BK = 32, STAGES = 3;
constexpr int CHUNK_KB = 4;   // k-blocks (of 32) per TMEM partial sum: 128-deep K chunks
constexpr int ACC_BUFS = 4;   // TMEM partial-sum buffers of BN (<= 128) columns
constexpr int NUM_THREADS = 192;
constexpr int A_PLANE_BYTES = BM * BK * 4;        // 16 KB
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 16;

struct Tail {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[ACC_BUFS];   // a K chunk's partial sum is in TMEM buffer b
  uint64_t tmem_empty[ACC_BUFS];  // the 4 epilogue warps have folded buffer b into registers
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

// x rounded to the 10-bit tf32 mantissa (nearest, ties away from zero), kept in fp32 layout with the
// 13 low mantissa bits clear: add half a tf32 unit (bit 12) to the magnitude, then truncate.
// Infinities and NaNs pass through.
__device__ __forceinline__ float tf32_round(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & 0xffffe000u;
  return __uint_as_float(u);
}

// Rows of src [rows, k] -> hi/lo planes [rows, kp] (kp >= k, zero padded).
__global__ void tf32_split_rows_pad_kernel(const float* __restrict__ src, float* __restrict__ hi,
                                           float* __restrict__ lo, int rows, int k, int kp) {
  const long long total = static_cast<long long>(rows) * kp;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / kp;
    const int c = static_cast<int>(i - r * kp);
    const float v = c < k ? src[r * k + c] : 0.0f;
    const float h = tf32_round(v);
    hi[i] = h;
    lo[i] = v - h;
  }
}

// im2col of an NCHW input as the K-major B^T planes of the conv GEMM: row j = (image, oh, ow),
// column kk = (c, kh, kw) (the OIHW weight order), zero outside the padded input and for kk >= k.
// A block takes IM2COL_ROWS rows at a time; a shared table maps kk to its input offset (c, dy, dx)
// once, so the inner loop has no division, and consecutive threads store consecutive columns.
constexpr int IM2COL_ROWS = 8;
constexpr int IM2COL_MAX_KP = 8192;
__global__ void __launch_bounds__(256) tf32_im2col_split_kernel(const float* __restrict__ x, float* __restrict__ hi,
                                                                float* __restrict__ lo, int rows, int k, int kp,
                                                                int in_c, int in_h, int in_w, int kh, int kw, int sh,
                                                                int sw, int ph, int pw, int oh, int ow) {
  __shared__ int tab[IM2COL_MAX_KP];  // (c << 16) | (dy << 8) | dx, or -1 for padding columns
  for (int kk = threadIdx.x; kk < kp; kk += blockDim.x) {
    if (kk < k) {
      const int c = kk / (kh * kw), r = kk - c * kh * kw, dy = r / kw;
      tab[kk] = (c << 16) | (dy << 8) | (r - dy * kw);
    } else {
      tab[kk] = -1;
    }
  }
  __syncthreads();
  const int pix = oh * ow;
  for (int j0 = blockIdx.x * IM2COL_ROWS; j0 < rows; j0 += gridDim.x * IM2COL_ROWS) {
    // Per row of the group: its image base and top-left input coordinate (rows past the end get
    // an empty window, so every load below is skipped for them).
    const float* xr[IM2COL_ROWS];
    int iy0[IM2COL_ROWS], ix0[IM2COL_ROWS];
#pragma unroll
    for (int jr = 0; jr < IM2COL_ROWS; ++jr) {
      const int j = min(j0 + jr, rows - 1);
      const int n = j / pix, pp = j - n * pix;
      const int y = pp / ow, xo = pp - y * ow;
      xr[jr] = x + static_cast<long long>(n) * in_c * in_h * in_w;
      iy0[jr] = j0 + jr < rows ? y * sh - ph : -(1 << 20);
      ix0[jr] = xo * sw - pw;
    }
    // kk outer, rows inner: the group's IM2COL_ROWS loads are independent and in flight together.
    for (int kk = threadIdx.x; kk < kp; kk += blockDim.x) {
      const int t = tab[kk];
      const int c = t >> 16, dy = (t >> 8) & 0xff, dx = t & 0xff;
      float v[IM2COL_ROWS];
#pragma unroll
      for (int jr = 0; jr < IM2COL_ROWS; ++jr) {
        const int iy = iy0[jr] + dy, ix = ix0[jr] + dx;
        v[jr] = (t >= 0 && iy >= 0 && iy < in_h && ix >= 0 && ix < in_w)
                    ? __ldg(xr[jr] + (static_cast<long long>(c) * in_h + iy) * in_w + ix)
                    : 0.0f;
      }
#pragma unroll
      for (int jr = 0; jr < IM2COL_ROWS; ++jr) {
        if (j0 + jr < rows) {
          const float h = tf32_round(v[jr]);
          hi[static_cast<long long>(j0 + jr) * kp + kk] = h;
          lo[static_cast<long long>(j0 + jr) * kp + kk] = v[jr] - h;
        }
      }
    }
  }
}

// The matmul's pre-pass in one launch: blocks [0, a_blocks) split A [M,K] into hi/lo planes
// (grid-stride over float4s), the rest split B [K,N] into the hi/lo planes of B^T [N,K] by 32x32
// tiles through shared memory; block 0 also zeroes the split-K counters of the GEMM that follows.
__global__ void __launch_bounds__(256) tf32_matmul_prep_kernel(const float4* __restrict__ a, float4* __restrict__ a_hi,
                                                               float4* __restrict__ a_lo, size_t na4, int a_blocks,
                                                               const float* __restrict__ b, float* __restrict__ bh_t,
                                                               float* __restrict__ bl_t, int K, int N, int bt_x,
                                                               unsigned* __restrict__ counters, int n_counters) {
  __shared__ float tile[32][33];
  griddep_launch_dependents();  // the GEMM may take its SMs now; it waits for these planes itself
  const int bid = static_cast<int>(blockIdx.x);
  if (bid == 0)
    for (int i = threadIdx.x; i < n_counters; i += blockDim.x) counters[i] = 0u;
  if (bid < a_blocks) {
    for (size_t i = static_cast<size_t>(bid) * 256 + threadIdx.x; i < na4; i += static_cast<size_t>(a_blocks) * 256) {
      const float4 v = a[i];
      float4 h;
      h.x = tf32_round(v.x);
      h.y = tf32_round(v.y);
      h.z = tf32_round(v.z);
      h.w = tf32_round(v.w);
      a_hi[i] = h;
      a_lo[i] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
    }
    return;
  }
  const int bt = bid - a_blocks;
  const int k0 = (bt / bt_x) * 32, n0 = (bt % bt_x) * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int r = ty; r < 32; r += 8) {
    const int k = k0 + r, n = n0 + tx;
    tile[r][tx] = (k < K && n < N) ? b[static_cast<size_t>(k) * N + n] : 0.0f;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const int n = n0 + r, k = k0 + tx;
    if (n < N && k < K) {
      const float v = tile[tx][r];
      const float h = tf32_round(v);
      bh_t[static_cast<size_t>(n) * K + k] = h;
      bl_t[static_cast<size_t>(n) * K + k] = v - h;
    }
  }
}

// Warp-uniform bounded wait (lane 0 polls, the verdict is broadcast) so the warp stays converged
// for the .sync.aligned TMEM loads that follow.
__device__ __forceinline__ bool warp_wait_gemm(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                               unsigned* err) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait_bounded(bar, parity, abort_flag, err, kErrGemmEpilogueWait) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& mb, int& nb) {
  const int group = GROUP_M * tiles_n;
  const int g = t / group;
  const int first_m = g * GROUP_M;
  const int gm = min(GROUP_M, tiles_m - first_m);
  const int r = t - g * group;
  mb = first_m + r % gm;
  nb = r / gm;
}

// BN_T: output columns per tile (128, or 64 when 128-wide tiles would leave SMs idle).
template <int BN_T>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap map_ahi, const __grid_constant__ CUtensorMap map_alo,
                       const __grid_constant__ CUtensorMap map_bhi, const __grid_constant__ CUtensorMap map_blo,
                       float* __restrict__ C, int M, int N, int K, int period, long long batch_stride,
                       long long row_stride, const float* __restrict__ row_bias, int relu, unsigned* err_word) {
  constexpr int BN = BN_T;
  constexpr int B_PLANE_BYTES = BN * BK * 4;
  constexpr int STAGE_BYTES = 2 * A_PLANE_BYTES + 2 * B_PLANE_BYTES;
  constexpr uint32_t IDESC = idesc_tf32_f32(BM, BN, /*a_mn_major=*/0, /*b_mn_major=*/0);
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // Stage layout: A_hi | A_lo | B_hi | B_lo.
  Tail* st = reinterpret_cast<Tail*>(smem + STAGES * STAGE_BYTES);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = (M + BM - 1) / BM;
  const int tiles_n = (N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&st->full[s], 1);
      mbar_init(&st->empty[s], 1);
    }
    for (int b = 0; b < ACC_BUFS; ++b) {
      mbar_init(&st->tmem_full[b], 1);
      mbar_init(&st->tmem_empty[b], 4);
    }
    mbar_init(&st->drain, 1);
    st->abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&map_ahi);
    tma_prefetch_desc(&map_alo);
    tma_prefetch_desc(&map_bhi);
    tma_prefetch_desc(&map_blo);
  }
  if (warp == 0) {
    tmem_alloc(&st->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = st->tmem_base;
  volatile int* abort_flag = &st->abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, tiles_m, tiles_n, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          // empty[stage] next completes for this stage's next use, which needs the loads below.
          if (!mbar_wait_bounded(&st->empty[stage], phase ^ 1u, abort_flag, err_word, kErrGemmProducerWait)) {
            ok = false;
            break;
          }
          uint8_t* base = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&st->full[stage], STAGE_BYTES);
          tma_load_2d(base, &map_ahi, kb * BK, mb * BM, &st->full[stage]);
          tma_load_2d(base + A_PLANE_BYTES, &map_alo, kb * BK, mb * BM, &st->full[stage]);
          tma_load_2d(base + 2 * A_PLANE_BYTES, &map_bhi, kb * BK, nb * BN, &st->full[stage]);
          tma_load_2d(base + 2 * A_PLANE_BYTES + B_PLANE_BYTES, &map_blo, kb * BK, nb * BN, &st->full[stage]);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA's shared memory goes away.
        for (int u = issued > STAGES ? issued - STAGES : 0; u < issued; ++u) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&st->full[u % STAGES], (u / STAGES) & 1) && globaltimer_ns() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The whole warp runs the loop (waits polled by every lane), one elected lane issues each MMA,
    // descriptors are advanced by constant adds: next to busy epilogue warps a loop run by lane 0
    // alone issues several times slower.
    {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true, issued = false;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        uint32_t d_tmem = tmem_base;
        for (int kb = 0; kb < num_kb; ++kb) {
          const int kc = kb % CHUNK_KB;
          if (kc == 0) {
            // Buffer acc was last committed ACC_BUFS chunks ago; tmem_empty[acc] next completes
            // only after the commit that follows this wait.
            if (!warp_wait_poll(&st->tmem_empty[acc], acc_phase ^ 1u, abort_flag, err_word, kErrGemmMmaWait)) {
              ok = false;
              break;
            }
            tc_fence_after();
            d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
          }
          // full[stage] next completes for the stage's next use, loaded only after the commit below.
          if (!warp_wait_poll(&st->full[stage], phase, abort_flag, err_word, kErrGemmMmaWait)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_hi = smem_u32(smem + stage * STAGE_BYTES);
          const uint64_t ahd0 = smem_desc_sw128(a_hi, 16, 1024);
          const uint64_t ald0 = smem_desc_sw128(a_hi + A_PLANE_BYTES, 16, 1024);
          const uint64_t bhd0 = smem_desc_sw128(a_hi + 2 * A_PLANE_BYTES, 16, 1024);
          const uint64_t bld0 = smem_desc_sw128(a_hi + 2 * A_PLANE_BYTES + B_PLANE_BYTES, 16, 1024);
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            // A and B^T: K-major SW128, rows 128 B apart, 8-row groups 1 KB apart; +32 B per K=8
            // step (+2 in the descriptor's address field, bytes / 16).
            const uint32_t first = (kc > 0 || k > 0) ? 1u : 0u;
            umma_tf32_ss_w(d_tmem, ald0 + k * 2, bhd0 + k * 2, IDESC, first);  // small terms first
            umma_tf32_ss_w(d_tmem, ahd0 + k * 2, bld0 + k * 2, IDESC, 1u);
            umma_tf32_ss_w(d_tmem, ahd0 + k * 2, bhd0 + k * 2, IDESC, 1u);
            issued = true;
          }
          umma_commit_w(&st->empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          if (kc == CHUNK_KB - 1 || kb == num_kb - 1) {
            umma_commit_w(&st->tmem_full[acc]);
            if (++acc == ACC_BUFS) {
              acc = 0;
              acc_phase ^= 1u;
            }
          }
        }
      }
      if (!ok && issued) {
        umma_commit_w(&st->drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&st->drain, 0) && globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5): chunk sums -> fp32 rows ----------------
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    // Vector stores need every segment start 16-byte aligned.
    const bool vec_ok = (period % 4) == 0 && (row_stride % 4) == 0 && (batch_stride % 4) == 0 &&
                        (reinterpret_cast<uintptr_t>(C) & 15u) == 0;
    const int chunks = (num_kb + CHUNK_KB - 1) / CHUNK_KB;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      int mb, nb;
      tile_coords(t, tiles_m, tiles_n, mb, nb);
      float sum[BN];
#pragma unroll
      for (int j = 0; j < BN; ++j) sum[j] = 0.0f;
      for (int ch = 0; ch < chunks; ++ch) {
        // tmem_full[acc] next completes after this warp releases the buffer (below).
        if (!warp_wait_gemm(&st->tmem_full[acc], acc_phase, abort_flag, err_word)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tbase =
            tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tbase + c0, r);
#pragma unroll
          for (int j = 0; j < 32; ++j) sum[c0 + j] = __fadd_rn(sum[c0 + j], __uint_as_float(r[j]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&st->tmem_empty[acc]);
        if (++acc == ACC_BUFS) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) break;
      // Element (row, col) goes to C + (col / period) * batch_stride + row * row_stride + col % period:
      // a plain row-major C (period = N), or NCHW conv output (period = OH*OW pixels of an image).
      const int row = mb * BM + row_in_tile;
      if (row < M) {
        const float bias = row_bias ? __ldg(row_bias + row) : 0.0f;
        if (row_bias || relu) {
#pragma unroll
          for (int j = 0; j < BN; ++j) {
            float v = sum[j] + bias;
            sum[j] = relu ? fmaxf(v, 0.0f) : v;
          }
        }
        const int col0 = nb * BN;
        const int img = col0 / period, pix = col0 - img * period;
        float* dst = C + static_cast<long long>(img) * batch_stride + static_cast<long long>(row) * row_stride + pix;
        if (vec_ok && col0 + BN <= N && pix + BN <= period) {
#pragma unroll
          for (int q = 0; q < BN / 4; ++q)
            reinterpret_cast<float4*>(dst)[q] = make_float4(sum[4 * q], sum[4 * q + 1], sum[4 * q + 2], sum[4 * q + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < BN; ++j) {
            const int col = col0 + j;
            if (col < N) {
              const int im = col / period;
              C[static_cast<long long>(im) * batch_stride + static_cast<long long>(row) * row_stride +
                (col - im * period)] = sum[j];
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---- cluster-pair variant ---------------------------------------------------------------------
// Two CTAs (two SMs) compute a 256 x BN tile with tcgen05.mma.cta_group::2.kind::tf32 (M = 256,
// N = BN, K = 8): each CTA stages its own 128 rows of the A planes and half of the B^T rows; the
// leader issues every MMA, its commits release the stage in both CTAs and hand each CTA its
// accumulator lanes chunk by chunk; each CTA's epilogue folds its rows' chunks into fp32 registers
// exactly as the one-CTA kernel does.
//
// Split K: a work item is (tile, split) with `kb_per` k-blocks per split.  With ksplit > 1 every
// epilogue warp writes its 32 rows x COLS partial sums to an L2 workspace and bumps its own
// counter; the warp that brings the counter to ksplit adds the partials (two splits: its own
// registers plus the other one, which is order-free; more: all of them in split order), so the
// bits never depend on which split finished last.  The counters are zeroed by the pre-pass of the
// same call.
namespace pairg {
template <int BN>
struct Cfg {
  static_assert(BN == 64 || BN == 128, "pair tile width");
  static constexpr int EPI_WARPS = 4;              // one per TMEM lane quarter
  static constexpr int COLS = BN * 4 / EPI_WARPS;  // columns per epilogue warp (the whole tile row)
  static constexpr int STAGES = 4;
  static constexpr int ACC = 4;                    // TMEM chunk buffers of BN columns
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int STAGE_BYTES = 2 * A_PLANE_BYTES + 2 * (BN / 2) * BK * 4;
};
struct Tail {
  uint64_t full[4];          // leader: both CTAs' bytes of the stage landed
  uint64_t empty[4];         // per CTA: the leader's MMAs reading this stage finished
  uint64_t tmem_full[4];     // per CTA: its lanes of a K chunk's partial sum are in buffer b
  uint64_t tmem_empty[4];    // leader: the epilogue warps of both CTAs folded buffer b
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
template <int BN>
constexpr size_t smem_bytes() {
  return 1024 + Cfg<BN>::STAGES * Cfg<BN>::STAGE_BYTES + sizeof(Tail);
}
}  // namespace pairg

template <int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pairg::Cfg<BN>::THREADS, 1)
    gemm_tf32x3_pair_kernel(const __grid_constant__ CUtensorMap map_ahi, const __grid_constant__ CUtensorMap map_alo,
                            const __grid_constant__ CUtensorMap map_bhi, const __grid_constant__ CUtensorMap map_blo,
                            float* __restrict__ C, int M, int N, int K, int period, long long batch_stride,
                            long long row_stride, const float* __restrict__ row_bias, int relu, int ksplit,
                            int kb_per, float* __restrict__ part, unsigned* __restrict__ counters,
                            unsigned* err_word) {
  using pairg::Tail;
  using CF = pairg::Cfg<BN>;
  constexpr int STAGES = CF::STAGES;
  constexpr int ACC = CF::ACC;
  constexpr int COLS = CF::COLS;
  constexpr int B_HALF_PLANE = (BN / 2) * BK * 4;
  constexpr int STAGE_BYTES = CF::STAGE_BYTES;  // A_hi | A_lo | B_hi | B_lo (this CTA's half)
  constexpr uint32_t IDESC = idesc_tf32_f32(2 * BM, BN, 0, 0);
  static_assert(ACC * BN <= TMEM_COLS, "TMEM chunk buffers");
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Tail* st = reinterpret_cast<Tail*>(smem + STAGES * STAGE_BYTES);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster_id = static_cast<int>(blockIdx.x) >> 1;
  const int num_clusters = static_cast<int>(gridDim.x) >> 1;
  const int tiles_m = (M + 2 * BM - 1) / (2 * BM);
  const int tiles_n = (N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = (K + BK - 1) / BK;
  const int num_items = num_tiles * ksplit;
  auto item_range = [&](int w, int& t, int& sp, int& kb0, int& kb1) {
    t = w / ksplit;
    sp = w - t * ksplit;
    kb0 = sp * kb_per;
    kb1 = min(num_kb, kb0 + kb_per);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&st->full[s], 1);
      mbar_init(&st->empty[s], 1);
    }
    for (int b = 0; b < ACC; ++b) {
      mbar_init(&st->tmem_full[b], 1);
      mbar_init(&st->tmem_empty[b], 2 * CF::EPI_WARPS);
    }
    mbar_init(&st->drain, 1);
    st->abort_flag = 0;
    fence_barrier_init_cluster();
    tma_prefetch_desc(&map_ahi);
    tma_prefetch_desc(&map_alo);
    tma_prefetch_desc(&map_bhi);
    tma_prefetch_desc(&map_blo);
  }
  if (warp == 0) {
    tmem_alloc_pair(&st->tmem_base, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barrier inits and the TMEM allocation visible to both CTAs
  tc_fence_after();
  griddep_wait();  // the split planes and counters come from the pre-pass
  const uint32_t tmem_base = st->tmem_base;
  volatile int* abort_flag = &st->abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int w = cluster_id; w < num_items && ok; w += num_clusters) {
        int t, sp, kb0, kb1, mb, nb;
        item_range(w, t, sp, kb0, kb1);
        tile_coords(t, tiles_m, tiles_n, mb, nb);
        const int row0 = mb * 2 * BM + static_cast<int>(rank) * BM;
        const int col0 = nb * BN + static_cast<int>(rank) * (BN / 2);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&st->empty[stage], phase ^ 1u, abort_flag, err_word, kErrGemmProducerWait)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&st->full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&st->full[stage], 2 * STAGE_BYTES);
          uint8_t* base = smem + stage * STAGE_BYTES;
          tma_load_2d_pair(base, &map_ahi, kb * BK, row0, full_leader);
          tma_load_2d_pair(base + A_PLANE_BYTES, &map_alo, kb * BK, row0, full_leader);
          tma_load_2d_pair(base + 2 * A_PLANE_BYTES, &map_bhi, kb * BK, col0, full_leader);
          tma_load_2d_pair(base + 2 * A_PLANE_BYTES + B_HALF_PLANE, &map_blo, kb * BK, col0, full_leader);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Tail: the leader's last commits on this CTA's empty barriers must land before exit.
      for (int u = issued > STAGES ? issued - STAGES : 0; u < issued; ++u) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&st->empty[u % STAGES], (u / STAGES) & 1) && !*abort_flag &&
               globaltimer_ns() - t0 < 200000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only) ----------------
    if (leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true, issued = false;
      for (int w = cluster_id; w < num_items && ok; w += num_clusters) {
        int t, sp, kb0, kb1;
        item_range(w, t, sp, kb0, kb1);
        uint32_t d_tmem = tmem_base;
        for (int kb = kb0; kb < kb1; ++kb) {
          const int kc = (kb - kb0) % CHUNK_KB;
          if (kc == 0) {
            if (!warp_wait_poll(&st->tmem_empty[acc], acc_phase ^ 1u, abort_flag, err_word, kErrGemmMmaWait)) {
              ok = false;
              break;
            }
            tc_fence_after();
            d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
          }
          if (!warp_wait_poll(&st->full[stage], phase, abort_flag, err_word, kErrGemmMmaWait)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_hi = smem_u32(smem + stage * STAGE_BYTES);
          const uint64_t ahd0 = smem_desc_sw128(a_hi, 16, 1024);
          const uint64_t ald0 = smem_desc_sw128(a_hi + A_PLANE_BYTES, 16, 1024);
          const uint64_t bhd0 = smem_desc_sw128(a_hi + 2 * A_PLANE_BYTES, 16, 1024);
          const uint64_t bld0 = smem_desc_sw128(a_hi + 2 * A_PLANE_BYTES + B_HALF_PLANE, 16, 1024);
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            const uint32_t first = (kc > 0 || k > 0) ? 1u : 0u;
            umma_tf32_ss_pair_w(d_tmem, ald0 + k * 2, bhd0 + k * 2, IDESC, first);  // small terms first
            umma_tf32_ss_pair_w(d_tmem, ahd0 + k * 2, bld0 + k * 2, IDESC, 1u);
            umma_tf32_ss_pair_w(d_tmem, ahd0 + k * 2, bhd0 + k * 2, IDESC, 1u);
            issued = true;
          }
          umma_commit_pair_w(&st->empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          if (kc == CHUNK_KB - 1 || kb == kb1 - 1) {
            umma_commit_pair_w(&st->tmem_full[acc], 0x3);
            if (++acc == ACC) {
              acc = 0;
              acc_phase ^= 1u;
            }
          }
        }
      }
      if (!ok && issued) {
        umma_commit_pair_w(&st->drain, 0x1);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&st->drain, 0) && globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2.. of both CTAs): chunk sums -> fp32 rows ----------------
    const int quarter = warp & 3;                  // TMEM lane quarter this warp may read
    const int ew = warp - 2;                       // epilogue warp index
    const int cbase = (ew >> 2) * COLS;            // this warp's first column of the tile
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    const bool vec_ok = (period % 4) == 0 && (row_stride % 4) == 0 && (batch_stride % 4) == 0 &&
                        (reinterpret_cast<uintptr_t>(C) & 15u) == 0;
    bool ok = true;
    for (int w = cluster_id; w < num_items && ok; w += num_clusters) {
      int t, sp, kb0, kb1, mb, nb;
      item_range(w, t, sp, kb0, kb1);
      tile_coords(t, tiles_m, tiles_n, mb, nb);
      const int chunks = (kb1 - kb0 + CHUNK_KB - 1) / CHUNK_KB;
      float sum[COLS];
#pragma unroll
      for (int j = 0; j < COLS; ++j) sum[j] = 0.0f;
      for (int ch = 0; ch < chunks; ++ch) {
        if (!warp_wait_gemm(&st->tmem_full[acc], acc_phase, abort_flag, err_word)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tbase = tmem_base + static_cast<uint32_t>(acc * BN + cbase) +
                               (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll
        for (int c0 = 0; c0 < COLS; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tbase + c0, r);
#pragma unroll
          for (int j = 0; j < 32; ++j) sum[c0 + j] = __fadd_rn(sum[c0 + j], __uint_as_float(r[j]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&st->tmem_empty[acc]), 0));
        if (++acc == ACC) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) break;
      if (ksplit > 1) {
        // This warp's partial block: [tile][split][rank][epilogue warp] of COLS/4 x 32 float4s
        // (quad q of lane l at q * 32 + l: every store and load of the warp is 512 contiguous bytes).
        const long long wblk = (static_cast<long long>(t) * 2 + rank) * CF::EPI_WARPS + ew;
        const long long span4 = static_cast<long long>(num_tiles) * 2 * CF::EPI_WARPS * (COLS / 4) * 32;
        float4* blk = reinterpret_cast<float4*>(part) + wblk * (COLS / 4) * 32 + lane;
#pragma unroll
        for (int q = 0; q < COLS / 4; ++q)
          __stcg(blk + sp * span4 + q * 32, make_float4(sum[4 * q], sum[4 * q + 1], sum[4 * q + 2], sum[4 * q + 3]));
        __threadfence();
        __syncwarp();
        unsigned prev = 0;
        if (lane == 0) prev = atomicAdd(counters + wblk, 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev != static_cast<unsigned>(ksplit - 1)) continue;  // another split finishes this block
        __threadfence();
        // Last split of this block.  Two splits: own + other (a + b == b + a, so the bits do not
        // depend on which split came last).  More: every partial from L2 in split order.  16
        // float4 loads are in flight per lane at a time.
        if (ksplit == 2) {
          const float4* other = blk + (1 - sp) * span4;
#pragma unroll
          for (int h = 0; h < COLS / 64; ++h) {
            float4 v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __ldcg(other + (h * 16 + i) * 32);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float* sj = sum + (h * 16 + i) * 4;
              sj[0] = __fadd_rn(sj[0], v[i].x);
              sj[1] = __fadd_rn(sj[1], v[i].y);
              sj[2] = __fadd_rn(sj[2], v[i].z);
              sj[3] = __fadd_rn(sj[3], v[i].w);
            }
          }
        } else {
#pragma unroll
          for (int h = 0; h < COLS / 64; ++h) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float4 v = __ldcg(blk + (h * 16 + i) * 32);
              float* sj = sum + (h * 16 + i) * 4;
              sj[0] = v.x, sj[1] = v.y, sj[2] = v.z, sj[3] = v.w;
            }
            for (int q = 1; q < ksplit; ++q) {
              float4 v[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) v[i] = __ldcg(blk + q * span4 + (h * 16 + i) * 32);
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                float* sj = sum + (h * 16 + i) * 4;
                sj[0] = __fadd_rn(sj[0], v[i].x);
                sj[1] = __fadd_rn(sj[1], v[i].y);
                sj[2] = __fadd_rn(sj[2], v[i].z);
                sj[3] = __fadd_rn(sj[3], v[i].w);
              }
            }
          }
        }
      }
      const int row = mb * 2 * BM + static_cast<int>(rank) * BM + row_in_tile;
      if (row < M) {
        const float bias = row_bias ? __ldg(row_bias + row) : 0.0f;
        if (row_bias || relu) {
#pragma unroll
          for (int j = 0; j < COLS; ++j) {
            float v = sum[j] + bias;
            sum[j] = relu ? fmaxf(v, 0.0f) : v;
          }
        }
        const int col0 = nb * BN + cbase;
        const int img = col0 / period, pix = col0 - img * period;
        float* dst = C + static_cast<long long>(img) * batch_stride + static_cast<long long>(row) * row_stride + pix;
        if (vec_ok && col0 + COLS <= N && pix + COLS <= period) {
#pragma unroll
          for (int q = 0; q < COLS / 4; ++q)
            reinterpret_cast<float4*>(dst)[q] = make_float4(sum[4 * q], sum[4 * q + 1], sum[4 * q + 2], sum[4 * q + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < COLS; ++j) {
            const int col = col0 + j;
            if (col < N) {
              const int im = col / period;
              C[static_cast<long long>(im) * batch_stride + static_cast<long long>(row) * row_stride +
                (col - im * period)] = sum[j];
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while the pair's MMAs, commits or arrivals can touch it
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// 2-D fp32 tensor map over row-major [rows, cols], box [box_rows, box_cols], 128-byte swizzle.
bool make_tmap_f32_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                      uint32_t box_cols) {
  auto enc = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 4};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool gemm_f32_tc_supported(const void* a, const void* b, const void* c, int m, int k, int n) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return m > 0 && k > 0 && n > 0 && (k % 4) == 0 && (n % 4) == 0 && al(a) && al(b) && al(c) &&
         tensor_map_encoder() != nullptr;
}

namespace {

struct Epi {
  float* c;
  int period;
  long long batch_stride, row_stride;
  const float* row_bias;
  int relu;
};

size_t smem_bytes_for(int bn) { return 1024 + STAGES * (2 * A_PLANE_BYTES + 2 * bn * BK * 4) + sizeof(Tail); }

// The GEMM on prepared planes A [m, kp] and B^T [n, kp] (hi and lo of each), with bn-column tiles
// (128, or 64 when 128-wide tiles would leave SMs idle: 1024^3 has 64 tiles of 128x128 for 148 SMs).
// The GEMM on prepared planes A [m, kp] and B^T [n, kp] (hi and lo of each) with the one-CTA
// kernel, bn-column tiles (128, or 64 when 128-wide tiles would leave SMs idle).
cudaError_t launch_planes(DeviceCtx* ctx, const float* a_hi, const float* a_lo, const float* b_hi, const float* b_lo,
                          int m, int n, int kp, const Epi& epi, cudaStream_t s, int bn = 128) {
  CUtensorMap mah, mal, mbh, mbl;
  if (!make_tmap_f32_2d(&mah, a_hi, m, kp, BM, BK) || !make_tmap_f32_2d(&mal, a_lo, m, kp, BM, BK) ||
      !make_tmap_f32_2d(&mbh, b_hi, n, kp, bn, BK) || !make_tmap_f32_2d(&mbl, b_lo, n, kp, bn, BK))
    return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> attr_done{0};  // devices with the attributes set
  {
    const cudaError_t ea = once_per_device(attr_done, [&]() -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(gemm_tf32x3_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem_bytes_for(128)));
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemm_tf32x3_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem_bytes_for(64)));
      if (e != cudaSuccess) return e;
      return cudaSuccess;
    });
    if (ea != cudaSuccess) return ea;
  }
  const int tiles = ((m + BM - 1) / BM) * ((n + bn - 1) / bn);
  const int grid = tiles < ctx->sm_count ? tiles : ctx->sm_count;
  if (bn == 64)
    gemm_tf32x3_kernel<64><<<grid, NUM_THREADS, smem_bytes_for(64), s>>>(
        mah, mal, mbh, mbl, epi.c, m, n, kp, epi.period, epi.batch_stride, epi.row_stride, epi.row_bias, epi.relu,
        ctx->err_word);
  else
    gemm_tf32x3_kernel<128><<<grid, NUM_THREADS, smem_bytes_for(128), s>>>(
        mah, mal, mbh, mbl, epi.c, m, n, kp, epi.period, epi.batch_stride, epi.row_stride, epi.row_bias, epi.relu,
        ctx->err_word);
  return cudaGetLastError();
}

// Work plan of the cluster-pair matmul: tile width, K splits and k-blocks per split.
struct PairPlan {
  int bn, ksplit, kb_per, tiles;
  size_t part_floats, counters;
};

PairPlan plan_pair(const DeviceCtx* ctx, int m, int n, int k, int bn) {
  PairPlan pl{};
  pl.bn = bn;
  const int clusters = ctx->sm_count / 2;
  const int num_kb = (k + BK - 1) / BK;
  pl.tiles = ((m + 2 * BM - 1) / (2 * BM)) * ((n + bn - 1) / bn);
  int ks = 1;
  // Fewer tiles than half the SM pairs: split K so the pairs fill up, keeping at least one
  // 128-deep chunk per split.
  if (pl.tiles * 2 <= clusters) ks = std::max(1, std::min(clusters / pl.tiles, num_kb / CHUNK_KB));
  pl.kb_per = (num_kb + ks - 1) / ks;
  pl.ksplit = (num_kb + pl.kb_per - 1) / pl.kb_per;  // every split non-empty
  const int epi_warps = pairg::Cfg<128>::EPI_WARPS;
  pl.part_floats = pl.ksplit > 1 ? static_cast<size_t>(pl.ksplit) * pl.tiles * 2 * BM * bn : 0;
  pl.counters = static_cast<size_t>(pl.tiles) * 2 * epi_warps;
  return pl;
}

template <int BN>
cudaError_t launch_pair_bn(const CUtensorMap& mah, const CUtensorMap& mal, const CUtensorMap& pbh,
                           const CUtensorMap& pbl, int m, int n, int kp, const Epi& epi, const PairPlan& pl,
                           float* part, unsigned* counters, unsigned* err_word, int clusters_max, cudaStream_t s) {
  static std::atomic<unsigned long long> attr_done{0};  // devices with the attributes set
  {
    const cudaError_t ea = once_per_device(attr_done, [&]() -> cudaError_t {
      const cudaError_t e = cudaFuncSetAttribute(gemm_tf32x3_pair_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(pairg::smem_bytes<BN>()));
      if (e != cudaSuccess) return e;
      return cudaSuccess;
    });
    if (ea != cudaSuccess) return ea;
  }
  const int items = pl.tiles * pl.ksplit;
  const int clusters = items < clusters_max ? items : clusters_max;
  return launch_pdl(gemm_tf32x3_pair_kernel<BN>, dim3(2 * clusters), dim3(pairg::Cfg<BN>::THREADS),
                    pairg::smem_bytes<BN>(), s, mah, mal, pbh, pbl, epi.c, m, n, kp, epi.period, epi.batch_stride,
                    epi.row_stride, epi.row_bias, epi.relu, pl.ksplit, pl.kb_per, part, counters, err_word);
}

// The matmul on prepared planes with CTA pairs (256-row tiles), per `pl`.
cudaError_t launch_pair(DeviceCtx* ctx, const float* a_hi, const float* a_lo, const float* b_hi, const float* b_lo,
                        int m, int n, int kp, const Epi& epi, const PairPlan& pl, float* part, unsigned* counters,
                        cudaStream_t s) {
  CUtensorMap mah, mal, pbh, pbl;  // B^T boxes of bn/2 rows: each CTA stages half of the tile's columns
  if (!make_tmap_f32_2d(&mah, a_hi, m, kp, BM, BK) || !make_tmap_f32_2d(&mal, a_lo, m, kp, BM, BK) ||
      !make_tmap_f32_2d(&pbh, b_hi, n, kp, pl.bn / 2, BK) || !make_tmap_f32_2d(&pbl, b_lo, n, kp, pl.bn / 2, BK))
    return cudaErrorInvalidValue;
  const int cmax = ctx->sm_count / 2;
  switch (pl.bn) {
    case 64:
      return launch_pair_bn<64>(mah, mal, pbh, pbl, m, n, kp, epi, pl, part, counters, ctx->err_word, cmax, s);
    default:
      return launch_pair_bn<128>(mah, mal, pbh, pbl, m, n, kp, epi, pl, part, counters, ctx->err_word, cmax, s);
  }
}

int grid_for(long long n) { return static_cast<int>(n / 256 + 1 < 148 * 8 ? n / 256 + 1 : 148 * 8); }

}  // namespace

cudaError_t gemm_f32_3xtf32(const float* a, const float* b, float* c, int m, int k, int n, cudaStream_t s) {
  DeviceCtx* ctx = device_ctx();
  if (!ctx) return cudaErrorNoDevice;
  if (ctx->sm_count < 2) return cudaErrorNotSupported;
  const size_t na = static_cast<size_t>(m) * k, nb = static_cast<size_t>(k) * n;
  // CTA pairs with 256x128 tiles; 256x64 when the wider tiles fill between a quarter and a half
  // of the SM pairs; with fewer tiles K is split across pairs (plan_pair).  Measured: 1024^3
  // 0.034 -> 0.029 ms (one-launch pre-pass, 256x128 tiles in two K splits), 2048^3 0.097 ms;
  // 256x256 tiles (eight epilogue warps, three stages) were slower at every size tried.
  const long long wide_tiles = static_cast<long long>((m + 2 * BM - 1) / (2 * BM)) * ((n + 127) / 128);
  const int bn = (wide_tiles < ctx->sm_count / 2 && wide_tiles * 4 > ctx->sm_count) ? 64 : 128;
  const PairPlan pl = plan_pair(ctx, m, n, k, bn);
  // Stream-ordered workspace: the split planes, the split-K partial sums and the counters.
  const size_t planes = 2 * (na + nb);
  float* ws = nullptr;
  cudaError_t e = workspace_alloc(ctx, reinterpret_cast<void**>(&ws),
                                  (planes + pl.part_floats + pl.counters) * sizeof(float), s);
  if (e != cudaSuccess) return e;
  float* a_hi = ws;
  float* a_lo = a_hi + na;
  float* b_hi = a_lo + na;
  float* b_lo = b_hi + nb;
  float* part = ws + planes;
  unsigned* counters = reinterpret_cast<unsigned*>(part + pl.part_floats);
  const int a_blocks = static_cast<int>(std::min<size_t>((na / 4 + 255) / 256, 1184));
  const int bt_x = (n + 31) / 32, bt_y = (k + 31) / 32;
  tf32_matmul_prep_kernel<<<a_blocks + bt_x * bt_y, 256, 0, s>>>(
      reinterpret_cast<const float4*>(a), reinterpret_cast<float4*>(a_hi), reinterpret_cast<float4*>(a_lo), na / 4,
      a_blocks, b, b_hi, b_lo, k, n, bt_x, counters, static_cast<int>(pl.counters));
  if ((e = cudaGetLastError()) == cudaSuccess)
    e = launch_pair(ctx, a_hi, a_lo, b_hi, b_lo, m, n, k, Epi{c, n, 0, n, nullptr, 0}, pl, part, counters, s);
  const cudaError_t ef = workspace_free(ws, s);
  return e != cudaSuccess ? e : ef;
}

// Conv as out_n[oc, p] = sum_kk W[oc, kk] col_n[kk, p] for all images at once: A = W [OC, C*kh*kw]
// (OIHW as is), B^T = the im2col rows [images*OH*OW, C*kh*kw]; the epilogue writes NCHW with
// bias and ReLU.  The reduction dimension is zero-padded to a multiple of 4 (TMA row pitch).
cudaError_t conv2d_nchw_f32_3xtf32(const float* x, const float* w, const float* bias, float* out, int batch, int in_c,
                                   int in_h, int in_w, int out_c, int kh, int kw, int sh, int sw, int ph, int pw,
                                   int relu, cudaStream_t s) {
  DeviceCtx* ctx = device_ctx();
  if (!ctx) return cudaErrorNoDevice;
  const int oh = (in_h + 2 * ph - kh) / sh + 1, ow = (in_w + 2 * pw - kw) / sw + 1;
  const int k = in_c * kh * kw, kp = (k + 3) & ~3;
  const long long rows = static_cast<long long>(batch) * oh * ow;
  if (rows > 0x7fffffffLL) return cudaErrorNotSupported;
  const size_t na = static_cast<size_t>(out_c) * kp, nb = static_cast<size_t>(rows) * kp;
  float* ws = nullptr;
  cudaError_t e = workspace_alloc(ctx, reinterpret_cast<void**>(&ws), 2 * (na + nb) * sizeof(float), s);
  if (e != cudaSuccess) return e;
  float* a_hi = ws;
  float* a_lo = a_hi + na;
  float* b_hi = a_lo + na;
  float* b_lo = b_hi + nb;
  tf32_split_rows_pad_kernel<<<grid_for(static_cast<long long>(na)), 256, 0, s>>>(w, a_hi, a_lo, out_c, k, kp);
  {
    const long long blocks = (rows + IM2COL_ROWS - 1) / IM2COL_ROWS;
    tf32_im2col_split_kernel<<<static_cast<unsigned>(blocks < 148 * 32 ? blocks : 148 * 32), 256, 0, s>>>(
        x, b_hi, b_lo, static_cast<int>(rows), k, kp, in_c, in_h, in_w, kh, kw, sh, sw, ph, pw, oh, ow);
  }
  if ((e = cudaGetLastError()) == cudaSuccess) {
    const int pix = oh * ow;
    e = launch_planes(ctx, a_hi, a_lo, b_hi, b_lo, out_c, static_cast<int>(rows), kp,
                      Epi{out, pix, static_cast<long long>(out_c) * pix, pix, bias, relu}, s);
  }
  const cudaError_t ef = workspace_free(ws, s);
  return e != cudaSuccess ? e : ef;
}

bool conv_tc_eligible(int in_c, int kh, int kw, int out_c) {
  const long long kp = (static_cast<long long>(in_c) * kh * kw + 3) & ~3LL;
  return out_c >= 32 && kp <= IM2COL_MAX_KP && kh < 256 && kw < 256 && in_c < 32768 && tensor_map_encoder() != nullptr;
}

bool conv_tune_key(size_t batch, size_t in_c, size_t in_h, size_t in_w, size_t out_c, size_t kh, size_t kw,
                   size_t sh, size_t sw, size_t ph, size_t pw, size_t* d0, size_t* d1, size_t* d2) {
  const size_t w32 = size_t(1) << 32;
  if (batch >= w32 || in_c >= w32 || out_c >= w32 || in_h >= w32 || in_w >= w32 || kh >= 256 || kw >= 256 ||
      sh >= 16 || sw >= 16 || ph >= 16 || pw >= 16)
    return false;
  *d0 = (in_c << 32) | out_c;
  *d1 = (in_h << 32) | in_w;
  *d2 = (batch << 32) | (kh << 24) | (kw << 16) | (sh << 12) | (sw << 8) | (ph << 4) | pw;
  return true;
}

// fp32 conv: a cached per-shape choice (lcConvAutotune / lcTuneCacheSet under LC_TUNE_CONV) when
// there is one; otherwise the implicit-GEMM tensor-core kernel for shapes it takes (>= 2^26
// multiply-adds), the im2col 3xTF32 GEMM for other large shapes (>= 2^28 multiply-adds, >= 32
// output channels), else the SIMT implicit GEMM.
cudaError_t conv2d_nchw_f32(const float* x, const float* w, const float* bias, float* out, int batch, int in_c,
                            int in_h, int in_w, int out_c, int kh, int kw, int sh, int sw, int ph, int pw, int relu,
                            cudaStream_t s) {
  const bool tc_ok = conv_tc_eligible(in_c, kh, kw, out_c);
  size_t d0, d1, d2;
  std::string cfg;
  if (conv_tune_key(batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, &d0, &d1, &d2) &&
      tune_lookup(LC_TUNE_CONV, d0, d1, d2, LC_DTYPE_F32, &cfg)) {
    if (cfg == kConvImplicitName && conv_implicit_supported(in_c, out_c, kh, kw))
      return conv2d_nchw_f32_implicit(x, w, bias, out, batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, relu, s);
    if (cfg == kConvTcName && tc_ok)
      return conv2d_nchw_f32_3xtf32(x, w, bias, out, batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, relu, s);
    if (cfg == "simt")
      return conv2d_nchw_f32_simt(x, w, bias, out, batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, relu, s);
  }
  const long long oh = (in_h + 2 * ph - kh) / sh + 1, ow = (in_w + 2 * pw - kw) / sw + 1;
  const long long macs = static_cast<long long>(out_c) * batch * oh * ow * in_c * kh * kw;
  if (macs >= (1LL << 26) && conv_implicit_supported(in_c, out_c, kh, kw))
    return conv2d_nchw_f32_implicit(x, w, bias, out, batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, relu, s);
  if (macs >= (1LL << 28) && out_c >= 32 && tc_ok)
    return conv2d_nchw_f32_3xtf32(x, w, bias, out, batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, relu, s);
  return conv2d_nchw_f32_simt(x, w, bias, out, batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, relu, s);
}

}  // namespace lcb
