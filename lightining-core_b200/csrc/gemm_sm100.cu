// bf16 GEMM on the 5th-generation tensor cores: C[M,N] (bf16) = A[M,K] (bf16) * B[K,N] (bf16),
// fp32 accumulation in TMEM.  Replaces the matmul2d hot loop (reference: ops::matMulWithPolicy,
// include/lightning_core/core/ops.hpp:354-459; CPU loop src/ops/matmul_cpu.cpp:49-60) for the
// bf16 configs.  Both operands keep the reference's row-major layout: A is K-major, B is
// N-major ("MN-major" in UMMA terms), so no transpose pass ever runs.
//
// Structure (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: A tile 128x64 (one 16 KB box) + B tile 64x256 (four 8 KB boxes of
//               64 N-columns), 128-byte swizzle, 4-stage mbarrier ring.
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=256, K=16) x 4 per stage,
//               commits the stage back to the producer, and commits a finished accumulator to
//               the epilogue.  Accumulators are double-buffered in TMEM (2 x 256 columns) so
//               the next tile's MMAs overlap the previous tile's epilogue.
//   warps 2..5  epilogue: tcgen05.ld 64 columns at a time (each warp owns the TMEM lane
//               quarter warp%4), convert to bf16 into a 128-byte-swizzled [32 x 64] staging box
//               in shared memory (two per warp), one TMA store per box.  Row-per-lane global
//               stores touched 32 lines per instruction and held the L1 near 75% busy on
//               short-K shapes: [16384, 1024, 4096] 0.100 -> 0.087 ms, 8192^3 0.707 -> 0.697 ms.
// Tiles are walked in groups of 16 M-blocks so the A and B panels in flight stay in L2.
// Every mbarrier wait is bounded (common.cuh); on a timeout the CTA drains and exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/lc_b200.h"
#include "common.cuh"
#include "lc_internal.hpp"

namespace lcb {
namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int NUM_THREADS = 192;
constexpr int A_STAGE_BYTES = BM * BK * 2;          // 16 KB
constexpr int B_CHUNK_BYTES = BK * 64 * 2;          // 8 KB: 64 K-rows x 64 N-cols
constexpr int B_STAGE_BYTES = BK * BN * 2;          // 32 KB
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int TMEM_COLS = 512;                      // 2 accumulators x 256 fp32 columns
constexpr int GROUP_M = 16;
constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN, /*a_mn_major=*/0, /*b_mn_major=*/1);

struct SharedTail {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
// Epilogue staging: per epilogue warp two [32 rows x 64 columns] bf16 boxes (4 KB each, 128-byte
// swizzle) that its TMA stores read from.
constexpr int C_BOX_BYTES = 32 * 64 * 2;
constexpr int C_STAGE_BYTES = 4 * 2 * C_BOX_BYTES;  // 32 KB
constexpr size_t SMEM_BYTES = 1024 /*align slack*/ + STAGES * STAGE_BYTES + C_STAGE_BYTES + sizeof(SharedTail);

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& mb, int& nb) {
  const int group = GROUP_M * tiles_n;
  const int g = t / group;
  const int first_m = g * GROUP_M;
  const int gm = min(GROUP_M, tiles_m - first_m);
  const int r = t - g * group;
  mb = first_m + r % gm;
  nb = r / gm;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                        const __grid_constant__ CUtensorMap map_c, int M, int N, int K, unsigned* err_word,
                        int stall_kb) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + STAGES * A_STAGE_BYTES;
  uint8_t* smem_c = smem + STAGES * STAGE_BYTES;
  SharedTail* st = reinterpret_cast<SharedTail*>(smem + STAGES * STAGE_BYTES + C_STAGE_BYTES);

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
    for (int b = 0; b < 2; ++b) {
      mbar_init(&st->tmem_full[b], 1);
      mbar_init(&st->tmem_empty[b], 4);
    }
    mbar_init(&st->drain, 1);
    st->abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
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
      int inflight_stage[STAGES];
      uint32_t inflight_phase[STAGES];
      int ninflight = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, tiles_m, tiles_n, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&st->empty[stage], phase ^ 1u, abort_flag, err_word, kErrGemmProducerWait)) {
            ok = false;
            break;
          }
          if (stall_kb == kb && t == 0) {
            // Test hook (lcTestStallNextGemm): CTA 0 never fills this stage, so the MMA warp's
            // bounded wait on it runs out and the CTA takes its abort path.
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          mbar_arrive_expect_tx(&st->full[stage], STAGE_BYTES);
          tma_load_2d(smem_a + stage * A_STAGE_BYTES, &map_a, kb * BK, mb * BM, &st->full[stage]);
          uint8_t* bdst = smem_b + stage * B_STAGE_BYTES;
#pragma unroll
          for (int c = 0; c < BN / 64; ++c)
            tma_load_2d(bdst + c * B_CHUNK_BYTES, &map_b, nb * BN + c * 64, kb * BK, &st->full[stage]);
          inflight_stage[ninflight % STAGES] = stage;
          inflight_phase[ninflight % STAGES] = phase;
          ++ninflight;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Abort path: let the copies already issued land before the CTA's shared memory goes away.
        const int n = ninflight < STAGES ? ninflight : STAGES;
        for (int i = 0; i < n; ++i) {
          const int idx = (ninflight - 1 - i) % STAGES;
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&st->full[inflight_stage[idx]], inflight_phase[idx]) &&
                 globaltimer_ns() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The whole warp runs the loop (waits polled by every lane), one elected lane issues.
    {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued = false;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!warp_wait_poll(&st->tmem_empty[acc], acc_phase ^ 1u, abort_flag, err_word, kErrGemmMmaWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!warp_wait_poll(&st->full[stage], phase, abort_flag, err_word, kErrGemmMmaWait)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // A: K-major SW128, rows 128 B apart, 8-row groups 1024 B apart; +32 B per K=16 step.
          // B: MN-major SW128, 64-column chunks 8 KB apart (LBO), 8-row K groups 1024 B apart
          // (SBO); +16 rows * 128 B per K=16 step.  Steps are added to the address field (bytes / 16).
          const uint64_t ad0 = smem_desc_sw128(smem_u32(smem_a + stage * A_STAGE_BYTES), 16, 1024);
          const uint64_t bd0 = smem_desc_sw128(smem_u32(smem_b + stage * B_STAGE_BYTES), B_CHUNK_BYTES, 1024);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            umma_f16_ss_w(d_tmem, ad0 + k * 2, bd0 + k * 128, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
            issued = true;
          }
          umma_commit_w(&st->empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_w(&st->tmem_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued) {
        // Abort path: wait (bounded) for every MMA already issued before TMEM is released.
        umma_commit_w(&st->drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&st->drain, 0) && globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    // As in the 2-SM kernel: 64-column chunks staged as swizzled bf16 boxes, one TMA store each.
    const int quarter = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    int nbox = 0;
    uint8_t* cbuf = smem_c + quarter * 2 * C_BOX_BYTES;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int mb, nb;
      tile_coords(t, tiles_m, tiles_n, mb, nb);
      if (!mbar_wait_bounded(&st->tmem_full[acc], acc_phase, abort_flag, err_word, kErrGemmEpilogueWait)) break;
      tc_fence_after();
      const int row0 = mb * BM + quarter * 32;
      const uint32_t tbase = tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 64) {
        uint32_t r[64];
        tmem_ld64(tbase + c0, r);
        if (c0 + 64 == BN) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&st->tmem_empty[acc]);
        }
        uint8_t* box = cbuf + (nbox & 1) * C_BOX_BYTES;
        if (lane == 0) bulk_wait_group_read1();
        __syncwarp();
        uint8_t* srow = box + lane * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          uint4 v;
          v.x = pack_bf16x2(__uint_as_float(r[q * 8 + 0]), __uint_as_float(r[q * 8 + 1]));
          v.y = pack_bf16x2(__uint_as_float(r[q * 8 + 2]), __uint_as_float(r[q * 8 + 3]));
          v.z = pack_bf16x2(__uint_as_float(r[q * 8 + 4]), __uint_as_float(r[q * 8 + 5]));
          v.w = pack_bf16x2(__uint_as_float(r[q * 8 + 6]), __uint_as_float(r[q * 8 + 7]));
          *reinterpret_cast<uint4*>(srow + ((q ^ (lane & 7)) << 4)) = v;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&map_c, box, nb * BN + c0, row0);
          bulk_commit_group();
        }
        ++nbox;
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_group0();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---- 2-SM variant ---------------------------------------------------------------------------
// A cluster of two CTAs (two SMs) computes a 256x256 tile with tcgen05.mma.cta_group::2
// (M=256, N=256, K=16): each CTA stages its own 128 rows of A and its own 128 columns of B, so
// per SM the operand traffic is 2/3 of the 1-SM 128x256 tile and the 32 KB stages allow a
// 6-deep ring.  The leader CTA (rank 0) arms the stage barrier for both CTAs' bytes and issues
// every MMA; its commits release the stage in both CTAs and hand each CTA's accumulator (its
// 128 TMEM lanes) to that CTA's epilogue.  No load uses multicast: each CTA fetches its own data.
namespace pair {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 6;  // BM, BN: this CTA's rows / the tile's columns
constexpr int TILE_M = 2 * BM;                           // rows per cluster tile
constexpr int NUM_THREADS = 192;
constexpr int A_STAGE_BYTES = BM * BK * 2;      // 16 KB
constexpr int B_CHUNK_BYTES = BK * 64 * 2;      // 8 KB
constexpr int B_STAGE_BYTES = BK * (BN / 2) * 2;  // 16 KB: this CTA's 128 columns
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 8;  // in 256-row blocks
constexpr uint32_t IDESC = idesc_bf16_f32(TILE_M, BN, /*a_mn_major=*/0, /*b_mn_major=*/1);

struct SharedTail {
  uint64_t full[STAGES];       // used in the leader only: both CTAs' bytes for the stage landed
  uint64_t empty[STAGES];      // per CTA: the leader's MMAs are done with this CTA's stage
  uint64_t tmem_full[2];       // per CTA: its accumulator half is final
  uint64_t tmem_empty[2];      // used in the leader only: 8 epilogue warps (both CTAs) drained it
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
// Epilogue staging: per epilogue warp two [32 rows x 64 columns] bf16 boxes (4 KB each, 128-byte
// swizzle) that its TMA stores read from.
constexpr int C_BOX_BYTES = 32 * 64 * 2;
constexpr int C_STAGE_BYTES = 4 * 2 * C_BOX_BYTES;  // 32 KB
constexpr size_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + C_STAGE_BYTES + sizeof(SharedTail);

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& mb, int& nb) {
  const int group = GROUP_M * tiles_n;
  const int g = t / group;
  const int first_m = g * GROUP_M;
  const int gm = min(GROUP_M, tiles_m - first_m);
  const int r = t - g * group;
  mb = first_m + r % gm;
  nb = r / gm;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_bf16_tc2_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                         const __grid_constant__ CUtensorMap map_c, int M, int N, int K, unsigned* err_word) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  // Both CTAs compute the same aligned offsets (the MMA descriptors name one offset for both).
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + STAGES * A_STAGE_BYTES;
  uint8_t* smem_c = smem + STAGES * STAGE_BYTES;
  SharedTail* st = reinterpret_cast<SharedTail*>(smem + STAGES * STAGE_BYTES + C_STAGE_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster_id = static_cast<int>(blockIdx.x) >> 1;
  const int num_clusters = static_cast<int>(gridDim.x) >> 1;
  const int tiles_m = (M + TILE_M - 1) / TILE_M;
  const int tiles_n = (N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&st->full[s], 1);
      mbar_init(&st->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&st->tmem_full[b], 1);
      mbar_init(&st->tmem_empty[b], 8);
    }
    mbar_init(&st->drain, 1);
    st->abort_flag = 0;
    fence_barrier_init_cluster();
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    tma_prefetch_desc(&map_c);
  }
  if (warp == 0) {
    tmem_alloc_pair(&st->tmem_base, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barrier inits and the TMEM allocation visible to both CTAs
  tc_fence_after();
  const uint32_t tmem_base = st->tmem_base;
  volatile int* abort_flag = &st->abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int t = cluster_id; t < num_tiles && ok; t += num_clusters) {
        int mb, nb;
        tile_coords(t, tiles_m, tiles_n, mb, nb);
        const int row0 = mb * TILE_M + static_cast<int>(rank) * BM;
        const int col0 = nb * BN + static_cast<int>(rank) * (BN / 2);
        for (int kb = 0; kb < num_kb; ++kb) {
          // empty[stage] (this CTA's) next completes for the use after this one, which needs the
          // load issued here: the parity wait is unambiguous.
          if (!mbar_wait_bounded(&st->empty[stage], phase ^ 1u, abort_flag, err_word, kErrGemmProducerWait)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&st->full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&st->full[stage], 2 * STAGE_BYTES);
          tma_load_2d_pair(smem_a + stage * A_STAGE_BYTES, &map_a, kb * BK, row0, full_leader);
          uint8_t* bdst = smem_b + stage * B_STAGE_BYTES;
#pragma unroll
          for (int c = 0; c < BN / 128; ++c)
            tma_load_2d_pair(bdst + c * B_CHUNK_BYTES, &map_b, col0 + c * 64, kb * BK, full_leader);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Tail: the leader's last commits on this CTA's empty barriers (and so every MMA read of
      // this CTA's stages) must land before the CTA may exit.  Bounded.
      // Use u of a stage is released by phase u / STAGES of its empty barrier.
      for (int u = issued > STAGES ? issued - STAGES : 0; u < issued; ++u) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&st->empty[u % STAGES], (u / STAGES) & 1) && !*abort_flag &&
               globaltimer_ns() - t0 < 200000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA only) ----------------
    // The whole warp runs the loop (waits polled by every lane), one elected lane issues.
    if (leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true, issued = false;
      for (int t = cluster_id; t < num_tiles && ok; t += num_clusters) {
        // tmem_empty[acc] next completes after this accumulator is committed again (below).
        if (!warp_wait_poll(&st->tmem_empty[acc], acc_phase ^ 1u, abort_flag, err_word, kErrGemmMmaWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          // full[stage] next completes for the stage's next use, whose loads wait on empty[stage],
          // committed only below.
          if (!warp_wait_poll(&st->full[stage], phase, abort_flag, err_word, kErrGemmMmaWait)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad0 = smem_desc_sw128(smem_u32(smem_a + stage * A_STAGE_BYTES), 16, 1024);
          const uint64_t bd0 = smem_desc_sw128(smem_u32(smem_b + stage * B_STAGE_BYTES), B_CHUNK_BYTES, 1024);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // +32 B (A) and +2 KB (B) per K=16 step: +2 and +128 in the address field (bytes / 16).
            umma_f16_ss_pair_w(d_tmem, ad0 + k * 2, bd0 + k * 128, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
            issued = true;
          }
          umma_commit_pair_w(&st->empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair_w(&st->tmem_full[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
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
    // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
    // Per 64-column chunk: two 32-column TMEM loads, bf16 rows into one of this warp's two
    // swizzled staging boxes (16-byte chunk k of row r at chunk k ^ (r & 7): conflict-free),
    // then one TMA store of the [32 x 64] box (rows past M / columns past N are clipped).  The
    // accumulator is released as soon as its last columns are in registers.
    const int quarter = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    int nbox = 0;  // boxes this warp has stored (selects the staging buffer)
    uint8_t* cbuf = smem_c + quarter * 2 * C_BOX_BYTES;
    for (int t = cluster_id; t < num_tiles; t += num_clusters) {
      int mb, nb;
      tile_coords(t, tiles_m, tiles_n, mb, nb);
      // tmem_full[acc] next completes after this warp releases the accumulator (below).
      if (!mbar_wait_bounded(&st->tmem_full[acc], acc_phase, abort_flag, err_word, kErrGemmEpilogueWait)) break;
      tc_fence_after();
      const int row0 = mb * TILE_M + static_cast<int>(rank) * BM + quarter * 32;
      const uint32_t tbase = tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 64) {
        uint32_t r[64];
        tmem_ld64(tbase + c0, r);
        if (c0 + 64 == BN) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&st->tmem_empty[acc]), 0));
        }
        uint8_t* box = cbuf + (nbox & 1) * C_BOX_BYTES;
        // The store issued from this buffer two boxes ago must have finished reading it.
        if (lane == 0) bulk_wait_group_read1();
        __syncwarp();
        uint8_t* srow = box + lane * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          uint4 v;
          v.x = pack_bf16x2(__uint_as_float(r[q * 8 + 0]), __uint_as_float(r[q * 8 + 1]));
          v.y = pack_bf16x2(__uint_as_float(r[q * 8 + 2]), __uint_as_float(r[q * 8 + 3]));
          v.z = pack_bf16x2(__uint_as_float(r[q * 8 + 4]), __uint_as_float(r[q * 8 + 5]));
          v.w = pack_bf16x2(__uint_as_float(r[q * 8 + 6]), __uint_as_float(r[q * 8 + 7]));
          *reinterpret_cast<uint4*>(srow + ((q ^ (lane & 7)) << 4)) = v;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&map_c, box, nb * BN + c0, row0);
          bulk_commit_group();
        }
        ++nbox;
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_group0();  // the stores complete before the CTA exits
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while the pair's MMAs, commits or loads can touch it
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace pair

// ---- host side ------------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

}  // namespace

// Resolves cuTensorMapEncodeTiled through the runtime so the library needs no -lcuda.
void* tensor_map_encoder() {
  static void* fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = p;
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with leading dimension ld (elements),
// box [box_rows, box_cols], 128-byte swizzle, zero fill out of bounds.
bool make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                       uint32_t box_rows, uint32_t box_cols) {
  auto enc = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool gemm_bf16_tc_supported(const void* a, const void* b, const void* c, int m, int k, int n) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return m > 0 && k > 0 && n > 0 && (k % 8) == 0 && (n % 8) == 0 && al(a) && al(b) && al(c) &&
         tensor_map_encoder() != nullptr;
}

cudaError_t gemm_bf16_tc(const __nv_bfloat16* a, const __nv_bfloat16* b, __nv_bfloat16* c, int m, int k, int n,
                         cudaStream_t s) {
  DeviceCtx* ctx = device_ctx();
  if (!ctx) return cudaErrorNoDevice;
  CUtensorMap ma, mb, mc;
  if (!make_tmap_bf16_2d(&ma, a, m, k, k, BM, BK)) return cudaErrorInvalidValue;
  if (!make_tmap_bf16_2d(&mb, b, k, n, n, BK, 64)) return cudaErrorInvalidValue;
  if (!make_tmap_bf16_2d(&mc, c, m, n, n, 32, 64)) return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> attr_done{0};  // devices with the attributes set
  {
    const cudaError_t ea = once_per_device(attr_done, [&]() -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(gemm_bf16_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(SMEM_BYTES));
      if (e != cudaSuccess) return e;
      return cudaSuccess;
    });
    if (ea != cudaSuccess) return ea;
  }
  const int tiles = ((m + BM - 1) / BM) * ((n + BN - 1) / BN);
  const int grid = tiles < ctx->sm_count ? tiles : ctx->sm_count;
  gemm_bf16_tc_kernel<<<grid, NUM_THREADS, SMEM_BYTES, s>>>(ma, mb, mc, m, n, k, ctx->err_word,
                                                            take_gemm_stall_kblock());
  return cudaGetLastError();
}

// 2-SM variant: clusters of two CTAs, 256x256 tiles.
cudaError_t gemm_bf16_tc2(const __nv_bfloat16* a, const __nv_bfloat16* b, __nv_bfloat16* c, int m, int k, int n,
                          cudaStream_t s) {
  DeviceCtx* ctx = device_ctx();
  if (!ctx) return cudaErrorNoDevice;
  CUtensorMap ma, mb;
  CUtensorMap mc;
  if (!make_tmap_bf16_2d(&ma, a, m, k, k, pair::BM, pair::BK)) return cudaErrorInvalidValue;
  if (!make_tmap_bf16_2d(&mb, b, k, n, n, pair::BK, 64)) return cudaErrorInvalidValue;
  if (!make_tmap_bf16_2d(&mc, c, m, n, n, 32, 64)) return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> attr_done{0};  // devices with the attributes set
  {
    const cudaError_t ea = once_per_device(attr_done, [&]() -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(pair::gemm_bf16_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(pair::SMEM_BYTES));
      if (e != cudaSuccess) return e;
      return cudaSuccess;
    });
    if (ea != cudaSuccess) return ea;
  }
  const int tiles = ((m + pair::TILE_M - 1) / pair::TILE_M) * ((n + pair::BN - 1) / pair::BN);
  const int clusters = tiles < ctx->sm_count / 2 ? tiles : ctx->sm_count / 2;
  pair::gemm_bf16_tc2_kernel<<<2 * clusters, pair::NUM_THREADS, pair::SMEM_BYTES, s>>>(ma, mb, mc, m, n, k,
                                                                                       ctx->err_word);
  return cudaGetLastError();
}

cudaError_t gemm_bf16(const __nv_bfloat16* a, const __nv_bfloat16* b, __nv_bfloat16* c, int m, int k, int n,
                      cudaStream_t s) {
  std::string cfg;
  const bool tuned = tune_lookup(LC_TUNE_MATMUL, m, k, n, 1 /*bf16*/, &cfg);
  if ((tuned && cfg == kGemvName && m <= 2) || (!tuned && m <= 2)) return gemv_bf16(a, b, c, m, k, n, s);
  if ((tuned && cfg == "simt") || !gemm_bf16_tc_supported(a, b, c, m, k, n)) return gemm_bf16_simt(a, b, c, m, k, n, s);
  if (tuned && cfg == kGemmTc2Name) return gemm_bf16_tc2(a, b, c, m, k, n, s);
  if (tuned && cfg == kGemmTcName) return gemm_bf16_tc(a, b, c, m, k, n, s);
  // Untuned: the 2-SM 256x256 tile once there are enough tiles to fill most of the SM pairs.
  const bool big = m >= 256 && static_cast<long long>(m) * n >= 64LL * 256 * 256;
  return big ? gemm_bf16_tc2(a, b, c, m, k, n, s) : gemm_bf16_tc(a, b, c, m, k, n, s);
}

}  // namespace lcb
