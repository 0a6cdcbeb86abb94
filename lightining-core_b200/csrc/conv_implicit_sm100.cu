// Strict-fp32 NCHW conv as an implicit GEMM on the 5th-generation tensor cores (3xTF32 split),
// with bias and ReLU in the epilogue and the output written straight in NCHW -- the layout the
// integrated pipeline reads as raw Q/K/V channel blocks.  Replaces the reference's conv2dNchw
// (include/lightning_core/core/ops.hpp:1044-1212: im2col + packed weights + bias/ReLU scatter;
// Metal 3x3 kernels src/ops/conv2d_metal.mm:76-390) for shapes with in_channels % 32 == 0 and
// 16 <= out_channels <= 256, out_channels % 16 == 0.
//
// GEMM view: out[n, oc, p] = sum_kk col[(n, p), kk] * W'[oc, kk] with the reduction index ordered
// kk = (dy * kw + dx) * C + c, so one 32-wide k-block is 32 consecutive input channels at one
// kernel tap (dy, dx).  M = output pixels of all images (128 per tile), N = out_channels (one MMA
// covers them all), K = C * kh * kw.
//   warps 0..7   producers: gather the im2col tile [128 pixels x 32 channels] straight from the
//                NCHW input (lanes walk consecutive pixels: coalesced loads), split each value into
//                tf32 hi + lo, and store both planes K-major with the 128-byte swizzle the MMA
//                descriptors expect; lane 0 of warp 0 also TMA-loads the matching [OC x 32] tiles
//                of the pre-split weight planes.  Nothing of the im2col matrix ever reaches HBM.
//   warp 8       MMA: three tcgen05.mma.kind::tf32 (M=128, N=OC, K=8) per K=8 step
//                (lo*hi + hi*lo + hi*hi, small terms first) into one of two TMEM accumulators.
//   warps 9..12  epilogue: TMEM -> + bias -> ReLU -> NCHW stores (a warp stores 32 consecutive
//                pixels of one channel per instruction), overlapping the next tile's MMAs.
// Every mbarrier wait is bounded (common.cuh): a CTA that gives up records the site, drains and
// exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/lc_b200.h"
#include "common.cuh"
#include "lc_internal.hpp"

namespace lcb {

void* tensor_map_encoder();

namespace {

constexpr int BM = 128;              // output pixels per tile (= TMEM lanes)
constexpr int BK = 32;               // channels per k-block (128 bytes of fp32: one swizzle row)
constexpr int STAGES = 2;
constexpr int NUM_PRODUCER_WARPS = 8;
constexpr int MMA_WARP = NUM_PRODUCER_WARPS;
constexpr int NUM_THREADS = (NUM_PRODUCER_WARPS + 1 + 4) * 32;
constexpr int A_PLANE_BYTES = BM * BK * 4;  // 16 KB
constexpr int MAX_OC = 256;
constexpr int B_PLANE_MAX = MAX_OC * BK * 4;  // 32 KB
constexpr int STAGE_MAX = 2 * A_PLANE_BYTES + 2 * B_PLANE_MAX;
constexpr uint32_t TMEM_COLS = 512;  // two accumulators of up to 256 columns

struct Tail {
  uint64_t full[STAGES];     // the 8 producer warps stored this stage's im2col planes
  uint64_t b_full[STAGES];   // the weight planes of this stage landed (TMA bytes)
  uint64_t empty[STAGES];    // the MMAs reading this stage finished
  uint64_t tmem_full[2];     // a tile's accumulator is final
  uint64_t tmem_empty[2];    // the 4 epilogue warps drained it
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

struct ConvParams {
  const float* x;
  float* out;
  const float* bias;
  int batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, oh, ow;
  int relu;
  int pixels;  // batch * oh * ow
  int num_kb;  // kh * kw * in_c / BK
  unsigned* err_word;
  QkvSplitOut qkv;  // fused integrated-pipeline epilogue (cluster-pair kernel only) when qkv.q_hi != nullptr
};

// x rounded to tf32 (nearest, ties away), the 13 low mantissa bits cleared; inf/NaN pass through.
__device__ __forceinline__ float tf32_hi(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & 0xffffe000u;
  return __uint_as_float(u);
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    conv_implicit_tf32x3_kernel(const __grid_constant__ CUtensorMap map_whi, const __grid_constant__ CUtensorMap map_wlo,
                                const ConvParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int b_plane = p.out_c * BK * 4;
  const int stage_bytes = 2 * A_PLANE_BYTES + 2 * b_plane;  // A_hi | A_lo | W_hi | W_lo
  Tail* st = reinterpret_cast<Tail*>(smem + STAGES * stage_bytes);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = (p.pixels + BM - 1) / BM;
  const int cblocks = p.in_c / BK;
  const int pix_img = p.oh * p.ow;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&st->full[s], NUM_PRODUCER_WARPS);
      mbar_init(&st->b_full[s], 1);
      mbar_init(&st->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&st->tmem_full[b], 1);
      mbar_init(&st->tmem_empty[b], 4);
    }
    mbar_init(&st->drain, 1);
    st->abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&map_whi);
    tma_prefetch_desc(&map_wlo);
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

  if (warp < NUM_PRODUCER_WARPS) {
    // ---------------- producers: im2col gather + tf32 split into swizzled smem ----------------
    const int row = (warp & 3) * 32 + lane;     // pixel row of the tile (= A row)
    const int ch0 = (warp >> 2) * 16;           // this warp's 16 channels of the 32-channel block
    const bool tma_thread = warp == 0 && lane == 0;
    int stage = 0;
    uint32_t phase = 0;
    int b_issued = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      const int gp = t * BM + row;
      const bool pix_ok = gp < p.pixels;
      const int n = pix_ok ? gp / pix_img : 0;
      const int pp = gp - n * pix_img;
      const int oy = pp / p.ow, ox = pp - oy * p.ow;
      const float* xn = p.x + static_cast<long long>(n) * p.in_c * p.in_h * p.in_w;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        // empty[stage] next completes for this stage's next use, which needs the stores below.
        if (!warp_wait_poll(&st->empty[stage], phase ^ 1u, abort_flag, p.err_word, kErrGemmProducerWait)) {
          ok = false;
          break;
        }
        uint8_t* base = smem + stage * stage_bytes;
        if (tma_thread) {
          mbar_arrive_expect_tx(&st->b_full[stage], 2 * b_plane);
          tma_load_2d(base + 2 * A_PLANE_BYTES, &map_whi, kb * BK, 0, &st->b_full[stage]);
          tma_load_2d(base + 2 * A_PLANE_BYTES + b_plane, &map_wlo, kb * BK, 0, &st->b_full[stage]);
          ++b_issued;
        }
        const int tap = kb / cblocks, c0 = (kb - tap * cblocks) * BK + ch0;
        const int dy = tap / p.kw, dx = tap - dy * p.kw;
        const int iy = oy * p.sh - p.ph + dy, ix = ox * p.sw - p.pw + dx;
        const bool in = pix_ok && iy >= 0 && iy < p.in_h && ix >= 0 && ix < p.in_w;
        const float* src = xn + (static_cast<long long>(c0) * p.in_h + iy) * p.in_w + ix;
        const long long cstride = static_cast<long long>(p.in_h) * p.in_w;
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = in ? __ldg(src + i * cstride) : 0.0f;
        uint8_t* arow_hi = base + row * 128;
        uint8_t* arow_lo = base + A_PLANE_BYTES + row * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float4 h, l;
          h.x = tf32_hi(v[4 * q + 0]);
          h.y = tf32_hi(v[4 * q + 1]);
          h.z = tf32_hi(v[4 * q + 2]);
          h.w = tf32_hi(v[4 * q + 3]);
          l.x = v[4 * q + 0] - h.x;
          l.y = v[4 * q + 1] - h.y;
          l.z = v[4 * q + 2] - h.z;
          l.w = v[4 * q + 3] - h.w;
          const int chunk = ((ch0 >> 2) + q) ^ (row & 7);  // 16-byte chunk within the 128-byte row
          *reinterpret_cast<float4*>(arow_hi + chunk * 16) = h;
          *reinterpret_cast<float4*>(arow_lo + chunk * 16) = l;
        }
        fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core's reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&st->full[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok && tma_thread) {
      // Let the weight copies already issued land before shared memory goes away.
      for (int u = b_issued > STAGES ? b_issued - STAGES : 0; u < b_issued; ++u) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&st->b_full[u % STAGES], (u / STAGES) & 1) && globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else if (warp == MMA_WARP) {
    // ---------------- MMA issuer (whole warp, one elected lane issues) ----------------
    const uint32_t idesc = idesc_tf32_f32(BM, p.out_c, 0, 0);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true, issued = false;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      if (!warp_wait_poll(&st->tmem_empty[acc], acc_phase ^ 1u, abort_flag, p.err_word, kErrGemmMmaWait)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * 256);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!warp_wait_poll(&st->full[stage], phase, abort_flag, p.err_word, kErrGemmMmaWait) ||
            !warp_wait_poll(&st->b_full[stage], phase, abort_flag, p.err_word, kErrGemmMmaWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_hi = smem_u32(smem + stage * stage_bytes);
        const uint64_t ahd = smem_desc_sw128(a_hi, 16, 1024);
        const uint64_t ald = smem_desc_sw128(a_hi + A_PLANE_BYTES, 16, 1024);
        const uint64_t bhd = smem_desc_sw128(a_hi + 2 * A_PLANE_BYTES, 16, 1024);
        const uint64_t bld = smem_desc_sw128(a_hi + 2 * A_PLANE_BYTES + b_plane, 16, 1024);
#pragma unroll
        for (int k = 0; k < BK / 8; ++k) {
          // K-major SW128 operands: rows 128 B apart, 8-row groups 1 KB apart; +32 B per K=8 step.
          const uint32_t first = (kb > 0 || k > 0) ? 1u : 0u;
          umma_tf32_ss_w(d_tmem, ald + k * 2, bhd + k * 2, idesc, first);
          umma_tf32_ss_w(d_tmem, ahd + k * 2, bld + k * 2, idesc, 1u);
          umma_tf32_ss_w(d_tmem, ahd + k * 2, bhd + k * 2, idesc, 1u);
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
      umma_commit_w(&st->drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&st->drain, 0) && globaltimer_ns() - t0 < 100000000ull) {
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> bias -> ReLU -> NCHW ----------------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      if (!warp_wait_poll(&st->tmem_full[acc], acc_phase, abort_flag, p.err_word, kErrGemmEpilogueWait)) break;
      tc_fence_after();
      const int gp = t * BM + row;
      const bool pix_ok = gp < p.pixels;
      const int n = pix_ok ? gp / pix_img : 0;
      const int pp = gp - n * pix_img;
      float* dst = p.out + static_cast<long long>(n) * p.out_c * pix_img + pp;
      const uint32_t tbase = tmem_base + static_cast<uint32_t>(acc * 256) + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
      for (int c0 = 0; c0 < p.out_c; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tbase + c0, r);
        if (pix_ok) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float v = __uint_as_float(r[j]) + (p.bias ? __ldg(p.bias + c0 + j) : 0.0f);
            if (p.relu) v = fmaxf(v, 0.0f);
            dst[static_cast<long long>(c0 + j) * pix_img] = v;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&st->tmem_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
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

// ---- cluster-pair kernel fed by TMA im2col loads -----------------------------------------------
// Two CTAs (two SMs) compute a 256-pixel tile with tcgen05.mma.cta_group::2 (M = 256, N = OC):
// each CTA TMA-loads the im2col planes of its own 128 pixels and half of the weight rows, so a
// stage is 32 KB + OC x 128 B (56 KB at OC = 192) and up to four stages fit.  The leader CTA arms
// each stage for both CTAs' bytes and issues every MMA; its commits release the stage in both CTAs
// and hand each CTA's accumulator lanes to that CTA's epilogue, which releases it with a remote
// arrival on the leader.  192 threads: warp 0 TMA, warp 1 MMA (leader), warps 2..5 epilogue.
namespace pairk {
constexpr int MAX_STAGES = 4;
constexpr int NUM_THREADS = 192;
constexpr size_t SMEM_LIMIT = 232448;  // opt-in shared memory per block on sm_100
struct Tail {
  uint64_t full[MAX_STAGES];    // leader: both CTAs' bytes of the stage landed
  uint64_t empty[MAX_STAGES];   // per CTA: the leader's MMAs reading this stage finished
  uint64_t tmem_full[2];        // per CTA: its lanes of a tile's accumulator are final
  uint64_t tmem_empty[2];       // leader: the 8 epilogue warps of both CTAs drained it
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
size_t stage_bytes(int out_c) { return 2 * A_PLANE_BYTES + static_cast<size_t>(out_c) * BK * 4; }
int stages(int out_c) {
  const int st = static_cast<int>((SMEM_LIMIT - 1024 - sizeof(Tail)) / stage_bytes(out_c));
  return st < MAX_STAGES ? st : MAX_STAGES;
}
}  // namespace pairk

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pairk::NUM_THREADS, 1)
    conv_im2col_pair_kernel(const __grid_constant__ CUtensorMap map_whi, const __grid_constant__ CUtensorMap map_wlo,
                            const __grid_constant__ CUtensorMap map_xhi, const __grid_constant__ CUtensorMap map_xlo,
                            const ConvParams p, int nstages) {
  using pairk::Tail;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  // Both CTAs compute the same aligned offsets (the MMA descriptors name one offset for both).
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int half_oc = p.out_c / 2;
  const int b_plane = half_oc * BK * 4;                     // this CTA's weight rows, one plane
  const int sbytes = 2 * A_PLANE_BYTES + 2 * b_plane;       // A_hi | A_lo | W_hi | W_lo
  const int STAGES = nstages;
  Tail* st = reinterpret_cast<Tail*>(smem + STAGES * sbytes);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster_id = static_cast<int>(blockIdx.x) >> 1;
  const int num_clusters = static_cast<int>(gridDim.x) >> 1;
  const int num_tiles = (p.pixels + 2 * BM - 1) / (2 * BM);
  const int cblocks = p.in_c / BK;
  const int pix_img = p.oh * p.ow;

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
    tma_prefetch_desc(&map_whi);
    tma_prefetch_desc(&map_wlo);
    tma_prefetch_desc(&map_xhi);
    tma_prefetch_desc(&map_xlo);
  }
  if (warp == 0) {
    tmem_alloc_pair(&st->tmem_base, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barrier inits and the TMEM allocation visible to both CTAs
  tc_fence_after();
  griddep_wait();  // the split planes of x come from the pre-pass
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
        const int gp = t * 2 * BM + static_cast<int>(rank) * BM;  // this CTA's first pixel
        const int n = gp / pix_img, pp = gp - n * pix_img;
        const int oy = pp / p.ow, ox = pp - oy * p.ow;
        const int w0 = ox * p.sw - p.pw, h0 = oy * p.sh - p.ph;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          // empty[stage] (this CTA's) next completes for the use after this one, which needs the
          // loads issued here: the parity wait is unambiguous.
          if (!mbar_wait_bounded(&st->empty[stage], phase ^ 1u, abort_flag, p.err_word, kErrGemmProducerWait)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&st->full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&st->full[stage], 2 * sbytes);
          uint8_t* base = smem + stage * sbytes;
          const int tap = kb / cblocks, c0 = (kb - tap * cblocks) * BK;
          const uint16_t dy = static_cast<uint16_t>(tap / p.kw), dx = static_cast<uint16_t>(tap % p.kw);
          tma_load_im2col_4d_pair(base, &map_xhi, c0, w0, h0, n, dx, dy, full_leader);
          tma_load_im2col_4d_pair(base + A_PLANE_BYTES, &map_xlo, c0, w0, h0, n, dx, dy, full_leader);
          const int wrow = static_cast<int>(rank) * half_oc;
          tma_load_2d_pair(base + 2 * A_PLANE_BYTES, &map_whi, kb * BK, wrow, full_leader);
          tma_load_2d_pair(base + 2 * A_PLANE_BYTES + b_plane, &map_wlo, kb * BK, wrow, full_leader);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Tail: the leader's last commits on this CTA's empty barriers (so every MMA read of this
      // CTA's stages) must land before the CTA may exit.  Use u of a stage: phase u / STAGES.
      for (int u = issued > STAGES ? issued - STAGES : 0; u < issued; ++u) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&st->empty[u % STAGES], (u / STAGES) & 1) && !*abort_flag &&
               globaltimer_ns() - t0 < 200000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA only) ----------------
    if (leader) {
      const uint32_t idesc = idesc_tf32_f32(2 * BM, p.out_c, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true, issued = false;
      for (int t = cluster_id; t < num_tiles && ok; t += num_clusters) {
        if (!warp_wait_poll(&st->tmem_empty[acc], acc_phase ^ 1u, abort_flag, p.err_word, kErrGemmMmaWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * 256);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!warp_wait_poll(&st->full[stage], phase, abort_flag, p.err_word, kErrGemmMmaWait)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_hi = smem_u32(smem + stage * sbytes);
          const uint64_t ahd = smem_desc_sw128(a_hi, 16, 1024);
          const uint64_t ald = smem_desc_sw128(a_hi + A_PLANE_BYTES, 16, 1024);
          const uint64_t bhd = smem_desc_sw128(a_hi + 2 * A_PLANE_BYTES, 16, 1024);
          const uint64_t bld = smem_desc_sw128(a_hi + 2 * A_PLANE_BYTES + b_plane, 16, 1024);
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            // K-major SW128 operands: rows 128 B apart, 8-row groups 1 KB apart; +32 B per K=8 step.
            const uint32_t first = (kb > 0 || k > 0) ? 1u : 0u;
            umma_tf32_ss_pair_w(d_tmem, ald + k * 2, bhd + k * 2, idesc, first);
            umma_tf32_ss_pair_w(d_tmem, ahd + k * 2, bld + k * 2, idesc, 1u);
            umma_tf32_ss_pair_w(d_tmem, ahd + k * 2, bhd + k * 2, idesc, 1u);
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
    // ---------------- epilogue (warps 2..5 of both CTAs): TMEM -> bias -> ReLU -> NCHW ----------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cluster_id; t < num_tiles; t += num_clusters) {
      if (!warp_wait_poll(&st->tmem_full[acc], acc_phase, abort_flag, p.err_word, kErrGemmEpilogueWait)) break;
      tc_fence_after();
      const int gp = t * 2 * BM + static_cast<int>(rank) * BM + row;
      const bool pix_ok = gp < p.pixels;
      const int n = pix_ok ? gp / pix_img : 0;
      const int pp = gp - n * pix_img;
      const uint32_t tbase = tmem_base + static_cast<uint32_t>(acc * 256) + (static_cast<uint32_t>(quarter * 32) << 16);
      if (!p.qkv.q_hi) {
        float* dst = p.out + static_cast<long long>(n) * p.out_c * pix_img + pp;
#pragma unroll 1
        for (int c0 = 0; c0 < p.out_c; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(tbase + c0, r);
          if (pix_ok) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float v = __uint_as_float(r[j]) + (p.bias ? __ldg(p.bias + c0 + j) : 0.0f);
              if (p.relu) v = fmaxf(v, 0.0f);
              dst[static_cast<long long>(c0 + j) * pix_img] = v;
            }
          }
        }
      } else {
        // Fused pipeline: channel c of image n is flat range [c*pix, (c+1)*pix) of the image's conv
        // output; with need a multiple of pix, channels [0, cpn) are Q, [cpn, 2cpn) K, [2cpn, 3cpn) V
        // (cpn a multiple of 16 here, so a 16-channel group lies in one operand).
        const int cpn = static_cast<int>(p.qkv.need / pix_img);
        const long long rowoff = static_cast<long long>(n) * p.qkv.need + pp;
#pragma unroll 1
        for (int c0 = 0; c0 < p.out_c && c0 < 3 * cpn; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(tbase + c0, r);
          const int seg = (c0 >= cpn) + (c0 >= 2 * cpn);
          const long long o = rowoff + static_cast<long long>(c0 - seg * cpn) * pix_img;
          if (pix_ok) {
            if (seg == 2) {
              float* d = p.qkv.v + o;
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                float v = __uint_as_float(r[j]) + (p.bias ? __ldg(p.bias + c0 + j) : 0.0f);
                if (p.relu) v = fmaxf(v, 0.0f);
                d[static_cast<long long>(j) * pix_img] = v;
              }
            } else {
              float* dh = (seg ? p.qkv.k_hi : p.qkv.q_hi) + o;
              float* dl = (seg ? p.qkv.k_lo : p.qkv.q_lo) + o;
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                float v = __uint_as_float(r[j]) + (p.bias ? __ldg(p.bias + c0 + j) : 0.0f);
                if (p.relu) v = fmaxf(v, 0.0f);
                const float h = tf32_hi(v);
                dh[static_cast<long long>(j) * pix_img] = h;
                dl[static_cast<long long>(j) * pix_img] = v - h;
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&st->tmem_empty[acc]), 0));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
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

// NCHW x -> hi / lo planes in NHWC (channels innermost, as the im2col TMA mode reads them):
// 32 channels x 32 pixels of one image per block through shared memory, coalesced both ways.
__global__ void nchw_to_nhwc_split_kernel(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                                          int c, int pix) {
  griddep_launch_dependents();  // the conv may take its SMs now; it waits for these planes itself
  __shared__ float tile[32][33];
  const int n = blockIdx.z, c0 = blockIdx.y * 32, p0 = blockIdx.x * 32;
  const float* xn = x + static_cast<long long>(n) * c * pix;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int ci = c0 + r, pi = p0 + threadIdx.x;
    tile[r][threadIdx.x] = (ci < c && pi < pix) ? xn[static_cast<long long>(ci) * pix + pi] : 0.0f;
  }
  __syncthreads();
  const long long base = static_cast<long long>(n) * pix * c;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int pi = p0 + r, ci = c0 + threadIdx.x;
    if (pi < pix && ci < c) {
      const float v = tile[threadIdx.x][r];
      const float h = tf32_hi(v);
      hi[base + static_cast<long long>(pi) * c + ci] = h;
      lo[base + static_cast<long long>(pi) * c + ci] = v - h;
    }
  }
}

// OIHW weights -> hi / lo planes [OC, kh*kw*C] with the reduction index (dy*kw + dx)*C + c.
__global__ void conv_weight_split_kernel(const float* __restrict__ w, float* __restrict__ hi, float* __restrict__ lo,
                                         int oc, int c, int kh, int kw) {
  const int k = c * kh * kw;
  const long long total = static_cast<long long>(oc) * k;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int o = static_cast<int>(i / k), kk = static_cast<int>(i - static_cast<long long>(o) * k);
    const int tap = kk / c, ci = kk - tap * c;
    const int dy = tap / kw, dx = tap - dy * kw;
    const float v = w[((static_cast<long long>(o) * c + ci) * kh + dy) * kw + dx];
    const float h = tf32_hi(v);
    hi[i] = h;
    lo[i] = v - h;
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [rows, cols] fp32 row-major, box [box_rows, 32 columns], 128-byte swizzle.
bool make_weight_map(CUtensorMap* map, const float* base, int rows, int cols, int box_rows) {
  auto enc = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!enc) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 4};
  cuuint32_t box[2] = {BK, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

using EncodeIm2colFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const int*, const int*, cuuint32_t, cuuint32_t,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeIm2colFn im2col_encoder() {
  static EncodeIm2colFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeIm2colFn>(f);
  });
  return fn;
}

// NHWC fp32 plane [n, h, w, c]: im2col boxes of BM output pixels x BK channels.  The pixel box
// runs over the output grid: its lower corner is -pad, its upper corner pad - (kernel - 1), and the
// traversal stride is the conv stride; the per-load offsets select the kernel tap.
bool make_im2col_map(CUtensorMap* map, const float* base, int n, int h, int w, int c, int kh, int kw, int sh, int sw,
                     int ph, int pw) {
  EncodeIm2colFn enc = im2col_encoder();
  if (!enc) return false;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(c), static_cast<cuuint64_t>(w), static_cast<cuuint64_t>(h),
                        static_cast<cuuint64_t>(n)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(c) * 4, static_cast<cuuint64_t>(w) * c * 4,
                           static_cast<cuuint64_t>(h) * w * c * 4};
  int lower[2] = {-pw, -ph};                      // {w, h}
  int upper[2] = {pw - (kw - 1), ph - (kh - 1)};  // {w, h}
  cuuint32_t estr[4] = {1, static_cast<cuuint32_t>(sw), static_cast<cuuint32_t>(sh), 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides, lower, upper, BK, BM,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool conv_implicit_supported(int in_c, int out_c, int kh, int kw) {
  return in_c % BK == 0 && out_c >= 16 && out_c <= MAX_OC && out_c % 16 == 0 && kh >= 1 && kw >= 1 &&
         static_cast<long long>(in_c) * kh * kw < (1LL << 24) && tensor_map_encoder() != nullptr;
}

namespace {
// The cluster-pair TMA-im2col path takes the shape (the input is large enough for the im2col tensor
// map, the kernel geometry fits its corner and stride ranges).
bool pair_path_ok(size_t x_elems, int kh, int kw, int sh, int sw, int ph, int pw) {
  return x_elems * 4 >= (size_t(128) << 10) && im2col_encoder() != nullptr && kh <= 128 && kw <= 128 && ph <= 127 &&
         pw <= 127 && sh <= 8 && sw <= 8;
}

cudaError_t conv_implicit_run(const float* x, const float* w, const float* bias, float* out, int batch, int in_c,
                              int in_h, int in_w, int out_c, int kh, int kw, int sh, int sw, int ph, int pw, int relu,
                              const QkvSplitOut* qkv, cudaStream_t s);
}  // namespace

bool conv_qkv_split_supported(int batch, int in_c, int in_h, int in_w, int out_c, int kh, int kw, int sh, int sw,
                              int ph, int pw) {
  (void)sh, (void)sw;
  return conv_implicit_supported(in_c, out_c, kh, kw) &&
         pair_path_ok(static_cast<size_t>(batch) * in_c * in_h * in_w, kh, kw, sh, sw, ph, pw);
}

cudaError_t conv2d_nchw_f32_implicit_qkv(const float* x, const float* w, const float* bias, int batch, int in_c,
                                         int in_h, int in_w, int out_c, int kh, int kw, int sh, int sw, int ph,
                                         int pw, int relu, const QkvSplitOut& qkv, cudaStream_t s) {
  if (!conv_qkv_split_supported(batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw)) return cudaErrorNotSupported;
  return conv_implicit_run(x, w, bias, nullptr, batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, relu, &qkv, s);
}

cudaError_t conv2d_nchw_f32_implicit(const float* x, const float* w, const float* bias, float* out, int batch,
                                     int in_c, int in_h, int in_w, int out_c, int kh, int kw, int sh, int sw, int ph,
                                     int pw, int relu, cudaStream_t s) {
  return conv_implicit_run(x, w, bias, out, batch, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, relu, nullptr, s);
}

namespace {
cudaError_t conv_implicit_run(const float* x, const float* w, const float* bias, float* out, int batch, int in_c,
                              int in_h, int in_w, int out_c, int kh, int kw, int sh, int sw, int ph, int pw, int relu,
                              const QkvSplitOut* qkv, cudaStream_t s) {
  if (!conv_implicit_supported(in_c, out_c, kh, kw)) return cudaErrorNotSupported;
  DeviceCtx* ctx = device_ctx();
  if (!ctx) return cudaErrorNoDevice;
  const int oh = (in_h + 2 * ph - kh) / sh + 1, ow = (in_w + 2 * pw - kw) / sw + 1;
  const long long pixels = static_cast<long long>(batch) * oh * ow;
  if (pixels > 0x7fffffffLL) return cudaErrorNotSupported;
  const int k = in_c * kh * kw;
  float* ws = nullptr;
  cudaError_t e = workspace_alloc(ctx, reinterpret_cast<void**>(&ws), 2 * static_cast<size_t>(out_c) * k * 4, s);
  if (e != cudaSuccess) return e;
  float* whi = ws;
  float* wlo = ws + static_cast<size_t>(out_c) * k;
  {
    const long long total = static_cast<long long>(out_c) * k;
    const int blocks = static_cast<int>(total / 256 + 1 < 1184 ? total / 256 + 1 : 1184);
    conv_weight_split_kernel<<<blocks, 256, 0, s>>>(w, whi, wlo, out_c, in_c, kh, kw);
    e = cudaGetLastError();
  }
  // The im2col TMA path (a CTA pair per 256-pixel tile) reads pre-split NHWC planes of x; a small
  // input (< 128 KB) keeps the 1-CTA kernel with gathering producers.
  const size_t x_elems = static_cast<size_t>(batch) * in_c * in_h * in_w;
  const bool tma_a = pair_path_ok(x_elems, kh, kw, sh, sw, ph, pw) && ctx->sm_count >= 2;
  if (qkv && !tma_a) {
    workspace_free(ws, s);
    return cudaErrorNotSupported;
  }
  CUtensorMap mhi, mlo, mxhi, mxlo;
  const int wbox = tma_a ? out_c / 2 : out_c;
  if (e == cudaSuccess && (!make_weight_map(&mhi, whi, out_c, k, wbox) || !make_weight_map(&mlo, wlo, out_c, k, wbox)))
    e = cudaErrorInvalidValue;
  float* xws = nullptr;
  if (e == cudaSuccess && tma_a) {
    e = workspace_alloc(ctx, reinterpret_cast<void**>(&xws), 2 * x_elems * 4, s);
    if (e == cudaSuccess) {
      const int pix = in_h * in_w;
      nchw_to_nhwc_split_kernel<<<dim3((pix + 31) / 32, (in_c + 31) / 32, batch), dim3(32, 8), 0, s>>>(
          x, xws, xws + x_elems, in_c, pix);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess && (!make_im2col_map(&mxhi, xws, batch, in_h, in_w, in_c, kh, kw, sh, sw, ph, pw) ||
                             !make_im2col_map(&mxlo, xws + x_elems, batch, in_h, in_w, in_c, kh, kw, sh, sw, ph, pw)))
      e = cudaErrorInvalidValue;
  }
  if (e == cudaSuccess) {
    // The largest size each kernel can take, once per device.
    static std::atomic<unsigned long long> attr_done{0};  // devices with the attributes set
    e = once_per_device(attr_done, []() -> cudaError_t {
      cudaError_t r = cudaFuncSetAttribute(conv_implicit_tf32x3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(1024 + STAGES * STAGE_MAX + sizeof(Tail)));
      if (r == cudaSuccess)
        r = cudaFuncSetAttribute(conv_im2col_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(pairk::SMEM_LIMIT));
      return r;
    });
  }
  if (e == cudaSuccess) {
    ConvParams p;
    p.x = x;
    p.out = out;
    p.bias = bias;
    p.batch = batch;
    p.in_c = in_c;
    p.in_h = in_h;
    p.in_w = in_w;
    p.out_c = out_c;
    p.kh = kh;
    p.kw = kw;
    p.sh = sh;
    p.sw = sw;
    p.ph = ph;
    p.pw = pw;
    p.oh = oh;
    p.ow = ow;
    p.relu = relu;
    p.pixels = static_cast<int>(pixels);
    p.num_kb = k / BK;
    p.err_word = ctx->err_word;
    p.qkv = qkv ? *qkv : QkvSplitOut{nullptr, nullptr, nullptr, nullptr, nullptr, 0};
    if (tma_a) {
      const int nst = pairk::stages(out_c);
      const size_t psmem = 1024 + nst * pairk::stage_bytes(out_c) + sizeof(pairk::Tail);
      const long long tiles = (pixels + 2 * BM - 1) / (2 * BM);
      const int max_clusters = ctx->sm_count / 2;
      const int clusters = static_cast<int>(tiles < max_clusters ? tiles : max_clusters);
      e = launch_pdl(conv_im2col_pair_kernel, dim3(2 * clusters), dim3(pairk::NUM_THREADS), psmem, s, mhi, mlo, mxhi,
                     mxlo, p, nst);
    } else {
      const long long tiles = (pixels + BM - 1) / BM;
      const int grid = static_cast<int>(tiles < ctx->sm_count ? tiles : ctx->sm_count);
      const size_t smem = 1024 + STAGES * (2 * A_PLANE_BYTES + 2 * static_cast<size_t>(out_c) * BK * 4) + sizeof(Tail);
      conv_implicit_tf32x3_kernel<<<grid, NUM_THREADS, smem, s>>>(mhi, mlo, p);
      e = cudaGetLastError();
    }
  }
  if (xws) {
    const cudaError_t ex = workspace_free(xws, s);
    if (e == cudaSuccess) e = ex;
  }
  const cudaError_t ef = workspace_free(ws, s);
  return e != cudaSuccess ? e : ef;
}

}  // namespace

}  // namespace lcb
