// Flash-attention forward on the 5th-generation tensor cores (bf16 in/out, fp32 softmax and
// accumulation), for head_dim 64 and 128.  Replaces the reference's attention forward
// (src/attention_cpu.cpp:38-101 arithmetic; Metal modes src/attention_metal.mm:342-576) for the
// batched bf16 config.  Output row i = sum_j softmax_j(q_i . k_j / sqrt(d)) v_j, j <= i if causal,
// then the optional postprocess out*scale + bias (ReLU) of src/attention.cpp:41-60.
//
// One CTA = one 128-row Q tile of one (batch, head) unit, two CTAs per SM; 224 threads:
//   warp 0      TMA: Q once, then K_j tiles (64 keys) into a 2-stage ring freed as soon as S_j
//               is done; warp 6 loads V_j into a 2-stage ring freed by PV_j (a separate thread,
//               so a late V slot never holds back K); L2 prefetch of upcoming tiles; 3-D tensor
//               maps [units, S, D] so rows past S read as zero; 128-byte swizzle.
//   warp 1      MMA (one thread): S_j = Q K_j^T into one of two TMEM score buffers (so S_{j+1}
//               overlaps the softmax of S_j), then O += P_j V_j with P_j read from TMEM (the A
//               operand of tcgen05.mma may live in tensor memory).
//   warps 2..5  softmax + epilogue: each thread owns one query row (= one TMEM lane), so row
//               max and sum need no shuffles.  Scores are scaled into the log2 domain; O is
//               rescaled in TMEM only when the running max grows by more than 8 (2^8), which
//               keeps exp2 values <= 256 and the final O / l exact.  P_j is written as packed
//               bf16 pairs over the first 32 columns of S_j's own TMEM buffer (tcgen05.st), so
//               it never touches shared memory.  The epilogue divides by l, applies
//               the postprocess, stages bf16 O in the (by then idle) Q buffer and writes it with
//               TMA stores.
// Causal: only KV tiles at or below the diagonal are visited; per-element masks only on the
// diagonal / sequence-tail tile.  CTAs run in groups of 16 units (heaviest Q tiles of the group
// first), so a wave of CTAs shares the K/V of few units in L2 and the light tiles run last.
// A persistent form of the same kernel (tune-cache name tcgen05_1qp) keeps two CTAs per SM
// resident and lets each claim Q tiles from a global counter; it is exact but measured no faster
// at config 3, so one CTA per Q tile stays the default.
// All mbarrier waits are bounded (common.cuh).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>
#include <string>

#include "../../include/lc_b200.h"
#include "common.cuh"
#include "lc_internal.hpp"

namespace lcb {

bool make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                       uint32_t box_rows, uint32_t box_cols);
void* tensor_map_encoder();

namespace {

constexpr int TILE = 128;               // query rows per CTA (= TMEM lanes)
constexpr int CHUNK_BYTES = 128 * 128;  // one [128 rows x 64 bf16] swizzled box = 16 KB
// KV tiles of TKV keys.  The TMEM score buffers take 128 columns whatever TKV is, so there are
// NB = 128 / TKV of them; the K and V rings have NB stages; P_j aliases score buffer j % NB, and
// S_{j+NB} can only be issued once P.V_j has read P_j.  The library launches TKV = 64; 32-key
// tiles (four buffers, three S tiles in flight) were exact but 23% slower at config 3 (0.186
// against 0.152 ms): the per-tile softmax costs, not the S -> P.V chain, then dominate.
constexpr int kMaxBufs = 4;
constexpr int NUM_THREADS = 224;  // 7 warps: K/Q loader, MMA, 4 softmax, V loader
constexpr uint32_t TMEM_COLS = 256;  // S buffers at 0 and 64, O at 128: two CTAs fit one SM
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_THRESHOLD = 8.0f;
// CTA order: units are taken in groups of kUnitGroup, and inside a group the heaviest Q tiles of
// all its units come first.  Heavy-first inside a group shortens the causal tail (light tiles run
// last); a group small enough to keep its units' K/V in L2 keeps DRAM reads at the algorithmic
// bytes.  Config 3 causal, one-tile kernel: 0.162 ms with one unit per group, 0.150-0.152 ms with
// 16 (256 CTAs per group), 0.156 ms with 128; a later sweep on one box gave 4: 0.162, 8: 0.158,
// 12: 0.164, 16: 0.154, 24: 0.166, 32: 0.154, 64: 0.154 ms.
constexpr int kUnitGroup = 16;

struct AttnTail {
  uint64_t q_full;
  uint64_t k_full[kMaxBufs];
  uint64_t v_full[kMaxBufs];
  uint64_t s_full[kMaxBufs];  // s_full[b]: S_j with j%NB == b is in TMEM (one commit)
  uint64_t p_full[kMaxBufs];  // p_full[b]: P_j with j%NB == b is in TMEM (4 warp arrivals)
  uint64_t o_done[kMaxBufs];  // o_done[b] completes for PV_j with j%NB == b (one phase per NB tiles)
  uint64_t drain;
  uint64_t o_staged;  // the 4 softmax warps have written the bf16 O tile into the Q buffer
  uint64_t item_full[4];   // persistent form: item ring published by the Q/K producer thread
  uint64_t item_empty[4];  // ... and released by the MMA warp, the V thread and 4 softmax warps
  int item_slot[4];
  uint32_t tmem_base;
  int abort_flag;
};

template <int D, int TKV>
struct Layout {
  static constexpr int NB = 128 / TKV;                    // score buffers = K/V ring stages
  static constexpr int NCH = D / 64;                      // 64-column chunks per row
  static constexpr int KCH = TKV * 128;                   // one [TKV rows x 64 bf16] swizzled box
  static constexpr int Q_BYTES = NCH * CHUNK_BYTES;
  static constexpr int KV_BYTES = NCH * KCH;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + Q_BYTES;
  static constexpr int V_OFF = K_OFF + NB * KV_BYTES;
  static constexpr int TAIL_OFF = V_OFF + NB * KV_BYTES;
  // No alignment slack: two CTAs must fit one SM's 228 KB.  The dynamic window of a kernel
  // without static shared memory starts 1 KB-aligned; the kernel checks this and bails out
  // with an error code otherwise.
  static constexpr size_t SMEM = TAIL_OFF + sizeof(AttnTail);
};

constexpr int kItemSlots = 4;

struct FaParams {
  __nv_bfloat16* out;
  unsigned* sched;  // persistent form: [next item counter, finished CTAs], zero at launch
  int units, seq, nq;  // nq = Q tiles per unit
  int group;           // causal CTA order: units per group, heaviest Q tiles of a group first
  int causal;
  float scale_log2;    // softmax scale * log2(e)
  float post_scale, post_bias;
  int post_relu, post;
  unsigned* err_word;
};

// 2^x with the hardware approximation (MUFU ex2, flush-to-zero): P is rounded to bf16 right
// after, and results below 2^-126 are irrelevant to a softmax weight.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32x2 arithmetic and the 3-input max of sm_100: half the FP instructions per score.
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void unpk2(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// 2^x for a pair of scores on the FMA pipes instead of MUFU: x = i + f with i = rint(x) (adding
// and subtracting 1.5 * 2^23), f in [-0.5, 0.5]; 2^f by a degree-3 polynomial whose coefficients
// are a weighted-least-squares minimax fit of 2^f on that interval (relative error 7.5e-5, far
// below the bf16 rounding of P); 2^i is added into the exponent field.  x is clamped at -125 so
// the result stays a normal number (a masked score gives 2^-125 instead of 0).
__device__ __forceinline__ void exp2_poly_pair(float x0, float x1, float& y0, float& y1) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  const uint64_t xx = pk2(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const uint64_t t = add2(xx, pk2(kRound, kRound));
  const uint64_t r = add2(t, pk2(-kRound, -kRound));
  const uint64_t f = fma2(r, pk2(-1.0f, -1.0f), xx);
  uint64_t q = fma2(pk2(0.05517132207751274f, 0.05517132207751274f), f,
                    pk2(0.24261054396629333f, 0.24261054396629333f));
  q = fma2(q, f, pk2(0.6932609677314758f, 0.6932609677314758f));
  q = fma2(q, f, pk2(0.9999281167984009f, 0.9999281167984009f));
  float q0, q1, t0, t1;
  unpk2(q, q0, q1);
  unpk2(t, t0, t1);
  y0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
  y1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 3-D TMA load: coordinates (d, row, unit).
__device__ __forceinline__ void load_rows(uint8_t* dst, const CUtensorMap* map, int nch, int chunk_bytes, int row,
                                          int unit, uint64_t* bar) {
  for (int c = 0; c < nch; ++c) tma_load_3d(dst + c * chunk_bytes, map, c * 64, row, unit, bar);
}

// Item b (0 <= b < nq * units) -> (Q tile, unit).  Units are taken in groups of p.group; inside a
// group the heaviest Q tiles of all its units come first.
__device__ __forceinline__ void fa_item(const FaParams& p, int b, int& qt, int& unit) {
  const int per_group = p.group * p.nq;
  const int g = b / per_group, r = b % per_group;
  const int gu = min(p.group, p.units - g * p.group);  // units in this (possibly short) group
  qt = p.nq - 1 - r / gu;
  unit = g * p.group + r % gu;
}
template <int TKV>
__device__ __forceinline__ int fa_kv_tiles(const FaParams& p, int qt) {
  const int kv_tiles_all = (p.seq + TKV - 1) / TKV;
  return p.causal ? min(kv_tiles_all, (qt * TILE + TILE - 1) / TKV + 1) : kv_tiles_all;
}

// The CTA's it-th item: blockIdx.x alone without PERSIST; otherwise read from the item ring
// (-1 = no more items).  Every reader releases the slot once it has the value.
template <bool PERSIST>
__device__ __forceinline__ bool fa_take_item(AttnTail* st, int it, int b0, int n_items, bool whole_warp,
                                             volatile int* abort_flag, unsigned* err, unsigned code, int& b) {
  if (!PERSIST) {
    b = (it == 0 && b0 < n_items) ? b0 : -1;
    return true;
  }
  const int r = it % kItemSlots;
  const uint32_t par = (it / kItemSlots) & 1;
  const bool ok = whole_warp ? warp_wait_poll(&st->item_full[r], par, abort_flag, err, code)
                             : mbar_wait_bounded(&st->item_full[r], par, abort_flag, err, code);
  if (!ok) return false;
  b = *reinterpret_cast<volatile int*>(&st->item_slot[r]);
  if (whole_warp) __syncwarp();
  if (!whole_warp || (threadIdx.x & 31) == 0) mbar_arrive(&st->item_empty[r]);
  return true;
}

// PERSIST = false: one CTA per item (grid = items), O staged in the idle Q buffer.
// PERSIST = true: two resident CTAs per SM; each starts with item blockIdx.x and then claims the
// next unclaimed item of the heavy-first order from a global counter (greedy, so the light items
// fill the tail).  Its Q/K producer thread claims and publishes items to the other roles through
// a 4-slot shared-memory ring.  The K/V rings, the TMEM score buffers and every barrier phase run
// on a global KV-step counter across items, so the next item's K/V loads and first score MMA
// overlap the previous item's last softmax and epilogue; the next Q is loaded as soon as the
// previous item's last S MMA is done, and O is written from registers, so the Q buffer is never
// needed for the epilogue.  This removes the per-CTA launch gap, set-up and cold Q wait, which
// the co-resident CTA had mostly hidden already: measured no faster at config 3.
template <int D, bool PERSIST, int TKV>
__global__ void __launch_bounds__(NUM_THREADS, 2)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                  const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
                  const FaParams p) {
  using LY = Layout<D, TKV>;
  constexpr int NB = LY::NB;
  constexpr int TK = TKV;
  constexpr int KCHUNK_BYTES = LY::KCH;
  constexpr int NCH = LY::NCH;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0) {  // the 128-byte swizzle atoms need 1 KB alignment
    if (threadIdx.x == 0) atomicCAS(p.err_word, 0u, static_cast<unsigned>(kErrAttnLoadWait) | 0x1000u);
    return;
  }
  uint8_t* smem = smem_raw;
  AttnTail* st = reinterpret_cast<AttnTail*>(smem + LY::TAIL_OFF);
  uint8_t* sQ = smem + LY::Q_OFF;
  uint8_t* sK = smem + LY::K_OFF;
  uint8_t* sV = smem + LY::V_OFF;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_items = p.nq * p.units;
  const int b0 = static_cast<int>(blockIdx.x);

  if (threadIdx.x == 0) {
    mbar_init(&st->q_full, 1);
    for (int s = 0; s < NB; ++s) {
      mbar_init(&st->k_full[s], 1);
      mbar_init(&st->v_full[s], 1);
      mbar_init(&st->s_full[s], 1);
      mbar_init(&st->p_full[s], 4);
      mbar_init(&st->o_done[s], 1);
    }
    mbar_init(&st->drain, 1);
    mbar_init(&st->o_staged, 4);
    for (int r = 0; r < kItemSlots; ++r) {
      mbar_init(&st->item_full[r], 1);
      mbar_init(&st->item_empty[r], 6);
    }
    st->abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_v);
    tma_prefetch_desc(&map_o);
    // The first Q tile (a cold HBM read) is requested before the TMEM allocation and the CTA barrier.
    if (b0 < n_items) {
      int qt, unit;
      fa_item(p, b0, qt, unit);
      mbar_arrive_expect_tx(&st->q_full, LY::Q_BYTES);
      load_rows(sQ, &map_q, NCH, CHUNK_BYTES, qt * TILE, unit, &st->q_full);
    }
  }
  if (warp == 0) {
    tmem_alloc(&st->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = st->tmem_base;
  volatile int* abort_flag = &st->abort_flag;

  // Bounded drain of copies already issued, so the CTA never exits with TMA writes in flight.
  auto drain = [](uint64_t* bar, uint32_t ph) {
    const uint64_t t1 = globaltimer_ns();
    while (!mbar_try_wait(bar, ph) && globaltimer_ns() - t1 < 100000000ull) {
    }
  };
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer: Q and K
    if (lane == 0) {
      bool ok = true;
      int g = 0;        // global KV step = K loads issued
      int q_loads = 1;  // Q tiles requested (the first one above)
      // Publish item `it` (b < 0: none left) once every reader has released its ring slot.
      auto publish = [&](int it, int b) -> bool {
        const int r = it % kItemSlots;
        if (it >= kItemSlots && !mbar_wait_bounded(&st->item_empty[r], ((it / kItemSlots) - 1) & 1, abort_flag,
                                                    p.err_word, kErrAttnLoadWait))
          return false;
        st->item_slot[r] = b;
        mbar_arrive(&st->item_full[r]);
        return true;
      };
      for (int b = b0, it = 0; ok; ++it) {
        if (PERSIST && !publish(it, b < n_items ? b : -1)) {
          ok = false;
          break;
        }
        if (b >= n_items) break;
        int qt, unit;
        fa_item(p, b, qt, unit);
        const int n_kv = fa_kv_tiles<TKV>(p, qt);
        int nxt = n_items;
        for (int j = 0; j < n_kv; ++j) {
          const int ks = g % NB;
          // The next item is claimed a few KV steps before this item ends: late enough that claims
          // follow the order CTAs run dry in (greedy balance), early enough that the atomic's
          // latency is hidden.
          if (PERSIST && j == (n_kv > 3 ? n_kv - 3 : 0)) nxt = static_cast<int>(gridDim.x + atomicAdd(p.sched, 1u));
          if (PERSIST && j == n_kv - 1 && nxt < n_items) {
            // Warm L2 with the next item's Q and first K/V tiles: their loads are issued at the
            // item boundary and would otherwise be cold HBM reads on the critical path.
            int nqt, nunit;
            fa_item(p, nxt, nqt, nunit);
            for (int c = 0; c < NCH; ++c) {
              tma_prefetch_l2_3d(&map_q, c * 64, nqt * TILE, nunit);
              tma_prefetch_l2_3d(&map_k, c * 64, 0, nunit);
              tma_prefetch_l2_3d(&map_k, c * 64, TK, nunit);
              tma_prefetch_l2_3d(&map_v, c * 64, 0, nunit);
              tma_prefetch_l2_3d(&map_v, c * 64, TK, nunit);
            }
          }
          if (j + NB < n_kv)  // warm L2 for the K tile that will take this slot next
            for (int c = 0; c < NCH; ++c) tma_prefetch_l2_3d(&map_k, c * 64, (j + NB) * TK, unit);
          // Slot ks last held the K of global step g-2: that S MMA must have finished reading it.
          // Every MMA group has exactly one commit (S_g -> s_full[g&1]), and this thread observes
          // S_0, S_1, ... in order, so each parity wait is unambiguous.
          if (g >= NB && !mbar_wait_bounded(&st->s_full[(g - NB) % NB], ((g - NB) / NB) & 1,
                                                  abort_flag, p.err_word, kErrAttnLoadWait)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&st->k_full[ks], LY::KV_BYTES);
          load_rows(sK + ks * LY::KV_BYTES, &map_k, NCH, KCHUNK_BYTES, j * TK, unit, &st->k_full[ks]);
          ++g;
          if (PERSIST && it > 0 && j == 0) {
            // This item's Q replaces the previous one once the previous item's last S MMA (global
            // step g-2 now) is done; the next completion of that barrier needs this Q, so the
            // parity wait is unambiguous.
            if (!mbar_wait_bounded(&st->s_full[(g - 2) % NB], ((g - 2) / NB) & 1, abort_flag, p.err_word,
                                   kErrAttnLoadWait)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&st->q_full, LY::Q_BYTES);
            load_rows(sQ, &map_q, NCH, CHUNK_BYTES, qt * TILE, unit, &st->q_full);
            ++q_loads;
          }
        }
        if (!PERSIST) break;
        b = nxt;
      }
      if (!ok) {
        drain(&st->q_full, (q_loads - 1) & 1);
        for (int x = g > NB ? g - NB : 0; x < g; ++x) drain(&st->k_full[x % NB], (x / NB) & 1);
      }
    }
  } else if (warp == 6) {
    // ------------------------------------------------------------ TMA producer: V
    // A separate thread, so a V slot that frees late never holds back the next K load.
    if (lane == 0) {
      bool ok = true;
      int g = 0;  // global KV step = V loads issued
      for (int it = 0; ok; ++it) {
        int b;
        if (!fa_take_item<PERSIST>(st, it, b0, n_items, false, abort_flag, p.err_word, kErrAttnLoadWait, b)) {
          ok = false;
          break;
        }
        if (b < 0) break;
        int qt, unit;
        fa_item(p, b, qt, unit);
        const int n_kv = fa_kv_tiles<TKV>(p, qt);
        for (int j = 0; j < n_kv; ++j) {
          const int vs = g % NB;
          if (j + NB < n_kv)
            for (int c = 0; c < NCH; ++c) tma_prefetch_l2_3d(&map_v, c * 64, (j + NB) * TK, unit);
          // Slot vs last held the V of step g-2: that PV (one commit: o_done[g%2]) must be done.
          // PV_g cannot complete before V_g is issued here, so the parity wait is unambiguous.
          if (g >= NB && !mbar_wait_bounded(&st->o_done[(g - NB) % NB], ((g - NB) / NB) & 1,
                                                  abort_flag, p.err_word, kErrAttnLoadWait)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&st->v_full[vs], LY::KV_BYTES);
          load_rows(sV + vs * LY::KV_BYTES, &map_v, NCH, KCHUNK_BYTES, j * TK, unit, &st->v_full[vs]);
          ++g;
        }
      }
      if (!ok)
        for (int x = g > NB ? g - NB : 0; x < g; ++x) drain(&st->v_full[x % NB], (x / NB) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the issue loop (waits polled by every lane) and one elected lane issues
    // each MMA, with descriptors advanced by constant adds.
    constexpr uint32_t IDESC_S = idesc_bf16_f32(TILE, TK, 0, 0);  // Q K-major, K K-major
    constexpr uint32_t IDESC_O = idesc_bf16_f32(TILE, D, 0, 1);   // P (TMEM) K-major, V MN-major
    const uint32_t q_addr = smem_u32(sQ);
    bool ok = true, issued = false;
    auto issue_s = [&](int gs) -> bool {  // S of global step gs into TMEM buffer gs&1
      const int s = gs % NB;
      if (!warp_wait_poll(&st->k_full[s], (gs / NB) & 1, abort_flag, p.err_word, kErrAttnMmaWait))
        return false;
      tc_fence_after();
      const uint64_t qd = smem_desc_sw128(q_addr, 16, 1024);
      const uint64_t kd = smem_desc_sw128(smem_u32(sK + s * LY::KV_BYTES), 16, 1024);
      const uint32_t d_tmem = tmem + static_cast<uint32_t>((gs % NB) * TK);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t qo16 = ((kk >> 2) * CHUNK_BYTES + (kk & 3) * 32) >> 4;  // address field: bytes / 16
        const uint32_t ko16 = ((kk >> 2) * KCHUNK_BYTES + (kk & 3) * 32) >> 4;
        umma_f16_ss_w(d_tmem, qd + qo16, kd + ko16, IDESC_S, kk > 0 ? 1u : 0u);
      }
      issued = true;
      umma_commit_w(&st->s_full[gs % NB]);  // the only commit of this MMA group
      return true;
    };
    int g = 0;  // global KV step of the item's first tile
    for (int it = 0; ok; ++it) {
      int b;
      if (!fa_take_item<PERSIST>(st, it, b0, n_items, true, abort_flag, p.err_word, kErrAttnMmaWait, b)) {
        ok = false;
        break;
      }
      if (b < 0) break;
      int qt, unit;
      fa_item(p, b, qt, unit);
      const int n_kv = fa_kv_tiles<TKV>(p, qt);
      // q_full completes once per item; the next Q needs this item's last S, so parity it&1 is unambiguous.
      ok = warp_wait_poll(&st->q_full, it & 1, abort_flag, p.err_word, kErrAttnMmaWait);
      // S runs NB-1 tiles ahead of P.V: S_{j+NB-1} goes into the buffer of P_{j-1}, which
      // P.V_{j-1} (issued before it, executed in order) has read.
      for (int j = 0; j < NB - 1 && j < n_kv && ok; ++j) ok = issue_s(g + j);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int gg = g + j;
        const int s = gg % NB;
        if (j + NB - 1 < n_kv && !issue_s(gg + NB - 1)) {
          ok = false;
          break;
        }
        // One barrier per TMEM buffer: p_full[gg%NB] next completes for P_{gg+NB}, which needs
        // S_{gg+NB}, issued only after this wait, so the parity wait is unambiguous.
        if (!warp_wait_poll(&st->p_full[gg % NB], (gg / NB) & 1, abort_flag, p.err_word, kErrAttnMmaWait) ||
            !warp_wait_poll(&st->v_full[s], (gg / NB) & 1, abort_flag, p.err_word, kErrAttnMmaWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t vd = smem_desc_sw128(smem_u32(sV + s * LY::KV_BYTES), KCHUNK_BYTES, 1024);
        const uint32_t o_tmem = tmem + NB * TK;
#pragma unroll
        for (int kk = 0; kk < TK / 16; ++kk) {
          // A = P in TMEM (lanes = rows, 2 keys per column): +8 columns per 16 keys.  B = V,
          // MN-major: 64-column d chunks 8 KB apart (LBO), +16 key rows * 128 B per step.  The
          // item's first PV overwrites O, which the softmax warps read out (previous item's
          // epilogue) before they hand over this item's first P.
          const uint32_t a_tmem = tmem + static_cast<uint32_t>((gg % NB) * TK + kk * 8);
          umma_f16_ts_w(o_tmem, a_tmem, vd + (kk * 2048 >> 4), IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit_w(&st->o_done[gg % NB]);  // the only commit of this MMA group
      }
      g += n_kv;
    }
    if (!ok && issued) {
      umma_commit_w(&st->drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&st->drain, 0) && globaltimer_ns() - t0 < 100000000ull) {
      }
    }
  } else if (warp >= 2 && warp <= 5) {
    // ------------------------------------------------------------ softmax + epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // row within the Q tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t o_tmem = tmem + lane_base + NB * TK;
    bool ok = true;
    int g = 0;        // global KV step of the item's first tile
    for (int it = 0; ok; ++it) {
      int b;
      if (!fa_take_item<PERSIST>(st, it, b0, n_items, true, abort_flag, p.err_word, kErrAttnSoftmaxWait, b)) {
        ok = false;
        break;
      }
      if (b < 0) break;
      int qt, unit;
      fa_item(p, b, qt, unit);
      const int n_kv = fa_kv_tiles<TKV>(p, qt);
      const int q0 = qt * TILE;
      const int qrow = q0 + row;
      float m = -INFINITY, l = 0.0f;
      for (int j = 0; j < n_kv; ++j) {
        const int gg = g + j;
        if (!warp_wait_poll(&st->s_full[gg % NB], (gg / NB) & 1, abort_flag, p.err_word, kErrAttnSoftmaxWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // Both 32-column score loads in flight before a single wait.
        uint32_t r[TK / 32][32];
        {
          const uint32_t s_tmem = tmem + lane_base + static_cast<uint32_t>((gg % NB) * TK);
#pragma unroll
          for (int c = 0; c < TK / 32; ++c) tmem_ld32(s_tmem + c * 32, r[c]);
          tmem_wait_ld();
        }
        const int kv0 = j * TK;
        // Keys allowed for this row: k < seq, and k <= qrow when causal.
        const int kmax = p.causal ? min(qrow, p.seq - 1) : p.seq - 1;
        if (kv0 + TK - 1 > kmax) {
#pragma unroll
          for (int e = 0; e < TK; ++e)
            if (kv0 + e > kmax) r[e >> 5][e & 31] = __float_as_uint(-INFINITY);
        }
        // Row max: 8 independent partial maxima fed two scores per 3-input max, in raw score
        // units (scale > 0, so max(s)*scale == max(s*scale)).
        float pm[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) pm[a] = __uint_as_float(r[0][a]);
#pragma unroll
        for (int e = 8; e < TK; e += 2)
          pm[(e >> 1) & 7] = max3(pm[(e >> 1) & 7], __uint_as_float(r[e >> 5][e & 31]),
                                  __uint_as_float(r[(e + 1) >> 5][(e + 1) & 31]));
        const float mx = max3(max3(pm[0], pm[1], pm[2]), max3(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7])) *
                         p.scale_log2;
        // P overwrites S in place.  The last reader of those columns before S_gg was PV_{gg-2},
        // issued before S_gg by the same thread; s_full[gg&1] therefore already covers it.
        const bool need = mx > m + RESCALE_THRESHOLD;
        float factor = 1.0f;
        if (need) {
          factor = (m == -INFINITY) ? 0.0f : exp2f(m - mx);
          l *= factor;
          m = mx;
        }
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          // O is rescaled in place: PV_{gg-1} must have landed first.
          if (!warp_wait_poll(&st->o_done[(gg - 1) % NB], ((gg - 1) / NB) & 1, abort_flag, p.err_word,
                              kErrAttnCorrectionWait)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < D; c += 16) {
            uint32_t o[16];
            tmem_ld16(o_tmem + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * factor);
            tmem_st16(o_tmem + c, o);
          }
          tmem_wait_st();
        }
        // p = exp2(s*scale - m), one FFMA + ex2 each; m is finite here (key 0 <= qrow is always
        // visible, so the first tile sets it).  Packed partial sums keep the adds independent.
        const uint64_t sc2 = pk2(p.scale_log2, p.scale_log2), nm2 = pk2(-m, -m);
        uint64_t ps2[4] = {0, 0, 0, 0};
        const uint32_t p_tmem = tmem + lane_base + static_cast<uint32_t>((gg % NB) * TK);
#pragma unroll
        for (int gq = 0; gq < TK / 32; ++gq) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int e = gq * 32 + 2 * i;
            // x = s*scale - m for two scores at once; masked scores are -inf, so ex2 gives 0.
            float x0, x1;
            unpk2(fma2(pk2(__uint_as_float(r[e >> 5][e & 31]), __uint_as_float(r[(e + 1) >> 5][(e + 1) & 31])),
                       sc2, nm2),
                  x0, x1);
            const float e0 = fast_exp2(x0), e1 = fast_exp2(x1);
            ps2[i & 3] = add2(ps2[i & 3], pk2(e0, e1));
            w[i] = pack_bf16x2(e0, e1);
          }
          tmem_st16(p_tmem + gq * 16, w);
        }
        float sum;
        {
          const uint64_t t = add2(add2(ps2[0], ps2[1]), add2(ps2[2], ps2[3]));
          float a, c;
          unpk2(t, a, c);
          sum = a + c;
        }
        l += sum;
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&st->p_full[gg % NB]);
      }
      if (!ok) break;
      // The last two PVs (one per P buffer) must have landed in O.  The next completion of either
      // barrier needs a P of the next item, which these warps have not handed over yet.
      const int gl = g + n_kv - 1;
      if (n_kv >= 2)
        ok = warp_wait_poll(&st->o_done[(gl - 1) % NB], ((gl - 1) / NB) & 1, abort_flag, p.err_word,
                            kErrAttnCorrectionWait);
      if (ok)
        ok = warp_wait_poll(&st->o_done[gl % NB], (gl / NB) & 1, abort_flag, p.err_word, kErrAttnCorrectionWait);
      if (!ok) break;
      tc_fence_after();
      const float inv = 1.0f / l;
      // O / l (+ postprocess) as bf16 pairs, 32 columns at a time, into a 128-byte-swizzled
      // [128 rows x 64 cols] box (16-byte chunk k of row r at chunk k ^ (r & 7): conflict-free).
      auto stage32 = [&](int c, uint8_t* box) {
        uint32_t rr[32];
        tmem_ld32(o_tmem + c, rr);
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float y0 = __uint_as_float(rr[2 * e]) * inv, y1 = __uint_as_float(rr[2 * e + 1]) * inv;
          if (p.post) {
            y0 = y0 * p.post_scale + p.post_bias;
            y1 = y1 * p.post_scale + p.post_bias;
            if (p.post_relu) {
              y0 = fmaxf(y0, 0.0f);
              y1 = fmaxf(y1, 0.0f);
            }
          }
          w[e] = pack_bf16x2(y0, y1);
        }
        uint8_t* srow = box + row * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int ch = ((c & 63) >> 3) + i;
          *reinterpret_cast<uint4*>(srow + ((ch ^ (row & 7)) << 4)) =
              make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      };
      if constexpr (!PERSIST) {
        // The Q buffer is idle (every S MMA completed before the last P.V): stage the whole tile
        // there and write it with one TMA store per 64-column box.  Rows past the sequence end
        // are clipped by the tensor map.
#pragma unroll
        for (int c = 0; c < D; c += 32) stage32(c, sQ + (c >> 6) * CHUNK_BYTES);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&st->o_staged);
        if (warp == 2 && lane == 0 &&
            mbar_wait_bounded(&st->o_staged, 0, abort_flag, p.err_word, kErrAttnCorrectionWait)) {
          for (int c = 0; c < NCH; ++c) tma_store_3d(&map_o, sQ + c * CHUNK_BYTES, c * 64, q0, unit);
          bulk_commit_group();
          bulk_wait_group_read0();  // shared memory must outlive the store's reads
        }
      } else {
        // Straight from registers: each thread writes its own row (256 contiguous bytes at
        // head_dim 128) with 16-byte stores that nothing waits for, so these warps go on to the
        // next item's scores at once.  tcgen05.ld is warp-collective, so every lane loads and
        // only the stores of rows past the sequence end are skipped.
        uint4* orow = reinterpret_cast<uint4*>(p.out + (static_cast<size_t>(unit) * p.seq + qrow) * D);
        const bool row_ok = qrow < p.seq;
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          uint32_t rr[32];
          tmem_ld32(o_tmem + c, rr);
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float y0 = __uint_as_float(rr[2 * e]) * inv, y1 = __uint_as_float(rr[2 * e + 1]) * inv;
            if (p.post) {
              y0 = y0 * p.post_scale + p.post_bias;
              y1 = y1 * p.post_scale + p.post_bias;
              if (p.post_relu) {
                y0 = fmaxf(y0, 0.0f);
                y1 = fmaxf(y1, 0.0f);
              }
            }
            w[e] = pack_bf16x2(y0, y1);
          }
          if (row_ok)
#pragma unroll
            for (int i = 0; i < 4; ++i)
              orow[c / 8 + i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
        tc_fence_before();  // these reads of O are ordered before the next item's first P hand-off
      }
      g += n_kv;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (PERSIST && threadIdx.x == 0) {
    // Every fetch of this CTA precedes this count, so the last CTA to finish can zero both words
    // for the next launch that uses this counter slot.
    __threadfence();
    if (atomicAdd(p.sched + 1, 1u) == gridDim.x - 1) {
      atomicExch(p.sched, 0u);
      atomicExch(p.sched + 1, 0u);
    }
  }
}

// ---- two Q tiles per CTA, 128-key tiles (head_dim 128) -------------------------------------
// One CTA per SM owns two 128-row Q tiles (A: rows q0..q0+127, B: q0+128..q0+255) of one unit,
// which share every K/V tile.  KV tiles are 128 keys, so S = Q K^T runs as M=128 N=128 K=16
// MMAs (operands 8 KB per MMA: the full tensor rate; 64-key tiles are bound by the 6 KB
// shared-memory operand traffic of an N=64 MMA).  TMEM (all 512 columns): S_A 0, S_B 128,
// O_A 256, O_B 384; P_h (bf16 pairs) overwrites the first 64 columns of S_h.  The MMA warp
// alternates the tiles: PV_A(j), S_A(j+1), PV_B(j), S_B(j+1), so each softmax warpgroup works on
// its tile while the tensor core serves the other one.
//   warp 0      TMA: Q_A, Q_B once, then K_j and V_j into 2-stage rings (freed by S_B(j) and
//               PV_B(j), the last reader of each).
//   warp 1      MMA issue (one thread).
//   warps 2..5  softmax + epilogue of tile A; warps 6..9 of tile B.
namespace q2 {
constexpr int D = 128;
constexpr int KT = 128;
constexpr int NCH = 2;                       // 64-column chunks per 128-column row
constexpr int CH = 128 * 128;                // one [128 rows x 64 bf16] swizzled box = 16 KB
constexpr int TILE_BYTES = NCH * CH;         // 32 KB: a Q tile, a K tile or a V tile
constexpr int Q_OFF = 0;                     // Q_A, Q_B
constexpr int K_OFF = 2 * TILE_BYTES;        // 2 stages
constexpr int V_OFF = K_OFF + 2 * TILE_BYTES;
constexpr int TAIL_OFF = V_OFF + 2 * TILE_BYTES;
constexpr int THREADS = 320;
constexpr int kPolyPairsOf8 = 2;  // exp2 pairs (of every 8) computed on the FMA pipes
struct Tail {
  uint64_t q_full[2];
  uint64_t k_full[2], v_full[2];
  uint64_t k_free[2], v_free[2];  // stage free: S_B(j) / PV_B(j) done (one commit each)
  uint64_t s_full[2];             // [tile]: S_h(j) in TMEM
  uint64_t p_full[2];             // [tile]: P_h(j) in TMEM (4 warp arrivals)
  uint64_t o_done[2];             // [tile]: PV_h(j) done
  uint64_t o_staged[2];           // [tile]: bf16 O staged in Q_h (4 warp arrivals)
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
constexpr size_t SMEM = 1024 + TAIL_OFF + sizeof(Tail);
}  // namespace q2

__global__ void __launch_bounds__(q2::THREADS, 1)
    fa2q_fwd_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_o,
                    const FaParams p) {
  using namespace q2;
  extern __shared__ __align__(16) uint8_t smem_raw2[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw2) + 1023) & ~uintptr_t(1023));
  Tail* st = reinterpret_cast<Tail*>(smem + TAIL_OFF);
  auto sQ = [&](int h) { return smem + Q_OFF + h * TILE_BYTES; };
  auto sK = [&](int s) { return smem + K_OFF + s * TILE_BYTES; };
  auto sV = [&](int s) { return smem + V_OFF + s * TILE_BYTES; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nq2 = (p.seq + 2 * 128 - 1) / (2 * 128);
  int qt, unit;  // groups of p.group units, heaviest tile pairs of a group first
  {
    const int b = static_cast<int>(blockIdx.x);
    const int per_group = p.group * nq2;
    const int g = b / per_group, r = b % per_group;
    const int gu = min(p.group, p.units - g * p.group);
    qt = nq2 - 1 - r / gu;
    unit = g * p.group + r % gu;
  }
  const int q0 = qt * 256;
  const int kv_all = (p.seq + KT - 1) / KT;
  int n_t[2];
  n_t[0] = p.causal ? min(kv_all, (q0 + 127) / KT + 1) : kv_all;
  n_t[1] = p.causal ? min(kv_all, (q0 + 255) / KT + 1) : kv_all;
  const int nA = n_t[0], nB = n_t[1];  // nB >= nA

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&st->q_full[b], 1);
      mbar_init(&st->k_full[b], 1);
      mbar_init(&st->v_full[b], 1);
      mbar_init(&st->k_free[b], 1);
      mbar_init(&st->v_free[b], 1);
      mbar_init(&st->s_full[b], 1);
      mbar_init(&st->p_full[b], 4);
      mbar_init(&st->o_done[b], 1);
      mbar_init(&st->o_staged[b], 4);
    }
    mbar_init(&st->drain, 1);
    st->abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_v);
    tma_prefetch_desc(&map_o);
    for (int h = 0; h < 2; ++h) {
      mbar_arrive_expect_tx(&st->q_full[h], TILE_BYTES);
      load_rows(sQ(h), &map_q, NCH, CH, q0 + h * 128, unit, &st->q_full[h]);
    }
  }
  if (warp == 0) {
    tmem_alloc(&st->tmem_base, 512);
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
    // ------------------------------------------------------------ TMA producer: K and V
    if (lane == 0) {
      bool ok = true;
      int k_issued = 0, v_issued = 0;
      for (int j = 0; j < nB && ok; ++j) {
        const int s = j & 1;
        // Stage s last held tile j-2, whose last readers are S_B(j-2) and PV_B(j-2); the next
        // completion of k_free[s] / v_free[s] needs tile j, loaded here, so the waits are
        // unambiguous.  PV_B(j-2) precedes S_B(j-1) in the MMA stream, so V never holds back K.
        if (j >= 2 && !mbar_wait_bounded(&st->k_free[s], ((j - 2) >> 1) & 1, abort_flag, p.err_word, kErrAttnLoadWait)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&st->k_full[s], TILE_BYTES);
        load_rows(sK(s), &map_k, NCH, CH, j * KT, unit, &st->k_full[s]);
        ++k_issued;
        if (j >= 2 && !mbar_wait_bounded(&st->v_free[s], ((j - 2) >> 1) & 1, abort_flag, p.err_word, kErrAttnLoadWait)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&st->v_full[s], TILE_BYTES);
        load_rows(sV(s), &map_v, NCH, CH, j * KT, unit, &st->v_full[s]);
        ++v_issued;
        if (j + 2 < nB)
          for (int c = 0; c < NCH; ++c) {
            tma_prefetch_l2_3d(&map_k, c * 64, (j + 2) * KT, unit);
            tma_prefetch_l2_3d(&map_v, c * 64, (j + 2) * KT, unit);
          }
      }
      if (!ok) {
        drain(&st->q_full[0], 0);
        drain(&st->q_full[1], 0);
        for (int j = k_issued > 2 ? k_issued - 2 : 0; j < k_issued; ++j) drain(&st->k_full[j & 1], (j >> 1) & 1);
        for (int j = v_issued > 2 ? v_issued - 2 : 0; j < v_issued; ++j) drain(&st->v_full[j & 1], (j >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the issue loop and one elected lane issues each MMA, with the
    // descriptors advanced by constant adds: beside eight busy softmax warps, a loop run by lane
    // 0 alone issues several times slower.
    {
      constexpr uint32_t IDESC_S = idesc_bf16_f32(128, KT, 0, 0);  // Q K-major, K K-major
      constexpr uint32_t IDESC_O = idesc_bf16_f32(128, D, 0, 1);   // P (TMEM) K-major, V MN-major
      bool ok = true, issued = false;
      auto wait = [&](uint64_t* bar, uint32_t ph) -> bool {
        return warp_wait_poll(bar, ph, abort_flag, p.err_word, kErrAttnMmaWait);
      };
      auto issue_s = [&](int h, int j) {
        const uint64_t qd = smem_desc_sw128(smem_u32(sQ(h)), 16, 1024);
        const uint64_t kd = smem_desc_sw128(smem_u32(sK(j & 1)), 16, 1024);
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(h * 128);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t o16 = ((kk >> 2) * CH + (kk & 3) * 32) >> 4;  // address field: bytes / 16
          umma_f16_ss_w(d_tmem, qd + o16, kd + o16, IDESC_S, kk > 0 ? 1u : 0u);
        }
        issued = true;
        umma_commit_w(&st->s_full[h]);
      };
      auto issue_pv = [&](int h, int j) {
        const uint64_t vd = smem_desc_sw128(smem_u32(sV(j & 1)), CH, 1024);
        const uint32_t o_tmem = tmem + 256 + static_cast<uint32_t>(h * 128);
        const uint32_t a_tmem = tmem + static_cast<uint32_t>(h * 128);
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk) {
          // A = P_h in TMEM (2 keys per column, +8 columns per 16 keys); B = V MN-major, the two
          // 64-column d chunks 16 KB apart (LBO), +16 key rows * 128 B per step.
          umma_f16_ts_w(o_tmem, a_tmem + kk * 8, vd + (kk * 2048 >> 4), IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit_w(&st->o_done[h]);
      };
      ok = wait(&st->q_full[0], 0) && wait(&st->k_full[0], 0);
      if (ok) issue_s(0, 0);
      if (ok) ok = wait(&st->q_full[1], 0);
      if (ok) {
        issue_s(1, 0);
        umma_commit_w(&st->k_free[0]);
      }
      for (int j = 0; j < nB && ok; ++j) {
        const int s = j & 1;
        const uint32_t par = (j >> 1) & 1;
        // p_full[h] next completes for P_h(j+1), which needs S_h(j+1), issued after this wait.
        if (!wait(&st->v_full[s], par)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (j < nA) {
          if (!wait(&st->p_full[0], j & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(0, j);
          if (j + 1 < nA) {
            if (!wait(&st->k_full[(j + 1) & 1], ((j + 1) >> 1) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(0, j + 1);
          }
        }
        if (!wait(&st->p_full[1], j & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_pv(1, j);
        umma_commit_w(&st->v_free[s]);
        if (j + 1 < nB) {
          if (!(j + 1 < nA) && !wait(&st->k_full[(j + 1) & 1], ((j + 1) >> 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(1, j + 1);
          umma_commit_w(&st->k_free[(j + 1) & 1]);
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
    // ------------------------------------------------------------ softmax + epilogue of tile h
    const int h = warp >= 6 ? 1 : 0;
    const int n = n_t[h];
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int qrow = q0 + h * 128 + row;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_tmem = tmem + lane_base + static_cast<uint32_t>(h * 128);
    const uint32_t o_tmem = tmem + lane_base + 256 + static_cast<uint32_t>(h * 128);
    const int kmax = p.causal ? min(qrow, p.seq - 1) : p.seq - 1;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      // s_full[h] next completes for S_h(j+1), which needs P_h(j) from these warps first.
      if (!warp_wait_poll(&st->s_full[h], j & 1, abort_flag, p.err_word, kErrAttnSoftmaxWait)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(s_tmem + c * 32, r[c]);
      tmem_wait_ld();
      const int kv0 = j * KT;
      if (kv0 + KT - 1 > kmax) {
#pragma unroll
        for (int e = 0; e < KT; ++e)
          if (kv0 + e > kmax) r[e >> 5][e & 31] = __float_as_uint(-INFINITY);
      }
      float pm[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) pm[a] = __uint_as_float(r[0][a]);
#pragma unroll
      for (int e = 8; e < KT; e += 2)
        pm[(e >> 1) & 7] = max3(pm[(e >> 1) & 7], __uint_as_float(r[e >> 5][e & 31]),
                                __uint_as_float(r[(e + 1) >> 5][(e + 1) & 31]));
      const float mx = max3(max3(pm[0], pm[1], pm[2]), max3(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7])) *
                       p.scale_log2;
      const bool need = mx > m + RESCALE_THRESHOLD;
      float factor = 1.0f;
      if (need) {
        factor = (m == -INFINITY) ? 0.0f : exp2f(m - mx);
        l *= factor;
        m = mx;
      }
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O_h is rescaled in place: PV_h(j-1) must have landed (o_done[h] next completes for
        // PV_h(j), which needs this tile's P).
        if (!warp_wait_poll(&st->o_done[h], (j - 1) & 1, abort_flag, p.err_word, kErrAttnCorrectionWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D; c += 16) {
          uint32_t o[16];
          tmem_ld16(o_tmem + c, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * factor);
          tmem_st16(o_tmem + c, o);
        }
        tmem_wait_st();
      }
      // P_h(j) over the first 64 columns of S_h(j) (all of S_h(j) is in registers already).
      const uint64_t sc2 = pk2(p.scale_log2, p.scale_log2), nm2 = pk2(-m, -m);
      uint64_t ps2[4] = {0, 0, 0, 0};
#pragma unroll
      for (int g = 0; g < KT / 32; ++g) {
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float x0, x1;
          unpk2(fma2(pk2(__uint_as_float(r[g][2 * i]), __uint_as_float(r[g][2 * i + 1])), sc2, nm2), x0, x1);
          // Two pairs in eight go to the FMA pipes, the rest to MUFU ex2 (measured best of 0, 2,
          // 3, 4 and 8 in eight: 0.251, 0.248, -, 0.272, 0.323 ms non-causal [128, 2048, 128]).
          float e0, e1;
          if ((i & 7) < kPolyPairsOf8) {
            exp2_poly_pair(x0, x1, e0, e1);
          } else {
            e0 = fast_exp2(x0);
            e1 = fast_exp2(x1);
          }
          ps2[i & 3] = add2(ps2[i & 3], pk2(e0, e1));
          w[i] = pack_bf16x2(e0, e1);
        }
        tmem_st16(s_tmem + g * 16, w);
      }
      {
        const uint64_t t = add2(add2(ps2[0], ps2[1]), add2(ps2[2], ps2[3]));
        float a, b;
        unpk2(t, a, b);
        l += a + b;
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&st->p_full[h]);
    }
    if (ok && warp_wait_poll(&st->o_done[h], (n - 1) & 1, abort_flag, p.err_word, kErrAttnCorrectionWait)) {
      tc_fence_after();
      // Epilogue: O / l (+ postprocess) as bf16 into Q_h (no MMA reads it any more: S_h(n-1)
      // completed before PV_h(n-1)), 128-byte-swizzled, then TMA stores clipped at seq.
      const float inv = 1.0f / l;
      uint8_t* sq = sQ(h);
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        uint32_t r[32];
        tmem_ld32(o_tmem + c, r);
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float y0 = __uint_as_float(r[2 * e]) * inv, y1 = __uint_as_float(r[2 * e + 1]) * inv;
          if (p.post) {
            y0 = y0 * p.post_scale + p.post_bias;
            y1 = y1 * p.post_scale + p.post_bias;
            if (p.post_relu) {
              y0 = fmaxf(y0, 0.0f);
              y1 = fmaxf(y1, 0.0f);
            }
          }
          w[e] = pack_bf16x2(y0, y1);
        }
        uint8_t* srow = sq + (c >> 6) * CH + row * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int ch = ((c & 63) >> 3) + i;
          *reinterpret_cast<uint4*>(srow + ((ch ^ (row & 7)) << 4)) =
              make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&st->o_staged[h]);
      // A tile wholly past the sequence end (short sequences) is never stored.
      if ((warp & 3) == 2 && lane == 0 && q0 + h * 128 < p.seq &&
          mbar_wait_bounded(&st->o_staged[h], 0, abort_flag, p.err_word, kErrAttnCorrectionWait)) {
        for (int c = 0; c < NCH; ++c) tma_store_3d(&map_o, sq + c * CH, c * 64, q0 + h * 128, unit);
        bulk_commit_group();
        bulk_wait_group_read0();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [units, seq, d] bf16, box [1, 128, 64], 128-byte swizzle, zero fill past seq.
bool make_tmap_heads(CUtensorMap* map, const void* base, int units, int seq, int d, int box_rows) {
  auto enc = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!enc) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(seq), static_cast<cuuint64_t>(units)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(d) * 2, static_cast<cuuint64_t>(seq) * d * 2};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


cudaError_t launch_fa2q(const AttnArgs& a, cudaStream_t s) {
  DeviceCtx* ctx = device_ctx();
  if (!ctx) return cudaErrorNoDevice;
  CUtensorMap mq, mk, mv, mo;
  if (!make_tmap_heads(&mq, a.q, a.units, a.seq, q2::D, 128) || !make_tmap_heads(&mk, a.k, a.units, a.seq, q2::D, 128) ||
      !make_tmap_heads(&mv, a.v, a.units, a.seq, q2::D, 128) || !make_tmap_heads(&mo, a.out, a.units, a.seq, q2::D, 128))
    return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> attr_done{0};  // devices with the attributes set
  {
    const cudaError_t ea = once_per_device(attr_done, [&]() -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(fa2q_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(q2::SMEM));
      if (e != cudaSuccess) return e;
      return cudaSuccess;
    });
    if (ea != cudaSuccess) return ea;
  }
  FaParams p;
  p.sched = nullptr;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.units = a.units;
  p.seq = a.seq;
  p.nq = (a.seq + 255) / 256;
  p.causal = a.causal;
  p.group = kUnitGroup;
  p.scale_log2 = a.scale * LOG2E;
  p.post_scale = a.post_scale;
  p.post_bias = a.post_bias;
  p.post_relu = a.post_relu;
  p.post = !(a.post_scale == 1.0f && a.post_bias == 0.0f && !a.post_relu);
  p.err_word = ctx->err_word;
  const long long blocks = static_cast<long long>(p.nq) * a.units;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  fa2q_fwd_kernel<<<static_cast<unsigned>(blocks), q2::THREADS, q2::SMEM, s>>>(mq, mk, mv, mo, p);
  return cudaGetLastError();
}


template <int D, bool PERSIST, int TKV = 64>
cudaError_t launch_fa(const AttnArgs& a, cudaStream_t s) {
  DeviceCtx* ctx = device_ctx();
  if (!ctx) return cudaErrorNoDevice;
  CUtensorMap mq, mk, mv, mo;
  if (!make_tmap_heads(&mq, a.q, a.units, a.seq, D, TILE) || !make_tmap_heads(&mk, a.k, a.units, a.seq, D, TKV) ||
      !make_tmap_heads(&mv, a.v, a.units, a.seq, D, TKV) || !make_tmap_heads(&mo, a.out, a.units, a.seq, D, TILE))
    return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> attr_done{0};  // devices with the attributes set
  {
    const cudaError_t ea = once_per_device(attr_done, [&]() -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(fa_fwd_kernel<D, PERSIST, TKV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(Layout<D, TKV>::SMEM));
      if (e != cudaSuccess) return e;
      e = cudaFuncSetAttribute(fa_fwd_kernel<D, PERSIST, TKV>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
      if (e != cudaSuccess) return e;
      return cudaSuccess;
    });
    if (ea != cudaSuccess) return ea;
  }
  FaParams p;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.units = a.units;
  p.seq = a.seq;
  p.nq = (a.seq + TILE - 1) / TILE;
  p.causal = a.causal;
  p.group = kUnitGroup;
  p.scale_log2 = a.scale * LOG2E;
  p.post_scale = a.post_scale;
  p.post_bias = a.post_bias;
  p.post_relu = a.post_relu;
  p.post = !(a.post_scale == 1.0f && a.post_bias == 0.0f && !a.post_relu);
  p.err_word = ctx->err_word;
  p.sched = PERSIST ? ctx->take_sched() : nullptr;
  const long long items = static_cast<long long>(p.nq) * a.units;
  if (items > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  // Persistent form: two resident CTAs per SM.
  const long long blocks = PERSIST ? std::min<long long>(items, 2LL * std::max(ctx->sm_count, 1)) : items;
  fa_fwd_kernel<D, PERSIST, TKV><<<static_cast<unsigned>(blocks), NUM_THREADS, Layout<D, TKV>::SMEM, s>>>(
      mq, mk, mv, mo, p);
  return cudaGetLastError();
}

}  // namespace

bool attention_bf16_tc_supported(const AttnArgs& a) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const long long hs = static_cast<long long>(a.seq) * a.d;
  return (a.d == 64 || a.d == 128) && a.proj_w == nullptr && a.q_unit_stride == hs && a.k_unit_stride == hs &&
         a.v_unit_stride == hs && a.out_unit_stride == hs && al(a.q) && al(a.k) && al(a.v) && al(a.out) &&
         tensor_map_encoder() != nullptr;
}

cudaError_t attention_bf16_by_name(const AttnArgs& a, const std::string& name, cudaStream_t s) {
  if (name == kAttnTc2qName) {
    if (!attention_bf16_tc_supported(a) || a.d != 128) return cudaErrorNotSupported;
    return launch_fa2q(a, s);
  }
  if (name == kAttnTc1qName) {
    if (!attention_bf16_tc_supported(a)) return cudaErrorNotSupported;
    return a.d == 64 ? launch_fa<64, false>(a, s) : launch_fa<128, false>(a, s);
  }
  if (name == kAttnTc1qPName) {
    if (!attention_bf16_tc_supported(a)) return cudaErrorNotSupported;
    return a.d == 64 ? launch_fa<64, true>(a, s) : launch_fa<128, true>(a, s);
  }
  if (name == "simt") return attention_bf16_simt(a, s);
  return cudaErrorInvalidValue;
}

cudaError_t attention_bf16(const AttnArgs& a, cudaStream_t s) {
  std::string cfg;
  const bool forced_simt =
      tune_lookup(LC_TUNE_ATTENTION, a.seq, a.d, a.causal, LC_DTYPE_BF16, &cfg) && cfg == "simt";
  if (!forced_simt && attention_bf16_tc_supported(a)) {
    // Two Q tiles per CTA for head_dim 128 without a causal mask (0.248 vs 0.264 ms at
    // [128, 2048, 128]); causal stays on the one-tile kernel, whose 64-key diagonal tiles
    // waste less (0.153 vs 0.164 ms), with one CTA per Q tile (the persistent form measured
    // 0.154-0.156 ms at config 3).  The tune cache can pin any of the three.
    if (cfg == kAttnTc1qName) return a.d == 64 ? launch_fa<64, false>(a, s) : launch_fa<128, false>(a, s);
    if (cfg == kAttnTc1qPName) return a.d == 64 ? launch_fa<64, true>(a, s) : launch_fa<128, true>(a, s);
    if (a.d == 128 && (cfg == kAttnTc2qName || !a.causal)) return launch_fa2q(a, s);
    return a.d == 64 ? launch_fa<64, false>(a, s) : launch_fa<128, false>(a, s);
  }
  return attention_bf16_simt(a, s);
}

}  // namespace lcb
