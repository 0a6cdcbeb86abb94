// Host-side internal interface between the C ABI (lc_api.cpp) and the kernel launchers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <string>

namespace lcb {

// Per-device state, created lazily on first use with that device current.
struct DeviceCtx {
  int device = -1;
  int sm_count = 0;
  unsigned* err_word = nullptr;  // device word written by kernels whose bounded waits gave up
  // Work counters of persistent kernels: kSchedSlots pairs of words, zero between launches (each
  // launch's last CTA zeroes its pair).  A launch takes the next pair in turn, so launches in
  // flight at the same time on different streams use different pairs (up to kSchedSlots).
  static constexpr int kSchedSlots = 64;
  unsigned* sched = nullptr;
  std::atomic<unsigned> sched_next{0};
  unsigned* take_sched() { return sched + 2 * (sched_next.fetch_add(1, std::memory_order_relaxed) % kSchedSlots); }
  // Stream-ordered pool for per-call workspaces (the 3xTF32 split planes): a call allocates on its
  // own stream and frees on it after its kernels, so calls on different streams never wait for
  // each other and no lock is held on the launch path.  Freed memory stays cached in the pool.
  cudaMemPool_t pool = nullptr;
};
DeviceCtx* device_ctx();

// Every device allocation of the library goes through these (so a test can make them fail).
cudaError_t device_malloc(void** p, size_t bytes);
// Stream-ordered workspace from the device pool; release with workspace_free on the same stream
// after the kernels that use it.
cudaError_t workspace_alloc(DeviceCtx* ctx, void** p, size_t bytes, cudaStream_t s);
cudaError_t workspace_free(void* p, cudaStream_t s);
// Test hook: when >= 0, the next 1-SM tcgen05 GEMM launch skips the loads of this k-block of its
// first tile (its MMA warp's bounded wait then runs out); consumed by that launch.
int take_gemm_stall_kblock();

// ---- auto-tune cache (tune_cache.cpp); kind: LC_TUNE_MATMUL / LC_TUNE_ATTENTION -------------
bool tune_lookup(int kind, size_t d0, size_t d1, size_t d2, int dtype, std::string* config);
void tune_store(int kind, size_t d0, size_t d1, size_t d2, int dtype, const std::string& config);

// ---- GEMM ---------------------------------------------------------------------------------
// Strict fp32 SIMT GEMM, C[m,n] = A[m,k] B[k,n], row-major.  tile < 0: default for the shape.
cudaError_t gemm_f32_tile(const float* a, const float* b, float* c, int m, int k, int n, int tile, cudaStream_t s);
int simt_tile_count();
const char* simt_tile_name(int tile);
int simt_tile_from_name(const char* name);
// Tuned dispatch: consults the matmul auto-tune cache for (m, k, n, dtype).
cudaError_t gemm_f32(const float* a, const float* b, float* c, int m, int k, int n, cudaStream_t s);
// Strict fp32 on tcgen05 by the 3xTF32 split (gemm_tf32x3.cu): k % 4 == 0, n % 4 == 0, 16-byte
// aligned pointers.
bool gemm_f32_tc_supported(const void* a, const void* b, const void* c, int m, int k, int n);
cudaError_t gemm_f32_3xtf32(const float* a, const float* b, float* c, int m, int k, int n, cudaStream_t s);
constexpr const char* kGemmTf32x3Name = "tcgen05_3xtf32";
// bf16 in, fp32 accumulate, bf16 out.  tcgen05/TMA kernel when k%8==0 && n%8==0 and the
// pointers are 16-byte aligned; otherwise a SIMT kernel with the same arithmetic contract.
cudaError_t gemm_bf16(const __nv_bfloat16* a, const __nv_bfloat16* b, __nv_bfloat16* c, int m, int k, int n,
                      cudaStream_t s);
cudaError_t gemm_bf16_simt(const __nv_bfloat16* a, const __nv_bfloat16* b, __nv_bfloat16* c, int m, int k, int n,
                           cudaStream_t s);
bool gemm_bf16_tc_supported(const void* a, const void* b, const void* c, int m, int k, int n);
// Small-M (m <= 2) matmul as a GEMV streaming B once (gemv.cu); tune-cache name "gemv".
cudaError_t gemv_f32(const float* a, const float* b, float* c, int m, int k, int n, cudaStream_t s);
cudaError_t gemv_bf16(const __nv_bfloat16* a, const __nv_bfloat16* b, __nv_bfloat16* c, int m, int k, int n,
                      cudaStream_t s);
constexpr const char* kGemvName = "gemv";
// The two tcgen05 kernels by their tune-cache names: 1-SM 128x256 tiles, 2-SM (cluster pair) 256x256.
constexpr const char* kGemmTcName = "tcgen05_128x256";
constexpr const char* kGemmTc2Name = "tcgen05_2sm_256x256";
cudaError_t gemm_bf16_tc(const __nv_bfloat16* a, const __nv_bfloat16* b, __nv_bfloat16* c, int m, int k, int n,
                         cudaStream_t s);
cudaError_t gemm_bf16_tc2(const __nv_bfloat16* a, const __nv_bfloat16* b, __nv_bfloat16* c, int m, int k, int n,
                          cudaStream_t s);

// ---- conv ---------------------------------------------------------------------------------
// Implicit-GEMM NCHW conv, fp32 strict; bias may be null.  Output NCHW, so channel blocks of an
// image are the raw [seq, d] slices the integrated pipeline reads as Q/K/V (no layout pass).
cudaError_t conv2d_nchw_f32(const float* x, const float* w, const float* bias, float* out, int batch, int in_c,
                            int in_h, int in_w, int out_c, int kh, int kw, int sh, int sw, int ph, int pw,
                            int relu, cudaStream_t s);
// The SIMT implicit-GEMM conv (never allocates) and the 3xTF32 tensor-core conv (split planes in
// the device's 3xTF32 workspace); conv2d_nchw_f32 picks by size.
cudaError_t conv2d_nchw_f32_simt(const float* x, const float* w, const float* bias, float* out, int batch, int in_c,
                            int in_h, int in_w, int out_c, int kh, int kw, int sh, int sw, int ph, int pw,
                            int relu, cudaStream_t s);
cudaError_t conv2d_nchw_f32_3xtf32(const float* x, const float* w, const float* bias, float* out, int batch, int in_c,
                            int in_h, int in_w, int out_c, int kh, int kw, int sh, int sw, int ph, int pw,
                            int relu, cudaStream_t s);
// Tensor-core conv eligibility (shape limits of the im2col split) and the tune-cache key of a conv
// shape (false: the shape does not fit the key packing and is never cached).
bool conv_tc_eligible(int in_c, int kh, int kw, int out_c);
bool conv_tune_key(size_t batch, size_t in_c, size_t in_h, size_t in_w, size_t out_c, size_t kh, size_t kw,
                   size_t sh, size_t sw, size_t ph, size_t pw, size_t* d0, size_t* d1, size_t* d2);
constexpr const char* kConvTcName = "tcgen05_3xtf32";
// Implicit-GEMM 3xTF32 conv (conv_implicit_sm100.cu): im2col gathered into shared memory by the
// kernel itself; in_channels % 32 == 0, 16 <= out_channels <= 256, out_channels % 16 == 0.
bool conv_implicit_supported(int in_c, int out_c, int kh, int kw);
cudaError_t conv2d_nchw_f32_implicit(const float* x, const float* w, const float* bias, float* out, int batch,
                                     int in_c, int in_h, int in_w, int out_c, int kh, int kw, int sh, int sw, int ph,
                                     int pw, int relu, cudaStream_t s);
constexpr const char* kConvImplicitName = "tcgen05_implicit";
// The integrated pipeline's fused conv epilogue: instead of the NCHW output, each image's flat conv
// output f (= c * OH*OW + pixel) goes to the attention's operands directly -- f < need: Q hi/lo
// planes, need <= f < 2*need: K hi/lo planes (tf32 split, [images, seq, head_dim] contiguous),
// 2*need <= f < 3*need: V unsplit ([images, need]); the rest is unused by the attention.  need must
// be a multiple of OH*OW (whole channels per operand).
struct QkvSplitOut {
  float *q_hi, *q_lo, *k_hi, *k_lo, *v;
  long long need;  // seq * head_dim
};
// True when conv2d_nchw_f32_implicit can write the fused QKV planes for this shape.
bool conv_qkv_split_supported(int batch, int in_c, int in_h, int in_w, int out_c, int kh, int kw, int sh, int sw,
                              int ph, int pw);
cudaError_t conv2d_nchw_f32_implicit_qkv(const float* x, const float* w, const float* bias, int batch, int in_c,
                                         int in_h, int in_w, int out_c, int kh, int kw, int sh, int sw, int ph,
                                         int pw, int relu, const QkvSplitOut& qkv, cudaStream_t s);
// Cyclic repeat of the first `have` floats of src into dst[0, total) (qkv_pack short case).
cudaError_t repeat_fill_f32(const float* src, size_t have, float* dst, size_t total, cudaStream_t s);

// ---- attention ------------------------------------------------------------------------------
struct AttnArgs {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  long long q_unit_stride, k_unit_stride, v_unit_stride, out_unit_stride;  // elements
  int units, seq, d, causal;
  float scale;           // softmax scale (1/sqrt(d))
  float post_scale, post_bias;
  int post_relu;         // out = relu?(out*post_scale + post_bias)
  const float* proj_w;   // optional [d, proj_cols] fused projection (fp32 path only)
  int proj_cols;
  float* lse;            // optional [units, seq] log-sum-exp of the scaled scores (fp32 path only)
};
cudaError_t attention_f32(const AttnArgs& a, cudaStream_t s);
// The SIMT fp32 kernels (any head_dim <= 256, LSE output, fused projection); never allocates.
cudaError_t attention_f32_simt(const AttnArgs& a, cudaStream_t s);
// Strict fp32 attention on tcgen05 by the 3xTF32 split (attention_tf32x3.cu), head_dim 64.
bool attention_f32_tc_supported(const AttnArgs& a);
cudaError_t attention_f32_tc(const AttnArgs& a, cudaStream_t s);
// The 3xTF32 attention on a caller-provided plane workspace [Q_hi | Q_lo | K_hi | K_lo | V^T_hi |
// V^T_lo] (attention_f32_tc_ws_floats) whose Q and K planes are already filled (the fused conv
// epilogue writes them); a.v is the unsplit V.  Same kernel and results as attention_f32_tc.
size_t attention_f32_tc_ws_floats(int units, int seq);
cudaError_t attention_f32_tc_presplit_qk(const AttnArgs& a, float* ws, cudaStream_t s);
// Train step pieces (fp32): dO = 2(O - T)/(seq*d) and per-unit sum of squared errors (double);
// then dV = P^T dO recomputed from Q, K and the forward's LSE, applied as v -= lr * dV in place.
cudaError_t attention_train_grad_out(const float* out, const float* target, float* dout, double* sse, int units,
                                     long long per_unit, cudaStream_t s);
cudaError_t attention_train_dv_update(const float* q, const float* k, float* v, const float* dout, const float* lse,
                                      int units, int seq, int d, int causal, float scale, float lr, cudaStream_t s);
cudaError_t attention_bf16(const AttnArgs& a, cudaStream_t s);
cudaError_t attention_bf16_simt(const AttnArgs& a, cudaStream_t s);
bool attention_bf16_tc_supported(const AttnArgs& a);
// The bf16 tensor-core kernels by their tune-cache names: one 128-row Q tile per CTA with 64-key
// tiles (two CTAs per SM), and two Q tiles per CTA with 128-key tiles (head_dim 128).
constexpr const char* kAttnTc1qName = "tcgen05_1q";
constexpr const char* kAttnTc2qName = "tcgen05_2q";
constexpr const char* kAttnTc1qPName = "tcgen05_1qp";  // one-tile kernel, persistent CTAs
// Strict fp32 attention on tcgen05 (3xTF32) by its tune-cache name.
constexpr const char* kAttnTf32x3Name = "tcgen05_3xtf32";
// Runs one bf16 attention kernel by its tune-cache name ("tcgen05_1q", "tcgen05_2q", "simt")
// without consulting the cache; cudaErrorNotSupported when that kernel cannot take the shape.
cudaError_t attention_bf16_by_name(const AttnArgs& a, const std::string& name, cudaStream_t s);

// ---- elementwise ----------------------------------------------------------------------------
cudaError_t vector_add_f32(const float* a, const float* b, float* out, size_t n, cudaStream_t s);
cudaError_t vector_add_f64(const double* a, const double* b, double* out, size_t n, cudaStream_t s);
// op 0: a - b, op 1: a / b (f64 selects double).
cudaError_t matrix_binary(int op, int f64, const void* a, const void* b, void* out, size_t n, cudaStream_t s);
cudaError_t layer_norm_f32(const float* x, float* out, size_t rows, size_t cols, float eps, cudaStream_t s);

}  // namespace lcb
