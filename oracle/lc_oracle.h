/* Test infrastructure only -- NOT the product path.
 *
 * Plain-C restatement of Lightning Core's CPU path for the attention / matmul2d /
 * conv->attention hot path.  Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may
 * load it, and only as the checker.  Each function cites the reference file:line it restates
 * (paths relative to the reference project root).  Pinned against the reference's own
 * known-answer tests and against fixtures produced by the reference itself compiled from its
 * sources (tests/golden/make_golden.py).
 */
#ifndef LC_ORACLE_H
#define LC_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* src/attention_cpu.cpp:38-101 (+ src/attention.cpp:41-60 postprocess). Single head [seq, d]. */
int orc_attention_forward(const float* q, const float* k, const float* v, float* out, size_t seq, size_t d,
                          int causal, float output_scale, float output_bias, int output_relu);
/* Same arithmetic, only output rows [row0, row1) -- used to sample large heads. */
int orc_attention_rows(const float* q, const float* k, const float* v, float* out_rows, size_t seq, size_t d,
                       int causal, size_t row0, size_t row1);
/* units independent heads [units, seq, d], fanned out over `threads` pthreads. */
int orc_attention_units(const float* q, const float* k, const float* v, float* out, size_t units, size_t seq,
                        size_t d, int causal, int threads);
/* src/attention_cpu.cpp:114-163: forward, MSE vs target, dV = P^T dO, v -= lr * dV. */
int orc_attention_train_step(const float* q, const float* k, float* v, const float* target, float* out, float lr,
                             size_t seq, size_t d, int causal, float* loss_out);

/* src/ops/matmul_cpu.cpp:49-60: C[m,n] = A[m,k] B[k,n], i-p-j order, fp32 accumulate. */
int orc_matmul(const float* a, const float* b, float* out, size_t m, size_t k, size_t n);
int orc_matmul_threads(const float* a, const float* b, float* out, size_t m, size_t k, size_t n, int threads);

/* include/lightning_core/core/ops.hpp:855-1212: NCHW x OIHW (+bias, optional ReLU) -> NCHW,
 * reduction order (c, ky, kx) as the im2col column order. bias may be NULL. */
int orc_conv2d_nchw(const float* x, const float* w, const float* bias, float* out, size_t batch, size_t in_c,
                    size_t in_h, size_t in_w, size_t out_c, size_t kh, size_t kw, size_t sh, size_t sw, size_t ph,
                    size_t pw, int apply_relu);

/* python/bindings/bind_integrated.cpp:707-729: Q/K/V = consecutive flat slices of the conv output,
 * cyclically repeated when the conv output is shorter than 3*need. packed has 3*need floats. */
void orc_qkv_pack(const float* conv, size_t conv_size, size_t need, float* packed);

/* Per image b: conv(x[b]) + ReLU -> qkv_pack -> attention(non-causal) -> optional @proj_w [d, proj_cols]
 * (include/lightning_core/core/graph.hpp:3529-3547). out: [images, seq, proj_w ? proj_cols : d]. */
int orc_conv_attention_images(const float* x, const float* w, const float* bias, const float* proj_w, float* out,
                              size_t images, size_t in_c, size_t in_h, size_t in_w, size_t out_c, size_t kh,
                              size_t kw, size_t sh, size_t sw, size_t ph, size_t pw, size_t seq, size_t d,
                              size_t proj_cols, int threads);

/* src/ops/vector_add_cpu.cpp:13-43 (scalar semantics). */
void orc_vector_add(const float* a, const float* b, float* out, size_t n);
/* src/ops/matrix_elemwise.cpp:8-29: out = a - b / a / b. */
void orc_matrix_sub(const float* a, const float* b, float* out, size_t n);
void orc_matrix_div(const float* a, const float* b, float* out, size_t n);
/* README.md:2267-2270 _layer_norm_np: (x - mean) / sqrt(var + eps), population variance, last axis. */
void orc_layer_norm(const float* x, float* out, size_t rows, size_t cols, float eps);

/* fp32 -> bf16 (round to nearest even, NaN kept quiet), returned as the widened fp32 value. */
float orc_bf16_round(float x);
void orc_bf16_round_array(const float* x, float* out, size_t n);

#ifdef __cplusplus
}
#endif
#endif
