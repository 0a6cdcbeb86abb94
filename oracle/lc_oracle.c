/* Test infrastructure only -- NOT the product path.  See lc_oracle.h.
 *
 * Plain-C restatement of the reference CPU path.  Arithmetic order follows the reference so
 * that results agree to fp32 rounding (the reference is built with -ffast-math, which may
 * re-associate its inner dot products; agreement is therefore to ~1e-6 relative, not bitwise).
 */
#define _POSIX_C_SOURCE 200809L
#include "lc_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---- attention: src/attention_cpu.cpp:38-101 ------------------------------------------ */

/* One output row i: scores_j = (q_i . k_j) * (1/sqrt(d)), causal j>i -> -1e30 (:55-63);
 * row max, e_j = exp(s_j - max), sum, p_j = e_j * (1/sum) (:67-84); out_i = sum_j p_j v_j (:86-95). */
static void attention_row(const float* q, const float* k, const float* v, float* out_row, float* scores,
                          size_t seq, size_t d, int causal, size_t i) {
  const float scale = 1.0f / sqrtf((float)d);
  const float* qi = q + i * d;
  for (size_t j = 0; j < seq; ++j) {
    if (causal && j > i) {
      scores[j] = -1e30f;
    } else {
      const float* kj = k + j * d;
      float s = 0.0f;
      for (size_t c = 0; c < d; ++c) s += qi[c] * kj[c];
      scores[j] = s * scale;
    }
  }
  float mx = scores[0];
  for (size_t j = 1; j < seq; ++j) mx = scores[j] > mx ? scores[j] : mx;
  float sum = 0.0f;
  for (size_t j = 0; j < seq; ++j) {
    float e = expf(scores[j] - mx);
    scores[j] = e;
    sum += e;
  }
  const float inv = 1.0f / sum;
  for (size_t j = 0; j < seq; ++j) scores[j] *= inv;
  for (size_t c = 0; c < d; ++c) out_row[c] = 0.0f;
  for (size_t j = 0; j < seq; ++j) {
    const float p = scores[j];
    const float* vj = v + j * d;
    for (size_t c = 0; c < d; ++c) out_row[c] += p * vj[c];
  }
}

int orc_attention_rows(const float* q, const float* k, const float* v, float* out_rows, size_t seq, size_t d,
                       int causal, size_t row0, size_t row1) {
  if (!q || !k || !v || !out_rows || seq == 0 || d == 0 || row1 > seq || row0 > row1) return 2;
  float* scores = (float*)malloc(sizeof(float) * seq);
  if (!scores) return 3;
  for (size_t i = row0; i < row1; ++i) attention_row(q, k, v, out_rows + (i - row0) * d, scores, seq, d, causal, i);
  free(scores);
  return 0;
}

/* src/attention.cpp:41-60: identity when scale==1, bias==0, !relu; else max(0?)(x*scale+bias). */
static void postprocess(float* out, size_t n, float scale, float bias, int relu) {
  if (scale == 1.0f && bias == 0.0f && !relu) return;
  for (size_t i = 0; i < n; ++i) {
    float x = out[i] * scale + bias;
    if (relu && x < 0.0f) x = 0.0f;
    out[i] = x;
  }
}

int orc_attention_forward(const float* q, const float* k, const float* v, float* out, size_t seq, size_t d,
                          int causal, float output_scale, float output_bias, int output_relu) {
  /* src/attention.cpp:145-148: null pointers or zero sizes -> kInvalidValue (2). */
  if (!q || !k || !v || !out || seq == 0 || d == 0) return 2;
  int rc = orc_attention_rows(q, k, v, out, seq, d, causal, 0, seq);
  if (rc == 0) postprocess(out, seq * d, output_scale, output_bias, output_relu);
  return rc;
}

typedef struct {
  size_t lo, hi;
  void* ctx;
  int (*fn)(void* ctx, size_t u);
  int rc;
} fan_job;

static void* fan_worker(void* arg) {
  fan_job* j = (fan_job*)arg;
  for (size_t u = j->lo; u < j->hi; ++u) {
    int r = j->fn(j->ctx, u);
    if (r) { j->rc = r; break; }
  }
  return NULL;
}

static int fan_out(size_t units, int threads, void* ctx, int (*fn)(void*, size_t)) {
  if (threads < 1) threads = 1;
  if ((size_t)threads > units) threads = units ? (int)units : 1;
  fan_job jobs[256];
  pthread_t tids[256];
  if (threads > 256) threads = 256;
  size_t per = (units + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    jobs[t].lo = t * per;
    jobs[t].hi = (t + 1) * per < units ? (t + 1) * per : units;
    jobs[t].ctx = ctx;
    jobs[t].fn = fn;
    jobs[t].rc = 0;
    pthread_create(&tids[t], NULL, fan_worker, &jobs[t]);
  }
  int rc = 0;
  for (int t = 0; t < threads; ++t) {
    pthread_join(tids[t], NULL);
    if (jobs[t].rc) rc = jobs[t].rc;
  }
  return rc;
}

typedef struct {
  const float *q, *k, *v;
  float* out;
  size_t seq, d;
  int causal;
} attn_ctx;

static int attn_unit(void* c, size_t u) {
  attn_ctx* a = (attn_ctx*)c;
  size_t s = a->seq * a->d;
  return orc_attention_rows(a->q + u * s, a->k + u * s, a->v + u * s, a->out + u * s, a->seq, a->d, a->causal, 0,
                            a->seq);
}

int orc_attention_units(const float* q, const float* k, const float* v, float* out, size_t units, size_t seq,
                        size_t d, int causal, int threads) {
  attn_ctx c = {q, k, v, out, seq, d, causal};
  return fan_out(units, threads, &c, attn_unit);
}

/* src/attention_cpu.cpp:114-163. */
int orc_attention_train_step(const float* q, const float* k, float* v, const float* target, float* out, float lr,
                             size_t seq, size_t d, int causal, float* loss_out) {
  if (!q || !k || !v || !target || !out || seq == 0 || d == 0) return 2;
  float* probs = (float*)malloc(sizeof(float) * seq * seq);
  float* grad_out = (float*)calloc(seq * d, sizeof(float));
  float* grad_v = (float*)calloc(seq * d, sizeof(float));
  if (!probs || !grad_out || !grad_v) { free(probs); free(grad_out); free(grad_v); return 3; }
  for (size_t i = 0; i < seq; ++i) attention_row(q, k, v, out + i * d, probs + i * seq, seq, d, causal, i);
  float loss = 0.0f;
  const float norm = 1.0f / (float)(seq * d);
  for (size_t i = 0; i < seq * d; ++i) {
    float diff = out[i] - target[i];
    loss += diff * diff;
    grad_out[i] = 2.0f * diff * norm;
  }
  for (size_t j = 0; j < seq; ++j)
    for (size_t i = 0; i < seq; ++i) {
      float p = probs[i * seq + j];
      for (size_t c = 0; c < d; ++c) grad_v[j * d + c] += p * grad_out[i * d + c];
    }
  for (size_t i = 0; i < seq * d; ++i) v[i] -= lr * grad_v[i];
  if (loss_out) *loss_out = loss * norm;
  free(probs); free(grad_out); free(grad_v);
  return 0;
}

/* ---- matmul: src/ops/matmul_cpu.cpp:49-60 --------------------------------------------- */

int orc_matmul(const float* a, const float* b, float* out, size_t m, size_t k, size_t n) {
  if (!a || !b || !out || m == 0 || k == 0 || n == 0) return 2;
  memset(out, 0, sizeof(float) * m * n);
  for (size_t i = 0; i < m; ++i)
    for (size_t p = 0; p < k; ++p) {
      const float av = a[i * k + p];
      const float* brow = b + p * n;
      float* crow = out + i * n;
      for (size_t j = 0; j < n; ++j) crow[j] += av * brow[j];
    }
  return 0;
}

typedef struct {
  const float *a, *b;
  float* out;
  size_t m, k, n, rows;
} mm_ctx;

static int mm_unit(void* c, size_t u) {
  mm_ctx* x = (mm_ctx*)c;
  size_t r0 = u * x->rows;
  if (r0 >= x->m) return 0;
  size_t r = x->m - r0 < x->rows ? x->m - r0 : x->rows;
  return orc_matmul(x->a + r0 * x->k, x->b, x->out + r0 * x->n, r, x->k, x->n);
}

int orc_matmul_threads(const float* a, const float* b, float* out, size_t m, size_t k, size_t n, int threads) {
  if (threads < 1) threads = 1;
  mm_ctx c = {a, b, out, m, k, n, (m + threads - 1) / threads};
  return fan_out((size_t)threads, threads, &c, mm_unit);
}

/* ---- conv: include/lightning_core/core/ops.hpp:855-1212 ------------------------------- */

/* im2col column col = (c*kh + ky)*kw + kx (:1082-1084), out2d = cols x packed_w accumulated in
 * column order (:1184 -> matmul i-p-j), then + bias (null -> 0) and ReLU, scattered to NCHW
 * (:1196-1210).  Out-of-image taps contribute the im2col zero fill. */
int orc_conv2d_nchw(const float* x, const float* w, const float* bias, float* out, size_t batch, size_t in_c,
                    size_t in_h, size_t in_w, size_t out_c, size_t kh, size_t kw, size_t sh, size_t sw, size_t ph,
                    size_t pw, int apply_relu) {
  if (!x || !w || !out || batch == 0 || in_c == 0 || in_h == 0 || in_w == 0 || out_c == 0 || kh == 0 ||
      kw == 0 || sh == 0 || sw == 0)
    return 2;
  if (in_h + 2 * ph < kh || in_w + 2 * pw < kw) return 2;
  const size_t oh = (in_h + 2 * ph - kh) / sh + 1;
  const size_t ow = (in_w + 2 * pw - kw) / sw + 1;
  for (size_t nb = 0; nb < batch; ++nb)
    for (size_t oc = 0; oc < out_c; ++oc)
      for (size_t oy = 0; oy < oh; ++oy)
        for (size_t ox = 0; ox < ow; ++ox) {
          float acc = 0.0f;
          for (size_t c = 0; c < in_c; ++c)
            for (size_t ky = 0; ky < kh; ++ky) {
              const size_t yn = oy * sh + ky;
              for (size_t kx = 0; kx < kw; ++kx) {
                const size_t xn = ox * sw + kx;
                float xv = 0.0f;
                if (yn >= ph && yn - ph < in_h && xn >= pw && xn - pw < in_w)
                  xv = x[((nb * in_c + c) * in_h + (yn - ph)) * in_w + (xn - pw)];
                acc += xv * w[((oc * in_c + c) * kh + ky) * kw + kx];
              }
            }
          float vv = acc + (bias ? bias[oc] : 0.0f);
          if (apply_relu && vv < 0.0f) vv = 0.0f;
          out[((nb * out_c + oc) * oh + oy) * ow + ox] = vv;
        }
  return 0;
}

/* python/bindings/bind_integrated.cpp:707-729. */
void orc_qkv_pack(const float* conv, size_t conv_size, size_t need, float* packed) {
  const size_t total = 3 * need;
  size_t copied = conv_size < total ? conv_size : total;
  memcpy(packed, conv, copied * sizeof(float));
  while (copied < total) {
    size_t chunk = copied < total - copied ? copied : total - copied;
    memcpy(packed + copied, packed, chunk * sizeof(float));
    copied += chunk;
  }
}

typedef struct {
  const float *x, *w, *bias, *proj_w;
  float* out;
  size_t in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, seq, d, proj_cols;
} ca_ctx;

static int ca_unit(void* c, size_t b) {
  ca_ctx* a = (ca_ctx*)c;
  const size_t oh = (a->in_h + 2 * a->ph - a->kh) / a->sh + 1;
  const size_t ow = (a->in_w + 2 * a->pw - a->kw) / a->sw + 1;
  const size_t conv_size = a->out_c * oh * ow;
  const size_t need = a->seq * a->d;
  const size_t out_cols = a->proj_w ? a->proj_cols : a->d;
  float* conv = (float*)malloc(sizeof(float) * conv_size);
  float* packed = (float*)malloc(sizeof(float) * 3 * need);
  float* attn = (float*)malloc(sizeof(float) * need);
  int rc = 3;
  if (conv && packed && attn) {
    rc = orc_conv2d_nchw(a->x + b * a->in_c * a->in_h * a->in_w, a->w, a->bias, conv, 1, a->in_c, a->in_h, a->in_w,
                         a->out_c, a->kh, a->kw, a->sh, a->sw, a->ph, a->pw, 1);
    if (!rc) {
      orc_qkv_pack(conv, conv_size, need, packed);
      rc = orc_attention_rows(packed, packed + need, packed + 2 * need, attn, a->seq, a->d, 0, 0, a->seq);
    }
    if (!rc) {
      if (a->proj_w)
        rc = orc_matmul(attn, a->proj_w, a->out + b * a->seq * out_cols, a->seq, a->d, a->proj_cols);
      else
        memcpy(a->out + b * need, attn, sizeof(float) * need);
    }
  }
  free(conv); free(packed); free(attn);
  return rc;
}

int orc_conv_attention_images(const float* x, const float* w, const float* bias, const float* proj_w, float* out,
                              size_t images, size_t in_c, size_t in_h, size_t in_w, size_t out_c, size_t kh,
                              size_t kw, size_t sh, size_t sw, size_t ph, size_t pw, size_t seq, size_t d,
                              size_t proj_cols, int threads) {
  if (!x || !w || !out || images == 0 || seq == 0 || d == 0) return 2;
  if (in_h + 2 * ph < kh || in_w + 2 * pw < kw || sh == 0 || sw == 0) return 2;
  ca_ctx c = {x, w, bias, proj_w, out, in_c, in_h, in_w, out_c, kh, kw, sh, sw, ph, pw, seq, d, proj_cols};
  return fan_out(images, threads, &c, ca_unit);
}

/* ---- elementwise ----------------------------------------------------------------------- */

void orc_vector_add(const float* a, const float* b, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

void orc_matrix_sub(const float* a, const float* b, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = a[i] - b[i];
}

void orc_matrix_div(const float* a, const float* b, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = a[i] / b[i];
}

/* README.md:2267-2270: mean and population variance over the last axis (numpy computes both
 * in float32 with pairwise sums; accumulated in double here, which is within fp32 rounding). */
void orc_layer_norm(const float* x, float* out, size_t rows, size_t cols, float eps) {
  for (size_t r = 0; r < rows; ++r) {
    const float* xr = x + r * cols;
    double s = 0.0;
    for (size_t c = 0; c < cols; ++c) s += xr[c];
    const double mean = s / (double)cols;
    double v = 0.0;
    for (size_t c = 0; c < cols; ++c) v += (xr[c] - mean) * (xr[c] - mean);
    const double inv = 1.0 / sqrt(v / (double)cols + (double)eps);
    for (size_t c = 0; c < cols; ++c) out[r * cols + c] = (float)((xr[c] - mean) * inv);
  }
}

float orc_bf16_round(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
    u |= 0x00400000u;
  } else {
    u += 0x7fffu + ((u >> 16) & 1u);
  }
  u &= 0xffff0000u;
  float y;
  memcpy(&y, &u, 4);
  return y;
}

void orc_bf16_round_array(const float* x, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = orc_bf16_round(x[i]);
}
