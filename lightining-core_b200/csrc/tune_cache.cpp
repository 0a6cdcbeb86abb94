// Per-shape auto-tune cache, re-keyed to sm_100a kernel configurations.
//
// Behaviour follows the reference's Metal tune caches (src/ops/matmul_metal.mm:416-577,
// src/attention_metal.mm:184-336): an in-memory map from shape to the chosen kernel
// configuration, persisted as CSV with a `#lc_tune_cache,<kind>,2` header and a `#columns,...`
// line; version 1 and 2 files load, a file with an unknown header is ignored as a whole; the file
// path comes from CJ_MATMUL_TUNE_CACHE_FILE / CJ_ATTN_TUNE_CACHE_FILE and is loaded on first use.
// Keys here are (m, k, n, dtype) for matmul, (seq, head_dim, causal, dtype) for attention and the
// packed conv shape (lcConvTuneKey; the reference's conv mode cache, src/ops/conv2d_metal.mm:577-672,
// is keyed on the conv shape the same way);
// values are kernel configuration names ("simt128x128", "tcgen05_128x256", "tcgen05_2q", ...).
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <mutex>
#include <sstream>
#include <string>
#include <tuple>
#include <vector>

#include "lc_host.hpp"
#include "lc_internal.hpp"

namespace lcb {
namespace {

using Key = std::tuple<size_t, size_t, size_t, int>;

struct Cache {
  std::map<Key, std::string> rows;
  bool loaded = false;  // env file consulted
};

std::mutex g_mu;
Cache g_cache[3];

const char* kind_name(int kind) {
  return kind == LC_TUNE_MATMUL ? "matmul" : kind == LC_TUNE_ATTENTION ? "attention" : "conv";
}
const char* env_name(int kind) {
  return kind == LC_TUNE_MATMUL      ? "CJ_MATMUL_TUNE_CACHE_FILE"
         : kind == LC_TUNE_ATTENTION ? "CJ_ATTN_TUNE_CACHE_FILE"
                                     : "CJ_CONV_TUNE_CACHE_FILE";
}
bool kind_ok(int kind) { return kind == LC_TUNE_MATMUL || kind == LC_TUNE_ATTENTION || kind == LC_TUNE_CONV; }
const char* dtype_name(int d) { return d == LC_DTYPE_BF16 ? "bf16" : d == LC_DTYPE_F64 ? "f64" : "f32"; }
int dtype_from(const std::string& s) { return s == "bf16" ? LC_DTYPE_BF16 : s == "f64" ? LC_DTYPE_F64 : LC_DTYPE_F32; }
const char* columns(int kind) {
  return kind == LC_TUNE_MATMUL      ? "#columns,m,k,n,dtype,config"
         : kind == LC_TUNE_ATTENTION ? "#columns,seq,dim,causal,dtype,config"
                                     : "#columns,channels,spatial,geometry,dtype,config";
}

// Comma-separated fields with surrounding blanks removed, so files saved with CRLF line ends or
// padded by hand load the same rows.
std::vector<std::string> split(const std::string& line) {
  std::vector<std::string> out;
  std::stringstream ss(line);
  std::string f;
  while (std::getline(ss, f, ',')) {
    const size_t b = f.find_first_not_of(" \t\r\n");
    const size_t e = f.find_last_not_of(" \t\r\n");
    out.push_back(b == std::string::npos ? std::string() : f.substr(b, e - b + 1));
  }
  return out;
}

// Loads rows into `into`; returns false when the file is missing or its header is unknown.
bool load_file(int kind, const std::string& path, std::map<Key, std::string>& into) {
  std::ifstream in(path);
  if (!in.is_open()) return false;
  std::string line;
  if (!std::getline(in, line)) return false;
  const auto h = split(line);
  if (h.size() != 3 || h[0] != "#lc_tune_cache" || h[1] != kind_name(kind)) return false;
  const int version = std::atoi(h[2].c_str());
  if (version != 1 && version != 2) return false;  // unknown format: drop every row
  std::map<Key, std::string> rows;
  while (std::getline(in, line)) {
    const auto f = split(line);
    if (f.empty() || f[0].empty() || f[0][0] == '#') continue;
    // v2: d0,d1,d2,dtype,config ; v1 (no dtype column): d0,d1,d2,config with dtype f32.
    if (version == 2 && f.size() == 5) {
      rows[Key{std::strtoull(f[0].c_str(), nullptr, 10), std::strtoull(f[1].c_str(), nullptr, 10),
               std::strtoull(f[2].c_str(), nullptr, 10), dtype_from(f[3])}] = f[4];
    } else if (version == 1 && f.size() == 4) {
      rows[Key{std::strtoull(f[0].c_str(), nullptr, 10), std::strtoull(f[1].c_str(), nullptr, 10),
               std::strtoull(f[2].c_str(), nullptr, 10), LC_DTYPE_F32}] = f[3];
    }
  }
  into.swap(rows);
  return true;
}

bool save_file(int kind, const std::string& path, const std::map<Key, std::string>& rows) {
  std::ofstream out(path, std::ios::out | std::ios::trunc);
  if (!out.is_open()) return false;
  out << "#lc_tune_cache," << kind_name(kind) << ",2\n" << columns(kind) << "\n";
  for (const auto& kv : rows)
    out << std::get<0>(kv.first) << "," << std::get<1>(kv.first) << "," << std::get<2>(kv.first) << ","
        << dtype_name(std::get<3>(kv.first)) << "," << kv.second << "\n";
  return out.good();
}

void ensure_env_loaded(int kind) {  // caller holds g_mu
  Cache& c = g_cache[kind];
  if (c.loaded) return;
  c.loaded = true;
  if (const char* p = std::getenv(env_name(kind)))
    if (p[0]) load_file(kind, p, c.rows);
}

void persist_env(int kind) {  // caller holds g_mu
  if (const char* p = std::getenv(env_name(kind)))
    if (p[0]) save_file(kind, p, g_cache[kind].rows);
}

}  // namespace

bool tune_lookup(int kind, size_t d0, size_t d1, size_t d2, int dtype, std::string* config) {
  std::lock_guard<std::mutex> lk(g_mu);
  ensure_env_loaded(kind);
  auto it = g_cache[kind].rows.find(Key{d0, d1, d2, dtype});
  if (it == g_cache[kind].rows.end()) return false;
  *config = it->second;
  return true;
}

void tune_store(int kind, size_t d0, size_t d1, size_t d2, int dtype, const std::string& config) {
  std::lock_guard<std::mutex> lk(g_mu);
  ensure_env_loaded(kind);
  g_cache[kind].rows[Key{d0, d1, d2, dtype}] = config;
  persist_env(kind);
}

// True when a kernel of the candidate just timed recorded an abort in the device error word;
// the word is cleared for the next candidate.
bool candidate_aborted() {
  DeviceCtx* ctx = device_ctx();
  if (!ctx) return false;
  unsigned w = 0;
  if (cudaMemcpy(&w, ctx->err_word, sizeof(w), cudaMemcpyDeviceToHost) != cudaSuccess || w == 0) return false;
  cudaMemset(ctx->err_word, 0, sizeof(unsigned));
  return true;
}

cudaError_t gemm_f32(const float* a, const float* b, float* c, int m, int k, int n, cudaStream_t s) {
  std::string cfg;
  const bool tc_ok = gemm_f32_tc_supported(a, b, c, m, k, n);
  if (tune_lookup(LC_TUNE_MATMUL, m, k, n, LC_DTYPE_F32, &cfg)) {
    if (cfg == kGemvName && m <= 2) return gemv_f32(a, b, c, m, k, n, s);
    if (cfg == kGemmTf32x3Name && tc_ok) return gemm_f32_3xtf32(a, b, c, m, k, n, s);
    return gemm_f32_tile(a, b, c, m, k, n, simt_tile_from_name(cfg.c_str()), s);
  }
  // Untuned: one or two rows are a GEMV over B (a 64x64 SIMT tile would idle 62 of its rows);
  // then the 3xTF32 tensor-core path once there is enough work to cover its pre-pass and
  // launches (measured: 512x64x512 is faster on the SIMT kernel, 1000x516x1004 2x faster here).
  if (m <= 2) return gemv_f32(a, b, c, m, k, n, s);
  if (tc_ok && m >= 256 && n >= 256 && static_cast<long long>(m) * n * k >= (1LL << 26))
    return gemm_f32_3xtf32(a, b, c, m, k, n, s);
  return gemm_f32_tile(a, b, c, m, k, n, -1, s);
}

}  // namespace lcb

using namespace lcb;

extern "C" {

lcError_t lcTuneCacheLoad(lcTuneKind kind, const char* path) {
  if (!kind_ok(kind)) return LC_INVALID_VALUE;
  const char* p = (path && path[0]) ? path : std::getenv(env_name(kind));
  if (!p || !p[0]) return LC_INVALID_VALUE;
  std::map<Key, std::string> rows;
  if (!load_file(kind, p, rows)) return LC_NOT_SUPPORTED;  // missing file or unknown header
  std::lock_guard<std::mutex> lk(g_mu);
  g_cache[kind].loaded = true;
  g_cache[kind].rows.swap(rows);
  return LC_SUCCESS;
}

lcError_t lcTuneCacheSave(lcTuneKind kind, const char* path) {
  if (!kind_ok(kind)) return LC_INVALID_VALUE;
  const char* p = (path && path[0]) ? path : std::getenv(env_name(kind));
  if (!p || !p[0]) return LC_INVALID_VALUE;
  std::lock_guard<std::mutex> lk(g_mu);
  return save_file(kind, p, g_cache[kind].rows) ? LC_SUCCESS : LC_UNKNOWN;
}

lcError_t lcTuneCacheReset(lcTuneKind kind) {
  if (!kind_ok(kind)) return LC_INVALID_VALUE;
  std::lock_guard<std::mutex> lk(g_mu);
  g_cache[kind].rows.clear();
  g_cache[kind].loaded = true;  // a reset cache does not reload the env file behind the caller's back
  return LC_SUCCESS;
}

size_t lcTuneCacheSize(lcTuneKind kind) {
  if (!kind_ok(kind)) return 0;
  std::lock_guard<std::mutex> lk(g_mu);
  ensure_env_loaded(kind);
  return g_cache[kind].rows.size();
}

lcError_t lcTuneCacheGet(lcTuneKind kind, size_t d0, size_t d1, size_t d2, lcDataType dtype, char* config,
                         size_t cap) {
  if (!kind_ok(kind) || !config || cap == 0) return LC_INVALID_VALUE;
  std::string c;
  if (!tune_lookup(kind, d0, d1, d2, dtype, &c)) return LC_NOT_SUPPORTED;
  std::snprintf(config, cap, "%s", c.c_str());
  return LC_SUCCESS;
}

lcError_t lcTuneCacheSet(lcTuneKind kind, size_t d0, size_t d1, size_t d2, lcDataType dtype, const char* config) {
  if (!kind_ok(kind) || !config || !config[0] || std::strchr(config, ','))
    return LC_INVALID_VALUE;
  tune_store(kind, d0, d1, d2, dtype, config);
  return LC_SUCCESS;
}

// Times every kernel configuration that can run the shape on the caller's device buffers
// (1 warm-up + median of 5 CUDA-event samples each, like autoTuneTile in
// src/ops/matmul_metal.mm:1643-1790), records the fastest in the cache and returns its name.
lcError_t lcMatMulAutotune(const void* a, const void* b, void* out, size_t m, size_t k, size_t n, lcDataType dtype,
                           lcStream_t stream, char* best, size_t cap) {
  if (!a || !b || !out || m == 0 || k == 0 || n == 0) return LC_INVALID_VALUE;
  if (dtype != LC_DTYPE_F32 && dtype != LC_DTYPE_BF16) return LC_NOT_SUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  struct Cand {
    std::string name;
    int tile;
  };
  std::vector<Cand> cands;
  if (m <= 2) cands.push_back({kGemvName, -5});
  if (dtype == LC_DTYPE_F32) {
    for (int t = 0; t < simt_tile_count(); ++t) cands.push_back({simt_tile_name(t), t});
    if (gemm_f32_tc_supported(a, b, out, (int)m, (int)k, (int)n)) cands.push_back({kGemmTf32x3Name, -4});
  } else {
    if (gemm_bf16_tc_supported(a, b, out, (int)m, (int)k, (int)n)) {
      cands.push_back({kGemmTcName, -2});
      cands.push_back({kGemmTc2Name, -3});
    }
    cands.push_back({"simt", -1});
  }
  auto run = [&](const Cand& c) -> cudaError_t {
    if (c.tile == -5)
      return dtype == LC_DTYPE_F32
                 ? gemv_f32(static_cast<const float*>(a), static_cast<const float*>(b), static_cast<float*>(out),
                            (int)m, (int)k, (int)n, s)
                 : gemv_bf16(static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b),
                             static_cast<__nv_bfloat16*>(out), (int)m, (int)k, (int)n, s);
    if (dtype == LC_DTYPE_F32 && c.tile == -4)
      return gemm_f32_3xtf32(static_cast<const float*>(a), static_cast<const float*>(b), static_cast<float*>(out),
                             (int)m, (int)k, (int)n, s);
    if (dtype == LC_DTYPE_F32)
      return gemm_f32_tile(static_cast<const float*>(a), static_cast<const float*>(b), static_cast<float*>(out),
                           (int)m, (int)k, (int)n, c.tile, s);
    const auto* A = static_cast<const __nv_bfloat16*>(a);
    const auto* B = static_cast<const __nv_bfloat16*>(b);
    auto* C = static_cast<__nv_bfloat16*>(out);
    if (c.tile == -2) return gemm_bf16_tc(A, B, C, (int)m, (int)k, (int)n, s);
    if (c.tile == -3) return gemm_bf16_tc2(A, B, C, (int)m, (int)k, (int)n, s);
    return gemm_bf16_simt(A, B, C, (int)m, (int)k, (int)n, s);
  };
  cudaEvent_t e0, e1;
  if (cudaEventCreate(&e0) != cudaSuccess) return LC_DRIVER_ERROR;
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    return LC_DRIVER_ERROR;
  }
  double best_ms = 1e30;
  std::string best_name;
  lcError_t st = LC_SUCCESS;
  for (const Cand& c : cands) {
    cudaError_t e = run(c);
    std::vector<float> ms;
    for (int rep = 0; rep < 5 && e == cudaSuccess; ++rep) {
      cudaEventRecord(e0, s);
      e = run(c);
      cudaEventRecord(e1, s);
      if (e == cudaSuccess) e = cudaEventSynchronize(e1);
      float t = 0.f;
      if (e == cudaSuccess) e = cudaEventElapsedTime(&t, e0, e1);
      ms.push_back(t);
    }
    if (e != cudaSuccess) {
      st = from_cuda(e);
      break;
    }
    // A kernel whose bounded wait gave up returns early and would look fastest: drop it.
    if (candidate_aborted()) continue;
    std::sort(ms.begin(), ms.end());
    if (ms[ms.size() / 2] < best_ms) {
      best_ms = ms[ms.size() / 2];
      best_name = c.name;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (st != LC_SUCCESS) return st;
  if (best_name.empty()) return LC_DRIVER_ERROR;  // every candidate gave up a bounded wait
  tune_store(LC_TUNE_MATMUL, m, k, n, dtype, best_name);
  if (best && cap) std::snprintf(best, cap, "%s", best_name.c_str());
  return LC_SUCCESS;
}

// Times every attention kernel that can run the shape on the caller's device buffers ([units,
// seq, head_dim] each, contiguous; 1 warm-up + median of 5 CUDA-event samples), records the fastest
// for (seq, head_dim, causal, dtype) and returns its name: the per-shape mode choice of the
// reference's autoTuneForwardMode (src/attention_metal.mm:1316-1420), over sm_100a kernels.
lcError_t lcAttentionAutotune(const void* q, const void* k, const void* v, void* out, size_t units, size_t seq,
                              size_t head_dim, int causal, lcDataType dtype, lcStream_t stream, char* best,
                              size_t cap) {
  if (!q || !k || !v || !out || units == 0 || seq == 0 || head_dim == 0) return LC_INVALID_VALUE;
  if (dtype != LC_DTYPE_F32 && dtype != LC_DTYPE_BF16) return LC_NOT_SUPPORTED;
  if (units > 65535 || seq > (size_t)INT_MAX || head_dim > 256) return LC_NOT_SUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  AttnArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.out = out;
  a.q_unit_stride = a.k_unit_stride = a.v_unit_stride = a.out_unit_stride = static_cast<long long>(seq * head_dim);
  a.units = static_cast<int>(units);
  a.seq = static_cast<int>(seq);
  a.d = static_cast<int>(head_dim);
  a.causal = causal ? 1 : 0;
  a.scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
  a.post_scale = 1.0f;
  a.post_bias = 0.0f;
  std::vector<std::string> cands;
  if (dtype == LC_DTYPE_F32) {
    if (attention_f32_tc_supported(a)) cands.push_back(kAttnTf32x3Name);
  } else if (attention_bf16_tc_supported(a)) {
    cands.push_back(kAttnTc1qName);
    cands.push_back(kAttnTc1qPName);
    if (head_dim == 128) cands.push_back(kAttnTc2qName);
  }
  cands.push_back("simt");
  auto run = [&](const std::string& c) -> cudaError_t {
    if (dtype == LC_DTYPE_F32) return c == kAttnTf32x3Name ? attention_f32_tc(a, s) : attention_f32_simt(a, s);
    return attention_bf16_by_name(a, c, s);
  };
  cudaEvent_t e0, e1;
  if (cudaEventCreate(&e0) != cudaSuccess) return LC_DRIVER_ERROR;
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    return LC_DRIVER_ERROR;
  }
  double best_ms = 1e30;
  std::string best_name;
  lcError_t st = LC_SUCCESS;
  for (const std::string& c : cands) {
    cudaError_t e = run(c);
    std::vector<float> ms;
    for (int rep = 0; rep < 5 && e == cudaSuccess; ++rep) {
      cudaEventRecord(e0, s);
      e = run(c);
      cudaEventRecord(e1, s);
      if (e == cudaSuccess) e = cudaEventSynchronize(e1);
      float t = 0.f;
      if (e == cudaSuccess) e = cudaEventElapsedTime(&t, e0, e1);
      ms.push_back(t);
    }
    if (e != cudaSuccess) {
      st = from_cuda(e);
      break;
    }
    // A kernel whose bounded wait gave up returns early and would look fastest: drop it.
    if (candidate_aborted()) continue;
    std::sort(ms.begin(), ms.end());
    if (ms[ms.size() / 2] < best_ms) {
      best_ms = ms[ms.size() / 2];
      best_name = c;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (st != LC_SUCCESS) return st;
  if (best_name.empty()) return LC_DRIVER_ERROR;  // every candidate gave up a bounded wait
  tune_store(LC_TUNE_ATTENTION, seq, head_dim, causal ? 1 : 0, dtype, best_name);
  if (best && cap) std::snprintf(best, cap, "%s", best_name.c_str());
  return LC_SUCCESS;
}

lcError_t lcConvTuneKey(size_t batch, size_t in_channels, size_t in_h, size_t in_w, size_t out_channels,
                        size_t kernel_h, size_t kernel_w, size_t stride_h, size_t stride_w, size_t pad_h,
                        size_t pad_w, size_t* d0, size_t* d1, size_t* d2) {
  if (!d0 || !d1 || !d2) return LC_INVALID_VALUE;
  return conv_tune_key(batch, in_channels, in_h, in_w, out_channels, kernel_h, kernel_w, stride_h, stride_w, pad_h,
                       pad_w, d0, d1, d2)
             ? LC_SUCCESS
             : LC_NOT_SUPPORTED;
}

lcError_t lcConvAutotune(const float* x, const float* w, const float* bias, float* out, size_t batch,
                         size_t in_channels, size_t in_h, size_t in_w, size_t out_channels, size_t kernel_h,
                         size_t kernel_w, size_t stride_h, size_t stride_w, size_t pad_h, size_t pad_w,
                         int apply_relu, lcStream_t stream, char* best, size_t cap) {
  if (!x || !w || !out || batch == 0 || in_channels == 0 || in_h == 0 || in_w == 0 || out_channels == 0 ||
      kernel_h == 0 || kernel_w == 0 || stride_h == 0 || stride_w == 0 || in_h + 2 * pad_h < kernel_h ||
      in_w + 2 * pad_w < kernel_w)
    return LC_INVALID_VALUE;
  if (!conv_dims_fit_int(in_channels, in_h, in_w, out_channels, kernel_h, kernel_w, stride_h, stride_w, pad_h, pad_w))
    return LC_NOT_SUPPORTED;
  const size_t oh = (in_h + 2 * pad_h - kernel_h) / stride_h + 1, ow = (in_w + 2 * pad_w - kernel_w) / stride_w + 1;
  if (batch * oh * ow > (size_t)INT_MAX) return LC_NOT_SUPPORTED;
  size_t d0, d1, d2;
  if (!conv_tune_key(batch, in_channels, in_h, in_w, out_channels, kernel_h, kernel_w, stride_h, stride_w, pad_h,
                     pad_w, &d0, &d1, &d2))
    return LC_NOT_SUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int B = (int)batch, C = (int)in_channels, H = (int)in_h, W = (int)in_w, OC = (int)out_channels,
            KH = (int)kernel_h, KW = (int)kernel_w, SH = (int)stride_h, SW = (int)stride_w, PH = (int)pad_h,
            PW = (int)pad_w, R = apply_relu ? 1 : 0;
  std::vector<std::string> cands = {"simt"};
  if (conv_tc_eligible(C, KH, KW, OC)) cands.push_back(kConvTcName);
  if (conv_implicit_supported(C, OC, KH, KW)) cands.push_back(kConvImplicitName);
  auto run = [&](const std::string& c) -> cudaError_t {
    if (c == kConvImplicitName)
      return conv2d_nchw_f32_implicit(x, w, bias, out, B, C, H, W, OC, KH, KW, SH, SW, PH, PW, R, s);
    return c == kConvTcName ? conv2d_nchw_f32_3xtf32(x, w, bias, out, B, C, H, W, OC, KH, KW, SH, SW, PH, PW, R, s)
                            : conv2d_nchw_f32_simt(x, w, bias, out, B, C, H, W, OC, KH, KW, SH, SW, PH, PW, R, s);
  };
  cudaEvent_t e0, e1;
  if (cudaEventCreate(&e0) != cudaSuccess) return LC_DRIVER_ERROR;
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    return LC_DRIVER_ERROR;
  }
  double best_ms = 1e30;
  std::string best_name;
  lcError_t st = LC_SUCCESS;
  for (const std::string& c : cands) {
    cudaError_t e = run(c);
    std::vector<float> ms;
    for (int rep = 0; rep < 5 && e == cudaSuccess; ++rep) {
      cudaEventRecord(e0, s);
      e = run(c);
      cudaEventRecord(e1, s);
      if (e == cudaSuccess) e = cudaEventSynchronize(e1);
      float t = 0.f;
      if (e == cudaSuccess) e = cudaEventElapsedTime(&t, e0, e1);
      ms.push_back(t);
    }
    if (e != cudaSuccess) {
      st = from_cuda(e);
      break;
    }
    if (candidate_aborted()) continue;
    std::sort(ms.begin(), ms.end());
    if (ms[ms.size() / 2] < best_ms) {
      best_ms = ms[ms.size() / 2];
      best_name = c;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (st != LC_SUCCESS) return st;
  if (best_name.empty()) return LC_DRIVER_ERROR;
  tune_store(LC_TUNE_CONV, d0, d1, d2, LC_DTYPE_F32, best_name);
  if (best && cap) std::snprintf(best, cap, "%s", best_name.c_str());
  return LC_SUCCESS;
}

}  // extern "C"
