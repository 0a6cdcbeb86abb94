// Device::kCUDA for the reference's own C++ operator API, served by liblc_b200.so.
//
// The reference's ops templates route Device::kCUDA to out-of-line hooks declared in
// include/lightning_core/core/detail/ops_backend.hpp (float overloads: vectorAddCudaWithPolicy
// :52-60, matMulCudaWithPolicy :209-219, matrixSubCudaWithPolicy :408-417, matrixDivCudaWithPolicy
// :558-567), dispatched from include/lightning_core/core/ops.hpp:115,
// :394, :1492, :1595.  The reference defines them as stubs that return kNotSupported, after which
// ops.hpp falls back to its CPU loops (src/ops/matmul_cpu.cpp:241-257, src/ops/vector_add_cpu.cpp
// :134-149).  This file defines the same four functions with the same signatures (taken from that
// header, so a mismatch does not compile) on top of the C ABI.  Linked into a program, or into a
// shared library loaded before the reference's, its definitions take the place of the stubs by
// ordinary symbol resolution, and nothing of the reference is edited.
//
// The policy flags keep the reference's meaning: upload_x set -> x is host memory, copied in;
// download_out set -> out is host memory; synchronize -> the call waits for its work.  A status
// other than success goes back to ops.hpp unchanged, so kNotSupported (say, a shape no kernel
// takes) still ends in the reference's CPU fallback, and the double/long double overloads keep
// the reference's stubs (liblc_b200.so computes in fp32 and bf16).
#include <atomic>
#include <cstddef>

#include "lc_b200.h"
#include "lightning_core/core/detail/ops_backend.hpp"

namespace {

std::atomic<unsigned long> g_routed{0};

lightning_core::runtime::Status to_status(lcError_t e) {
  using S = lightning_core::runtime::Status;
  switch (e) {
    case LC_SUCCESS: g_routed.fetch_add(1, std::memory_order_relaxed); return S::kSuccess;
    case LC_NOT_INITIALIZED: return S::kNotInitialized;
    case LC_INVALID_VALUE: return S::kInvalidValue;
    case LC_OUT_OF_MEMORY: return S::kOutOfMemory;
    case LC_NOT_SUPPORTED: return S::kNotSupported;
    case LC_DRIVER_ERROR: return S::kDriverError;
    default: return S::kUnknown;
  }
}

lcVectorAddIoPolicy elem_policy(bool upload_a, bool upload_b, bool download_out, bool synchronize) {
  lcVectorAddIoPolicy p;
  p.upload_a = upload_a;
  p.upload_b = upload_b;
  p.download_out = download_out;
  p.synchronize = synchronize;
  return p;
}

}  // namespace

// Calls of the four hooks that liblc_b200.so completed (a test reads it to tell the kCUDA route
// from the reference's silent CPU fallback).
extern "C" unsigned long lcReferenceHookCalls() { return g_routed.load(std::memory_order_relaxed); }

namespace lightning_core::detail {

runtime::Status vectorAddCudaWithPolicy(const float* a, const float* b, float* out, std::size_t n, bool upload_a,
                                        bool upload_b, bool download_out, bool synchronize) {
  const lcVectorAddIoPolicy p = elem_policy(upload_a, upload_b, download_out, synchronize);
  return to_status(lcVectorAdd(a, b, out, n, LC_DTYPE_F32, &p, nullptr));
}

runtime::Status matMulCudaWithPolicy(const float* a, const float* b, float* out, std::size_t m, std::size_t k,
                                     std::size_t n, bool upload_a, bool upload_b, bool download_out,
                                     bool synchronize) {
  lcMatMulIoPolicy p;
  p.upload_a = upload_a;
  p.upload_b = upload_b;
  p.download_out = download_out;
  p.synchronize = synchronize;
  return to_status(lcMatMul(a, b, out, m, k, n, LC_DTYPE_F32, &p, nullptr));
}

runtime::Status matrixSubCudaWithPolicy(const float* a, const float* b, float* out, std::size_t rows,
                                        std::size_t cols, bool upload_a, bool upload_b, bool download_out,
                                        bool synchronize) {
  const lcVectorAddIoPolicy p = elem_policy(upload_a, upload_b, download_out, synchronize);
  return to_status(lcMatrixSub(a, b, out, rows, cols, LC_DTYPE_F32, &p, nullptr));
}

runtime::Status matrixDivCudaWithPolicy(const float* a, const float* b, float* out, std::size_t rows,
                                        std::size_t cols, bool upload_a, bool upload_b, bool download_out,
                                        bool synchronize) {
  const lcVectorAddIoPolicy p = elem_policy(upload_a, upload_b, download_out, synchronize);
  return to_status(lcMatrixDiv(a, b, out, rows, cols, LC_DTYPE_F32, &p, nullptr));
}

}  // namespace lightning_core::detail
