// Host-only helpers shared by the C ABI translation units.
#pragma once

#include <cuda_runtime.h>

#include "../../include/lc_b200.h"

namespace lcb {

// RuntimeTraceEventType values (reference include/lightning_core/core/runtime.hpp:50-62).
enum TraceType {
  kTraceMalloc = 0,
  kTraceFree,
  kTraceMemcpy,
  kTraceDeviceSynchronize,
  kTraceApplySyncPolicy,
  kTraceGetDeviceCount,
  kTraceIsCudaAvailable,
  kTraceIsMetalAvailable,
  kTracePreferredDeviceFor,
  kTraceBackendName,
  kTraceOpDispatch
};
// RuntimeTraceOpKind values (runtime.hpp:65-73).
enum TraceOp { kOpUnknown = 0, kOpMatMul, kOpVectorAdd, kOpMatrixSub, kOpMatrixDiv, kOpConv2dNchw, kOpAttention };

lcError_t from_cuda(cudaError_t e);

// The conv launchers take int dimensions and form C*kh*kw and padded extents in int: every size
// argument, the padded input extents and the reduction length must fit.
inline bool conv_dims_fit_int(size_t in_c, size_t in_h, size_t in_w, size_t out_c, size_t kh, size_t kw, size_t sh,
                              size_t sw, size_t ph, size_t pw) {
  const size_t lim = 0x7fffffff;
  if (in_c > lim || in_h > lim || in_w > lim || out_c > lim || kh > lim || kw > lim || sh > lim || sw > lim ||
      ph > lim || pw > lim)
    return false;
  if (in_h + 2 * ph > lim || in_w + 2 * pw > lim) return false;
  if (kh * kw > lim || in_c > lim / (kh * kw)) return false;
  return true;
}
void trace_event(int type, lcError_t status, size_t bytes, int d0, int d1);
void trace_op(int op_kind, size_t workload_hint);

}  // namespace lcb
