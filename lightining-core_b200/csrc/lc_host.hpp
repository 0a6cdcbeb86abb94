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
void trace_event(int type, lcError_t status, size_t bytes, int d0, int d1);
void trace_op(int op_kind, size_t workload_hint);

}  // namespace lcb
