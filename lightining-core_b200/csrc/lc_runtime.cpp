// Runtime half of the C ABI: the reference's lc* runtime symbols on a real CUDA memory model
// (reference: src/runtime.cpp and src/lightning_core_c_api.cpp:179-353), the runtime trace
// ring (src/runtime.cpp:63-99, 620-760), per-device contexts and the device error word.
#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/lc_b200.h"
#include "lc_internal.hpp"
#include "lc_host.hpp"

namespace lcb {

// ---- error mapping ------------------------------------------------------------------------
lcError_t from_cuda(cudaError_t e) {
  switch (e) {
    case cudaSuccess:
      return LC_SUCCESS;
    case cudaErrorMemoryAllocation:
      return LC_OUT_OF_MEMORY;
    case cudaErrorInvalidValue:
    case cudaErrorInvalidDevicePointer:
    case cudaErrorInvalidConfiguration:
      return LC_INVALID_VALUE;
    case cudaErrorNotSupported:
      return LC_NOT_SUPPORTED;
    case cudaErrorInitializationError:
    case cudaErrorNoDevice:
    case cudaErrorInsufficientDriver:
      return LC_NOT_INITIALIZED;
    default:
      return LC_DRIVER_ERROR;
  }
}

// ---- trace ring -----------------------------------------------------------------------------
namespace {
constexpr size_t kTraceCap = 4096;  // src/runtime.cpp:63 (same capacity)
std::mutex g_trace_mu;
std::vector<lcRuntimeTraceEvent> g_trace(kTraceCap);
size_t g_trace_head = 0, g_trace_count = 0;
std::atomic<int> g_trace_enabled{0};
std::atomic<int> g_sync_mode{LC_SYNC_AUTO};
std::atomic<int> g_sync_trace{0};

uint64_t now_ns() {
  return static_cast<uint64_t>(
      std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
          .count());
}
}  // namespace

void trace_event(int type, lcError_t status, size_t bytes, int d0, int d1) {
  if (!g_trace_enabled.load(std::memory_order_relaxed)) return;
  std::lock_guard<std::mutex> lk(g_trace_mu);
  lcRuntimeTraceEvent& e = g_trace[g_trace_head];
  e.type = type;
  e.status = status;
  e.timestamp_ns = now_ns();
  e.size_bytes = bytes;
  e.detail0 = d0;
  e.detail1 = d1;
  g_trace_head = (g_trace_head + 1) % kTraceCap;
  if (g_trace_count < kTraceCap) ++g_trace_count;
}

void trace_op(int op_kind, size_t workload_hint) {
  // requested = selected = CUDA (1), no fallback: the encoding of src/runtime.cpp:703-708.
  trace_event(kTraceOpDispatch, LC_SUCCESS, workload_hint, op_kind, 1 | (1 << 4));
}

// ---- device contexts ------------------------------------------------------------------------
namespace {
std::mutex g_ctx_mu;
DeviceCtx* g_ctx[64] = {};
}  // namespace

std::mutex g_fail_mu;
int g_fail_after = 0, g_fail_count = 0;  // test hook: let `after` allocations pass, fail `count`
std::atomic<int> g_fail_armed{0};
std::atomic<int> g_gemm_stall{-1};

bool injected_alloc_failure() {
  if (!g_fail_armed.load(std::memory_order_relaxed)) return false;
  std::lock_guard<std::mutex> lk(g_fail_mu);
  if (g_fail_after > 0) {
    --g_fail_after;
    return false;
  }
  if (g_fail_count > 0) {
    if (--g_fail_count == 0) g_fail_armed.store(0);
    return true;
  }
  return false;
}

cudaError_t device_malloc(void** p, size_t bytes) {
  if (injected_alloc_failure()) {
    *p = nullptr;
    return cudaErrorMemoryAllocation;
  }
  return cudaMalloc(p, bytes);
}

cudaError_t workspace_alloc(DeviceCtx* ctx, void** p, size_t bytes, cudaStream_t s) {
  if (injected_alloc_failure()) {
    *p = nullptr;
    return cudaErrorMemoryAllocation;
  }
  return cudaMallocFromPoolAsync(p, bytes, ctx->pool, s);
}

cudaError_t workspace_free(void* p, cudaStream_t s) { return p ? cudaFreeAsync(p, s) : cudaSuccess; }

int take_gemm_stall_kblock() { return g_gemm_stall.exchange(-1); }

DeviceCtx* device_ctx() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  DeviceCtx* c = g_ctx[dev];
  if (c) return c;
  std::lock_guard<std::mutex> lk(g_ctx_mu);
  if (g_ctx[dev]) return g_ctx[dev];
  c = new DeviceCtx();
  c->device = dev;
  // One allocation: the error word, padding to 256 bytes, then the persistent-kernel counters.
  constexpr size_t kCtxWords = 64 + 2 * DeviceCtx::kSchedSlots;
  cudaMemPoolProps props = {};
  props.allocType = cudaMemAllocationTypePinned;
  props.location.type = cudaMemLocationTypeDevice;
  props.location.id = dev;
  if (cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaMalloc(&c->err_word, kCtxWords * sizeof(unsigned)) != cudaSuccess ||
      cudaMemset(c->err_word, 0, kCtxWords * sizeof(unsigned)) != cudaSuccess ||
      cudaMemPoolCreate(&c->pool, &props) != cudaSuccess) {
    if (c->err_word) cudaFree(c->err_word);
    delete c;
    return nullptr;
  }
  c->sched = c->err_word + 64;
  uint64_t keep = ~0ull;  // keep freed workspace cached in the pool instead of returning it
  cudaMemPoolSetAttribute(c->pool, cudaMemPoolAttrReleaseThreshold, &keep);
  g_ctx[dev] = c;
  return c;
}

}  // namespace lcb

using lcb::from_cuda;
using lcb::trace_event;

extern "C" {

lcError_t lcMalloc(void** ptr, size_t size_bytes) {
  lcError_t st;
  if (ptr == nullptr || size_bytes == 0) {
    st = LC_INVALID_VALUE;
  } else {
    st = from_cuda(lcb::device_malloc(ptr, size_bytes));
  }
  trace_event(lcb::kTraceMalloc, st, size_bytes, 0, 0);
  return st;
}

lcError_t lcFree(void* ptr) {
  lcError_t st = ptr == nullptr ? LC_SUCCESS : from_cuda(cudaFree(ptr));
  trace_event(lcb::kTraceFree, st, 0, 0, 0);
  return st;
}

lcError_t lcMemcpy(void* dst, const void* src, size_t size_bytes, lcMemcpyKind kind) {
  lcError_t st;
  if (dst == nullptr || src == nullptr) {
    st = LC_INVALID_VALUE;
  } else {
    cudaMemcpyKind k = cudaMemcpyDefault;
    switch (kind) {
      case LC_MEMCPY_HOST_TO_HOST: k = cudaMemcpyHostToHost; break;
      case LC_MEMCPY_HOST_TO_DEVICE: k = cudaMemcpyHostToDevice; break;
      case LC_MEMCPY_DEVICE_TO_HOST: k = cudaMemcpyDeviceToHost; break;
      case LC_MEMCPY_DEVICE_TO_DEVICE: k = cudaMemcpyDeviceToDevice; break;
    }
    st = from_cuda(cudaMemcpy(dst, src, size_bytes, k));
  }
  trace_event(lcb::kTraceMemcpy, st, size_bytes, static_cast<int>(kind), 0);
  return st;
}

lcError_t lcDeviceSynchronize(void) {
  lcError_t st = from_cuda(cudaDeviceSynchronize());
  trace_event(lcb::kTraceDeviceSynchronize, st, 0, 0, 0);
  return st;
}

lcError_t lcGetDeviceCount(int* count) {
  if (count == nullptr) return LC_INVALID_VALUE;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  *count = e == cudaSuccess ? n : 0;
  lcError_t st = e == cudaSuccess ? LC_SUCCESS : LC_NOT_SUPPORTED;
  trace_event(lcb::kTraceGetDeviceCount, st, 0, *count, 0);
  return st;
}

int lcIsCudaAvailable(void) {
  int n = 0;
  return (cudaGetDeviceCount(&n) == cudaSuccess && n > 0) ? 1 : 0;
}

int lcIsMetalAvailable(void) { return 0; }

lcError_t lcGetPreferredDeviceForInference(lcDeviceKind* device) {
  if (device == nullptr) return LC_INVALID_VALUE;
  *device = lcIsCudaAvailable() ? LC_DEVICE_CUDA : LC_DEVICE_CPU;
  return LC_SUCCESS;
}

lcError_t lcGetPreferredDeviceForTraining(lcDeviceKind* device) { return lcGetPreferredDeviceForInference(device); }

lcMemoryModel lcGetMemoryModel(void) { return LC_MEMORY_NATIVE_DEVICE; }

const char* lcGetMemoryModelName(lcMemoryModel model) {
  return model == LC_MEMORY_NATIVE_DEVICE ? "native-device" : "host-managed-compat";
}

lcError_t lcSetDefaultSyncPolicy(lcSyncPolicy policy) {
  lcb::g_sync_mode.store(policy.mode);
  lcb::g_sync_trace.store(policy.trace_sync_boundary);
  return LC_SUCCESS;
}

lcSyncPolicy lcGetDefaultSyncPolicy(void) {
  lcSyncPolicy p;
  const int m = lcb::g_sync_mode.load();
  p.mode = (m == LC_SYNC_ALWAYS || m == LC_SYNC_NEVER) ? static_cast<lcSyncMode>(m) : LC_SYNC_AUTO;
  p.trace_sync_boundary = lcb::g_sync_trace.load();
  return p;
}

// src/runtime.cpp:454-479: never -> no-op; always -> device sync; auto -> sync when a GPU exists.
lcError_t lcApplySyncPolicy(lcSyncPolicy policy) {
  lcError_t st = LC_SUCCESS;
  if (policy.mode == LC_SYNC_ALWAYS || (policy.mode == LC_SYNC_AUTO && lcIsCudaAvailable()))
    st = from_cuda(cudaDeviceSynchronize());
  trace_event(lcb::kTraceApplySyncPolicy, st, 0, static_cast<int>(policy.mode), policy.trace_sync_boundary ? 1 : 0);
  return st;
}

lcError_t lcApplyDefaultSyncPolicy(void) { return lcApplySyncPolicy(lcGetDefaultSyncPolicy()); }

static lcBackendCapabilities caps_for(lcDeviceKind device) {
  lcBackendCapabilities c;
  std::memset(&c, 0, sizeof(c));
  c.device = device;
  c.runtime_trace_surface = 1;
  c.sync_policy_surface = 1;
  c.memory_model = LC_MEMORY_NATIVE_DEVICE;
  if (device == LC_DEVICE_CUDA) {
    c.built = 1;
    c.available = lcIsCudaAvailable();
    c.compute_surface = c.available;
    c.memory_surface = c.available;
    c.sync_surface = c.available;
    c.profiling_surface = c.available;
  } else if (device == LC_DEVICE_CPU) {
    // This library has no CPU compute path: the CPU backend is host memory only.
    c.built = 1;
    c.available = 1;
    c.memory_surface = 1;
    c.sync_surface = 1;
  }
  return c;
}

lcError_t lcGetBackendCapabilities(lcDeviceKind device, lcBackendCapabilities* out_caps) {
  if (out_caps == nullptr) return LC_INVALID_VALUE;
  *out_caps = caps_for(device);
  return LC_SUCCESS;
}

lcError_t lcGetActiveBackendCapabilities(lcBackendCapabilities* out_caps) {
  return lcGetBackendCapabilities(LC_DEVICE_CUDA, out_caps);
}

lcError_t lcGetBackendInterfaceContract(lcDeviceKind device, lcBackendInterfaceContract* out) {
  if (out == nullptr) return LC_INVALID_VALUE;
  std::memset(out, 0, sizeof(*out));
  out->device = device;
  out->capabilities = caps_for(device);
  const bool cuda = device == LC_DEVICE_CUDA;
  // Driver tags as in src/runtime.cpp:541-580.
  out->compute.available = out->capabilities.compute_surface;
  out->compute.op_dispatch_trace_surface = 1;
  out->compute.driver_tag = cuda ? "cuda.runtime.dispatch" : device == LC_DEVICE_METAL ? "metal.compute.dispatch"
                                                                                       : "cpu.eager.dispatch";
  out->memory.available = out->capabilities.memory_surface;
  out->memory.allocator_surface = out->capabilities.memory_surface;
  out->memory.memcpy_surface = out->capabilities.memory_surface;
  out->memory.memory_model = LC_MEMORY_NATIVE_DEVICE;
  out->memory.driver_tag = cuda ? "cuda.memory" : device == LC_DEVICE_METAL ? "metal.host_managed_memory"
                                                                            : "cpu.host_memory";
  out->sync.available = out->capabilities.sync_surface;
  out->sync.sync_policy_surface = 1;
  out->sync.trace_sync_boundary_surface = 1;
  out->sync.driver_tag = cuda ? "cuda.device_sync" : device == LC_DEVICE_METAL ? "metal.command_sync"
                                                                               : "cpu.noop_sync";
  out->profiler.available = 1;
  out->profiler.runtime_trace_surface = 1;
  out->profiler.op_dispatch_trace_surface = 1;
  out->profiler.trace_capacity = lcb::kTraceCap;
  out->profiler.driver_tag = "runtime.trace.ring";
  return LC_SUCCESS;
}

lcError_t lcGetActiveBackendInterfaceContract(lcBackendInterfaceContract* out) {
  return lcGetBackendInterfaceContract(LC_DEVICE_CUDA, out);
}

lcError_t lcGetApiVersion(int* out_major, int* out_minor, int* out_patch) {
  if (!out_major || !out_minor || !out_patch) return LC_INVALID_VALUE;
  *out_major = LC_API_VERSION_MAJOR;
  *out_minor = LC_API_VERSION_MINOR;
  *out_patch = LC_API_VERSION_PATCH;
  return LC_SUCCESS;
}

const char* lcGetApiVersionString(void) { return LC_API_VERSION_STRING; }

size_t lcGetStructSize(lcStructId id) {
  switch (id) {
    case LC_STRUCT_BACKEND_CAPABILITIES: return sizeof(lcBackendCapabilities);
    case LC_STRUCT_COMPUTE_INTERFACE_CONTRACT: return sizeof(lcComputeInterfaceContract);
    case LC_STRUCT_MEMORY_INTERFACE_CONTRACT: return sizeof(lcMemoryInterfaceContract);
    case LC_STRUCT_SYNC_INTERFACE_CONTRACT: return sizeof(lcSyncInterfaceContract);
    case LC_STRUCT_PROFILER_INTERFACE_CONTRACT: return sizeof(lcProfilerInterfaceContract);
    case LC_STRUCT_BACKEND_INTERFACE_CONTRACT: return sizeof(lcBackendInterfaceContract);
    default: return 0;
  }
}

int lcCheckStructSize(lcStructId id, size_t observed) {
  const size_t e = lcGetStructSize(id);
  return (e != 0 && e == observed) ? 1 : 0;
}

const char* lcBackendName(void) { return lcIsCudaAvailable() ? "cuda" : "cpu"; }

// src/runtime.cpp:762-781 strings.
const char* lcGetErrorString(lcError_t error) {
  switch (error) {
    case LC_SUCCESS: return "success";
    case LC_NOT_INITIALIZED: return "not initialized";
    case LC_INVALID_VALUE: return "invalid value";
    case LC_OUT_OF_MEMORY: return "out of memory";
    case LC_NOT_SUPPORTED: return "not supported";
    case LC_DRIVER_ERROR: return "driver error";
    default: return "unknown error";
  }
}

// ---- trace + error word --------------------------------------------------------------------
void lcRuntimeTraceSetEnabled(int enabled) { lcb::g_trace_enabled.store(enabled ? 1 : 0); }
int lcRuntimeTraceIsEnabled(void) { return lcb::g_trace_enabled.load(); }
void lcRuntimeTraceClear(void) {
  std::lock_guard<std::mutex> lk(lcb::g_trace_mu);
  lcb::g_trace_head = 0;
  lcb::g_trace_count = 0;
}
size_t lcRuntimeTraceCount(void) {
  std::lock_guard<std::mutex> lk(lcb::g_trace_mu);
  return lcb::g_trace_count;
}
size_t lcRuntimeTraceCapacity(void) { return lcb::kTraceCap; }
lcError_t lcRuntimeTraceGet(size_t index, lcRuntimeTraceEvent* out) {
  if (out == nullptr) return LC_INVALID_VALUE;
  std::lock_guard<std::mutex> lk(lcb::g_trace_mu);
  if (index >= lcb::g_trace_count) return LC_INVALID_VALUE;
  const size_t first = (lcb::g_trace_head + lcb::kTraceCap - lcb::g_trace_count) % lcb::kTraceCap;
  *out = lcb::g_trace[(first + index) % lcb::kTraceCap];
  return LC_SUCCESS;
}

lcError_t lcGetDeviceErrorWord(unsigned int* code) {
  if (code == nullptr) return LC_INVALID_VALUE;
  lcb::DeviceCtx* c = lcb::device_ctx();
  if (!c) return LC_NOT_INITIALIZED;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return from_cuda(e);
  e = cudaMemcpy(code, c->err_word, sizeof(unsigned), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return from_cuda(e);
  return *code ? LC_DRIVER_ERROR : LC_SUCCESS;
}

lcError_t lcClearDeviceErrorWord(void) {
  lcb::DeviceCtx* c = lcb::device_ctx();
  if (!c) return LC_NOT_INITIALIZED;
  return from_cuda(cudaMemset(c->err_word, 0, sizeof(unsigned)));
}

void lcTestFailAllocations(int after, int count) {
  std::lock_guard<std::mutex> lk(lcb::g_fail_mu);
  lcb::g_fail_after = after < 0 ? 0 : after;
  lcb::g_fail_count = count < 0 ? 0 : count;
  lcb::g_fail_armed.store(lcb::g_fail_count > 0 ? 1 : 0);
}

void lcTestStallNextGemm(int kblock) { lcb::g_gemm_stall.store(kblock < 0 ? -1 : kblock); }

}  // extern "C"
