/* lc_b200.h -- C ABI of liblc_b200.so, the B200 (sm_100a) build of Lightning Core's
 * attention / matmul2d / conv->attention hot path.
 *
 * Part 1 keeps every runtime symbol, enum and struct of the reference's C ABI with identical
 * names, values and layouts (include/lightning_core/lightning_core.h:1-141 of the reference;
 * implementation src/lightning_core_c_api.cpp:179-353), so existing C callers relink unchanged.
 * Part 2 adds the op entry points the reference only exposes through C++ templates and pybind.
 *
 * Conventions of the op entry points (part 2):
 *  - Errors are returned as lcError_t, never thrown.  Null or zero-sized arguments ->
 *    LC_INVALID_VALUE (reference: src/attention.cpp:145-148, ops.hpp:366-369); a shape the
 *    kernels cannot take -> LC_NOT_SUPPORTED; a CUDA failure or a kernel-side bounded wait that
 *    gave up -> LC_DRIVER_ERROR.  There is no CPU fallback on any path.
 *  - IO policies carry the reference's meaning on explicit device memory: an upload_* flag set
 *    means that pointer is HOST memory and is copied in with cudaMemcpyAsync; clear means it
 *    is already a DEVICE pointer (or, for sessions, that the session's resident buffer is
 *    reused).  download_out set means `out` is host memory and the result is copied back;
 *    synchronize set means cudaStreamSynchronize(stream) before returning.  A NULL policy
 *    means "all device pointers, asynchronous".
 *  - `stream` is a cudaStream_t (NULL = the legacy default stream).
 *  - Tensors are dense row-major; "units" are independent heads/images stacked outermost.
 */
#ifndef LC_B200_H
#define LC_B200_H

#include <stddef.h>
#include <stdint.h>

#define LC_API_VERSION_MAJOR 0
#define LC_API_VERSION_MINOR 6
#define LC_API_VERSION_PATCH 0
#define LC_API_VERSION_STRING "0.6.0-rc0"

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ===================== Part 1: reference runtime ABI (lightning_core.h) ================= */

typedef enum lcError {
  LC_SUCCESS = 0,
  LC_NOT_INITIALIZED,
  LC_INVALID_VALUE,
  LC_OUT_OF_MEMORY,
  LC_NOT_SUPPORTED,
  LC_DRIVER_ERROR,
  LC_UNKNOWN
} lcError_t;

typedef enum lcMemcpyKind {
  LC_MEMCPY_HOST_TO_HOST = 0,
  LC_MEMCPY_HOST_TO_DEVICE,
  LC_MEMCPY_DEVICE_TO_HOST,
  LC_MEMCPY_DEVICE_TO_DEVICE
} lcMemcpyKind;

typedef enum lcDeviceKind { LC_DEVICE_CPU = 0, LC_DEVICE_CUDA, LC_DEVICE_METAL } lcDeviceKind;

typedef enum lcMemoryModel { LC_MEMORY_NATIVE_DEVICE = 0, LC_MEMORY_HOST_MANAGED_COMPAT } lcMemoryModel;

typedef enum lcSyncMode { LC_SYNC_AUTO = 0, LC_SYNC_ALWAYS, LC_SYNC_NEVER } lcSyncMode;

typedef struct lcSyncPolicy {
  lcSyncMode mode;
  int trace_sync_boundary;
} lcSyncPolicy;

typedef struct lcBackendCapabilities {
  lcDeviceKind device;
  int built;
  int available;
  int compute_surface;
  int memory_surface;
  int sync_surface;
  int profiling_surface;
  int runtime_trace_surface;
  int sync_policy_surface;
  lcMemoryModel memory_model;
} lcBackendCapabilities;

typedef struct lcComputeInterfaceContract {
  int available;
  int op_dispatch_trace_surface;
  const char* driver_tag;
} lcComputeInterfaceContract;

typedef struct lcMemoryInterfaceContract {
  int available;
  int allocator_surface;
  int memcpy_surface;
  lcMemoryModel memory_model;
  const char* driver_tag;
} lcMemoryInterfaceContract;

typedef struct lcSyncInterfaceContract {
  int available;
  int sync_policy_surface;
  int trace_sync_boundary_surface;
  const char* driver_tag;
} lcSyncInterfaceContract;

typedef struct lcProfilerInterfaceContract {
  int available;
  int runtime_trace_surface;
  int op_dispatch_trace_surface;
  size_t trace_capacity;
  const char* driver_tag;
} lcProfilerInterfaceContract;

typedef struct lcBackendInterfaceContract {
  lcDeviceKind device;
  lcBackendCapabilities capabilities;
  lcComputeInterfaceContract compute;
  lcMemoryInterfaceContract memory;
  lcSyncInterfaceContract sync;
  lcProfilerInterfaceContract profiler;
} lcBackendInterfaceContract;

typedef enum lcStructId {
  LC_STRUCT_BACKEND_CAPABILITIES = 1,
  LC_STRUCT_COMPUTE_INTERFACE_CONTRACT = 2,
  LC_STRUCT_MEMORY_INTERFACE_CONTRACT = 3,
  LC_STRUCT_SYNC_INTERFACE_CONTRACT = 4,
  LC_STRUCT_PROFILER_INTERFACE_CONTRACT = 5,
  LC_STRUCT_BACKEND_INTERFACE_CONTRACT = 6
} lcStructId;

/* lightning_core.h:113-137 (reference). lcMalloc is cudaMalloc on the current device. */
lcError_t lcMalloc(void** ptr, size_t size_bytes);
lcError_t lcFree(void* ptr);
lcError_t lcMemcpy(void* dst, const void* src, size_t size_bytes, lcMemcpyKind kind);
lcError_t lcDeviceSynchronize(void);
lcError_t lcGetDeviceCount(int* count);
lcError_t lcGetPreferredDeviceForInference(lcDeviceKind* device);
lcError_t lcGetPreferredDeviceForTraining(lcDeviceKind* device);
int lcIsCudaAvailable(void);
int lcIsMetalAvailable(void);
lcMemoryModel lcGetMemoryModel(void);
const char* lcGetMemoryModelName(lcMemoryModel model);
lcError_t lcSetDefaultSyncPolicy(lcSyncPolicy policy);
lcSyncPolicy lcGetDefaultSyncPolicy(void);
lcError_t lcApplySyncPolicy(lcSyncPolicy policy);
lcError_t lcApplyDefaultSyncPolicy(void);
lcError_t lcGetBackendCapabilities(lcDeviceKind device, lcBackendCapabilities* out_caps);
lcError_t lcGetActiveBackendCapabilities(lcBackendCapabilities* out_caps);
lcError_t lcGetBackendInterfaceContract(lcDeviceKind device, lcBackendInterfaceContract* out_contract);
lcError_t lcGetActiveBackendInterfaceContract(lcBackendInterfaceContract* out_contract);
lcError_t lcGetApiVersion(int* out_major, int* out_minor, int* out_patch);
const char* lcGetApiVersionString(void);
size_t lcGetStructSize(lcStructId struct_id);
int lcCheckStructSize(lcStructId struct_id, size_t observed_size);
const char* lcBackendName(void);
const char* lcGetErrorString(lcError_t error);

/* ===================== Part 2: hot-path op entry points (new in this build) =============== */

typedef enum lcDataType {
  LC_DTYPE_F32 = 0,  /* fp32 in/out, fp32-accurate: 3xTF32 on tcgen05, SIMT FFMA for small shapes */
  LC_DTYPE_BF16 = 1, /* bf16 in/out, fp32 accumulate/softmax on tcgen05 tensor cores */
  LC_DTYPE_F64 = 2   /* vector add only                                             */
} lcDataType;

typedef void* lcStream_t; /* a cudaStream_t */

/* include/lightning_core/core/attention.hpp:16-32 (AttentionIoPolicy), ints for bools. */
typedef struct lcAttentionIoPolicy {
  int upload_q, upload_k, upload_v, upload_target;
  int download_out, download_v, synchronize;
  int loss_every;
  float output_scale, output_bias; /* out = max(0?)(out*scale + bias), relu if output_relu */
  int output_relu;
} lcAttentionIoPolicy;

/* include/lightning_core/core/ops/policy.hpp:8-34. */
typedef struct lcMatMulIoPolicy { int upload_a, upload_b, download_out, synchronize; } lcMatMulIoPolicy;
typedef struct lcVectorAddIoPolicy { int upload_a, upload_b, download_out, synchronize; } lcVectorAddIoPolicy;
typedef struct lcConv2dIoPolicy { int upload_x, upload_w, upload_bias, download_out, synchronize; } lcConv2dIoPolicy;

/* Fills the reference defaults (everything true, loss_every=1, scale 1, bias 0, no relu). */
void lcAttentionIoPolicyDefault(lcAttentionIoPolicy* p);
void lcMatMulIoPolicyDefault(lcMatMulIoPolicy* p);
void lcConv2dIoPolicyDefault(lcConv2dIoPolicy* p);
void lcVectorAddIoPolicyDefault(lcVectorAddIoPolicy* p);

/* Resident-loop presets, include/lightning_core/core/ops/policy.hpp:37-71
 * (start: upload, no download, no sync; run: nothing; finish: download+sync; sync: sync). */
typedef enum lcLoopStage { LC_LOOP_START = 0, LC_LOOP_RUN, LC_LOOP_FINISH, LC_LOOP_SYNC } lcLoopStage;
void lcMatMulPolicyForStage(lcLoopStage stage, lcMatMulIoPolicy* p);
/* The same presets for vector add and the matrix elementwise ops (makeVectorPolicyForLoop /
 * makeElemwisePolicyForLoop, include/lightning_core/core/model_customization.hpp:120-144, over the
 * resident presets of ops/policy.hpp:73-150); both ops take lcVectorAddIoPolicy. */
void lcVectorPolicyForStage(lcLoopStage stage, lcVectorAddIoPolicy* p);
void lcElemwisePolicyForStage(lcLoopStage stage, lcVectorAddIoPolicy* p);
/* makeAttentionPolicyForLoop (model_customization.hpp:146-185): sets only the transfer and sync
 * flags of *p (loss_every and the output postprocess are the caller's): start uploads q, k, v and
 * target; run moves nothing; finish downloads out (and v when `training`) and synchronizes; sync
 * only synchronizes. */
void lcAttentionPolicyForStage(lcLoopStage stage, int training, lcAttentionIoPolicy* p);

/* Attention forward over `units` independent heads laid out [units, seq, head_dim].
 * Replaces attentionForwardWithPolicy (src/attention.cpp:137-201) for Device::kCUDA, batched.
 * scale = 1/sqrt(head_dim); causal masks j > i. f32: strict fp32, any head_dim <= 256.
 * bf16: tcgen05 flash attention for head_dim 64/128 (others: fp32-math SIMT kernel). */
lcError_t lcAttentionForward(const void* q, const void* k, const void* v, void* out, size_t units, size_t seq,
                             size_t head_dim, int causal, lcDataType dtype, const lcAttentionIoPolicy* policy,
                             lcStream_t stream);

/* C[m,n] = A[m,k] B[k,n], row-major, no transposes; replaces ops::matMulWithPolicy<T>
 * (include/lightning_core/core/ops.hpp:354-459) for Device::kCUDA.  bf16: tcgen05 GEMM with
 * fp32 accumulation (needs k%8==0 and n%8==0, else a SIMT kernel). f32: strict fp32. */
lcError_t lcMatMul(const void* a, const void* b, void* out, size_t m, size_t k, size_t n, lcDataType dtype,
                   const lcMatMulIoPolicy* policy, lcStream_t stream);

/* attentionTrainStepWithPolicy (src/attention.cpp:216-242; CPU src/attention_cpu.cpp:114-163):
 * forward (written to `out`), MSE loss against `target`, dV = P^T dO with dO = 2(out - target)/(seq*d),
 * v -= learning_rate * dV in place.  fp32, head_dim <= 128, `units` heads [units, seq, head_dim].
 * learning_rate <= 0 -> LC_INVALID_VALUE.  loss_out (host, may be NULL) receives one loss per unit
 * (mean squared error, as the reference).  Policy: upload_q/k/v/target mark host inputs;
 * download_out / download_v copy `out` / the updated `v` back to host memory. */
lcError_t lcAttentionTrainStep(const float* q, const float* k, float* v, const float* target, float* out,
                               float learning_rate, size_t units, size_t seq, size_t head_dim, int causal,
                               float* loss_out, const lcAttentionIoPolicy* policy, lcStream_t stream);

/* NCHW x OIHW (+bias, may be NULL) -> NCHW, optional ReLU; replaces ops::conv2dNchw<float>
 * (include/lightning_core/core/ops.hpp:855-1212).  fp32 strict implicit GEMM. */
lcError_t lcConv2dNchw(const float* x, const float* w, const float* bias, float* out, size_t batch,
                       size_t in_channels, size_t in_h, size_t in_w, size_t out_channels, size_t kernel_h,
                       size_t kernel_w, size_t stride_h, size_t stride_w, size_t pad_h, size_t pad_w,
                       int apply_relu, const lcConv2dIoPolicy* policy, lcStream_t stream);

/* Integrated conv2d+ReLU -> QKV arrange -> non-causal attention -> optional projection.
 * Replaces convAttentionTorchstrongNchwIntoDirect (python/bindings/bind_integrated.cpp:614-730)
 * plus the attention_qkv_proj pattern (include/lightning_core/core/graph.hpp:3529-3547).
 *   per_image = 0: the reference's semantics for any batch: one attention over the first
 *                  3*seq*head_dim floats of the flat conv output (cyclically repeated if short);
 *                  out is [seq, cols].
 *   per_image = 1: image b runs those batch-1 semantics on x[b]; out is [batch, seq, cols].
 * cols = proj_cols when proj_w ([head_dim, proj_cols]) is given, else head_dim.
 * Policy flags refer to x/w/bias/proj_w (upload_x .. upload_bias; proj_w follows upload_w). */
lcError_t lcConvAttentionNchw(const float* x, const float* w, const float* bias, const float* proj_w, float* out,
                              size_t batch, size_t in_channels, size_t in_h, size_t in_w, size_t out_channels,
                              size_t kernel_h, size_t kernel_w, size_t stride_h, size_t stride_w, size_t pad_h,
                              size_t pad_w, size_t seq, size_t head_dim, size_t proj_cols, int per_image,
                              const lcConv2dIoPolicy* policy, lcStream_t stream);

/* No counterpart in the reference.  lcConvAttentionNchw for callers that cannot allocate GPU
 * memory (code running where cudaMalloc may not be called -- a host callback, a real-time loop,
 * a plugin whose host owns every device allocation).  Same arguments and results as
 * lcConvAttentionNchw, but every pointer is a DEVICE pointer (no IO policy) and the conv
 * intermediate lives in a fixed 64 MiB array compiled into the library (16 Mi floats), which
 * every GPU that loads the library holds until exit.  Needs batch*out_channels*out_h*out_w
 * floats of it (plus units*3*seq*head_dim when the conv output is shorter than 3*seq*head_dim);
 * larger calls return LC_INVALID_VALUE.  Allocates nothing: no cudaMalloc/cudaFree.  The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress), so make that
 * first call before any stream capture.  All calls share the array: calls that overlap on the
 * GPU race -- keep them on one stream.  Asynchronous on `stream`. */
lcError_t lcConvAttentionNchwNoAlloc(const float* x, const float* w, const float* bias, const float* proj_w,
                                     float* out, size_t batch, size_t in_channels, size_t in_h, size_t in_w,
                                     size_t out_channels, size_t kernel_h, size_t kernel_w, size_t stride_h,
                                     size_t stride_w, size_t pad_h, size_t pad_w, size_t seq, size_t head_dim,
                                     size_t proj_cols, int per_image, lcStream_t stream);

/* Graph fused pattern attention_proj_v1 (GraphIR::executeAttentionProjFusedNodeTyped,
 * include/lightning_core/core/graph.hpp:3454-3555): out[u] = attention(q[u], k[u], v[u]) @ proj_w,
 * q/k/v [units, seq, head_dim], proj_w [head_dim, proj_cols], out [units, seq, proj_cols], scale
 * 1/sqrt(head_dim); the graph passes causal = 0.  f32: one fused kernel (the projection runs in the
 * attention epilogue) when head_dim, proj_cols <= 128, else attention then GEMM; bf16: tcgen05
 * attention then tcgen05 GEMM.  Policy: upload_q/k/v as for attention, proj_w follows upload_q;
 * the output postprocess fields must be neutral (scale 1, bias 0, no ReLU). */
lcError_t lcAttentionProjForward(const void* q, const void* k, const void* v, const void* proj_w, void* out,
                                 size_t units, size_t seq, size_t head_dim, size_t proj_cols, int causal,
                                 lcDataType dtype, const lcAttentionIoPolicy* policy, lcStream_t stream);

/* Graph fused pattern attention_qkv_proj_v1 (graph.hpp:3556-3584 with the kQkvPackRepeat node,
 * graph.hpp:3138-3185): Q, K, V are the consecutive [seq, head_dim] flat slices of `packed`
 * (packed_len floats, repeated cyclically when shorter than 3*seq*head_dim), then non-causal
 * attention and the projection as above.  f32 only, like the reference's pack node.  `packed`
 * follows upload_q, proj_w too. */
lcError_t lcAttentionQkvProjForward(const float* packed, size_t packed_len, const float* proj_w, float* out,
                                    size_t seq, size_t head_dim, size_t proj_cols,
                                    const lcAttentionIoPolicy* policy, lcStream_t stream);

/* out = a + b (f32 or f64); replaces vectorAddCuda (src/ops/vector_add_cuda.cu:12-86). */
lcError_t lcVectorAdd(const void* a, const void* b, void* out, size_t n, lcDataType dtype,
                      const lcVectorAddIoPolicy* policy, lcStream_t stream);

/* ops::matrixSub / matrixDiv (include/lightning_core/core/ops.hpp:31-49, CPU
 * src/ops/matrix_elemwise.cpp:8-29): out = a - b / a / b elementwise over rows x cols, f32 or f64,
 * IEEE arithmetic (sub is bit-identical to the reference CPU loop; the reference's -ffast-math
 * build divides approximately, so div agrees to rounding).  The policy struct has the fields of
 * the reference's MatrixElementwiseIoPolicy (ops/policy.hpp:15-20). */
lcError_t lcMatrixSub(const void* a, const void* b, void* out, size_t rows, size_t cols, lcDataType dtype,
                      const lcVectorAddIoPolicy* policy, lcStream_t stream);
lcError_t lcMatrixDiv(const void* a, const void* b, void* out, size_t rows, size_t cols, lcDataType dtype,
                      const lcVectorAddIoPolicy* policy, lcStream_t stream);

/* (x - mean)/sqrt(var + eps) over the last axis, population variance, no affine
 * (the reference's LN formula, README.md:2267-2270).  Device pointers, fp32. */
lcError_t lcLayerNorm(const float* x, float* out, size_t rows, size_t cols, float eps, lcStream_t stream);

/* ---- device-resident sessions ----------------------------------------------------------------
 * AttentionSession (include/lightning_core/core/attention.hpp:86-129, src/attention.cpp:247-343) and
 * MatMulMetalResidentSession (include/lightning_core/core/ops.hpp:1339-1379): a handle bound to one
 * shape owning device buffers that persist between calls.  Policy flags: upload_* set -> copy that
 * HOST pointer into the session buffer; clear -> reuse the buffer as it is (pointer may be NULL);
 * download_out set -> copy the result to HOST `out`; synchronize -> wait on `stream`.  Buffers can be
 * filled or read directly through lcAttentionSessionBuffer / lcMatMulSessionBuffer (device
 * pointers; which = 0 q|a, 1 k|b, 2 v (attention) / out (matmul), 3 out (attention)).  Calls on one
 * session from several threads serialise on a per-session lock. */
typedef struct lcAttentionSession* lcAttentionSession_t;
typedef struct lcMatMulSession* lcMatMulSession_t;
lcError_t lcAttentionSessionCreate(lcAttentionSession_t* out, size_t units, size_t seq, size_t head_dim, int causal,
                                   lcDataType dtype);
lcError_t lcAttentionSessionDestroy(lcAttentionSession_t s);
/* Default policy for calls that pass NULL; starts as the reference session default
 * (everything uploaded/downloaded, synchronize = 0). */
lcError_t lcAttentionSessionSetDefaultPolicy(lcAttentionSession_t s, const lcAttentionIoPolicy* policy);
lcError_t lcAttentionSessionBuffer(lcAttentionSession_t s, int which, void** dev_ptr);
lcError_t lcAttentionSessionForward(lcAttentionSession_t s, const void* q, const void* k, const void* v, void* out,
                                    const lcAttentionIoPolicy* policy, lcStream_t stream);
/* AttentionSession::trainStepWithPolicy (src/attention.cpp:301-343): one train step on the
 * session's resident q/k/v (v updated in place, so repeated steps train it); `target` follows
 * upload_target.  With loss_out, the loss is computed every loss_every-th step (0 -> the
 * reference's shape-aware default) and the last sampled loss is returned in between. */
lcError_t lcAttentionSessionTrainStep(lcAttentionSession_t s, const float* q, const float* k, float* v,
                                      const float* target, float* out, float learning_rate, float* loss_out,
                                      const lcAttentionIoPolicy* policy, lcStream_t stream);
lcError_t lcMatMulSessionCreate(lcMatMulSession_t* out, size_t m, size_t k, size_t n, lcDataType dtype);
lcError_t lcMatMulSessionDestroy(lcMatMulSession_t s);
lcError_t lcMatMulSessionBuffer(lcMatMulSession_t s, int which, void** dev_ptr);
/* One call; drive a resident loop with lcMatMulPolicyForStage(START / RUN / FINISH / SYNC). */
lcError_t lcMatMulSessionRun(lcMatMulSession_t s, const void* a, const void* b, void* out,
                             const lcMatMulIoPolicy* policy, lcStream_t stream);
/* runBatchSync / runBatchSyncNoDownload (ops.hpp:251-352): upload a / b when non-NULL, launch
 * `repeat` times on the resident buffers, synchronize once, download when out != NULL. */
lcError_t lcMatMulSessionRunBatch(lcMatMulSession_t s, const void* a, const void* b, void* out, size_t repeat,
                                  lcStream_t stream);

/* ---- per-shape auto-tune cache (src/ops/matmul_metal.mm:416-577, src/attention_metal.mm:184-336) */
/* CSV `#lc_tune_cache,<matmul|attention>,2` + `#columns,...`; keys (m,k,n,dtype) for matmul and
 * (seq,head_dim,causal,dtype) for attention; values are sm_100a kernel configuration names
 * (matmul: "simt128x128", "simt128x64", "simt64x64", "tcgen05_128x256", "tcgen05_2sm_256x256",
 * "tcgen05_3xtf32", "simt"; attention: "tcgen05_1q", "tcgen05_1qp", "tcgen05_2q", "tcgen05_3xtf32", "simt").  A NULL path
 * means CJ_MATMUL_TUNE_CACHE_FILE / CJ_ATTN_TUNE_CACHE_FILE, which is also loaded on first use and
 * rewritten whenever an entry is added.  Load rejects a file with an unknown header
 * (LC_NOT_SUPPORTED) and keeps the current rows. */
typedef enum lcTuneKind { LC_TUNE_MATMUL = 0, LC_TUNE_ATTENTION = 1, LC_TUNE_CONV = 2 } lcTuneKind;
lcError_t lcTuneCacheLoad(lcTuneKind kind, const char* path);
lcError_t lcTuneCacheSave(lcTuneKind kind, const char* path);
/* Clears the cache (the reference's matMulMetalResetTuning, src/ops/matmul_metal.mm:1803-1834). */
lcError_t lcTuneCacheReset(lcTuneKind kind);
size_t lcTuneCacheSize(lcTuneKind kind);
lcError_t lcTuneCacheGet(lcTuneKind kind, size_t d0, size_t d1, size_t d2, lcDataType dtype, char* config,
                         size_t cap);
lcError_t lcTuneCacheSet(lcTuneKind kind, size_t d0, size_t d1, size_t d2, lcDataType dtype, const char* config);
/* Times every configuration that can run the shape on the given device buffers (1 warm-up +
 * median of 5, CUDA events; like autoTuneTile, src/ops/matmul_metal.mm:1643-1790), stores the
 * fastest and writes its name to `best`.  Synchronizes `stream`. */
lcError_t lcMatMulAutotune(const void* a, const void* b, void* out, size_t m, size_t k, size_t n, lcDataType dtype,
                           lcStream_t stream, char* best, size_t cap);
/* The same for attention over device [units, seq, head_dim] q / k / v / out (the per-shape mode
 * auto-tune of autoTuneForwardMode, src/attention_metal.mm:1316-1420): every kernel that can take
 * the shape is timed and the fastest is stored under (seq, head_dim, causal, dtype). */
lcError_t lcAttentionAutotune(const void* q, const void* k, const void* v, void* out, size_t units, size_t seq,
                              size_t head_dim, int causal, lcDataType dtype, lcStream_t stream, char* best,
                              size_t cap);

/* ---- multi-GPU: one process per GPU, NCCL over NVLink -----------------------------------
 * No counterpart in the reference, which runs on one device and has no collective (its batched
 * workloads are independent units: attention heads, matmul rows, conv->attention images).  These
 * shard those units across the ranks of a communicator and assemble the full output on every
 * rank with one in-place NCCL all-gather (grouped broadcasts when units do not divide evenly).
 * NCCL is loaded at run time (dlopen "libnccl.so.2"); lcCommAvailable() says whether it was found.
 * A communicator belongs to the device that was current at lcCommInitRank; call it with that
 * device current.  Shards are contiguous and balanced: rank r owns [lo, hi) of lcShardRange. */
typedef struct lcComm* lcComm_t;
typedef struct lcCommUniqueId { char internal[128]; } lcCommUniqueId; /* ncclUniqueId bytes */
int lcCommAvailable(void);
/* Rank 0 creates the id and hands it to the other ranks by any host channel. */
lcError_t lcCommGetUniqueId(lcCommUniqueId* id);
/* Collective over the nranks processes (ncclCommInitRank); binds the current device. */
lcError_t lcCommInitRank(lcComm_t* comm, int nranks, const lcCommUniqueId* id, int rank);
lcError_t lcCommDestroy(lcComm_t comm);
/* Tears the communicator down without waiting for peers (ncclCommAbort): the way out after a
 * peer failed. */
lcError_t lcCommAbort(lcComm_t comm);
lcError_t lcCommRankInfo(lcComm_t comm, int* rank, int* nranks);
lcError_t lcShardRange(size_t total, int rank, int nranks, size_t* lo, size_t* hi);
/* In-place all-gather of total_rows rows of row_bytes: this rank's rows [lo, hi) are in place in
 * the device buffer `buf`; on return (stream order) every rank holds all rows. */
lcError_t lcCommAllGatherRows(lcComm_t comm, void* buf, size_t total_rows, size_t row_bytes, lcStream_t stream);
/* lcAttentionForward / lcMatMul / lcConvAttentionNchw (per_image = 1) over a communicator.
 * Arguments describe the FULL problem, identical on every rank; each rank computes its shard of
 * units / rows of A / images.  Policies keep their single-GPU meaning per pointer:
 *   - device output (download_out = 0): after the call every rank holds the full output;
 *   - host output (download_out = 1): each rank downloads only its own rows into `out`
 *     (no gather: the host buffers of the ranks are separate);
 *   - host inputs are uploaded per shard; the matmul's replicated B (upload_b = 1) is uploaded as a
 *     1/N row slice per rank and all-gathered over NVLink into a buffer the communicator owns.
 * synchronize (or a host output) waits for the stream and reports NCCL's asynchronous errors and
 * the device error word. */
lcError_t lcAttentionForwardSharded(lcComm_t comm, const void* q, const void* k, const void* v, void* out,
                                    size_t units, size_t seq, size_t head_dim, int causal, lcDataType dtype,
                                    const lcAttentionIoPolicy* policy, lcStream_t stream);
lcError_t lcMatMulSharded(lcComm_t comm, const void* a, const void* b, void* out, size_t m, size_t k, size_t n,
                          lcDataType dtype, const lcMatMulIoPolicy* policy, lcStream_t stream);
lcError_t lcConvAttentionNchwSharded(lcComm_t comm, const float* x, const float* w, const float* bias,
                                     const float* proj_w, float* out, size_t batch, size_t in_channels, size_t in_h,
                                     size_t in_w, size_t out_channels, size_t kernel_h, size_t kernel_w,
                                     size_t stride_h, size_t stride_w, size_t pad_h, size_t pad_w, size_t seq,
                                     size_t head_dim, size_t proj_cols, const lcConv2dIoPolicy* policy,
                                     lcStream_t stream);

/* Conv kernel-mode cache: the reference chooses the 3x3 conv kernel per shape and remembers it
 * (chooseModeWithAutotune, src/ops/conv2d_metal.mm:577-672).  Here the LC_TUNE_CONV cache maps a
 * conv shape to "simt" (implicit-GEMM CUDA-core kernel), "tcgen05_implicit" (implicit-GEMM 3xTF32
 * tensor-core kernel: in_channels % 32 == 0, 16 <= out_channels <= 256, out_channels % 16 == 0) or
 * "tcgen05_3xtf32" (tensor-core 3xTF32 GEMM over an im2col split held in a workspace);
 * CJ_CONV_TUNE_CACHE_FILE persists it like the other kinds.  The shape
 * is packed into the cache's three key columns by lcConvTuneKey (channels in d0, spatial size in
 * d1, batch and kernel geometry in d2); shapes whose fields do not fit the packing
 * (channels/extent >= 2^32, batch >= 2^32, kernel >= 256, stride/pad >= 16) return
 * LC_NOT_SUPPORTED and are never cached. */
lcError_t lcConvTuneKey(size_t batch, size_t in_channels, size_t in_h, size_t in_w, size_t out_channels,
                        size_t kernel_h, size_t kernel_w, size_t stride_h, size_t stride_w, size_t pad_h,
                        size_t pad_w, size_t* d0, size_t* d1, size_t* d2);
/* Times every conv kernel that can take the shape on the given device buffers (1 warm-up + median
 * of 5), stores the fastest under the shape's key and writes its name to `best`.  Synchronizes. */
lcError_t lcConvAutotune(const float* x, const float* w, const float* bias, float* out, size_t batch,
                         size_t in_channels, size_t in_h, size_t in_w, size_t out_channels, size_t kernel_h,
                         size_t kernel_w, size_t stride_h, size_t stride_w, size_t pad_h, size_t pad_w,
                         int apply_relu, lcStream_t stream, char* best, size_t cap);

/* ---- device error word: kernels' bounded waits record where they gave up ---------------- */
/* Returns LC_DRIVER_ERROR and the recorded code if any kernel on the current device gave up a
 * bounded wait since the last clear; LC_SUCCESS otherwise.  Synchronizes the device. */
lcError_t lcGetDeviceErrorWord(unsigned int* code);
lcError_t lcClearDeviceErrorWord(void);

/* ---- test hooks (no counterpart in the reference) -----------------------------------------
 * For failure-path tests only; inert unless called.
 * lcTestFailAllocations(after, count): of the library's next device allocations, `after` succeed
 *   and the `count` after them fail (the op that needed them returns LC_OUT_OF_MEMORY, having
 *   released what it already held); count = 0 disarms.
 * lcTestStallNextGemm(kb): the next 1-SM tcgen05 GEMM launch ("tcgen05_128x256") leaves k-block kb
 *   of its first tile unloaded, so the MMA warp's bounded mbarrier wait (2 s) runs out: the kernel
 *   records the code in the device error word, drains its in-flight copies and MMAs, frees TMEM
 *   and exits; a synchronising call returns LC_DRIVER_ERROR.  No fault, trap or hang is involved. */
void lcTestFailAllocations(int after, int count);
void lcTestStallNextGemm(int kblock);

/* ---- runtime trace ring (src/runtime.cpp:63-99,620-760) ---------------------------------- */
typedef struct lcRuntimeTraceEvent {
  int type;   /* RuntimeTraceEventType: 0 malloc .. 10 op_dispatch          */
  int status; /* lcError_t                                                   */
  uint64_t timestamp_ns;
  size_t size_bytes;
  int detail0; /* op kind for op_dispatch (1 matmul .. 6 attention_forward)  */
  int detail1; /* requested | selected<<4 | fallback<<8                      */
} lcRuntimeTraceEvent;
void lcRuntimeTraceSetEnabled(int enabled);
int lcRuntimeTraceIsEnabled(void);
void lcRuntimeTraceClear(void);
size_t lcRuntimeTraceCount(void);
size_t lcRuntimeTraceCapacity(void);
lcError_t lcRuntimeTraceGet(size_t index, lcRuntimeTraceEvent* out_event);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif /* LC_B200_H */
