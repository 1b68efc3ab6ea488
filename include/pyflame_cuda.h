/*
 * pyflame_cuda.h — C ABI of the B200 graph executor for PyFlame IR graphs.
 *
 * This library evaluates a materialised PyFlame lazy IR graph (the nodes of an
 * `ir::Graph`, include/pyflame/ir/graph.hpp:17-215 in PyFlame) on an NVIDIA
 * B200 (sm_100a).  It takes the place of the ROCm executor behind PyFlame's
 * executor boundary:
 *
 *   PyFlame                                   this header
 *   -------------------------------------     -----------------------------------
 *   backend::Backend (executor.cpp:138-145)   PFC_BACKEND_CUDA added by the adapter
 *   backend::ExecutorConfig (:163-168)        pfc_executor_config
 *   backend::ExecutionResult (:148-160)       pfc_execution_result + caller buffers
 *   rocm::ROCmExecutor (rocm_executor.hpp:37) pfc_executor_*
 *   rocm::ROCmExecutor::execute (:71-74)      pfc_executor_execute
 *   rocm::get_device_count/... (rocm_backend.hpp:119-139)   pfc_cuda_*
 *   rocm::MemoryStats (rocm_memory.hpp:14-21) pfc_memory_stats
 *   kernels::launch_* extern "C" launchers (rocm_kernels.hip:740-806)
 *                                             pfk_* kernel entry points
 *
 * Conventions: every function returns 0 (PFC_OK) on success or a negative
 * PFC_ERR_* code; no C++ exception crosses this boundary.  The text of the
 * last error on the calling thread is available from pfc_last_error().
 * Pointers are plain host or device pointers; sizes are in bytes unless the
 * name says elements.  Node ids are PyFlame NodeIds (uint64, node.hpp:19).
 */
#ifndef PYFLAME_CUDA_H
#define PYFLAME_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PFC_API __attribute__((visibility("default")))
#else
#define PFC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define PFC_ABI_VERSION 1

/* ---- status codes -------------------------------------------------------- */
#define PFC_OK 0
#define PFC_ERR_INVALID_ARGUMENT (-1)
#define PFC_ERR_UNSUPPORTED (-2)
#define PFC_ERR_CUDA (-3)
#define PFC_ERR_OUT_OF_MEMORY (-4)
#define PFC_ERR_NO_DEVICE (-5)
#define PFC_ERR_GRAPH (-6)      /* malformed graph: cycle, size limit, bad edge */
#define PFC_ERR_JIT (-7)        /* NVRTC compile or module load failed */
#define PFC_ERR_TIMEOUT (-8)    /* a device-side bounded wait gave up */
#define PFC_ERR_INTERNAL (-9)

/* ---- IR enums (numeric values are PyFlame's) ----------------------------- */
/* NodeType, include/pyflame/ir/node.hpp:22-27 */
enum pfc_node_type {
    PFC_NODE_CONSTANT = 0,
    PFC_NODE_INPUT = 1,
    PFC_NODE_PARAMETER = 2,
    PFC_NODE_OPERATION = 3
};

/* DType, include/pyflame/core/dtype.hpp:11-21 */
enum pfc_dtype {
    PFC_DTYPE_FLOAT32 = 0,
    PFC_DTYPE_FLOAT16 = 1,
    PFC_DTYPE_BFLOAT16 = 2,
    PFC_DTYPE_INT32 = 3,
    PFC_DTYPE_INT16 = 4,
    PFC_DTYPE_INT8 = 5,
    PFC_DTYPE_BOOL = 6,
    PFC_DTYPE_FLOAT64 = 7,
    PFC_DTYPE_INT64 = 8
};

/* OpType codes are PyFlame's OpType values (include/pyflame/ir/op_type.hpp:9-124),
 * passed as int. */

/* Attribute value types: the C++ type a PyFlame producer stores in the node's
 * std::any attribute map (node.hpp:119-165).  The executor reads attributes
 * by the names and types the producers write (tensor_impl.cpp:530-533,
 * tensor.cpp:281-283,687, conv.cpp:114-117, normalization.cpp:85-89,246-248,
 * pooling.cpp:57-59,163-164). */
enum pfc_attr_type {
    PFC_ATTR_INT32 = 0,     /* int */
    PFC_ATTR_INT64 = 1,     /* int64_t */
    PFC_ATTR_FLOAT32 = 2,   /* float */
    PFC_ATTR_FLOAT64 = 3,   /* double */
    PFC_ATTR_BOOL = 4,      /* bool */
    PFC_ATTR_INT64_VEC = 5, /* std::vector<int64_t> */
    PFC_ATTR_INT32_VEC = 6, /* std::vector<int> */
    PFC_ATTR_FLOAT32_VEC = 7
};

/* Flags for constant payloads (pfc_graph_set_constant). */
#define PFC_CONST_COPY 0x1     /* copy the bytes now (default: borrow; the pointer must stay valid while
                                  the graph is executed) */
#define PFC_CONST_RESIDENT 0x2 /* immutable weights: the device copy is kept across execute calls under
                                  (cache_key, size); payloads with equal key and size must hold equal bytes */

/* Matmul precision for fp32 contractions. */
enum pfc_precision {
    PFC_PRECISION_TF32X3 = 0, /* fp32-accurate: 3 tcgen05 kind::tf32 products of split hi/lo operands */
    PFC_PRECISION_BF16 = 1    /* bf16 operands, fp32 accumulate: one kind::f16 product */
};

/* ---- device functions (mirror rocm_backend.hpp:119-139) ------------------ */
typedef struct pfc_device_info {
    int device_id;
    char name[256];
    char architecture[32]; /* "sm_100" */
    size_t total_memory;
    size_t free_memory;
    int compute_units;     /* SM count */
    int max_threads_per_block;
    int warp_size;
} pfc_device_info;

PFC_API int pfc_cuda_is_available(void); /* 1 if at least one sm_100 device is visible */
PFC_API int pfc_cuda_get_device_count(int* count);
PFC_API int pfc_cuda_get_device_info(int device_id, pfc_device_info* info);
PFC_API int pfc_cuda_set_device(int device_id);
PFC_API int pfc_cuda_get_device(int* device_id);
PFC_API int pfc_cuda_synchronize(void);

PFC_API const char* pfc_last_error(void);
PFC_API int pfc_abi_version(void);

/* ---- graph description --------------------------------------------------- */
/* A pfc_graph holds the nodes of one PyFlame ir::Graph: the same ids, node
 * types, OpTypes, output TensorSpecs (shape + dtype), input edges, typed
 * attributes and constant payloads.  It is built once and may be executed
 * many times; the executor caches its compiled plan against the graph's
 * structure. */
typedef struct pfc_graph pfc_graph;

PFC_API int pfc_graph_create(pfc_graph** out);
PFC_API int pfc_graph_destroy(pfc_graph* g);
/* Graph::create_constant/create_input/create_parameter/create_op (graph.hpp:31-100) */
PFC_API int pfc_graph_add_node(pfc_graph* g, uint64_t id, int node_type, int op_type, int dtype,
                       int ndim, const int64_t* shape, int n_inputs, const uint64_t* input_ids);
/* Node::set_attr (node.hpp:119-121).  `count` is the element count of vector
 * types; scalar types read one element of the matching C type from `value`. */
PFC_API int pfc_graph_set_attr(pfc_graph* g, uint64_t id, const char* key, int attr_type,
                       const void* value, int64_t count);
/* Node::set_constant_data (node.hpp:175-177).  `bytes` must equal the node's
 * TensorSpec::size_bytes (node.hpp:46-48).  `cache_key` names the payload
 * for PFC_CONST_RESIDENT (ignored otherwise); it must never be reused for
 * different bytes of the same size. */
PFC_API int pfc_graph_set_constant(pfc_graph* g, uint64_t id, const void* data, size_t bytes,
                           uint32_t flags, uint64_t cache_key);
/* Graph::mark_output (graph.hpp:109-113) */
PFC_API int pfc_graph_mark_output(pfc_graph* g, uint64_t id);
PFC_API int pfc_graph_num_nodes(const pfc_graph* g, int64_t* n);

/* ---- executor ------------------------------------------------------------ */
typedef struct pfc_executor pfc_executor;

/* rocm::ROCmExecutor::Config (rocm_executor.hpp:40-47) plus the B200 additions. */
typedef struct pfc_executor_config {
    int device_id;            /* GPU device to use */
    int enable_profiling;     /* time each launch with CUDA events (pfc_executor_last_profile) */
    int sync_after_launch;    /* synchronise and check after each launch (debug) */
    size_t workspace_size_mb; /* pool release threshold: bytes kept cached between calls */
    int precision;            /* pfc_precision for fp32 MATMUL/CONV2D */
    int use_cuda_graph;       /* replay a captured CUDA graph of each compiled plan */
    int fail_after_n_allocations; /* >0: the Nth device allocation fails (host-side fault injection) */
} pfc_executor_config;

PFC_API void pfc_executor_config_default(pfc_executor_config* cfg);

/* ExecutionResult (executor.cpp:148-160) minus the output map: outputs are
 * written into the caller's buffers. */
typedef struct pfc_execution_result {
    int success;
    char error_message[1024];
    double compile_time_ms;
    double transfer_time_ms;
    double compute_time_ms;
    double total_time_ms;
    int64_t kernel_launches; /* device launches issued by this call */
    uint64_t h2d_bytes;      /* host->device bytes this call copied (inputs, constants not yet resident) */
    uint64_t d2h_bytes;      /* device->host bytes this call copied (outputs) */
} pfc_execution_result;

/* rocm::MemoryStats (rocm_memory.hpp:14-21) */
typedef struct pfc_memory_stats {
    size_t total_allocated;
    size_t peak_allocated;
    size_t total_allocations;
    size_t total_deallocations;
    size_t cache_hits;
    size_t cache_misses;
    size_t resident_constant_bytes;
} pfc_memory_stats;

PFC_API int pfc_executor_create(const pfc_executor_config* cfg, pfc_executor** out);
PFC_API int pfc_executor_destroy(pfc_executor* ex);

/* ROCmExecutor::execute (rocm_executor.cpp:66-161): evaluate `output_ids` of
 * `g`.  Constants are uploaded (or found resident), the plan runs on the
 * executor's stream, and each requested output is copied into
 * `out_host[i]`, a host buffer of `out_bytes[i]` bytes (dense row-major, the
 * node's dtype).  Ids not present in the graph fail the call.  On failure
 * `result->success` is 0 and `result->error_message` says why; the return
 * value is the matching PFC_ERR_* code. */
PFC_API int pfc_executor_execute(pfc_executor* ex, pfc_graph* g, const uint64_t* output_ids,
                         int n_outputs, void* const* out_host, const size_t* out_bytes,
                         pfc_execution_result* result);

/* Device-resident variant: the data of the INPUT/CONSTANT nodes listed in
 * `input_ids` is read from device pointers `in_dev` (dense row-major) instead
 * of host payloads, and outputs are written to device pointers `out_dev`.
 * Work is issued on `stream` (a cudaStream_t; NULL = the executor's stream)
 * and the call returns without synchronising. */
PFC_API int pfc_executor_execute_device(pfc_executor* ex, pfc_graph* g, const uint64_t* input_ids,
                                int n_inputs, const void* const* in_dev,
                                const uint64_t* output_ids, int n_outputs,
                                void* const* out_dev, void* stream,
                                pfc_execution_result* result);

/* Streamed host-buffer execution for graphs whose rows are independent (no
 * op mixes rows of dim 0, as for batch sharding): `g` describes one chunk of
 * rows, and the host arrays hold `n_chunks` chunks back to back (input i of
 * chunk c at in_host[i] + c * size_bytes(input_ids[i]), outputs likewise).
 * Chunk c+1's inputs are copied in and chunk c-1's outputs copied out while
 * chunk c computes (three streams, two device slots per tensor), so a step
 * costs about the largest of the three instead of their sum.  Host memory
 * must be pinned for the copies to overlap.  Synchronous: returns when every
 * output is on the host.  No counterpart in the reference (ROCmExecutor
 * copies and computes one graph serially, rocm_executor.cpp:66-161). */
PFC_API int pfc_executor_execute_streamed(pfc_executor* ex, pfc_graph* g, const uint64_t* input_ids,
                                          int n_inputs, const void* const* in_host,
                                          const uint64_t* output_ids, int n_outputs,
                                          void* const* out_host, int n_chunks,
                                          pfc_execution_result* result);

PFC_API int pfc_executor_get_device_info(pfc_executor* ex, pfc_device_info* info);
PFC_API int pfc_executor_get_memory_stats(pfc_executor* ex, pfc_memory_stats* stats);
/* Drop every resident constant and compiled plan. */
PFC_API int pfc_executor_release_constants(pfc_executor* ex);
/* Use caller-owned device memory as the resident copy of every constant
 * whose payload key is `cache_key` and whose size is `bytes` (the pair given
 * to pfc_graph_set_constant with PFC_CONST_RESIDENT), instead of uploading
 * the host payload.  For weights that arrive on the device by other means,
 * e.g. broadcast from rank 0 over NCCL.  The executor reads the memory and
 * never writes or frees it; it must stay valid and unchanged until
 * pfc_executor_release_constants or pfc_executor_destroy.  Tensor-core
 * operands derived from earlier contents are rebuilt on next use.  No
 * counterpart in the reference (ROCmExecutor re-uploads constants on every
 * call, rocm_executor.cpp:93-103). */
PFC_API int pfc_executor_set_resident(pfc_executor* ex, uint64_t cache_key, const void* dev_ptr,
                                      size_t bytes);
/* Human-readable description of the compiled plan for (g, output_ids):
 * kernels, fusion groups and buffers.  Writes a NUL-terminated string. */
PFC_API int pfc_executor_describe_plan(pfc_executor* ex, pfc_graph* g, const uint64_t* output_ids,
                               int n_outputs, char* buf, size_t buf_len);
/* Build the plan for (g, output_ids) and compile every generated kernel for
 * sm_100a, without a device (no allocation, no launch).  Writes the plan
 * description.  Used to check graphs and code generation on build hosts. */
PFC_API int pfc_compile_check(pfc_graph* g, const uint64_t* output_ids, int n_outputs, int precision,
                              char* buf, size_t buf_len);
/* Per-launch device times of the last execute (enable_profiling=1):
 * up to `cap` entries of (kernel name, milliseconds). */
PFC_API int pfc_executor_last_profile(pfc_executor* ex, char (*names)[64], double* ms, int cap,
                              int* count);

/* ---- kernel entry points ------------------------------------------------- */
/* Each takes device pointers and launches on `stream` (cudaStream_t, may be
 * NULL).  They allocate nothing, except where a comment says otherwise. */

/* Split an fp32 matrix view into tcgen05 operands: hi = x with the low 13
 * mantissa bits cleared, lo = x - hi, each [batch][rows][kpad] K-major,
 * zero padded for k >= cols.  Element (b, r, k) of the source is read at
 * src[b*sb + r*sr + k*sk]. */
PFC_API int pfk_split_tf32(const float* src, int64_t batch, int64_t rows, int64_t cols, int64_t sb,
                   int64_t sr, int64_t sk, float* hi, float* lo, int64_t kpad, void* stream);
/* Same view converted to bf16 (round to nearest even), K padded to kpad. */
PFC_API int pfk_convert_bf16(const float* src, int64_t batch, int64_t rows, int64_t cols, int64_t sb,
                     int64_t sr, int64_t sk, uint16_t* out, int64_t kpad, void* stream);

/* Epilogue of the tensor-core GEMM: v = alpha*acc (+ bias[n]); v = act(v);
 * (+ residual[b,m,n]); C[b,m,n] = v.  act: 0 none, 1 relu, 2 gelu(tanh form),
 * 3 sigmoid, 4 tanh, 5 silu. */
typedef struct pfk_gemm_epilogue {
    float alpha;
    const float* bias;        /* [N] or NULL */
    int act;
    const float* residual;    /* or NULL */
    int64_t res_sb, res_sm, res_sn;
} pfk_gemm_epilogue;

/* C[b,m,n] = sum_k A[b,m,k] * B[b,n,k] on tcgen05 tensor cores, TMA-fed,
 * accumulating in TMEM.  precision PFC_PRECISION_TF32X3: a_hi/a_lo/b_hi/b_lo
 * are pfk_split_tf32 outputs; PFC_PRECISION_BF16: a_hi/b_hi are bf16
 * (pfk_convert_bf16) and a_lo/b_lo are ignored.  kpad is the padded K of the
 * operands (multiple of 32 for tf32x3, of 64 for bf16).  a_sb/b_sb are batch
 * strides in elements (0 broadcasts).  C element (b,m,n) is at
 * c[b*c_sb + m*c_sm + n*c_sn].  `err` is a device int that receives a
 * nonzero code if a bounded wait inside the kernel expired. */
PFC_API int pfk_gemm(int precision, const void* a_hi, const void* a_lo, int64_t a_sb, const void* b_hi,
             const void* b_lo, int64_t b_sb, int64_t batch, int64_t M, int64_t N, int64_t K,
             int64_t kpad, float* c, int64_t c_sb, int64_t c_sm, int64_t c_sn,
             const pfk_gemm_epilogue* epi, int* err, void* stream);

/* im2col for Conv2d as implicit GEMM (conv.cpp:75-131 attribute contract):
 * x is [N,C,H,W] addressed through strides (sn,sc,sh,sw) in elements; row
 * m = ((n*OH)+oh)*OW+ow, column k = (c*KH+kh)*KW+kw, zero outside the padded
 * input.  Output is tf32x3 hi/lo (or bf16 when lo == NULL and bf16 != NULL). */
PFC_API int pfk_im2col(const float* x, int64_t n, int64_t c, int64_t h, int64_t w, int64_t sn,
               int64_t sc, int64_t sh, int64_t sw, int64_t kh, int64_t kw, int64_t stride_h,
               int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dil_h, int64_t dil_w,
               int64_t oh, int64_t ow, float* hi, float* lo, uint16_t* bf16, int64_t kpad,
               void* stream);

/* MaxPool2d / AvgPool2d (pooling.cpp:38-63,97-122) and AdaptiveAvgPool2d
 * (pooling.cpp:150-168) over a strided [N,C,H,W] view; output dense NCHW or
 * through output strides.  mode: 0 max, 1 avg (count includes padding, like
 * PyTorch's default), 2 adaptive avg. */
typedef struct pfk_pool_params {
    int mode;
    int64_t n, c, h, w;
    int64_t sn, sc, sh, sw;
    int64_t kh, kw, stride_h, stride_w, pad_h, pad_w;
    int64_t oh, ow;
    int64_t osn, osc, osh, osw;
} pfk_pool_params;
PFC_API int pfk_pool2d(const float* x, float* y, const pfk_pool_params* p, void* stream);

/* C[M,N] = A[M,K] @ B[K,N], all fp32 dense row-major, on the 3xTF32 tcgen05
 * GEMM, allocating nothing: the split operands and the wait-timeout flag live
 * in a fixed 64 MiB device array inside the library (one per device), for
 * hosts that cannot grant the library device memory or must not call
 * cudaMalloc/cudaFree on this path.  It has no counterpart in the reference.
 * The array occupies 64 MiB on every device once this library's device code
 * is loaded there (under CUDA_MODULE_LOADING=EAGER, at context creation),
 * whether or not this entry point is ever called.  Needs 256 + 2*ru(4*M*Kp) + 2*ru(4*N*Kp) bytes, Kp = K rounded up to 32,
 * ru = round up to 256; larger problems return PFC_ERR_INVALID_ARGUMENT.
 * All calls share the array, so overlapping calls race: serialise them (one
 * stream).  The first call on a device sets up the array's address; make it
 * before any stream capture begins.  `err`: optional device int receiving the
 * kernel's wait-timeout code (0 = none) in stream order. */
PFC_API int pfk_matmul_tf32x3_static(const float* a, const float* b, float* c, int64_t M, int64_t N,
                                     int64_t K, int* err, void* stream);

/* Self-check of the failure path every tensor-core kernel shares: launches
 * one CTA whose mbarrier wait can never complete, bounded by the global timer
 * like all device waits here; after `limit_us` (at most 5 s) it records
 * PFC_ERR_TIMEOUT in the device int *err (left as is if already non-zero)
 * and the kernel returns.  Nothing faults or hangs and the context stays
 * usable.  No counterpart in the reference. */
PFC_API int pfk_check_bounded_wait(int* err, int64_t limit_us, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PYFLAME_CUDA_H */
