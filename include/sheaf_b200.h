/*
 * sheaf_b200.h - C ABI of libsheafb200, the B200 (sm_100a) execution backend
 * for Sheaf's JIT-compiled StableHLO graphs.
 *
 * The library takes the place of the IREE compile-and-run layer that Sheaf
 * drives through its hand-written FFI (sheaf/src/runtime/iree_ffi.rs:133-275).
 * Conventions kept from that interface:
 *   - status objects: a NULL `sb_status*` means success; a non-NULL status is
 *     heap-allocated and owned by the caller, who frees it with
 *     sb_status_free (iree_status_t, iree_ffi.rs:17, 129-131);
 *   - element type codes are IREE's (iree_ffi.rs:32-34);
 *   - buffers are reference counted (retain/release) like
 *     iree_hal_buffer_view_t;
 *   - functions are called by qualified name "<module>.<function>"
 *     (iree_runtime_session_call_by_name, iree_ffi.rs:190-195).
 * Instead of a precompiled .vmfb, a module is loaded from the StableHLO text
 * that Sheaf emits (sheaf/src/lowering/stablehlo/emit.rs:253-273); the library
 * plans, fuses and compiles it for the GPU itself.
 */
#ifndef SHEAF_B200_H_
#define SHEAF_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SB_API __attribute__((visibility("default")))

typedef struct sb_status sb_status;
typedef struct sb_session sb_session;
typedef struct sb_buffer sb_buffer;

typedef enum sb_status_code {
  SB_STATUS_OK = 0,
  SB_STATUS_INVALID_ARGUMENT = 3,
  SB_STATUS_DEADLINE_EXCEEDED = 4,
  SB_STATUS_NOT_FOUND = 5,
  SB_STATUS_RESOURCE_EXHAUSTED = 8,
  SB_STATUS_FAILED_PRECONDITION = 9,
  SB_STATUS_UNIMPLEMENTED = 12,
  SB_STATUS_INTERNAL = 13,
  SB_STATUS_UNAVAILABLE = 14,
} sb_status_code;

/* Element types: the IREE HAL codes (iree_ffi.rs:32-34). */
#define SB_ELEMENT_TYPE_FLOAT_32 ((0x21u << 24) | 32u)
#define SB_ELEMENT_TYPE_BFLOAT_16 ((0x31u << 24) | 16u)
#define SB_ELEMENT_TYPE_INT_32 ((0x11u << 24) | 32u)

/* Arithmetic used for dot_general contractions of f32 tensors.  Other ops
 * compute in the graph's types (f32; bf16 tensors as bf16, rounding every op's
 * result).  A dot_general of bf16 tensors always runs on tcgen05 kind::f16. */
typedef enum sb_precision {
  SB_PRECISION_FP32 = 0, /* f32 FMA on CUDA cores */
  SB_PRECISION_TF32 = 1, /* tcgen05 kind::tf32 on operands rounded to nearest TF32, f32 accumulate */
  SB_PRECISION_BF16 = 2, /* GEMM operands converted to bf16 (round to nearest even), tcgen05 kind::f16,
                            f32 accumulate; fused attention in TF32 */
} sb_precision;

/* How an output of a data-parallel call is combined across ranks. */
typedef enum sb_reduce_op {
  SB_REDUCE_NONE = 0, /* keep the local value */
  SB_REDUCE_SUM = 1,
  SB_REDUCE_MEAN = 2,
} sb_reduce_op;

typedef struct sb_session_options {
  int32_t device_ordinal;       /* CUDA device used by this session */
  int32_t precision;            /* sb_precision */
  int32_t rank;                 /* data-parallel rank (0 when world_size == 1) */
  int32_t world_size;           /* number of ranks; 1 = single GPU, no NCCL */
  uint8_t nccl_unique_id[128];  /* from sb_nccl_get_unique_id on rank 0 */
  int64_t collective_timeout_ms;/* host deadline for collectives; <= 0 = 600000 */
  const char* kernel_cache_dir; /* compiled-kernel cache; NULL = $SHEAF_B200_CACHE or default */
  uint32_t flags;               /* SB_SESSION_FLAG_* */
} sb_session_options;

/* Launch every call's kernels one by one.  By default a function's calls from
 * the second on replay a CUDA graph of its steps (one launch per call). */
#define SB_SESSION_FLAG_NO_CUDA_GRAPH 1u
/* TF32: keep the attention region on the generic fused-loop + GEMM path instead
 * of the fused tcgen05 attention kernels (for A/B parity checks). */
#define SB_SESSION_FLAG_NO_ATTENTION_FUSION 2u
/* Data parallel (world_size > 1): all-reduce the reduced outputs (the
 * gradients) in buckets on a second stream as soon as the backward has
 * written them, overlapping the rest of the backward; without it one grouped
 * all-reduce runs after the last step. */
#define SB_SESSION_FLAG_OVERLAP_ALLREDUCE 4u

typedef struct sb_allocator_stats {
  /* field meaning follows iree_hal_allocator_statistics_t as read by
   * sheaf/src/interpreter/mem_profile.rs:123 */
  uint64_t host_bytes_peak, host_bytes_allocated, host_bytes_freed;
  uint64_t device_bytes_peak, device_bytes_allocated, device_bytes_freed;
} sb_allocator_stats;

/* --- status (iree_status_t: iree_ffi.rs:17, 129-131, 268-269) ------------ */
SB_API sb_status_code sb_status_code_of(const sb_status* status);
SB_API const char* sb_status_message(const sb_status* status);
SB_API void sb_status_free(sb_status* status);

/* --- session (iree_runtime_instance/session_create*: iree_ffi.rs:141-177;
 *     IreeSession::new, sheaf/src/runtime/iree_session.rs:174) ----------- */
SB_API void sb_session_options_initialize(sb_session_options* options);
SB_API sb_status* sb_session_create(const sb_session_options* options, sb_session** out_session);
SB_API void sb_session_release(sb_session* session);
SB_API sb_status* sb_session_synchronize(sb_session* session);
SB_API sb_status* sb_session_allocator_stats(sb_session* session, sb_allocator_stats* out_stats);
/* The cudaStream_t all of the session's work is ordered on (for event timing
 * and for ordering work of other CUDA users against the session). */
SB_API void* sb_session_cuda_stream(sb_session* session);
/* Per-step CUDA-event timing (the B200 counterpart of `--jit-profile`,
 * sheaf/src/runtime/iree_session.rs:158-167, 813-849).  While enabled, every
 * kernel launch of every call is bracketed by events on the session stream. */
SB_API sb_status* sb_session_set_profiling(sb_session* session, int enable);
/* CSV, one row per plan step with accumulated device time:
 * function,step,kind,kernel,calls,total_ms,elements,bytes,flops,launches_per_call
 * Synchronizes the stream.  `reset` clears the accumulators afterwards. */
SB_API sb_status* sb_session_profile_report(sb_session* session, int reset, char* out, size_t capacity,
                                            size_t* out_length);

/* --- module loading (replaces `iree-compile` + append_bytecode_module_from_memory:
 *     sheaf/src/runtime/jit/vag.rs:726-794, iree_ffi.rs:180-184,
 *     IreeSession::load_vmfb, iree_session.rs:373) ------------------------ */
SB_API sb_status* sb_session_load_stablehlo(sb_session* session, const char* text, size_t length);
SB_API int sb_session_has_function(sb_session* session, const char* qualified_name);

/* --- calls (iree_runtime_session_call_by_name: iree_ffi.rs:187-192;
 *     IreeSession::call_device, iree_session.rs:574) ---------------------- *
 * inputs are borrowed; each returned output carries one reference owned by the
 * caller.  `output_reduce` (may be NULL) gives an sb_reduce_op per output for
 * data-parallel sessions; NULL means SB_REDUCE_NONE for every output.
 * From the second call of a function on, the call replays a CUDA graph of its
 * steps (and, data parallel, of its all-reduce): the outputs then live in one
 * of up to 4 output sets of the function, reused by a later call once every
 * output of the set has been released; a call finding all sets held runs
 * eagerly into fresh buffers.  Inputs whose address changes between calls are
 * copied into library-owned staging buffers by the replay. */
SB_API sb_status* sb_session_call(sb_session* session, const char* qualified_name,
                                  sb_buffer* const* inputs, size_t input_count,
                                  const int32_t* output_reduce,
                                  sb_buffer** outputs, size_t output_capacity,
                                  size_t* out_output_count);

/* --- buffers (iree_hal_buffer_view_*: iree_ffi.rs:195-242) --------------- */
SB_API sb_status* sb_buffer_allocate_copy(sb_session* session, size_t rank, const uint64_t* shape,
                                          uint32_t element_type, const void* host_data,
                                          size_t byte_length, sb_buffer** out_buffer);
/* Wraps caller-owned device memory without copying; the caller keeps it alive.
 * The pointer must be 16-byte aligned (vector loads and TMA read it directly). */
SB_API sb_status* sb_buffer_wrap_device(sb_session* session, size_t rank, const uint64_t* shape,
                                        uint32_t element_type, void* device_ptr, size_t byte_length,
                                        sb_buffer** out_buffer);
/* Blocking device-to-host copy (iree_hal_device_transfer_d2h, iree_ffi.rs:223-231),
 * bounded by timeout_ms (<= 0: no bound). */
SB_API sb_status* sb_buffer_d2h(sb_session* session, sb_buffer* buffer, void* host_data,
                                size_t byte_length, int64_t timeout_ms);
SB_API void sb_buffer_retain(sb_buffer* buffer);
SB_API void sb_buffer_release(sb_buffer* buffer);
SB_API size_t sb_buffer_rank(const sb_buffer* buffer);
SB_API uint64_t sb_buffer_dim(const sb_buffer* buffer, size_t index);
SB_API uint32_t sb_buffer_element_type(const sb_buffer* buffer);
SB_API size_t sb_buffer_byte_length(const sb_buffer* buffer);
SB_API void* sb_buffer_device_pointer(const sb_buffer* buffer);

/* --- ahead-of-time bundles (the `sheaf build` .vmfb path) ------------------ *
 * Replaces compiling a module to a .vmfb ahead of time and loading it
 * (runtime/vmfb_loader.rs:24; the __sheaf__/ manifest cache, jit/support.rs:
 * 131-164).  sb_module_build_bundle plans `text` and compiles every fused
 * kernel for sm_100a on the host (no GPU needed) into one self-contained
 * buffer: call with out = NULL to get the size in *out_length, then with a
 * buffer of at least that size.  sb_session_load_bundle loads it without
 * compiling anything (the plan is rebuilt from the embedded text, the cubins
 * come from the bundle); the session's precision and planning flags must be
 * the ones the bundle was built with, and a bundle from another library
 * version whose kernels differ is rejected. */
SB_API sb_status* sb_module_build_bundle(const char* text, size_t length, int32_t precision, uint32_t flags,
                                         uint8_t* out, size_t capacity, size_t* out_length);
SB_API sb_status* sb_session_load_bundle(sb_session* session, const uint8_t* data, size_t length);

/* --- fused optimizer step -------------------------------------------------- *
 * Replaces lib/optim.shf:72-83 (global-norm, clip-by-global-norm) followed by
 * lib/optim.shf:36-58 (adamw-step), as examples/nanoGPT/train.shf:26-33 calls
 * them after every value-and-grad.  For each leaf i (params[i], grads[i],
 * m[i], v[i]: f32 buffers of one element count, on this session's device),
 * in place on the session stream:
 *   norm = sqrt(sum over all leaves of sum(g^2))        (before clipping)
 *   g'   = g * min(1, max_grad_norm / (norm + 1e-8))     (if max_grad_norm > 0)
 *   m    = beta1 m + (1 - beta1) g'
 *   v    = beta2 v + (1 - beta2) g'^2
 *   p    = p - lr (weight_decay p + (m bc_m) / (sqrt(v bc_v) + epsilon)),
 *          bc_m = 1 / (1 - beta1^(step+1)), bc_v = 1 / (1 - beta2^(step+1)).
 * `step` is the t passed to adamw-step (the update uses t + 1; the caller
 * keeps t).  Gradients are read only.  The norm is a fixed-order sum:
 * results are deterministic.  When out_global_norm is non-NULL the call waits
 * for the step and stores the pre-clip norm there; otherwise it returns once
 * the work is enqueued. */
typedef struct sb_adamw_options {
  float learning_rate, beta1, beta2, epsilon, weight_decay;
  float max_grad_norm; /* > 0: clip by global norm first; <= 0: no clipping */
  int64_t step;
} sb_adamw_options;
SB_API void sb_adamw_options_initialize(sb_adamw_options* options);
SB_API sb_status* sb_optimizer_adamw_step(sb_session* session, size_t leaf_count, sb_buffer* const* params,
                                          sb_buffer* const* grads, sb_buffer* const* m, sb_buffer* const* v,
                                          const sb_adamw_options* options, float* out_global_norm);

/* --- allocation-free GEMM --------------------------------------------------- *
 * No counterpart in the reference.  For callers that must not allocate device
 * memory: code running under another framework's memory manager, which owns
 * every device byte, or latency-critical paths that may not touch the CUDA
 * allocator.  Computes C = A @ B for row-major f32 device matrices A (m x k),
 * B (k x n), C (m x n) on the current device with the CUDA-core GEMM, enqueued
 * on `cuda_stream` (NULL = default stream); it allocates nothing.  When the
 * output has too few tiles to fill the GPU, K is split and the partial
 * products go to a static device array of SB_GEMM_SPLITK_NOALLOC_MAX_FLOATS
 * floats (16 MiB, present on every GPU that loads this library until the
 * process exits).  Calls whose partials would exceed it return
 * SB_STATUS_RESOURCE_EXHAUSTED and launch nothing.  The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress); make that first
 * call before any stream capture.  The address is kept for the life of the
 * device's primary context: after a device reset in the same process this
 * entry point must not be called again.  m is at most 65535 * 128 (one
 * CUDA-core launch); larger m returns SB_STATUS_INVALID_ARGUMENT.  All calls
 * on a device share the array:
 * calls that overlap on the GPU race on it, so serialize them.  Returns
 * SB_STATUS_OK, SB_STATUS_INVALID_ARGUMENT, SB_STATUS_RESOURCE_EXHAUSTED,
 * SB_STATUS_UNAVAILABLE (no device / array not reachable) or
 * SB_STATUS_INTERNAL (launch failure). */
#define SB_GEMM_SPLITK_NOALLOC_MAX_FLOATS (4u << 20)
SB_API sb_status_code sb_gemm_f32_splitk_noalloc(const float* a, const float* b, float* c, int64_t m, int64_t n,
                                                 int64_t k, void* cuda_stream);

/* --- collectives ---------------------------------------------------------- */
SB_API sb_status* sb_nccl_get_unique_id(uint8_t out_id[128]);

/* --- host-only inspection (no GPU needed) --------------------------------- *
 * Parses and plans `text`, compiles its fused kernels, and writes a one-line
 * summary per function into `report` (NUL-terminated, truncated to capacity). */
SB_API sb_status* sb_module_inspect(const char* text, size_t length, int32_t precision,
                                    char* report, size_t report_capacity);
/* CSV of the execution plan of one function, one row per step:
 * step,kind,kernel,elements,bytes,flops,batch,M,N,K,sab,sam,sak,sbb,sbk,sbn,epi,deferred_sums,root_offset
 * (epi: 1 when a GEMM step also writes gelu of its result, fused into its
 * epilogue; deferred_sums: column sums of a row group that the runtime may
 * finish later, batched with other steps'; root_offset: byte offset of the
 * step's result (of the copy, for an operand conversion) in the call's work
 * arena, -1 for a returned value, which has a buffer of its own) */
SB_API sb_status* sb_module_plan_steps(const char* text, size_t length, const char* function, int32_t precision,
                                       char* out, size_t capacity, size_t* out_length);
/* Writes the generated CUDA source of one function (for diagnostics). */
SB_API sb_status* sb_module_kernel_source(const char* text, size_t length, const char* function,
                                          char* out, size_t capacity, size_t* out_length);

/* Library version string. */
SB_API const char* sb_version(void);

/* Number of CUDA kernels this library has launched in this process (all
 * sessions and devices): generated loop / reduction kernels, tensor-core
 * GEMMs and their split-K reductions and operand copies, attention, sort and
 * optimizer kernels.  Diagnostics: the difference across a call is the
 * number of kernels that call launched. */
SB_API uint64_t sb_kernel_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* SHEAF_B200_H_ */
