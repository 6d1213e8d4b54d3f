/*
 * b2g.h — C ABI of the B200 (sm_100a) fp16/bf16 GEMM family: C[M,N] = A[M,K] · B[K,N], fp32 accumulate.
 *
 * This ABI replaces what the reference compiles just in time through Triton:
 *   - `_matmul_kernel` launch            kernels/triton_matmul.py:38-82 (kernel), :120-130 (SPLIT_K == 1 launch)
 *   - `_splitk_reduce_kernel` launch     kernels/triton_matmul.py:85-92 (kernel), :132-146 (SPLIT_K > 1 launch)
 *   - `TritonMatmul.make_runner`          kernels/triton_matmul.py:103-147 (allocate once, launch many times)
 *   - `even_k`, `grid`                    kernels/triton_matmul.py:95-100
 *   - the compile failures `validate` turns into invalid candidates   tune/correctness.py:147-149
 *
 * Plain pointers and sizes only: no torch types cross this boundary. Device pointers are raw CUDA device addresses on
 * the calling thread's current device; `stream` is a cudaStream_t passed as void*. Every entry point is re-entrant:
 * the library keeps no mutable global state besides per-device one-time kernel attribute set-up behind a mutex.
 *
 * Errors: functions return B2G_OK (0) or a negative B2G_ERR_* code. `b2g_last_error()` returns a thread-local
 * message describing the last failure on the calling thread. A kernel whose bounded device-side wait ran out writes a
 * non-zero code into the caller's device status word (see b2g_status_string) and returns; the context stays usable.
 */
#ifndef B2G_H_
#define B2G_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2G_ABI_VERSION 1

/* return codes */
#define B2G_OK 0
#define B2G_ERR_INVALID_ARG (-1)  /* null pointer, negative size, bad dtype */
#define B2G_ERR_UNSUPPORTED (-2)  /* config/shape/layout combination this family cannot run; reason in last_error */
#define B2G_ERR_WORKSPACE (-3)    /* workspace missing or smaller than b2g_workspace_size() */
#define B2G_ERR_CUDA (-4)         /* a CUDA runtime/driver call failed; message in last_error */

/* element types of A, B and C (A and B always share one type; C has it too) */
#define B2G_DTYPE_F16 0
#define B2G_DTYPE_BF16 1

/* tile schedules */
#define B2G_SCHED_PERSISTENT 0 /* one CTA per SM slot walks the tiles (default) */
#define B2G_SCHED_TILE 1       /* one CTA per (tile, split): the reference's launch grid, kernels/triton_matmul.py:99-100 */
#define B2G_SCHED_STREAMK 2    /* persistent workers share tiles x K blocks evenly; split tiles are finished in K order
                                  by the worker holding their first K block. Needs SPLIT_K = 1 and a workspace whose
                                  first bytes (the fix-up flags) are zero before the first launch; the kernels leave
                                  them zero. After a device status error, zero the workspace again. */

/*
 * One kernel variant. The first seven fields mean what MatmulConfig's fields mean (kernels/triton_matmul.py:20-28):
 * output tile BLOCK_M x BLOCK_N, K step BLOCK_K, GROUP_M tile-rows per L2 group, SPLIT_K deterministic K splits.
 * num_warps is the number of epilogue warps (4 or 8); num_stages the depth of the shared-memory ring.
 * BLOCK_M <= 64 selects the swapped-operand (skinny M) form: the tensor-core M side covers BLOCK_N columns of C and
 * the N side covers BLOCK_M rows of C.
 * cluster = 2 computes each tile with a CTA pair on two SMs (cta_group::2 MMAs of M = 256): BLOCK_M = 256 (or, in the
 * skinny form, BLOCK_N = 256) is split into two 128-row halves, each CTA loading its half of A and half of B.
 */
typedef struct b2g_config {
  int32_t block_m;
  int32_t block_n;
  int32_t block_k;
  int32_t num_warps;
  int32_t num_stages;
  int32_t group_m;
  int32_t split_k;
  int32_t schedule; /* B2G_SCHED_* */
  int32_t cluster;  /* 1: one CTA per tile; 2: a CTA pair per tile */
  /* Limit of every bounded device-side wait, in microseconds; 0 selects the default of one second. A wait that runs
     out writes its code to the status word and the kernel stops early (C is then incomplete). Single-CTA variants
     only: with cluster = 2 a non-zero value is B2G_ERR_UNSUPPORTED, because a pair that stops early cannot wait out
     the copies its second CTA already issued. */
  int32_t wait_limit_us;
  int32_t reserved[6];
} b2g_config;

/*
 * Problem: element (i, j) of X lives at X + i*stride_x0 + j*stride_x1 (element strides). The reference passes the same
 * six strides to its kernel (kernels/triton_matmul.py:42, :124). Any strides are accepted; layouts the tensor-memory
 * loader cannot read directly are staged through the workspace first.
 */
typedef struct b2g_problem {
  int64_t M, N, K;
  int64_t stride_am, stride_ak;
  int64_t stride_bk, stride_bn;
  int64_t stride_cm, stride_cn;
  int32_t dtype; /* B2G_DTYPE_* */
  int32_t reserved;
} b2g_problem;

typedef struct b2g_plan b2g_plan; /* opaque: tensor maps + launch geometry for one (config, problem, pointers) */

/* library identity */
int32_t b2g_abi_version(void);
const char* b2g_version(void);
/* hash of the CUDA sources and build flags this library was compiled from; a stored config key names the kernel that
   hash identifies (the role kernel_src_hash plays for the Triton source, tune/winner_cache.py:76-79) */
const char* b2g_source_hash(void);
const char* b2g_last_error(void);
const char* b2g_error_string(int32_t code);
/* text for a device status word written by a kernel (0 = ok) */
const char* b2g_status_string(int32_t status);

/* B2G_OK if `cfg` can run `prob`, else B2G_ERR_UNSUPPORTED with the reason copied into `reason` (may be NULL). Host
   only; needs no GPU. The shape rules the config space prunes with are kernels/config_space.py:69-90. */
int32_t b2g_check(const b2g_config* cfg, const b2g_problem* prob, char* reason, size_t reason_len);

/* bytes of device workspace a plan for (cfg, prob, A, B) needs: split-K fp32 partials (the reference's
   [SPLIT_K, M, N] buffer, kernels/triton_matmul.py:133) plus staging for operands TMA cannot read in place
   (a base that is not 16-byte aligned, or a leading dimension that is not a multiple of 8 elements). A and B are
   only inspected for alignment; NULL means "16-byte aligned". Host only. */
int32_t b2g_workspace_size(const b2g_config* cfg, const b2g_problem* prob, const void* A, const void* B,
                           size_t* bytes);

/* dynamic shared memory bytes one CTA of this variant uses (the number the config space's smem rule compares with
   the device limit). Host only. */
int32_t b2g_smem_bytes(const b2g_config* cfg, const b2g_problem* prob, size_t* bytes);

/* Build a launch plan on the current device. `workspace` may be NULL when b2g_workspace_size() is 0. `status` is a
   device int32 the kernels write on a bounded-wait timeout (may be NULL: then a timeout is only visible as wrong
   output). Pointers are captured in the plan: a plan runs on exactly these buffers. */
int32_t b2g_plan_create(const b2g_config* cfg, const b2g_problem* prob, const void* A, const void* B, void* C,
                        void* workspace, size_t workspace_bytes, int32_t* status, b2g_plan** out);
/* Enqueue the plan's kernels on `stream` (cudaStream_t, a stream of the plan's device). No allocation, no host
   synchronisation: capturable into a CUDA graph. Returns B2G_OK, B2G_ERR_INVALID_ARG when the current device is not
   the one the plan was made on (nothing is launched), or B2G_ERR_CUDA (launch error). */
int32_t b2g_plan_launch(const b2g_plan* plan, void* stream);
/* Point an existing plan at new A, B and C of the same shape, strides and alignment class (each pointer's address
   modulo 16 unchanged): only the tensor maps of operands whose address changed are re-encoded, nothing is
   allocated, and the launch geometry is kept. The per-call path of a dispatcher that sees the same shape with new
   buffers (the reference caches one runner per call site and pointers, lscli/client.py:328-345). Returns
   B2G_ERR_INVALID_ARG, leaving the plan as it was, when the alignment class or the tensor-map form would change:
   then create a new plan. Not safe while another thread launches the same plan. */
int32_t b2g_plan_rebind(b2g_plan* plan, const void* A, const void* B, void* C);
/* number of kernels b2g_plan_launch enqueues (packing, GEMM, split-K reduce) */
int32_t b2g_plan_num_kernels(const b2g_plan* plan);
/* grid size (CTAs) of the plan's GEMM kernel */
int32_t b2g_plan_grid(const b2g_plan* plan);
int32_t b2g_plan_destroy(b2g_plan* plan);

/* One-shot: plan, launch, destroy. */
int32_t b2g_gemm(const b2g_config* cfg, const b2g_problem* prob, const void* A, const void* B, void* C,
                 void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/* The deterministic split-K reduction alone (kernels/triton_matmul.py:85-92): C[i,j] = cast(sum_{s<split} ws[s,i,j])
   summed in increasing s, ws contiguous [split, M, N] fp32. split == 0 writes zeros. */
int32_t b2g_splitk_reduce(const float* ws, void* C, int64_t M, int64_t N, int64_t stride_cm, int64_t stride_cn,
                          int32_t split, int32_t dtype, void* stream);

/* ---- timing support (the candidate timer's stream gate; no counterpart in the reference, whose timer queues a
   calibrated device sleep instead, tune/timing.py:151-154) ----
   A 4-byte flag in mapped, pinned host memory: *host_ptr for the host, *device_ptr for kernels. */
int32_t b2g_host_flag_create(int32_t** host_ptr, int32_t** device_ptr);
/* store `value` into the flag (sequentially consistent; the device sees it on its next read) */
int32_t b2g_host_flag_set(int32_t* host_ptr, int32_t value);
int32_t b2g_host_flag_destroy(int32_t* host_ptr);
/* Enqueue on `stream` a one-thread kernel that returns once *device_flag == expect, so the work queued after it
   starts only when the host sets the flag. Bounded: after timeout_ns it writes 0x201 into *status (may be NULL) and
   returns. */
int32_t b2g_hold(const int32_t* device_flag, int32_t expect, uint64_t timeout_ns, int32_t* status, void* stream);

/* ---- selector support ----
   Scores of a tree ensemble (the learned ranker's model, stored as arrays; no counterpart in the reference, which
   calls LightGBM's own predictor, analysis/learned.py:488-516). Node n: feature[n] (-1 for a leaf), threshold[n],
   children left[n] / right[n] (indices into the same arrays), missing_left[n] (direction of a NaN), value[n] (a
   leaf's output). roots[t] is tree t's root. out[r] = base + sum over t in order of the leaf value row r reaches,
   going left when X[r, feature] <= threshold. X is row-major [n_rows, n_features] double. Host only. */
int32_t b2g_forest_predict(const int32_t* feature, const double* threshold, const int32_t* left, const int32_t* right,
                           const uint8_t* missing_left, const double* value, const int32_t* roots, int32_t n_trees,
                           double base, const double* X, int64_t n_rows, int32_t n_features, double* out,
                           int32_t threads);

/* Allocation-free GEMM. It has no counterpart in the reference: the reference always allocates its split-K workspace
   with torch (kernels/triton_matmul.py:133).
   For callers that may not allocate device memory themselves: plugin hosts that hand a library only its input and
   output buffers, processes whose device memory is already fully reserved by another allocator, and code running
   while a stream is being captured in global mode, where cudaMalloc is not permitted. This entry point allocates
   nothing (no cudaMalloc, no cudaFree, no allocating library call). The caller passes A, B and C (and optionally a
   device status word); split-K partials go to a fixed scratch array that lives in the library's module image, 32 MiB
   on every GPU that loads the library, held until the process exits.
   Limits and rules:
   - split-K partials larger than 32 MiB (4 * SPLIT_K * M * N bytes) are rejected with B2G_ERR_WORKSPACE and a
     message naming both sizes; operands that would need staging (unaligned bases or leading dimensions) and the
     stream-K schedule (its fix-up flags must start zeroed in a caller workspace) are rejected with
     B2G_ERR_UNSUPPORTED. K = 0 needs no partials whatever SPLIT_K is.
   - The first call on each device looks up the scratch array's device address (cudaGetSymbolAddress) with that
     device current; make that first call before any stream capture begins.
   - All calls share the one scratch array, which keeps the contents of the last call. Nothing in it needs to start
     at zero: every partial a call reads is written by the same call. Calls whose kernels overlap on the GPU (other
     streams, other threads) race on the array: serialise them.
   Returns B2G_OK after enqueueing the kernels on `stream`. */
int32_t b2g_gemm_noalloc(const b2g_config* cfg, const b2g_problem* prob, const void* A, const void* B, void* C,
                         int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* B2G_H_ */
