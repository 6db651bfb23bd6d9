/*
 * fa_b200.h - C ABI of the B200 (sm_100a) FlashAttention-2 forward library.
 *
 * This is the drop-in boundary under the `_flash_attn_metal` Python module.
 * Every entry point takes plain pointers, sizes and a CUDA stream handle
 * (passed as void*), so any FFI (ctypes, cffi, pybind11, JNI, cgo) can bind it.
 *
 * Reference interfaces replaced (harvestingmoon/flash_attn_metal_cpp):
 *   fa_params            <- struct FlashAttentionParams     include/flash_attn_core.hpp:31-46
 *   fa_init              <- MetalDevice::initialize          src/flash_attn_core.cpp:50-64
 *                           and py_initialize                python/bindings.cpp:42-50
 *   fa_device_info       <- MetalDevice::device_name / max_buffer_length
 *                                                            src/flash_attn_core.cpp:83-91
 *                           and py_get_device_info           python/bindings.cpp:94-109
 *   fa_forward           <- FlashAttentionForward::execute (kernel part: bind + dispatch)
 *                                                            src/flash_attn_core.cpp:352-385
 *   fa_forward_host      <- FlashAttentionForward::execute (whole call: stage in, dispatch,
 *                           wait, copy out)                  src/flash_attn_core.cpp:276-407
 *   fa_workspace_size    <- buffer sizing in execute         src/flash_attn_core.cpp:299-305
 *   fa_tensor_bytes      <- compute_tensor_size              src/flash_attn_core.cpp:445-448
 *   fa_pool_stats        <- BufferPool hit/miss/bytes stats  include/flash_attn_core.hpp:99-101
 *   fa_pool_clear        <- BufferPool::clear                src/flash_attn_core.cpp:236-246
 *   fa_rope_tables       <- host cos/sin tables bound in execute
 *                                                            src/flash_attn_core.cpp:343-349
 *   fa_forward_partial   <- (no counterpart) split-KV partial used by the multi-GPU
 *                           long-context path; same kernel as fa_forward
 *   fa_combine           <- (no counterpart) (O, LSE) merge of split-KV partials
 *   fa_forward_range     <- (no counterpart) row/key-range forward with optional
 *                           output routing to peer devices (split-KV over NVLink)
 *   fa_ipc_*             <- (no counterpart) CUDA IPC staging buffers for the routing
 *   fa_last_error       <- std::cerr messages / RuntimeError text
 *                                                            python/bindings.cpp:46-49,224-232
 *
 * Layout contract (same as the reference API, python/bindings.cpp:142-159):
 *   Q, O : (batch, seqlen_q, num_heads_q, head_dim)   row-major
 *   K, V : (batch, seqlen_k, num_heads_k, head_dim)   row-major
 *   LSE  : (batch, num_heads_q, seqlen_q) float32, natural-log log-sum-exp
 * Element strides may be given per tensor (0 = contiguous BSHD), which
 * allows zero-copy head/batch slices and (B,H,S,D) tensors.
 *
 * Semantics: O = softmax(softmax_scale * Q K^T + mask) V with fp32
 * accumulation; the causal mask is top-left aligned (key k is masked for
 * query q iff k > q), as in the reference test oracle (test.py:80-82).
 * GQA maps query head h to key/value head h / (num_heads_q / num_heads_k).
 * Rotate-half RoPE is applied to Q and K when has_rotary is set.
 */
#ifndef FA_B200_H
#define FA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum fa_status {
    FA_OK = 0,
    FA_ERR_INVALID_ARG = 1,   /* bad shape, pointer, stride or alignment */
    FA_ERR_UNSUPPORTED = 2,   /* valid request that this build does not implement */
    FA_ERR_CUDA = 3,          /* a CUDA runtime/driver call failed */
    FA_ERR_TIMEOUT = 4,       /* a bounded in-kernel wait ran out (kernel returned early) */
    FA_ERR_RANGE = 5,         /* reserved: no longer returned (operands beyond the fp16
                                 range are rescaled by a power of two, see fa_forward) */
    FA_ERR_NOT_INITIALIZED = 6,
    FA_ERR_NO_DEVICE = 7
} fa_status;

typedef enum fa_dtype {
    FA_F16 = 0,
    FA_BF16 = 1,
    FA_F32 = 2
} fa_dtype;

/* Launch parameters. The first block mirrors FlashAttentionParams
 * (include/flash_attn_core.hpp:31-46) field by field. */
typedef struct fa_params {
    uint32_t batch_size;
    uint32_t seqlen_q;
    uint32_t seqlen_k;
    uint32_t num_heads_q;
    uint32_t num_heads_k;
    uint32_t head_dim;
    float softmax_scale;      /* used as given; 0 gives uniform weights, as in the reference */
    int32_t is_causal;
    int32_t window_left;      /* sliding window (common.metal:95-104): key k is masked for */
    int32_t window_right;     /* query q if k - q < -window_left or k - q > window_right;
                                 a negative value leaves that side unbounded (-1 = none) */
    float dropout_p;          /* must be 0 (UNSUPPORTED otherwise) */
    int32_t has_alibi;        /* add alibi_slopes[h] * (k - q) to the scaled scores
                                 (common.metal:123-128); needs alibi_slopes */
    int32_t has_rotary;       /* apply rotate-half RoPE to Q and K */
    uint32_t gqa_group_size;  /* 0 = derive num_heads_q / num_heads_k; else must equal it */

    /* Additions of this library. */
    int32_t dtype;            /* fa_dtype of Q, K and V */
    int32_t out_dtype;        /* fa_dtype of O; -1 = same as dtype */
    float rope_theta;         /* when has_rotary and no cos/sin tables: inv_freq_i = theta^(-2i/D) */
    /* Element strides (batch, seq, head); the head_dim stride is always 1.
     * All zero = contiguous BSHD for that tensor. */
    int64_t q_stride[3];
    int64_t k_stride[3];
    int64_t v_stride[3];
    int64_t o_stride[3];
    /* float32 [num_heads_q] ALiBi slopes when has_alibi: device memory for
     * fa_forward / fa_forward_range / fa_forward_partial / fa_forward_noalloc,
     * host memory for fa_forward_host. */
    const float* alibi_slopes;
} fa_params;

/* Fill `p` with the reference defaults (scale 0, no mask, no RoPE, contiguous). */
void fa_params_init(fa_params* p);

/* Select and initialise CUDA device `device` for the calling thread
 * (-1: the thread's current device, left selected). */
fa_status fa_init(int device);

/* Device name (NUL-terminated, truncated to name_len), total global memory
 * in bytes, and whether fa_init succeeded on it (-1: the current device).
 * Any output may be NULL. */
fa_status fa_device_info(int device, char* name, size_t name_len,
                         uint64_t* total_mem, int* initialized);

/* Bytes of device scratch fa_forward needs for `p` (0 when none). */
size_t fa_workspace_size(const fa_params* p);

/* Bytes of one (B,S,H,D) tensor of element type `dtype`. */
size_t fa_tensor_bytes(uint32_t batch, uint32_t seq, uint32_t heads,
                       uint32_t dim, int32_t dtype);

/* Attention forward on device pointers, enqueued on `stream` (cudaStream_t;
 * NULL = legacy default stream). Returns without synchronising.
 *   q, k, v   : device inputs (dtype p->dtype)
 *   o         : device output (dtype p->out_dtype)
 *   lse       : optional device output [B, Hq, Sq] float32 (NULL = skip)
 *   cos, sin  : optional device RoPE tables, float32 [max(Sq,Sk), D/2],
 *               row = position (layout of src/flash_attn_core.cpp:343-349);
 *               NULL with has_rotary set = build from rope_theta
 *   workspace : device scratch of fa_workspace_size(p) bytes, or NULL to use
 *               the library's cached per-stream workspace.
 * On the tensor-core path, fp16/bf16 operands are staged as fp16 (RoPE
 * applied, bf16 converted); a staged tensor whose largest magnitude exceeds
 * 65504 is stored scaled by the smallest power of two 2^-e that keeps it
 * finite, and the kernel multiplies the scores (Q, K) or O (V) back by 2^e,
 * so inputs anywhere in the bf16 range give correct results. */
fa_status fa_forward(const fa_params* p, const void* q, const void* k,
                     const void* v, void* o, float* lse, const float* cos,
                     const float* sin, void* workspace, size_t workspace_bytes,
                     void* stream);

/* Whole-call path on HOST pointers: copies Q/K/V (and tables) to device
 * buffers from the library pool, runs fa_forward, copies O (and LSE when
 * non-NULL) back and synchronises, like FlashAttentionForward::execute.
 * Large calls are pipelined over query-row blocks (copy in, compute, copy
 * out on three streams). Host buffers may be pinned or pageable: pageable
 * inputs are copied into pinned staging by a few worker threads (set their
 * number with the FA_HOST_COPY_THREADS environment variable) piece by
 * piece, each piece DMA'd as soon as it is staged; pageable outputs are
 * staged the same way on the way back. */
fa_status fa_forward_host(const fa_params* p, const void* q, const void* k,
                          const void* v, void* o, float* lse, const float* cos,
                          const float* sin);

/* Pinned (page-locked) host memory from the library's pool (no counterpart
 * in the reference, whose Metal buffers are shared with the host). Outputs
 * the caller lets the library allocate (the Python module's NumPy results)
 * live here, so fa_forward_host copies them back by DMA at full link speed;
 * fa_host_free returns a buffer to the pool (freed unused buffers beyond a
 * few GB go back to the system; fa_pool_clear releases the rest). */
fa_status fa_host_alloc(size_t bytes, void** ptr);
void fa_host_free(void* ptr);

/* Split-KV partial: attention of every query row over the keys in
 * [kv_begin, kv_end) only (after the causal mask). Writes the row-normalised
 * partial O (float32, contiguous BSHD) and its LSE [B, Hq, Sq]; rows with no
 * visible key get O = 0 and LSE = -inf. Only query rows in
 * [q_begin, q_end) are computed and written. */
fa_status fa_forward_partial(const fa_params* p, const void* q, const void* k,
                             const void* v, float* o_partial, float* lse_partial,
                             const float* cos, const float* sin,
                             uint32_t q_begin, uint32_t q_end,
                             uint32_t kv_begin, uint32_t kv_end,
                             void* workspace, size_t workspace_bytes, void* stream);

/* Merge n_splits partials for rows [q_begin, q_end):
 *   o_parts   : n_splits consecutive float32 BSHD tensors (Hq heads)
 *   lse_parts : n_splits consecutive [B, Hq, Sq] float32 arrays
 *   o         : output of dtype out_dtype (BSHD, p->o_stride honoured)
 *   lse       : optional merged LSE [B, Hq, Sq] (NULL = skip)
 * LSE = log sum_j exp(LSE_j), O = sum_j exp(LSE_j - LSE) O_j. */
fa_status fa_combine(const fa_params* p, const float* o_parts,
                     const float* lse_parts, int32_t n_splits, void* o,
                     float* lse, uint32_t q_begin, uint32_t q_end, void* stream);

/* fa_combine where partial j holds only rows [part_row_begin[j], ...)
 * (part_row_begin: DEVICE array of n_splits int32, NULL = every row): rows
 * before it ignore that partial, whose staging there may be stale. */
fa_status fa_combine_ranges(const fa_params* p, const float* o_parts,
                            const float* lse_parts, int32_t n_splits,
                            const int32_t* part_row_begin, void* o, float* lse,
                            uint32_t q_begin, uint32_t q_end, void* stream);

/* Output routing for a split-KV partial spread over devices. Query rows are
 * owned in blocks of owner_rows (a multiple of 128): row r belongs to owner
 * r / owner_rows. `table` is a DEVICE array of 2 * n_owners addresses:
 *   table[o]            O slot of owner o: [batch, owner_rows, Hq, D] of
 *                       p->out_dtype, contiguous, 16-byte aligned
 *   table[n_owners + o] LSE slot of owner o: [batch, Hq, owner_rows] float32
 * Slots may be peer-device memory (fa_ipc_open): the kernel's epilogue then
 * stores each finished tile straight over NVLink. */
typedef struct fa_route {
  const uint64_t* table;
  int32_t n_owners;
  uint32_t owner_rows;
} fa_route;

/* Rows [q_begin, q_end) of softmax(scale Q K^T + mask) V restricted to keys
 * [kv_begin, kv_end) (no counterpart in the reference; the building block of
 * the multi-GPU paths). Output dtype p->out_dtype; rows are written to o /
 * lse (lse may be NULL) or, when route != NULL, to the owners' slots (o and
 * lse are ignored; q_begin must then be a multiple of 128 and
 * n_owners * owner_rows >= q_end). Rows that see no key of the range get O = 0 and
 * LSE = -inf. Query and key positions are absolute (RoPE tables and the
 * causal mask use them). */
fa_status fa_forward_range(const fa_params* p, const void* q, const void* k,
                           const void* v, void* o, float* lse,
                           const float* cos, const float* sin,
                           uint32_t q_begin, uint32_t q_end,
                           uint32_t kv_begin, uint32_t kv_end,
                           const fa_route* route, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Device memory shared between the processes of one node (CUDA IPC; no
 * counterpart in the reference). fa_ipc_alloc allocates on the current
 * device and returns a handle another process passes to fa_ipc_open to map
 * the same memory (peer access over NVLink). fa_ipc_close unmaps an opened
 * handle; fa_ipc_free releases an allocation (after every peer closed it). */
typedef struct fa_ipc_handle {
  unsigned char bytes[64];
} fa_ipc_handle;

fa_status fa_ipc_alloc(size_t bytes, void** dev_ptr, fa_ipc_handle* handle);
fa_status fa_ipc_free(void* dev_ptr);
fa_status fa_ipc_open(const fa_ipc_handle* handle, void** dev_ptr);
fa_status fa_ipc_close(void* dev_ptr);

/* Build float32 cos/sin tables [rows, head_dim/2] on the host:
 * angle(pos, i) = pos * theta^(-2i/head_dim). */
fa_status fa_rope_tables(float* cos_out, float* sin_out, uint32_t rows,
                         uint32_t head_dim, float theta);

/* Device-pool statistics of the calling thread's current device. */
fa_status fa_pool_stats(uint64_t* hits, uint64_t* misses, uint64_t* bytes_reserved);

/* Synchronise the calling thread's current device, then free every cached
 * buffer of it: the host-path pool, the per-stream workspaces of fa_forward
 * calls made without one, the RoPE tables built from rope_theta, and the
 * buffers those caches replaced when they grew. Calls in flight on other
 * host threads must have finished enqueuing. */
fa_status fa_pool_clear(void);

/* Read and clear the in-kernel status word of the current device (after the
 * stream has been synchronised). Returns FA_ERR_TIMEOUT when a kernel of
 * this library (other than fa_forward_noalloc's) gave up a wait since the
 * last call, else FA_OK. */
fa_status fa_check_device_status(void);

/* Wall-clock limit of every in-kernel wait of later launches, in seconds
 * (default 2 s; process-wide). A wait that runs out makes its kernel record
 * FA_ERR_TIMEOUT, release its resources and return early. Raise it when the
 * GPU is time-sliced with other work for long periods. */
fa_status fa_set_wait_limit(double seconds);
double fa_get_wait_limit(void);

/* Test hook (no counterpart in the reference): the next tensor-core launch
 * of the calling thread withholds K tile `k_tile` (counted from the first
 * key tile) from its first CTA, so that CTA's waits run out after the wait
 * limit and the kernel takes its timeout path; the status word then reads
 * FA_ERR_TIMEOUT. Only tests use it. */
fa_status fa_test_stall_next_launch(int32_t k_tile);

/* Number of kernels this library launched on the calling thread so far. */
uint64_t fa_launch_count(void);

/* Kernel timing (no counterpart in the reference): while enabled, every
 * launch of the attention kernel on the calling thread is bracketed by CUDA
 * events recorded on its own stream. fa_kernel_timing_read synchronises
 * those events and returns the summed duration (ms) and the launch count
 * since the last enable, then disables timing. */
fa_status fa_kernel_timing_enable(void);
fa_status fa_kernel_timing_read(double* total_ms, uint64_t* launches);

/* Text of the last error raised on the calling thread ("" if none). */
const char* fa_last_error(void);

/* Allocation-free forward. No counterpart in the reference: it exists for
 * callers that may not allocate device memory, e.g. a plugin inside a host
 * application that owns every device allocation and forbids cudaMalloc.
 * Same arguments and results as fa_forward without the workspace: the caller
 * passes device inputs and outputs, and the library's scratch (fp16 staging
 * of Q/K/V, zero-padded operands and output for head dims other than 64 and
 * 128, RoPE tables built from rope_theta) lives in one fixed 64 MiB device
 * array that every GPU loading the library's module keeps until the process
 * exits. Calls no cudaMalloc/cudaFree and no allocating library routine.
 * A problem whose scratch exceeds 64 MiB is rejected with FA_ERR_INVALID_ARG
 * and a message giving the size it needs.
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make it before any
 * stream capture. Only the primary context of each device is supported.
 * All calls share the array: calls that may overlap on the GPU (several
 * streams or host threads) race and must be serialised by the caller.
 * In-kernel timeouts of this entry point are reported by
 * fa_noalloc_check_status. */
fa_status fa_forward_noalloc(const fa_params* p, const void* q, const void* k,
                             const void* v, void* o, float* lse, const float* cos,
                             const float* sin, void* stream);

/* Status of fa_forward_noalloc's kernels on the current device (after the
 * stream has been synchronised): reads and clears their status word with
 * cudaMemcpy / cudaMemset, allocating nothing. FA_ERR_TIMEOUT when a wait
 * ran out since the last call (that call's output is invalid), else FA_OK. */
fa_status fa_noalloc_check_status(void);

#ifdef __cplusplus
}
#endif

#endif /* FA_B200_H */
