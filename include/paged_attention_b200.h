/*
 * paged_attention_b200.h — C ABI of the B200 (sm_100a) paged-attention decode path.
 *
 * Two operations make up one decode step of one transformer layer:
 *
 *   pa_kv_append  scatters the step's new K/V rows into the paged KV cache.
 *                 Replaces the scatter loop of GpuKVBlockPool.write_tokens_batch
 *                 (runtime/phase2/paged_kv_kernel.py:176-227) and, through the
 *                 slot_mapping form, the north-star `slot_mapping` argument.
 *   pa_decode     attends every query row of every sequence over that sequence's
 *                 blocks, reached through its block table.  Replaces
 *                 _paged_attention_decode_batched_triton and its Triton kernels
 *                 (runtime/phase2/paged_attention_triton.py:148-243, 245-336,
 *                 338-412, 414-457, 460-660).
 *
 * Conventions
 *   - Every pointer is a device pointer unless the name says host.  The library
 *     never allocates device memory; the caller owns every buffer.
 *   - Strides are in ELEMENTS.  The innermost (head_dim) stride is always 1.
 *   - `stream` is a cudaStream_t passed as void*; every launch goes on it.
 *   - Every function returns a pa_status (0 = PA_OK).  pa_last_error() gives a
 *     human-readable reason for the last failure on the calling host thread.
 *   - Device-detected input errors (a block id outside the pool, a sequence
 *     longer than its block table, a slot outside the pool) never fault: the
 *     kernel skips the access and ORs a PA_DEVERR_* bit into the status word at
 *     the start of the workspace (or into `error_flags` for pa_kv_append).
 *     pa_read_device_errors() reads it back.
 *   - Launch-time work is graph-capture safe: no host synchronisation, no
 *     allocation, grid sizes depend only on host-side shapes.
 */
#ifndef PAGED_ATTENTION_B200_H_
#define PAGED_ATTENTION_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PA_API __attribute__((visibility("default")))
#else
#define PA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (host) -------------------------------------------------- */
typedef enum pa_status {
  PA_OK = 0,
  PA_ERR_INVALID_ARGUMENT = 1, /* bad shape / stride / null pointer  -> ValueError  */
  PA_ERR_UNSUPPORTED = 2,      /* valid but not implemented (head_dim, block size) -> ValueError */
  PA_ERR_WORKSPACE = 3,        /* workspace missing or too small      -> RuntimeError */
  PA_ERR_CUDA = 4,             /* CUDA runtime / launch failure       -> RuntimeError */
  PA_ERR_DEVICE = 5            /* device error word non-zero          -> IndexError   */
} pa_status;

/* ---- element types -------------------------------------------------------- */
typedef enum pa_dtype {
  PA_DTYPE_FLOAT32 = 0,
  PA_DTYPE_FLOAT16 = 1,
  PA_DTYPE_BFLOAT16 = 2
} pa_dtype;

/* ---- device error bits (status word / error_flags) ------------------------ */
#define PA_DEVERR_BLOCK_ID_RANGE 0x1u /* block-table entry outside [0, num_blocks)       */
#define PA_DEVERR_TABLE_UNDERRUN 0x2u /* sequence needs more blocks than max_blocks      */
#define PA_DEVERR_SLOT_RANGE 0x4u     /* slot_mapping entry outside the pool             */
#define PA_DEVERR_WAIT_TIMEOUT 0x8u   /* a bounded wait on a bulk copy ran out           */

/* A paged cache view: [num_blocks, num_kv_heads, block_size, head_dim], head_dim
 * contiguous.  For GpuKVBlockPool's per-layer view (paged_kv_kernel.py:124-134)
 * stride_block = num_layers * num_kv_heads * block_size * head_dim. */
typedef struct pa_cache_view {
  void* data;
  int64_t num_blocks;
  int64_t stride_block;
  int64_t stride_head;
  int64_t stride_token;
} pa_cache_view;

/* Arguments of pa_kv_append.
 * New rows `key`/`value` are [batch, num_kv_heads, q_len, head_dim] (HF layout).
 * Token i = b * q_len + t is written to
 *   slot = slot_mapping[i]                                 (slot_mapping != NULL)
 *   slot = block_tables[b, p / bs] * bs + p % bs,
 *          p = positions[b] + position_offset + t                      (otherwise)
 * and lands in cache[slot / bs, h, slot % bs, :].  A negative slot_mapping entry
 * marks a padding token and is skipped. */
typedef struct pa_kv_append_args {
  const void* key;
  int64_t key_stride_b, key_stride_h, key_stride_t;
  const void* value;
  int64_t value_stride_b, value_stride_h, value_stride_t;
  pa_cache_view key_cache;
  pa_cache_view value_cache;
  const int64_t* slot_mapping;  /* [batch * q_len] or NULL */
  const int32_t* block_tables;  /* [batch, >= max_blocks] (used when slot_mapping == NULL) */
  int64_t block_table_stride;
  int32_t max_blocks;
  const void* positions;        /* [batch] start position of token t=0 (slot_mapping == NULL) */
  int32_t positions_is_int64;   /* 0: int32, 1: int64 */
  int32_t position_offset;      /* added to every position (e.g. -q_len for post-append lengths) */
  int32_t batch, q_len, num_kv_heads, head_dim, block_size;
  int32_t dtype;                /* pa_dtype of key, value and both caches */
  uint32_t* error_flags;        /* device word that receives PA_DEVERR_* bits (may be NULL) */
} pa_kv_append_args;

/* Arguments of pa_decode.
 * query [batch, num_q_heads, q_len, head_dim]; out has the same shape and dtype.
 * Sequence b attends L_b = context_lens[b] + len_offset tokens.  Query token t of
 * row b sits at absolute position L_b - q_len + t and attends positions
 * 0 .. L_b - q_len + t (causal over the q_len new tokens; q_len = 1 is plain decode).
 * Query head hq reads KV head hq / (num_q_heads / num_kv_heads).
 *   len_offset = q_len : context_lens counts the tokens cached BEFORE this step;
 *   len_offset = 0     : context_lens already includes them (the reference's
 *                        seq_lens, paged_attention_triton.py:50). */
typedef struct pa_decode_args {
  const void* query;
  int64_t query_stride_b, query_stride_h, query_stride_t;
  pa_cache_view key_cache;
  pa_cache_view value_cache;
  const int32_t* block_tables;  /* [batch, >= max_blocks] */
  int64_t block_table_stride;
  int32_t max_blocks;
  const int32_t* context_lens;  /* [batch] */
  int32_t len_offset;
  void* out;
  int64_t out_stride_b, out_stride_h, out_stride_t;
  int32_t batch, q_len, num_q_heads, num_kv_heads, head_dim, block_size;
  int32_t dtype;                /* pa_dtype of query, caches and out */
  float scale;                  /* softmax scale applied to q.k */
  void* workspace;              /* device scratch, pa_decode_workspace_bytes() long,
                                   zero-filled once before first use (pa_workspace_init) */
  size_t workspace_bytes;
  int32_t allow_overlap_with_previous; /* 1: programmatic dependent launch on the kernel
                                          launched just before on `stream` (pa_kv_append) */
  /* Per-SM shares of large fp16/bf16 decode calls (no counterpart in the
   * reference; NULL / 0: equal shares).  sm_weights is host memory, one
   * relative speed per SM of the device (num_sm_weights = its SM count); it is
   * read at the call, so a launch (or a captured graph) keeps the shares it was
   * given.  A call whose work gives every warp at least 64 units (16 tokens of
   * one KV head) splits its cost in proportion to them, SM by SM.  With
   * sm_timing_tag != 0 such a call also writes one pa_sm_timing record per SM
   * at PA_WS_SM_TIMING_OFFSET in the workspace, tagged with it, so the caller
   * can derive the speeds (see paged_attention.py). */
  const float* sm_weights;
  int32_t num_sm_weights;
  uint32_t sm_timing_tag;
} pa_decode_args;

/* One SM's share of a large decode call: when it started and finished (the
 * GPU's global timer, ns), the cost units it held (16-token units plus a
 * fixed cost per row), the SM it ran on and the call's tag. */
typedef struct pa_sm_timing {
  uint64_t t_start_ns, t_end_ns;
  uint32_t cost, smid, tag, pad;
} pa_sm_timing;
#define PA_WS_SM_TIMING_OFFSET 256
#define PA_MAX_SM_WEIGHTS 160

/* Scatter new K/V rows into the paged cache.  Bit-exact copy.
 * Replaces: GpuKVBlockPool.write_tokens_batch, runtime/phase2/paged_kv_kernel.py:176-227
 * (and write_tokens :136-174, which delegates to it for batch 1). */
PA_API int pa_kv_append(const pa_kv_append_args* args, void* stream);

/* Paged decode attention (split-K over the whole batch with an in-kernel
 * log-sum-exp merge).  fp16/bf16 use tensor-core tiles; fp32 stays on CUDA cores.
 * head_dim: fp16/bf16 any multiple of 8 up to 128 (tiles of 64 or 128 columns,
 * the columns past head_dim zero-filled by TMA), fp32 any value up to 128; the
 * reference's kernels take any head_dim (a power-of-two tile with a mask,
 * paged_attention_triton.py:497).  Others return PA_ERR_UNSUPPORTED.
 * Replaces: paged_attention_decode_batched -> _paged_attention_decode_batched_triton,
 * runtime/phase2/paged_attention_triton.py:460-552 and :745-775, with the kernels at
 * :148-243 (direct batched), :245-336 (split), :338-412 (direct single) and
 * :414-457 (log-sum-exp combine). */
PA_API int pa_decode(const pa_decode_args* args, void* stream);

/* Sequences whose block tables start with the same physical blocks (a shared
 * prompt prefix), in groups.  Device arrays except the two host bounds:
 *   members of group g  = member_seqs[member_offsets[g] .. member_offsets[g+1])
 *   prefix_lens[g]      = tokens at positions 0 .. prefix_lens[g]-1 that every
 *                         member of g reads through the SAME physical blocks
 *                         (the first member's table is the one read);
 *   seq_group[b]        = group of batch row b, -1 for a row in no group.
 * A row belongs to at most one group.  max_members and max_prefix_len bound the
 * device values (they size the grid); a group with more members or a longer
 * prefix is an argument error the kernels flag (PA_DEVERR_PREFIX). */
typedef struct pa_prefix_groups {
  int32_t num_groups;
  int32_t max_members;            /* host: >= members of any group */
  int32_t max_prefix_len;         /* host: >= prefix_lens[g] of any group */
  const int32_t* member_offsets;  /* [num_groups + 1] */
  const int32_t* member_seqs;     /* [member_offsets[num_groups]] */
  const int32_t* prefix_lens;     /* [num_groups] */
  const int32_t* seq_group;       /* [batch] */
} pa_prefix_groups;

#define PA_DEVERR_PREFIX 0x10u /* a member's table differs from its group's in the prefix,
                                  or a group exceeds max_members / max_prefix_len */

/* pa_decode over sequences that share prompt prefixes (cascade attention): each
 * group's query rows attend the shared prefix blocks together, once per group,
 * on the tcgen05 multi-query kernel; the decode kernel then attends each
 * sequence's own tokens and merges both parts (log-sum-exp) before writing the
 * output.  Same result as pa_decode on the same tables, reading each shared
 * block once per group instead of once per member.  The reference shares
 * prefixes by copying blocks (GpuKVBlockPool.copy_blocks,
 * runtime/phase2/paged_kv_kernel.py:233-250; callers worker_server.py:1266-1272)
 * and then attends every copy; it has no counterpart of this call.
 * Needs pa_cascade_workspace_bytes() of workspace.  fp32 calls and calls whose
 * query / out rows are not 16-byte aligned run pa_decode unchanged. */
PA_API int pa_decode_cascade(const pa_decode_args* args, const pa_prefix_groups* groups, void* stream);

/* Workspace bytes of pa_decode_cascade: pa_decode's plus the prefix partials. */
PA_API size_t pa_cascade_workspace_bytes(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                         int32_t q_len, int32_t head_dim, int32_t dtype, int32_t device,
                                         int32_t num_groups, int32_t max_members, int32_t max_prefix_len);

/* ---- KV-head-sharded decode with the all-gather fused in (one process per GPU) ----
 * Each rank attends its own KV heads of every sequence; the decode kernel writes
 * every finished output row straight into EVERY rank's gathered output
 * [batch, total query heads, q_len, head_dim] (peer memory over NVLink), then
 * the grid's last warp raises this rank's flag at every rank and waits, for at
 * most wait_ns, until every rank has raised its own.  Replaces the local decode
 * + all-gather (an NCCL collective plus a copy) of the sharded layout; the
 * reference runs on one GPU and has no counterpart.
 * Buffers of other ranks are reached through CUDA IPC: pa_ipc_export on the
 * owner, pa_ipc_import in every other process. */
#define PA_IPC_HANDLE_BYTES 64
typedef struct pa_ipc_handle {
  unsigned char bytes[PA_IPC_HANDLE_BYTES]; /* cudaIpcMemHandle_t of the allocation */
  int64_t offset;                           /* of the exported pointer within it */
} pa_ipc_handle;

/* Handle for `device_ptr` (any pointer into a cudaMalloc'd allocation). */
PA_API int pa_ipc_export(const void* device_ptr, pa_ipc_handle* handle);
/* Map another process's exported pointer into this one (*device_ptr receives it). */
PA_API int pa_ipc_import(const pa_ipc_handle* handle, void** device_ptr);
/* Unmap a pointer pa_ipc_import returned. */
PA_API int pa_ipc_release(void* device_ptr);

typedef struct pa_gather_args {
  int32_t num_ranks, rank;
  int32_t head_offset;           /* first query head of this rank in the gathered output */
  void* const* out_ranks;        /* device array [num_ranks]: every rank's gathered output
                                    (this process's mapping); args->out must be out_ranks[rank] */
  uint32_t* const* flags_ranks;  /* device array [num_ranks]: every rank's flag words [num_ranks] */
  uint32_t* epoch;               /* this rank's call counter (device, starts at 0 like the flags) */
  uint32_t* done_warps;          /* this rank's warp counter (device, zero between calls) */
  int64_t wait_ns;               /* bound on the wait for the other ranks' flags */
} pa_gather_args;

/* The ranks of a fused gather fell out of step: a wait ran out, or a peer's
 * flag skipped calls.  The rank that sees it sets bit 31 of its epoch and of
 * its flag at every rank, so every later pa_decode_gather call on every rank
 * reports this bit at once, without waiting, until the ranks start again from
 * fresh (zeroed) flags and epochs. */
#define PA_DEVERR_GATHER 0x20u

/* pa_decode for the local KV heads, output rows written to every rank's gathered
 * output at query-head offset head_offset (args->out_stride_* are the gathered
 * output's strides).  fp16/bf16 only.  A rank whose flag does not arrive in time
 * is reported as PA_DEVERR_WAIT_TIMEOUT | PA_DEVERR_GATHER; no wait is
 * unbounded. */
PA_API int pa_decode_gather(const pa_decode_args* args, const pa_gather_args* gather, void* stream);

/* Size of the scratch array behind pa_decode_static_workspace (16 MiB). */
#define PA_STATIC_WORKSPACE_BYTES (16u << 20)

/* pa_decode for callers that cannot allocate device memory.  No counterpart in
 * the reference (its decode allocates scratch on first use per shape).
 * Takes the same arguments as pa_decode but ignores args->workspace and
 * args->workspace_bytes: the scratch is a 16 MiB __device__ array inside this
 * library.  The CUDA runtime loads device code lazily, so the array is created
 * in a GPU's memory by the first call on that GPU and held there until the
 * process exits; that first call also looks up the array's device address
 * (cudaGetSymbolAddress, that device current).  Make it before giving the rest
 * of the free memory to the KV pool and before any stream capture.  After it,
 * nothing is allocated: a plugin host that hands its kernels only inputs and
 * outputs, or a serving loop that has given all free HBM to the KV pool, can
 * call it.  Every call shares the array: each clears the error word and merge
 * counters on its stream before the decode, and calls that overlap on the GPU
 * race.  Shapes needing more scratch than PA_STATIC_WORKSPACE_BYTES
 * (pa_decode_workspace_bytes) are rejected with PA_ERR_WORKSPACE; on a 148-SM
 * B200 that is more than 13 query rows per KV head (G * q_len) at head_dim 128.
 * The kernels still skip invalid block ids, but their device error word stays
 * inside the array: this entry point reports host-side errors only. */
PA_API int pa_decode_static_workspace(const pa_decode_args* args, void* stream);

/* Bytes of workspace pa_decode needs on `device` for these shapes.
 * Replaces the scratch caches _decode_scratch_buffers / _direct_out_buffer
 * (runtime/phase2/paged_attention_triton.py:90-115); unlike them the output is
 * never aliased to scratch. */
PA_API size_t pa_decode_workspace_bytes(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                 int32_t q_len, int32_t head_dim, int32_t dtype, int32_t device);

/* Zero a workspace (its merge counters and status word) on `stream`.  Needed
 * once after allocation; pa_decode leaves the counters at zero after each call.
 * No counterpart in the reference (its scratch needs no initialisation). */
PA_API int pa_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/* Copy the device status word at the start of `workspace` (or any device
 * uint32 word) to *host_flags, optionally clearing it.  Synchronises `stream`.
 * Stands in for the host-side checks that raise IndexError in the reference
 * (paged_kv_kernel.py:118-119, :167-170, :221-222). */
PA_API int pa_read_device_errors(void* device_word, uint32_t* host_flags, int32_t clear, void* stream);

/* Text for the last failure on this host thread ("" when none). */
PA_API const char* pa_last_error(void);

/* Name of the kernel the last pa_decode / pa_decode_cascade call on this host
 * thread launched ("pa::decode_mma_kernel", "pa::decode_f32_kernel",
 * "pa::prefill_mma_kernel", "pa::prefill_umma_kernel", or for the cascade
 * "pa::prefill_umma_kernel<prefix> + pa::decode_mma_kernel").  No counterpart in the reference, whose
 * dispatch (paged_attention_triton.py:460-552) is visible in Python. */
PA_API const char* pa_last_kernel(void);

/* Library version: major * 10000 + minor * 100 + patch. */
PA_API int32_t pa_version(void);

#ifdef __cplusplus
}
#endif

#endif /* PAGED_ATTENTION_B200_H_ */
