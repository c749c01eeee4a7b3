/*
 * b200_paged_attn.h -- C ABI of the sm_100a paged-attention backend.
 *
 * Device operations over the minivllm KV layout
 *   k_pool / v_pool : contiguous [L, P, S, H, D]
 *   element (l, p, s, h, d) at (((l*P + p)*S + s)*H + h)*D + d
 * (minivllm/kv_block_pool.py:50-68 of zyyh-ops/mini-gpt-inference).
 *
 * Every entry point:
 *   - takes plain device pointers, element strides and sizes (no torch types);
 *   - validates its host-visible arguments and returns a non-zero status
 *     (B200_ERR_*) without launching anything when they are invalid; the
 *     message is available through b200_last_error();
 *   - enqueues its kernels on `stream` (a cudaStream_t passed as void*) and
 *     never synchronises the stream and never allocates device memory;
 *   - checks device-resident metadata (block-table entries, slots, context
 *     lengths) inside the kernel: an out-of-range value is skipped, never
 *     dereferenced, and ORed into the optional `status` word (B200_DEV_*),
 *     which the caller may read after the stream has been synchronised.
 *
 * Thread-safety: the functions keep no per-call global state except the
 * thread-local last-error message and a per-device cache of kernel
 * attributes; concurrent calls on different streams are allowed.
 */
#ifndef B200_PAGED_ATTN_H_
#define B200_PAGED_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_PAGED_ATTN_ABI_VERSION 1

/* Exported symbols (the library is built with hidden default visibility). */
#if defined(__GNUC__)
#define B200_API __attribute__((visibility("default")))
#else
#define B200_API
#endif

/* Element types of q / k / v / pools / outputs. */
typedef enum {
  B200_DTYPE_F32 = 0,
  B200_DTYPE_BF16 = 1,
  B200_DTYPE_F16 = 2
} b200_dtype_t;

/* Integer types of block tables, context lengths and slot mappings. */
typedef enum {
  B200_INDEX_I32 = 0,
  B200_INDEX_I64 = 1
} b200_index_t;

/* Host-side return codes. */
enum {
  B200_OK = 0,
  B200_ERR_INVALID_ARGUMENT = 1, /* the reference raises ValueError here   */
  B200_ERR_UNSUPPORTED = 2,      /* shape/dtype outside the kernels' range */
  B200_ERR_WORKSPACE = 3,        /* workspace missing or too small         */
  B200_ERR_CUDA = 4              /* a CUDA runtime/driver call failed       */
};

/* Bits ORed into the optional device status word by the kernels. */
enum {
  B200_DEV_BAD_BLOCK = 1,    /* block-table entry outside [0, P)           */
  B200_DEV_BAD_LENGTH = 2,   /* context length < 1 or > M*S                */
  B200_DEV_BAD_SLOT = 4,     /* slot outside [0, P*S)                      */
  B200_DEV_WAIT_TIMEOUT = 8, /* a bounded pipeline wait gave up            */
  B200_DEV_SLOT_MISMATCH = 16 /* fused write: slot is not the slot of the
                                 sequence's last context position           */
};

/* Paged KV pool descriptor: two contiguous [L, P, S, H, D] tensors. */
typedef struct {
  void* k;                 /* device pointer, 16-byte aligned              */
  void* v;                 /* device pointer, 16-byte aligned              */
  int64_t num_layers;      /* L */
  int64_t num_blocks;      /* P */
  int64_t block_size;      /* S */
  int64_t num_heads;       /* H */
  int64_t head_dim;        /* D */
  b200_dtype_t dtype;      /* f32 or bf16                                   */
} b200_kv_pool_t;

/*
 * Slot-mapping scatter: for n in [0, N):
 *   pool.k[layer, slot[n] / S, slot[n] % S, :, :] = k[n, :, :]   (and v)
 * with a dtype conversion when k/v and the pool differ.
 * Replaces the decode write of minivllm/attention.py:370-392 and the
 * per-token prefill write loop of minivllm/attention.py:193-208
 * (KVBlockPool.write_layer, minivllm/kv_block_pool.py:91-109).
 */
typedef struct {
  b200_kv_pool_t pool;
  int64_t layer_idx;
  int64_t num_tokens;               /* N (0 is a no-op)                     */
  const void* k;                    /* [N, H, D], strides in elements       */
  const void* v;
  int64_t k_stride[3];
  int64_t v_stride[3];
  b200_dtype_t kv_in_dtype;         /* dtype of k and v                     */
  const void* slot_mapping;         /* device [N]                           */
  int64_t slot_stride;
  b200_index_t slot_dtype;
  int32_t* status;                  /* optional device word (may be NULL)   */
} b200_kv_scatter_args_t;

/*
 * Batched paged decode attention (one query token per sequence):
 *   out[b, h, :] = softmax(q[b, h, :] . K_b^T / sqrt(D)) V_b
 * over the first context_lengths[b] logical positions of sequence b, whose
 * logical block j lives in physical block block_tables[b, j].
 * Optionally fused with the decode KV write: when k_new, v_new and
 * slot_mapping are all non-NULL the kernel first stores k_new[b] / v_new[b]
 * at slot_mapping[b] (which must be the slot of logical position
 * context_lengths[b] - 1 of sequence b, as minivllm's ModelRunner builds it)
 * and then attends over it.
 * Replaces paged_attention_batch_triton_v0 (minivllm/triton_paged_decode.py:102)
 * and the reference backend paged_attention_batch_online_v1
 * (minivllm/paged_attention_batch.py:121) behind the selector at
 * minivllm/attention.py:394-416, plus the KV write at attention.py:370-392.
 *
 * Split-K: long contexts are cut into splits processed by different CTAs;
 * partial results go to `workspace` and the last CTA of a (sequence, head
 * group) combines them.  `workspace` must hold
 * b200_paged_decode_workspace_size(...) bytes; its contents need not be
 * initialised (the launch clears the split counters on `stream` first).
 *
 * Virtual-batch mode (used by the fp32 chunked prefill): when
 * context_lengths is NULL, context_lengths[b] = ctx_base + b + 1 and
 * block_table_stride[0] may be 0 so that every row shares one table.
 */
typedef struct {
  b200_kv_pool_t pool;
  int64_t layer_idx;
  int64_t batch;                    /* B >= 1                               */
  int64_t table_width;              /* M >= 1 (columns of block_tables)     */
  const void* q;                    /* [B, H, D] any strides                */
  int64_t q_stride[3];
  b200_dtype_t q_dtype;             /* f32 / bf16                           */
  void* out;                        /* [B, H, D] strides, dtype = out_dtype */
  int64_t out_stride[3];
  b200_dtype_t out_dtype;
  const void* block_tables;         /* device [B, M]                        */
  int64_t block_table_stride[2];
  b200_index_t block_table_dtype;
  const void* context_lengths;      /* device [B] or NULL (virtual batch)   */
  int64_t context_length_stride;
  b200_index_t context_length_dtype;
  int64_t ctx_base;                 /* used only when context_lengths==NULL */
  /* fused decode KV write (all three NULL for attention only) */
  const void* k_new;                /* [B, H, D] strides                    */
  const void* v_new;
  int64_t k_new_stride[3];
  int64_t v_new_stride[3];
  b200_dtype_t kv_new_dtype;
  const void* slot_mapping;         /* device [B]                           */
  int64_t slot_stride;
  b200_index_t slot_dtype;
  /* split-K scratch */
  void* workspace;
  size_t workspace_bytes;
  int32_t* status;                  /* optional device word (may be NULL)   */
  int32_t max_splits_hint;          /* 0 = automatic                        */
} b200_decode_args_t;

/*
 * Prefix-aware chunked prefill attention for one sequence:
 *   query i (absolute position prefix_len + i, 0 <= i < T) attends to keys
 *   0 .. prefix_len + i, all read from the paged pool through block_table.
 * The chunk's own K/V must already be in the pool (b200_kv_scatter first),
 * exactly as minivllm writes them before attention (attention.py:193-208).
 * out[i, h, :] is written for every head.
 * Replaces the prefix-aware SDPA v2 branch (minivllm/attention.py:229-267),
 * the first-chunk SDPA branch (attention.py:215-227) for prefix_len == 0,
 * and the per-token reference loop (attention.py:269-299).
 * bf16 pools with D in {64, 128} run on tcgen05 tensor cores (TMEM
 * accumulators, TMA-fed); f32 pools run the CUDA-core split-K kernel in
 * virtual-batch mode (exact fp32, TF32 never used) and need `workspace`
 * sized by b200_chunked_prefill_workspace_size().  A bf16 launch of fewer
 * CTAs than about 85 % of the SMs (one sequence's chunk) splits each chunk's
 * keys over several CTAs when `workspace` holds their partial rows (the same
 * size query; batched calls use seqs[0]'s workspace and split only as far as
 * it holds); without a workspace it runs unsplit, with the same results.
 */
typedef struct {
  b200_kv_pool_t pool;
  int64_t layer_idx;
  int64_t num_tokens;               /* T >= 1                               */
  int64_t prefix_len;               /* >= 0                                 */
  const void* q;                    /* [T, H, D] any strides                */
  int64_t q_stride[3];
  b200_dtype_t q_dtype;
  void* out;                        /* [T, H, D] strides                    */
  int64_t out_stride[3];
  b200_dtype_t out_dtype;
  const void* block_table;          /* device [>= ceil((prefix+T)/S)]       */
  int64_t block_table_len;
  int64_t block_table_stride;
  b200_index_t block_table_dtype;
  void* workspace;
  size_t workspace_bytes;
  int32_t* status;
} b200_prefill_args_t;

/* Batched variant: `num_seqs` independent prefill chunks in one launch. */
typedef struct {
  int64_t num_seqs;
  const b200_prefill_args_t* seqs;  /* host array, same pool/layer/dtypes   */
} b200_prefill_batch_args_t;

B200_API int b200_kv_scatter(const b200_kv_scatter_args_t* args, void* stream);
B200_API int b200_paged_decode(const b200_decode_args_t* args, void* stream);
B200_API int b200_chunked_prefill(const b200_prefill_args_t* args, void* stream);
B200_API int b200_chunked_prefill_batch(const b200_prefill_batch_args_t* args, void* stream);

/*
 * Paged decode that allocates nothing -- no counterpart in the reference.
 * For callers that may not allocate device memory (an engine that owns all
 * memory up front, a plugin restricted to the buffers it is given, a step
 * loop that must not call cudaMalloc): same arguments and results as
 * b200_paged_decode, but args->workspace / workspace_bytes are ignored and
 * the split-K scratch is a static device array of
 * B200_NO_ALLOC_SCRATCH_BYTES held by every GPU that loads the library.
 * Arguments are checked exactly as by b200_paged_decode first; calls needing
 * more scratch are then rejected with B200_ERR_UNSUPPORTED.  The first call
 * in a CUDA context looks up the array's address in that context (make it
 * before any stream capture); a later context on the same device, e.g.
 * after cudaDeviceReset, gets its own lookup.  All calls share the array:
 * calls that overlap on the GPU race and must be serialised by the caller.
 */
#define B200_NO_ALLOC_SCRATCH_BYTES (4u << 20)
B200_API int b200_paged_decode_no_alloc(const b200_decode_args_t* args, void* stream);

/*
 * Fused QKV projection with the KV write in its epilogue (bf16, tcgen05):
 *   y[t, :] = x[t, :] . W^T           W: [3C, C] weight of the bias-free
 *                                     `qkv` Linear (minivllm/attention.py:79-83)
 *   q_out[t, :] = y[t, 0:C]
 *   pool.k[layer, slot[t] / S, slot[t] % S, :, :] = y[t, C:2C]   (H * D = C)
 *   pool.v[layer, slot[t] / S, slot[t] % S, :, :] = y[t, 2C:3C]
 * with f32 accumulation and one round-to-nearest-even bf16 rounding per
 * output.  Replaces the projection, chunk(3) split and KV write of
 * forward_prefill_chunk (minivllm/attention.py:177-208, through
 * KVBlockPool.write_layer, minivllm/kv_block_pool.py:91-109) and of
 * forward_decode_batch (minivllm/attention.py:360-392); the attention call
 * that follows reads k/v from the pool (decode without k_new).
 * A slot outside [0, P*S) skips that token's k/v and sets B200_DEV_BAD_SLOT
 * in *status; its q row is still written.
 */
typedef struct {
  b200_kv_pool_t pool;              /* bf16, num_heads * head_dim == hidden */
  int64_t layer_idx;
  int64_t num_tokens;               /* T (0 is a no-op)                     */
  int64_t hidden;                   /* C: a multiple of 64                  */
  const void* x;                    /* [T, C] bf16, unit inner stride       */
  int64_t x_row_stride;             /* elements, a multiple of 8            */
  const void* weight;               /* [3C, C] bf16, contiguous             */
  void* q_out;                      /* [T, C] bf16, unit inner stride       */
  int64_t q_row_stride;             /* elements, a multiple of 8            */
  const void* slot_mapping;         /* device [T]                           */
  int64_t slot_stride;
  b200_index_t slot_dtype;
  int32_t* status;                  /* optional device word (may be NULL)   */
} b200_qkv_kv_write_args_t;

B200_API int b200_qkv_kv_write(const b200_qkv_kv_write_args_t* args, void* stream);

/* The kernel b200_qkv_kv_write launches for num_tokens x hidden on the
 * current device: *kind = 0 single CTAs (128 x *tile_n tiles), 1 CTA pairs
 * (256 x *tile_n tiles, *tile_n 192 or 256), 2 split-K clusters of *splits
 * CTAs (128 x *tile_n tiles).  A diagnostic with no counterpart in the reference. */
B200_API int b200_qkv_kv_write_plan(int64_t num_tokens, int64_t hidden, int32_t* kind,
                                    int32_t* tile_n, int32_t* splits);

/* Workspace bytes the decode launch needs for these sizes. */
B200_API size_t b200_paged_decode_workspace_size(int64_t batch, int64_t num_heads,
                                        int64_t head_dim, int64_t table_width,
                                        int64_t block_size, b200_dtype_t kv_dtype,
                                        int32_t max_splits_hint);
/* Workspace bytes one prefill call of `num_tokens` queries needs (0 when the
 * tensor-core path serves it). */
B200_API size_t b200_chunked_prefill_workspace_size(int64_t num_tokens, int64_t num_heads,
                                           int64_t head_dim, int64_t block_table_len,
                                           int64_t block_size, b200_dtype_t kv_dtype);

/* Copies the calling thread's last error message (NUL-terminated) into buf
 * and returns its full length. */
B200_API size_t b200_last_error(char* buf, size_t len);

/*
 * Failure-path self-test.  No counterpart in the reference: it exercises,
 * on the device, the bounded waits every kernel pipeline uses.  One warp
 * waits (through the same wait routine) on a barrier phase that nothing
 * completes; after limit_ns (0 < limit_ns <= 2e9) the kernel ORs
 * B200_DEV_WAIT_TIMEOUT into *status (a device word) and returns normally,
 * so the context stays usable.  Nothing faults, traps or hangs.
 */
B200_API int b200_selftest_bounded_wait(int32_t* status, int64_t limit_ns, void* stream);

/* ABI version and the compute capability the library was built for. */
B200_API int b200_abi_version(void);
B200_API int b200_built_arch(void);

#ifdef __cplusplus
}
#endif
#endif /* B200_PAGED_ATTN_H_ */
