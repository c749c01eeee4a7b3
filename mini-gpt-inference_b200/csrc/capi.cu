// capi.cu -- the extern "C" entry points: host-side argument validation
// (mirroring the ValueError checks of minivllm/triton_paged_decode.py:109-144)
// and dispatch to the kernel launchers.
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "host_util.h"
#include "kernels.h"

namespace b200 {
namespace {

#define B200_CHECK(cond, code, msg)          \
  do {                                       \
    if (!(cond)) return fail((code), (msg)); \
  } while (0)

bool valid_dtype(int d) {
  return d == B200_DTYPE_F32 || d == B200_DTYPE_BF16 || d == B200_DTYPE_F16;
}
bool valid_index(int d) { return d == B200_INDEX_I32 || d == B200_INDEX_I64; }

int check_pool(const b200_kv_pool_t& p, int64_t layer_idx) {
  B200_CHECK(p.k != nullptr && p.v != nullptr, B200_ERR_INVALID_ARGUMENT,
             "KV pool pointers must be non-null");
  B200_CHECK(p.num_layers > 0 && p.num_blocks > 0 && p.block_size > 0 && p.num_heads > 0 &&
                 p.head_dim > 0,
             B200_ERR_INVALID_ARGUMENT, "KV pool dimensions must be nonzero");
  B200_CHECK(p.dtype == B200_DTYPE_F32 || p.dtype == B200_DTYPE_BF16, B200_ERR_UNSUPPORTED,
             "KV pool dtype must be float32 or bfloat16");
  B200_CHECK(0 <= layer_idx && layer_idx < p.num_layers, B200_ERR_INVALID_ARGUMENT,
             "layer_idx outside KV pool");
  B200_CHECK(is_pow2(p.block_size) && p.block_size <= 256, B200_ERR_UNSUPPORTED,
             "block_size must be a power of two <= 256");
  B200_CHECK(p.head_dim <= 128, B200_ERR_UNSUPPORTED, "head_dim must be <= 128");
  const int64_t es = static_cast<int64_t>(dtype_size(p.dtype));
  B200_CHECK((p.head_dim * es) % 16 == 0, B200_ERR_UNSUPPORTED,
             "head_dim * element size must be a multiple of 16 bytes");
  B200_CHECK((reinterpret_cast<uintptr_t>(p.k) % 16) == 0 &&
                 (reinterpret_cast<uintptr_t>(p.v) % 16) == 0,
             B200_ERR_INVALID_ARGUMENT, "KV pool base pointers must be 16-byte aligned");
  B200_CHECK(p.num_layers * p.num_blocks * p.block_size < (int64_t(1) << 31),
             B200_ERR_UNSUPPORTED, "KV pool has more than 2^31 token rows");
  return B200_OK;
}

int check_decode(const b200_decode_args_t& a) {
  int rc = check_pool(a.pool, a.layer_idx);
  if (rc != B200_OK) return rc;
  B200_CHECK(a.batch >= 1, B200_ERR_INVALID_ARGUMENT, "q dimensions must be nonzero");
  B200_CHECK(a.batch < (int64_t(1) << 24), B200_ERR_UNSUPPORTED, "batch too large");
  B200_CHECK(a.table_width >= 1, B200_ERR_INVALID_ARGUMENT,
             "block_tables need at least one block column");
  B200_CHECK(a.q != nullptr && a.out != nullptr, B200_ERR_INVALID_ARGUMENT,
             "q and out must be non-null");
  B200_CHECK(valid_dtype(a.q_dtype) && valid_dtype(a.out_dtype), B200_ERR_INVALID_ARGUMENT,
             "q/out dtype must be float32, bfloat16 or float16");
  B200_CHECK(a.block_tables != nullptr, B200_ERR_INVALID_ARGUMENT,
             "block_tables must be non-null");
  B200_CHECK(valid_index(a.block_table_dtype), B200_ERR_INVALID_ARGUMENT,
             "block_tables must contain integer indices");
  if (a.context_lengths != nullptr)
    B200_CHECK(valid_index(a.context_length_dtype), B200_ERR_INVALID_ARGUMENT,
               "context_lengths must be integer");
  else
    B200_CHECK(a.ctx_base >= 0, B200_ERR_INVALID_ARGUMENT, "ctx_base must be >= 0");
  const bool any_new = a.k_new || a.v_new || a.slot_mapping;
  const bool all_new = a.k_new && a.v_new && a.slot_mapping;
  B200_CHECK(any_new == all_new, B200_ERR_INVALID_ARGUMENT,
             "k_new, v_new and slot_mapping must be given together");
  if (all_new) {
    B200_CHECK(valid_dtype(a.kv_new_dtype), B200_ERR_INVALID_ARGUMENT,
               "k_new/v_new dtype must be float32, bfloat16 or float16");
    B200_CHECK(valid_index(a.slot_dtype), B200_ERR_INVALID_ARGUMENT,
               "slot_mapping must be integer");
    B200_CHECK(a.context_lengths != nullptr, B200_ERR_INVALID_ARGUMENT,
               "the fused KV write needs context_lengths");
  }
  return B200_OK;
}

int check_prefill(const b200_prefill_args_t& a) {
  int rc = check_pool(a.pool, a.layer_idx);
  if (rc != B200_OK) return rc;
  B200_CHECK(a.num_tokens >= 1, B200_ERR_INVALID_ARGUMENT, "prefill chunk must be nonempty");
  B200_CHECK(a.prefix_len >= 0, B200_ERR_INVALID_ARGUMENT, "prefix_len must be >= 0");
  // Positions are 32-bit in the kernels; the fp32 path runs the chunk as a
  // decode batch, whose size limit it shares.
  B200_CHECK(a.num_tokens < (int64_t(1) << 24) && a.prefix_len + a.num_tokens < (int64_t(1) << 31),
             B200_ERR_UNSUPPORTED, "prefill chunk too large (num_tokens < 2^24, positions < 2^31)");
  B200_CHECK(a.q != nullptr && a.out != nullptr, B200_ERR_INVALID_ARGUMENT,
             "q and out must be non-null");
  B200_CHECK(valid_dtype(a.q_dtype) && valid_dtype(a.out_dtype), B200_ERR_INVALID_ARGUMENT,
             "q/out dtype must be float32, bfloat16 or float16");
  B200_CHECK(a.block_table != nullptr, B200_ERR_INVALID_ARGUMENT,
             "block_table must be non-null");
  B200_CHECK(valid_index(a.block_table_dtype), B200_ERR_INVALID_ARGUMENT,
             "block_table must contain integer indices");
  B200_CHECK(a.block_table_len * a.pool.block_size >= a.prefix_len + a.num_tokens,
             B200_ERR_INVALID_ARGUMENT, "incomplete KV block table for prefix and chunk");
  return B200_OK;
}

// The f32 (and odd-shaped bf16) prefill runs the split-K decode kernel in
// virtual-batch mode: query i is a decode "sequence" of context length
// prefix_len + i + 1 over the shared block table.
b200_decode_args_t prefill_as_decode(const b200_prefill_args_t& a) {
  b200_decode_args_t d{};
  d.pool = a.pool;
  d.layer_idx = a.layer_idx;
  d.batch = a.num_tokens;
  d.table_width = a.block_table_len;
  d.q = a.q;
  memcpy(d.q_stride, a.q_stride, sizeof(d.q_stride));
  d.q_dtype = a.q_dtype;
  d.out = a.out;
  memcpy(d.out_stride, a.out_stride, sizeof(d.out_stride));
  d.out_dtype = a.out_dtype;
  d.block_tables = a.block_table;
  d.block_table_stride[0] = 0;
  d.block_table_stride[1] = a.block_table_stride;
  d.block_table_dtype = a.block_table_dtype;
  d.context_lengths = nullptr;
  d.ctx_base = a.prefix_len;
  d.workspace = a.workspace;
  d.workspace_bytes = a.workspace_bytes;
  d.status = a.status;
  return d;
}

int sm_count() {
  DeviceInfo dev;
  if (current_device_info(&dev) != B200_OK) return 148;
  return dev.num_sms;
}

}  // namespace

int validate_decode_args(const b200_decode_args_t& a) { return check_decode(a); }

}  // namespace b200

using namespace b200;

extern "C" {

int b200_abi_version(void) { return B200_PAGED_ATTN_ABI_VERSION; }

int b200_selftest_bounded_wait(int32_t* status, int64_t limit_ns, void* stream) {
  clear_error();
  if (status == nullptr) return fail(B200_ERR_INVALID_ARGUMENT, "selftest: status must be a device word");
  if (limit_ns <= 0 || limit_ns > 2000000000LL)
    return fail(B200_ERR_INVALID_ARGUMENT, "selftest: limit_ns must be in (0, 2e9]");
  return launch_bounded_wait_selftest(status, limit_ns, static_cast<cudaStream_t>(stream));
}
int b200_built_arch(void) { return 100; }

size_t b200_last_error(char* buf, size_t len) {
  const std::string& msg = last_error();
  if (buf != nullptr && len > 0) {
    const size_t n = std::min(len - 1, msg.size());
    memcpy(buf, msg.data(), n);
    buf[n] = '\0';
  }
  return msg.size();
}

int b200_kv_scatter(const b200_kv_scatter_args_t* args, void* stream) {
  clear_error();
  if (args == nullptr) return fail(B200_ERR_INVALID_ARGUMENT, "null arguments");
  const b200_kv_scatter_args_t& a = *args;
  int rc = check_pool(a.pool, a.layer_idx);
  if (rc != B200_OK) return rc;
  if (a.num_tokens < 0) return fail(B200_ERR_INVALID_ARGUMENT, "num_tokens must be >= 0");
  if (a.num_tokens == 0) return B200_OK;
  // One CTA per token: the grid's x extent bounds N (a pool holds < 2^31 rows anyway).
  if (a.num_tokens >= (int64_t(1) << 31) - 1)
    return fail(B200_ERR_UNSUPPORTED, "kv scatter: num_tokens must be < 2^31 - 1");
  if (a.k == nullptr || a.v == nullptr || a.slot_mapping == nullptr)
    return fail(B200_ERR_INVALID_ARGUMENT, "k, v and slot_mapping must be non-null");
  if (!valid_dtype(a.kv_in_dtype))
    return fail(B200_ERR_INVALID_ARGUMENT, "k/v dtype must be float32, bfloat16 or float16");
  if (!valid_index(a.slot_dtype))
    return fail(B200_ERR_INVALID_ARGUMENT, "slot_mapping must be integer");
  return launch_kv_scatter(a, static_cast<cudaStream_t>(stream));
}

int b200_qkv_kv_write(const b200_qkv_kv_write_args_t* args, void* stream) {
  clear_error();
  if (args == nullptr) return fail(B200_ERR_INVALID_ARGUMENT, "null arguments");
  const b200_qkv_kv_write_args_t& a = *args;
  int rc = check_pool(a.pool, a.layer_idx);
  if (rc != B200_OK) return rc;
  if (a.num_tokens < 0) return fail(B200_ERR_INVALID_ARGUMENT, "num_tokens must be >= 0");
  if (a.num_tokens == 0) return B200_OK;
  B200_CHECK(a.x != nullptr && a.weight != nullptr && a.q_out != nullptr && a.slot_mapping != nullptr,
             B200_ERR_INVALID_ARGUMENT, "x, weight, q_out and slot_mapping must be non-null");
  B200_CHECK(a.pool.dtype == B200_DTYPE_BF16, B200_ERR_UNSUPPORTED,
             "qkv projection: the KV pool must be bfloat16");
  B200_CHECK(a.hidden >= 64 && a.hidden % 64 == 0, B200_ERR_UNSUPPORTED,
             "qkv projection: hidden size must be a positive multiple of 64");
  B200_CHECK(a.pool.num_heads * a.pool.head_dim == a.hidden, B200_ERR_INVALID_ARGUMENT,
             "qkv projection: num_heads * head_dim must equal the hidden size");
  B200_CHECK(a.hidden <= (int64_t(1) << 20) && a.num_tokens < (int64_t(1) << 31) / 2,
             B200_ERR_UNSUPPORTED, "qkv projection: sizes too large");
  // Tile indices are 32-bit: bound the finest tiling (128 tokens x 32 features).
  B200_CHECK(ceil_div(a.num_tokens, 128) * ceil_div(3 * a.hidden, 32) < (int64_t(1) << 31),
             B200_ERR_UNSUPPORTED, "qkv projection: too many output tiles (split the tokens)");
  B200_CHECK(a.x_row_stride >= a.hidden && a.x_row_stride % 8 == 0 &&
                 a.q_row_stride >= a.hidden && a.q_row_stride % 8 == 0,
             B200_ERR_UNSUPPORTED,
             "qkv projection: x and q_out rows must be 16-byte aligned and not overlap");
  B200_CHECK(reinterpret_cast<uintptr_t>(a.x) % 16 == 0 &&
                 reinterpret_cast<uintptr_t>(a.weight) % 16 == 0 &&
                 reinterpret_cast<uintptr_t>(a.q_out) % 16 == 0,
             B200_ERR_UNSUPPORTED, "qkv projection: x, weight and q_out must be 16-byte aligned");
  B200_CHECK(valid_index(a.slot_dtype), B200_ERR_INVALID_ARGUMENT, "slot_mapping must be integer");
  return launch_qkv_kv_write(a, static_cast<cudaStream_t>(stream));
}

int b200_qkv_kv_write_plan(int64_t num_tokens, int64_t hidden, int32_t* kind, int32_t* tile_n,
                           int32_t* splits) {
  clear_error();
  B200_CHECK(kind != nullptr && tile_n != nullptr && splits != nullptr, B200_ERR_INVALID_ARGUMENT,
             "null output pointer");
  B200_CHECK(num_tokens >= 1 && hidden >= 64 && hidden % 64 == 0, B200_ERR_INVALID_ARGUMENT,
             "qkv projection plan: num_tokens >= 1 and hidden a positive multiple of 64");
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc != B200_OK) return rc;
  const QkvPlan plan = qkv_plan(num_tokens, hidden, dev);
  *kind = plan.kind;
  *tile_n = plan.bn;
  *splits = plan.splits;
  return B200_OK;
}

int b200_paged_decode(const b200_decode_args_t* args, void* stream) {
  clear_error();
  if (args == nullptr) return fail(B200_ERR_INVALID_ARGUMENT, "null arguments");
  int rc = check_decode(*args);
  if (rc != B200_OK) return rc;
  return launch_paged_decode(*args, static_cast<cudaStream_t>(stream));
}

int b200_chunked_prefill(const b200_prefill_args_t* args, void* stream) {
  clear_error();
  if (args == nullptr) return fail(B200_ERR_INVALID_ARGUMENT, "null arguments");
  int rc = check_prefill(*args);
  if (rc != B200_OK) return rc;
  if (prefill_tc_supported(*args)) return launch_prefill_tc(args, 1, static_cast<cudaStream_t>(stream));
  return launch_paged_decode(prefill_as_decode(*args), static_cast<cudaStream_t>(stream));
}

int b200_chunked_prefill_batch(const b200_prefill_batch_args_t* args, void* stream) {
  clear_error();
  if (args == nullptr || (args->num_seqs > 0 && args->seqs == nullptr))
    return fail(B200_ERR_INVALID_ARGUMENT, "null arguments");
  const int64_t n = args->num_seqs;
  if (n == 0) return B200_OK;
  bool all_tc = true;
  for (int64_t i = 0; i < n; ++i) {
    const b200_prefill_args_t& s = args->seqs[i];
    int rc = check_prefill(s);
    if (rc != B200_OK) return rc;
    const b200_prefill_args_t& s0 = args->seqs[0];
    if (s.pool.k != s0.pool.k || s.pool.v != s0.pool.v || s.pool.dtype != s0.pool.dtype ||
        s.pool.num_blocks != s0.pool.num_blocks || s.pool.block_size != s0.pool.block_size ||
        s.pool.num_heads != s0.pool.num_heads || s.pool.head_dim != s0.pool.head_dim ||
        s.pool.num_layers != s0.pool.num_layers || s.layer_idx != s0.layer_idx ||
        s.q_dtype != s0.q_dtype || s.out_dtype != s0.out_dtype)
      return fail(B200_ERR_INVALID_ARGUMENT,
                  "batched prefill sequences must share pool, layer and dtypes");
    all_tc = all_tc && prefill_tc_supported(s);
  }
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (all_tc) return launch_prefill_tc(args->seqs, n, st);
  for (int64_t i = 0; i < n; ++i) {
    int rc = launch_paged_decode(prefill_as_decode(args->seqs[i]), st);
    if (rc != B200_OK) return rc;
  }
  return B200_OK;
}

size_t b200_paged_decode_workspace_size(int64_t batch, int64_t num_heads, int64_t head_dim,
                                        int64_t table_width, int64_t block_size,
                                        b200_dtype_t kv_dtype, int32_t max_splits_hint) {
  const size_t es = dtype_size(kv_dtype);
  if (es == 0 || batch < 1 || num_heads < 1 || head_dim < 1 || table_width < 1 ||
      block_size < 1)
    return 0;
  return decode_workspace_bytes(batch, num_heads, head_dim, table_width, block_size,
                                max_splits_hint, es, sm_count());
}

size_t b200_chunked_prefill_workspace_size(int64_t num_tokens, int64_t num_heads,
                                           int64_t head_dim, int64_t block_table_len,
                                           int64_t block_size, b200_dtype_t kv_dtype) {
  b200_prefill_args_t probe{};
  probe.pool.dtype = kv_dtype;
  probe.pool.head_dim = head_dim;
  probe.pool.num_heads = num_heads;
  probe.pool.block_size = block_size;
  probe.num_tokens = num_tokens;
  if (prefill_tc_supported(probe))
    return prefill_tc_workspace_bytes(num_tokens, num_heads, head_dim, block_table_len * block_size,
                                      sm_count());
  return b200_paged_decode_workspace_size(num_tokens, num_heads, head_dim, block_table_len,
                                          block_size, kv_dtype, 0);
}

}  // extern "C"
