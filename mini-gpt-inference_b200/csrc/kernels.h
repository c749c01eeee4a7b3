// kernels.h -- launcher entry points of the device kernels (host side).
// Arguments arrive already validated by capi.cu.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "b200_paged_attn.h"

namespace b200 {

using DecodeLaunch = b200_decode_args_t;

// The host-side checks b200_paged_decode runs on its arguments (capi.cu):
// B200_OK, or the status and message it would return.
int validate_decode_args(const b200_decode_args_t& a);

int launch_paged_decode(const DecodeLaunch& a, cudaStream_t stream);
int launch_kv_scatter(const b200_kv_scatter_args_t& a, cudaStream_t stream);
// tcgen05 prefill over `n` sequences sharing one pool (bf16, D in {64,128}).
int launch_prefill_tc(const b200_prefill_args_t* seqs, int64_t n, cudaStream_t stream);
bool prefill_tc_supported(const b200_prefill_args_t& a);
// Workspace for a key split over CTAs of one bf16 sequence's chunk (T tokens,
// at most `keys` keys); 0 when its launch needs none.
size_t prefill_tc_workspace_bytes(int64_t T, int64_t H, int64_t D, int64_t keys, int num_sms);
// One warp waiting on an mbarrier nothing arrives on, with the given limit.
// Fused QKV projection + KV write (tcgen05, bf16).  qkv_plan is the kernel
// and tile shape it launches for T tokens of hidden size C: single CTAs with
// BN-wide tiles, CTA pairs with 256 x 256 tiles, or split-K clusters.
struct QkvPlan {
  enum Kind { kSingle = 0, kPair = 1, kSplit = 2 };
  int kind;
  int bn;      // output features per tile
  int splits;  // reduction split (cluster size) of kSplit
  int xrows;   // x box rows of kSplit
};
int launch_qkv_kv_write(const b200_qkv_kv_write_args_t& a, cudaStream_t stream);
struct DeviceInfo;
QkvPlan qkv_plan(int64_t T, int64_t C, const DeviceInfo& dev);
int launch_bounded_wait_selftest(int32_t* status, int64_t limit_ns, cudaStream_t stream);

// Split-K planning shared by the launcher and the workspace query.
size_t decode_workspace_bytes(int64_t B, int64_t H, int64_t D, int64_t M, int64_t S,
                              int32_t hint, size_t es, int num_sms);

}  // namespace b200
