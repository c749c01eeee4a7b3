// paged_decode_no_alloc.cu -- b200_paged_decode_no_alloc: the paged decode
// for callers that cannot allocate device memory.
//
// Some hosts embed this library where no allocator is available to it: a
// runtime that owns every byte of device memory up front (a serving engine
// with a fixed memory plan, an inference server plugin that may only use the
// buffers handed to it) or code that must not call cudaMalloc, which can
// synchronise the device, between its steps.  For those callers the split-K
// scratch of the decode comes from one file-scope device array instead of a
// caller-provided workspace.
//
// The array is B200_NO_ALLOC_SCRATCH_BYTES large; every GPU that loads the
// library holds it until the process exits.  Its device address is looked up
// with cudaGetSymbolAddress once per device, by the first call made while
// that device is current (so that first call should come before any stream
// capture).  All calls share the array and it keeps the last call's
// contents: the split counters are cleared on the stream by every launch and
// the partial results are always written before they are read, but two calls
// that overlap on the GPU (different streams, or different host threads) race
// on it and must be serialised by the caller.
#include <stdio.h>

#include <mutex>

#include "host_util.h"
#include "kernels.h"

namespace b200 {
namespace {

static __device__ __align__(256) uint8_t g_decode_scratch[B200_NO_ALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of g_decode_scratch on the current device (set up once).
int scratch_address(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[device] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(decode scratch)");
    g_scratch_ptr[device] = p;
  }
  *out = g_scratch_ptr[device];
  return B200_OK;
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" int b200_paged_decode_no_alloc(const b200_decode_args_t* args, void* stream) {
  clear_error();
  if (args == nullptr) return fail(B200_ERR_INVALID_ARGUMENT, "null arguments");
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc != B200_OK) return rc;
  if (dev.device < 0 || dev.device >= kMaxDevices)
    return fail(B200_ERR_UNSUPPORTED, "device ordinal out of range");
  const b200_decode_args_t& a = *args;
  const size_t es = dtype_size(a.pool.dtype);
  if (es != 0 && a.batch >= 1 && a.pool.num_heads >= 1 && a.pool.head_dim >= 1 &&
      a.table_width >= 1 && a.pool.block_size >= 1) {
    const size_t need = decode_workspace_bytes(a.batch, a.pool.num_heads, a.pool.head_dim,
                                               a.table_width, a.pool.block_size,
                                               a.max_splits_hint, es, dev.num_sms);
    if (need > static_cast<size_t>(B200_NO_ALLOC_SCRATCH_BYTES)) {
      char buf[200];
      snprintf(buf, sizeof(buf),
               "paged decode (no-alloc) needs %zu bytes of split-K scratch, more than the "
               "%zu-byte static scratch; use b200_paged_decode with a workspace",
               need, static_cast<size_t>(B200_NO_ALLOC_SCRATCH_BYTES));
      return fail(B200_ERR_UNSUPPORTED, buf);
    }
  }
  void* scratch = nullptr;
  rc = scratch_address(dev.device, &scratch);
  if (rc != B200_OK) return rc;
  b200_decode_args_t local = a;
  local.workspace = scratch;
  local.workspace_bytes = B200_NO_ALLOC_SCRATCH_BYTES;
  return b200_paged_decode(&local, stream);
}
