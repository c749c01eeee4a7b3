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
// library holds it until the process exits.  In host code its name is only a
// host-side stand-in, so the launch needs its device address: that is looked
// up with cudaGetSymbolAddress, with the device current, by the first call
// made in a CUDA context, and cached per device together with the context's
// unique id.  A call made in another context of the same device (after a
// cudaDeviceReset, or from a driver-API context) looks the address up again,
// so a cached address never outlives its context.  The first call in a
// context should therefore come before any stream capture.  All calls share
// the array and it keeps the last call's contents: the split counters are
// cleared on the stream by every launch and the partial results are always
// written before they are read, but two calls that overlap on the GPU
// (different streams, or different host threads) race on it and must be
// serialised by the caller.
#include <stdio.h>

#include <mutex>

#include "host_util.h"
#include "kernels.h"

namespace b200 {
namespace {

static __device__ __align__(256) uint8_t g_decode_scratch[B200_NO_ALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;

struct ScratchSlot {
  void* ptr = nullptr;
  unsigned long long ctx_id = 0;  // cuCtxGetId of the context ptr belongs to
};

std::mutex g_scratch_mu;
ScratchSlot g_scratch[kMaxDevices];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// The driver's cuCtxGetCurrent / cuCtxGetId, fetched through the runtime's
// entry-point query (the library links no libcuda).  Both stay null when the
// driver does not offer them; the address is then looked up on every call.
struct CtxQueries {
  CtxGetCurrentFn get_current = nullptr;
  CtxGetIdFn get_id = nullptr;
  CtxQueries() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  }
};

// Unique id of the calling thread's current context, or 0 when unknown.
unsigned long long current_ctx_id() {
  static const CtxQueries fns;
  if (fns.get_current == nullptr || fns.get_id == nullptr) return 0;
  CUcontext ctx = nullptr;
  if (fns.get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (fns.get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of g_decode_scratch in the current context of `device`.
int scratch_address(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchSlot& slot = g_scratch[device];
  const unsigned long long id = current_ctx_id();
  if (slot.ptr == nullptr || id == 0 || slot.ctx_id != id) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(decode scratch)");
    slot.ptr = p;
    // The lookup above creates the context if none was current yet.
    slot.ctx_id = id != 0 ? id : current_ctx_id();
  }
  *out = slot.ptr;
  return B200_OK;
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" int b200_paged_decode_no_alloc(const b200_decode_args_t* args, void* stream) {
  clear_error();
  if (args == nullptr) return fail(B200_ERR_INVALID_ARGUMENT, "null arguments");
  const b200_decode_args_t& a = *args;
  // The same checks and messages as b200_paged_decode, before any size
  // arithmetic on the arguments.
  int rc = validate_decode_args(a);
  if (rc != B200_OK) return rc;
  DeviceInfo dev;
  rc = current_device_info(&dev);
  if (rc != B200_OK) return rc;
  if (dev.device < 0 || dev.device >= kMaxDevices)
    return fail(B200_ERR_UNSUPPORTED, "device ordinal out of range");
  const size_t need = decode_workspace_bytes(a.batch, a.pool.num_heads, a.pool.head_dim,
                                             a.table_width, a.pool.block_size,
                                             a.max_splits_hint, dtype_size(a.pool.dtype),
                                             dev.num_sms);
  if (need > static_cast<size_t>(B200_NO_ALLOC_SCRATCH_BYTES)) {
    char buf[200];
    snprintf(buf, sizeof(buf),
             "paged decode (no-alloc) needs %zu bytes of split-K scratch, more than the "
             "%zu-byte static scratch; use b200_paged_decode with a workspace",
             need, static_cast<size_t>(B200_NO_ALLOC_SCRATCH_BYTES));
    return fail(B200_ERR_UNSUPPORTED, buf);
  }
  void* scratch = nullptr;
  rc = scratch_address(dev.device, &scratch);
  if (rc != B200_OK) return rc;
  b200_decode_args_t local = a;
  local.workspace = scratch;
  local.workspace_bytes = B200_NO_ALLOC_SCRATCH_BYTES;
  return b200_paged_decode(&local, stream);
}
