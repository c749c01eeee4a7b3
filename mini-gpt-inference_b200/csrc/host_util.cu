// host_util.cu -- error plumbing, TMA descriptor encoding and device queries.
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "host_util.h"

namespace b200 {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }
void clear_error() { g_last_error.clear(); }
const std::string& last_error() { return g_last_error; }

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                  cudaGetErrorString(e) + ")";
  return fail(B200_ERR_CUDA, m);
}

size_t dtype_size(int dtype) {
  switch (dtype) {
    case B200_DTYPE_F32: return 4;
    case B200_DTYPE_BF16: return 2;
    case B200_DTYPE_F16: return 2;
    default: return 0;
  }
}

// cuTensorMapEncodeTiled is a driver API function; it is fetched through the
// runtime's entry-point query so the library does not link libcuda directly.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType type, int rank, void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes,
                      const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, type, static_cast<cuuint32_t>(rank), base,
                  reinterpret_cast<const cuuint64_t*>(dims),
                  reinterpret_cast<const cuuint64_t*>(strides_bytes),
                  reinterpret_cast<const cuuint32_t*>(box), elem_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    snprintf(buf, sizeof(buf),
             "cuTensorMapEncodeTiled failed (CUresult %d): rank %d dims [%llu %llu %llu] "
             "box [%u %u %u]",
             static_cast<int>(r), rank, (unsigned long long)dims[0],
             (unsigned long long)(rank > 1 ? dims[1] : 0),
             (unsigned long long)(rank > 2 ? dims[2] : 0), box[0], rank > 1 ? box[1] : 0,
             rank > 2 ? box[2] : 0);
    return fail(B200_ERR_CUDA, buf);
  }
  return B200_OK;
}

int current_device_info(DeviceInfo* info) {
  static std::mutex mu;
  static DeviceInfo cache[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(B200_ERR_CUDA, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(mu);
  DeviceInfo& d = cache[dev];
  if (d.device != dev) {
    DeviceInfo n;
    n.device = dev;
    if ((e = cudaDeviceGetAttribute(&n.num_sms, cudaDevAttrMultiProcessorCount, dev)) !=
        cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    if ((e = cudaDeviceGetAttribute(&n.max_smem_optin,
                                    cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) !=
        cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute(smem)");
    if ((e = cudaDeviceGetAttribute(&n.cc_major, cudaDevAttrComputeCapabilityMajor, dev)) !=
        cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute(cc major)");
    if ((e = cudaDeviceGetAttribute(&n.cc_minor, cudaDevAttrComputeCapabilityMinor, dev)) !=
        cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute(cc minor)");
    d = n;
  }
  *info = d;
  return B200_OK;
}

}  // namespace b200
