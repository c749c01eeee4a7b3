// host_util.h -- host-side helpers shared by the launchers: error messages,
// TMA descriptor encoding through the driver entry point, device queries.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "b200_paged_attn.h"

namespace b200 {

// Thread-local last-error message (returned by b200_last_error).
void set_error(const std::string& msg);
void clear_error();
const std::string& last_error();

// Returns B200_OK or sets the error message and returns `code`.
int fail(int code, const std::string& msg);

// cudaError_t -> B200_ERR_CUDA with a message naming `what`.
int cuda_fail(cudaError_t e, const char* what);

size_t dtype_size(int dtype);

// Encodes a tiled tensor map (no swizzle unless requested, no interleave,
// zero fill for out-of-bounds elements).  dims / strides are innermost
// first; strides are in bytes for dims 1..rank-1.
int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType type, int rank, void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes,
                      const uint32_t* box, CUtensorMapSwizzle swizzle);

struct DeviceInfo {
  int device = -1;
  int num_sms = 0;
  int max_smem_optin = 0;
  int cc_major = 0;
  int cc_minor = 0;
};

// Cached per-device properties of the current device.
int current_device_info(DeviceInfo* info);

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline bool is_pow2(int64_t x) { return x > 0 && (x & (x - 1)) == 0; }
inline int log2i(int64_t x) {
  int r = 0;
  while ((int64_t(1) << r) < x) ++r;
  return r;
}

}  // namespace b200
