// kv_scatter.cu -- slot-mapping KV-cache scatter.
//
// For every token n the H*D elements of k[n] (and v[n]) are stored as one
// contiguous run at pool[layer, slot[n] / S, slot[n] % S, :, :].  The pool run
// is contiguous, so the kernel writes it with 16-byte vector stores; source
// rows are read with 16-byte loads when their innermost stride is 1 and
// aligned, else element by element (q/k/v arrive as strided views of the
// fused QKV projection, minivllm/attention.py:180-191 and :360-368).
// Semantics: minivllm/attention.py:370-392 (decode) and :193-208 via
// KVBlockPool.write_layer (minivllm/kv_block_pool.py:91-109) (prefill).
#include <algorithm>

#include "common.cuh"
#include "host_util.h"
#include "kernels.h"

namespace b200 {

struct ScatterParams {
  int64_t N, H, D, S, P;
  int64_t layer_row0;  // layer * P * S
  const void* k;
  const void* v;
  int64_t ks0, ks1, ks2, vs0, vs1, vs2;
  int32_t in_dtype;
  void* kp;
  void* vp;
  int32_t pool_dtype;
  const void* slots;
  int64_t ss;
  int32_t slots_i64;
  int32_t vec_ok;  // 16-byte loads legal for both k and v
  int32_t* status;
};

// Same-dtype copy of tokens whose H*D run is contiguous in k, v and the pool
// (q/k/v views of a fused projection have head stride D): a flat 16-byte
// copy of H*D*es bytes per tensor.  Each thread issues all of its loads (up
// to kFlatIter chunks of k and of v) before its stores, with streaming
// cache hints (the data is read and written once).
constexpr int kFlatIter = 4;
struct FlatParams {
  int64_t P, S;
  int64_t layer_row0;
  int64_t run;        // 16-byte chunks per token per tensor
  int64_t k_tok, v_tok;  // token stride of k / v in 16-byte chunks
  const uint4* k;
  const uint4* v;
  uint4* kp;
  uint4* vp;
  const void* slots;
  int64_t ss;
  int32_t slots_i64;
  int32_t* status;
};

__global__ void __launch_bounds__(256) kv_scatter_flat_kernel(const FlatParams p) {
  const int64_t n = blockIdx.x;
  const int64_t slot = load_index(p.slots, n * p.ss, p.slots_i64);
  if (slot < 0 || slot >= p.P * p.S) {
    if (threadIdx.x == 0) report(p.status, B200_DEV_BAD_SLOT);
    return;
  }
  const uint4* ks = p.k + n * p.k_tok;
  const uint4* vs = p.v + n * p.v_tok;
  uint4* kd = p.kp + (p.layer_row0 + slot) * p.run;
  uint4* vd = p.vp + (p.layer_row0 + slot) * p.run;
  const int run = static_cast<int>(p.run);
  for (int base = threadIdx.x; base < run; base += kFlatIter * blockDim.x) {
    uint4 a[kFlatIter], b[kFlatIter];
#pragma unroll
    for (int i = 0; i < kFlatIter; ++i) {
      const int c = base + i * blockDim.x;
      if (c < run) {
        a[i] = __ldcs(ks + c);
        b[i] = __ldcs(vs + c);
      }
    }
#pragma unroll
    for (int i = 0; i < kFlatIter; ++i) {
      const int c = base + i * blockDim.x;
      if (c < run) {
        __stcs(kd + c, a[i]);
        __stcs(vd + c, b[i]);
      }
    }
  }
}

template <typename PoolT>
struct Pack;
template <>
struct Pack<float> {
  static constexpr int N = 4;
  __device__ __forceinline__ static uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
};
template <>
struct Pack<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ __forceinline__ static uint4 pack(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

// Reads N consecutive d-elements of row (n, h) starting at d0 as floats.
template <int N>
__device__ __forceinline__ void read_run(const void* base, int64_t off, int64_t sd, int dtype,
                                         bool vec, int64_t d0, int64_t D, float* f) {
  if (vec && d0 + N <= D) {
    if (dtype == B200_DTYPE_F32) {
#pragma unroll
      for (int i = 0; i < N; i += 4) {
        const float4 x = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + off + i);
        f[i] = x.x;
        f[i + 1] = x.y;
        f[i + 2] = x.z;
        f[i + 3] = x.w;
      }
      return;
    }
    if (dtype == B200_DTYPE_BF16) {
#pragma unroll
      for (int i = 0; i < N; i += 8) {
        const uint4 raw = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(base) + off + i);
        Elem<__nv_bfloat16>::unpack(raw, f + i);
      }
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i)
    f[i] = (d0 + i < D) ? load_elem(base, off + i * sd, dtype) : 0.f;
}

// One CTA per token: the token's H*D elements form one contiguous run in the
// pool, and (for q/k/v views of a fused projection) one contiguous run in the
// source as well, so the CTA copies 16-byte chunks with no index division.
// Rows whose heads are not contiguous fall back to per-head addressing with
// 32-bit arithmetic.
template <typename PoolT>
__global__ void __launch_bounds__(256) kv_scatter_kernel(const ScatterParams p) {
  constexpr int NE = Pack<PoolT>::N;
  const int64_t n = blockIdx.x;
  const int64_t slot = load_index(p.slots, n * p.ss, p.slots_i64);
  if (slot < 0 || slot >= p.P * p.S) {
    if (threadIdx.x == 0) report(p.status, B200_DEV_BAD_SLOT);
    return;
  }
  const int D = static_cast<int>(p.D);
  const int cpr = (D + NE - 1) / NE;               // chunks per head row
  const int chunks = static_cast<int>(p.H) * cpr;  // chunks per token
  const bool full_chunks = (D % NE) == 0;
  const int64_t dst0 = (p.layer_row0 + slot) * p.H * p.D;
  const int64_t ks0 = n * p.ks0, vs0 = n * p.vs0;
  for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
    const int h = c / cpr;
    const int d0 = (c - h * cpr) * NE;
    float fk[NE], fv[NE];
    read_run<NE>(p.k, ks0 + h * p.ks1 + d0 * p.ks2, p.ks2, p.in_dtype, p.vec_ok, d0, p.D, fk);
    read_run<NE>(p.v, vs0 + h * p.vs1 + d0 * p.vs2, p.vs2, p.in_dtype, p.vec_ok, d0, p.D, fv);
    const int64_t dst = dst0 + static_cast<int64_t>(h) * D + d0;
    if (full_chunks) {
      *reinterpret_cast<uint4*>(static_cast<PoolT*>(p.kp) + dst) = Pack<PoolT>::pack(fk);
      *reinterpret_cast<uint4*>(static_cast<PoolT*>(p.vp) + dst) = Pack<PoolT>::pack(fv);
    } else {
      for (int e = 0; e < NE && d0 + e < D; ++e) {
        store_elem(p.kp, dst + e, p.pool_dtype, fk[e]);
        store_elem(p.vp, dst + e, p.pool_dtype, fv[e]);
      }
    }
  }
}

int launch_kv_scatter(const b200_kv_scatter_args_t& a, cudaStream_t stream) {
  if (a.num_tokens == 0) return B200_OK;
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc != B200_OK) return rc;
  ScatterParams p{};
  p.N = a.num_tokens;
  p.H = a.pool.num_heads;
  p.D = a.pool.head_dim;
  p.S = a.pool.block_size;
  p.P = a.pool.num_blocks;
  p.layer_row0 = a.layer_idx * a.pool.num_blocks * a.pool.block_size;
  p.k = a.k;
  p.v = a.v;
  p.ks0 = a.k_stride[0];
  p.ks1 = a.k_stride[1];
  p.ks2 = a.k_stride[2];
  p.vs0 = a.v_stride[0];
  p.vs1 = a.v_stride[1];
  p.vs2 = a.v_stride[2];
  p.in_dtype = a.kv_in_dtype;
  p.kp = a.pool.k;
  p.vp = a.pool.v;
  p.pool_dtype = a.pool.dtype;
  p.slots = a.slot_mapping;
  p.ss = a.slot_stride;
  p.slots_i64 = a.slot_dtype == B200_INDEX_I64;
  p.status = a.status;
  // Vector loads need unit innermost stride, 16-byte aligned rows and a
  // 16-byte multiple for the head stride and token stride.
  const size_t es = dtype_size(a.kv_in_dtype);
  const int ne = a.pool.dtype == B200_DTYPE_F32 ? 4 : 8;
  auto aligned = [&](const void* ptr, const int64_t* st) {
    return st[2] == 1 && (reinterpret_cast<uintptr_t>(ptr) % 16) == 0 &&
           ((st[0] * es) % 16) == 0 && ((st[1] * es) % 16) == 0 && (ne * es) % 16 == 0;
  };
  p.vec_ok = (a.kv_in_dtype != B200_DTYPE_F16) && aligned(a.k, a.k_stride) && aligned(a.v, a.v_stride);
  if (p.N > 0x7fffffffLL) return fail(B200_ERR_UNSUPPORTED, "kv_scatter: too many tokens");
  // Flat path: same dtype, each token's H*D run contiguous in k, v and the
  // pool, 16-byte aligned rows (checked by vec_ok) and a run of whole chunks.
  const int64_t run_bytes = p.H * p.D * static_cast<int64_t>(es);
  if (p.vec_ok && a.kv_in_dtype == a.pool.dtype && a.k_stride[1] == p.D &&
      a.v_stride[1] == p.D && run_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(a.pool.k) % 16) == 0 &&
      (reinterpret_cast<uintptr_t>(a.pool.v) % 16) == 0) {
    FlatParams f{};
    f.P = p.P;
    f.S = p.S;
    f.layer_row0 = p.layer_row0;
    f.run = run_bytes / 16;
    f.k_tok = a.k_stride[0] * static_cast<int64_t>(es) / 16;
    f.v_tok = a.v_stride[0] * static_cast<int64_t>(es) / 16;
    f.k = static_cast<const uint4*>(a.k);
    f.v = static_cast<const uint4*>(a.v);
    f.kp = static_cast<uint4*>(a.pool.k);
    f.vp = static_cast<uint4*>(a.pool.v);
    f.slots = a.slot_mapping;
    f.ss = a.slot_stride;
    f.slots_i64 = p.slots_i64;
    f.status = a.status;
    const int threads = static_cast<int>(std::min<int64_t>(
        256, std::max<int64_t>(32, (f.run + kFlatIter - 1) / kFlatIter + 31) / 32 * 32));
    kv_scatter_flat_kernel<<<static_cast<unsigned>(p.N), threads, 0, stream>>>(f);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "kv_scatter launch");
    return B200_OK;
  }
  const int64_t chunks = p.H * ((p.D + ne - 1) / ne);
  const int threads = chunks >= 256 ? 256 : static_cast<int>((chunks + 31) / 32 * 32);
  const unsigned blocks = static_cast<unsigned>(p.N);
  if (a.pool.dtype == B200_DTYPE_F32)
    kv_scatter_kernel<float><<<blocks, threads, 0, stream>>>(p);
  else
    kv_scatter_kernel<__nv_bfloat16><<<blocks, threads, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kv_scatter launch");
  return B200_OK;
}

}  // namespace b200
