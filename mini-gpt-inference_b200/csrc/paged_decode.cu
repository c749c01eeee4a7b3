// paged_decode.cu -- fused KV-write + split-K paged decode attention for
// sm_100a (CUDA cores; decode is a bandwidth-bound GEMV).
//
// Work decomposition: one CTA per (sequence b, head group of G heads, split).
// A split is a run of `tiles_per_split` tiles of TILE logical KV rows.
//   * warp G (producer): walks the block table and issues one 3-D TMA load
//     per (KV block or block part, K/V) into a STAGES-deep shared-memory ring
//     guarded by full/empty mbarriers.  Boxes are {D_PAD, G heads, rbox rows}
//     of the [L*P*S rows, H, D] view of the pool, so one load moves G heads'
//     rows of one block with 128-bit coalesced transactions.
//   * warps 0..G-1 (consumers, one per head): each lane owns one 16-byte
//     chunk of a row; q.k partial dot products of a tile are combined with a
//     butterfly reduce-scatter over the chunk lanes (NI values -> NF values
//     in log2(CPR) shuffle steps), then an online-softmax update in the
//     log2 domain and the p.V accumulation from the same smem tile.
//   * split-K: a CTA whose sequence has more than one split writes
//     (m, l, acc) to the workspace; the last CTA of the (sequence, head
//     group) to finish (atomic counter, no waiting) combines them and resets
//     the counter to zero.
//   * fused decode write: the CTA that owns the last tile of sequence b
//     stores k_new/v_new at slot_mapping[b] before its pipeline starts
//     (generic stores + fence.proxy.async + CTA barrier before any TMA read).
//
// Semantics follow paged_attention_batch_online_v1
// (minivllm/paged_attention_batch.py:121-278): scale 1/sqrt(D) (:131), keys
// beyond the context masked to -inf before the max (:193-211), masked rows
// never multiplied into the output (:234-240, 0*NaN), and block-table -1
// padding beyond ceil(ctx/S) never read (triton_paged_decode.py:5-7).
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "host_util.h"
#include "kernels.h"

namespace b200 {

struct DecodeParams {
  int64_t P, S, H, D;
  int64_t layer;
  int64_t M;
  int32_t B;
  int32_t s_shift;  // log2(S)
  const void* q;
  int64_t qs0, qs1, qs2;
  int32_t q_dtype;
  void* out;
  int64_t os0, os1, os2;
  int32_t out_dtype;
  const void* tables;
  int64_t ts0, ts1;
  int32_t tables_i64;
  const void* lens;
  int64_t ls;
  int32_t lens_i64;
  int64_t ctx_base;
  // fused write
  int32_t fused;
  void* k_pool;
  void* v_pool;
  int32_t pool_dtype;
  const void* k_new;
  const void* v_new;
  int64_t kns0, kns1, kns2, vns0, vns1, vns2;
  int32_t new_dtype;
  const void* slots;
  int64_t ss;
  int32_t slots_i64;
  // geometry
  int32_t tiles_per_split;
  int32_t max_splits;
  int32_t num_hg;
  int32_t gbox;        // heads per TMA box (min(G, H))
  int32_t rbox;        // rows per TMA box (min(S, TILE))
  int32_t rb_shift;    // log2(rbox)
  int32_t box_stride;  // bytes between boxes in a stage (128-aligned)
  int32_t nbox;        // boxes per K (or V) tile
  int32_t box_bytes;   // bytes one box transfers
  int32_t stage_bytes;
  float* ws_acc;  // [B][H][max_splits][D_PAD]
  float* ws_ml;   // [B][H][max_splits][2]
  int32_t* ws_cnt;  // [B][num_hg]
  int32_t* status;
  float qscale;  // (1/sqrt(D)) * log2(e)
};

template <typename KV, int DPAD, int G, int STAGES>
struct DecodeCfg {
  static constexpr int ES = sizeof(KV);
  static constexpr int EPC = 16 / ES;         // elements per 16-byte chunk
  static constexpr int CPR = DPAD * ES / 16;  // chunks per row (1..32)
  static constexpr int RPL = 32 / CPR;        // rows per warp-wide load
  static constexpr int TILE = RPL > 16 ? RPL : 16;  // logical rows per stage
  static constexpr int NI = TILE / RPL;       // row loads per lane per tile
  static constexpr int DUP = CPR > NI ? CPR / NI : 1;  // lanes holding one score
  static constexpr int NF = NI > CPR ? NI / CPR : 1;   // scores held per lane
  static constexpr int THREADS = (G + 1) * 32;
  static_assert(CPR >= 1 && CPR <= 32, "row must span 1..32 chunks");
  static_assert(STAGES * 2 * 8 <= 128, "barriers live in the first 128 bytes");
};

// Butterfly reduce-scatter of NI per-lane partial sums over the lane bits
// [0, log2(CPR)).  Upper-half lanes keep the upper half of the values at
// each halving step, so afterwards lane chunk c holds the complete sums of
// value indices (c / DUP) * NF + f, f < NF.
template <int N, int BIT>
struct RowReduce {
  __device__ __forceinline__ static void run(float* s, int lane) {
    if constexpr (BIT == 0) {
      return;
    } else if constexpr (N > 1) {
      const bool upper = (lane & BIT) != 0;
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
        const float send = upper ? s[i] : s[i + N / 2];
        const float keep = upper ? s[i + N / 2] : s[i];
        s[i] = keep + __shfl_xor_sync(0xffffffffu, send, BIT);
      }
      RowReduce<N / 2, BIT / 2>::run(s, lane);
    } else {
      s[0] += __shfl_xor_sync(0xffffffffu, s[0], BIT);
      RowReduce<1, BIT / 2>::run(s, lane);
    }
  }
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename KV, int DPAD, int G, int STAGES>
__global__ void __launch_bounds__((G + 1) * 32)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv, const DecodeParams p) {
  using C = DecodeCfg<KV, DPAD, G, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // The launch reserves 128 spare bytes so the ring can start 128-aligned
  // (TMA destinations) whatever alignment the dynamic window has.
  uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int idx = blockIdx.x;
  const int split = idx % p.max_splits;
  idx /= p.max_splits;
  const int hg = idx % p.num_hg;
  const int b = idx / p.num_hg;
  const int h0 = hg * G;

  const int64_t ctx = p.lens != nullptr ? load_index(p.lens, b * p.ls, p.lens_i64)
                                        : p.ctx_base + b + 1;
  if (ctx < 1 || ctx > p.M * p.S) {
    // Invalid length: write zeros once (split 0) and report; never read KV.
    if (split == 0) {
      if (threadIdx.x == 0) report(p.status, B200_DEV_BAD_LENGTH);
      if (warp < G && h0 + warp < p.H)
        for (int d = lane; d < p.D; d += 32)
          store_elem(p.out, b * p.os0 + (h0 + warp) * p.os1 + d * p.os2, p.out_dtype, 0.f);
    }
    return;
  }
  const int n_tiles = static_cast<int>((ctx + C::TILE - 1) / C::TILE);
  const int nsplit = (n_tiles + p.tiles_per_split - 1) / p.tiles_per_split;
  if (split >= nsplit) return;
  const int t0 = split * p.tiles_per_split;
  const int t1 = min(n_tiles, t0 + p.tiles_per_split);

  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + STAGES;
  int32_t& s_is_last = *reinterpret_cast<int32_t*>(smem + 120);
  uint8_t* tiles = smem + 128;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], G);
    }
    fence_mbar_init();
  }
  if (warp == G && lane == 0) {
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmv);
  }

  // Fused decode KV write (before any TMA read of the pool by this CTA).
  if (p.fused && t1 == n_tiles && warp < G && h0 + warp < p.H) {
    const int h = h0 + warp;
    const int64_t slot = load_index(p.slots, b * p.ss, p.slots_i64);
    if (slot < 0 || slot >= p.P * p.S) {
      if (lane == 0) report(p.status, B200_DEV_BAD_SLOT);
    } else {
      const int64_t pos = ctx - 1;
      const int64_t phys = load_index(p.tables, b * p.ts0 + (pos >> p.s_shift) * p.ts1,
                                      p.tables_i64);
      if (lane == 0 && phys * p.S + (pos & (p.S - 1)) != slot)
        report(p.status, B200_DEV_SLOT_MISMATCH);
      const int64_t base = ((p.layer * p.P * p.S + slot) * p.H + h) * p.D;
      for (int d = lane; d < p.D; d += 32) {
        const float kv = load_elem(p.k_new, b * p.kns0 + h * p.kns1 + d * p.kns2, p.new_dtype);
        const float vv = load_elem(p.v_new, b * p.vns0 + h * p.vns1 + d * p.vns2, p.new_dtype);
        store_elem(p.k_pool, base + d, p.pool_dtype, kv);
        store_elem(p.v_pool, base + d, p.pool_dtype, vv);
      }
      fence_proxy_async_global();
    }
  }
  __syncthreads();

  const int row_bytes = p.gbox * DPAD * C::ES;

  if (warp == G) {
    // ------------------------------------------------------------ producer
    int64_t j_base = -(int64_t(1) << 40);
    int64_t my_entry = 0;
    const int64_t row_layer = p.layer * p.P;
    int issued = 0;
    for (int t = t0; t < t1; ++t) {
      const int it = t - t0;
      const int stage = it % STAGES;
      const uint32_t ph = static_cast<uint32_t>(it / STAGES) & 1u;
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&empty[stage], ph ^ 1u) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) report(p.status, B200_DEV_WAIT_TIMEOUT);
        break;
      }
      const int64_t row0 = static_cast<int64_t>(t) * C::TILE;
      const int64_t rows_left = ctx - row0;
      const int nvb = static_cast<int>(min(static_cast<int64_t>(p.nbox), (rows_left + p.rbox - 1) >> p.rb_shift));
      if (lane == 0) mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(2 * nvb * p.box_bytes));
      uint8_t* kdst = tiles + static_cast<size_t>(stage) * p.stage_bytes;
      uint8_t* vdst = kdst + static_cast<size_t>(p.nbox) * p.box_stride;
      for (int k = 0; k < nvb; ++k) {
        const int64_t r = row0 + (static_cast<int64_t>(k) << p.rb_shift);
        const int64_t j = r >> p.s_shift;
        if (j < j_base || j >= j_base + 32) {
          j_base = j;
          my_entry = (j + lane < p.M)
                         ? load_index(p.tables, b * p.ts0 + (j + lane) * p.ts1, p.tables_i64)
                         : -1;
        }
        int64_t phys = __shfl_sync(0xffffffffu, my_entry, static_cast<int>(j - j_base));
        if (phys < 0 || phys >= p.P) {
          if (lane == 0) report(p.status, B200_DEV_BAD_BLOCK);
          phys = 0;  // load an in-bounds block; the status word flags the result
        }
        if (lane == 0) {
          const int32_t row = static_cast<int32_t>((row_layer + phys) * p.S + (r & (p.S - 1)));
          tma_load_3d(kdst + k * p.box_stride, &tmk, &full[stage], 0, h0, row);
          tma_load_3d(vdst + k * p.box_stride, &tmv, &full[stage], 0, h0, row);
        }
      }
      ++issued;
    }
    // Drain: make sure no TMA write into this CTA's smem is still in flight.
    if (lane == 0) {
      const int first = issued > STAGES ? issued - STAGES : 0;
      for (int it = first; it < issued; ++it)
        if (!mbar_wait(&full[it % STAGES], static_cast<uint32_t>(it / STAGES) & 1u)) {
          report(p.status, B200_DEV_WAIT_TIMEOUT);
          break;
        }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int h = h0 + warp;
    const bool active = (h < p.H) && (warp < p.gbox);
    const int c = lane % C::CPR;
    const int rg = lane / C::CPR;
    float qv[C::EPC];
#pragma unroll
    for (int e = 0; e < C::EPC; ++e) {
      const int d = c * C::EPC + e;
      qv[e] = (active && d < p.D)
                  ? load_elem(p.q, b * p.qs0 + h * p.qs1 + d * p.qs2, p.q_dtype) * p.qscale
                  : 0.f;
    }
    float m = -INFINITY, l = 0.f;
    float acc[C::EPC];
#pragma unroll
    for (int e = 0; e < C::EPC; ++e) acc[e] = 0.f;
    const int head_off = warp * DPAD * C::ES + c * 16;

    for (int t = t0; t < t1; ++t) {
      const int it = t - t0;
      const int stage = it % STAGES;
      const uint32_t ph = static_cast<uint32_t>(it / STAGES) & 1u;
      if (!mbar_wait(&full[stage], ph)) {
        if (lane == 0) report(p.status, B200_DEV_WAIT_TIMEOUT);
        break;
      }
      if (active) {
        const uint8_t* kt = tiles + static_cast<size_t>(stage) * p.stage_bytes;
        const uint8_t* vt = kt + static_cast<size_t>(p.nbox) * p.box_stride;
        const int nvalid = static_cast<int>(min(static_cast<int64_t>(C::TILE), ctx - static_cast<int64_t>(t) * C::TILE));
        float s[C::NI];
#pragma unroll
        for (int i = 0; i < C::NI; ++i) {
          const int r = i * C::RPL + rg;
          float acc_d = 0.f;
          if (r < nvalid) {
            const int off = (r >> p.rb_shift) * p.box_stride + (r & (p.rbox - 1)) * row_bytes + head_off;
            const uint4 raw = *reinterpret_cast<const uint4*>(kt + off);
            float kf[C::EPC];
            Elem<KV>::unpack(raw, kf);
#pragma unroll
            for (int e = 0; e < C::EPC; ++e) acc_d = fmaf(qv[e], kf[e], acc_d);
          }
          s[i] = acc_d;
        }
        RowReduce<C::NI, C::CPR / 2>::run(s, lane);
        float mx = -INFINITY;
#pragma unroll
        for (int f = 0; f < C::NF; ++f) {
          const int r = ((c / C::DUP) * C::NF + f) * C::RPL + rg;
          if (r >= nvalid) s[f] = -INFINITY;
          mx = fmaxf(mx, s[f]);
        }
        mx = warp_max(mx);
        const float m_new = fmaxf(m, mx);
        const float alpha = fast_exp2(m - m_new);
        float psum = 0.f;
#pragma unroll
        for (int f = 0; f < C::NF; ++f) {
          s[f] = fast_exp2(s[f] - m_new);
          psum += s[f];
        }
        psum = warp_sum(psum) * (1.0f / C::DUP);
        l = l * alpha + psum;
        m = m_new;
#pragma unroll
        for (int e = 0; e < C::EPC; ++e) acc[e] *= alpha;
#pragma unroll
        for (int i = 0; i < C::NI; ++i) {
          const int r = i * C::RPL + rg;
          const float pr = __shfl_sync(0xffffffffu, s[i % C::NF], rg * C::CPR + (i / C::NF) * C::DUP);
          if (r < nvalid) {
            const int off = (r >> p.rb_shift) * p.box_stride + (r & (p.rbox - 1)) * row_bytes + head_off;
            const uint4 raw = *reinterpret_cast<const uint4*>(vt + off);
            float vf[C::EPC];
            Elem<KV>::unpack(raw, vf);
#pragma unroll
            for (int e = 0; e < C::EPC; ++e) acc[e] = fmaf(pr, vf[e], acc[e]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
    }

    // Combine the row groups (lanes with equal chunk index).
#pragma unroll
    for (int bit = C::CPR; bit < 32; bit <<= 1)
#pragma unroll
      for (int e = 0; e < C::EPC; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], bit);

    if (active) {
      if (nsplit == 1) {
        if (rg == 0) {
          const float inv = 1.0f / l;
#pragma unroll
          for (int e = 0; e < C::EPC; ++e) {
            const int d = c * C::EPC + e;
            if (d < p.D) store_elem(p.out, b * p.os0 + h * p.os1 + d * p.os2, p.out_dtype, acc[e] * inv);
          }
        }
      } else {
        const int64_t slot = (static_cast<int64_t>(b) * p.H + h) * p.max_splits + split;
        if (rg == 0) {
#pragma unroll
          for (int e = 0; e < C::EPC; ++e) p.ws_acc[slot * DPAD + c * C::EPC + e] = acc[e];
        }
        if (lane == 0) {
          p.ws_ml[slot * 2] = m;
          p.ws_ml[slot * 2 + 1] = l;
        }
        __threadfence();
      }
    }
  }

  if (nsplit == 1) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(&p.ws_cnt[b * p.num_hg + hg], 1);
    s_is_last = (old == nsplit - 1) ? 1 : 0;
  }
  __syncthreads();
  if (!s_is_last) return;
  __threadfence();
  if (warp < G) {
    const int h = h0 + warp;
    if (h < p.H) {
      const int64_t base = (static_cast<int64_t>(b) * p.H + h) * p.max_splits;
      float mg = -INFINITY;
      for (int i = 0; i < nsplit; ++i) mg = fmaxf(mg, __ldcg(&p.ws_ml[(base + i) * 2]));
      float lg = 0.f;
      for (int i = 0; i < nsplit; ++i) {
        const float w = fast_exp2(__ldcg(&p.ws_ml[(base + i) * 2]) - mg);
        lg += w * __ldcg(&p.ws_ml[(base + i) * 2 + 1]);
      }
      const float inv = 1.0f / lg;
      for (int d = lane; d < p.D; d += 32) {
        float o = 0.f;
        for (int i = 0; i < nsplit; ++i) {
          const float w = fast_exp2(__ldcg(&p.ws_ml[(base + i) * 2]) - mg);
          o = fmaf(w, __ldcg(&p.ws_acc[(base + i) * DPAD + d]), o);
        }
        store_elem(p.out, b * p.os0 + h * p.os1 + d * p.os2, p.out_dtype, o * inv);
      }
    }
  }
  if (threadIdx.x == 0) p.ws_cnt[b * p.num_hg + hg] = 0;
}

// ------------------------------------------------------------------ host
namespace {

struct Plan {
  int g, stages, dpad, tile;
  int64_t num_hg, max_tiles, tiles_per_split, max_splits;
};

int pick_dpad(int64_t D, size_t es) {
  int64_t d = static_cast<int64_t>(16 / es);
  while (d < D) d <<= 1;
  return static_cast<int>(d);
}

// Heads per CTA and pipeline depth for a KV element size.
void pick_shape(size_t es, int* g, int* stages) {
  *g = es == 2 ? 4 : 2;
  *stages = 4;
}

int tile_rows(int dpad, size_t es) {
  const int cpr = static_cast<int>(dpad * es / 16);
  const int rpl = 32 / cpr;
  return rpl > 16 ? rpl : 16;
}

}  // namespace

size_t decode_workspace_bytes(int64_t B, int64_t H, int64_t D, int64_t M, int64_t S,
                              int32_t hint, size_t es, int num_sms) {
  const int dpad = pick_dpad(D, es);
  int g, stages;
  pick_shape(es, &g, &stages);
  const int tile = tile_rows(dpad, es);
  const int64_t max_tiles = ceil_div(M * S, tile);
  const int64_t num_hg = ceil_div(H, g);
  int64_t tps = decode_tiles_per_split(B * num_hg, max_tiles, hint, num_sms);
  const int64_t max_splits = ceil_div(max_tiles, tps);
  if (max_splits <= 1) return 0;
  size_t bytes = static_cast<size_t>(B * H * max_splits) * (dpad + 2) * sizeof(float);
  bytes = (bytes + 255) & ~size_t(255);
  bytes += static_cast<size_t>(B * num_hg) * sizeof(int32_t);
  return (bytes + 255) & ~size_t(255);
}

int64_t decode_tiles_per_split(int64_t units, int64_t max_tiles, int32_t hint, int num_sms) {
  if (hint > 0) return ceil_div(max_tiles, std::min<int64_t>(hint, max_tiles));
  // Aim for about 4 CTAs per SM over the whole grid; never split below 8 tiles.
  const int64_t target_ctas = 4 * static_cast<int64_t>(num_sms);
  int64_t splits = ceil_div(target_ctas, std::max<int64_t>(units, 1));
  splits = std::max<int64_t>(1, std::min<int64_t>(splits, ceil_div(max_tiles, 8)));
  return ceil_div(max_tiles, splits);
}

template <typename KV, int DPAD, int G, int STAGES>
static int launch_cfg(const DecodeParams& prm, const CUtensorMap& tk, const CUtensorMap& tv,
                      int64_t grid, size_t smem, cudaStream_t stream) {
  auto kern = paged_decode_kernel<KV, DPAD, G, STAGES>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && configured[dev] < static_cast<int>(smem)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(paged_decode)");
    configured[dev] = static_cast<int>(smem);
  }
  kern<<<static_cast<unsigned>(grid), DecodeCfg<KV, DPAD, G, STAGES>::THREADS, smem, stream>>>(
      tk, tv, prm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "paged_decode launch");
  return B200_OK;
}

template <typename KV, int G, int STAGES>
static int launch_dpad(int dpad, const DecodeParams& prm, const CUtensorMap& tk,
                       const CUtensorMap& tv, int64_t grid, size_t smem, cudaStream_t stream) {
  switch (dpad) {
    case 4:
      if constexpr (sizeof(KV) == 4) return launch_cfg<KV, 4, G, STAGES>(prm, tk, tv, grid, smem, stream);
      break;
    case 8: return launch_cfg<KV, 8, G, STAGES>(prm, tk, tv, grid, smem, stream);
    case 16: return launch_cfg<KV, 16, G, STAGES>(prm, tk, tv, grid, smem, stream);
    case 32: return launch_cfg<KV, 32, G, STAGES>(prm, tk, tv, grid, smem, stream);
    case 64: return launch_cfg<KV, 64, G, STAGES>(prm, tk, tv, grid, smem, stream);
    case 128: return launch_cfg<KV, 128, G, STAGES>(prm, tk, tv, grid, smem, stream);
    default: break;
  }
  return fail(B200_ERR_UNSUPPORTED, "paged decode: head_dim padding not instantiated");
}

int launch_paged_decode(const DecodeLaunch& a, cudaStream_t stream) {
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc != B200_OK) return rc;
  const size_t es = dtype_size(a.pool.dtype);
  const int dpad = pick_dpad(a.pool.head_dim, es);
  int g, stages;
  pick_shape(es, &g, &stages);
  const int tile = tile_rows(dpad, es);
  const int64_t S = a.pool.block_size, H = a.pool.num_heads, D = a.pool.head_dim;
  const int64_t P = a.pool.num_blocks, L = a.pool.num_layers;
  const int64_t max_tiles = ceil_div(a.table_width * S, tile);
  const int64_t num_hg = ceil_div(H, g);
  const int64_t tps = decode_tiles_per_split(a.batch * num_hg, max_tiles, a.max_splits_hint, dev.num_sms);
  const int64_t max_splits = ceil_div(max_tiles, tps);

  DecodeParams prm{};
  prm.P = P;
  prm.S = S;
  prm.H = H;
  prm.D = D;
  prm.layer = a.layer_idx;
  prm.M = a.table_width;
  prm.B = static_cast<int32_t>(a.batch);
  prm.s_shift = log2i(S);
  prm.q = a.q;
  prm.qs0 = a.q_stride[0];
  prm.qs1 = a.q_stride[1];
  prm.qs2 = a.q_stride[2];
  prm.q_dtype = a.q_dtype;
  prm.out = a.out;
  prm.os0 = a.out_stride[0];
  prm.os1 = a.out_stride[1];
  prm.os2 = a.out_stride[2];
  prm.out_dtype = a.out_dtype;
  prm.tables = a.block_tables;
  prm.ts0 = a.block_table_stride[0];
  prm.ts1 = a.block_table_stride[1];
  prm.tables_i64 = a.block_table_dtype == B200_INDEX_I64;
  prm.lens = a.context_lengths;
  prm.ls = a.context_length_stride;
  prm.lens_i64 = a.context_length_dtype == B200_INDEX_I64;
  prm.ctx_base = a.ctx_base;
  prm.fused = a.k_new != nullptr;
  prm.k_pool = a.pool.k;
  prm.v_pool = a.pool.v;
  prm.pool_dtype = a.pool.dtype;
  prm.k_new = a.k_new;
  prm.v_new = a.v_new;
  prm.kns0 = a.k_new_stride[0];
  prm.kns1 = a.k_new_stride[1];
  prm.kns2 = a.k_new_stride[2];
  prm.vns0 = a.v_new_stride[0];
  prm.vns1 = a.v_new_stride[1];
  prm.vns2 = a.v_new_stride[2];
  prm.new_dtype = a.kv_new_dtype;
  prm.slots = a.slot_mapping;
  prm.ss = a.slot_stride;
  prm.slots_i64 = a.slot_dtype == B200_INDEX_I64;
  prm.tiles_per_split = static_cast<int32_t>(tps);
  prm.max_splits = static_cast<int32_t>(max_splits);
  prm.num_hg = static_cast<int32_t>(num_hg);
  prm.gbox = static_cast<int32_t>(std::min<int64_t>(g, H));
  prm.rbox = static_cast<int32_t>(std::min<int64_t>(S, tile));
  prm.rb_shift = log2i(prm.rbox);
  prm.box_bytes = static_cast<int32_t>(prm.rbox * prm.gbox * dpad * es);
  prm.box_stride = (prm.box_bytes + 127) & ~127;
  prm.nbox = tile / prm.rbox;
  prm.stage_bytes = 2 * prm.nbox * prm.box_stride;
  prm.status = a.status;
  prm.qscale = static_cast<float>(1.0 / sqrt(static_cast<double>(D)) * 1.4426950408889634);

  if (max_splits > 1) {
    const size_t need = decode_workspace_bytes(a.batch, H, D, a.table_width, S,
                                               a.max_splits_hint, es, dev.num_sms);
    if (a.workspace == nullptr || a.workspace_bytes < need) {
      char buf[160];
      snprintf(buf, sizeof(buf), "paged decode needs %zu workspace bytes, got %zu", need,
               a.workspace_bytes);
      return fail(B200_ERR_WORKSPACE, buf);
    }
    uint8_t* ws = static_cast<uint8_t*>(a.workspace);
    const size_t acc_bytes = static_cast<size_t>(a.batch * H * max_splits) * dpad * sizeof(float);
    const size_t ml_bytes = static_cast<size_t>(a.batch * H * max_splits) * 2 * sizeof(float);
    prm.ws_acc = reinterpret_cast<float*>(ws);
    prm.ws_ml = reinterpret_cast<float*>(ws + acc_bytes);
    size_t cnt_off = (acc_bytes + ml_bytes + 255) & ~size_t(255);
    prm.ws_cnt = reinterpret_cast<int32_t*>(ws + cnt_off);
    // The counters' location depends on (B, H, splits), so a workspace
    // reused across calls of other shapes may hold stale data there; clear
    // them on the stream before the launch (an async memset, no allocation).
    cudaError_t me = cudaMemsetAsync(prm.ws_cnt, 0, static_cast<size_t>(a.batch * num_hg) * sizeof(int32_t), stream);
    if (me != cudaSuccess) return cuda_fail(me, "cudaMemsetAsync(split-K counters)");
  }

  // Tensor maps over the [L*P*S rows, H, D] views of the pools.
  CUtensorMap tk, tv;
  const CUtensorMapDataType ttype =
      es == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(H),
                            static_cast<uint64_t>(L * P * S)};
  const uint64_t strides[2] = {static_cast<uint64_t>(D * es), static_cast<uint64_t>(H * D * es)};
  const uint32_t box[3] = {static_cast<uint32_t>(dpad), static_cast<uint32_t>(prm.gbox),
                           static_cast<uint32_t>(prm.rbox)};
  rc = encode_tensor_map(&tk, ttype, 3, a.pool.k, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc != B200_OK) return rc;
  rc = encode_tensor_map(&tv, ttype, 3, a.pool.v, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc != B200_OK) return rc;

  const size_t smem = 256 + static_cast<size_t>(stages) * prm.stage_bytes;
  if (smem > static_cast<size_t>(dev.max_smem_optin))
    return fail(B200_ERR_UNSUPPORTED, "paged decode: stage ring exceeds shared memory");
  const int64_t grid = a.batch * num_hg * max_splits;
  if (grid > 0x7fffffffLL) return fail(B200_ERR_UNSUPPORTED, "paged decode: grid too large");

  if (es == 4) return launch_dpad<float, 2, 4>(dpad, prm, tk, tv, grid, smem, stream);
  return launch_dpad<__nv_bfloat16, 4, 4>(dpad, prm, tk, tv, grid, smem, stream);
}

}  // namespace b200
