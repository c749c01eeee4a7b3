// paged_decode.cu -- fused KV-write + split-K paged decode attention for
// sm_100a (CUDA cores; decode is a bandwidth-bound GEMV).
//
// Work decomposition: one CTA per (sequence b, head group of G heads, split).
// A split is a run of `tiles_per_split` tiles of TILE logical KV rows.
//   * last warp (producer): walks the block table (32 entries per coalesced
//     warp load) and issues one 3-D TMA load per (KV block or block part,
//     K/V) into a STAGES-deep shared-memory ring guarded by full/empty
//     mbarriers.  Boxes are {D_PAD, G heads, rbox rows} of the
//     [L*P*S rows, H, D] view of the pool, so one load moves G heads' rows of
//     one block with 128-bit coalesced transactions.
//   * G*WPH consumer warps, WPH per head: warp (g, sub) owns head g and the
//     rows [sub*TILE/WPH, (sub+1)*TILE/WPH) of every tile.  Each lane owns one
//     16-byte chunk of a row; q.k partial dot products (packed fp32x2 FMAs on
//     exactly unpacked bf16 pairs) are combined with a butterfly
//     reduce-scatter over the chunk lanes, then an online-softmax update in
//     the log2 domain and the p.V accumulation from the same smem tile.  The
//     WPH partial states of a head are merged through shared memory at the
//     end of the split.
//   * split-K: a CTA whose sequence has more than one split writes
//     (m, l, acc) to the workspace; the last CTA of the (sequence, head
//     group) to finish (atomic counter, no waiting) combines them.  The launch
//     clears the counters on the stream first.
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
#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <type_traits>

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

template <typename KV, int DPAD, int G, int WPH, int STAGES>
struct DecodeCfg {
  static constexpr int ES = sizeof(KV);
  static constexpr int EPC = 16 / ES;         // elements per 16-byte chunk
  static constexpr int CPR = DPAD * ES / 16;  // chunks per row (1..32)
  static constexpr int RPL = 32 / CPR;        // rows per warp-wide load
  static constexpr int TILE = RPL > 16 ? RPL : 16;  // logical rows per stage
  static constexpr int NI = TILE / RPL;       // row loads per tile per head
  static constexpr int NIW = NI / WPH;        // row loads per tile per warp
  static constexpr int DUP = CPR > NIW ? CPR / NIW : 1;  // lanes holding one score
  static constexpr int NF = NIW > CPR ? NIW / CPR : 1;   // scores held per lane
  static constexpr int CONSUMERS = G * WPH;
  static constexpr int THREADS = (CONSUMERS + 1) * 32;
  static_assert(CPR >= 1 && CPR <= 32, "row must span 1..32 chunks");
  static_assert(NI % WPH == 0 && NIW >= 1, "tile rows must split evenly across a head's warps");
  static_assert(STAGES * 2 * 8 <= 112, "barriers live in the first 128 bytes");
  static_assert(EPC % 2 == 0, "chunks hold element pairs");
};

// Butterfly reduce-scatter of N per-lane partial sums over the lane bits
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

// q.chunk for one 16-byte chunk of a K row (exact unpack, packed FMAs).
template <typename KV>
__device__ __forceinline__ float chunk_dot(const float2* q2, const uint4& raw) {
  float2 acc = make_float2(0.f, 0.f);
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  if constexpr (sizeof(KV) == 2) {
#pragma unroll
    for (int i = 0; i < 4; ++i) acc = ffma2(q2[i], bf16x2_to_float2(w[i]), acc);
  } else {
#pragma unroll
    for (int i = 0; i < 2; ++i)
      acc = ffma2(q2[i], make_float2(__uint_as_float(w[2 * i]), __uint_as_float(w[2 * i + 1])), acc);
  }
  return acc.x + acc.y;
}

// acc += p * chunk of a V row.
template <typename KV>
__device__ __forceinline__ void chunk_axpy(float2* acc2, float pr, const uint4& raw) {
  const float2 p2 = make_float2(pr, pr);
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  if constexpr (sizeof(KV) == 2) {
#pragma unroll
    for (int i = 0; i < 4; ++i) acc2[i] = ffma2(p2, bf16x2_to_float2(w[i]), acc2[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 2; ++i)
      acc2[i] = ffma2(p2, make_float2(__uint_as_float(w[2 * i]), __uint_as_float(w[2 * i + 1])),
                      acc2[i]);
  }
}

template <typename KV, int DPAD, int G, int WPH, int STAGES>
__global__ void __launch_bounds__(DecodeCfg<KV, DPAD, G, WPH, STAGES>::THREADS)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv, const DecodeParams p) {
  using C = DecodeCfg<KV, DPAD, G, WPH, STAGES>;
  constexpr int NP = C::EPC / 2;  // float2 pairs per chunk
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // The launch reserves spare bytes so the ring can start 128-aligned
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
  float* mrg = reinterpret_cast<float*>(tiles + static_cast<size_t>(STAGES) * p.stage_bytes);

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], C::CONSUMERS);
    }
    fence_mbar_init();
  }
  if (warp == C::CONSUMERS && lane == 0) {
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmv);
  }

  const int g = warp / WPH;    // head of this consumer warp within the group
  const int sub = warp % WPH;  // row slice of this consumer warp

  // Fused decode KV write (before any TMA read of the pool by this CTA).
  if (p.fused && t1 == n_tiles && warp < C::CONSUMERS && sub == 0 && h0 + g < p.H) {
    const int h = h0 + g;
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
  float m = -INFINITY, l = 0.f;
  float2 acc2[NP];
#pragma unroll
  for (int e = 0; e < NP; ++e) acc2[e] = make_float2(0.f, 0.f);
  const int c = lane % C::CPR;
  const int rg = lane / C::CPR;
  const int h = h0 + g;
  const bool active = warp < C::CONSUMERS && (h < p.H) && (g < p.gbox);

  if (warp == C::CONSUMERS) {
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
      const int nvb = static_cast<int>(
          min(static_cast<int64_t>(p.nbox), (rows_left + p.rbox - 1) >> p.rb_shift));
      if (lane == 0)
        mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(2 * nvb * p.box_bytes));
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
    float2 q2[NP];
#pragma unroll
    for (int e = 0; e < NP; ++e) {
      float f[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int d = c * C::EPC + 2 * e + u;
        f[u] = (active && d < p.D)
                   ? load_elem(p.q, b * p.qs0 + h * p.qs1 + d * p.qs2, p.q_dtype) * p.qscale
                   : 0.f;
      }
      q2[e] = make_float2(f[0], f[1]);
    }
    // Byte offsets (within a K or V tile) of this lane's rows: loop-invariant.
    int roff[C::NIW];
#pragma unroll
    for (int k = 0; k < C::NIW; ++k) {
      const int r = (sub * C::NIW + k) * C::RPL + rg;
      roff[k] = (r >> p.rb_shift) * p.box_stride + (r & (p.rbox - 1)) * row_bytes +
                g * DPAD * C::ES + c * 16;
    }

    // One tile; FULL = every row of the tile is inside the context.
    auto tile = [&](const uint8_t* kt, const uint8_t* vt, int nvalid, auto full_tag) {
      constexpr bool FULL = decltype(full_tag)::value;
      float s[C::NIW];
#pragma unroll
      for (int k = 0; k < C::NIW; ++k) {
        const int r = (sub * C::NIW + k) * C::RPL + rg;
        s[k] = 0.f;
        if (FULL || r < nvalid)
          s[k] = chunk_dot<KV>(q2, *reinterpret_cast<const uint4*>(kt + roff[k]));
      }
      RowReduce<C::NIW, C::CPR / 2>::run(s, lane);
      float mx = -INFINITY;
#pragma unroll
      for (int f = 0; f < C::NF; ++f) {
        const int r = (sub * C::NIW + (c / C::DUP) * C::NF + f) * C::RPL + rg;
        if (!FULL && r >= nvalid) s[f] = -INFINITY;
        mx = fmaxf(mx, s[f]);
      }
      mx = warp_max(mx);
      if (mx == -INFINITY) return;  // no row of this warp's slice is in the context
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
      const float2 a2 = make_float2(alpha, alpha);
      const float2 z2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int e = 0; e < NP; ++e) acc2[e] = ffma2(acc2[e], a2, z2);
#pragma unroll
      for (int k = 0; k < C::NIW; ++k) {
        const int r = (sub * C::NIW + k) * C::RPL + rg;
        const float pr = __shfl_sync(0xffffffffu, s[k % C::NF],
                                     rg * C::CPR + (k / C::NF) * C::DUP);
        if (FULL || r < nvalid)
          chunk_axpy<KV>(acc2, pr, *reinterpret_cast<const uint4*>(vt + roff[k]));
      }
    };

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
        const int nvalid = static_cast<int>(
            min(static_cast<int64_t>(C::TILE), ctx - static_cast<int64_t>(t) * C::TILE));
        if (nvalid == C::TILE)
          tile(kt, vt, nvalid, std::true_type{});
        else
          tile(kt, vt, nvalid, std::false_type{});
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
    }

    // Combine the row groups (lanes with equal chunk index).
#pragma unroll
    for (int bit = C::CPR; bit < 32; bit <<= 1)
#pragma unroll
      for (int e = 0; e < NP; ++e) {
        acc2[e].x += __shfl_xor_sync(0xffffffffu, acc2[e].x, bit);
        acc2[e].y += __shfl_xor_sync(0xffffffffu, acc2[e].y, bit);
      }
  }

  // Merge the WPH row slices of each head through shared memory.
  if constexpr (WPH > 1) {
    if (active) {
      float* pa = mrg + warp * (DPAD + 2);
      if (rg == 0) {
#pragma unroll
        for (int e = 0; e < NP; ++e) {
          pa[c * C::EPC + 2 * e] = acc2[e].x;
          pa[c * C::EPC + 2 * e + 1] = acc2[e].y;
        }
      }
      if (lane == 0) {
        pa[DPAD] = m;
        pa[DPAD + 1] = l;
      }
    }
    __syncthreads();
    if (active && sub == 0) {
      float mg = -INFINITY;
#pragma unroll
      for (int w = 0; w < WPH; ++w) mg = fmaxf(mg, mrg[(warp + w) * (DPAD + 2) + DPAD]);
      float lg = 0.f;
      float2 ag[NP];
#pragma unroll
      for (int e = 0; e < NP; ++e) ag[e] = make_float2(0.f, 0.f);
#pragma unroll
      for (int w = 0; w < WPH; ++w) {
        const float* pa = mrg + (warp + w) * (DPAD + 2);
        const float wt = fast_exp2(pa[DPAD] - mg);  // 0 for a slice that saw no row
        lg += wt * pa[DPAD + 1];
        const float2 w2 = make_float2(wt, wt);
#pragma unroll
        for (int e = 0; e < NP; ++e)
          ag[e] = ffma2(w2, make_float2(pa[c * C::EPC + 2 * e], pa[c * C::EPC + 2 * e + 1]), ag[e]);
      }
      m = mg;
      l = lg;
#pragma unroll
      for (int e = 0; e < NP; ++e) acc2[e] = ag[e];
    }
  }

  if (active && sub == 0) {
    if (nsplit == 1) {
      if (rg == 0) {
        const float inv = 1.0f / l;
#pragma unroll
        for (int e = 0; e < NP; ++e) {
          const int d = c * C::EPC + 2 * e;
          if (d < p.D)
            store_elem(p.out, b * p.os0 + h * p.os1 + d * p.os2, p.out_dtype, acc2[e].x * inv);
          if (d + 1 < p.D)
            store_elem(p.out, b * p.os0 + h * p.os1 + (d + 1) * p.os2, p.out_dtype,
                       acc2[e].y * inv);
        }
      }
    } else {
      const int64_t slot = (static_cast<int64_t>(b) * p.H + h) * p.max_splits + split;
      if (rg == 0) {
#pragma unroll
        for (int e = 0; e < NP; ++e) {
          p.ws_acc[slot * DPAD + c * C::EPC + 2 * e] = acc2[e].x;
          p.ws_acc[slot * DPAD + c * C::EPC + 2 * e + 1] = acc2[e].y;
        }
      }
      if (lane == 0) {
        p.ws_ml[slot * 2] = m;
        p.ws_ml[slot * 2 + 1] = l;
      }
      __threadfence();
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
    const int hh = h0 + warp;
    if (hh < p.H) {
      const int64_t base = (static_cast<int64_t>(b) * p.H + hh) * p.max_splits;
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
        store_elem(p.out, b * p.os0 + hh * p.os1 + d * p.os2, p.out_dtype, o * inv);
      }
    }
  }
  if (threadIdx.x == 0) p.ws_cnt[b * p.num_hg + hg] = 0;
}

// ------------------------------------------------------------------ host
namespace {

// CTA shape of one instantiation: heads per CTA, warps per head, ring depth
// and the number of CTAs it is sized to keep resident per SM.
struct Shape {
  int g, wph, stages, ctas_per_sm;
};

int pick_dpad(int64_t D, size_t es) {
  int64_t d = static_cast<int64_t>(16 / es);
  while (d < D) d <<= 1;
  return static_cast<int>(d);
}

int tile_rows(int dpad, size_t es) {
  const int cpr = static_cast<int>(dpad * es / 16);
  const int rpl = 32 / cpr;
  return rpl > 16 ? rpl : 16;
}

// Shapes instantiated for head_dim 128 (the production shape); the first
// entry is the default.  Other head dims use the fixed small shapes.
constexpr Shape kShapesBf16[] = {{4, 2, 3, 2}, {4, 1, 4, 1}, {2, 2, 4, 3}, {4, 4, 3, 2},
                                 {8, 1, 3, 1}, {2, 4, 4, 3}};
constexpr Shape kShapesF32[] = {{2, 2, 3, 2}, {2, 1, 4, 1}, {4, 2, 3, 1}, {2, 4, 3, 2}};
constexpr int kNumShapesBf16 = sizeof(kShapesBf16) / sizeof(Shape);
constexpr int kNumShapesF32 = sizeof(kShapesF32) / sizeof(Shape);
constexpr Shape kSmallBf16 = {4, 1, 4, 2};
constexpr Shape kSmallF32 = {2, 1, 4, 2};

// Tuning override of the head_dim-128 shape:
// B200ATTN_DECODE_SHAPE=<index into the table of the pool's dtype>.
int shape_override() {
  static int v = -1;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* e = getenv("B200ATTN_DECODE_SHAPE");
    v = e ? atoi(e) : -1;
  });
  return v;
}

Shape pick_shape(size_t es, int dpad) {
  if (dpad != 128) return es == 2 ? kSmallBf16 : kSmallF32;
  const int o = shape_override();
  if (es == 2) return kShapesBf16[(o >= 0 && o < kNumShapesBf16) ? o : 0];
  return kShapesF32[(o >= 0 && o < kNumShapesF32) ? o : 0];
}

struct Plan {
  Shape shape;
  int dpad, tile;
  int64_t num_hg, max_tiles, tiles_per_split, max_splits;
};

// Split-K plan (at most 64 splits, each >= 8 tiles).  Each split costs a
// CTA's setup and ring fill, its partial write and a share of the combine,
// so the plan takes the fewest splits that give about one wave of CTAs
// (85 % of the resident slots), as long as a CTA then covers at most
// kOneWaveTokens context tokens.  Longer CTAs need balance more: then the
// smallest count that gives at least two waves with the last wave >= 95 %
// full (the largest allowed count when none does).  Measured with the fused
// write on one B200 (bf16, 32 heads of 128): at 1 x 32768, 8 x 4096,
// 32 x 1024, 4 x 16384, 2 x 8192 and 16 x 2048 tokens, one wave ran
// 9-35 % faster than two or more; 64 x 32768 ran 6-8 % slower with one or
// two splits than with four.
constexpr int64_t kOneWaveTokens = 8192;
int64_t choose_tiles_per_split(int64_t units, int64_t max_tiles, int32_t hint, int num_sms,
                               int ctas_per_sm, int tile) {
  if (hint > 0) return ceil_div(max_tiles, std::min<int64_t>(hint, max_tiles));
  const int64_t slots = static_cast<int64_t>(num_sms) * ctas_per_sm;
  const int64_t smax = std::max<int64_t>(1, std::min<int64_t>(64, ceil_div(max_tiles, 8)));
  const int64_t s_one = std::min<int64_t>(smax, std::max<int64_t>(1, ceil_div(ceil_div(slots * 85, 100), units)));
  if (ceil_div(max_tiles, s_one) * tile <= kOneWaveTokens) return ceil_div(max_tiles, s_one);
  int64_t best = smax;
  for (int64_t s = 1; s <= smax; ++s) {
    const int64_t ctas = units * s;
    if (ctas < 2 * slots) continue;
    const double waves = static_cast<double>(ctas) / static_cast<double>(slots);
    if (waves / ceil(waves) >= 0.95) {
      best = s;
      break;
    }
  }
  return ceil_div(max_tiles, best);
}

Plan make_plan(int64_t B, int64_t H, int64_t D, int64_t M, int64_t S, int32_t hint, size_t es,
               int num_sms) {
  Plan pl;
  pl.dpad = pick_dpad(D, es);
  pl.shape = pick_shape(es, pl.dpad);
  pl.tile = tile_rows(pl.dpad, es);
  pl.max_tiles = ceil_div(M * S, pl.tile);
  pl.num_hg = ceil_div(H, pl.shape.g);
  pl.tiles_per_split = choose_tiles_per_split(B * pl.num_hg, pl.max_tiles, hint, num_sms,
                                              pl.shape.ctas_per_sm, pl.tile);
  pl.max_splits = ceil_div(pl.max_tiles, pl.tiles_per_split);
  return pl;
}

}  // namespace

size_t decode_workspace_bytes(int64_t B, int64_t H, int64_t D, int64_t M, int64_t S,
                              int32_t hint, size_t es, int num_sms) {
  const Plan pl = make_plan(B, H, D, M, S, hint, es, num_sms);
  if (pl.max_splits <= 1) return 0;
  size_t bytes = static_cast<size_t>(B * H * pl.max_splits) * (pl.dpad + 2) * sizeof(float);
  bytes = (bytes + 255) & ~size_t(255);
  bytes += static_cast<size_t>(B * pl.num_hg) * sizeof(int32_t);
  return (bytes + 255) & ~size_t(255);
}



template <typename KV, int DPAD, int G, int WPH, int STAGES>
static int launch_cfg(const DecodeParams& prm, const CUtensorMap& tk, const CUtensorMap& tv,
                      int64_t grid, size_t smem, cudaStream_t stream) {
  auto kern = paged_decode_kernel<KV, DPAD, G, WPH, STAGES>;
  // The attribute only ever grows (under a lock, so that concurrent first
  // calls with different sizes cannot lower it below a size in use).
  static std::atomic<int> configured[64];
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 &&
      configured[dev].load(std::memory_order_acquire) < static_cast<int>(smem)) {
    std::lock_guard<std::mutex> lock(mu);
    if (configured[dev].load(std::memory_order_relaxed) < static_cast<int>(smem)) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(paged_decode)");
      configured[dev].store(static_cast<int>(smem), std::memory_order_release);
    }
  }
  kern<<<static_cast<unsigned>(grid), DecodeCfg<KV, DPAD, G, WPH, STAGES>::THREADS, smem,
         stream>>>(tk, tv, prm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "paged_decode launch");
  return B200_OK;
}

template <typename KV, int DPAD, int I = 0>
static int launch_d128(const Shape& s, const DecodeParams& prm, const CUtensorMap& tk,
                       const CUtensorMap& tv, int64_t grid, size_t smem, cudaStream_t stream) {
  constexpr bool BF = sizeof(KV) == 2;
  constexpr int N = BF ? kNumShapesBf16 : kNumShapesF32;
  if constexpr (I < N) {
    constexpr Shape c = BF ? kShapesBf16[I] : kShapesF32[I];
    if (s.g == c.g && s.wph == c.wph && s.stages == c.stages)
      return launch_cfg<KV, DPAD, c.g, c.wph, c.stages>(prm, tk, tv, grid, smem, stream);
    return launch_d128<KV, DPAD, I + 1>(s, prm, tk, tv, grid, smem, stream);
  } else {
    return fail(B200_ERR_UNSUPPORTED, "paged decode: CTA shape not instantiated");
  }
}

template <typename KV>
static int launch_small(int dpad, const DecodeParams& prm, const CUtensorMap& tk,
                        const CUtensorMap& tv, int64_t grid, size_t smem, cudaStream_t stream) {
  constexpr Shape sh = sizeof(KV) == 2 ? kSmallBf16 : kSmallF32;
  constexpr int G = sh.g, W = sh.wph, ST = sh.stages;
  switch (dpad) {
    case 4:
      if constexpr (sizeof(KV) == 4) return launch_cfg<KV, 4, G, W, ST>(prm, tk, tv, grid, smem, stream);
      break;
    case 8: return launch_cfg<KV, 8, G, W, ST>(prm, tk, tv, grid, smem, stream);
    case 16: return launch_cfg<KV, 16, G, W, ST>(prm, tk, tv, grid, smem, stream);
    case 32: return launch_cfg<KV, 32, G, W, ST>(prm, tk, tv, grid, smem, stream);
    case 64: return launch_cfg<KV, 64, G, W, ST>(prm, tk, tv, grid, smem, stream);
    default: break;
  }
  return fail(B200_ERR_UNSUPPORTED, "paged decode: head_dim padding not instantiated");
}

int launch_paged_decode(const DecodeLaunch& a, cudaStream_t stream) {
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc != B200_OK) return rc;
  const size_t es = dtype_size(a.pool.dtype);
  const int64_t S = a.pool.block_size, H = a.pool.num_heads, D = a.pool.head_dim;
  const int64_t P = a.pool.num_blocks, L = a.pool.num_layers;
  const Plan pl = make_plan(a.batch, H, D, a.table_width, S, a.max_splits_hint, es, dev.num_sms);
  const int dpad = pl.dpad;
  const int g = pl.shape.g;

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
  prm.tiles_per_split = static_cast<int32_t>(pl.tiles_per_split);
  prm.max_splits = static_cast<int32_t>(pl.max_splits);
  prm.num_hg = static_cast<int32_t>(pl.num_hg);
  prm.gbox = static_cast<int32_t>(std::min<int64_t>(g, H));
  prm.rbox = static_cast<int32_t>(std::min<int64_t>(S, pl.tile));
  prm.rb_shift = log2i(prm.rbox);
  prm.box_bytes = static_cast<int32_t>(prm.rbox * prm.gbox * dpad * es);
  prm.box_stride = (prm.box_bytes + 127) & ~127;
  prm.nbox = pl.tile / prm.rbox;
  prm.stage_bytes = 2 * prm.nbox * prm.box_stride;
  prm.status = a.status;
  prm.qscale = static_cast<float>(1.0 / sqrt(static_cast<double>(D)) * 1.4426950408889634);

  if (pl.max_splits > 1) {
    const size_t need = decode_workspace_bytes(a.batch, H, D, a.table_width, S,
                                               a.max_splits_hint, es, dev.num_sms);
    if (a.workspace == nullptr || a.workspace_bytes < need) {
      char buf[160];
      snprintf(buf, sizeof(buf), "paged decode needs %zu workspace bytes, got %zu", need,
               a.workspace_bytes);
      return fail(B200_ERR_WORKSPACE, buf);
    }
    uint8_t* ws = static_cast<uint8_t*>(a.workspace);
    const size_t acc_bytes =
        static_cast<size_t>(a.batch * H * pl.max_splits) * dpad * sizeof(float);
    const size_t ml_bytes = static_cast<size_t>(a.batch * H * pl.max_splits) * 2 * sizeof(float);
    prm.ws_acc = reinterpret_cast<float*>(ws);
    prm.ws_ml = reinterpret_cast<float*>(ws + acc_bytes);
    size_t cnt_off = (acc_bytes + ml_bytes + 255) & ~size_t(255);
    prm.ws_cnt = reinterpret_cast<int32_t*>(ws + cnt_off);
    // The counters' location depends on (B, H, splits), so a workspace
    // reused across calls of other shapes may hold stale data there; clear
    // them on the stream before the launch (an async memset, no allocation).
    cudaError_t me = cudaMemsetAsync(
        prm.ws_cnt, 0, static_cast<size_t>(a.batch * pl.num_hg) * sizeof(int32_t), stream);
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

  const size_t merge_bytes = static_cast<size_t>(g * pl.shape.wph) * (dpad + 2) * sizeof(float);
  const size_t smem = 256 + static_cast<size_t>(pl.shape.stages) * prm.stage_bytes + merge_bytes;
  if (smem > static_cast<size_t>(dev.max_smem_optin))
    return fail(B200_ERR_UNSUPPORTED, "paged decode: stage ring exceeds shared memory");
  const int64_t grid = a.batch * pl.num_hg * pl.max_splits;
  if (grid > 0x7fffffffLL) return fail(B200_ERR_UNSUPPORTED, "paged decode: grid too large");

  if (dpad == 128) {
    if (es == 4) return launch_d128<float, 128>(pl.shape, prm, tk, tv, grid, smem, stream);
    return launch_d128<__nv_bfloat16, 128>(pl.shape, prm, tk, tv, grid, smem, stream);
  }
  if (es == 4) return launch_small<float>(dpad, prm, tk, tv, grid, smem, stream);
  return launch_small<__nv_bfloat16>(dpad, prm, tk, tv, grid, smem, stream);
}

}  // namespace b200
