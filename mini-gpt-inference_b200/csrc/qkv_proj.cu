// qkv_proj.cu -- the attention's fused QKV projection with the KV-cache write
// in its epilogue, on tcgen05 tensor cores (bf16 operands, f32 accumulate).
//
//   y = x W^T            x [T, C], W [3C, C]: the bias-free `qkv` Linear of
//                        minivllm/attention.py:79-83
//   q_out[t]                    = y[t, 0:C]
//   pool.k[layer, slot[t] / S, slot[t] % S] = y[t, C:2C]
//   pool.v[layer, slot[t] / S, slot[t] % S] = y[t, 2C:3C]
//
// The reference computes qkv(x), splits it with chunk(3) and views
// (attention.py:177-191, :360-368), then writes k and v into the pool per
// token (attention.py:193-208 through KVBlockPool.write_layer) or by
// index_put (attention.py:370-392).  A pool row (one token of one block, all
// heads) is H * D = C contiguous elements, exactly the k (or v) third of an
// output row, so the epilogue stores each run of a row straight into the
// row's slot and k and v never exist as a separate tensor.
//
// Three kernels share the warp roles below; qkv_plan picks one per call:
//   CTA pairs   129+ tokens: 256 x BN tiles, tcgen05.mma.cta_group::2 (BN =
//               192 up to 256 tokens, where it keeps more SMs busy, else 256);
//   single CTA  128 x BN tiles (BN = 64 or 128) where those waves are
//               cheaper than pair waves, and 97-256 tokens where one wave
//               of them keeps more SMs busy than the pairs;
//   split-K     decode-size token counts (<= 96, or <= 128 where single-CTA
//               tiles need more than one wave): one output tile per
//               cluster, the reduction split over the cluster's CTAs.
// The persistent ones (one CTA per SM) walk the output tiles in the grouped
// order of tile_coords.  Warp roles (6 warps):
//   warp 0     TMA producer: the x tile (128 x 64) and the W tile (BN x 64)
//              of each k-step, 128-byte swizzle, into a STAGES-deep ring;
//   warp 1     TMEM allocation and MMA issue: D[acc] += A B^T with M = 128,
//              N = BN, K = 16 per instruction (both operands K-major); two
//              TMEM accumulators, so the epilogue of one tile overlaps the
//              MMAs of the next;
//   warps 2-5  epilogue: thread r owns output row r (TMEM lane r), reads 64
//              columns at a time and rounds them to bf16 (nearest even);
//              the warp stores its 32 rows' 128-byte runs to q_out or to
//              the rows' pool slots through shared staging rows (whole
//              lines per store instruction).
// Rows past T and columns past 3C are zero-filled by TMA (or, past the
// x box of a short token tile, left stale) and not stored.
// A slot outside [0, P*S) sets B200_DEV_BAD_SLOT and skips that row's k and
// v (q is still written).  Every mbarrier wait is bounded; on a timeout the
// CTA reports B200_DEV_WAIT_TIMEOUT, lets its own copies and MMAs finish,
// frees TMEM and exits.
#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "host_util.h"
#include "kernels.h"
#include "tcgen05.cuh"

namespace b200 {
namespace {

constexpr int kBM = 128;                 // tokens per tile (TMEM lanes)
constexpr int kBK = 64;                  // reduction elements per stage (one 128-byte row)
constexpr int kThreads = 192;            // producer, MMA issuer, 4 epilogue warps
constexpr int kRingBytes = 192 * 1024;   // operand ring (1 CTA per SM)
// Epilogue stores of the tile kernels.  An epilogue warp holds 32 token
// rows of an accumulator, one per lane; stored from registers, each 16-byte
// store of the warp would touch 32 rows (32 memory requests per
// instruction).  Instead each 64-column batch is rounded to bf16, written
// to the warp's staging rows in shared memory and read back so that 8
// consecutive lanes store one row's 128 contiguous bytes: 4 rows, whole
// lines, per instruction.  Staging rows are kEpiPitch = 128 + 16 bytes
// apart, so both the row-wise writes and the line-wise reads of 8 lanes
// fall in distinct banks.
constexpr int kEpiPitch = 144;
constexpr int kEpiWarpBytes = 32 * kEpiPitch;
constexpr int kEpiBytes = 4 * kEpiWarpBytes;  // the four epilogue warps

template <int BN>
struct QkvCfg {
  static constexpr int A_BYTES = kBM * 128;  // x tile: 128 rows of 64 bf16
  static constexpr int B_BYTES = BN * 128;   // W tile: BN rows of 64 bf16
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGES = kRingBytes / STAGE;  // 6 / 8 for BN 128 / 64
  static constexpr int BAR = STAGES * STAGE;
  static constexpr int EPI = BAR + 256;  // the epilogue warps' staging rows
  static constexpr int BYTES = EPI + kEpiBytes;
  static constexpr int TMEM_COLS = 2 * BN;  // two f32 accumulators
  static_assert(STAGE % 1024 == 0, "stages must keep the 1024-byte swizzle alignment");
  static_assert((2 * STAGES + 5) * 8 + 8 <= 256, "barrier area too small");
};

struct QkvParams {
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_pool;
  __nv_bfloat16* v_pool;
  const void* slots;
  int64_t q_rs;     // q_out row stride (elements)
  int64_t ss;       // slot stride (elements)
  int64_t T, C;
  int64_t row0;     // layer * P * S: the layer's first pool row
  int64_t nslots;   // P * S
  int32_t slots_i64;
  int32_t m_tiles, n_tiles, k_iters;
  int32_t x_rows;  // token rows per x box of a CTA (128, or fewer for one short tile)
  int32_t* status;
};

// Tile order: token tiles run fastest inside groups covering kGroupRows
// tokens, and a group sweeps every weight tile before the next group
// starts, so the CTAs running at once share a few MB of x and of W in L2
// (the 126 MB L2 holds neither all of x nor all of W at prefill sizes).
constexpr int kGroupRows = 4096;
__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int group, int& mt,
                                            int& nt) {
  const int per_group = group * n_tiles;
  const int g = t / per_group;
  const int first = g * group;
  const int rows = min(group, m_tiles - first);
  const int r = t - g * per_group;
  mt = first + r % rows;
  nt = r / rows;
}

// Stores RW f32 values as RW bf16 (2 * RW contiguous bytes, 16-byte aligned).
template <int RW>
__device__ __forceinline__ void store_run(__nv_bfloat16* dst, const float* v) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < RW / 8; ++i)
    d[i] = make_uint4(pack_bf16(v[8 * i], v[8 * i + 1]), pack_bf16(v[8 * i + 2], v[8 * i + 3]),
                      pack_bf16(v[8 * i + 4], v[8 * i + 5]), pack_bf16(v[8 * i + 6], v[8 * i + 7]));
}

// Destination of columns [n, n + 64) of token row `row`, or nullptr when
// they are not stored (a row past the tokens, columns past 3C, a bad
// slot).  n and C are multiples of 64, so the run lies in one of q, k, v;
// dst_row is the token's first element in the layer's pool rows (< 0: no
// slot).
__device__ __forceinline__ __nv_bfloat16* epi_dst(const QkvParams& p, bool live, int64_t row,
                                                  int64_t dst_row, int64_t n) {
  if (!live || n >= 3 * p.C) return nullptr;
  if (n < p.C) return p.q_out + row * p.q_rs + n;
  if (dst_row < 0) return nullptr;
  return n < 2 * p.C ? p.k_pool + dst_row + (n - p.C) : p.v_pool + dst_row + (n - 2 * p.C);
}

// Loads 64 accumulator columns at TMEM address `taddr` (this warp's lane
// quarter) and stores lane l's row to dst (per lane; nullptr: skipped)
// through the warp's staging rows `stage`.  Warp-collective.
__device__ __forceinline__ void epi_store64(uint32_t taddr, uint8_t* stage, __nv_bfloat16* dst,
                                            int lane) {
  float v[64];
  __syncwarp();  // tcgen05.ld is warp-collective; the staging rows are free
  tmem_ld32(taddr, v);
  tmem_ld32(taddr + 32u, v + 32);
  tmem_wait_ld();
  uint4* srow = reinterpret_cast<uint4*>(stage + lane * kEpiPitch);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    srow[i] = make_uint4(pack_bf16(v[8 * i], v[8 * i + 1]), pack_bf16(v[8 * i + 2], v[8 * i + 3]),
                         pack_bf16(v[8 * i + 4], v[8 * i + 5]), pack_bf16(v[8 * i + 6], v[8 * i + 7]));
  __syncwarp();
  const unsigned long long d = reinterpret_cast<unsigned long long>(dst);
  const int part = lane & 7;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = (lane >> 3) + 4 * i;
    const unsigned long long rd = __shfl_sync(0xffffffffu, d, r);
    const uint4 val = *reinterpret_cast<const uint4*>(stage + r * kEpiPitch + part * 16);
    if (rd != 0ull) reinterpret_cast<uint4*>(rd)[part] = val;
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    qkv_kv_write_kernel(const __grid_constant__ CUtensorMap tmx,
                        const __grid_constant__ CUtensorMap tmw, const QkvParams p) {
  using Cfg = QkvCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::BAR);  // [STAGES] operands landed
  uint64_t* empty = full + STAGES;                                // [STAGES] MMAs read them
  uint64_t* acc_full = empty + STAGES;                            // [2] accumulator complete
  uint64_t* acc_empty = acc_full + 2;                             // [2] epilogue drained it
  uint64_t* drain = acc_empty + 2;                                // all MMAs done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int32_t* abort_flag = reinterpret_cast<int32_t*>(tmem_slot + 1);
  volatile int32_t* abort_v = abort_flag;

  if (threadIdx.x == 0) {
    // The tensor maps are fetched while the barriers and TMEM are set up.
    tma_prefetch_desc(&tmx);
    tma_prefetch_desc(&tmw);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(Cfg::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int ntiles = p.m_tiles * p.n_tiles;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int64_t issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
        int mt, nt;
        tile_coords(t, p.m_tiles, p.n_tiles, kGroupRows / kBM, mt, nt);
        const int m0 = mt * kBM;
        const int n0 = nt * BN;
        for (int kb = 0; kb < p.k_iters; ++kb) {
          const int st = static_cast<int>(issued % STAGES);
          const uint32_t use = static_cast<uint32_t>(issued / STAGES);
          if (*abort_v || !mbar_wait(&empty[st], (use & 1u) ^ 1u)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(p.x_rows * 128 + Cfg::B_BYTES));
          uint8_t* a = smem + st * Cfg::STAGE;
          tma_load_2d(a, &tmx, &full[st], kb * kBK, m0);
          tma_load_2d(a + Cfg::A_BYTES, &tmw, &full[st], kb * kBK, n0);
          ++issued;
        }
      }
      if (!ok) {
        report(p.status, B200_DEV_WAIT_TIMEOUT);
        *abort_v = 1;
      }
      // Each of the last (up to) STAGES loads must land before the CTA
      // exits; earlier ones were waited for before their stage was reused.
      for (int64_t j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j)
        if (!mbar_wait(&full[j % STAGES], static_cast<uint32_t>(j / STAGES) & 1u)) {
          report(p.status, B200_DEV_WAIT_TIMEOUT);
          break;
        }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop (values stay warp-uniform); every lane
    // waits on the barriers and a vote makes the outcome uniform;
    // elect.sync picks the issuing lane.
    auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, *abort_v == 0 && mbar_wait(bar, parity)) != 0;
    };
    constexpr uint32_t idesc = idesc_bf16(kBM, BN, false);
    // Stage bases are 1024-aligned; a k-step of 16 elements is 32 bytes
    // inside the 128-byte swizzle row (+2 in the descriptor's address
    // field, which cannot carry: shared memory is < 256 KB).
    const uint64_t da0 = smem_desc_sw128(smem_u32(smem), 16, 1024);
    int64_t consumed = 0;
    bool ok = true;
    int i = 0;
    for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x, ++i) {
      const int acc = i & 1;
      const uint32_t use = static_cast<uint32_t>(i >> 1);
      if (!wait_all(&acc_empty[acc], (use & 1u) ^ 1u)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t td = tmem + static_cast<uint32_t>(acc * BN);
      for (int kb = 0; kb < p.k_iters; ++kb, ++consumed) {
        const int st = static_cast<int>(consumed % STAGES);
        if (!wait_all(&full[st], static_cast<uint32_t>(consumed / STAGES) & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t da = da0 + static_cast<uint64_t>((st * Cfg::STAGE) >> 4);
        const uint64_t db = da + static_cast<uint64_t>(Cfg::A_BYTES >> 4);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          mma_bf16(td, da + static_cast<uint64_t>(kk * 2), db + static_cast<uint64_t>(kk * 2), idesc,
                   (kb > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&empty[st]);  // the stage is free once these MMAs have read it
      }
      if (!ok) break;
      mma_commit(&acc_full[acc]);
    }
    if (!ok && lane == 0) {
      report(p.status, B200_DEV_WAIT_TIMEOUT);
      *abort_v = 1;
    }
    // Every MMA this thread issued completes before TMEM is freed.
    mma_commit(drain);
    if (!__all_sync(0xffffffffu, mbar_wait(drain, 0)) && lane == 0)
      report(p.status, B200_DEV_WAIT_TIMEOUT);
  } else {
    // ------------------------------------------------------------ epilogue
    // A warp may only touch TMEM lanes [32 * (warp % 4), +32): warps 2-5
    // cover quarters 2, 3, 0, 1.
    const int qd = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(qd * 32) << 16;
    uint8_t* stage = smem + Cfg::EPI + qd * kEpiWarpBytes;
    int i = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
      const int acc = i & 1;
      const uint32_t use = static_cast<uint32_t>(i >> 1);
      // The row's destination (its slot is a global load) is resolved while
      // the tile's MMAs still run.
      int mt, nt;
      tile_coords(t, p.m_tiles, p.n_tiles, kGroupRows / kBM, mt, nt);
      const int64_t row = static_cast<int64_t>(mt) * kBM + qd * 32 + lane;
      const int64_t n0 = static_cast<int64_t>(nt) * BN;
      const bool live = row < p.T;
      // The slot is needed only when the tile reaches the k / v columns.
      int64_t dst_row = -1;
      if (live && n0 + BN > p.C) {
        const int64_t slot = load_index(p.slots, row * p.ss, p.slots_i64);
        if (slot >= 0 && slot < p.nslots) {
          dst_row = (p.row0 + slot) * p.C;
        } else {
          report(p.status, B200_DEV_BAD_SLOT);
        }
      }
      if (!__all_sync(0xffffffffu, *abort_v == 0 && mbar_wait(&acc_full[acc], use & 1u))) {
        if (lane == 0) {
          report(p.status, B200_DEV_WAIT_TIMEOUT);
          *abort_v = 1;
        }
        break;
      }
      tc_fence_after();
      const uint32_t tacc = tmem + lane_base + static_cast<uint32_t>(acc * BN);
      // BN and n0 are multiples of 64: every batch lies in one of q, k, v.
#pragma unroll 1
      for (int c = 0; c < BN; c += 64)
        epi_store64(tacc + static_cast<uint32_t>(c), stage, epi_dst(p, live, row, dst_row, n0 + c), lane);
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(Cfg::TMEM_COLS)
                 : "memory");
  }
}

// ------------------------------------------------------------------ CTA pairs
// For long token runs the tiles are 256 tokens x BN features, computed by
// a cluster of two CTAs with tcgen05.mma.cta_group::2: CTA r of the pair
// loads token rows [128r, +128) of the x tile (a single tile of at most 256
// tokens is split evenly instead: `x_rows` rows per CTA, the A rows past
// them left stale, reaching only accumulator rows that are never stored)
// and feature rows [BN/2 * r, +BN/2) of the W tile, and the pair MMA (issued by CTA 0 only)
// multiplies the pair's 256 x rows by all BN W rows, each CTA's TMEM receiving the
// accumulator rows of its own tokens.  Per SM this halves the W bytes
// staged in shared memory for the same tensor work, which a single CTA
// with 256-wide tiles is limited by.  Both CTAs' copies complete on CTA 0's
// stage barrier; CTA 0's MMA commits release the stage in both CTAs and
// publish each accumulator to both epilogues; each epilogue warp of either
// CTA returns an accumulator to CTA 0 with one remote arrival.  Each CTA
// loads only its own rows: every TMA copy writes the issuing CTA's shared
// memory alone.  BN is 256 for long token runs (the fewest staged bytes
// per MAC) or 192 for 129-256 tokens (3C / 192 pairs keep more SMs busy).
constexpr int kPairBN = 256;
constexpr int kPairBNNarrow = 192;
template <int BN>
struct PairCfg {
  static constexpr int A_BYTES = kBM * 128;        // this CTA's 128 x rows
  static constexpr int B_BYTES = (BN / 2) * 128;   // this CTA's BN/2 W rows
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGES = kRingBytes / STAGE;  // 6
  static constexpr int BAR = STAGES * STAGE;
  static constexpr int EPI = BAR + 256;  // the epilogue warps' staging rows
  static constexpr int BYTES = EPI + kEpiBytes;
  static constexpr int TMEM_COLS = 512;            // two BN-column accumulators (a power of 2)
  static_assert(2 * BN <= TMEM_COLS, "two accumulators must fit the allocation");
  static_assert(STAGE % 1024 == 0, "stages must keep the 1024-byte swizzle alignment");
  static_assert((2 * STAGES + 5) * 8 + 8 <= 256, "barrier area too small");
};

template <int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    qkv_kv_write_pair_kernel(const __grid_constant__ CUtensorMap tmx,
                             const __grid_constant__ CUtensorMap tmw, const QkvParams p) {
  using Cfg = PairCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::BAR);  // [STAGES] (CTA 0's are used)
  uint64_t* empty = full + STAGES;                                // [STAGES] this CTA's stage free
  uint64_t* acc_full = empty + STAGES;                            // [2] in both CTAs
  uint64_t* acc_empty = acc_full + 2;                             // [2] (CTA 0's are used)
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int32_t* abort_flag = reinterpret_cast<int32_t*>(tmem_slot + 1);
  volatile int32_t* abort_v = abort_flag;

  if (threadIdx.x == 0) {
    // The tensor maps are fetched while the barriers and TMEM are set up.
    tma_prefetch_desc(&tmx);
    tma_prefetch_desc(&tmw);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 8);  // one arrival per epilogue warp of either CTA
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(Cfg::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  // Both CTAs' barriers exist before any copy or commit of the pair targets them.
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int m_tiles = static_cast<int>((p.T + 2 * kBM - 1) / (2 * kBM));
  const int ntiles = m_tiles * p.n_tiles;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (warp == 0) {
    // ------------------------------------------------------------ producers (both CTAs)
    if (lane == 0) {
      const uint32_t full0 = map_to_rank(full, 0);
      int64_t issued = 0;
      bool ok = true;
      for (int t = pair; ok && t < ntiles; t += npairs) {
        int mt, nt;
        tile_coords(t, m_tiles, p.n_tiles, kGroupRows / (2 * kBM), mt, nt);
        const int m0 = mt * 2 * kBM + static_cast<int>(rank) * p.x_rows;
        const int n0 = nt * BN + static_cast<int>(rank) * (BN / 2);
        for (int kb = 0; kb < p.k_iters; ++kb) {
          const int st = static_cast<int>(issued % STAGES);
          const uint32_t use = static_cast<uint32_t>(issued / STAGES);
          if (*abort_v || !mbar_wait(&empty[st], (use & 1u) ^ 1u)) {
            ok = false;
            break;
          }
          // CTA 0's stage barrier counts the bytes of both CTAs' copies.
          if (rank == 0) mbar_arrive_expect_tx(&full[st], 2u * static_cast<uint32_t>(p.x_rows * 128 + Cfg::B_BYTES));
          uint8_t* a = smem + st * Cfg::STAGE;
          const uint32_t bar = full0 + static_cast<uint32_t>(st * 8);
          tma_load_2d_pair(a, &tmx, bar, kb * kBK, m0);
          tma_load_2d_pair(a + Cfg::A_BYTES, &tmw, bar, kb * kBK, n0);
          ++issued;
        }
      }
      if (!ok) {
        report(p.status, B200_DEV_WAIT_TIMEOUT);
        *abort_v = 1;
      }
      // CTA 0 sees every copy of the pair land on its stage barriers.
      if (rank == 0)
        for (int64_t j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j)
          if (!mbar_wait(&full[j % STAGES], static_cast<uint32_t>(j / STAGES) & 1u)) {
            report(p.status, B200_DEV_WAIT_TIMEOUT);
            break;
          }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (CTA 0)
    if (rank == 0) {
      auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
        return __all_sync(0xffffffffu, *abort_v == 0 && mbar_wait(bar, parity)) != 0;
      };
      constexpr uint32_t idesc = idesc_bf16(2 * kBM, BN, false);
      const uint64_t da0 = smem_desc_sw128(smem_u32(smem), 16, 1024);
      int64_t consumed = 0;
      bool ok = true;
      int i = 0;
      for (int t = pair; ok && t < ntiles; t += npairs, ++i) {
        const int acc = i & 1;
        const uint32_t use = static_cast<uint32_t>(i >> 1);
        if (!wait_all(&acc_empty[acc], (use & 1u) ^ 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t td = tmem + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < p.k_iters; ++kb, ++consumed) {
          const int st = static_cast<int>(consumed % STAGES);
          if (!wait_all(&full[st], static_cast<uint32_t>(consumed / STAGES) & 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = da0 + static_cast<uint64_t>((st * Cfg::STAGE) >> 4);
          const uint64_t db = da + static_cast<uint64_t>(Cfg::A_BYTES >> 4);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_bf16_pair(td, da + static_cast<uint64_t>(kk * 2), db + static_cast<uint64_t>(kk * 2),
                          idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          mma_commit_pair_both(&empty[st]);
        }
        if (!ok) break;
        mma_commit_pair_both(&acc_full[acc]);
      }
      if (!ok && lane == 0) {
        report(p.status, B200_DEV_WAIT_TIMEOUT);
        *abort_v = 1;
      }
      mma_commit_pair_local(drain);
      if (!__all_sync(0xffffffffu, mbar_wait(drain, 0)) && lane == 0)
        report(p.status, B200_DEV_WAIT_TIMEOUT);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int qd = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(qd * 32) << 16;
    uint8_t* stage = smem + Cfg::EPI + qd * kEpiWarpBytes;
    const uint32_t acc_empty0 = map_to_rank(acc_empty, 0);
    int i = 0;
    for (int t = pair; t < ntiles; t += npairs, ++i) {
      const int acc = i & 1;
      const uint32_t use = static_cast<uint32_t>(i >> 1);
      // The row's destination (its slot is a global load) is resolved while
      // the tile's MMAs still run.
      int mt, nt;
      tile_coords(t, m_tiles, p.n_tiles, kGroupRows / (2 * kBM), mt, nt);
      const int lr = qd * 32 + lane;  // accumulator row (TMEM lane) of this CTA
      const int64_t row = static_cast<int64_t>(mt) * 2 * kBM + rank * p.x_rows + lr;
      const int64_t n0 = static_cast<int64_t>(nt) * BN;
      const bool live = lr < p.x_rows && row < p.T;
      int64_t dst_row = -1;
      if (live && n0 + BN > p.C) {
        const int64_t slot = load_index(p.slots, row * p.ss, p.slots_i64);
        if (slot >= 0 && slot < p.nslots) {
          dst_row = (p.row0 + slot) * p.C;
        } else {
          report(p.status, B200_DEV_BAD_SLOT);
        }
      }
      if (!__all_sync(0xffffffffu, *abort_v == 0 && mbar_wait(&acc_full[acc], use & 1u))) {
        if (lane == 0) {
          report(p.status, B200_DEV_WAIT_TIMEOUT);
          *abort_v = 1;
        }
        break;
      }
      tc_fence_after();
      const uint32_t tacc = tmem + lane_base + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN; c += 64)
        epi_store64(tacc + static_cast<uint32_t>(c), stage, epi_dst(p, live, row, dst_row, n0 + c), lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(acc_empty0 + static_cast<uint32_t>(acc * 8));
    }
  }
  // Neither CTA frees TMEM or exits while the pair's MMAs, copies or
  // arrivals may still touch it (every wait above is bounded, so both CTAs
  // get here).
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(Cfg::TMEM_COLS)
                 : "memory");
  }
}

// ------------------------------------------------------------------ split K
// Few tokens (decode): reading the 3C x C weight dominates, and TMA brings
// at most ~90 GB/s into one SM, so the weight stream must be spread over
// nearly every SM with as few bytes per SM as possible.  One tile per CTA
// of 256 features would use only 3C / 256 SMs (48 at C = 4096); instead
// the tile width (a multiple of 16, <= 256) and a split of the reduction
// over a cluster of `splits` CTAs are chosen per call: CTA r of a cluster
// accumulates k-steps [r * kpb, +kpb) of one output tile in its own TMEM.
// The x box is only as tall as the live tokens (rows of the A operand past
// it hold stale data, which only reaches accumulator rows that are never
// stored).  The live token rows are divided into `splits` contiguous
// ranges of `per` rows, CTA r owning range r.  Once this CTA's accumulator
// is complete, each thread reads its TMEM row and writes it to the row's
// owner: into
// its own staging rows, or with st.async into the owner's receive slot for
// this CTA, completing as transaction bytes on the owner's recv_full
// barrier; each sender's abort flag travels the same way.  The receive
// slots sit after the operand ring, so a CTA sends as soon as its own
// accumulator is complete, without waiting for its peers'.  The owner then
// sums its rows' partials in rank order (the same order every run) from
// its own shared memory, rounds once to bf16 and stores 32- (or 16-)
// column runs; the (row, run) items are spread over all of the CTA's
// threads.  The slot of each owned row is read while the MMAs run.  No CTA
// reads another's shared memory, and every CTA written to waits for its
// bytes, so no barrier is needed at the end.
constexpr int kSplitMaxBN = 256;
// A stage holds kc (1 or 2) consecutive 64-column chunks of x and W,
// fetched by one 3-D box per operand ({64 columns, rows, chunks}; the chunk
// dimension strides 128 bytes through the row).  Two chunks per box halve
// the copies per byte, whose per-box cost bounds short token counts; one
// chunk keeps the ring at >= 3 stages when the x rows are many.
constexpr int kSplitMaxKC = 2;
constexpr int kSplitMaxStages = 24;
// The operand ring, reused for the reduction rows once the MMAs are done;
// then the barriers and the slot of each token row.
constexpr int kSplitAreaBytes = 224 * 1024;
constexpr int kSplitBarOffset = kSplitAreaBytes;
constexpr int kSplitSlotOffset = kSplitBarOffset + 512;
constexpr int kSplitBytes = kSplitSlotOffset + kBM * 8;
constexpr int kSplitMaxCluster = 8;  // splits per cluster
static_assert((2 * kSplitMaxStages + 3) * 8 + 8 + 4 * kSplitMaxCluster <= 512, "barrier area too small");

struct SplitShape {
  int bn;           // output features per tile (multiple of 16, <= 256)
  int xrows;        // x box rows (multiple of 8, <= 128)
  int kc;           // 64-column chunks per stage (1 or 2)
  int stage_bytes;  // kc * (xrows + bn) * 128
  int stages;
  int splits;
  int kpb;          // k-steps per split
  int recv_off;     // byte offset of the receive slots after the ring, or 0:
                    // the slots follow this CTA's own rows in the ring
};

// Bytes of the receive slots of a split plan (a multiple of 1024): per
// peer, ceil(rows / splits) rows of bn + 4 floats.  Where they fit without
// costing the operand ring a stage they sit after it, so peers may write
// them while this CTA's MMAs still run; otherwise they follow this CTA's
// own rows in the ring, written once every CTA of the cluster is done.
int64_t split_recv_bytes(int rows, int bn, int splits) {
  const int64_t b = static_cast<int64_t>(splits - 1) * ((rows + splits - 1) / splits) * (bn + 4) * 4;
  return (b + 1023) / 1024 * 1024;
}

// A split plan fits when this CTA's own rows and the receive slots fit the
// reduction area (the slots may have to share the ring), and the ring holds
// at least two one-chunk stages (plus the M = 128 MMA's 16 KB A window past
// the last one).
bool split_fits(int rows, int bn, int splits) {
  const int64_t own = static_cast<int64_t>((rows + splits - 1) / splits) * (bn + 4) * 4;
  const int64_t stage = static_cast<int64_t>(rows + bn) * 128;
  return own + split_recv_bytes(rows, bn, splits) <= kSplitAreaBytes &&
         (kSplitAreaBytes - kBM * 128) / stage + 1 >= 2;
}

// 16-byte store into a cluster peer's shared memory, counted as 16
// transaction bytes on the peer's mbarrier (both shared::cluster addresses).
__device__ __forceinline__ void st_async_f4(uint32_t dst, float a, float b, float c, float d,
                                            uint32_t bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];"
      ::"r"(dst), "f"(a), "f"(b), "f"(c), "f"(d), "r"(bar)
      : "memory");
}

// 4-byte form of st_async_f4.
__device__ __forceinline__ void st_async_b32(uint32_t dst, int32_t v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];"
               ::"r"(dst), "r"(v), "r"(bar)
               : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    qkv_kv_write_split_kernel(const __grid_constant__ CUtensorMap tmx,
                              const __grid_constant__ CUtensorMap tmw, const QkvParams p,
                              const SplitShape sh) {
  const int STAGES = sh.stages;
  const int splits = sh.splits;
  const int bn = sh.bn;
  const int a_bytes = sh.kc * sh.xrows * 128;  // [chunk][x row][128 B]
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSplitBarOffset);
  uint64_t* empty = full + kSplitMaxStages;
  uint64_t* acc_full = empty + kSplitMaxStages;
  uint64_t* drain = acc_full + 1;
  uint64_t* recv_full = drain + 1;  // the peers' partials of this CTA's rows landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_full + 1);
  int32_t* abort_flag = reinterpret_cast<int32_t*>(tmem_slot + 1);
  // The abort flag of each sender of this CTA's rows (slot order), pushed
  // with the rows.
  int32_t* peer_flag = abort_flag + 1;  // [kSplitMaxCluster - 1]
  volatile int32_t* abort_v = abort_flag;
  int64_t* row_slot = reinterpret_cast<int64_t*>(smem + kSplitSlotOffset);  // [kBM]

  if (threadIdx.x == 0) {
    // The tensor maps are fetched while the barriers and TMEM are set up.
    tma_prefetch_desc(&tmx);
    tma_prefetch_desc(&tmw);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    mbar_init(recv_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kSplitMaxBN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Receive slots after the ring: every CTA of the cluster arrives once its
  // barriers exist and waits (below) before writing into a peer's shared
  // memory.  In the ring: one full cluster barrier after the MMAs.
  const bool early = sh.recv_off != 0;
  if (early) asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const int tile = blockIdx.x / splits;
  const int m0 = (tile % p.m_tiles) * kBM;
  const int n0 = (tile / p.m_tiles) * bn;
  const int k0 = static_cast<int>(rank) * sh.kpb;
  const int k1 = min(p.k_iters, k0 + sh.kpb);
  const int live = static_cast<int>(p.T - m0 < kBM ? p.T - m0 : kBM);
  // Up to 64 token rows the MMAs are M = 64: they read half the A rows.  The
  // M = 64 accumulator puts rows 16q .. 16q + 15 in TMEM lanes 32q .. 32q + 15;
  // acc_row gives the row that lane `lane` of lane quarter q holds (-1: none).
  const int mma_m = sh.xrows <= 64 ? 64 : kBM;
  auto acc_row = [&](int q, int ln) { return mma_m == 64 ? (ln < 16 ? q * 16 + ln : -1) : q * 32 + ln; };
  // Reduction rows: this CTA's own rows over the ring once its MMAs are
  // done, at (row - own_lo) * rs floats; the receive slots after the ring,
  // `per` rows per sender (sender q's slot is q, or q - 1 past this CTA's
  // rank).
  // Rows are bn + 4 floats apart: 16-byte aligned, and the 16-byte accesses
  // of a warp's 32 consecutive rows fall in distinct banks.
  const int rs = bn + 4;
  const int per = (live + splits - 1) / splits;
  auto own_lo = [&](int q) { return min(live, q * per); };
  auto own_n = [&](int q) { return min(live, q * per + per) - min(live, q * per); };
  auto slot_of = [&](int sender, int owner) { return sender < owner ? sender : sender - 1; };
  float* stage_rows = reinterpret_cast<float*>(smem);
  float* recv_rows = early ? reinterpret_cast<float*>(smem + sh.recv_off) : stage_rows + per * rs;

  if (warp == 0) {
    if (lane == 0) {
      // Every CTA of a split reads the same x columns; starting each tile's
      // walk at its own k-step spreads those reads over the L2 slices
      // instead of all CTAs requesting one chunk at a time.
      const int nk = k1 - k0;
      const int rot = nk > 0 ? tile % nk : 0;
      int issued = 0;
      for (; issued < nk; ++issued) {
        const int kb = k0 + (issued + rot) % nk;
        const int st = issued % STAGES;
        if (*abort_v || !mbar_wait(&empty[st], ((issued / STAGES) & 1) ^ 1)) {
          report(p.status, B200_DEV_WAIT_TIMEOUT);
          *abort_v = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(sh.stage_bytes));
        uint8_t* a = smem + st * sh.stage_bytes;
        tma_load_3d(a, &tmx, &full[st], 0, m0, kb * sh.kc);
        tma_load_3d(a + a_bytes, &tmw, &full[st], 0, n0, kb * sh.kc);
      }
      for (int j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j)
        if (!mbar_wait(&full[j % STAGES], (j / STAGES) & 1)) {
          report(p.status, B200_DEV_WAIT_TIMEOUT);
          break;
        }
    }
  } else if (warp == 1) {
    const uint32_t idesc = idesc_bf16(mma_m, bn, false);
    const uint64_t da0 = smem_desc_sw128(smem_u32(smem), 16, 1024);
    bool ok = true;
    for (int kb = k0, j = 0; kb < k1; ++kb, ++j) {
      const int st = j % STAGES;
      if (!__all_sync(0xffffffffu, *abort_v == 0 && mbar_wait(&full[st], (j / STAGES) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint64_t da = da0 + static_cast<uint64_t>((st * sh.stage_bytes) >> 4);
      const uint64_t db = da + static_cast<uint64_t>(a_bytes >> 4);
#pragma unroll
      for (int c = 0; c < kSplitMaxKC; ++c)
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          if (c < sh.kc)
            mma_bf16(tmem, da + static_cast<uint64_t>((c * sh.xrows * 128 + kk * 32) >> 4),
                     db + static_cast<uint64_t>((c * bn * 128 + kk * 32) >> 4), idesc,
                     (j > 0 || c > 0 || kk > 0) ? 1u : 0u);
        }
      mma_commit(&empty[st]);
    }
    if (ok) {
      mma_commit(acc_full);
    } else if (lane == 0) {
      report(p.status, B200_DEV_WAIT_TIMEOUT);
      *abort_v = 1;
    }
    mma_commit(drain);
    if (!__all_sync(0xffffffffu, mbar_wait(drain, 0)) && lane == 0)
      report(p.status, B200_DEV_WAIT_TIMEOUT);
  } else {
    const int r = acc_row(warp & 3, lane);
    // The slots of the rows this CTA stores, read while the MMAs run.
    if (r >= own_lo(rank) && r < own_lo(rank) + own_n(rank) && n0 + bn > p.C)
      row_slot[r] = load_index(p.slots, (m0 + r) * p.ss, p.slots_i64);
    if (warp == 2 && lane == 0)
      mbar_arrive_expect_tx(recv_full, static_cast<uint32_t>(
                                           own_n(rank) > 0 ? (splits - 1) * (own_n(rank) * bn * 4 + 4) : 0));
    if (!__all_sync(0xffffffffu, *abort_v == 0 && mbar_wait(acc_full, 0)) && lane == 0) {
      report(p.status, B200_DEV_WAIT_TIMEOUT);
      *abort_v = 1;
    }
    tc_fence_before();
  }
  __syncthreads();
  if (early)
    // Every peer's barriers exist (arrived long ago: this does not wait for
    // the peers' MMAs; the receive slots are not part of the ring).
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  else
    cluster_sync_all();  // every CTA's MMAs are done and its ring idle
  if (warp >= 2) {
    // Each thread sends its TMEM row to the row's owner; the thread holding
    // an owner's first row also sends this CTA's abort flag.  A CTA whose
    // accumulator was abandoned sends zeros, so that every owner's byte
    // count completes; its flag tells the owner to store nothing.  No CTA
    // reads another's shared memory, so none need wait for the others at
    // the end: an owner leaves only once its bytes have landed.
    tc_fence_after();
    const int qd = warp & 3;
    const int r = acc_row(qd, lane);
    const int owner = r >= 0 && r < live ? r / per : -1;
    const int32_t my_flag = *abort_v;
    const bool mine_ok = my_flag == 0;
    const uint32_t trow = tmem + (static_cast<uint32_t>(qd * 32) << 16);
    float* local = stage_rows;
    uint32_t remote = 0, bar = 0;
    if (owner == static_cast<int>(rank)) {
      local = stage_rows + (r - own_lo(owner)) * rs;
    } else if (owner >= 0) {
      const uint32_t o = static_cast<uint32_t>(owner);
      const int slot = slot_of(static_cast<int>(rank), owner);
      remote = map_to_rank(recv_rows + (slot * per + (r - own_lo(owner))) * rs, o);
      bar = map_to_rank(recv_full, o);
      if (r == own_lo(owner)) st_async_b32(map_to_rank(peer_flag + slot, o), my_flag, bar);
    }
    // The next 32 columns load from TMEM while the current ones are sent.
    float v[2][32];
    if (mine_ok) tmem_ld32(trow, v[0]);
#pragma unroll
    for (int i = 0; i < kSplitMaxBN / 32; ++i) {
      const int c = i * 32;
      if (c >= bn) break;
      float* cur = v[i & 1];
      if (mine_ok) {
        tmem_wait_ld();
        if (c + 32 < bn) tmem_ld32(trow + static_cast<uint32_t>(c + 32), v[(i + 1) & 1]);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) cur[e] = 0.f;
      }
      // Only the tile's bn columns are sent (bn may end half-way into a
      // 32-column load).
      if (owner == static_cast<int>(rank)) {
        float4* dst = reinterpret_cast<float4*>(local + c);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (c + 4 * e < bn)
            dst[e] = make_float4(cur[4 * e], cur[4 * e + 1], cur[4 * e + 2], cur[4 * e + 3]);
      } else if (owner >= 0) {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (c + 4 * e < bn)
            st_async_f4(remote + static_cast<uint32_t>((c + 4 * e) * 4), cur[4 * e], cur[4 * e + 1],
                        cur[4 * e + 2], cur[4 * e + 3], bar);
      }
    }
    tc_fence_before();
  }
  __syncthreads();  // this CTA's own rows are staged
  {
    const int lo = own_lo(static_cast<int>(rank));
    const int n_own = own_n(static_cast<int>(rank));
    bool ready = n_own > 0;
    if (ready && !mbar_wait(recv_full, 0)) {
      report(p.status, B200_DEV_WAIT_TIMEOUT);
      ready = false;
    }
    bool all_ok = *abort_v == 0;
    for (int q = 0; q < splits - 1; ++q) all_ok = all_ok && (!ready || peer_flag[q] == 0);
    // Items (owned row, RW-column run), rows fastest: a warp's 16-byte
    // loads of one run cover consecutive rows.  Runs are 32 columns, or 16
    // when bn is not a multiple of 32 (a 32-column run could then straddle
    // the q / k / v boundaries, which are multiples of 64).
    auto sum_pass = [&](auto run_width) {
      constexpr int RW = decltype(run_width)::value;
      const int items = ready && all_ok ? n_own * (bn / RW) : 0;
      for (int it = threadIdx.x; it < items; it += kThreads) {
        const int lr = it % n_own;
        const int c = (it / n_own) * RW;
        const int64_t n = n0 + c;
        if (n >= 3 * p.C) continue;
        float acc[RW];
#pragma unroll
        for (int i = 0; i < RW; ++i) acc[i] = 0.f;
        for (int q = 0; q < splits; ++q) {
          const float* src = q == static_cast<int>(rank)
                                 ? stage_rows + lr * rs + c
                                 : recv_rows + (slot_of(q, static_cast<int>(rank)) * per + lr) * rs + c;
#pragma unroll
          for (int i = 0; i < RW / 4; ++i) {
            const float4 v = reinterpret_cast<const float4*>(src)[i];
            acc[4 * i] += v.x;
            acc[4 * i + 1] += v.y;
            acc[4 * i + 2] += v.z;
            acc[4 * i + 3] += v.w;
          }
        }
        const int64_t row = m0 + lo + lr;
        if (n < p.C) {
          store_run<RW>(p.q_out + row * p.q_rs + n, acc);
        } else {
          const int64_t slot = row_slot[lo + lr];
          if (slot < 0 || slot >= p.nslots) {
            report(p.status, B200_DEV_BAD_SLOT);
          } else if (n < 2 * p.C) {
            store_run<RW>(p.k_pool + (p.row0 + slot) * p.C + (n - p.C), acc);
          } else {
            store_run<RW>(p.v_pool + (p.row0 + slot) * p.C + (n - 2 * p.C), acc);
          }
        }
      }
    };
    if (bn % 32 == 0)
      sum_pass(std::integral_constant<int, 32>{});
    else
      sum_pass(std::integral_constant<int, 16>{});
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kSplitMaxBN)
                 : "memory");
  }
}

// Shared-memory clocks per 16-deep k-step on one SM: the MMA reads the A
// and B rows of the step and TMA writes the same bytes into the ring, at
// 128 bytes per clock between them (above the tensor clocks for every
// single-CTA tile width: M128 x N takes N/2 clocks).  A CTA pair with
// 256-wide tiles stages 128 A rows and 128 B rows per SM: 128 clocks, equal
// to its tensor clocks.
int step_clocks(int bn) { return (kBM + bn) / 2; }
constexpr int kPairStepClocks = 128;

// Tensor map of a bf16 [rows, cols] matrix (row stride in elements, a
// multiple of 8): boxes of 64 columns x box_rows rows, 128-byte swizzle.
int encode_rows(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t row_stride,
                int box_rows) {
  const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {static_cast<uint64_t>(row_stride * 2)};
  const uint32_t box[2] = {static_cast<uint32_t>(kBK), static_cast<uint32_t>(box_rows)};
  return encode_tensor_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                           strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Guards the first-call setup per device (kernel attributes, occupancy
// queries); later calls read the cached results without locking.
std::mutex g_setup_mu;

// Kernel parameters of one call: tiles of tile_m tokens x tile_n features,
// k-steps of step_k reduction columns.
QkvParams make_params(const b200_qkv_kv_write_args_t& a, int tile_m, int tile_n, int step_k) {
  QkvParams prm;
  memset(&prm, 0, sizeof(prm));
  prm.q_out = static_cast<__nv_bfloat16*>(a.q_out);
  prm.k_pool = static_cast<__nv_bfloat16*>(a.pool.k);
  prm.v_pool = static_cast<__nv_bfloat16*>(a.pool.v);
  prm.slots = a.slot_mapping;
  prm.q_rs = a.q_row_stride;
  prm.ss = a.slot_stride;
  prm.T = a.num_tokens;
  prm.C = a.hidden;
  prm.row0 = a.layer_idx * a.pool.num_blocks * a.pool.block_size;
  prm.nslots = a.pool.num_blocks * a.pool.block_size;
  prm.slots_i64 = a.slot_dtype == B200_INDEX_I64;
  prm.m_tiles = static_cast<int32_t>(ceil_div(a.num_tokens, tile_m));
  prm.n_tiles = static_cast<int32_t>(ceil_div(3 * a.hidden, tile_n));
  prm.k_iters = static_cast<int32_t>(ceil_div(a.hidden, step_k));
  prm.status = a.status;
  return prm;
}

template <int BN>
int launch_bn(const b200_qkv_kv_write_args_t& a, cudaStream_t stream, const DeviceInfo& dev) {
  using Cfg = QkvCfg<BN>;
  const int64_t T = a.num_tokens, C = a.hidden;
  const size_t smem = static_cast<size_t>(Cfg::BYTES) + 1024;
  if (smem > static_cast<size_t>(dev.max_smem_optin))
    return fail(B200_ERR_UNSUPPORTED, "qkv projection: not enough shared memory");

  // A single token tile stages only its live rows (rounded up to 8): the A
  // rows past them are stale and reach only accumulator rows never stored.
  const int rows = T < kBM ? static_cast<int>((T + 7) / 8 * 8) : kBM;
  CUtensorMap tx, tw;
  int rc = encode_rows(&tx, a.x, T, C, a.x_row_stride, rows);
  if (rc == B200_OK) rc = encode_rows(&tw, a.weight, 3 * C, C, C, BN);
  if (rc != B200_OK) return rc;
  static std::atomic<int> configured[64];
  if (dev.device >= 0 && dev.device < 64 && !configured[dev.device].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    cudaError_t e = cudaFuncSetAttribute(qkv_kv_write_kernel<BN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(qkv_kv_write)");
    configured[dev.device].store(1, std::memory_order_release);
  }
  QkvParams prm = make_params(a, kBM, BN, kBK);
  prm.x_rows = rows;
  const int64_t tiles = static_cast<int64_t>(prm.m_tiles) * prm.n_tiles;
  const int grid = static_cast<int>(std::min<int64_t>(tiles, dev.num_sms));
  qkv_kv_write_kernel<BN><<<grid, kThreads, smem, stream>>>(tx, tw, prm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "qkv_kv_write launch");
  return B200_OK;
}

template <int BN>
int launch_pair(const b200_qkv_kv_write_args_t& a, cudaStream_t stream, const DeviceInfo& dev) {
  using Cfg = PairCfg<BN>;
  const int64_t T = a.num_tokens, C = a.hidden;
  const size_t smem = static_cast<size_t>(Cfg::BYTES) + 1024;
  if (smem > static_cast<size_t>(dev.max_smem_optin))
    return fail(B200_ERR_UNSUPPORTED, "qkv projection: not enough shared memory");
  // One tile of at most 256 tokens: each CTA takes half of the tokens
  // (rounded up to 8 rows) so that neither stages more x rows than needed.
  const int rows = T <= 2 * kBM ? static_cast<int>(std::min<int64_t>(kBM, (ceil_div(T, 2) + 7) / 8 * 8))
                                : kBM;
  CUtensorMap tx, tw;
  int rc = encode_rows(&tx, a.x, T, C, a.x_row_stride, rows);
  if (rc == B200_OK) rc = encode_rows(&tw, a.weight, 3 * C, C, C, BN / 2);  // this CTA's half
  if (rc != B200_OK) return rc;
  static std::atomic<int> max_pairs[64];
  int pairs = dev.num_sms / 2;
  if (dev.device >= 0 && dev.device < 64) {
    if (max_pairs[dev.device].load(std::memory_order_acquire) == 0) {
      std::lock_guard<std::mutex> lock(g_setup_mu);
      cudaError_t e = cudaFuncSetAttribute(qkv_kv_write_pair_kernel<BN>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(qkv_kv_write_pair)");
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(dev.num_sms & ~1), 1, 1);
      cfg.blockDim = dim3(kThreads, 1, 1);
      cfg.dynamicSmemBytes = smem;
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, qkv_kv_write_pair_kernel<BN>, &cfg);
      if (e != cudaSuccess || n < 1) {
        (void)cudaGetLastError();
        n = dev.num_sms / 2;
      }
      max_pairs[dev.device].store(n, std::memory_order_release);
    }
    pairs = max_pairs[dev.device].load(std::memory_order_acquire);
  }
  QkvParams prm = make_params(a, 2 * kBM, BN, kBK);
  prm.x_rows = rows;
  const int64_t tiles = static_cast<int64_t>(prm.m_tiles) * prm.n_tiles;
  const int grid = 2 * static_cast<int>(std::min<int64_t>(tiles, pairs));
  qkv_kv_write_pair_kernel<BN><<<grid, kThreads, smem, stream>>>(tx, tw, prm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "qkv_kv_write_pair launch");
  return B200_OK;
}

// Clusters of `cluster` split-K CTAs that can be resident at once (cached).
int split_capacity(int cluster, const DeviceInfo& dev) {
  static std::atomic<int> cache[64][9];
  if (cluster == 1) return dev.num_sms;
  if (dev.device < 0 || dev.device >= 64 || cluster < 2 || cluster > 8) return 0;
  std::atomic<int>& slot = cache[dev.device][cluster];
  if (slot.load(std::memory_order_acquire) == 0) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    const size_t smem = static_cast<size_t>(kSplitBytes) + 1024;
    cudaError_t e = cudaFuncSetAttribute(qkv_kv_write_split_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    int n = 0;
    if (e == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = static_cast<unsigned>(cluster);
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.gridDim = dim3(static_cast<unsigned>(cluster * (dev.num_sms / cluster)), 1, 1);
      cfg.blockDim = dim3(kThreads, 1, 1);
      cfg.dynamicSmemBytes = smem;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      e = cudaOccupancyMaxActiveClusters(&n, qkv_kv_write_split_kernel, &cfg);
    }
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
    slot.store(n > 0 ? n : -1, std::memory_order_release);
  }
  const int cap = slot.load(std::memory_order_acquire);
  return cap > 0 ? cap : 0;
}

int launch_split(const b200_qkv_kv_write_args_t& a, cudaStream_t stream, const QkvPlan& plan,
                 const DeviceInfo& dev) {
  const int64_t T = a.num_tokens, C = a.hidden;
  const size_t smem = static_cast<size_t>(kSplitBytes) + 1024;
  static std::atomic<int> configured[64];
  if (dev.device >= 0 && dev.device < 64 && !configured[dev.device].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    cudaError_t e = cudaFuncSetAttribute(qkv_kv_write_split_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(qkv_kv_write_split)");
    configured[dev.device].store(1, std::memory_order_release);
  }
  SplitShape sh;
  sh.bn = plan.bn;
  sh.xrows = plan.xrows;
  // The M = 128 MMA reads 16 KB of A rows from each chunk's base, past the
  // chunk when the x box is short: the last stage's last A window must
  // still end inside the ring.
  sh.splits = plan.splits;
  if (sh.splits < 1 || sh.splits > kSplitMaxCluster || !split_fits(sh.xrows, sh.bn, sh.splits))
    return fail(B200_ERR_UNSUPPORTED, "qkv projection: split plan exceeds the reduction area");
  // Ring stages for a ring of ring_bytes; the receive slots go after the
  // ring when that costs it neither a stage nor its two-chunk stages.
  auto ring_stages = [&](int ring_bytes, int kc) {
    const int sb = kc * (sh.xrows + sh.bn) * 128;
    return std::min({kSplitMaxStages, ring_bytes / sb,
                     (ring_bytes - kBM * 128 - (kc - 1) * sh.xrows * 128) / sb + 1});
  };
  auto ring_shape = [&](int ring_bytes, int& kc, int& stages) {
    kc = ring_stages(ring_bytes, 2) >= 3 ? 2 : 1;
    stages = ring_stages(ring_bytes, kc);
  };
  int kc_full, stages_full, kc_short, stages_short;
  const int short_ring = kSplitAreaBytes - static_cast<int>(split_recv_bytes(sh.xrows, sh.bn, sh.splits));
  ring_shape(kSplitAreaBytes, kc_full, stages_full);
  ring_shape(short_ring, kc_short, stages_short);
  const bool after = sh.splits > 1 && kc_short == kc_full && stages_short == stages_full;
  sh.kc = after ? kc_short : kc_full;
  sh.stages = after ? stages_short : stages_full;
  sh.recv_off = after ? short_ring : 0;
  sh.stage_bytes = sh.kc * (sh.xrows + sh.bn) * 128;
  if (sh.stages < 2)
    return fail(B200_ERR_UNSUPPORTED, "qkv projection: split plan leaves too small an operand ring");
  CUtensorMap tx, tw;
  {
    // {64 columns, token rows, 64-column chunks}: the chunk dimension
    // steps 128 bytes along the row.
    const uint64_t dims[3] = {static_cast<uint64_t>(kBK), static_cast<uint64_t>(T),
                              static_cast<uint64_t>(C / kBK)};
    const uint64_t strides[2] = {static_cast<uint64_t>(a.x_row_stride * 2),
                                 static_cast<uint64_t>(kBK * 2)};
    const uint32_t box[3] = {static_cast<uint32_t>(kBK), static_cast<uint32_t>(sh.xrows),
                             static_cast<uint32_t>(sh.kc)};
    int rc = encode_tensor_map(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(a.x),
                               dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != B200_OK) return rc;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(kBK), static_cast<uint64_t>(3 * C),
                              static_cast<uint64_t>(C / kBK)};
    const uint64_t strides[2] = {static_cast<uint64_t>(C * 2), static_cast<uint64_t>(kBK * 2)};
    const uint32_t box[3] = {static_cast<uint32_t>(kBK), static_cast<uint32_t>(sh.bn),
                             static_cast<uint32_t>(sh.kc)};
    int rc = encode_tensor_map(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                               const_cast<void*>(a.weight), dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != B200_OK) return rc;
  }
  const QkvParams prm = make_params(a, kBM, sh.bn, sh.kc * kBK);  // k-steps of kc chunks
  sh.kpb = static_cast<int>(ceil_div(prm.k_iters, sh.splits));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(sh.splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(prm.m_tiles * prm.n_tiles * sh.splits), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, qkv_kv_write_split_kernel, tx, tw, prm, sh);
  if (e != cudaSuccess) return cuda_fail(e, "qkv_kv_write_split launch");
  return B200_OK;
}

}  // namespace

QkvPlan qkv_plan(int64_t T, int64_t C, const DeviceInfo& dev) {
  const int num_sms = dev.num_sms;
  const int64_t m_tiles = ceil_div(T, kBM);
  if (m_tiles <= 2 && T > 96) {
    // 97..256 tokens: a tile per CTA (128 x BN) or per CTA pair (256 x BN)
    // beats split-K clusters.  Measured with every call on another layer's
    // weights (CUDA graphs, one B200):
    //  - hidden 4096: 104-128 tokens take 24.2-24.3 us on 128-wide single
    //    CTAs against 24.6-25.5 us split-K (96 tokens: level), and 256
    //    tokens 27.0 us on 192-wide pairs against 33 us;
    //  - hidden 2048: 128 tokens take 11.9 us on 64-wide single CTAs (96
    //    CTAs) against 12.8 us on 128-wide ones (48), and 192-256 tokens 13.0
    //    us on 128-wide single CTAs (96) against 14.4 us on 192-wide pairs
    //    (64 CTAs): with the tiles in one wave, more CTAs win;
    //  - hidden 8192, 129-256 tokens: no layout fits one wave; persistent
    //    192-wide pairs take 88-93 us, 256-wide ones 96-100 us and 128-wide
    //    single CTAs 104-112 us.
    const int64_t single64 = m_tiles * ceil_div(3 * C, 64);
    const int64_t single128 = m_tiles * ceil_div(3 * C, 128);
    const int64_t pairs192 = ceil_div(3 * C, kPairBNNarrow);
    if (m_tiles == 1) {
      if (single64 <= num_sms) return {QkvPlan::kSingle, 64, 1, kBM};
      if (single128 <= num_sms) return {QkvPlan::kSingle, 128, 1, kBM};
    } else {
      if (single128 <= num_sms && single128 > 2 * pairs192) return {QkvPlan::kSingle, 128, 1, kBM};
      if (pairs192 <= num_sms / 2) return {QkvPlan::kPair, kPairBNNarrow, 1, kBM};
      if (ceil_div(3 * C, kPairBN) <= num_sms / 2) return {QkvPlan::kPair, kPairBN, 1, kBM};
      return {QkvPlan::kPair, kPairBNNarrow, 1, kBM};
    }
  }
  if (m_tiles <= 2) {
    // Few tokens (decode): the weights dominate and are read once, at a
    // per-SM rate that TMA caps.  Pick the tile width and reduction split
    // that stage the fewest bytes per CTA with every CTA resident at once
    // (splits keep >= 8 chunks each).  Each split past the first also costs
    // its exchange and a shorter pipeline, counted as 6 x-rows per live row
    // block: at hidden 2048, 96-wide tiles over 2 splits take 10.0-10.9 us
    // at 1-96 tokens against 11.0-14.2 us for 192-wide tiles over 4.
    const int64_t k_iters = C / kBK;
    const int xrows = m_tiles == 1 ? static_cast<int>((T + 7) / 8 * 8) : kBM;
    QkvPlan best{QkvPlan::kSplit, 0, 0, 0};
    int64_t best_cost = -1;
    for (int bn = kSplitMaxBN; bn >= 32; bn -= 16) {
      const int64_t tiles = m_tiles * ceil_div(3 * C, bn);
      for (int s = 1; s <= 8; ++s) {
        if (tiles * s > num_sms || (s > 1 && k_iters / s < 8)) continue;
        if (!split_fits(xrows, bn, s)) continue;
        if (s > 1 && tiles > split_capacity(s, dev)) continue;
        const int64_t cost = ceil_div(k_iters, s) * (xrows + bn) + (s - 1) * 6 * xrows;
        if (best_cost < 0 || cost < best_cost) {
          best = {QkvPlan::kSplit, bn, s, xrows};
          best_cost = cost;
        }
      }
    }
    if (best_cost >= 0) return best;
    // More 32-wide tiles than SMs: one 128-wide tile per CTA, several waves.
    return {QkvPlan::kSingle, 128, 1, kBM};
  }
  // Otherwise: fewest shared-memory-bound clocks per SM, counting the
  // partial last wave; CTA pairs (256 x 256 tiles) unless a single-CTA
  // tile width is cheaper.
  const int cand[2] = {128, 64};
  QkvPlan best{QkvPlan::kPair, kPairBN, 1, kBM};
  int64_t best_cost = ceil_div(ceil_div(T, 2 * kBM) * ceil_div(3 * C, kPairBN), num_sms / 2) *
                      kPairStepClocks;
  for (int bn : cand) {
    const int64_t tiles = m_tiles * ceil_div(3 * C, bn);
    const int64_t cost = ceil_div(tiles, num_sms) * step_clocks(bn);
    // On a tie the single-CTA tiles win: their last wave is fuller (384
    // tokens at hidden 4096: 42.9 us against 51.4 us on CTA pairs).
    if (cost <= best_cost) {
      best = {QkvPlan::kSingle, bn, 1, kBM};
      best_cost = cost;
    }
  }
  return best;
}

int launch_qkv_kv_write(const b200_qkv_kv_write_args_t& a, cudaStream_t stream) {
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc != B200_OK) return rc;
  const QkvPlan plan = qkv_plan(a.num_tokens, a.hidden, dev);
  if (plan.kind == QkvPlan::kPair)
    return plan.bn == kPairBNNarrow ? launch_pair<kPairBNNarrow>(a, stream, dev)
                                    : launch_pair<kPairBN>(a, stream, dev);
  if (plan.kind == QkvPlan::kSplit) return launch_split(a, stream, plan, dev);
  switch (plan.bn) {
    case 128:
      return launch_bn<128>(a, stream, dev);
    default:
      return launch_bn<64>(a, stream, dev);
  }
}

}  // namespace b200
