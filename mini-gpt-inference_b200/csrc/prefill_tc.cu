// prefill_tc.cu -- prefix-aware chunked-prefill attention on tcgen05 tensor
// cores (bf16 KV pool, head_dim 64 or 128, block size >= 8).
//
// One CTA per (sequence, head, pair of 128-query tiles).  Query i of a chunk
// sits at absolute position prefix_len + i and attends to keys
// 0 .. prefix_len + i (minivllm/attention.py:256-265), all read from the
// paged pool.  The two query tiles share every K/V tile and ping-pong on the
// tensor core: while one softmax group works on its scores, the MMAs of the
// other group run.
//
// Key tiles are BN = 64 (two S buffers per query tile, so S(k+1) is computed
// while the softmax works on S(k)) or BN = 128 (one S buffer; launches of
// single-tile chunks, where a CTA's two softmax groups split the keys).
//
// Warp roles (12 warps):
//   warps 0, 10  TMA producers of K and V: for each key tile they walk the
//            block table and load, per KV block, boxes {64 d, 1 head, rbox
//            rows} with 128-byte swizzle into this CTA's K ring and V ring;
//            warp 0 also loads the Q tiles.
//   warp 1   TMEM allocation (512 columns) and the S issuer (whole warp, one
//            elected lane issues): S_w = Q_w K^T (M=128, N=BN) into the
//            group's S buffer; it releases K stages.
//   warp 11  the P.V issuer: O_w += P_w V (M=128, N=D), P read from TMEM as
//            the A operand; it releases V stages.  Q, K and P are K-major
//            SW128 operands; V is read MN-major.
//   warps 2-5, 6-9  softmax / correction / epilogue of query tile 0 / 1:
//            thread r of a group owns query row r = TMEM lane r: pass 1
//            reads its S row and takes the masked max, pass 2 writes the
//            bf16 probabilities over the S columns; the running max is kept
//            unless it grows by more than 2^8 (lazy rescale of O in TMEM).
// V rows beyond the last valid key of the last tile are zeroed in smem
// before the P.V MMA: unwritten pool rows can hold NaN and 0 * NaN is NaN
// inside the tensor core as well (minivllm/paged_attention_batch.py:234-240).
// Launches of few CTAs (one sequence's chunk) may split each query pair's
// keys over CTAs (blockIdx.z): each writes its unnormalised rows with their
// max and sum to the caller's workspace, and the last CTA to arrive, found
// by an atomic counter (no spin-wait), combines them.
// Every mbarrier wait is bounded; on a timeout the CTA reports
// B200_DEV_WAIT_TIMEOUT, waits for its own MMAs and copies, frees TMEM and
// exits.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "host_util.h"
#include "kernels.h"
#include "tcgen05.cuh"

namespace b200 {
namespace {

constexpr int kMaxSeqs = 64;   // sequences per launch (host splits larger batches)
constexpr int kMaxWork = 2048; // (sequence, query pair) items per launch
constexpr int kThreads = 384;  // K producer, S issuer, two 4-warp softmax groups, V producer, P.V issuer
constexpr int kBM = 128;       // queries per query tile (two tiles per CTA)
// Key-tile configurations.  BN = 64: S is double-buffered per query tile
// (the MMAs of tile k+1 run during the softmax of tile k); used when the
// launch has 256-query CTAs.  BN = 128: one S buffer, twice the keys per
// barrier round trip and TMA burst; used when every CTA has a single query
// tile (short chunks), where per-tile overheads dominate.
template <int BN> struct TileCfg;
template <> struct TileCfg<64> {
  static constexpr int KS = 5, VS = 4, NBUF = 2;  // K / V ring depths, S buffers
};
template <> struct TileCfg<128> {
  static constexpr int KS = 3, VS = 2, NBUF = 1;
};

struct SeqDesc {
  const void* q;
  void* out;
  const void* table;
  int64_t qs0, qs1, qs2;
  int64_t os0, os1, os2;
  int64_t ts;
  int32_t prefix;
  int32_t T;
  int32_t table_len;
  int32_t pad;
};

struct PrefillParams {
  CUtensorMap qmap[kMaxSeqs];  // per-sequence Q maps (valid when q_tma)
  int64_t P, S, H, D;
  int64_t layer;
  int32_t q_dtype, out_dtype, table_i64;
  int32_t q_vec, out_vec;  // 16-byte row access is legal for every sequence
  int32_t q_tma;           // every sequence's q is bf16 and TMA-addressable
  int32_t rbox, rb_shift, s_shift;
  int32_t nseq;
  int32_t max_qtiles;
  int32_t* status;
  float scale_log2;
  // Key split (ksplits > 1): CTA z of (item, head) covers the z-th of
  // ksplits equal ranges of the item's key tiles and writes its unnormalised
  // O rows with their (max, sum) to `part`; the last CTA to arrive (count)
  // combines them.  part: [item][H][ksplits][D + 2][2 * kBM rows] fp32 (O
  // by feature, then the row max and sum: a warp's 32 rows are contiguous);
  // count: [item][H], zeroed before the launch.
  int32_t ksplits;
  float* part;
  int32_t* count;
  SeqDesc seq[kMaxSeqs];
  // Work items, longest first: sequence | query pair << 8.  blockIdx.y picks
  // one, blockIdx.x is the head, so the CTAs with the most key tiles start
  // first and the short ones fill the tail of the launch.
  uint32_t work[kMaxWork];
};
// Kernel parameters (two K/V maps + this struct) stay under the 32764-byte limit.
static_assert(sizeof(PrefillParams) + 2 * sizeof(CUtensorMap) <= 32764, "kernel parameters too large");

// Hardware base-2 exponential (MUFU), flushing denormal results to zero.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (three-input max, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Byte offset of 16-byte chunk `ch` (0..7) of row `r` in a 128-byte-swizzled
// tile of 128-byte rows.
__device__ __forceinline__ uint32_t sw128(int r, int ch) {
  return static_cast<uint32_t>(r) * 128u + (static_cast<uint32_t>(ch ^ (r & 7)) << 4);
}

// Pass 2 of the softmax for this thread's S row (128 columns in TMEM at
// `srow`): p = 2^(s * scale - m) for keys c <= lim (all keys when !MASK),
// written as bf16 pairs over the S columns already read (chunk [c, c+32) ->
// P columns [c/2, c/2 + 16)).  The next 32-column chunk is loaded while the
// current one is computed.  Returns the row sum of p.
template <bool MASK, int kBN>
__device__ __forceinline__ float p_pass(uint32_t srow, float scale, float neg_m, int lim) {
  const float2 sc2 = make_float2(scale, scale);
  const float2 nm2 = make_float2(neg_m, neg_m);
  const float2 one2 = make_float2(1.f, 1.f);
  float2 rs[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                  make_float2(0.f, 0.f)};
  float sv[2][32];
  tmem_ld32(srow, sv[0]);
  tmem_wait_ld();
#pragma unroll
  for (int c = 0; c < kBN; c += 32) {
    const int cur = (c >> 5) & 1;
    if (c + 32 < kBN) tmem_ld32(srow + c + 32, sv[cur ^ 1]);
    uint32_t pk[16];
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
      const float2 a = ffma2(make_float2(sv[cur][e], sv[cur][e + 1]), sc2, nm2);
      float p0 = ex2_approx(a.x);
      float p1 = ex2_approx(a.y);
      if (MASK) {
        p0 = c + e <= lim ? p0 : 0.f;
        p1 = c + e + 1 <= lim ? p1 : 0.f;
      }
      rs[(e >> 1) & 3] = ffma2(make_float2(p0, p1), one2, rs[(e >> 1) & 3]);
      pk[e >> 1] = pack_bf16(p0, p1);
    }
    tmem_st16(srow + (c >> 1), pk);
    if (c + 32 < kBN) tmem_wait_ld();
  }
  return ((rs[0].x + rs[0].y) + (rs[1].x + rs[1].y)) + ((rs[2].x + rs[2].y) + (rs[3].x + rs[3].y));
}

// Pass 2 from the S row already in registers (sv, loaded by pass 1): the
// same probabilities and P stores as p_pass without re-reading TMEM.  Used
// with 64-key tiles, whose row costs 64 registers.
template <bool MASK, int kBN>
__device__ __forceinline__ float p_regs(const float* sv, uint32_t srow, float scale, float neg_m,
                                        int lim) {
  const float2 sc2 = make_float2(scale, scale);
  const float2 nm2 = make_float2(neg_m, neg_m);
  const float2 one2 = make_float2(1.f, 1.f);
  float2 rs[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                  make_float2(0.f, 0.f)};
#pragma unroll
  for (int c = 0; c < kBN; c += 32) {
    uint32_t pk[16];
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
      const float2 a = ffma2(make_float2(sv[c + e], sv[c + e + 1]), sc2, nm2);
      float p0 = ex2_approx(a.x);
      float p1 = ex2_approx(a.y);
      if (MASK) {
        p0 = c + e <= lim ? p0 : 0.f;
        p1 = c + e + 1 <= lim ? p1 : 0.f;
      }
      rs[(e >> 1) & 3] = ffma2(make_float2(p0, p1), one2, rs[(e >> 1) & 3]);
      pk[e >> 1] = pack_bf16(p0, p1);
    }
    tmem_st16(srow + (c >> 1), pk);
  }
  return ((rs[0].x + rs[0].y) + (rs[1].x + rs[1].y)) + ((rs[2].x + rs[2].y) + (rs[3].x + rs[3].y));
}

// Shared-memory layout (offsets from a 1024-aligned base).
template <int D, int kBN>
struct Smem {
  static constexpr int kKStages = TileCfg<kBN>::KS;
  static constexpr int kVStages = TileCfg<kBN>::VS;
  static constexpr int HALVES = D / 64;               // 64-element (128-byte) column halves
  static constexpr int QHALF = kBM * 128;             // one column half of a Q tile
  static constexpr int QTILE = HALVES * QHALF;        // a 128-query tile
  static constexpr int KVHALF = kBN * 128;            // one column half of a K/V tile
  static constexpr int KVTILE = HALVES * KVHALF;      // a 64-key tile
  static constexpr int Q0 = 0;                        // Q tiles 0 and 1
  static constexpr int K0 = Q0 + 2 * QTILE;           // K ring
  static constexpr int V0 = K0 + kKStages * KVTILE;   // V ring
  static constexpr int BAR = V0 + kVStages * KVTILE;
  static constexpr int BYTES = BAR + 512;
};

// Loads query row i (zeros past T) of head h into row r of a swizzled Q tile.
template <int D>
__device__ __forceinline__ void load_q_row(uint8_t* tile, int r, int i, int h, const SeqDesc& sd,
                                           int q_dtype, int q_vec) {
  constexpr int HALVES = D / 64;
#pragma unroll
  for (int half = 0; half < HALVES; ++half) {
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      const int d0 = half * 64 + ch * 8;
      uint4 w = make_uint4(0, 0, 0, 0);
      if (i < sd.T) {
        const int64_t off = i * sd.qs0 + h * sd.qs1 + d0 * sd.qs2;
        if (q_vec && q_dtype == B200_DTYPE_BF16) {
          w = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(sd.q) + off);
        } else if (q_vec && q_dtype == B200_DTYPE_F32) {
          const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(sd.q) + off);
          const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(sd.q) + off + 4);
          w = make_uint4(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w), pack_bf16(b.x, b.y),
                         pack_bf16(b.z, b.w));
        } else {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = load_elem(sd.q, off + e * sd.qs2, q_dtype);
          w = make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]),
                         pack_bf16(f[6], f[7]));
        }
      }
      *reinterpret_cast<uint4*>(tile + half * 16384 + sw128(r, ch)) = w;
    }
  }
}

// Key tiles [*j0, return value) that key split z of `splits` covers for
// query tile w of the query pair starting at i0 (empty when j0 >= the
// returned end): the pair's key tiles (those of its last query) are cut into
// `splits` equal ranges, and each tile's own causal end clips them.
__device__ __forceinline__ int key_split_range(const SeqDesc& sd, int i0, int w, int bn, int splits,
                                               int z, int* j0) {
  const int lo = i0 + w * kBM;
  const int full = lo < sd.T ? static_cast<int>((sd.prefix + min(sd.T, lo + kBM) + bn - 1) / bn) : 0;
  if (splits <= 1) {
    *j0 = 0;
    return full;
  }
  const int last = static_cast<int>((sd.prefix + min(sd.T, i0 + 2 * kBM) + bn - 1) / bn);
  const int per = (last + splits - 1) / splits;
  *j0 = z * per;
  return max(*j0, min(full, *j0 + per));
}

// Per-CTA bookkeeping shared by the roles.
struct Geom {
  int i0;          // first query of the CTA
  int j0;          // first key tile of the CTA's range (key split), else 0
  int nkt[2];      // key tiles of query tile 0 / 1 (0 = tile inactive)
  int nmax;        // max(nkt): key tiles streamed through the rings
  int64_t total;   // keys any query of the CTA may see
  // Key split: with one query tile (and >= 2 key tiles) both softmax groups
  // work on it, group w taking key tiles w, w+2, w+4, ... with its own O,
  // max and sum; group 0 merges the two at the end.
  bool split;
  int cnt[2];      // key tiles group w processes
  __device__ int tile(int w, int k) const { return split ? 2 * k + w : k; }
  __device__ int qtile(int w) const { return split ? 0 : w; }
  // The last group whose S or P.V reads key tile j (releases its stages).
  __device__ int last_user(int j) const { return split ? (j & 1) : (j < nkt[1] ? 1 : 0); }
};

template <int D, int kBN>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const __grid_constant__ PrefillParams p) {
  using L = Smem<D, kBN>;
  constexpr int kKStages = TileCfg<kBN>::KS;
  constexpr int kVStages = TileCfg<kBN>::VS;
  constexpr int kNBuf = TileCfg<kBN>::NBUF;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t item = p.work[blockIdx.y];
  const int seq = static_cast<int>(item & 0xFFu);
  const int qp = static_cast<int>(item >> 8);
  const int h = blockIdx.x;
  const SeqDesc& sd = p.seq[seq];
  Geom g;
  g.i0 = qp * 2 * kBM;
  if (g.i0 >= sd.T) return;
  const int64_t prefix = sd.prefix;
  const int ksplit = static_cast<int>(blockIdx.z);
  // Key tiles of query tile w (all keys up to its last query), clipped to
  // this CTA's range under a key split; tile indices below stay relative to
  // the range (ring stages and barrier phases start afresh in every CTA) and
  // key positions add g.j0 back.
  g.j0 = 0;
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    const int j1 = key_split_range(sd, g.i0, w, kBN, p.ksplits, ksplit, &g.j0);
    g.nkt[w] = j1 - g.j0;
  }
  g.nmax = max(g.nkt[0], g.nkt[1]);
  g.total = prefix + min(sd.T, g.i0 + 2 * kBM);
  g.split = g.nkt[1] == 0 && g.nkt[0] >= 2;
  g.cnt[0] = g.split ? (g.nkt[0] + 1) / 2 : g.nkt[0];
  g.cnt[1] = g.split ? g.nkt[0] / 2 : g.nkt[1];

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint64_t* k_full = bars;                      // [kKStages]
  uint64_t* k_empty = k_full + kKStages;        // [kKStages]
  uint64_t* v_full = k_empty + kKStages;        // [kVStages]
  uint64_t* v_empty = v_full + kVStages;        // [kVStages]
  // Per group w and tile parity b = k & 1 (index 2w + b): S(k) complete, P(k)
  // written, P.V(k) complete.  A barrier of parity b completes once every
  // other tile, and tile k+2 of a group cannot reach it before P.V(k) has
  // been issued, so no waiter is ever two phases behind: every wait's parity
  // is unambiguous even when some phases are never waited for.
  uint64_t* s_full = v_empty + kVStages;        // [2 groups][2]
  uint64_t* p_full = s_full + 4;                // [2 groups][2]
  uint64_t* o_done = p_full + 4;                // [2 groups][2]
  uint64_t* mma_idle = o_done + 4;              // [2]: S issuer, P.V issuer
  uint64_t* q_full = mma_idle + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_full + 1);
  int32_t* abort_flag = reinterpret_cast<int32_t*>(q_full + 2);
  static_assert((2 * kKStages + 2 * kVStages + 17) * 8 <= 512, "barrier area too small");

  if (threadIdx.x == 0) {
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 4; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 128);
      mbar_init(&o_done[s], 1);
    }
    mbar_init(&mma_idle[0], 1);
    mbar_init(&mma_idle[1], 1);
    mbar_init(q_full, p.q_tma ? 1 : 256);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // Q tiles: softmax group w loads query tile w; row r of a 128-row tile is
  // TMEM lane r, and a warp may only touch lanes [32*(warp%4), +32), so rows
  // follow (warp % 4, lane).
  const int wg = (warp >= 2 && warp < 10) ? (warp - 2) >> 2 : -1;  // softmax group
  const int r = (warp & 3) * 32 + lane;             // row within the group's tile
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Q tiles: by TMA from the K producer (zero-filled past T), else loaded
  // here by the softmax threads; either way the MMA issuer waits on q_full,
  // and K/V prefetch starts at once.
  if (!p.q_tma && wg >= 0) {
    load_q_row<D>(smem + L::Q0 + wg * L::QTILE, r, g.i0 + wg * kBM + r, h, sd, p.q_dtype, p.q_vec);
    fence_proxy_async_shared();
    mbar_arrive(q_full);
  }
  const uint32_t tmem = *tmem_slot;
  // TMEM columns.  kBN = 64: group w has S buffers [256w, +64) and
  // [256w+64, +64) and O [256w+128, +D).  kBN = 128: S_w [128w, +128),
  // O_w [256+128w, +D).
  auto tmem_s = [&](int w, int b) {
    return tmem + static_cast<uint32_t>(kNBuf == 2 ? w * 256 + b * 64 : w * 128);
  };
  auto tmem_o = [&](int w) {
    return tmem + static_cast<uint32_t>(kNBuf == 2 ? w * 256 + 128 : 256 + w * 128);
  };

  if (warp == 0 || warp == 10) {
    // ------------------------------------------------------------ producers
    // Warp 0 streams K, warp 10 streams V, each through its own ring.  Every
    // lane issues TMA boxes: a tile is (keys/rbox blocks) x (D/64 column
    // halves) small boxes, and spreading their issue over the warp keeps the
    // copy engine fed.
    const bool is_k = warp == 0;
    const int NS = is_k ? kKStages : kVStages;
    uint64_t* full = is_k ? k_full : v_full;
    uint64_t* empty = is_k ? k_empty : v_empty;
    uint8_t* ring = smem + (is_k ? L::K0 : L::V0);
    const CUtensorMap* map = is_k ? &tmk : &tmv;
    const int box_bytes = 64 * p.rbox * 2;
    const int boxes_per_tile = kBN / p.rbox;
    if (is_k && p.q_tma && lane == 0) {
      const int ntiles = g.nkt[1] > 0 ? 2 : 1;
      mbar_arrive_expect_tx(q_full, static_cast<uint32_t>(ntiles * L::HALVES * kBM * 128));
      for (int w = 0; w < ntiles; ++w)
        for (int half = 0; half < L::HALVES; ++half)
          tma_load_3d(smem + L::Q0 + w * L::QTILE + half * L::QHALF, &p.qmap[seq], q_full, half * 64,
                      h, g.i0 + w * kBM);
    }
    // A tile has at most 16 boxes (rbox >= 8, two column halves), so each
    // lane issues at most one: lane -> (block b, half).
    const int b = lane / L::HALVES;
    const int half = lane % L::HALVES;
    int issued = 0;
    // Block-table entries are read one tile ahead: the load for tile j+1 is
    // issued before tile j's slot wait, and an entry is checked only when it
    // is used, so the load's latency overlaps the wait and the copies.
    auto boxes = [&](int j) {
      return static_cast<int>(min(static_cast<int64_t>(boxes_per_tile),
                                  (g.total - static_cast<int64_t>(g.j0 + j) * kBN + p.rbox - 1) >> p.rb_shift));
    };
    auto entry = [&](int j) -> int64_t {
      if (j >= g.nmax || lane >= boxes(j) * L::HALVES) return 0;
      const int64_t blk = (static_cast<int64_t>(g.j0 + j) * kBN + (static_cast<int64_t>(b) << p.rb_shift)) >> p.s_shift;
      return blk < sd.table_len ? load_index(sd.table, blk * sd.ts, p.table_i64) : -1;
    };
    int64_t raw_next = entry(0);
    for (int j = 0; j < g.nmax; ++j) {
      const int st = j % NS;
      const uint32_t use = static_cast<uint32_t>(j / NS);
      const int64_t key0 = static_cast<int64_t>(g.j0 + j) * kBN;
      const int nb = boxes(j);
      const bool mine = lane < nb * L::HALVES;
      const int64_t key = key0 + (static_cast<int64_t>(b) << p.rb_shift);
      const int64_t raw = raw_next;
      raw_next = entry(j + 1);
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&empty[st], (use & 1u) ^ 1u) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok || *reinterpret_cast<volatile int32_t*>(abort_flag)) {
        if (lane == 0 && !ok) {
          report(p.status, B200_DEV_WAIT_TIMEOUT);
          *abort_flag = 1;
        }
        break;
      }
      if (lane == 0)
        mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(nb * L::HALVES * box_bytes));
      __syncwarp();
      int64_t phys = raw;
      if (mine && (phys < 0 || phys >= p.P)) {
        report(p.status, B200_DEV_BAD_BLOCK);
        phys = 0;
      }
      if (mine) {
        uint8_t* dst = ring + st * L::KVTILE;
        const int32_t row = static_cast<int32_t>((p.layer * p.P + phys) * p.S + (key & (p.S - 1)));
        tma_load_3d(dst + half * L::KVHALF + b * p.rbox * 128, map, &full[st], half * 64, h, row);
      }
      ++issued;
    }
    if (lane == 0) {
      const int first = issued > NS ? issued - NS : 0;
      for (int j = first; j < issued; ++j)
        if (!mbar_wait(&full[j % NS], static_cast<uint32_t>(j / NS) & 1u)) {
          report(p.status, B200_DEV_WAIT_TIMEOUT);
          break;
        }
      if (is_k && p.q_tma && !mbar_wait(q_full, 0)) report(p.status, B200_DEV_WAIT_TIMEOUT);
    }
  } else if (warp == 1 || warp == 11) {
    // ------------------------------------------------------------ MMA issuers
    // Warp 1 issues every S (and releases K stages), warp 11 every P.V (and
    // releases V stages), so that one issuer's barrier waits and commits
    // overlap the other's MMAs.  Each runs its loop as a whole warp (values
    // stay warp-uniform); every lane waits on the barriers itself and a vote
    // makes the outcome uniform; elect.sync picks the issuing lane.
    auto wait_all = [&](uint64_t* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity)) != 0;
    };
    bool ok = true;
    // Descriptors of the tile bases; a step's descriptor adds its byte
    // offset / 16 to the 14-bit address field (no carry: smem < 256 KB).
    if (warp == 1) {
      constexpr uint32_t idesc_s = idesc_bf16(128, kBN, false);
      const uint64_t dq0 = smem_desc_sw128(smem_u32(smem + L::Q0), 16, 1024);
      const uint64_t dk0 = smem_desc_sw128(smem_u32(smem + L::K0), 16, 1024);
      // S of group w's k-th key tile, into its S buffer k % kNBuf.
      auto issue_s = [&](int w, int k) -> bool {
        const int j = g.tile(w, k);
        const int st = j % kKStages;
        if (!wait_all(&k_full[st], static_cast<uint32_t>(j / kKStages) & 1u)) return false;
        tc_fence_after();
        const uint64_t dq = dq0 + static_cast<uint64_t>(g.qtile(w) * (L::QTILE >> 4));
        const uint64_t dk = dk0 + static_cast<uint64_t>(st * (L::KVTILE >> 4));
        const uint32_t ts = tmem_s(w, k % kNBuf);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t qoff = static_cast<uint64_t>(((kk >> 2) * L::QHALF + (kk & 3) * 32) >> 4);
          const uint64_t koff = static_cast<uint64_t>(((kk >> 2) * L::KVHALF + (kk & 3) * 32) >> 4);
          mma_bf16(ts, dq + qoff, dk + koff, idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[w * 2 + (k & 1)]);
        // The last S MMA of tile j releases its K stage.
        if (w == g.last_user(j)) mma_commit(&k_empty[st]);
        return true;
      };
      // Each group's first kNBuf S (all its S buffers) go out at once.  S(k)
      // for k >= kNBuf overwrites P(k - kNBuf), so it waits for that P.V to
      // complete (every o_done phase is waited for here, in order).  With two
      // buffers the softmax of tile k+1 never waits for the MMAs of tile k.
      ok = wait_all(q_full, 0);
      for (int k = 0; k < kNBuf; ++k)
        for (int w = 0; w < 2; ++w)
          if (ok && k < g.cnt[w]) ok = issue_s(w, k);
      const int rounds = max(g.cnt[0], g.cnt[1]);
      for (int k = kNBuf; ok && k < rounds; ++k) {
        for (int w = 0; ok && w < 2; ++w) {
          if (k >= g.cnt[w]) continue;
          const int kp = k - kNBuf;
          if (!wait_all(&o_done[w * 2 + (kp & 1)], static_cast<uint32_t>(kp >> 1) & 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (!issue_s(w, k)) ok = false;
        }
      }
    } else {
      constexpr uint32_t idesc_o = idesc_bf16(128, D, true);
      const uint64_t dv0 = smem_desc_sw128(smem_u32(smem + L::V0), L::KVHALF, 1024);
      int v_ready = -1;  // the last key tile whose V has been waited for
      const int rounds = max(g.cnt[0], g.cnt[1]);
      for (int k = 0; ok && k < rounds; ++k) {
        for (int w = 0; ok && w < 2; ++w) {
          if (k >= g.cnt[w]) continue;
          const int j = g.tile(w, k);
          const int vst = j % kVStages;
          const uint64_t dv = dv0 + static_cast<uint64_t>(vst * (L::KVTILE >> 4));
          if (!wait_all(&p_full[w * 2 + (k & 1)], static_cast<uint32_t>(k >> 1) & 1u)) {
            ok = false;
            break;
          }
          if (v_ready != j && !wait_all(&v_full[vst], static_cast<uint32_t>(j / kVStages) & 1u)) {
            ok = false;
            break;
          }
          v_ready = j;
          tc_fence_after();
          // P (bf16 pairs over S_w's first columns) is the TMEM A operand;
          // 16 keys per step = 8 columns.
          const uint32_t to = tmem_o(w), ts = tmem_s(w, k % kNBuf);
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk)
            mma_bf16_ts(to, ts + kk * 8, dv + static_cast<uint64_t>(kk * 128), idesc_o,
                        (k > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&o_done[w * 2 + (k & 1)]);
          // The tile's last P.V releases its V stage.
          if (w == g.last_user(j)) mma_commit(&v_empty[vst]);
        }
      }
    }
    if (!ok && lane == 0) {
      report(p.status, B200_DEV_WAIT_TIMEOUT);
      *abort_flag = 1;
    }
    // Wait until every MMA this warp issued has completed.
    uint64_t* idle = &mma_idle[warp == 1 ? 0 : 1];
    mma_commit(idle);
    if (!wait_all(idle, 0) && lane == 0) report(p.status, B200_DEV_WAIT_TIMEOUT);
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int w = wg;
    const int qt = g.qtile(w);                         // this group's query tile
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int iq = g.i0 + qt * kBM + r;                // this thread's query
    const int i = min(iq, sd.T - 1);                   // rows past T mirror the last query
    const int64_t qpos = prefix + i;
    // A warp whose 32 rows are all past T has nothing to compute (its rows of
    // P and O are never used); it only keeps the barrier protocol.
    const bool warp_live = g.i0 + qt * kBM + (warp & 3) * 32 < sd.T;
    const int nk = g.cnt[w];
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int k = 0; k < nk; ++k) {
      const int j = g.tile(w, k);
      const int sb = k & 1;          // barrier parity of this tile
      const int buf = k % kNBuf;     // S buffer of this tile
      if (!mbar_wait(&s_full[w * 2 + sb], static_cast<uint32_t>(k >> 1) & 1u)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int64_t key0 = static_cast<int64_t>(g.j0 + j) * kBN;
      const bool need_mask = key0 + kBN - 1 > prefix + g.i0 + qt * kBM;  // some key may be masked
      float alpha = 1.f, m_use = m;
      bool rescale = false;
      // Keys c <= lim of this tile are visible to this row (int32, clamped).
      const int lim = static_cast<int>(max(min(qpos - key0, static_cast<int64_t>(kBN - 1)),
                                           static_cast<int64_t>(-1)));
      float sv[kBN];  // the S row (kept for pass 2 with 64-key tiles)
      if (warp_live) {
        // Pass 1: row max of the masked raw scores (the scale is positive, so
        // it is applied once to the max).
        float mx;
        {
#pragma unroll
          for (int c = 0; c < kBN; c += 32) tmem_ld32(tmem_s(w, buf) + lane_base + c, sv + c);
          tmem_wait_ld();
          // Eight independent chains of three-input max, then a tree.
          float mp[8];
          if (need_mask) {
#pragma unroll
            for (int a = 0; a < 8; ++a)
              mp[a] = fmaxf(2 * a <= lim ? sv[2 * a] : -INFINITY,
                            2 * a + 1 <= lim ? sv[2 * a + 1] : -INFINITY);
#pragma unroll
            for (int e = 16; e < kBN; e += 16)
#pragma unroll
              for (int a = 0; a < 8; ++a)
                mp[a] = fmax3(mp[a], e + 2 * a <= lim ? sv[e + 2 * a] : -INFINITY,
                              e + 2 * a + 1 <= lim ? sv[e + 2 * a + 1] : -INFINITY);
          } else {
#pragma unroll
            for (int a = 0; a < 8; ++a) mp[a] = fmaxf(sv[2 * a], sv[2 * a + 1]);
#pragma unroll
            for (int e = 16; e < kBN; e += 16)
#pragma unroll
              for (int a = 0; a < 8; ++a) mp[a] = fmax3(mp[a], sv[e + 2 * a], sv[e + 2 * a + 1]);
          }
          mx = fmax3(fmax3(mp[0], mp[1], mp[2]), fmax3(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
        }
        mx *= p.scale_log2;
        // Lazy rescale: keep the old max unless the new one exceeds it by
        // more than 8 (probabilities then stay below 2^8, exact in fp32).
        if (mx > m + 8.f) m_use = mx;
        rescale = __any_sync(0xffffffffu, m_use != m) && k > 0;
        // (A row may see no key of its group's first tiles under the key
        // split: m stays -inf and alpha must stay 1.)
        alpha = m_use == m ? 1.f : ex2_approx(m - m_use);
      }
      if (warp_live) {
        // Pass 2: probabilities, written back as bf16 pairs over the S
        // columns already consumed; the masked variant is a separate
        // instantiation so unmasked tiles carry no per-element selects.
        const uint32_t srow = tmem_s(w, buf) + lane_base;
        float rsum;
        if (kBN == 64)  // the row is still in registers
          rsum = need_mask ? p_regs<true, kBN>(sv, srow, p.scale_log2, -m_use, lim)
                           : p_regs<false, kBN>(sv, srow, p.scale_log2, -m_use, lim);
        else
          rsum = need_mask ? p_pass<true, kBN>(srow, p.scale_log2, -m_use, lim)
                           : p_pass<false, kBN>(srow, p.scale_log2, -m_use, lim);
        l = l * alpha + rsum;
        m = m_use;
      }
      if (rescale) {
        // P.V(k-1) must have completed before O is rescaled (only then is
        // the softmax held back by the MMAs of an earlier tile).
        const int kp = k - 1;
        if (!mbar_wait(&o_done[w * 2 + (kp & 1)], static_cast<uint32_t>(kp >> 1) & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (warp_live) {
#pragma unroll
          for (int c = 0; c < D; c += 32) {
            float o[32];
            tmem_ld32(tmem_o(w) + lane_base + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= alpha;
            tmem_st32(tmem_o(w) + lane_base + c, o);
          }
        }
      }
      tmem_wait_st();
      // Zero V rows past the last valid key of the last tile (pool rows there
      // may be unwritten); the group issuing the tile's first P.V does it.
      const int64_t valid = g.total - key0;
      const int first_w = g.split ? (j & 1) : (j < g.nkt[0] ? 0 : 1);
      if (w == first_w && valid < kBN) {
        // V of this tile must have landed before its rows are cleared.
        if (!mbar_wait(&v_full[j % kVStages], static_cast<uint32_t>(j / kVStages) & 1u)) {
          ok = false;
          break;
        }
      }
      if (w == first_w && valid < kBN && r >= valid && r < kBN) {
        uint8_t* vrow = smem + L::V0 + (j % kVStages) * L::KVTILE + r * 128;
#pragma unroll
        for (int half = 0; half < L::HALVES; ++half)
#pragma unroll
          for (int ch = 0; ch < 8; ++ch)
            *reinterpret_cast<uint4*>(vrow + half * L::KVHALF + ((ch ^ (r & 7)) << 4)) =
                make_uint4(0, 0, 0, 0);
        fence_proxy_async_shared();
      }
      tc_fence_before();
      mbar_arrive(&p_full[w * 2 + sb]);
    }
    // The last P.V completing implies all earlier ones have (issue order).
    if (nk > 0 && ok &&
        !mbar_wait(&o_done[w * 2 + ((nk - 1) & 1)], static_cast<uint32_t>((nk - 1) >> 1) & 1u))
      ok = false;
    if (!ok) {
      if (r == 0) report(p.status, B200_DEV_WAIT_TIMEOUT);
      *abort_flag = 1;
    }
    // Row weights of the output: O_w / l in the two-query-tile case; under
    // the key split group 0 writes (O_0 2^(m_0-M) + O_1 2^(m_1-M)) /
    // (l_0 2^(m_0-M) + l_1 2^(m_1-M)), M = max(m_0, m_1).
    bool write = ok && nk > 0 && warp_live;
    float a_self = 1.f, a_other = 0.f, inv = 0.f, m_row = m, l_row = l;
    if (g.split) {
      // Group 1 hands its row max and sum over through its S columns, free
      // once its last P.V has completed; group 0's thread r reads the same
      // TMEM lane.  Both groups meet at named barrier 1 (256 threads).
      if (w == 1 && write) {
        tmem_st2(tmem_s(1, 0) + lane_base, __float_as_uint(m), __float_as_uint(l));
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      asm volatile("bar.sync 1, 256;" ::: "memory");
      tc_fence_after();
      write = write && w == 0 && *reinterpret_cast<volatile int32_t*>(abort_flag) == 0;
      if (write) {
        uint32_t mb, lb;
        tmem_ld2(tmem_s(1, 0) + lane_base, mb, lb);
        tmem_wait_ld();
        const float m1 = __uint_as_float(mb), l1 = __uint_as_float(lb);
        const float mm = fmaxf(m, m1);
        // (Under a key split over CTAs a row may see no key of this CTA's
        // range at all: mm = -inf, and the row's partial is empty.)
        a_self = m == -INFINITY ? 0.f : ex2_approx(m - mm);
        a_other = m1 == -INFINITY ? 0.f : ex2_approx(m1 - mm);
        m_row = mm;
        l_row = l * a_self + l1 * a_other;
        inv = 1.0f / l_row;
      }
    } else if (write) {
      inv = 1.0f / l;
    }
    if (p.ksplits > 1) {
      // Key split over CTAs: this CTA's unnormalised rows O (relative to the
      // row max m_row) with (m_row, l_row) go to its slot; the last CTA of
      // the (item, head) to arrive combines every split's rows.
      const int64_t slot0 = (static_cast<int64_t>(blockIdx.y) * p.H + h) * p.ksplits;
      constexpr int kRows = 2 * kBM;
      constexpr int64_t kSlot = static_cast<int64_t>(D + 2) * kRows;
      if (write) {
        tc_fence_after();
        float* prow = p.part + (slot0 + ksplit) * kSlot + qt * kBM + r;
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          float o[32];
          tmem_ld32(tmem_o(w) + lane_base + c, o);
          if (g.split) {
            float o1[32];
            tmem_ld32(tmem_o(1) + lane_base + c, o1);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = o[e] * a_self + o1[e] * a_other;
          } else {
            tmem_wait_ld();
          }
#pragma unroll
          for (int e = 0; e < 32; ++e) prow[(c + e) * kRows] = o[e];
        }
        prow[D * kRows] = m_row;
        prow[(D + 1) * kRows] = l_row;
      }
      // The ticket's outcome is shared through the word after the abort flag.
      volatile int32_t* last_cta = reinterpret_cast<volatile int32_t*>(abort_flag) + 1;
      __threadfence();
      asm volatile("bar.sync 2, 256;" ::: "memory");
      if (warp == 2 && lane == 0)
        *last_cta = atomicAdd(&p.count[static_cast<int64_t>(blockIdx.y) * p.H + h], 1) == p.ksplits - 1;
      asm volatile("bar.sync 2, 256;" ::: "memory");
      if (*last_cta) {
        __threadfence();
        // Thread r of group w combines row r of query tile w over the splits
        // whose range is not empty for that tile.
        const int t = w;
        const int iq_t = g.i0 + t * kBM + r;
        if (iq_t < sd.T) {
          auto row = [&](int z) { return p.part + (slot0 + z) * kSlot + t * kBM + r; };
          // Splits whose range is empty for this tile wrote nothing for it.
          uint32_t live_z = 0;
          for (int z = 0; z < p.ksplits; ++z) {
            int zj0;
            if (key_split_range(sd, g.i0, t, kBN, p.ksplits, z, &zj0) > zj0) live_z |= 1u << z;
          }
          float M = -INFINITY;
          for (uint32_t zs = live_z; zs; zs &= zs - 1) M = fmaxf(M, __ldcg(row(__ffs(zs) - 1) + D * kRows));
          float L = 0.f;
          for (uint32_t zs = live_z; zs; zs &= zs - 1) {
            const float* src = row(__ffs(zs) - 1);
            const float mz = __ldcg(src + D * kRows);
            if (mz != -INFINITY) L += ex2_approx(mz - M) * __ldcg(src + (D + 1) * kRows);
          }
          const float linv = 1.0f / L;
          const bool vec = p.out_vec && p.out_dtype == B200_DTYPE_BF16;
#pragma unroll 1
          for (int c = 0; c < D; c += 32) {
            float o[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = 0.f;
            for (uint32_t zs = live_z; zs; zs &= zs - 1) {
              const float* src = row(__ffs(zs) - 1);
              const float mz = __ldcg(src + D * kRows);
              if (mz == -INFINITY) continue;
              const float f = ex2_approx(mz - M) * linv;
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] += f * __ldcg(src + (c + e) * kRows);
            }
            const int64_t base = iq_t * sd.os0 + h * sd.os1 + c * sd.os2;
            if (vec) {
#pragma unroll
              for (int e = 0; e < 32; e += 8) {
                const uint4 wv = make_uint4(pack_bf16(o[e], o[e + 1]), pack_bf16(o[e + 2], o[e + 3]),
                                            pack_bf16(o[e + 4], o[e + 5]), pack_bf16(o[e + 6], o[e + 7]));
                *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(sd.out) + base + e) = wv;
              }
            } else {
#pragma unroll
              for (int e = 0; e < 32; ++e) store_elem(sd.out, base + e * sd.os2, p.out_dtype, o[e]);
            }
          }
        }
      }
    } else if (write) {
      tc_fence_after();
      const bool vec = p.out_vec && p.out_dtype == B200_DTYPE_BF16;
      const float ws = a_self * inv, wo = a_other * inv;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        float o[32];
        tmem_ld32(tmem_o(w) + lane_base + c, o);
        if (g.split) {
          float o1[32];
          tmem_ld32(tmem_o(1) + lane_base + c, o1);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = o[e] * ws + o1[e] * wo;
        } else {
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] *= ws;
        }
        if (iq < sd.T) {
          const int64_t base = iq * sd.os0 + h * sd.os1 + c * sd.os2;
          if (vec) {
#pragma unroll
            for (int e = 0; e < 32; e += 8) {
              const uint4 wv = make_uint4(pack_bf16(o[e], o[e + 1]), pack_bf16(o[e + 2], o[e + 3]),
                                          pack_bf16(o[e + 4], o[e + 5]), pack_bf16(o[e + 6], o[e + 7]));
              *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(sd.out) + base + e) = wv;
            }
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) store_elem(sd.out, base + e * sd.os2, p.out_dtype, o[e]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512)
                 : "memory");
  }
}

}  // namespace

namespace {

// Key split over CTAs.  A launch of fewer CTAs than about 85 % of the SMs
// (one CTA fits an SM) leaves the GPU mostly idle: one sequence's chunk of
// 64 tokens over a 4032-token prefix at 32 heads is 32 CTAs, reading its KV
// at 1.3 TB/s.  Its items' keys are then cut into ks ranges (>= 16 key
// tiles each, so that a range outweighs its partial rows' write and
// combine; ks <= 32), as many as the caller's workspace holds.
constexpr int64_t kSplitRows = 2 * kBM;  // partial rows per (item, head, split)

size_t split_workspace_bytes(int64_t items, int64_t H, int64_t ks, int64_t D) {
  const size_t counters = (static_cast<size_t>(items * H) * sizeof(int32_t) + 255) & ~size_t(255);
  return counters + static_cast<size_t>(items * H * ks * kSplitRows * (D + 2)) * sizeof(float);
}

int64_t plan_key_splits(int64_t items, int64_t H, int64_t key_tiles, int num_sms) {
  const int64_t ctas = items * H;
  if (ctas * 100 >= 85 * static_cast<int64_t>(num_sms)) return 1;
  int64_t ks = ceil_div(85 * static_cast<int64_t>(num_sms), ctas * 100);
  ks = std::min<int64_t>({ks, 32, key_tiles / 16});
  return std::max<int64_t>(ks, 1);
}

}  // namespace

size_t prefill_tc_workspace_bytes(int64_t T, int64_t H, int64_t D, int64_t keys, int num_sms) {
  const int64_t bn = T <= kBM ? 128 : 64;
  const int64_t items = ceil_div(T, 2 * kBM);
  const int64_t ks = plan_key_splits(items, H, ceil_div(keys, bn), num_sms);
  return ks > 1 ? split_workspace_bytes(items, H, ks, D) : 0;
}

bool prefill_tc_supported(const b200_prefill_args_t& a) {
  if (a.pool.dtype != B200_DTYPE_BF16) return false;
  if (a.pool.head_dim != 64 && a.pool.head_dim != 128) return false;
  if (a.pool.block_size < 8 || !is_pow2(a.pool.block_size)) return false;
  return true;
}

template <int D_, int BN>
int launch_tc(const b200_prefill_args_t* seqs, int64_t n, cudaStream_t stream,
              const DeviceInfo& dev) {
  int rc = B200_OK;
  const b200_prefill_args_t& a0 = seqs[0];
  const int64_t D = a0.pool.head_dim, H = a0.pool.num_heads, S = a0.pool.block_size;
  const int64_t P = a0.pool.num_blocks, Ly = a0.pool.num_layers;
  const size_t smem = static_cast<size_t>(Smem<D_, BN>::BYTES) + 1024;
  if (smem > static_cast<size_t>(dev.max_smem_optin))
    return fail(B200_ERR_UNSUPPORTED, "tensor-core prefill: not enough shared memory");

  CUtensorMap tk, tv;
  const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(H),
                            static_cast<uint64_t>(Ly * P * S)};
  const uint64_t strides[2] = {static_cast<uint64_t>(D * 2), static_cast<uint64_t>(H * D * 2)};
  const int64_t rbox = std::min<int64_t>(S, BN);
  const uint32_t box[3] = {64u, 1u, static_cast<uint32_t>(rbox)};
  rc = encode_tensor_map(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a0.pool.k, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != B200_OK) return rc;
  rc = encode_tensor_map(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a0.pool.v, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != B200_OK) return rc;

  static std::atomic<int> configured[64];
  static std::mutex mu;
  if (dev.device >= 0 && dev.device < 64 &&
      !configured[dev.device].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(mu);
    cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel<D_, BN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(prefill_tc)");
    configured[dev.device].store(1, std::memory_order_release);
  }

  for (int64_t base = 0; base < n; base += kMaxSeqs) {
    const int64_t cnt = std::min<int64_t>(kMaxSeqs, n - base);
    PrefillParams prm;
    memset(&prm, 0, sizeof(prm));
    prm.P = P;
    prm.S = S;
    prm.H = H;
    prm.D = D;
    prm.layer = a0.layer_idx;
    prm.q_dtype = a0.q_dtype;
    prm.out_dtype = a0.out_dtype;
    prm.table_i64 = a0.block_table_dtype == B200_INDEX_I64;
    prm.rbox = static_cast<int32_t>(rbox);
    prm.rb_shift = log2i(rbox);
    prm.s_shift = log2i(S);
    prm.nseq = static_cast<int32_t>(cnt);
    prm.status = a0.status;
    prm.scale_log2 = static_cast<float>(1.4426950408889634 / sqrt(static_cast<double>(D)));
    int64_t max_qt = 0;
    bool q_vec = true, out_vec = true;
    for (int64_t i = 0; i < cnt; ++i) {
      const b200_prefill_args_t& s = seqs[base + i];
      if (s.block_table_dtype != a0.block_table_dtype)
        return fail(B200_ERR_INVALID_ARGUMENT, "batched prefill: block tables must share a dtype");
      if (s.num_tokens > (int64_t(1) << 30) || s.prefix_len > (int64_t(1) << 30))
        return fail(B200_ERR_UNSUPPORTED, "prefill chunk too long");
      SeqDesc& d = prm.seq[i];
      d.q = s.q;
      d.out = s.out;
      d.table = s.block_table;
      d.qs0 = s.q_stride[0];
      d.qs1 = s.q_stride[1];
      d.qs2 = s.q_stride[2];
      d.os0 = s.out_stride[0];
      d.os1 = s.out_stride[1];
      d.os2 = s.out_stride[2];
      d.ts = s.block_table_stride;
      d.prefix = static_cast<int32_t>(s.prefix_len);
      d.T = static_cast<int32_t>(s.num_tokens);
      d.table_len = static_cast<int32_t>(std::min<int64_t>(s.block_table_len, INT32_MAX));
      max_qt = std::max<int64_t>(max_qt, ceil_div(s.num_tokens, 2 * kBM));
      const size_t qes = dtype_size(s.q_dtype);
      const bool qv = s.q_stride[2] == 1 && (reinterpret_cast<uintptr_t>(s.q) % 16) == 0 &&
                      (s.q_stride[0] * static_cast<int64_t>(qes)) % 16 == 0 &&
                      (s.q_stride[1] * static_cast<int64_t>(qes)) % 16 == 0;
      const bool ov = s.out_stride[2] == 1 && (reinterpret_cast<uintptr_t>(s.out) % 16) == 0 &&
                      (s.out_stride[0] * 2) % 16 == 0 && (s.out_stride[1] * 2) % 16 == 0;
      q_vec = q_vec && qv;
      out_vec = out_vec && ov;
    }
    prm.max_qtiles = static_cast<int32_t>(max_qt);
    // Q by TMA when every q is bf16 with unit innermost stride and 16-byte
    // aligned rows/heads: dims {D, H, T}, box {64, 1, 128 rows}, swizzle 128B.
    bool q_tma = a0.q_dtype == B200_DTYPE_BF16;
    for (int64_t i = 0; i < cnt && q_tma; ++i) {
      const b200_prefill_args_t& sq = seqs[base + i];
      q_tma = sq.q_stride[2] == 1 && (reinterpret_cast<uintptr_t>(sq.q) % 16) == 0 &&
              (sq.q_stride[0] * 2) % 16 == 0 && (sq.q_stride[1] * 2) % 16 == 0 &&
              sq.q_stride[0] > 0 && sq.q_stride[1] > 0;
    }
    for (int64_t i = 0; i < cnt && q_tma; ++i) {
      const b200_prefill_args_t& sq = seqs[base + i];
      const uint64_t qd[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(H),
                              static_cast<uint64_t>(sq.num_tokens)};
      const uint64_t qs[2] = {static_cast<uint64_t>(sq.q_stride[1] * 2),
                              static_cast<uint64_t>(sq.q_stride[0] * 2)};
      const uint32_t qb[3] = {64u, 1u, static_cast<uint32_t>(kBM)};
      if (encode_tensor_map(&prm.qmap[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                            const_cast<void*>(sq.q), qd, qs, qb,
                            CU_TENSOR_MAP_SWIZZLE_128B) != B200_OK) {
        q_tma = false;  // fall back to thread loads for this launch
        clear_error();
      }
    }
    prm.q_tma = q_tma ? 1 : 0;
    prm.q_vec = q_vec ? 1 : 0;
    prm.out_vec = out_vec ? 1 : 0;
    // Work list: every (sequence, query pair) with its key-tile count, sorted
    // longest first (stable, so equal items keep sequence order).
    std::vector<std::pair<int64_t, uint32_t>> items;
    for (int64_t i = 0; i < cnt; ++i) {
      const b200_prefill_args_t& s = seqs[base + i];
      for (int64_t qp = 0; qp * 2 * kBM < s.num_tokens; ++qp) {
        int64_t tiles = 0;
        for (int w = 0; w < 2; ++w) {
          const int64_t lo = qp * 2 * kBM + w * kBM;
          if (lo < s.num_tokens)
            tiles += ceil_div(s.prefix_len + std::min<int64_t>(s.num_tokens, lo + kBM), BN);
        }
        items.emplace_back(tiles, static_cast<uint32_t>(i) | (static_cast<uint32_t>(qp) << 8));
      }
    }
    std::stable_sort(items.begin(), items.end(),
                     [](const auto& a, const auto& b) { return a.first > b.first; });
    for (size_t w0 = 0; w0 < items.size(); w0 += kMaxWork) {
      const size_t nw = std::min<size_t>(kMaxWork, items.size() - w0);
      int64_t key_tiles = 0;  // the longest item's key tiles (those of its last query)
      for (size_t k = 0; k < nw; ++k) {
        const uint32_t it = items[w0 + k].second;
        prm.work[k] = it;
        const b200_prefill_args_t& s = seqs[base + (it & 0xFFu)];
        const int64_t last_q = std::min<int64_t>(s.num_tokens, (static_cast<int64_t>(it >> 8) + 1) * 2 * kBM);
        key_tiles = std::max<int64_t>(key_tiles, ceil_div(s.prefix_len + last_q, BN));
      }
      int64_t ks = a0.workspace != nullptr
                       ? plan_key_splits(static_cast<int64_t>(nw), H, key_tiles, dev.num_sms)
                       : 1;
      while (ks > 1 && split_workspace_bytes(static_cast<int64_t>(nw), H, ks, D) > a0.workspace_bytes)
        --ks;
      prm.ksplits = static_cast<int32_t>(ks);
      prm.count = nullptr;
      prm.part = nullptr;
      if (ks > 1) {
        const size_t counters = static_cast<size_t>(nw * H) * sizeof(int32_t);
        prm.count = static_cast<int32_t*>(a0.workspace);
        prm.part = reinterpret_cast<float*>(static_cast<char*>(a0.workspace) + ((counters + 255) & ~size_t(255)));
        cudaError_t e = cudaMemsetAsync(prm.count, 0, counters, stream);
        if (e != cudaSuccess) return cuda_fail(e, "prefill split counters");
      }
      const dim3 grid(static_cast<unsigned>(H), static_cast<unsigned>(nw), static_cast<unsigned>(ks));
      prefill_tc_kernel<D_, BN><<<grid, kThreads, smem, stream>>>(tk, tv, prm);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return cuda_fail(e, "prefill_tc launch");
    }
  }
  return B200_OK;
}


int launch_prefill_tc(const b200_prefill_args_t* seqs, int64_t n, cudaStream_t stream) {
  if (n <= 0) return B200_OK;
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc != B200_OK) return rc;
  // 128-key tiles when every CTA holds a single query tile, else 64-key tiles
  // with double-buffered S.
  int64_t max_t = 0;
  for (int64_t i = 0; i < n; ++i) max_t = std::max<int64_t>(max_t, seqs[i].num_tokens);
  const bool short_chunks = max_t <= kBM;
  if (seqs[0].pool.head_dim == 128)
    return short_chunks ? launch_tc<128, 128>(seqs, n, stream, dev)
                        : launch_tc<128, 64>(seqs, n, stream, dev);
  return short_chunks ? launch_tc<64, 128>(seqs, n, stream, dev)
                      : launch_tc<64, 64>(seqs, n, stream, dev);
}

}  // namespace b200
