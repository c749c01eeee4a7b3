// prefill_tc.cu -- prefix-aware chunked-prefill attention on tcgen05 tensor
// cores (bf16 KV pool, head_dim 64 or 128, block size >= 8).
//
// One CTA per (sequence, head, tile of 128 queries).  Query i of a chunk sits
// at absolute position prefix_len + i and attends to keys 0 .. prefix_len + i
// (minivllm/attention.py:256-265), all read from the paged pool.
//
// Warp roles (6 warps):
//   warp 0   TMA producer: for each 128-key tile walks the block table and
//            loads, per KV block, boxes {64 d, 1 head, rbox rows} of K and V
//            with 128-byte swizzle into a 2-stage ring of this CTA.
//   warp 1   TMEM allocation (256 columns) and the MMA issuer (one thread):
//              S   = Q K^T   -> TMEM columns [0, 128)         (M=128,N=128)
//              O  += P V     -> TMEM columns [128, 128+D)      (M=128,N=D)
//            Q, K and P are K-major SW128 operands; V is read MN-major.
//   warps 2-5 softmax / correction / epilogue: thread r of the warpgroup owns
//            query row r = TMEM lane r: it loads its S row (tcgen05.ld),
//            applies the causal mask on absolute positions, updates the
//            running max/sum in the log2 domain, rescales its O row in TMEM
//            when the max grew, and writes its bf16 P row into the swizzled
//            smem tile that the P.V MMA reads.
// V rows beyond the last valid key of the last tile are zeroed in smem
// before the P.V MMA: unwritten pool rows can hold NaN and 0 * NaN is NaN
// inside the tensor core as well (minivllm/paged_attention_batch.py:234-240).
// Every mbarrier wait is bounded; on a timeout the CTA reports
// B200_DEV_WAIT_TIMEOUT, waits for its own MMAs and copies, frees TMEM and
// exits.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "host_util.h"
#include "kernels.h"

namespace b200 {
namespace {

constexpr int kMaxSeqs = 128;  // sequences per launch (host splits larger batches)
constexpr int kThreads = 192;
constexpr int kBM = 128;       // queries per CTA
constexpr int kBN = 128;       // keys per tile

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
  int64_t P, S, H, D;
  int64_t layer;
  int32_t q_dtype, out_dtype, table_i64;
  int32_t rbox, rb_shift, s_shift;
  int32_t nseq;
  int32_t max_qtiles;
  int32_t* status;
  float scale_log2;
  SeqDesc seq[kMaxSeqs];
};

// ------------------------------------------------------------ tcgen05 PTX
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor: f32 accumulate, bf16 A and B, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn_major ? (1u << 16) : 0u) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Byte offset of 16-byte chunk `ch` (0..7) of row `r` in a 128-byte-swizzled
// tile of 128-byte rows.
__device__ __forceinline__ uint32_t sw128(int r, int ch) {
  return static_cast<uint32_t>(r) * 128u + (static_cast<uint32_t>(ch ^ (r & 7)) << 4);
}

// Shared-memory layout (offsets from a 1024-aligned base).
template <int D>
struct Smem {
  static constexpr int HALVES = D / 64;           // 64-element (128-byte) column halves
  static constexpr int TILE = HALVES * 128 * 128;  // one 128-row operand tile
  static constexpr int Q = 0;
  static constexpr int K0 = Q + TILE;              // K stage 0, K stage 1
  static constexpr int V0 = K0 + 2 * TILE;         // V stage 0, V stage 1
  static constexpr int PT = V0 + 2 * TILE;         // P tile: 128 x 128 bf16
  static constexpr int BAR = PT + 2 * 128 * 128;
  static constexpr int BYTES = BAR + 256;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const __grid_constant__ PrefillParams p) {
  using L = Smem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int seq = blockIdx.y;
  const int h = blockIdx.x % static_cast<int>(p.H);
  const int qt = blockIdx.x / static_cast<int>(p.H);
  const SeqDesc& sd = p.seq[seq];
  const int i0 = qt * kBM;
  if (i0 >= sd.T) return;
  const int64_t prefix = sd.prefix;
  const int q_hi = min(sd.T, i0 + kBM);                // queries [i0, q_hi)
  const int64_t total = prefix + q_hi;                   // keys this CTA may see
  const int nkt = static_cast<int>((total + kBN - 1) / kBN);

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint64_t* kv_full = bars + 0;   // [2]
  uint64_t* kv_empty = bars + 2;  // [2]
  uint64_t* s_full = bars + 4;
  uint64_t* p_full = bars + 5;
  uint64_t* o_done = bars + 6;
  uint64_t* mma_idle = bars + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
  int32_t* abort_flag = reinterpret_cast<int32_t*>(bars + 9);

  if (threadIdx.x == 0) {
    mbar_init(&kv_full[0], 1);
    mbar_init(&kv_full[1], 1);
    mbar_init(&kv_empty[0], 1);
    mbar_init(&kv_empty[1], 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    mbar_init(mma_idle, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // Q tile: softmax thread r loads query row i0 + r (zeros past T) into the
  // swizzled K-major tile, converting to bf16.
  if (warp >= 2) {
    // Row r of every 128-row tile is TMEM lane r; a warp may only touch the
    // 32 lanes [32*(warp%4), +32), so rows follow (warp % 4, lane).
    const int r = (warp & 3) * 32 + lane;
    const int i = i0 + r;
    uint8_t* qt_base = smem + L::Q;
#pragma unroll
    for (int half = 0; half < L::HALVES; ++half) {
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int d = half * 64 + ch * 8 + e;
          f[e] = (i < sd.T) ? load_elem(sd.q, i * sd.qs0 + h * sd.qs1 + d * sd.qs2, p.q_dtype) : 0.f;
        }
        uint4 w = make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]),
                             pack_bf16(f[6], f[7]));
        *reinterpret_cast<uint4*>(qt_base + half * 16384 + sw128(r, ch)) = w;
      }
    }
    fence_proxy_async_shared();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem;        // columns [0, 128)
  const uint32_t tmem_o = tmem + 128;  // columns [128, 128 + D)

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const int box_bytes = 64 * p.rbox * 2;
    const int boxes_per_tile = kBN / p.rbox;
    int64_t j_base = -(int64_t(1) << 40);
    int64_t my_entry = 0;
    int issued = 0;
    for (int j = 0; j < nkt; ++j) {
      const int st = j & 1;
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok || *reinterpret_cast<volatile int32_t*>(abort_flag)) {
        if (lane == 0 && !ok) {
          report(p.status, B200_DEV_WAIT_TIMEOUT);
          *abort_flag = 1;
        }
        break;
      }
      const int64_t key0 = static_cast<int64_t>(j) * kBN;
      const int nb = static_cast<int>(min(static_cast<int64_t>(boxes_per_tile),
                                          (total - key0 + p.rbox - 1) >> p.rb_shift));
      if (lane == 0)
        mbar_arrive_expect_tx(&kv_full[st], static_cast<uint32_t>(nb * 2 * L::HALVES * box_bytes));
      uint8_t* kdst = smem + L::K0 + st * L::TILE;
      uint8_t* vdst = smem + L::V0 + st * L::TILE;
      for (int b = 0; b < nb; ++b) {
        const int64_t key = key0 + (static_cast<int64_t>(b) << p.rb_shift);
        const int64_t blk = key >> p.s_shift;
        if (blk < j_base || blk >= j_base + 32) {
          j_base = blk;
          my_entry = (blk + lane < sd.table_len)
                         ? load_index(sd.table, (blk + lane) * sd.ts, p.table_i64)
                         : -1;
        }
        int64_t phys = __shfl_sync(0xffffffffu, my_entry, static_cast<int>(blk - j_base));
        if (phys < 0 || phys >= p.P) {
          if (lane == 0) report(p.status, B200_DEV_BAD_BLOCK);
          phys = 0;
        }
        if (lane == 0) {
          const int32_t row = static_cast<int32_t>((p.layer * p.P + phys) * p.S + (key & (p.S - 1)));
#pragma unroll
          for (int half = 0; half < L::HALVES; ++half) {
            const uint32_t off = half * 16384 + b * p.rbox * 128;
            tma_load_3d(kdst + off, &tmk, &kv_full[st], half * 64, h, row);
            tma_load_3d(vdst + off, &tmv, &kv_full[st], half * 64, h, row);
          }
        }
      }
      ++issued;
    }
    if (lane == 0) {
      const int first = issued > 2 ? issued - 2 : 0;
      for (int j = first; j < issued; ++j)
        if (!mbar_wait(&kv_full[j & 1], (j >> 1) & 1)) {
          report(p.status, B200_DEV_WAIT_TIMEOUT);
          break;
        }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16(128, 128, false);
      constexpr uint32_t idesc_o = idesc_bf16(128, D, true);
      const uint32_t q_addr = smem_u32(smem + L::Q);
      const uint32_t p_addr = smem_u32(smem + L::PT);
      bool ok = true;
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&kv_full[st], (j >> 1) & 1)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + L::K0 + st * L::TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t koff = (kk >> 2) * 16384 + (kk & 3) * 32;
          mma_bf16(tmem_s, smem_desc_sw128(q_addr + koff, 16, 1024),
                   smem_desc_sw128(k_addr + koff, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(s_full);
        return true;
      };
      ok = issue_s(0);
      for (int j = 0; ok && j < nkt; ++j) {
        if (!mbar_wait(p_full, j & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int st = j & 1;
        const uint32_t v_addr = smem_u32(smem + L::V0 + st * L::TILE);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint32_t poff = (kk >> 2) * 16384 + (kk & 3) * 32;
          mma_bf16(tmem_o, smem_desc_sw128(p_addr + poff, 16, 1024),
                   smem_desc_sw128(v_addr + kk * 2048, 16384, 1024), idesc_o,
                   (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&kv_empty[st]);
        mma_commit(o_done);
        if (j + 1 < nkt && !issue_s(j + 1)) {
          ok = false;
          break;
        }
      }
      if (!ok) {
        report(p.status, B200_DEV_WAIT_TIMEOUT);
        *abort_flag = 1;
      }
      // Wait until every MMA this thread issued has completed.
      mma_commit(mma_idle);
      if (!mbar_wait(mma_idle, 0)) report(p.status, B200_DEV_WAIT_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int r = (warp & 3) * 32 + lane;    // query row == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int i = min(i0 + r, sd.T - 1);     // rows past T mirror the last query
    const int64_t qpos = prefix + i;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkt; ++j) {
      if (!mbar_wait(s_full, j & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kBN];
#pragma unroll
      for (int c = 0; c < kBN; c += 32) tmem_ld32(tmem_s + lane_base + c, s + c);
      tmem_wait_ld();
      const int64_t key0 = static_cast<int64_t>(j) * kBN;
      float mx = -INFINITY;
      if (key0 + kBN - 1 <= qpos) {
#pragma unroll
        for (int c = 0; c < kBN; ++c) {
          s[c] *= p.scale_log2;
          mx = fmaxf(mx, s[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < kBN; ++c) {
          s[c] = (key0 + c <= qpos) ? s[c] * p.scale_log2 : -INFINITY;
          mx = fmaxf(mx, s[c]);
        }
      }
      const float m_new = fmaxf(m, mx);
      const float alpha = fast_exp2(m - m_new);
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < kBN; ++c) {
        s[c] = fast_exp2(s[c] - m_new);
        rs += s[c];
      }
      l = l * alpha + rs;
      m = m_new;
      if (j > 0) {
        // P.V of the previous tile must be done before O is rescaled and
        // before the P tile is overwritten.
        if (!mbar_wait(o_done, (j - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
          for (int c = 0; c < D; c += 32) {
            float o[32];
            tmem_ld32(tmem_o + lane_base + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= alpha;
            tmem_st32(tmem_o + lane_base + c, o);
          }
          tmem_wait_st();
        }
      }
      // Zero V rows past the last valid key of the tile (pool rows there may
      // be unwritten); thread r clears row r of both column halves.
      const int64_t valid = total - key0;
      if (valid < kBN && r >= valid) {
        uint8_t* vrow = smem + L::V0 + (j & 1) * L::TILE + r * 128;
#pragma unroll
        for (int half = 0; half < L::HALVES; ++half)
#pragma unroll
          for (int ch = 0; ch < 8; ++ch)
            *reinterpret_cast<uint4*>(vrow + half * 16384 + ch * 16) = make_uint4(0, 0, 0, 0);
      }
      uint8_t* pt = smem + L::PT;
#pragma unroll
      for (int ch = 0; ch < 16; ++ch) {
        const int c = ch * 8;
        uint4 w = make_uint4(pack_bf16(s[c], s[c + 1]), pack_bf16(s[c + 2], s[c + 3]),
                             pack_bf16(s[c + 4], s[c + 5]), pack_bf16(s[c + 6], s[c + 7]));
        *reinterpret_cast<uint4*>(pt + (ch >> 3) * 16384 + sw128(r, ch & 7)) = w;
      }
      fence_proxy_async_shared();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && !mbar_wait(o_done, (nkt - 1) & 1)) ok = false;
    if (!ok) {
      if (r == 0) report(p.status, B200_DEV_WAIT_TIMEOUT);
      *abort_flag = 1;
    } else {
      tc_fence_after();
      const int iq = i0 + r;
      const float inv = 1.0f / l;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        float o[32];
        tmem_ld32(tmem_o + lane_base + c, o);
        tmem_wait_ld();
        if (iq < sd.T) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            store_elem(sd.out, iq * sd.os0 + h * sd.os1 + (c + e) * sd.os2, p.out_dtype, o[e] * inv);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256)
                 : "memory");
  }
}

}  // namespace

bool prefill_tc_supported(const b200_prefill_args_t& a) {
  if (a.pool.dtype != B200_DTYPE_BF16) return false;
  if (a.pool.head_dim != 64 && a.pool.head_dim != 128) return false;
  if (a.pool.block_size < 8 || !is_pow2(a.pool.block_size)) return false;
  return true;
}

int launch_prefill_tc(const b200_prefill_args_t* seqs, int64_t n, cudaStream_t stream) {
  if (n <= 0) return B200_OK;
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc != B200_OK) return rc;
  const b200_prefill_args_t& a0 = seqs[0];
  const int64_t D = a0.pool.head_dim, H = a0.pool.num_heads, S = a0.pool.block_size;
  const int64_t P = a0.pool.num_blocks, Ly = a0.pool.num_layers;
  const size_t smem = static_cast<size_t>(D == 128 ? Smem<128>::BYTES : Smem<64>::BYTES) + 1024;
  if (smem > static_cast<size_t>(dev.max_smem_optin))
    return fail(B200_ERR_UNSUPPORTED, "tensor-core prefill: not enough shared memory");

  CUtensorMap tk, tv;
  const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(H),
                            static_cast<uint64_t>(Ly * P * S)};
  const uint64_t strides[2] = {static_cast<uint64_t>(D * 2), static_cast<uint64_t>(H * D * 2)};
  const int64_t rbox = std::min<int64_t>(S, kBN);
  const uint32_t box[3] = {64u, 1u, static_cast<uint32_t>(rbox)};
  rc = encode_tensor_map(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a0.pool.k, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != B200_OK) return rc;
  rc = encode_tensor_map(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a0.pool.v, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != B200_OK) return rc;

  static int configured[64][2] = {{0}};
  const int slot = D == 128 ? 1 : 0;
  if (dev.device >= 0 && dev.device < 64 && !configured[dev.device][slot]) {
    cudaError_t e = D == 128
                        ? cudaFuncSetAttribute(prefill_tc_kernel<128>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem))
                        : cudaFuncSetAttribute(prefill_tc_kernel<64>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(prefill_tc)");
    configured[dev.device][slot] = 1;
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
      max_qt = std::max<int64_t>(max_qt, ceil_div(s.num_tokens, kBM));
    }
    prm.max_qtiles = static_cast<int32_t>(max_qt);
    const dim3 grid(static_cast<unsigned>(max_qt * H), static_cast<unsigned>(cnt));
    if (D == 128)
      prefill_tc_kernel<128><<<grid, kThreads, smem, stream>>>(tk, tv, prm);
    else
      prefill_tc_kernel<64><<<grid, kThreads, smem, stream>>>(tk, tv, prm);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "prefill_tc launch");
  }
  return B200_OK;
}

}  // namespace b200
