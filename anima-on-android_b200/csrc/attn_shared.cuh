// attn_shared.cuh -- pieces shared by the attention kernels (128-key tiles in
// attn_fwd.cu, 64-key tiles in attn_fwd64.cu): warp roles and register split, call
// parameters, the segment walk of the three schedules (one CTA per unit, persistent whole
// units, and the cut last round), and the staged output epilogue.
#pragma once
#include <type_traits>

#include "common.cuh"

namespace anima {
namespace attn {

constexpr int kD = 128;
constexpr int kBM = 128;               // query rows per tile (TMEM lanes)
constexpr int kNT = 2;                 // query tiles per unit
constexpr int kUnitRows = kBM * kNT;   // 256
constexpr int kKvWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kQWarp = 10;
constexpr int kThreads = 384;          // 3 warpgroups
// Launch budget 384 x 168 registers; the control warpgroup gives registers back to the
// two softmax warpgroups: 2*128*200 + 128*104 = 64512 = 384*168.
constexpr uint32_t kRegsSoftmax = 200;
constexpr uint32_t kRegsControl = 104;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
#ifndef ANIMA_POLY_PER8
#define ANIMA_POLY_PER8 0
#endif
// Of every 8 column pairs, how many take the FMA-pipe polynomial exp2 instead of MUFU.
// 0 by default: the extra softmax instructions take issue slots from the MMA and TMA
// warps that share the SM sub-partitions and sit on the critical path; 1/8 measured 14 %
// slower, 2/8 22 %.
constexpr int kPolyPer8 = ANIMA_POLY_PER8;
// One partial of a split unit: O fp32 (unnormalised) quad-major, [32 column quads][256 rows]
// [4], so 32 consecutive rows of one quad are 512 contiguous bytes; then m [256], l [256].
constexpr int kPartFloats = kUnitRows * kD + 2 * kUnitRows;
constexpr int kSemBytes = 4096;         // arrival counters at the start of the workspace


constexpr int kMaxPeers = 8;  // output destinations of one call (ranks of one NVLink domain)

struct Params {
  int B, H, S_q, S_kv;
  float scale_log2;
  unsigned flags;
  const int* kv_valid;
  void* out;
  long long ob, oh, os;
  int* status;
  int nqb;             // query units per (batch, head)
  int units;           // B * H * nqb
  int split;           // 1: persistent grid (whole-unit rounds, then the cut last round)
  int n_kv;            // key tiles per unit (split mode)
  int rounds;          // whole-unit rounds: CTA c owns units c + r * gridDim.x (< units)
  int tail_base;       // first unit of the cut last round (rounds * gridDim.x)
  int tail_tiles;      // key-tile steps of the last round
  int tail_ctas;       // CTAs sharing the last round (<= gridDim.x)
  int* sem;            // arrival counters [tail unit][tile], zero between calls
  float* part;         // partial slots [tail_ctas][2][kPartFloats]
  int tma_out;         // 1: output blocks leave by TMA tensor stores (map passed separately)
  int tma_hs;          // output map axes (D, H, S, B) (1) or (D, S, H, B) (0)
  int n_peers;         // > 0: output blocks go to peer_out bases instead of out
  void* peer_out[kMaxPeers];
  int peer_rows;       // 0: every block to every base (all-gather); > 0: row scatter, global
                       // row g = b * S_q + s to base g / peer_rows at local row g % peer_rows
  long long peer_row_stride;  // row scatter: elements between a destination's rows
  int peer_head0;      // row scatter: this call's first head in a destination row
};

// Slice of the last round owned by CTA c: key-tile steps [slice_lo(c), slice_lo(c+1)).
__device__ __forceinline__ int slice_lo(const Params& p, int c) {
  return (int)((long long)c * p.tail_tiles / p.tail_ctas);
}
// The CTA whose slice holds key-tile step t of the last round.
__device__ __forceinline__ int slice_of(const Params& p, int t) {
  return (int)((((long long)t + 1) * p.tail_ctas + p.tail_tiles - 1) / p.tail_tiles) - 1;
}

// One piece of work of a CTA: key tiles [k0, k1) of unit `unit`.
struct Seg {
  int unit, k0, k1;
  int full;            // covers every key tile of the unit
  int slot;            // partial slot (0: starts the CTA's slice, 1: ends it)
};

// Key tiles of a unit in unit mode (mask / causal aware).
__device__ __forceinline__ int unit_kv_len(const Params& p, int unit) {
  const int b = (unit / p.nqb) / p.H;
  int kv_len = p.S_kv;
  if (p.flags & ANIMA_FLAG_MASK) kv_len = min(max(p.kv_valid[b], 0), p.S_kv);
  return kv_len;
}
// kBN: keys per key tile of the calling kernel.
// In split mode (persistent grid) a unit has p.n_kv key tiles, or fewer when its sample's
// keys are masked (masked calls run whole units only, never cut).
template <int kBN>
__device__ __forceinline__ int unit_tiles(const Params& p, int unit) {
  if (p.split && !(p.flags & ANIMA_FLAG_MASK)) return p.n_kv;
  int n = (unit_kv_len(p, unit) + kBN - 1) / kBN;
  if (p.flags & ANIMA_FLAG_CAUSAL) {
    const int q0 = (unit % p.nqb) * kUnitRows;
    const int last_row = min(q0 + kUnitRows, p.S_q) - 1;
    n = min(n, last_row / kBN + 1);
  }
  return n;
}

// Segment iterator: every role walks the same sequence.
template <int kBN>
struct SegIter {
  int r;          // whole-unit rounds handed out so far
  int t, lo, hi;  // this CTA's slice of the last round (key-tile steps)
  __device__ __forceinline__ SegIter(const Params& p) : r(0) {
    if (!p.split) {
      lo = 0;
      hi = 1;
    } else if ((int)blockIdx.x < p.tail_ctas) {
      lo = slice_lo(p, blockIdx.x);
      hi = slice_lo(p, blockIdx.x + 1);
    } else {
      lo = hi = 0;
    }
    t = lo;
  }
  __device__ __forceinline__ bool next(const Params& p, Seg& s) {
    if (!p.split) {
      if (t >= hi) return false;
      s.unit = blockIdx.x;
      s.k0 = 0;
      s.k1 = unit_tiles<kBN>(p, s.unit);
      s.full = 1;
      s.slot = 0;
      t = hi;
      return true;
    }
    const int n = p.n_kv;
    if (r < p.rounds) {
      s.unit = blockIdx.x + r * gridDim.x;
      ++r;
      if (s.unit < p.units) {
        s.k0 = 0;
        s.k1 = unit_tiles<kBN>(p, s.unit);
        s.full = 1;
        s.slot = 0;
        return true;
      }
      r = p.rounds;  // the last whole round leaves this CTA out
    }
    if (t >= hi) return false;
    const int ut = t / n;
    const int ubeg = ut * n, uend = ubeg + n;
    s.unit = p.tail_base + ut;
    s.k0 = t - ubeg;
    s.k1 = min(uend, hi) - ubeg;
    s.full = (s.k0 == 0 && s.k1 == n);
    s.slot = (t == lo) ? 0 : 1;
    t = min(uend, hi);
    return true;
  }
};

// Bounded wait that only gives up on its time limit; used to drain in-flight copies
// and MMAs on the exit path after an abort.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return;
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) return;
  }
}

// Barrier over the 128 threads of one softmax warpgroup (ids 1, 2; 0 is __syncthreads).
__device__ __forceinline__ void wg_sync(int id) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(kBM) : "memory");
}

template <int kOp>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return kOp == ANIMA_DTYPE_BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}

// True in every thread of softmax warpgroup barrier `id` if `v` is true in any of them.
__device__ __forceinline__ bool wg_any(int id, bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n"
      " selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(kBM)
      : "memory");
  return r != 0;
}

// Stores columns [32 c, 32 c + 32) of the warp's 32 output rows; lane = row on entry (its
// values v, scaled by inv).  The block goes through the warp's 4 KB staging buffer
// (16-byte chunks XOR-swizzled by row, so neither the row-wise writes nor the transposed
// reads conflict on banks) and leaves as whole row segments: 4 rows x 128 B per fp32 store
// instruction, 8 rows x 64 B for 16-bit, instead of 32 scattered 16-byte pieces.  Rows
// >= nvalid are not written.
// The warp's 32 x 32 block (lane = row, v = its 32 columns, times inv) into the staging
// buffer: fp32 rows of 128 B with 16-byte chunks XOR-swizzled by (row & 7), 16-bit rows of
// 64 B swizzled by ((row >> 1) & 3), so neither this write nor the transposed read conflicts
// on banks.  These are the 128-byte and 64-byte swizzle layouts of a TMA tile.
template <int kOut>
__device__ __forceinline__ void stage_block(const float (&v)[32], float inv, float4* stage,
                                            int lane) {
  if (kOut == ANIMA_DTYPE_F32) {
#pragma unroll
    for (int e = 0; e < 8; ++e)
      stage[lane * 8 + (e ^ (lane & 7))] =
          make_float4(v[4 * e] * inv, v[4 * e + 1] * inv, v[4 * e + 2] * inv, v[4 * e + 3] * inv);
  } else {
    uint4* st = reinterpret_cast<uint4*>(stage);
#pragma unroll
    for (int e = 0; e < 4; ++e)
      st[lane * 4 + (e ^ ((lane >> 1) & 3))] = make_uint4(
          pack2<kOut>(v[8 * e] * inv, v[8 * e + 1] * inv),
          pack2<kOut>(v[8 * e + 2] * inv, v[8 * e + 3] * inv),
          pack2<kOut>(v[8 * e + 4] * inv, v[8 * e + 5] * inv),
          pack2<kOut>(v[8 * e + 6] * inv, v[8 * e + 7] * inv));
  }
}

template <int kOut>
__device__ __forceinline__ void store_block(char* out_w, long long row_bytes, int nvalid,
                                            const float (&v)[32], int c, float inv,
                                            float4* stage, int lane) {
  stage_block<kOut>(v, inv, stage, lane);
  __syncwarp();
  if (kOut == ANIMA_DTYPE_F32) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int r = 4 * k + (lane >> 3), q = lane & 7;
      const float4 x = stage[r * 8 + (q ^ (r & 7))];
      if (r < nvalid)
        *reinterpret_cast<float4*>(out_w + r * row_bytes + (c * 32 + q * 4) * 4) = x;
    }
  } else {
    const uint4* st = reinterpret_cast<const uint4*>(stage);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int r = 8 * k + (lane >> 2), q = lane & 3;
      const uint4 x = st[r * 4 + (q ^ ((r >> 1) & 3))];
      if (r < nvalid) *reinterpret_cast<uint4*>(out_w + r * row_bytes + (c * 32 + q * 8) * 2) = x;
    }
  }
  __syncwarp();  // the buffer is free for the next block
}

// The warp's 32 x 32 block, staged once, stored to every destination base p.peer_out[0 ..
// n_peers) at byte offset `off` (+ row r * row_bytes + column): the all-gather of the head
// outputs over NVLink, folded into the epilogue (the other ranks' bases are peer mappings).
template <int kOut>
__device__ __forceinline__ void store_block_peers(const Params& p, long long off,
                                                  long long row_bytes, int nvalid,
                                                  const float (&v)[32], int c, float inv,
                                                  float4* stage, int lane) {
  stage_block<kOut>(v, inv, stage, lane);
  __syncwarp();
  if (kOut == ANIMA_DTYPE_F32) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int r = 4 * k + (lane >> 3), q = lane & 7;
      const float4 x = stage[r * 8 + (q ^ (r & 7))];
      const long long o = off + r * row_bytes + (c * 32 + q * 4) * 4;
#pragma unroll
      for (int i = 0; i < kMaxPeers; ++i)
        if (i < p.n_peers && r < nvalid)
          *reinterpret_cast<float4*>(static_cast<char*>(p.peer_out[i]) + o) = x;
    }
  } else {
    const uint4* st = reinterpret_cast<const uint4*>(stage);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int r = 8 * k + (lane >> 2), q = lane & 3;
      const uint4 x = st[r * 4 + (q ^ ((r >> 1) & 3))];
      const long long o = off + r * row_bytes + (c * 32 + q * 8) * 2;
#pragma unroll
      for (int i = 0; i < kMaxPeers; ++i)
        if (i < p.n_peers && r < nvalid)
          *reinterpret_cast<uint4*>(static_cast<char*>(p.peer_out[i]) + o) = x;
    }
  }
  __syncwarp();  // the buffer is free for the next block
}

// Output tile map of a call (om != nullptr): the staged block leaves as one TMA tensor store
// issued by lane 0, which only waits, before the next block, for the bulk engine to have
// read the buffer; rows past S_q are clipped by the map.  (x, y, z, w) are the block's map
// coordinates: column 32c, then the head/token axes in the map's order, then the batch.
template <int kOut>
__device__ __forceinline__ void store_block_tma(const CUtensorMap* om, int x, int y, int z, int w,
                                                const float (&v)[32], float inv, float4* stage,
                                                int lane) {
  if (lane == 0) bulk_wait_read_all();  // the previous block's store has read the buffer
  __syncwarp();
  stage_block<kOut>(v, inv, stage, lane);
  fence_proxy_async_smem();  // these generic-proxy writes, before the async-proxy read
  __syncwarp();
  if (lane == 0) {
    tma_store_4d(om, stage, x, y, z, w);
    bulk_commit_group();
  }
}

// Output of one segment of query tile i: O in tensor memory at tO (this warp's lane
// quarter), m and l the row's running max and sum.  A whole unit is normalised and
// stored; a slice of a cut unit is stored as an fp32 partial, or merged with the other
// slices' partials by the last warpgroup to finish the unit's tile.  `stage` is the warp's
// 4 KB staging buffer.
template <int kOut>
__device__ __forceinline__ void segment_epilogue(const Params& p, const Seg& sg, int n, int i,
                                                 int row, int lane, int b, int bh, int grow,
                                                 uint32_t tO, float m, float l, float4* stage,
                                                 const CUtensorMap* om = nullptr) {
  // The warp's first output row, and how many of its 32 rows exist.
  constexpr int kEsize = kOut == ANIMA_DTYPE_F32 ? 4 : 2;
  const long long row_bytes = p.os * kEsize;
  char* const out_w = reinterpret_cast<char*>(p.out) +
                      ((long long)b * p.ob + (long long)(bh % p.H) * p.oh +
                       (long long)(grow - lane) * p.os) *
                          kEsize;
  const int nvalid = p.S_q - (grow - lane);
  // TMA coordinates of this warp's blocks: (32c, head or token, token or head, batch).
  const int h_ = bh % p.H, s_ = grow - lane;
  const int ty = p.tma_hs ? h_ : s_, tz = p.tma_hs ? s_ : h_;
  const long long off = ((long long)b * p.ob + (long long)(bh % p.H) * p.oh +
                         (long long)(grow - lane) * p.os) * kEsize;
  auto put = [&](const float (&v)[32], int c, float inv) {
    if (p.n_peers > 0 && p.peer_rows > 0) {
      // the all-to-all back to the token owners: the 32 rows of this block belong to one
      // rank (S_q and peer_rows are multiples of 32)
      const int g0 = b * p.S_q + s_;
      const int d = g0 / p.peer_rows, r0 = g0 - d * p.peer_rows;
      char* base = nullptr;
#pragma unroll
      for (int k = 0; k < kMaxPeers; ++k)  // constant indices: no local copy of the params
        if (k == d) base = static_cast<char*>(p.peer_out[k]);
      if (nvalid > 0)
        store_block<kOut>(base + ((long long)r0 * p.peer_row_stride +
                                  (long long)(p.peer_head0 + h_) * kD) * kEsize,
                          p.peer_row_stride * kEsize, nvalid, v, c, inv, stage, lane);
    } else if (p.n_peers > 0) {
      store_block_peers<kOut>(p, off, row_bytes, nvalid, v, c, inv, stage, lane);
    } else if (om != nullptr) {
      if (nvalid > 0) store_block_tma<kOut>(om, c * 32, ty, tz, b, v, inv, stage, lane);
    } else {
      store_block<kOut>(out_w, row_bytes, nvalid, v, c, inv, stage, lane);
    }
  };
  if (sg.full) {
    const float inv = (l > 0.f) ? 1.f / l : 0.f;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float v[32];
      if (n > 0) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(o[e]);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = 0.f;
      }
      put(v, c, inv);
    }
  } else {
    // A slice of a cut unit.  The warpgroup that completes the unit tile's arrival
    // count merges every slice of it,
    //   out = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s,  M = max_s m_s,
    // its own slice straight from tensor memory and the others from their partials.
    // A warpgroup that finds every other slice already counted is last before it
    // stores anything, and skips its own partial.
    const int ut = sg.unit - p.tail_base;
    const int r = i * kBM + row;
    const int t0 = ut * p.n_kv, t1 = t0 + p.n_kv;
    const int c0 = slice_of(p, t0), c1 = slice_of(p, t1 - 1);
    const int me = blockIdx.x;
    int* const cnt = &p.sem[ut * kNT + i];
    auto part_of = [&](int c) {
      const int lo_c = slice_lo(p, c);
      return p.part + ((long long)c * 2 + (max(t0, lo_c) == lo_c ? 0 : 1)) * kPartFloats;
    };
    bool last = wg_any(1 + i, row == 0 && *reinterpret_cast<volatile int*>(cnt) == c1 - c0);
    if (!last) {
      float* const part = part_of(me);
      float4* const dst = reinterpret_cast<float4*>(part) + r;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 8; ++e)
          dst[(c * 8 + e) * kUnitRows] =
              make_float4(__uint_as_float(o[4 * e]), __uint_as_float(o[4 * e + 1]),
                          __uint_as_float(o[4 * e + 2]), __uint_as_float(o[4 * e + 3]));
      }
      part[kUnitRows * kD + r] = m;
      part[kUnitRows * kD + kUnitRows + r] = l;
      __threadfence();
      wg_sync(1 + i);
      int prev = 0;
      if (row == 0) prev = atomicAdd(cnt, 1);
      last = wg_any(1 + i, row == 0 && prev == c1 - c0);
    }
    if (last) {
      __threadfence();
      const int nothers = c1 - c0;  // this CTA is one of the unit's slices
      auto other = [&](int k) { return c0 + k + (c0 + k >= me ? 1 : 0); };
      // Pass 1: M and the denominator over all slices of this row.
      float M = m, den = l;
#pragma unroll 2
      for (int k = 0; k < nothers; ++k) {
        const float* pc = part_of(other(k));
        const float mc = __ldcg(pc + kUnitRows * kD + r);
        const float lc = __ldcg(pc + kUnitRows * kD + kUnitRows + r);
        const float mn = fmaxf(M, mc);
        den = den * exp2f(M - mn) + lc * exp2f(mc - mn);
        M = mn;
      }
      const float inv = den > 0.f ? 1.f / den : 0.f;
      const float w_own = exp2f(m - M) * inv;
      // Pass 2 in tensor memory: the own O scaled in place, then each other slice's partial
      // added into it with all four 32-column chunks loaded at once (one L2 round trip per
      // slice, 32 loads in flight, quad-major rows: one 512-byte run per warp load), then the
      // merged rows stored.
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * w_own);
        tmem_st32(tO + c * 32, o);
      }
      tmem_st_wait();
#pragma unroll 1
      for (int k = 0; k < nothers; ++k) {
        const float* pc = part_of(other(k));
        const float wc = exp2f(__ldcg(pc + kUnitRows * kD + r) - M) * inv;
        const float4* src = reinterpret_cast<const float4*>(pc) + r;
        float4 x[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] = __ldcg(src + j * kUnitRows);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float4 xe = x[c * 8 + e];
            o[4 * e] = __float_as_uint(__uint_as_float(o[4 * e]) + wc * xe.x);
            o[4 * e + 1] = __float_as_uint(__uint_as_float(o[4 * e + 1]) + wc * xe.y);
            o[4 * e + 2] = __float_as_uint(__uint_as_float(o[4 * e + 2]) + wc * xe.z);
            o[4 * e + 3] = __float_as_uint(__uint_as_float(o[4 * e + 3]) + wc * xe.w);
          }
          tmem_st32(tO + c * 32, o);
        }
        tmem_st_wait();
      }
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + c * 32, o);
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(o[e]);
        put(v, c, 1.f);
      }
      if (row == 0) *cnt = 0;  // leave the counter zero for the next call
    }
  }
}

}  // namespace attn
}  // namespace anima
