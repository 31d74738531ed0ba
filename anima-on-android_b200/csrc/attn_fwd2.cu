// attn_fwd2.cu -- flash-attention forward on CTA pairs (2-SM tcgen05 MMA), sm_100a.
//
// Same math and softmax as attn_fwd.cu (anima::cpu::flash_attention,
// anima_rt/include/cpu/flash_attention.h:55-208), but the two CTAs of a cluster pair
// issue their matrix products together: the leader's MMA warp runs
// tcgen05.mma.cta_group::2 with M = 256 (each CTA's 128 query rows), so each SM supplies
// only HALF of every K tile (64 of its 128 keys) and HALF of every V tile (64 of the 128
// head-dim columns).  A QK^T step then reads 96 B/clk of shared memory per SM instead of
// 128, and a key-tile step moves 160 KB through each SM's shared memory instead of 256 KB,
// which is what bounded the one-SM kernel.
//
// Work unit = 512 query rows of one (batch, head): CTA rank r owns rows [256r, 256r+256)
// as two 128-row tiles.  One cluster per unit.
//
// Per CTA (384 threads): warps 0-7 softmax (tile = warp / 4, thread = row = TMEM lane),
// warp 8 K/V producer (own halves), warp 9 TMEM owner (+ MMA issuer in the leader),
// warp 10 Q producer, warp 11 idle.  TMEM per CTA as in the one-SM kernel:
// S_0 S_1 O_0 O_1, 128 columns each, P over the first 64 columns of S.
//
// Hand-offs: TMA loads of both CTAs count on the leader's full barriers; the leader's
// commits arrive on both CTAs' barriers (tcgen05.commit multicast); the peer's softmax
// threads arrive on the leader's P barriers through cluster addresses.  No TMA multicast.
#include "common.cuh"

namespace anima {
namespace attn2 {

constexpr int kD = 128;
constexpr int kBM = 128;                 // rows per tile per CTA
constexpr int kNT = 2;                   // tiles per CTA
constexpr int kUnitRows = 2 * kNT * kBM; // 512 rows per cluster
constexpr int kBN = 128;                 // keys per step (64 per CTA for K)
constexpr int kStages = 8;               // K/V half-tile ring slots
constexpr int kQPanel = 128 * 128;       // [128 rows][64 x 16-bit], 16 KB
constexpr int kQTile = 2 * kQPanel;      // 32 KB
constexpr int kKPanel = 64 * 128;        // [64 keys][64 x 16-bit], 8 KB
constexpr int kSlot = 16 * 1024;         // K half (2 x 8 KB panels) or V half (one 16 KB panel)
constexpr int kKvWarp = 8, kMmaWarp = 9, kQWarp = 10;
constexpr int kThreads = 384;
constexpr uint32_t kRegsSoftmax = 200;
constexpr uint32_t kRegsControl = 104;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;
constexpr int kPolyPer8 = 0;

struct Smem {
  uint8_t q[kNT][kQTile];
  uint8_t kv[kStages][kSlot];
  uint64_t q_full;                 // leader: 2 arrivals (one per CTA) + bytes
  uint64_t kv_full[kStages];       // leader: 2 arrivals + bytes
  uint64_t kv_empty[kStages];      // every CTA: leader's multicast commit
  uint64_t s_full[kNT];            // every CTA: multicast commit
  uint64_t p_full[kNT];            // leader: 256 arrivals (both CTAs' softmax threads)
  uint64_t o_full[kNT];            // every CTA: multicast commit
  uint64_t mma_done;               // every CTA: multicast commit
  uint32_t tmem_base;
  int abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

struct Params {
  int B, H, S_q, S_kv;
  float scale_log2;
  unsigned flags;
  const int* kv_valid;
  void* out;
  long long ob, oh, os;
  int* status;
  int nqb;  // 512-row units per (batch, head)
};

__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait_cluster(bar, parity)) return;
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) return;
  }
}

template <int kOp>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return kOp == ANIMA_DTYPE_BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}

template <int kOut>
__device__ __forceinline__ void store_row(char* out_row, const uint32_t (&o)[32], int c,
                                          float inv) {
  if (kOut == ANIMA_DTYPE_F32) {
    float4* dst = reinterpret_cast<float4*>(out_row) + c * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      dst[e] = make_float4(__uint_as_float(o[4 * e]) * inv, __uint_as_float(o[4 * e + 1]) * inv,
                           __uint_as_float(o[4 * e + 2]) * inv, __uint_as_float(o[4 * e + 3]) * inv);
  } else {
    uint4* dst = reinterpret_cast<uint4*>(out_row) + c * 4;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      dst[e] = make_uint4(
          pack2<kOut>(__uint_as_float(o[8 * e]) * inv, __uint_as_float(o[8 * e + 1]) * inv),
          pack2<kOut>(__uint_as_float(o[8 * e + 2]) * inv, __uint_as_float(o[8 * e + 3]) * inv),
          pack2<kOut>(__uint_as_float(o[8 * e + 4]) * inv, __uint_as_float(o[8 * e + 5]) * inv),
          pack2<kOut>(__uint_as_float(o[8 * e + 6]) * inv, __uint_as_float(o[8 * e + 7]) * inv));
  }
}

template <int kOp, int kOut>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    attn_fwd_pair_kernel(const __grid_constant__ CUtensorMap tmap_q,
                         const __grid_constant__ CUtensorMap tmap_k,
                         const __grid_constant__ CUtensorMap tmap_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + pad);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int unit = blockIdx.x >> 1;
  const int bh = unit / p.nqb;
  const int b = bh / p.H;
  const int q0 = (unit % p.nqb) * kUnitRows + (int)rank * (kNT * kBM);  // this CTA's rows
  volatile int* abort = &sm.abort;

  int kv_len = p.S_kv;
  if (p.flags & ANIMA_FLAG_MASK) kv_len = min(max(p.kv_valid[b], 0), p.S_kv);
  int n_kv = (kv_len + kBN - 1) / kBN;
  if (p.flags & ANIMA_FLAG_CAUSAL) {  // the pair agrees on the tile count of its 512 rows
    const int last_row = min((unit % p.nqb) * kUnitRows + kUnitRows, p.S_q) - 1;
    n_kv = min(n_kv, last_row / kBN + 1);
  }

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 2);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 2);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int i = 0; i < kNT; ++i) {
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.p_full[i], 2 * kBM);
      mbar_init(&sm.o_full[i], 1);
    }
    mbar_init(&sm.mma_done, 1);
    sm.abort = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc_pair(&sm.tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist and the pair's TMEM is allocated
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  // The leader's barriers that both CTAs of the pair arrive on.
  const uint32_t lead_q_full = mapa_shared(smem_u32(&sm.q_full), 0);
  const uint32_t lead_kv_full0 = mapa_shared(smem_u32(&sm.kv_full[0]), 0);
  const uint32_t lead_p_full0 = mapa_shared(smem_u32(&sm.p_full[0]), 0);

  if (warp >= 8) {
    regs_dec<kRegsControl>();
    if (warp == kKvWarp && lane == 0 && n_kv > 0) {
      // ------------------------------------------------ K/V producer: this CTA's halves
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_v);
      int item = 0;
      bool ok = true;
      for (int j = 0; j < n_kv && ok; ++j) {
        for (int kind = 0; kind < 2; ++kind, ++item) {
          const int slot = item % kStages;
          const uint32_t round = (uint32_t)(item / kStages);
          if (!mbar_wait_cluster(&sm.kv_empty[slot], (round & 1u) ^ 1u, abort, p.status,
                                 ANIMA_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          const uint32_t full = lead_kv_full0 + slot * 8;
          mbar_arrive_expect_tx_cluster(full, kSlot);
          if (kind == 0) {  // K: keys [128j + 64r, +64), both head-dim panels
            const int y = j * kBN + (int)rank * 64;
            tma_load_3d_pair(sm.kv[slot], &tmap_k, full, 0, y, bh);
            tma_load_3d_pair(sm.kv[slot] + kKPanel, &tmap_k, full, 64, y, bh);
          } else {          // V: keys [128j, +128), head-dim panel r
            tma_load_3d_pair(sm.kv[slot], &tmap_v, full, (int)rank * 64, j * kBN, bh);
          }
        }
      }
      // Copies of this CTA complete on the leader's barrier.  Each slot's last copy has
      // landed once the leader released that slot; wait (bounded) for those releases so
      // no copy into this CTA's shared memory is in flight when it exits.
      for (int s = 0; s < kStages; ++s) {
        int last = -1;
        for (int c = s; c < item; c += kStages) last = c;
        if (last >= 0) drain_wait(&sm.kv_empty[s], (uint32_t)(last / kStages) & 1u);
      }
    } else if (warp == kQWarp && lane == 0 && n_kv > 0) {
      // ------------------------------------------------ Q producer: this CTA's 2 tiles
      tma_prefetch_desc(&tmap_q);
      mbar_arrive_expect_tx_cluster(lead_q_full, kNT * kQTile);
      for (int i = 0; i < kNT; ++i)
        for (int pn = 0; pn < 2; ++pn)
          tma_load_3d_pair(sm.q[i] + pn * kQPanel, &tmap_q, lead_q_full, pn * 64, q0 + i * kBM, bh);
    } else if (warp == kMmaWarp && lane == 0 && rank == 0 && n_kv > 0) {
      // ------------------------------------------------ MMA issuer (leader only)
      constexpr uint32_t ab = kOp == ANIMA_DTYPE_BF16 ? 1u : 0u;
      constexpr uint32_t idesc_qk = make_idesc_f16(ab, 2 * kBM, kBN, 0);  // M 256, N 128 keys
      constexpr uint32_t idesc_pv = make_idesc_f16(ab, 2 * kBM, kD, 1);   // M 256, N 128 dims
      const uint32_t q_base = smem_u32(sm.q[0]);
      const uint32_t kv_base = smem_u32(sm.kv[0]);
      auto issue_qk = [&](int i, int slot) {
        const uint32_t d = tmem + i * 128;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t ao = (kk >> 2) * kQPanel + (kk & 3) * 32;
          const uint32_t bo = (kk >> 2) * kKPanel + (kk & 3) * 32;
          umma_ss_pair(d, sdesc_sw128(q_base + i * kQTile + ao, 16, 1024),
                       sdesc_sw128(kv_base + slot * kSlot + bo, 16, 1024), idesc_qk, kk > 0);
        }
      };
      auto issue_pv = [&](int i, int slot, bool acc) {
        const uint32_t d = tmem + 256 + i * 128;
        const uint32_t a = tmem + i * 128;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          umma_ts_pair(d, a + kk * 8, sdesc_sw128(kv_base + slot * kSlot + kk * 2048, kSlot, 1024),
                       idesc_pv, (acc || kk > 0) ? 1u : 0u);
      };
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return mbar_wait_cluster(bar, parity, abort, p.status, ANIMA_ERR_TIMEOUT);
      };
      auto slot_of = [](int item) { return item % kStages; };
      auto par_of = [](int item) { return (uint32_t)(item / kStages) & 1u; };
      bool ok = wait(&sm.q_full, 0);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int ik = 2 * j;
        if (!(ok = wait(&sm.kv_full[slot_of(ik)], par_of(ik)))) break;
        if (j == 0) {
          tc_fence_after();
          issue_qk(0, slot_of(ik));
          umma_commit_pair(&sm.s_full[0], 0x3);
          issue_qk(1, slot_of(ik));
          umma_commit_pair(&sm.s_full[1], 0x3);
          umma_commit_pair(&sm.kv_empty[slot_of(ik)], 0x3);
        } else {
          const int iv = 2 * (j - 1) + 1;
          const uint32_t pp = (uint32_t)(j - 1) & 1u;
          ok = wait(&sm.kv_full[slot_of(iv)], par_of(iv)) && wait(&sm.p_full[0], pp);
          if (!ok) break;
          tc_fence_after();
          issue_pv(0, slot_of(iv), j > 1);
          issue_qk(0, slot_of(ik));
          umma_commit_pair(&sm.s_full[0], 0x3);
          if (!(ok = wait(&sm.p_full[1], pp))) break;
          tc_fence_after();
          issue_pv(1, slot_of(iv), j > 1);
          umma_commit_pair(&sm.kv_empty[slot_of(iv)], 0x3);
          issue_qk(1, slot_of(ik));
          umma_commit_pair(&sm.s_full[1], 0x3);
          umma_commit_pair(&sm.kv_empty[slot_of(ik)], 0x3);
        }
      }
      if (ok) {
        const int iv = 2 * (n_kv - 1) + 1;
        const uint32_t pp = (uint32_t)(n_kv - 1) & 1u;
        ok = wait(&sm.kv_full[slot_of(iv)], par_of(iv)) && wait(&sm.p_full[0], pp);
        if (ok) {
          tc_fence_after();
          issue_pv(0, slot_of(iv), n_kv > 1);
          umma_commit_pair(&sm.o_full[0], 0x3);
          if (wait(&sm.p_full[1], pp)) {
            tc_fence_after();
            issue_pv(1, slot_of(iv), n_kv > 1);
            umma_commit_pair(&sm.o_full[1], 0x3);
            umma_commit_pair(&sm.kv_empty[slot_of(iv)], 0x3);
          }
        }
      }
      umma_commit_pair(&sm.mma_done, 0x3);
    }
    __syncwarp();
    if (warp == kMmaWarp && lane == 0 && n_kv > 0) drain_wait(&sm.mma_done, 0);
    __syncwarp();
    tc_fence_before();
    cluster_sync();  // no CTA leaves while its pair may still touch its smem or TMEM
    if (warp == kMmaWarp) {
      tc_fence_after();
      tmem_dealloc_pair(tmem, kTmemCols);
    }
    return;
  } else {
    regs_inc<kRegsSoftmax>();
    const int i = warp >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_field = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_field + i * 128;
    const uint32_t tO = tmem + lane_field + 256 + i * 128;
    const bool causal = (p.flags & ANIMA_FLAG_CAUSAL) != 0;
    const float sl2 = p.scale_log2;
    const int grow = q0 + i * kBM + row;
    const uint32_t p_full_lead = lead_p_full0 + i * 8;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int jj = 0; jj < n_kv; ++jj) {
      const int j = jj;
      const bool got = mbar_wait_cluster(&sm.s_full[i], (uint32_t)jj & 1u, abort, p.status,
                                         ANIMA_ERR_TIMEOUT);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, r[c]);
      tmem_ld_wait();
      int lim = kv_len - j * kBN;
      if (causal) lim = min(lim, grow - j * kBN + 1);
      const bool full = lim >= kBN;
      if (!full) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (c * 32 + e >= lim) r[c][e] = __float_as_uint(-INFINITY);
      }
#define SV(e) __uint_as_float(r[(e) >> 5][(e) & 31])
      // Row max: 8 independent 3-input-max chains, then a small tree.
      float acc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = fmaxf(SV(2 * k), SV(2 * k + 1));
#pragma unroll
      for (int e = 16; e < 128; e += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] = max3f(acc[k], SV(e + 2 * k), SV(e + 2 * k + 1));
      const float mx = max3f(max3f(acc[0], acc[1], acc[2]), max3f(acc[3], acc[4], acc[5]),
                             fmaxf(acc[6], acc[7]));
      const float m_tile = mx * sl2;
      float m_use = m, alpha = 1.f;
      if (m == -INFINITY) {
        m_use = m_tile;
        alpha = 0.f;
      } else if (m_tile > m + kRescaleThreshold) {
        m_use = m_tile;
        alpha = ex2_approx(m - m_tile);
      }
      const float neg_base = (m_use == -INFINITY) ? 0.f : -m_use;
      const uint64_t scale2 = f2pack(sl2, sl2), base2 = f2pack(neg_base, neg_base);
      uint64_t sum2[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) sum2[k] = 0ull;
      // P = 2^(s*scale*log2e - m): pairs of columns through the packed FMA pipe; in full
      // tiles kPolyPer8 of every 8 pairs take the polynomial exp2, the rest MUFU ex2.
      uint32_t pk[2][32];
      if (full) {
#pragma unroll
        for (int pr = 0; pr < 64; ++pr) {
          float x0, x1;
          f2unpack(fma2(f2pack(SV(2 * pr), SV(2 * pr + 1)), scale2, base2), x0, x1);
          if ((pr & 7) < kPolyPer8) {
            exp2_poly_pair(x0, x1);
          } else {
            x0 = ex2_approx(x0);
            x1 = ex2_approx(x1);
          }
          sum2[pr & 3] = add2(sum2[pr & 3], f2pack(x0, x1));
          pk[pr >> 5][pr & 31] = pack2<kOp>(x0, x1);
        }
      } else {
#pragma unroll
        for (int pr = 0; pr < 64; ++pr) {
          float x0, x1;
          f2unpack(fma2(f2pack(SV(2 * pr), SV(2 * pr + 1)), scale2, base2), x0, x1);
          x0 = ex2_approx(x0);
          x1 = ex2_approx(x1);
          sum2[pr & 3] = add2(sum2[pr & 3], f2pack(x0, x1));
          pk[pr >> 5][pr & 31] = pack2<kOp>(x0, x1);
        }
      }
      tmem_st32(tS, pk[0]);
      tmem_st32(tS + 32, pk[1]);
#undef SV
      float sa, sb;
      f2unpack(add2(add2(sum2[0], sum2[1]), add2(sum2[2], sum2[3])), sa, sb);
      const float sum = sa + sb;
      l = l * alpha + sum;
      if (__any_sync(0xffffffffu, jj > 0 && alpha != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(tO + c * 32, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive_cluster(p_full_lead);
      m = m_use;
    }
    if (ok && n_kv > 0) {
      const bool got = mbar_wait_cluster(&sm.o_full[i], 0, abort, p.status, ANIMA_ERR_TIMEOUT);
      ok = __all_sync(0xffffffffu, got);
      tc_fence_after();
    }
    if (ok) {
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      char* out_row = reinterpret_cast<char*>(p.out) +
                      ((long long)b * p.ob + (long long)(bh % p.H) * p.oh + (long long)grow * p.os) *
                          (kOut == ANIMA_DTYPE_F32 ? 4 : 2);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        if (n_kv > 0) {
          tmem_ld32(tO + c * 32, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (grow < p.S_q) store_row<kOut>(out_row, o, c, inv);
      }
    }
    tc_fence_before();
    cluster_sync();  // pairs with the control warpgroup's teardown
  }
}

}  // namespace attn2

// ---------------------------------------------------------------- host launcher
typedef CUresult (*EncodeTiledFn2)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn2 get_encode_fn2() {
  static EncodeTiledFn2 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<EncodeTiledFn2>(ptr);
  }
  return fn;
}

// [bh][rows][128] 16-bit tensor, box [64 elements][box_rows rows][1], 128-byte swizzle.
static int make_map2(CUtensorMap* map, const void* base, int op_dtype, int bh, int rows,
                     int box_rows) {
  EncodeTiledFn2 enc = get_encode_fn2();
  if (!enc) return ANIMA_ERR_CUDA;
  const CUtensorMapDataType dt = op_dtype == ANIMA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)bh};
  cuuint64_t strides[2] = {128 * 2, (cuuint64_t)rows * 128 * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ANIMA_OK : ANIMA_ERR_CUDA;
}

template <int kOp, int kOut>
static int launch_pair(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                       const attn2::Params& prm, int grid, cudaStream_t st) {
  auto kern = attn2::attn_fwd_pair_kernel<kOp, kOut>;
  static int attr_dev_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask & (1 << (dev & 31)))) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)attn2::kSmemBytes) != cudaSuccess)
      return ANIMA_ERR_CUDA;
    attr_dev_mask |= 1 << (dev & 31);
  }
  kern<<<grid, attn2::kThreads, attn2::kSmemBytes, st>>>(mq, mk, mv, prm);
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

// One cluster (CTA pair) per 512-row unit.
int attn_fwd_pair_launch(const AnimaAttnArgs* a, int* status, cudaStream_t st) {
  if (a->D != attn2::kD) return ANIMA_ERR_SHAPE;
  if (a->op_dtype != ANIMA_DTYPE_BF16 && a->op_dtype != ANIMA_DTYPE_F16) return ANIMA_ERR_ARG;
  const int bh = a->B * a->H;
  if (a->B <= 0 || a->H <= 0 || a->S_q <= 0 || a->S_kv <= 0) return ANIMA_ERR_SHAPE;
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = make_map2(&mq, a->q, a->op_dtype, bh, a->S_q, 128))) return rc;
  if ((rc = make_map2(&mk, a->k, a->op_dtype, bh, a->S_kv, 64))) return rc;
  if ((rc = make_map2(&mv, a->v, a->op_dtype, bh, a->S_kv, 128))) return rc;
  attn2::Params prm;
  prm.B = a->B;
  prm.H = a->H;
  prm.S_q = a->S_q;
  prm.S_kv = a->S_kv;
  prm.scale_log2 = a->scale * 1.4426950408889634f;
  prm.flags = a->flags;
  prm.kv_valid = a->kv_valid_len;
  prm.out = a->out;
  prm.ob = a->out_stride[0];
  prm.oh = a->out_stride[1];
  prm.os = a->out_stride[2];
  prm.status = status;
  prm.nqb = (a->S_q + attn2::kUnitRows - 1) / attn2::kUnitRows;
  const long long units = (long long)bh * prm.nqb;
  if (2 * units > 0x7fffffffLL) return ANIMA_ERR_SHAPE;
  const int grid = (int)(2 * units);
  const bool bf = a->op_dtype == ANIMA_DTYPE_BF16;
  switch (a->out_dtype) {
    case ANIMA_DTYPE_F32:
      return bf ? launch_pair<ANIMA_DTYPE_BF16, ANIMA_DTYPE_F32>(mq, mk, mv, prm, grid, st)
                : launch_pair<ANIMA_DTYPE_F16, ANIMA_DTYPE_F32>(mq, mk, mv, prm, grid, st);
    case ANIMA_DTYPE_BF16:
      return bf ? launch_pair<ANIMA_DTYPE_BF16, ANIMA_DTYPE_BF16>(mq, mk, mv, prm, grid, st)
                : launch_pair<ANIMA_DTYPE_F16, ANIMA_DTYPE_BF16>(mq, mk, mv, prm, grid, st);
    case ANIMA_DTYPE_F16:
      return bf ? launch_pair<ANIMA_DTYPE_BF16, ANIMA_DTYPE_F16>(mq, mk, mv, prm, grid, st)
                : launch_pair<ANIMA_DTYPE_F16, ANIMA_DTYPE_F16>(mq, mk, mv, prm, grid, st);
  }
  return ANIMA_ERR_ARG;
}

}  // namespace anima
