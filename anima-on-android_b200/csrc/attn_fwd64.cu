// attn_fwd64.cu -- flash-attention forward for sm_100a with 64-key tiles and P in tensor
// memory columns of its own (ANIMA_FLAG_KV64).  Same call, schedules, softmax arithmetic
// and epilogue as attn_fwd.cu (anima::cpu::flash_attention,
// anima_rt/include/cpu/flash_attention.h:55-208); what differs is the per-tile chain.
//
// In attn_fwd.cu, P_i(j) overlays S_i, so QK^T_i(j+1), which rewrites S_i, can only start
// once PV_i(j) has read P_i(j): per key tile, a query tile's softmax, its PV and its next
// QK^T run one after the other, and the tensor pipe idles for part of every step.  Here
// each query tile i owns 256 tensor-memory columns (base 256 i):
//     S_i  [0, 64)     fp32 scores of one 64-key tile
//     P_i  [64, 96) and [96, 128)   16-bit pairs, two buffers used by alternate steps
//     O_i  [128, 256)  fp32 accumulator
// The softmax copies S_i(j) into registers and signals s_free at once, so QK^T_i(j+1) is
// issued while the softmax of step j still runs; PV_i(j) follows when P_i(j) is stored.
// Each query tile has its own MMA-issuing thread (warp 9 for tile 0, warp 11 for tile 1),
// so neither tile's MMAs queue behind the other's softmax.  The softmax keeps its scores
// in registers for the rare re-check of the running max, and waits for PV_i(j-1) only
// when it must rescale O_i.  P buffer b has its own p_full / pv_done barriers, completed
// once per use of the buffer (every other step): a softmax that runs a step ahead of the
// MMA thread can then never advance a barrier by two phases before it is waited on.
//
// Per 64-key step and query tile the tensor pipe runs QK^T (M128 N64 K128: 8 MMAs) and
// PV (M128 N128 K64: 4 MMAs), 256 cycles each.  K and V tiles are 16 KB; the ring holds 8.
// Warp roles, register split, schedules and the output epilogue are those of
// attn_shared.cuh.
#include "attn_shared.cuh"

namespace anima {
namespace attn64 {
using namespace attn;

constexpr int kBN = 64;                   // keys per K/V tile
constexpr int kStages = 8;                // K/V ring slots
constexpr int kQPanel = 128 * 128;        // Q: [128 rows][64 x 16-bit], 128B-swizzled = 16 KB
constexpr int kQTile = 2 * kQPanel;       // [128 rows][128 x 16-bit] = 32 KB
constexpr int kKvPanel = 64 * 128;        // K/V: [64 rows][64 x 16-bit] = 8 KB
constexpr int kKvTile = 2 * kKvPanel;     // [64 rows][128 x 16-bit] = 16 KB
constexpr int kColS = 0, kColP = 64, kColO = 128, kTileCols = 256;
constexpr int kMmaWarp1 = 11;             // MMA issuer of query tile 1 (warp 9: tile 0)

struct Smem {
  uint8_t q[kNT][kQTile];
  uint8_t kv[kStages][kKvTile];
  float4 stage[8][256];  // per softmax warp: one 32 x 32 fp32 block on its way to global
  uint64_t q_full, q_empty;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[kNT];   // QK^T_i done: S_i holds the step's scores
  uint64_t s_free[kNT];   // the softmax has S_i in registers: S_i may be rewritten
  uint64_t p_full[kNT][2];   // P_i stored in buffer b (steps b, b+2, ...)
  uint64_t pv_done[kNT][2];  // PV_i that read buffer b done
  uint64_t o_full[kNT];   // the segment's last PV_i done: O_i final
  uint64_t o_empty[kNT];  // the epilogue has read O_i
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + slack to align the base to 1 KB
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

// Four chained MMAs D (+)= A_k * B_k with A in tensor memory (one 64-deep K block in
// 16-deep steps); the first accumulates iff acc0 != 0, the rest always do.
__device__ __forceinline__ void umma_ts_x4(uint32_t d, const uint32_t (&a)[4],
                                           const uint64_t (&b)[4], uint32_t idesc,
                                           uint32_t acc0) {
  asm volatile(
      "{\n\t.reg .pred p0, p1;\n\t"
      "setp.ne.b32 p0, %10, 0;\n\t"
      "setp.eq.b32 p1, %10, %10;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %5, %9, p0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %6, %9, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%3], %7, %9, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %8, %9, p1;\n\t}" ::"r"(d),
      "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]),
      "r"(idesc), "r"(acc0)
      : "memory");
}

template <int kOp, int kOut>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd64_kernel(const __grid_constant__ CUtensorMap tmap_q,
                      const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + pad);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort = &sm.abort;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_empty, kNT);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], kNT);  // one commit from each tile's MMA thread
    }
    for (int i = 0; i < kNT; ++i) {
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_free[i], kBM);
      for (int b = 0; b < 2; ++b) {
        mbar_init(&sm.p_full[i][b], kBM);
        mbar_init(&sm.pv_done[i][b], 1);
      }
      mbar_init(&sm.o_full[i], 1);
      mbar_init(&sm.o_empty[i], kBM);
    }
    mbar_init(&sm.mma_done, kNT);
    sm.abort = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp >= 8) {
    regs_dec<kRegsControl>();
    if (warp == kKvWarp && lane == 0) {
      // ---------------------------------------------------------- K/V producer
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_v);
      SegIter<kBN> it(p);
      Seg sg;
      int item = 0;  // K of tile-step g is item 2g, V is item 2g+1
      bool ok = true;
      while (ok && it.next(p, sg)) {
        const int bh = sg.unit / p.nqb;
        for (int j = sg.k0; j < sg.k1 && ok; ++j) {
          for (int kind = 0; kind < 2; ++kind, ++item) {
            const int slot = item % kStages;
            const uint32_t round = (uint32_t)(item / kStages);
            if (!mbar_wait(&sm.kv_empty[slot], (round & 1u) ^ 1u, abort, p.status,
                           ANIMA_ERR_TIMEOUT)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&sm.kv_full[slot], kKvTile);
            const CUtensorMap* m = kind ? &tmap_v : &tmap_k;
            tma_load_3d(sm.kv[slot], m, &sm.kv_full[slot], 0, j * kBN, bh);
            tma_load_3d(sm.kv[slot] + kKvPanel, m, &sm.kv_full[slot], 64, j * kBN, bh);
          }
        }
      }
      // Every copy this thread started must land before the CTA may exit.
      for (int s = 0; s < kStages; ++s) {
        int last = -1;
        for (int c = s; c < item; c += kStages) last = c;
        if (last >= 0) drain_wait(&sm.kv_full[s], (uint32_t)(last / kStages) & 1u);
      }
    } else if (warp == kQWarp && lane == 0) {
      // ---------------------------------------------------------- Q producer
      tma_prefetch_desc(&tmap_q);
      SegIter<kBN> it(p);
      Seg sg;
      int a = 0;  // active (non-empty) segments so far
      bool ok = true;
      while (ok && it.next(p, sg)) {
        if (sg.k1 <= sg.k0) continue;
        if (a > 0 && !mbar_wait(&sm.q_empty, (uint32_t)(a - 1) & 1u, abort, p.status,
                                ANIMA_ERR_TIMEOUT)) {
          ok = false;
          break;
        }
        const int bh = sg.unit / p.nqb;
        const int q0 = (sg.unit % p.nqb) * kUnitRows;
        mbar_arrive_expect_tx(&sm.q_full, kNT * kQTile);
        for (int i = 0; i < kNT; ++i)
          for (int pn = 0; pn < 2; ++pn)
            tma_load_3d(sm.q[i] + pn * kQPanel, &tmap_q, &sm.q_full, pn * 64, q0 + i * kBM, bh);
        ++a;
      }
      if (a > 0) drain_wait(&sm.q_full, (uint32_t)(a - 1) & 1u);
    } else if ((warp == kMmaWarp || warp == kMmaWarp1) && lane == 0) {
      // ---------------------------------------------------------- MMA issuer of tile i
      const int i = warp == kMmaWarp ? 0 : 1;
      constexpr uint32_t ab = kOp == ANIMA_DTYPE_BF16 ? 1u : 0u;  // idesc: 0 f16, 1 bf16
      constexpr uint32_t idesc_qk = make_idesc_f16(ab, kBM, kBN, 0);
      constexpr uint32_t idesc_pv = make_idesc_f16(ab, kBM, kD, 1);
      // K-major K tile: K-step kk starts at panel kk / 4, 32 bytes per step inside it;
      // MN-major V tile: K-step kk (16 keys) at row 16 kk, 2 KiB per step; its two
      // 64-dimension panels are kKvPanel apart.
      const uint64_t dk0 = sdesc_sw128(smem_u32(sm.kv[0]), 16, 1024);
      const uint64_t dv0 = sdesc_sw128(smem_u32(sm.kv[0]), kKvPanel, 1024);
      uint64_t dq[8];
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        dq[kk] = sdesc_sw128(smem_u32(sm.q[i]) + (kk >> 2) * kQPanel + (kk & 3) * 32, 16, 1024);
      const uint32_t tS = tmem + i * kTileCols + kColS;
      const uint32_t tP = tmem + i * kTileCols + kColP;
      const uint32_t tO = tmem + i * kTileCols + kColO;

      auto issue_qk = [&](int slot) {
        const uint64_t kb = desc_plus(dk0, (uint32_t)slot * kKvTile);
        uint64_t b[8];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) b[kk] = desc_plus(kb, (kk >> 2) * kKvPanel + (kk & 3) * 32);
        umma_ss_x8(tS, dq, b, idesc_qk, 0u);
      };
      auto issue_pv = [&](int slot, int buf, bool acc) {
        const uint64_t vb = desc_plus(dv0, (uint32_t)slot * kKvTile);
        uint64_t b[4];
        uint32_t a[4];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          b[kk] = desc_plus(vb, kk * 2048);
          a[kk] = tP + buf * 32 + kk * 8;  // 16 keys per step
        }
        umma_ts_x4(tO, a, b, idesc_pv, acc ? 1u : 0u);
      };
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return mbar_wait(bar, parity, abort, p.status, ANIMA_ERR_TIMEOUT);
      };
      auto slot_of = [](int item) { return item % kStages; };
      auto par_of = [](int item) { return (uint32_t)(item / kStages) & 1u; };

      SegIter<kBN> it(p);
      Seg sg;
      int g = 0;  // global tile-step counter
      int a = 0;  // active segments so far
      bool ok = true;
      while (ok && it.next(p, sg)) {
        const int n = sg.k1 - sg.k0;
        if (n <= 0) continue;
        const uint32_t pa = (uint32_t)(a - 1) & 1u;  // parity of the previous segment
        if (!(ok = wait(&sm.q_full, (uint32_t)a & 1u))) break;
        // Scores of the segment's first key tile, once the softmax has taken the previous
        // step's scores into registers.
        {
          const int ik = 2 * g;
          if (!(ok = wait(&sm.kv_full[slot_of(ik)], par_of(ik)))) break;
          if (g > 0 && !(ok = wait(&sm.s_free[i], (uint32_t)(g - 1) & 1u))) break;
          tc_fence_after();
          issue_qk(slot_of(ik));
          umma_commit(&sm.s_full[i]);
          umma_commit(&sm.kv_empty[slot_of(ik)]);
          if (n == 1) umma_commit(&sm.q_empty);
        }
        for (int jj = 0; jj < n && ok; ++jj) {
          const int gj = g + jj;
          const int ik = 2 * (gj + 1), iv = 2 * gj + 1;
          const bool more = jj + 1 < n;
          // next scores, then this step's P V
          if (more) {
            ok = wait(&sm.kv_full[slot_of(ik)], par_of(ik)) && wait(&sm.s_free[i], (uint32_t)gj & 1u);
            if (!ok) break;
            tc_fence_after();
            issue_qk(slot_of(ik));
            umma_commit(&sm.s_full[i]);
            umma_commit(&sm.kv_empty[slot_of(ik)]);
            if (jj + 2 == n) umma_commit(&sm.q_empty);  // the segment's last QK^T issued
          }
          ok = wait(&sm.kv_full[slot_of(iv)], par_of(iv)) &&
               wait(&sm.p_full[i][gj & 1], (uint32_t)(gj >> 1) & 1u);
          if (ok && jj == 0 && a > 0) ok = wait(&sm.o_empty[i], pa);
          if (!ok) break;
          tc_fence_after();
          issue_pv(slot_of(iv), gj & 1, jj > 0);
          umma_commit(&sm.pv_done[i][gj & 1]);
          umma_commit(&sm.kv_empty[slot_of(iv)]);
          if (!more) umma_commit(&sm.o_full[i]);
        }
        if (!ok) break;
        g += n;
        ++a;
      }
      // Let every MMA this thread issued retire (and the other issuer's) before TMEM is
      // released.
      umma_commit(&sm.mma_done);
      drain_wait(&sm.mma_done, 0);
    }
    __syncwarp();
    // Teardown of the control warpgroup: TMEM is released once every warp is done.
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
      tc_fence_after();
      tmem_dealloc(tmem, kTmemCols);
    }
    return;
  } else {
    regs_inc<kRegsSoftmax>();
    // ------------------------------------------------------------ softmax / epilogue
    const int i = warp >> 2;            // query tile of this warpgroup
    const int quarter = warp & 3;       // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const uint32_t lane_field = (uint32_t)(quarter * 32) << 16;
    const uint32_t tbase = tmem + lane_field + i * kTileCols;
    const uint32_t tS = tbase + kColS, tP = tbase + kColP, tO = tbase + kColO;
    const bool causal = (p.flags & ANIMA_FLAG_CAUSAL) != 0;
    const float sl2 = p.scale_log2;

    SegIter<kBN> it(p);
    Seg sg;
    int g = 0;
    int a = 0;
    bool ok = true;
    while (ok && it.next(p, sg)) {
      const int bh = sg.unit / p.nqb;
      const int b = bh / p.H;
      const int grow = (sg.unit % p.nqb) * kUnitRows + i * kBM + row;
      const int kv_len = unit_kv_len(p, sg.unit);
      const int n = sg.k1 - sg.k0;
      float m = -INFINITY;  // running max, scaled log2 units
      float l = 0.f;        // running sum of P
      for (int jj = 0; jj < n; ++jj, ++g) {
        const int j = sg.k0 + jj;  // key tile index within the unit
        const bool got = mbar_wait(&sm.s_full[i], (uint32_t)g & 1u, abort, p.status,
                                   ANIMA_ERR_TIMEOUT);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r[2][32];
        tmem_ld32(tS, r[0]);
        tmem_ld32(tS + 32, r[1]);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(&sm.s_free[i]);  // the scores live in r now
        int lim = kv_len - j * kBN;
        if (causal) lim = min(lim, grow - j * kBN + 1);
        const bool full = lim >= kBN;
        if (!full) {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (c * 32 + e >= lim) r[c][e] = __float_as_uint(-INFINITY);
        }
#define SV(e) __uint_as_float(r[(e) >> 5][(e) & 31])
        // Row max: 8 independent 3-input-max chains, then a small tree.
        auto row_max = [&]() {
          float acc[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) acc[k] = fmaxf(SV(2 * k), SV(2 * k + 1));
#pragma unroll
          for (int e = 16; e < kBN; e += 16)
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[k] = max3f(acc[k], SV(e + 2 * k), SV(e + 2 * k + 1));
          return max3f(max3f(acc[0], acc[1], acc[2]), max3f(acc[3], acc[4], acc[5]),
                       fmaxf(acc[6], acc[7]));
        };
        uint64_t sum2[4];
        uint32_t pk[32];
        // P = 2^(s*scale*log2e - mu) for pairs of columns through the packed FMA pipe, the
        // row sum and the 16-bit pack, in one pass over the scores in r (which it keeps).
        auto exp_pass = [&](float mu) {
          const float nb = (mu == -INFINITY) ? 0.f : -mu;
          const uint64_t scale2 = f2pack(sl2, sl2), base2 = f2pack(nb, nb);
#pragma unroll
          for (int k = 0; k < 4; ++k) sum2[k] = 0ull;
#pragma unroll
          for (int pr = 0; pr < kBN / 2; ++pr) {
            float x0, x1;
            f2unpack(fma2(f2pack(SV(2 * pr), SV(2 * pr + 1)), scale2, base2), x0, x1);
            if (full && (pr & 7) < kPolyPer8) {
              exp2_poly_pair(x0, x1);
            } else {
              x0 = ex2_approx(x0);
              x1 = ex2_approx(x1);
            }
            sum2[pr & 3] = add2(sum2[pr & 3], f2pack(x0, x1));
            pk[pr] = pack2<kOp>(x0, x1);
          }
        };
        auto row_sum = [&]() {
          float sa, sb;
          f2unpack(add2(add2(sum2[0], sum2[1]), add2(sum2[2], sum2[3])), sa, sb);
          return sa + sb;
        };
        // Online softmax with the lazy rescale and sum-certified running max of
        // attn_fwd.cu: the first tile of a segment takes its row max first; later tiles
        // compute P with the running max m and keep it if the row sum certifies that no P
        // exceeds 2^kRescaleThreshold, else redo the pass with the exact tile max (from
        // the scores still in registers) under the lazy rule.
        float m_use = m, alpha = 1.f, sum;
        if (jj == 0) {
          m_use = row_max() * sl2;
          alpha = 0.f;  // nothing accumulated yet
          exp_pass(m_use);
          sum = row_sum();
        } else {
          exp_pass(m);
          sum = row_sum();
          const bool check = !(sum <= 256.f) || (m == -INFINITY && sum > 0.f);
          if (__any_sync(0xffffffffu, check)) {
            const float m_tile = row_max() * sl2;
            if (m == -INFINITY) {
              m_use = m_tile;
              alpha = 0.f;
            } else if (m_tile > m + kRescaleThreshold) {
              m_use = m_tile;
              alpha = ex2_approx(m - m_tile);
            }
            exp_pass(m_use);
            sum = row_sum();
          }
        }
#undef SV
        l = l * alpha + sum;
        // The P buffer of this step was last read by PV_i(g-2).  (Its completion is also
        // implied by S_i(g): the tile's MMA thread issued QK^T_i(g) after PV_i(g-2), and
        // its MMAs run in order; the wait never stalls.)
        if (g >= 2) {
          const bool got2 = mbar_wait(&sm.pv_done[i][g & 1], (uint32_t)((g - 2) >> 1) & 1u,
                                      abort, p.status, ANIMA_ERR_TIMEOUT);
          if (!__all_sync(0xffffffffu, got2)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        if (__any_sync(0xffffffffu, jj > 0 && alpha != 1.f)) {
          // O_i must hold PV_i(g-1) before it is rescaled.
          const bool got3 = mbar_wait(&sm.pv_done[i][(g - 1) & 1], (uint32_t)((g - 1) >> 1) & 1u,
                                      abort, p.status, ANIMA_ERR_TIMEOUT);
          if (!__all_sync(0xffffffffu, got3)) {
            ok = false;
            break;
          }
          tc_fence_after();
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
        tmem_st32(tP + (g & 1) * 32, pk);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&sm.p_full[i][g & 1]);
        m = m_use;
      }
      if (!ok) break;
      if (n > 0) {
        const bool got = mbar_wait(&sm.o_full[i], (uint32_t)a & 1u, abort, p.status,
                                   ANIMA_ERR_TIMEOUT);
        if (!(ok = __all_sync(0xffffffffu, got))) break;
        tc_fence_after();
      }
      segment_epilogue<kOut>(p, sg, n, i, row, lane, b, bh, grow, tO, m, l, sm.stage[warp]);
      if (n > 0) {
        tc_fence_before();
        mbar_arrive(&sm.o_empty[i]);
        ++a;
      }
    }
    tc_fence_before();
    __syncthreads();  // pairs with the control warpgroup's teardown barrier
  }
}

template <int kOp, int kOut>
static int launch_t(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                    const Params& prm, int grid, cudaStream_t st) {
  auto kern = attn_fwd64_kernel<kOp, kOut>;
  static int attr_dev_mask = 0;  // devices on which the smem attribute was raised
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask & (1 << (dev & 31)))) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemBytes) != cudaSuccess)
      return ANIMA_ERR_CUDA;
    attr_dev_mask |= 1 << (dev & 31);
  }
  kern<<<grid, kThreads, kSmemBytes, st>>>(mq, mk, mv, prm);
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

}  // namespace attn64

// Launch of the 64-key-tile kernel; the caller built K/V maps with 64-row boxes and
// counted prm.n_kv / the cut slices in 64-key tiles.
int attn64_launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                  const attn::Params& prm, int grid, int op_dtype, int out_dtype,
                  cudaStream_t st) {
  const bool bf = op_dtype == ANIMA_DTYPE_BF16;
  switch (out_dtype) {
    case ANIMA_DTYPE_F32:
      return bf ? attn64::launch_t<ANIMA_DTYPE_BF16, ANIMA_DTYPE_F32>(mq, mk, mv, prm, grid, st)
                : attn64::launch_t<ANIMA_DTYPE_F16, ANIMA_DTYPE_F32>(mq, mk, mv, prm, grid, st);
    case ANIMA_DTYPE_BF16:
      return bf ? attn64::launch_t<ANIMA_DTYPE_BF16, ANIMA_DTYPE_BF16>(mq, mk, mv, prm, grid, st)
                : attn64::launch_t<ANIMA_DTYPE_F16, ANIMA_DTYPE_BF16>(mq, mk, mv, prm, grid, st);
    default:
      return bf ? attn64::launch_t<ANIMA_DTYPE_BF16, ANIMA_DTYPE_F16>(mq, mk, mv, prm, grid, st)
                : attn64::launch_t<ANIMA_DTYPE_F16, ANIMA_DTYPE_F16>(mq, mk, mv, prm, grid, st);
  }
}

}  // namespace anima
