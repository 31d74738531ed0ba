// attn_fwd.cu -- flash-attention forward for sm_100a: TMA-staged tiles, tcgen05.mma
// with TMEM accumulators, fp32 online softmax; non-causal, causal and key-padding
// masked.  Replaces anima::cpu::flash_attention
// (anima_rt/include/cpu/flash_attention.h:55-208): out = softmax(Q K^T * scale) V per
// (batch, head), D = 128.
//
// Work unit = 256 query rows (two 128-row tiles) of one (batch, head) against its keys,
// streamed in 128-key tiles.  Three schedules share one kernel (plan_split chooses):
//   unit         one CTA per unit (causal calls, long masked units, calls of at most one wave that
//                keep most SMs busy, and long units, where the hardware's dynamic hand-out
//                of CTAs balances best);
//   whole        a persistent grid of one CTA per SM.  Whole units are dealt round-robin
//                (CTA c takes units c, c+G, ...), so the CTAs in flight share heads and
//                their K/V stay in L2, and a CTA moves to its next unit without start-up;
//   cut          whole-unit rounds as above, and the units of the last, partial round cut
//                into equal slices of key tiles spread over all CTAs, so that round is not
//                left half idle.  A call of one wave that would leave most SMs idle (a few
//                heads per GPU) has no whole round: all its units are cut.  A CTA holding a slice writes an fp32 partial (O, running
//                max, running sum); the last warpgroup to finish a cut unit, told by an
//                arrival counter, merges the partials and writes the output.  No CTA waits
//                on another.
//
// Warp roles (384 threads, 3 warpgroups):
//   warps 0-7  two softmax warpgroups, one per query tile; thread = query row = TMEM
//              lane.  Reads its S row from TMEM, updates running max / sum, writes P
//              (16-bit) back over S, rescales its O row when the max moved, and at the
//              end of a segment stores O (or the partial) and frees O for the next one.
//   warp 8     TMA producer of K_j / V_j through a 4-slot ring.
//   warp 9     MMA issuer (one thread) + TMEM owner:
//                S_i  = Q_i K_j^T   (SS form, both operands in shared memory)
//                O_i += P_i V_j     (TS form, P read from tensor memory)
//   warp 10    TMA producer of the Q tiles of each segment.
//   warp 11    idle.  Warps 8-11 give registers to the softmax warpgroups (setmaxnreg).
//
// Tensor memory (512 columns x 128 lanes, fp32): S_0 [0,128) S_1 [128,256)
// O_0 [256,384) O_1 [384,512); P_i overlays the first 64 columns of S_i.  The two query
// tiles ping-pong: while warpgroup 0 runs the softmax of tile 0 the tensor core works
// on tile 1, and vice versa.
//
// Online softmax in the exp2 domain (scores scaled by scale*log2(e)) with a lazy
// rescale: the max used for P moves only when the new row max exceeds it by more than
// 8 (a factor 256), so the O correction is rare after the first tiles.
#include <algorithm>
#include <cstring>

#include "attn_shared.cuh"

namespace anima {
namespace attn {

constexpr int kBN = 128;               // keys per K/V tile
constexpr int kStages = 4;             // K/V ring slots
constexpr int kPanel = 128 * 128;      // [128 rows][64 x 16-bit], 128B-swizzled = 16 KB
constexpr int kTile = 2 * kPanel;      // [128 rows][128 x 16-bit] = 32 KB
constexpr int kMinSliceTiles = 4;       // shortest key-tile slice of the last round (512 keys)

struct Smem {
  uint8_t q[kNT][kTile];
  uint8_t kv[kStages][kTile];
  float4 stage[8][256];  // per softmax warp: one 32 x 32 fp32 block on its way to global
  uint64_t q_full, q_empty;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[kNT];
  uint64_t p_full[kNT];
  uint64_t o_full[kNT];
  uint64_t o_empty[kNT];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + slack to align the base to 1 KB
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");


template <int kOp, int kOut>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmap_q,
                    const __grid_constant__ CUtensorMap tmap_k,
                    const __grid_constant__ CUtensorMap tmap_v,
                    const __grid_constant__ CUtensorMap tmap_o, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + pad);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort = &sm.abort;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_empty, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int i = 0; i < kNT; ++i) {
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.p_full[i], kBM);
      mbar_init(&sm.o_full[i], 1);
      mbar_init(&sm.o_empty[i], kBM);
    }
    mbar_init(&sm.mma_done, 1);
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
  // Launched as a programmatic dependent of the kernel before it on the stream (the
  // prologue): the set-up above overlaps that kernel's tail; no global memory is touched
  // before the previous grid has completed and its writes are visible.
  grid_dependency_wait();

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
            const int slot = (int)(item % kStages);
            const uint32_t round = (uint32_t)(item / kStages);
            if (!mbar_wait(&sm.kv_empty[slot], (round & 1u) ^ 1u, abort, p.status,
                           ANIMA_ERR_TIMEOUT)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&sm.kv_full[slot], kTile);
            const CUtensorMap* m = kind ? &tmap_v : &tmap_k;
            tma_load_3d(sm.kv[slot], m, &sm.kv_full[slot], 0, j * kBN, bh);
            tma_load_3d(sm.kv[slot] + kPanel, m, &sm.kv_full[slot], 64, j * kBN, bh);
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
        mbar_arrive_expect_tx(&sm.q_full, kNT * kTile);
        for (int i = 0; i < kNT; ++i)
          for (int pn = 0; pn < 2; ++pn)
            tma_load_3d(sm.q[i] + pn * kPanel, &tmap_q, &sm.q_full, pn * 64, q0 + i * kBM, bh);
        ++a;
      }
      if (a > 0) drain_wait(&sm.q_full, (uint32_t)(a - 1) & 1u);
    } else if (warp == kMmaWarp && lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t ab = kOp == ANIMA_DTYPE_BF16 ? 1u : 0u;  // idesc: 0 f16, 1 bf16
      constexpr uint32_t idesc_qk = make_idesc_f16(ab, kBM, kBN, 0);
      constexpr uint32_t idesc_pv = make_idesc_f16(ab, kBM, kD, 1);
      // Descriptors are built once; per MMA only the start address moves (desc_plus).
      // K-step kk of a K-major tile starts at panel kk / 4, 32 bytes per step inside it;
      // of the MN-major V tile at row 16 * kk (2 KiB per step).
      const uint64_t dk0 = sdesc_sw128(smem_u32(sm.kv[0]), 16, 1024);      // K, slot 0
      const uint64_t dv0 = sdesc_sw128(smem_u32(sm.kv[0]), kPanel, 1024);  // V, slot 0
      const uint64_t dq0 = sdesc_sw128(smem_u32(sm.q[0]), 16, 1024);  // Q tile 0, step 0

      // The Q descriptors are recomputed per call (one add each) rather than held: a table
      // of all 16 held 32 registers of this thread's budget and made it spill.
      auto issue_qk = [&](int i, int slot) {
        const uint64_t kb = desc_plus(dk0, (uint32_t)slot * kTile);
        uint64_t b[8], aq[8];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          b[kk] = desc_plus(kb, (kk >> 2) * kPanel + (kk & 3) * 32);
          aq[kk] = desc_plus(dq0, (uint32_t)i * kTile + (kk >> 2) * kPanel + (kk & 3) * 32);
        }
        umma_ss_x8(tmem + i * 128, aq, b, idesc_qk, 0u);
      };
      auto issue_pv = [&](int i, int slot, bool acc) {
        const uint64_t vb = desc_plus(dv0, (uint32_t)slot * kTile);
        uint64_t b[8];
        uint32_t a[8];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          b[kk] = desc_plus(vb, kk * 2048);
          a[kk] = tmem + i * 128 + kk * 8;  // P_i, 16 keys (8 columns) per step
        }
        umma_ts_x8(tmem + 256 + i * 128, a, b, idesc_pv, acc ? 1u : 0u);
      };
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return mbar_wait(bar, parity, abort, p.status, ANIMA_ERR_TIMEOUT);
      };
      auto slot_of = [](int item) { return item % kStages; };
      auto par_of = [](int item) { return (uint32_t)(item / kStages) & 1u; };

      SegIter<kBN> it(p);
      Seg sg;
      int g = 0;        // global tile-step counter
      int a = 0;        // active segments so far
      bool ok = true;
      while (ok && it.next(p, sg)) {
        const int n = sg.k1 - sg.k0;
        if (n <= 0) continue;
        const uint32_t pa = (uint32_t)(a - 1) & 1u;  // parity of the previous segment
        if (!(ok = wait(&sm.q_full, (uint32_t)a & 1u))) break;
        tc_fence_after();
        for (int jj = 0; jj < n && ok; ++jj, ++g) {
          const int ik = 2 * g;
          if (!(ok = wait(&sm.kv_full[slot_of(ik)], par_of(ik)))) break;
          if (jj == 0) {
            tc_fence_after();
            issue_qk(0, slot_of(ik));
            umma_commit(&sm.s_full[0]);
            issue_qk(1, slot_of(ik));
            umma_commit(&sm.s_full[1]);
            umma_commit(&sm.kv_empty[slot_of(ik)]);
          } else {
            const int iv = 2 * (g - 1) + 1;
            const uint32_t pp = (uint32_t)(g - 1) & 1u;
            ok = wait(&sm.kv_full[slot_of(iv)], par_of(iv)) && wait(&sm.p_full[0], pp);
            if (ok && jj == 1 && a > 0) ok = wait(&sm.o_empty[0], pa);
            if (!ok) break;
            tc_fence_after();
            issue_pv(0, slot_of(iv), jj > 1);
            issue_qk(0, slot_of(ik));
            umma_commit(&sm.s_full[0]);
            ok = wait(&sm.p_full[1], pp);
            if (ok && jj == 1 && a > 0) ok = wait(&sm.o_empty[1], pa);
            if (!ok) break;
            tc_fence_after();
            issue_pv(1, slot_of(iv), jj > 1);
            umma_commit(&sm.kv_empty[slot_of(iv)]);
            issue_qk(1, slot_of(ik));
            umma_commit(&sm.s_full[1]);
            umma_commit(&sm.kv_empty[slot_of(ik)]);
          }
          if (jj == n - 1) umma_commit(&sm.q_empty);  // all QK^T of this segment issued
        }
        if (!ok) break;
        // tail: P V of the segment's last key tile, then O is final
        const int iv = 2 * (g - 1) + 1;
        const uint32_t pp = (uint32_t)(g - 1) & 1u;
        ok = wait(&sm.kv_full[slot_of(iv)], par_of(iv)) && wait(&sm.p_full[0], pp);
        if (ok && n == 1 && a > 0) ok = wait(&sm.o_empty[0], pa);
        if (!ok) break;
        tc_fence_after();
        issue_pv(0, slot_of(iv), n > 1);
        umma_commit(&sm.o_full[0]);
        ok = wait(&sm.p_full[1], pp);
        if (ok && n == 1 && a > 0) ok = wait(&sm.o_empty[1], pa);
        if (!ok) break;
        tc_fence_after();
        issue_pv(1, slot_of(iv), n > 1);
        umma_commit(&sm.o_full[1]);
        umma_commit(&sm.kv_empty[slot_of(iv)]);
        ++a;
      }
      // Let every MMA this thread issued retire before TMEM is released.
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
    const uint32_t tS = tmem + lane_field + i * 128;
    const uint32_t tO = tmem + lane_field + 256 + i * 128;
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
        uint32_t r[4][32];
        int lim = kv_len - j * kBN;
        if (causal) lim = min(lim, grow - j * kBN + 1);
        const bool full = lim >= kBN;
        // S row from tensor memory; columns >= lim (padding, causal) become -inf.
        auto load_s = [&]() {
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, r[c]);
          tmem_ld_wait();
          if (!full) {
#pragma unroll
            for (int c = 0; c < 4; ++c)
#pragma unroll
              for (int e = 0; e < 32; ++e)
                if (c * 32 + e >= lim) r[c][e] = __float_as_uint(-INFINITY);
          }
        };
#define SV(e) __uint_as_float(r[(e) >> 5][(e) & 31])
        // Row max: 8 independent 3-input-max chains, then a small tree.
        auto row_max = [&]() {
          float acc[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) acc[k] = fmaxf(SV(2 * k), SV(2 * k + 1));
#pragma unroll
          for (int e = 16; e < 128; e += 16)
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[k] = max3f(acc[k], SV(e + 2 * k), SV(e + 2 * k + 1));
          return max3f(max3f(acc[0], acc[1], acc[2]), max3f(acc[3], acc[4], acc[5]),
                       fmaxf(acc[6], acc[7]));
        };
        uint64_t sum2[4];
        uint32_t pk[2][32];
        // P = 2^(s*scale*log2e - mu) for pairs of columns through the packed FMA pipe, the
        // row sum and the 16-bit pack, in one pass that consumes r.  In full tiles
        // kPolyPer8 of every 8 pairs take the polynomial exp2, the rest MUFU ex2.
        auto exp_pass = [&](float mu) {
          const float nb = (mu == -INFINITY) ? 0.f : -mu;
          const uint64_t scale2 = f2pack(sl2, sl2), base2 = f2pack(nb, nb);
#pragma unroll
          for (int k = 0; k < 4; ++k) sum2[k] = 0ull;
          // The polynomial share is fixed per pair at compile time, and the test of `full`
          // sits outside the unrolled loop: a runtime test per pair makes the compiler branch
          // or evaluate both exponentials, which saves no MUFU work.
          auto pass = [&](auto pc) {
            constexpr bool kPoly = decltype(pc)::value;
#pragma unroll
            for (int pr = 0; pr < 64; ++pr) {
              float x0, x1;
              f2unpack(fma2(f2pack(SV(2 * pr), SV(2 * pr + 1)), scale2, base2), x0, x1);
              if (kPoly && (pr & 7) < kPolyPer8) {
                exp2_poly_pair(x0, x1);
              } else {
                x0 = ex2_approx(x0);
                x1 = ex2_approx(x1);
              }
              sum2[pr & 3] = add2(sum2[pr & 3], f2pack(x0, x1));
              pk[pr >> 5][pr & 31] = pack2<kOp>(x0, x1);
            }
          };
          if (kPolyPer8 > 0 && full)
            pass(std::true_type{});
          else
            pass(std::false_type{});
        };
        auto row_sum = [&]() {
          float sa, sb;
          f2unpack(add2(add2(sum2[0], sum2[1]), add2(sum2[2], sum2[3])), sa, sb);
          return sa + sb;
        };
        // Online softmax with a lazy rescale: the max used for P (m_use) moves only when
        // the tile's row max exceeds it by more than kRescaleThreshold.
        //  * first tile of a segment: row max first, then P;
        //  * later tiles: P with the running max m straight away.  The row sum, computed
        //    anyway, certifies it: sum <= 2^kRescaleThreshold means every P <= 2^8, so the
        //    tile max is within the threshold and m stays.  Otherwise (rare once the running
        //    max has settled) the warp reloads S, takes the exact max and redoes the pass
        //    with the max the lazy rule picks.  This removes the row-max pass from the
        //    steady-state critical path.
        load_s();
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
            load_s();
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
        tmem_st32(tS, pk[0]);
        tmem_st32(tS + 32, pk[1]);
#undef SV
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
        mbar_arrive(&sm.p_full[i]);
        m = m_use;
      }
      if (!ok) break;
      if (n > 0) {
        const bool got = mbar_wait(&sm.o_full[i], (uint32_t)a & 1u, abort, p.status,
                                   ANIMA_ERR_TIMEOUT);
        if (!(ok = __all_sync(0xffffffffu, got))) break;
        tc_fence_after();
      }
      segment_epilogue<kOut>(p, sg, n, i, row, lane, b, bh, grow, tO, m, l, sm.stage[warp],
                             p.tma_out ? &tmap_o : nullptr);
      if (n > 0) {
        tc_fence_before();
        mbar_arrive(&sm.o_empty[i]);
        ++a;
      }
    }
    if (p.tma_out && lane == 0) bulk_wait_read_all();  // stores done reading shared memory
    tc_fence_before();
    __syncthreads();  // pairs with the control warpgroup's teardown barrier
  }
}

}  // namespace attn

// ---------------------------------------------------------------- no-allocation scratch
// Scratch of the split schedule for anima_attn_fwd_noalloc, for callers that cannot
// allocate device memory.  Sized for GPUs with up to kNoAllocMaxCtas SMs: 4 KiB of
// arrival counters plus two fp32 partial slots per CTA (about 40.6 MB).  Every GPU that
// loads this library holds it until the process exits.  Zero at module load; each call
// clears the counters again before its kernel runs.
namespace attn {
constexpr int kNoAllocMaxCtas = 160;
constexpr size_t kNoAllocScratchBytes =
    kSemBytes + (size_t)kNoAllocMaxCtas * 2 * kPartFloats * sizeof(float);
}  // namespace attn
static __device__ __align__(256) unsigned char g_noalloc_scratch[attn::kNoAllocScratchBytes];

// ---------------------------------------------------------------- host launcher
// The 64-key-tile kernel (attn_fwd64.cu).
int attn64_launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                  const attn::Params& prm, int grid, int op_dtype, int out_dtype,
                  cudaStream_t st);

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// [bh][rows][128] 16-bit tensor, box [64 elements][box_rows rows][1], 128-byte swizzle.
static int make_head_map(CUtensorMap* map, const void* base, int op_dtype, int bh, int rows,
                         int box_rows = 128) {
  EncodeTiledFn enc = get_encode_fn();
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

// Output [B, S_q, H, 128] addressed by element strides (ob, oh, os) as a TMA tile map for
// the epilogue's 32 x 32 blocks (box: 32 columns x 32 tokens of one head), axes ordered by
// stride: (D, H, S, B) when heads are closer than tokens (token-major output), else
// (D, S, H, B).  Swizzle 128 B (fp32) / 64 B (16-bit), the staging buffer's layout.
// Returns false when the strides or alignment do not allow a map (then plain stores).
static bool make_out_map(CUtensorMap* map, const AnimaAttnArgs* a, int* hs) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const int esz = a->out_dtype == ANIMA_DTYPE_F32 ? 4 : 2;
  const long long ob = a->out_stride[0], oh = a->out_stride[1], os = a->out_stride[2];
  if ((reinterpret_cast<uintptr_t>(a->out) & 15u) != 0 || ob <= 0 || oh <= 0 || os <= 0) return false;
  if ((ob * esz) % 16 || (oh * esz) % 16 || (os * esz) % 16) return false;
  const CUtensorMapDataType dt = a->out_dtype == ANIMA_DTYPE_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : a->out_dtype == ANIMA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  *hs = oh <= os ? 1 : 0;
  cuuint64_t dims[4] = {128, (cuuint64_t)(*hs ? a->H : a->S_q), (cuuint64_t)(*hs ? a->S_q : a->H),
                        (cuuint64_t)a->B};
  cuuint64_t strides[3] = {(cuuint64_t)((*hs ? oh : os) * esz), (cuuint64_t)((*hs ? os : oh) * esz),
                           (cuuint64_t)(ob * esz)};
  cuuint32_t box[4] = {32, (cuuint32_t)(*hs ? 1 : 32), (cuuint32_t)(*hs ? 32 : 1), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, dt, 4, a->out, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         esz == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                         CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int kOp, int kOut>
static int launch_t(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                    const CUtensorMap& mo, const attn::Params& prm, int grid, cudaStream_t st) {
  auto kern = attn::attn_fwd_kernel<kOp, kOut>;
  static int attr_dev_mask = 0;  // devices on which the smem attribute was raised
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask & (1 << (dev & 31)))) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)attn::kSmemBytes) != cudaSuccess)
      return ANIMA_ERR_CUDA;
    attr_dev_mask |= 1 << (dev & 31);
  }
  // Programmatic dependent launch: the CTAs may start (barriers, TMEM, descriptor
  // prefetch) while the previous kernel on the stream drains; the kernel waits for it
  // (griddepcontrol.wait) before its first global access.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(attn::kThreads);
  cfg.dynamicSmemBytes = attn::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, mo, prm) != cudaSuccess) {
    cudaGetLastError();
    return ANIMA_ERR_CUDA;
  }
  return ANIMA_OK;
}

// Schedule of a call: one CTA per unit, or a persistent grid of whole-unit rounds, or
// whole-unit rounds plus the last round cut into slices (needs `bytes` of workspace).
enum { kSchedUnit = 0, kSchedWhole = 1, kSchedCut = 2 };
struct SplitPlan {
  int mode, rounds, tail_units, tail_tiles, tail_ctas;
  size_t bytes;  // workspace: counters + partial slots (kSchedCut only)
};

// allow_cut = false plans for a call without a usable workspace.  The decisions are taken
// in 128-key tiles; the cut slices are counted in the kernel's own key tiles (bn keys).
static SplitPlan plan_split(int bh, int S_q, int S_kv, unsigned flags, int sm_count,
                            bool allow_cut = true) {
  const int bn = (flags & ANIMA_FLAG_KV64) ? 64 : attn::kBN;
  SplitPlan sp = {kSchedUnit, 0, 0, 0, 0, 0};
  if (flags & (ANIMA_FLAG_CAUSAL | ANIMA_FLAG_UNIT) || sm_count < 2)
    return sp;  // causal units differ in length along the diagonal: the hardware balances them
  const long long units = (long long)bh * ((S_q + attn::kUnitRows - 1) / attn::kUnitRows);
  const long long n = (S_kv + attn::kBN - 1) / attn::kBN;
  if (units > 0x7fffffffLL) return sp;
  if (flags & ANIMA_FLAG_MASK) {
    // Key-padding masks shorten every unit of a sample alike (the DiT's cross-attention:
    // 512 context keys, 4 tiles, fewer when padded).  Short units pay their start-up
    // (TMEM allocation, barriers, the first loads) once per unit in one-CTA-per-unit mode,
    // so calls of more than one wave of units of at most 16 key tiles run persistent whole
    // units (never cut: the cut's slices assume every unit has n tiles).  Longer masked
    // units keep one CTA per unit, which balances units of different lengths.
    if ((flags & ANIMA_FLAG_KV64) || units <= sm_count) return sp;
    if (n > 16 && !(flags & ANIMA_FLAG_WHOLE)) return sp;
    sp.mode = kSchedWhole;
    sp.rounds = (int)((units + sm_count - 1) / sm_count);
    return sp;
  }
  const long long rounds = units / sm_count, tail = units - rounds * sm_count;
  // Cutting the last round saves the idle share of the unit grid's last wave, (sm - tail)/sm
  // of one unit's time, and costs segment set-up, partial stores and merges, which do not
  // grow with the unit's n key tiles.  The cut is the default when the idle share exceeds
  // 0.15 + 5/n: with B=2, H=16, bf16 that picks the faster schedule at every shape measured
  // (cut at L = 2560, 3072, 4096, 5120, 6144 and S_q x S_kv = 4096 x 2048; not at 2048,
  // 8192, 16384, where the idle share is 0.27, 0.08 and 0.16, nor at 4096 x 512 / 1024).
  const bool worth = (sm_count - tail) * n * 100 > (long long)sm_count * (15 * n + 500);
  if (units <= sm_count) {
    // One wave: one CTA per unit, unless most SMs would idle (a few heads per GPU, e.g.
    // B=2 with 2 heads at L = 4096: 64 units on 148 SMs).  Then every unit is cut into
    // key-tile slices over all SMs, as the last round of a longer call is.  Here every
    // unit pays a merge, so the rule compares step counts: cut ~ max(kMinSliceTiles,
    // units * n / sm) + 5 steps of merge against n for one CTA per unit, taken below 0.9 n.
    // Measured (B=2, L=4096, TFLOP/s unit -> cut): 2 heads 507 -> 668, 1 head 242 -> 377;
    // 4 heads 893 = 892 (stays unit); at 1024 tokens (n = 8) the cut lost 3-5 %.
    const long long cut_steps_x_sm =
        std::max((long long)attn::kMinSliceTiles * sm_count, units * n) + 5LL * sm_count;
    const bool one_wave_worth = 10 * cut_steps_x_sm < 9 * n * sm_count;
    if (units == sm_count || (flags & ANIMA_FLAG_WHOLE) || !allow_cut || !one_wave_worth)
      return sp;
    if (2LL * tail * (long long)sizeof(int) > attn::kSemBytes) return sp;
  }
  // Persistent grid of whole units: a CTA moves from unit to unit without its start-up
  // (TMEM allocation, barrier set-up, the first Q and K loads from DRAM) and with the next
  // unit's K/V already streaming, ~1.5 key-tile steps less overhead per unit than one CTA
  // per unit; but the units are dealt statically, while the hardware hands one-CTA units
  // to whichever SM is free, and that balance is worth ~4 %.  Measured (B=2, H=16):
  // whole units win for short units (n = 4: +13 %, 8: +9 %, 16: +3-4 %, 32: +1 %) and lose
  // for long ones (48: -0.7 %, 64: -1.5 %, 128: -3.4 %), so without a cut the plan takes
  // whole units up to n = 32 key tiles and one CTA per unit beyond.
  SplitPlan whole = sp;
  whole.mode = kSchedWhole;
  whole.rounds = (int)((units + sm_count - 1) / sm_count);
  if (flags & ANIMA_FLAG_WHOLE) return whole;
  const SplitPlan nocut = (rounds == 0 || n > 32) ? sp : whole;
  if (!allow_cut || tail == 0 || tail * n > 0x7fffffffLL) return nocut;  // whole rounds
  if (2LL * tail * (long long)sizeof(int) > attn::kSemBytes) return nocut;
  if (rounds > 0 && !(flags & ANIMA_FLAG_SPLIT) && !worth) return nocut;
  sp.mode = kSchedCut;
  sp.rounds = (int)rounds;
  sp.tail_units = (int)tail;
  const long long nt = (S_kv + bn - 1) / bn;  // the kernel's key tiles per unit
  if (tail * nt > 0x7fffffffLL) return nocut;
  sp.tail_tiles = (int)(tail * nt);
  long long ctas = sp.tail_tiles / (attn::kMinSliceTiles * attn::kBN / bn);
  if (ctas > sm_count) ctas = sm_count;
  if (ctas < 1) ctas = 1;
  sp.tail_ctas = (int)ctas;
  sp.bytes = attn::kSemBytes + (size_t)ctas * 2 * attn::kPartFloats * sizeof(float);
  return sp;
}

size_t attn_workspace_bytes(int B, int H, int S_q, int S_kv, unsigned flags, int sm_count) {
  return plan_split(B * H, S_q, S_kv, flags, sm_count).bytes;
}

int attn_schedule_mode(int B, int H, int S_q, int S_kv, unsigned flags, int sm_count) {
  static_assert((int)kSchedUnit == (int)ANIMA_SCHED_UNIT && (int)kSchedWhole == (int)ANIMA_SCHED_WHOLE &&
                    (int)kSchedCut == (int)ANIMA_SCHED_CUT,
                "schedule codes of the header");
  return plan_split(B * H, S_q, S_kv, flags, sm_count).mode;
}

int attn_fwd_launch(const AnimaAttnArgs* a, int* status, int sm_count, cudaStream_t st,
                    void* const* peers, int n_peers, int peer_rows, long long peer_row_stride,
                    int peer_head0) {
  if (a->D != attn::kD) return ANIMA_ERR_SHAPE;
  if (a->op_dtype != ANIMA_DTYPE_BF16 && a->op_dtype != ANIMA_DTYPE_F16) return ANIMA_ERR_ARG;
  if (a->out_dtype != ANIMA_DTYPE_F32 && a->out_dtype != ANIMA_DTYPE_BF16 &&
      a->out_dtype != ANIMA_DTYPE_F16)
    return ANIMA_ERR_ARG;
  const int bh = a->B * a->H;
  if (a->B <= 0 || a->H <= 0 || a->S_q <= 0 || a->S_kv <= 0) return ANIMA_ERR_SHAPE;
  CUtensorMap mq, mk, mv;
  int rc;
  const bool kv64 = (a->flags & ANIMA_FLAG_KV64) != 0;
  const int bn = kv64 ? 64 : attn::kBN;  // keys per key tile of the kernel that runs
  if ((rc = make_head_map(&mq, a->q, a->op_dtype, bh, a->S_q))) return rc;
  if ((rc = make_head_map(&mk, a->k, a->op_dtype, bh, a->S_kv, bn))) return rc;
  if ((rc = make_head_map(&mv, a->v, a->op_dtype, bh, a->S_kv, bn))) return rc;
  attn::Params prm;
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
  prm.nqb = (a->S_q + attn::kUnitRows - 1) / attn::kUnitRows;
  prm.n_kv = (a->S_kv + bn - 1) / bn;
  const long long units = (long long)bh * prm.nqb;
  if (units > 0x7fffffffLL) return ANIMA_ERR_SHAPE;
  prm.units = (int)units;
  SplitPlan sp = plan_split(bh, a->S_q, a->S_kv, a->flags, sm_count);
  if (sp.mode == kSchedCut &&
      !(a->workspace && a->workspace_bytes >= sp.bytes &&
        (reinterpret_cast<uintptr_t>(a->workspace) & 255u) == 0))
    sp = plan_split(bh, a->S_q, a->S_kv, a->flags, sm_count, false);
  prm.split = sp.mode != kSchedUnit ? 1 : 0;
  prm.rounds = sp.rounds;
  prm.tail_base = sp.mode == kSchedCut ? sp.rounds * sm_count : (int)units;
  prm.tail_tiles = sp.mode == kSchedCut ? sp.tail_tiles : 0;
  prm.tail_ctas = sp.mode == kSchedCut ? sp.tail_ctas : 0;
  prm.sem = static_cast<int*>(a->workspace);
  prm.part = reinterpret_cast<float*>(static_cast<char*>(a->workspace) + attn::kSemBytes);
  const int grid = prm.split ? sm_count : (int)units;
  prm.tma_out = 0;
  prm.tma_hs = 0;
  prm.n_peers = n_peers;
  for (int i = 0; i < attn::kMaxPeers; ++i) prm.peer_out[i] = i < n_peers ? peers[i] : nullptr;
  prm.peer_rows = peer_rows;
  prm.peer_row_stride = peer_row_stride;
  prm.peer_head0 = peer_head0;
  if (kv64) return attn64_launch(mq, mk, mv, prm, grid, a->op_dtype, a->out_dtype, st);
  CUtensorMap mo;
  memset(&mo, 0, sizeof(mo));
  prm.tma_out = n_peers == 0 && make_out_map(&mo, a, &prm.tma_hs) ? 1 : 0;
  const bool bf = a->op_dtype == ANIMA_DTYPE_BF16;
  switch (a->out_dtype) {
    case ANIMA_DTYPE_F32:
      return bf ? launch_t<ANIMA_DTYPE_BF16, ANIMA_DTYPE_F32>(mq, mk, mv, mo, prm, grid, st)
                : launch_t<ANIMA_DTYPE_F16, ANIMA_DTYPE_F32>(mq, mk, mv, mo, prm, grid, st);
    case ANIMA_DTYPE_BF16:
      return bf ? launch_t<ANIMA_DTYPE_BF16, ANIMA_DTYPE_BF16>(mq, mk, mv, mo, prm, grid, st)
                : launch_t<ANIMA_DTYPE_F16, ANIMA_DTYPE_BF16>(mq, mk, mv, mo, prm, grid, st);
    default:
      return bf ? launch_t<ANIMA_DTYPE_BF16, ANIMA_DTYPE_F16>(mq, mk, mv, mo, prm, grid, st)
                : launch_t<ANIMA_DTYPE_F16, ANIMA_DTYPE_F16>(mq, mk, mv, mo, prm, grid, st);
  }
}

// Device address of g_noalloc_scratch on the current device.  Host code must use this
// address: the array's name in host code is a host-side stand-in.
cudaError_t noalloc_scratch_address(void** ptr) { return cudaGetSymbolAddress(ptr, g_noalloc_scratch); }

// Same launch as attn_fwd_launch, with the split schedule's scratch taken from
// g_noalloc_scratch (its device address `scratch`, from noalloc_scratch_address) instead of
// the caller's workspace.
int attn_fwd_launch_noalloc(const AnimaAttnArgs* a, int* status, int sm_count, void* scratch,
                            cudaStream_t st, const char** why) {
  const SplitPlan sp = plan_split(a->B * a->H, a->S_q, a->S_kv, a->flags, sm_count);
  if (sp.bytes > attn::kNoAllocScratchBytes) {
    *why = "this call's split schedule needs more scratch than the no-allocation entry's "
           "static array holds (it is sized for GPUs with up to 160 SMs)";
    return ANIMA_ERR_SHAPE;
  }
  if (sp.bytes > 0 && cudaMemsetAsync(scratch, 0, attn::kSemBytes, st) != cudaSuccess) {
    cudaGetLastError();
    *why = "clearing the no-allocation scratch counters failed";
    return ANIMA_ERR_CUDA;
  }
  AnimaAttnArgs b = *a;
  b.workspace = scratch;
  b.workspace_bytes = attn::kNoAllocScratchBytes;
  return attn_fwd_launch(&b, status, sm_count, st, nullptr, 0, 0, 0, 0);
}

}  // namespace anima
