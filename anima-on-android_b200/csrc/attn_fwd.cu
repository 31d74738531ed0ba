// attn_fwd.cu -- non-causal / causal / key-padding-masked flash-attention forward for
// sm_100a: TMA-staged tiles, tcgen05.mma with TMEM accumulators, fp32 online softmax.
//
// Replaces anima::cpu::flash_attention (anima_rt/include/cpu/flash_attention.h:55-208):
// out = softmax(Q K^T * scale) V per (batch, head), D = 128.  The reference tiles
// queries by 256/64/32 and keys by 512 on one CPU thread; here one CTA owns 256 query
// rows of one head and streams 128-key tiles:
//
//   warp 8     TMA producer: Q (2 tiles, once), then K_j / V_j into a 4-slot ring
//   warp 9     MMA issuer (one thread) + TMEM owner:
//                S_i  = Q_i K_j^T          (SS form, both operands in shared memory)
//                O_i += P_i V_j            (TS form, P read from tensor memory)
//   warps 10-11 idle (they complete the third warpgroup, which donates its registers)
//   warps 0-7  two softmax warpgroups, one per 128-row Q tile; thread = query row =
//              TMEM lane.  Each reads its S row from TMEM, updates the running max
//              and sum, writes P (16-bit) back over S, rescales its O row when the
//              max moved, and finally normalises O and stores it.
//
// Tensor memory (512 columns x 128 lanes, fp32): S_0 [0,128) S_1 [128,256)
// O_0 [256,384) O_1 [384,512); P_i overlays the first 64 columns of S_i (two 16-bit
// values per column).  The two query tiles ping-pong: while warpgroup 0 runs the
// softmax of tile 0, the tensor core computes tile 1, and vice versa.
//
// Online softmax in the exp2 domain (scores scaled by scale*log2(e)), with a lazy
// rescale: the running max used for P moves only when the new row max exceeds it by
// more than 8 (a factor 256), so the O correction is rare after the first tiles.
#include "common.cuh"

namespace anima {
namespace attn {

constexpr int kD = 128;
constexpr int kBM = 128;               // query rows per tile (TMEM lanes)
constexpr int kNT = 2;                 // query tiles per CTA
constexpr int kBN = 128;               // keys per K/V tile
constexpr int kStages = 4;             // K/V ring slots
constexpr int kPanel = 128 * 128;      // [128 rows][64 x 16-bit], 128B-swizzled = 16 KB
constexpr int kTile = 2 * kPanel;      // [128 rows][128 x 16-bit] = 32 KB
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 384;              // 3 warpgroups
// Launch budget 384 x 168 registers; the control warpgroup gives registers back to the
// two softmax warpgroups: 2*128*208 + 128*80 = 63488 <= 384*168.
constexpr uint32_t kRegsSoftmax = 208;
constexpr uint32_t kRegsControl = 80;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
#ifndef ANIMA_POLY_PER8
#define ANIMA_POLY_PER8 2
#endif
constexpr int kPolyPer8 = ANIMA_POLY_PER8;  // of every 8 column pairs, polynomial exp2

struct Smem {
  uint8_t q[kNT][kTile];
  uint8_t kv[kStages][kTile];
  uint64_t bar_q;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[kNT];
  uint64_t p_full[kNT];
  uint64_t o_full[kNT];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + slack to align the base to 1 KB
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

struct Params {
  int B, H, S_q, S_kv;
  float scale_log2;
  unsigned flags;
  const int* kv_valid;
  void* out;
  long long ob, oh, os;
  int* status;
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

template <int kOp>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return kOp == ANIMA_DTYPE_BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}

template <int kOp, int kOut>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmap_q,
                    const __grid_constant__ CUtensorMap tmap_k,
                    const __grid_constant__ CUtensorMap tmap_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + pad);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int b = bh / p.H;
  const int q0 = blockIdx.x * (kBM * kNT);

  int kv_len = p.S_kv;
  if (p.flags & ANIMA_FLAG_MASK) kv_len = min(max(p.kv_valid[b], 0), p.S_kv);
  int n_kv = (kv_len + kBN - 1) / kBN;
  if (p.flags & ANIMA_FLAG_CAUSAL) {
    const int last_row = min(q0 + kBM * kNT, p.S_q) - 1;
    n_kv = min(n_kv, last_row / kBN + 1);
  }
  volatile int* abort = &sm.abort;

  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_q, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int i = 0; i < kNT; ++i) {
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.p_full[i], kBM);
      mbar_init(&sm.o_full[i], 1);
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

  if (warp >= 8) {
    regs_dec<kRegsControl>();
  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_q);
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_v);
      mbar_arrive_expect_tx(&sm.bar_q, kNT * kTile);
      for (int i = 0; i < kNT; ++i)
        for (int pn = 0; pn < 2; ++pn)
          tma_load_3d(sm.q[i] + pn * kPanel, &tmap_q, &sm.bar_q, pn * 64, q0 + i * kBM, bh);
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < n_kv && ok; ++j) {
        for (int kind = 0; kind < 2; ++kind) {
          const int c = 2 * j + kind;
          const int slot = c % kStages;
          const uint32_t round = c / kStages;
          if (!mbar_wait(&sm.kv_empty[slot], (round & 1u) ^ 1u, abort, p.status,
                         ANIMA_ERR_TIMEOUT)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sm.kv_full[slot], kTile);
          const CUtensorMap* m = kind ? &tmap_v : &tmap_k;
          tma_load_3d(sm.kv[slot], m, &sm.kv_full[slot], 0, j * kBN, bh);
          tma_load_3d(sm.kv[slot] + kPanel, m, &sm.kv_full[slot], 64, j * kBN, bh);
          ++issued;
        }
      }
      // Every copy this thread started must land before the CTA may exit.
      drain_wait(&sm.bar_q, 0);
      for (int s = 0; s < kStages; ++s) {
        int last = -1;
        for (int c = s; c < issued; c += kStages) last = c;
        if (last >= 0) drain_wait(&sm.kv_full[s], (uint32_t)(last / kStages) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t ab = kOp == ANIMA_DTYPE_BF16 ? 1u : 0u;  // idesc: 0 f16, 1 bf16
      constexpr uint32_t idesc_qk = make_idesc_f16(ab, kBM, kBN, 0);
      constexpr uint32_t idesc_pv = make_idesc_f16(ab, kBM, kD, 1);
      const uint32_t q_base = smem_u32(sm.q[0]);    // tile i at + i * kTile
      const uint32_t kv_base = smem_u32(sm.kv[0]);  // slot s at + s * kTile

      auto issue_qk = [&](int i, int slot) {
        const uint32_t d = tmem + i * 128;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kPanel + (kk & 3) * 32;
          umma_ss(d, sdesc_sw128(q_base + i * kTile + off, 16, 1024),
                  sdesc_sw128(kv_base + slot * kTile + off, 16, 1024), idesc_qk, kk > 0);
        }
      };
      auto issue_pv = [&](int i, int slot, bool acc) {
        const uint32_t d = tmem + 256 + i * 128;
        const uint32_t a = tmem + i * 128;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          umma_ts(d, a + kk * 8, sdesc_sw128(kv_base + slot * kTile + kk * 2048, kPanel, 1024),
                  idesc_pv, (acc || kk > 0) ? 1u : 0u);
        }
      };
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return mbar_wait(bar, parity, abort, p.status, ANIMA_ERR_TIMEOUT);
      };

      bool ok = wait(&sm.bar_q, 0) && wait(&sm.kv_full[0], 0);
      if (ok) {
        tc_fence_after();
        issue_qk(0, 0);
        umma_commit(&sm.s_full[0]);
        issue_qk(1, 0);
        umma_commit(&sm.s_full[1]);
        umma_commit(&sm.kv_empty[0]);
      }
      for (int j = 1; j < n_kv && ok; ++j) {
        const int ck = 2 * j, cv = 2 * (j - 1) + 1;
        const int sk = ck % kStages, sv = cv % kStages;
        const uint32_t pk = (uint32_t)(ck / kStages) & 1u, pv = (uint32_t)(cv / kStages) & 1u;
        const uint32_t pp = (uint32_t)(j - 1) & 1u;
        ok = wait(&sm.kv_full[sk], pk) && wait(&sm.kv_full[sv], pv) && wait(&sm.p_full[0], pp);
        if (!ok) break;
        tc_fence_after();
        issue_pv(0, sv, j - 1 > 0);
        issue_qk(0, sk);
        umma_commit(&sm.s_full[0]);
        if (!(ok = wait(&sm.p_full[1], pp))) break;
        tc_fence_after();
        issue_pv(1, sv, j - 1 > 0);
        umma_commit(&sm.kv_empty[sv]);
        issue_qk(1, sk);
        umma_commit(&sm.s_full[1]);
        umma_commit(&sm.kv_empty[sk]);
      }
      if (ok) {
        const int j = n_kv - 1;
        const int cv = 2 * j + 1, sv = cv % kStages;
        const uint32_t pv = (uint32_t)(cv / kStages) & 1u, pp = (uint32_t)j & 1u;
        ok = wait(&sm.kv_full[sv], pv) && wait(&sm.p_full[0], pp);
        if (ok) {
          tc_fence_after();
          issue_pv(0, sv, j > 0);
          umma_commit(&sm.o_full[0]);
          if (wait(&sm.p_full[1], pp)) {
            tc_fence_after();
            issue_pv(1, sv, j > 0);
            umma_commit(&sm.o_full[1]);
            umma_commit(&sm.kv_empty[sv]);
          }
        }
      }
      // Let every MMA this thread issued retire before TMEM is released.
      umma_commit(&sm.mma_done);
      drain_wait(&sm.mma_done, 0);
    }
    __syncwarp();
  }
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
    const int grow = q0 + i * kBM + row;
    const uint32_t lane_field = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_field + i * 128;
    const uint32_t tO = tmem + lane_field + 256 + i * 128;
    const bool causal = (p.flags & ANIMA_FLAG_CAUSAL) != 0;
    const float sl2 = p.scale_log2;

    float m = -INFINITY;  // running max, scaled log2 units
    float l = 0.f;        // running sum of P
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const bool got = mbar_wait(&sm.s_full[i], (uint32_t)j & 1u, abort, p.status,
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
      uint32_t pk[2][32];
      // P = 2^(s*scale*log2e - m): pairs of columns through the packed FMA pipe; in full
      // tiles kPolyPer8 of every 8 pairs take the polynomial exp2, the rest MUFU ex2.
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
#undef SV
      float sa, sb;
      f2unpack(add2(add2(sum2[0], sum2[1]), add2(sum2[2], sum2[3])), sa, sb);
      const float sum = sa + sb;
      l = l * alpha + sum;
      tmem_st32(tS, pk[0]);
      tmem_st32(tS + 32, pk[1]);
      if (__any_sync(0xffffffffu, j > 0 && alpha != 1.f)) {
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

    if (ok && n_kv > 0) {
      const bool got = mbar_wait(&sm.o_full[i], 0, abort, p.status, ANIMA_ERR_TIMEOUT);
      ok = __all_sync(0xffffffffu, got);
      tc_fence_after();
    }
    if (ok) {
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      const bool live = grow < p.S_q;
      char* out_row = reinterpret_cast<char*>(p.out) +
                      ((long long)b * p.ob + (long long)(bh % p.H) * p.oh +
                       (long long)grow * p.os) *
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
        if (live) {
          if (kOut == ANIMA_DTYPE_F32) {
            float4* dst = reinterpret_cast<float4*>(out_row) + c * 8;
#pragma unroll
            for (int e = 0; e < 8; ++e)
              dst[e] = make_float4(__uint_as_float(o[4 * e]) * inv,
                                   __uint_as_float(o[4 * e + 1]) * inv,
                                   __uint_as_float(o[4 * e + 2]) * inv,
                                   __uint_as_float(o[4 * e + 3]) * inv);
          } else {
            uint4* dst = reinterpret_cast<uint4*>(out_row) + c * 4;
#pragma unroll
            for (int e = 0; e < 4; ++e)
              dst[e] = make_uint4(
                  pack_bf16x2(__uint_as_float(o[8 * e]) * inv, __uint_as_float(o[8 * e + 1]) * inv),
                  pack_bf16x2(__uint_as_float(o[8 * e + 2]) * inv, __uint_as_float(o[8 * e + 3]) * inv),
                  pack_bf16x2(__uint_as_float(o[8 * e + 4]) * inv, __uint_as_float(o[8 * e + 5]) * inv),
                  pack_bf16x2(__uint_as_float(o[8 * e + 6]) * inv, __uint_as_float(o[8 * e + 7]) * inv));
          }
        }
      }
    }
    tc_fence_before();
    __syncthreads();  // pairs with the control warpgroup's teardown barrier
  }
}

}  // namespace attn

// ---------------------------------------------------------------- host launcher
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

// [bh][rows][128] 16-bit tensor, box [64 elements][128 rows][1], 128-byte swizzle.
static int make_head_map(CUtensorMap* map, const void* base, int op_dtype, int bh, int rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return ANIMA_ERR_CUDA;
  const CUtensorMapDataType dt = op_dtype == ANIMA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)bh};
  cuuint64_t strides[2] = {128 * 2, (cuuint64_t)rows * 128 * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ANIMA_OK : ANIMA_ERR_CUDA;
}

template <int kOp, int kOut>
static int launch_t(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                    const attn::Params& prm, dim3 grid, cudaStream_t st) {
  auto kern = attn::attn_fwd_kernel<kOp, kOut>;
  static bool attr_set = false;  // per instantiation
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)attn::kSmemBytes) != cudaSuccess)
      return ANIMA_ERR_CUDA;
    attr_set = true;
  }
  kern<<<grid, attn::kThreads, attn::kSmemBytes, st>>>(mq, mk, mv, prm);
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

int attn_fwd_launch(const AnimaAttnArgs* a, int* status, cudaStream_t st) {
  if (a->D != attn::kD) return ANIMA_ERR_SHAPE;
  if (a->op_dtype != ANIMA_DTYPE_BF16 && a->op_dtype != ANIMA_DTYPE_F16) return ANIMA_ERR_ARG;
  if (a->out_dtype != ANIMA_DTYPE_F32 && a->out_dtype != ANIMA_DTYPE_BF16) return ANIMA_ERR_ARG;
  const int bh = a->B * a->H;
  if (bh <= 0 || a->S_q <= 0 || a->S_kv <= 0) return ANIMA_ERR_SHAPE;
  if (bh > 65535) return ANIMA_ERR_SHAPE;
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = make_head_map(&mq, a->q, a->op_dtype, bh, a->S_q))) return rc;
  if ((rc = make_head_map(&mk, a->k, a->op_dtype, bh, a->S_kv))) return rc;
  if ((rc = make_head_map(&mv, a->v, a->op_dtype, bh, a->S_kv))) return rc;
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
  dim3 grid((a->S_q + attn::kBM * attn::kNT - 1) / (attn::kBM * attn::kNT), bh);
  const bool bf = a->op_dtype == ANIMA_DTYPE_BF16;
  const bool of32 = a->out_dtype == ANIMA_DTYPE_F32;
  if (bf && of32) return launch_t<ANIMA_DTYPE_BF16, ANIMA_DTYPE_F32>(mq, mk, mv, prm, grid, st);
  if (bf) return launch_t<ANIMA_DTYPE_BF16, ANIMA_DTYPE_BF16>(mq, mk, mv, prm, grid, st);
  if (of32) return launch_t<ANIMA_DTYPE_F16, ANIMA_DTYPE_F32>(mq, mk, mv, prm, grid, st);
  return launch_t<ANIMA_DTYPE_F16, ANIMA_DTYPE_BF16>(mq, mk, mv, prm, grid, st);
}

}  // namespace anima
