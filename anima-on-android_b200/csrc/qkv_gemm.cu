// qkv_gemm.cu -- the q/k/v projection GEMM with the attention prologue in its epilogue.
//
// The reference projects, then normalises, rotates and transposes in separate passes
// (anima_rt/scripts/numpy_dit.py:276-291; src/predict2.py:174-193):
//   q = x Wq^T, k = ctx Wk^T, v = ctx Wv^T     [B, S, H*128]
//   q, k <- RMSNorm per head (eps 1e-6, weight [128])
//   q, k <- RoPE (self-attention)
//   [B, S, H, 128] -> [B, H, S, 128]
// Here one tcgen05 GEMM computes C = X W^T tile by tile in tensor memory and its epilogue
// applies all of that to the fp32 accumulator before the only store: the attention core's
// head-major 16-bit operands [B*H, S, 128].  The projection output never reaches HBM, and
// the norm sees the fp32 accumulator instead of a 16-bit rounding of it.
//
// Tiles of 128 rows (tokens) x 256 columns (two 128-column heads), K in steps of 64 (one
// 128-byte swizzle row of 16-bit values).  Persistent grid, one CTA per SM:
//   warp 0     TMA producer: A (X rows) and B (W rows) tiles through a 4-stage ring
//   warp 1     MMA issuer + TMEM owner: tcgen05.mma kind::f16, M128 N256 K16, into one of
//              two 256-column fp32 accumulators, so a tile's epilogue overlaps the next
//              tile's main loop
//   warps 4-7  epilogue: thread = token row = TMEM lane; RMSNorm statistics per head from
//              the fp32 accumulator, then 16-pair chunks of both heads: norm scale, RoPE
//              pairs (p, 64 + p) (q, k), pack to 16 bit and store 32-byte row pieces through
//              shared memory (32 consecutive tokens of one head are 32 consecutive rows of
//              the head-major output)
// Every wait is bounded (see common.cuh); a CTA that gives up records ANIMA_ERR_TIMEOUT.
#include <cstring>

#include "attn_shared.cuh"

namespace anima {
namespace qkv {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kStages = 4;
constexpr int kThreads = 256;  // the setup loads both 128-float norm weight rows, one per thread
constexpr int kATile = kBM * kBK * 2;  // 16 KB
constexpr int kBTile = kBN * kBK * 2;  // 32 KB
constexpr uint32_t kTmemCols = 512;    // two 256-column accumulators

struct Smem {
  uint8_t a[kStages][kATile];
  uint8_t b[kStages][kBTile];
  uint4 stage[4][64];     // per epilogue warp: 32 rows x 16 columns on their way to HBM
  float norm_w[2][128];   // q, k RMSNorm weights (1 where none is given)
  uint64_t full[kStages], empty[kStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

constexpr int kMaxDest = 8;

struct Params {
  int M, N, K;            // GEMM: token rows, columns n_tensors*H*128, depth
  int L, H;               // tokens per sample, heads per tensor
  int n_tiles_n, n_tiles; // column tiles, all tiles
  int tensor0;            // tensor (0 q, 1 k, 2 v) of the first 128-column block
  const float* norm_w[2]; // q, k RMSNorm weights (nullptr: weight 1)
  unsigned norm_mask;     // bit c: normalise tensor c
  const float* freqs;     // [L, 64, 2, 2]; nullptr: no RoPE (applied to q and k)
  float eps;
  // Head-major [B*Hd, L, 128] outputs: global head hg (of H per tensor) goes to destination
  // hg / Hd as its local head hg % Hd (one destination: this call's own q/k/v; several: the
  // ranks of a head split, reached through peer mappings).  Rows are tokens row0 + m of
  // the [B, L] token grid.
  int row0, Hd, n_dest;
  void* dest[kMaxDest][3];
  void* y;                // GELU epilogue: row-major [M, N] output, row stride ldy elements
  long long ldy;
  int* status;
};

enum { kEpiQkv = 0, kEpiGelu = 1 };

// 32 rows (one per lane) x 16 columns from column c0 of rows of 16-bit values, row_bytes
// apart: packed into the warp's staging buffer, then written as whole 32-byte row pieces
// (two lanes per row).  The swizzle (piece ^ bit 2 of the row) keeps both phases free of bank
// conflicts.  Rows >= nvalid are not written.
template <int kDt>
__device__ __forceinline__ void store_half(char* out_w, long long row_bytes, int nvalid,
                                           const float (&v)[16], int c0, uint4* st, int lane) {
#pragma unroll
  for (int e = 0; e < 2; ++e)
    st[lane * 2 + (e ^ ((lane >> 2) & 1))] = make_uint4(
        attn::pack2<kDt>(v[8 * e], v[8 * e + 1]), attn::pack2<kDt>(v[8 * e + 2], v[8 * e + 3]),
        attn::pack2<kDt>(v[8 * e + 4], v[8 * e + 5]), attn::pack2<kDt>(v[8 * e + 6], v[8 * e + 7]));
  __syncwarp();
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int r = 16 * k + (lane >> 1), q = lane & 1;
    const uint4 x = st[r * 2 + (q ^ ((r >> 2) & 1))];
    if (r < nvalid) *reinterpret_cast<uint4*>(out_w + r * row_bytes + (c0 + q * 8) * 2) = x;
  }
  __syncwarp();  // the buffer is free for the next piece
}

template <int kDt, int kEpi>
__global__ void __launch_bounds__(kThreads, 1)
    qkv_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_b, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + pad);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort = &sm.abort;
  const int nk = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(&sm.mma_done, 1);
    sm.abort = 0;
    fence_barrier_init();
  }
  {
    const int c = threadIdx.x >> 7, e = threadIdx.x & 127;  // 256 threads: both weight rows
    const float* w = c == 0 ? p.norm_w[0] : p.norm_w[1];  // no dynamic index into params
    sm.norm_w[c][e] = w ? w[e] : 1.0f;
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA producer
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.n_tiles && ok; t += gridDim.x) {
      const int m0 = (t / p.n_tiles_n) * kBM, n0 = (t % p.n_tiles_n) * kBN;
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const int s = it % kStages;
        if (!mbar_wait(&sm.empty[s], ((uint32_t)(it / kStages) & 1u) ^ 1u, abort, p.status,
                       ANIMA_ERR_TIMEOUT)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.full[s], kATile + kBTile);
        tma_load_2d(sm.a[s], &tmap_a, &sm.full[s], kb * kBK, m0);
        tma_load_2d(sm.b[s], &tmap_b, &sm.full[s], kb * kBK, n0);
      }
    }
    for (int s = 0; s < kStages; ++s) {  // every copy started must land before exit
      int last = -1;
      for (int c = s; c < it; c += kStages) last = c;
      if (last >= 0) attn::drain_wait(&sm.full[s], (uint32_t)(last / kStages) & 1u);
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t ab = kDt == ANIMA_DTYPE_BF16 ? 1u : 0u;
    constexpr uint32_t idesc = make_idesc_f16(ab, kBM, kBN, 0);
    const uint64_t da0 = sdesc_sw128(smem_u32(sm.a[0]), 16, 1024);
    const uint64_t db0 = sdesc_sw128(smem_u32(sm.b[0]), 16, 1024);
    int it = 0, tl = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.n_tiles && ok; t += gridDim.x, ++tl) {
      const int buf = tl & 1;
      if (tl >= 2 && !mbar_wait(&sm.acc_empty[buf], (uint32_t)((tl >> 1) - 1) & 1u, abort,
                                p.status, ANIMA_ERR_TIMEOUT)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t acc = tmem + (uint32_t)buf * kBN;
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const int s = it % kStages;
        if (!mbar_wait(&sm.full[s], (uint32_t)(it / kStages) & 1u, abort, p.status,
                       ANIMA_ERR_TIMEOUT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t da = desc_plus(da0, (uint32_t)s * kATile);
        const uint64_t db = desc_plus(db0, (uint32_t)s * kBTile);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          umma_ss(acc, desc_plus(da, kk * 32), desc_plus(db, kk * 32), idesc,
                  (kb | kk) != 0 ? 1u : 0u);
        umma_commit(&sm.empty[s]);
      }
      if (!ok) break;
      umma_commit(&sm.acc_full[buf]);
    }
    umma_commit(&sm.mma_done);
    attn::drain_wait(&sm.mma_done, 0);
  } else if (warp >= 4 && kEpi == kEpiGelu) {
    // ------------------------------------------------------------ GELU epilogue
    // y = GELU(C) (exact, x (1 + erf(x / sqrt 2)) / 2) on the fp32 accumulator, 16 columns
    // at a time, stored row-major as 16-bit.
    const int quarter = warp & 3;
    const uint32_t lane_field = (uint32_t)(quarter * 32) << 16;
    int tl = 0;
    for (int t = blockIdx.x; t < p.n_tiles; t += gridDim.x, ++tl) {
      const int buf = tl & 1;
      const int m0 = (t / p.n_tiles_n) * kBM, n0 = (t % p.n_tiles_n) * kBN;
      const int wm = m0 + quarter * 32;
      const int nvalid = min(32, p.M - wm);
      const int nchunks = min(kBN, p.N - n0) / 16;  // N is a multiple of 16
      const bool got = mbar_wait(&sm.acc_full[buf], (uint32_t)(tl >> 1) & 1u, abort, p.status,
                                 ANIMA_ERR_TIMEOUT);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const uint32_t tb = tmem + lane_field + (uint32_t)buf * kBN;
      char* const yw = static_cast<char*>(p.y) + ((long long)max(wm, 0) * p.ldy + n0) * 2;
#pragma unroll 1
      for (int j = 0; j < nchunks; ++j) {
        uint32_t r[16];
        tmem_ld16(tb + 16 * j, r);
        tmem_ld_wait();
        if (j == nchunks - 1) {  // the last TMEM read of this buffer is done
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
        }
        float v[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float x = __uint_as_float(r[e]);
          v[e] = 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
        }
        store_half<kDt>(yw, p.ldy * 2, nvalid, v, 16 * j, sm.stage[quarter], lane);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    // Pass 1 reads each normalised head's 128 columns for the sum of squares; pass 2
    // walks 16-pair chunks (columns 16j..16j+15 and 64+16j..64+16j+15 of both heads),
    // applying the norm scale and the rotation and storing.  The RoPE table rows of the
    // tile's tokens serve both heads, and the next chunk's rows are loaded while the
    // current one is processed.
    const int quarter = warp & 3;
    const uint32_t lane_field = (uint32_t)(quarter * 32) << 16;
    const float4* const f4 = reinterpret_cast<const float4*>(p.freqs);
    int tl = 0;
    for (int t = blockIdx.x; t < p.n_tiles; t += gridDim.x, ++tl) {
      const int buf = tl & 1;
      const int m0 = (t / p.n_tiles_n) * kBM, n0 = (t % p.n_tiles_n) * kBN;
      const int wm = m0 + quarter * 32;        // the warp's first token row of x
      const int gw = p.row0 + wm;              // ... in the [B, L] token grid
      const int b = gw / p.L, s0 = gw - b * p.L;
      const int nvalid = min(32, p.M - wm);    // rows of the warp inside the GEMM
      bool hval[2], hnorm[2], hrope[2];
      int hc[2], hh_[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int ncol = n0 + hh * 128;
        const int hb = ncol / 128;
        hval[hh] = ncol < p.N;                 // uniform over the CTA
        hc[hh] = p.tensor0 + hb / p.H;
        hh_[hh] = hb % p.H;
        hnorm[hh] = hval[hh] && hc[hh] < 2 && ((p.norm_mask >> hc[hh]) & 1u);
        hrope[hh] = hval[hh] && hc[hh] < 2 && f4 != nullptr;
      }
      const bool any_rope = hrope[0] || hrope[1];
      // s0 + lane < L (L is a multiple of 32), so the table row is in bounds for every lane
      const float4* const fr = any_rope ? f4 + (long long)(s0 + lane) * 64 : nullptr;
      float4 fc[16];
      if (any_rope) {
#pragma unroll
        for (int e = 0; e < 16; ++e) fc[e] = __ldg(fr + e);
      }
      const bool got = mbar_wait(&sm.acc_full[buf], (uint32_t)(tl >> 1) & 1u, abort, p.status,
                                 ANIMA_ERR_TIMEOUT);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const uint32_t tb = tmem + lane_field + (uint32_t)buf * kBN;
      float rs[2] = {1.f, 1.f};
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        if (!hnorm[hh]) continue;
        float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t r[32];
          tmem_ld32(tb + hh * 128 + q * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float x = __uint_as_float(r[e]);
            s4[e & 3] = fmaf(x, x, s4[e & 3]);
          }
        }
        const float ss = (s4[0] + s4[1]) + (s4[2] + s4[3]);
        rs[hh] = 1.0f / sqrtf(ss / 128.0f + p.eps);
      }
      const int last_hh = hval[1] ? 1 : 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float4 fn[16];
        if (any_rope && j < 3) {
#pragma unroll
          for (int e = 0; e < 16; ++e) fn[e] = __ldg(fr + 16 * (j + 1) + e);
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          if (!hval[hh]) continue;
          uint32_t lo[16], hi[16];
          tmem_ld16(tb + hh * 128 + 16 * j, lo);
          tmem_ld16(tb + hh * 128 + 64 + 16 * j, hi);
          tmem_ld_wait();
          if (j == 3 && hh == last_hh) {       // the last TMEM read of this buffer is done
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
          }
          float a[16], d[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            a[e] = __uint_as_float(lo[e]);
            d[e] = __uint_as_float(hi[e]);
          }
          if (hnorm[hh]) {
            const float* w = sm.norm_w[hc[hh]];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              a[e] *= rs[hh] * w[16 * j + e];
              d[e] *= rs[hh] * w[64 + 16 * j + e];
            }
          }
          if (hrope[hh]) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {    // fc[e] = [cos, -sin, sin, cos] of pair 16j+e
              const float x = a[e], y = d[e];
              a[e] = fc[e].x * x + fc[e].y * y;
              d[e] = fc[e].z * x + fc[e].w * y;
            }
          }
          const int dd = hh_[hh] / p.Hd, hl = hh_[hh] - dd * p.Hd;
          void* base = nullptr;
#pragma unroll
          for (int k = 0; k < kMaxDest; ++k)  // constant indices: no local copy of the params
            if (k == dd)
              base = hc[hh] == 0 ? p.dest[k][0] : hc[hh] == 1 ? p.dest[k][1] : p.dest[k][2];
          char* const out_w = static_cast<char*>(base) +
                              (((long long)b * p.Hd + hl) * p.L + s0) * 256;
          store_half<kDt>(out_w, 256, nvalid, a, 16 * j, sm.stage[quarter], lane);
          store_half<kDt>(out_w, 256, nvalid, d, 64 + 16 * j, sm.stage[quarter], lane);
        }
        if (any_rope && j < 3) {
#pragma unroll
          for (int e = 0; e < 16; ++e) fc[e] = fn[e];
        }
      }
    }
  }
  // teardown: TMEM is released once every warp is done
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace qkv

typedef CUresult (*EncodeTiledFnQ)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFnQ get_encode_fn_q() {
  static EncodeTiledFnQ fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<EncodeTiledFnQ>(ptr);
  }
  return fn;
}

// Row-major [rows, K] 16-bit matrix, box [64 elements][box_rows], 128-byte swizzle.
static int make_rows_map(CUtensorMap* map, const void* base, int dtype, int rows, int K,
                         int box_rows) {
  EncodeTiledFnQ enc = get_encode_fn_q();
  if (!enc) return ANIMA_ERR_CUDA;
  const CUtensorMapDataType dt = dtype == ANIMA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ANIMA_OK : ANIMA_ERR_CUDA;
}

template <int kDt, int kEpi>
static int qkv_launch_t(const CUtensorMap& ma, const CUtensorMap& mb, const qkv::Params& prm,
                        int grid, cudaStream_t st) {
  auto kern = qkv::qkv_gemm_kernel<kDt, kEpi>;
  static int attr_dev_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask & (1 << (dev & 31)))) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)qkv::kSmemBytes) != cudaSuccess)
      return ANIMA_ERR_CUDA;
    attr_dev_mask |= 1 << (dev & 31);
  }
  kern<<<grid, qkv::kThreads, qkv::kSmemBytes, st>>>(ma, mb, prm);
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

int qkv_projection_launch(const AnimaQkvProjArgs* a, int* status, int sm_count, cudaStream_t st) {
  if (a->dtype != ANIMA_DTYPE_F16 && a->dtype != ANIMA_DTYPE_BF16) return ANIMA_ERR_ARG;
  if (a->B <= 0 || a->L <= 0 || a->H <= 0 || a->K <= 0) return ANIMA_ERR_SHAPE;
  if (a->L % 32 != 0 || a->K % 8 != 0) return ANIMA_ERR_SHAPE;
  if (a->n_tensors < 1 || a->first_tensor < 0 || a->first_tensor + a->n_tensors > 3)
    return ANIMA_ERR_ARG;
  void* outs[3] = {a->q_out, a->k_out, a->v_out};
  for (int c = a->first_tensor; c < a->first_tensor + a->n_tensors; ++c)
    if (!outs[c] || (reinterpret_cast<uintptr_t>(outs[c]) & 15u)) return ANIMA_ERR_ARG;
  if (!a->x || !a->w || ((reinterpret_cast<uintptr_t>(a->x) | reinterpret_cast<uintptr_t>(a->w)) & 15u))
    return ANIMA_ERR_ARG;
  const bool rope = (a->flags & ANIMA_FLAG_ROPE) != 0;
  if (rope && (!a->rope_freqs || (reinterpret_cast<uintptr_t>(a->rope_freqs) & 15u)))
    return ANIMA_ERR_ARG;
  const long long M = (long long)a->B * a->L, N = (long long)a->n_tensors * a->H * 128;
  if (M > 0x7fffffffLL || N > 0x7fffffffLL) return ANIMA_ERR_SHAPE;
  CUtensorMap ma, mb;
  int rc;
  if ((rc = make_rows_map(&ma, a->x, a->dtype, (int)M, a->K, qkv::kBM))) return rc;
  if ((rc = make_rows_map(&mb, a->w, a->dtype, (int)N, a->K, qkv::kBN))) return rc;
  qkv::Params prm;
  prm.M = (int)M;
  prm.N = (int)N;
  prm.K = a->K;
  prm.L = a->L;
  prm.H = a->H;
  prm.n_tiles_n = (int)((N + qkv::kBN - 1) / qkv::kBN);
  const long long tiles = ((M + qkv::kBM - 1) / qkv::kBM) * prm.n_tiles_n;
  if (tiles > 0x7fffffffLL) return ANIMA_ERR_SHAPE;
  prm.n_tiles = (int)tiles;
  prm.tensor0 = a->first_tensor;
  prm.norm_w[0] = a->q_norm_w;
  prm.norm_w[1] = a->k_norm_w;
  prm.norm_mask = ((a->flags & ANIMA_FLAG_QNORM) ? 1u : 0u) | ((a->flags & ANIMA_FLAG_KNORM) ? 2u : 0u);
  prm.freqs = rope ? a->rope_freqs : nullptr;
  prm.eps = a->eps;
  prm.row0 = 0;
  prm.Hd = a->H;
  prm.n_dest = 1;
  for (int d = 0; d < qkv::kMaxDest; ++d)
    for (int c = 0; c < 3; ++c) prm.dest[d][c] = d == 0 ? outs[c] : nullptr;
  prm.status = status;
  const int grid = (int)(tiles < sm_count ? tiles : sm_count);
  prm.y = nullptr;
  prm.ldy = 0;
  return a->dtype == ANIMA_DTYPE_BF16
             ? qkv_launch_t<ANIMA_DTYPE_BF16, qkv::kEpiQkv>(ma, mb, prm, grid, st)
             : qkv_launch_t<ANIMA_DTYPE_F16, qkv::kEpiQkv>(ma, mb, prm, grid, st);
}

// The projection of `rows` token rows (tokens row0 .. of the [B, L] grid) for all heads of a
// head split over n_dest ranks (a->H heads each), each head's operand rows stored into the
// buffers of the rank that owns the head: dest[d * 3 + c] is rank d's head-major
// [B * a->H, L, 128] buffer of tensor c (q, k, v).  This is the projection GEMM and the
// all-to-all of its output in one kernel.
int qkv_projection_scatter_launch(const AnimaQkvProjArgs* a, int rows, int row0,
                                  void* const* dest, int n_dest, int* status, int sm_count,
                                  cudaStream_t st) {
  if (a->dtype != ANIMA_DTYPE_F16 && a->dtype != ANIMA_DTYPE_BF16) return ANIMA_ERR_ARG;
  if (a->B <= 0 || a->L <= 0 || a->H <= 0 || a->K <= 0 || rows <= 0 || row0 < 0)
    return ANIMA_ERR_SHAPE;
  if (a->L % 32 != 0 || a->K % 8 != 0 || row0 % 32 != 0) return ANIMA_ERR_SHAPE;
  if ((long long)row0 + rows > (long long)a->B * a->L) return ANIMA_ERR_SHAPE;
  if (n_dest < 1 || n_dest > qkv::kMaxDest || !dest) return ANIMA_ERR_ARG;
  if (a->n_tensors < 1 || a->first_tensor < 0 || a->first_tensor + a->n_tensors > 3)
    return ANIMA_ERR_ARG;
  for (int d = 0; d < n_dest; ++d)
    for (int c = a->first_tensor; c < a->first_tensor + a->n_tensors; ++c) {
      const void* q = dest[d * 3 + c];
      if (!q || (reinterpret_cast<uintptr_t>(q) & 15u)) return ANIMA_ERR_ARG;
    }
  if (!a->x || !a->w || ((reinterpret_cast<uintptr_t>(a->x) | reinterpret_cast<uintptr_t>(a->w)) & 15u))
    return ANIMA_ERR_ARG;
  const bool rope = (a->flags & ANIMA_FLAG_ROPE) != 0;
  if (rope && (!a->rope_freqs || (reinterpret_cast<uintptr_t>(a->rope_freqs) & 15u)))
    return ANIMA_ERR_ARG;
  const long long H = (long long)a->H * n_dest;  // heads per tensor over all ranks
  const long long N = (long long)a->n_tensors * H * 128;
  if (N > 0x7fffffffLL) return ANIMA_ERR_SHAPE;
  CUtensorMap ma, mb;
  int rc;
  if ((rc = make_rows_map(&ma, a->x, a->dtype, rows, a->K, qkv::kBM))) return rc;
  if ((rc = make_rows_map(&mb, a->w, a->dtype, (int)N, a->K, qkv::kBN))) return rc;
  qkv::Params prm;
  memset(&prm, 0, sizeof(prm));
  prm.M = rows;
  prm.N = (int)N;
  prm.K = a->K;
  prm.L = a->L;
  prm.H = (int)H;
  prm.n_tiles_n = (int)((N + qkv::kBN - 1) / qkv::kBN);
  const long long tiles = (long long)((rows + qkv::kBM - 1) / qkv::kBM) * prm.n_tiles_n;
  if (tiles > 0x7fffffffLL) return ANIMA_ERR_SHAPE;
  prm.n_tiles = (int)tiles;
  prm.tensor0 = a->first_tensor;
  prm.norm_w[0] = a->q_norm_w;
  prm.norm_w[1] = a->k_norm_w;
  prm.norm_mask = ((a->flags & ANIMA_FLAG_QNORM) ? 1u : 0u) | ((a->flags & ANIMA_FLAG_KNORM) ? 2u : 0u);
  prm.freqs = rope ? a->rope_freqs : nullptr;
  prm.eps = a->eps;
  prm.row0 = row0;
  prm.Hd = a->H;
  prm.n_dest = n_dest;
  for (int d = 0; d < n_dest; ++d)
    for (int c = 0; c < 3; ++c) prm.dest[d][c] = dest[d * 3 + c];
  prm.status = status;
  const int grid = (int)(tiles < sm_count ? tiles : sm_count);
  return a->dtype == ANIMA_DTYPE_BF16
             ? qkv_launch_t<ANIMA_DTYPE_BF16, qkv::kEpiQkv>(ma, mb, prm, grid, st)
             : qkv_launch_t<ANIMA_DTYPE_F16, qkv::kEpiQkv>(ma, mb, prm, grid, st);
}

// y [M, N] = GELU(x [M, K] W[N, K]^T), 16-bit row-major (the first layer of the DiT block's
// MLP with its activation, predict2.py:45: the cuBLAS GEMM + GELU pass it replaces read and
// wrote the hidden layer once more).
int gemm_gelu_launch(const void* x, const void* w, void* y, int M, int N, int K, int dtype,
                     int* status, int sm_count, cudaStream_t st) {
  if (dtype != ANIMA_DTYPE_F16 && dtype != ANIMA_DTYPE_BF16) return ANIMA_ERR_ARG;
  if (M <= 0 || N <= 0 || K <= 0 || N % 16 != 0 || K % 8 != 0) return ANIMA_ERR_SHAPE;
  if (!x || !w || !y ||
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
        reinterpret_cast<uintptr_t>(y)) & 15u))
    return ANIMA_ERR_ARG;
  CUtensorMap ma, mb;
  int rc;
  if ((rc = make_rows_map(&ma, x, dtype, M, K, qkv::kBM))) return rc;
  if ((rc = make_rows_map(&mb, w, dtype, N, K, qkv::kBN))) return rc;
  qkv::Params prm;
  memset(&prm, 0, sizeof(prm));
  prm.M = M;
  prm.N = N;
  prm.K = K;
  prm.L = 1;
  prm.H = 1;
  prm.n_tiles_n = (N + qkv::kBN - 1) / qkv::kBN;
  const long long tiles = (long long)((M + qkv::kBM - 1) / qkv::kBM) * prm.n_tiles_n;
  if (tiles > 0x7fffffffLL) return ANIMA_ERR_SHAPE;
  prm.n_tiles = (int)tiles;
  prm.y = y;
  prm.ldy = N;
  prm.status = status;
  const int grid = (int)(tiles < sm_count ? tiles : sm_count);
  return dtype == ANIMA_DTYPE_BF16
             ? qkv_launch_t<ANIMA_DTYPE_BF16, qkv::kEpiGelu>(ma, mb, prm, grid, st)
             : qkv_launch_t<ANIMA_DTYPE_F16, qkv::kEpiGelu>(ma, mb, prm, grid, st);
}

}  // namespace anima
