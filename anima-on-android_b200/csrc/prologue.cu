// prologue.cu -- the HBM-bound passes around the attention core.
//
// prologue_kernel: one pass over the projections that replaces, per attention call,
//   q/k RMSNorm   anima_rt/include/cpu/rmsnorm_kernel.h:11-33 (via anima_rt.cpp:45-50,
//                 called per (token, head) row of D = 128 at numpy_dit.py:285-286)
//   RoPE          anima_rt/include/cpu/rope_kernel.h:30-62 / predict2.py:31-38
//                 (pairs (p, 64 + p), table [S, 64, 2, 2] = [cos, -sin, sin, cos])
//   transpose     numpy_dit.py:291 ([B,S,H,D] -> [B,H,S,D])
//   cast          fp32 -> bf16/f16 operands for the tensor cores
// One warp owns one token (b, s) of one tensor and walks its H head rows, so the RoPE
// row of that token is read once and reused for every head (layout in prologue_kernel);
// every lane moves 16 bytes per load for fp32 and 16-bit inputs alike.
//
// rmsnorm_kernel / rope_kernel: the stand-alone drop-ins behind anima_rt_run_rmsnorm
// and anima_rt_run_rope (fp32 in, fp32 out, any row length / even head size).
#include "common.cuh"

namespace anima {

struct PrologueParams {
  const void* in[3];
  long long sb[3], ss[3], sh[3];
  void* out[3];
  int S[3];
  int B, H;
  const float* w[2];  // q, k norm weights (nullptr = 1)
  unsigned norm_mask; // bit t: normalise tensor t
  const float* freqs; // nullptr = no RoPE
  float eps;
  long long tokens_q, tokens_k;  // B*S_q, B*S_kv
};

// One 16-byte load: 4 fp32 or 8 16-bit elements of a row, kept raw until used.
template <typename Tin>
__device__ __forceinline__ uint4 load16(const Tin* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// Raw 16 bytes -> E floats.
template <typename Tin>
__device__ __forceinline__ void widen(const uint4& u, float* f);
template <>
__device__ __forceinline__ void widen<float>(const uint4& u, float* f) {
  f[0] = __uint_as_float(u.x);
  f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z);
  f[3] = __uint_as_float(u.w);
}
template <>
__device__ __forceinline__ void widen<__half>(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}
template <>
__device__ __forceinline__ void widen<__nv_bfloat16>(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

template <int kOp>
__device__ __forceinline__ uint32_t pack_op(float lo, float hi) {
  return kOp == ANIMA_DTYPE_BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}

// E floats -> E 16-bit operands at p (E = 4: 8 bytes, E = 8: 16 bytes).
template <int E, int kOp>
__device__ __forceinline__ void store_op(void* p, const float* v) {
  if constexpr (E == 4) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_op<kOp>(v[0], v[1]), pack_op<kOp>(v[2], v[3]));
  } else {
    *reinterpret_cast<uint4*>(p) = make_uint4(pack_op<kOp>(v[0], v[1]), pack_op<kOp>(v[2], v[3]),
                                              pack_op<kOp>(v[4], v[5]), pack_op<kOp>(v[6], v[7]));
  }
}

// One RoPE pair (a, c) with table entry f = [cos, -sin, sin, cos]; products and sums
// rounded separately as in the reference (no FMA contraction).
__device__ __forceinline__ void rot(float& a, float& c, float4 f) {
  const float x = __fadd_rn(__fmul_rn(f.x, a), __fmul_rn(f.y, c));
  const float y = __fadd_rn(__fmul_rn(f.z, a), __fmul_rn(f.w, c));
  a = x;
  c = y;
}

// Work item = one token (b, s) of one tensor; the warp walks that token's H head rows,
// so the token's RoPE row is read once and reused for every head.
// A head row (D = 128) is held by R = 64 / E lanes, E = 16 / sizeof(Tin) elements per
// 16-byte load: lane l of the group holds elements [E*l, E*l + E) and 64 + the same,
// i.e. RoPE pairs p = E*l .. E*l + E - 1, so the rotation needs no shuffles and the norm
// reduces over the R lanes.  The warp's 32 / R lane groups take consecutive heads, and
// kPasses such passes are loaded before any is processed: 16 heads (fp32: 8) and 4 KiB
// per warp in flight.
// Occupancy: three 256-thread blocks per SM for fp32 input (80 registers; 9 % faster than
// two), two for 16-bit input.
template <typename Tin, int kOp>
__global__ void __launch_bounds__(256, sizeof(Tin) == 4 ? 3 : 2) prologue_kernel(const PrologueParams p) {
  constexpr int E = 16 / (int)sizeof(Tin);
  constexpr int R = 64 / E;       // lanes per head row
  constexpr int G = 32 / R;       // head rows per pass
  constexpr int kPasses = 4;
  constexpr int HB = G * kPasses; // heads per batch of loads
  const int lane = threadIdx.x & 31;
  const int gl = lane % R;        // lane within the row group
  const int grp = lane / R;
  const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  const long long total = p.tokens_q + 2 * p.tokens_k;
  // The attention kernel that follows may begin its set-up; it reads nothing of ours
  // before this grid has completed.
  grid_dependents_launch();

  for (long long item = warp0; item < total; item += nwarps) {
    int t;
    long long tok;
    if (item < p.tokens_q) {
      t = 0;
      tok = item;
    } else if (item < p.tokens_q + p.tokens_k) {
      t = 1;
      tok = item - p.tokens_q;
    } else {
      t = 2;
      tok = item - p.tokens_q - p.tokens_k;
    }
    const int S = p.S[t];
    const int b = (int)(tok / S);
    const int s = (int)(tok - (long long)b * S);
    const Tin* src = reinterpret_cast<const Tin*>(p.in[t]) + (long long)b * p.sb[t] +
                     (long long)s * p.ss[t] + E * gl;
    const long long sh = p.sh[t];
    char* dst = reinterpret_cast<char*>(p.out[t]);
    const bool norm = (p.norm_mask >> t) & 1u;
    const bool rope = (p.freqs != nullptr) && t < 2;

    float wl[E], wh[E];
    {
      const float* w = t < 2 ? p.w[t] : nullptr;
#pragma unroll
      for (int e = 0; e < E; e += 4) {
        const float4 a = (norm && w) ? __ldg(reinterpret_cast<const float4*>(w + E * gl + e))
                                     : make_float4(1.f, 1.f, 1.f, 1.f);
        const float4 c = (norm && w) ? __ldg(reinterpret_cast<const float4*>(w + 64 + E * gl + e))
                                     : make_float4(1.f, 1.f, 1.f, 1.f);
        wl[e] = a.x; wl[e + 1] = a.y; wl[e + 2] = a.z; wl[e + 3] = a.w;
        wh[e] = c.x; wh[e + 1] = c.y; wh[e + 2] = c.z; wh[e + 3] = c.w;
      }
    }
    float4 f[E];
    if (rope) {
      const float4* fr = reinterpret_cast<const float4*>(p.freqs + (long long)s * 256) + E * gl;
#pragma unroll
      for (int k = 0; k < E; ++k) f[k] = __ldg(fr + k);
    }

    for (int h0 = 0; h0 < p.H; h0 += HB) {
      uint4 lo[kPasses], hi[kPasses];
#pragma unroll
      for (int u = 0; u < kPasses; ++u) {
        const int h = h0 + G * u + grp;
        if (h < p.H) {
          const Tin* row = src + (long long)h * sh;
          lo[u] = load16<Tin>(row);
          hi[u] = load16<Tin>(row + 64);
        } else {
          lo[u] = hi[u] = make_uint4(0u, 0u, 0u, 0u);
        }
      }
#pragma unroll
      for (int u = 0; u < kPasses; ++u) {
        const int h = h0 + G * u + grp;
        float a[E], c[E];
        widen<Tin>(lo[u], a);
        widen<Tin>(hi[u], c);
        if (norm) {
          float ss = 0.f;
#pragma unroll
          for (int e = 0; e < E; ++e) ss += a[e] * a[e] + c[e] * c[e];
#pragma unroll
          for (int o = R / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          const float inv = 1.0f / sqrtf(ss / 128.0f + p.eps);
          // x * inv * w with both products rounded (the reference's order)
#pragma unroll
          for (int e = 0; e < E; ++e) {
            a[e] = __fmul_rn(__fmul_rn(a[e], inv), wl[e]);
            c[e] = __fmul_rn(__fmul_rn(c[e], inv), wh[e]);
          }
        }
        if (rope) {
#pragma unroll
          for (int e = 0; e < E; ++e) rot(a[e], c[e], f[e]);
        }
        if (h < p.H) {
          char* orow = dst + ((((long long)b * p.H + h) * S + s) * 128 + E * gl) * 2;
          store_op<E, kOp>(orow, a);
          store_op<E, kOp>(orow + 128, c);
        }
      }
    }
  }
}

// y = x * (1/sqrt(mean(x^2) + eps)) (* w), fp32 [m, d]; one warp per row.
__global__ void __launch_bounds__(256)
    rmsnorm_kernel(const float* x, const float* w, float* y, long long m, int d, float eps) {
  const int lane = threadIdx.x & 31;
  const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long r = warp0; r < m; r += nwarps) {
    const float* xr = x + r * d;
    float ss = 0.f;
    for (int j = lane; j < d; j += 32) ss += xr[j] * xr[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf(ss / (float)d + eps);
    float* yr = y + r * d;
    for (int j = lane; j < d; j += 32) {
      float v = __fmul_rn(xr[j], inv);
      if (w) v = __fmul_rn(v, w[j]);
      yr[j] = v;
    }
  }
}

// Half-split RoPE on t [N, S, D]; one thread per (n, s, pair).  Products and the sum
// are rounded separately, as in the reference, so results are bit-identical.
__global__ void __launch_bounds__(256)
    rope_kernel(const float* t, const float* f, float* out, int N, int S, int D) {
  const int half = D / 2;
  const long long total = (long long)N * S * half;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int pr = (int)(idx % half);
    const long long ns = idx / half;
    const int s = (int)(ns % S);
    const float* x = t + ns * D;
    const float* fr = f + (long long)s * D * 2 + 4 * pr;
    const float a = x[pr], c = x[half + pr];
    out[ns * D + pr] = __fadd_rn(__fmul_rn(fr[0], a), __fmul_rn(fr[1], c));
    out[ns * D + half + pr] = __fadd_rn(__fmul_rn(fr[2], a), __fmul_rn(fr[3], c));
  }
}

// RoPE on a strided fp32 view [O, S, Hn, D] (D contiguous) into another: t at element
// offset o*ts[0] + s*ts[1] + h*ts[2], out likewise with os_[].  Same arithmetic as
// rope_kernel.  Covers the reference's [N, S, D] (O = N, Hn = 1) and predict2's
// [B, S, H, D] (apply_rotary_pos_emb) without a transpose copy.
__global__ void __launch_bounds__(256)
    rope_strided_kernel(const float* t, long long ts0, long long ts1, long long ts2,
                        const float* f, float* out, long long os0, long long os1, long long os2,
                        int O, int S, int Hn, int D) {
  const int half = D / 2;
  const long long total = (long long)O * S * Hn * half;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int pr = (int)(idx % half);
    long long r = idx / half;
    const int h = (int)(r % Hn);
    r /= Hn;
    const int s = (int)(r % S);
    const long long o = r / S;
    const float* x = t + o * ts0 + s * ts1 + h * ts2;
    float* y = out + o * os0 + s * os1 + h * os2;
    const float* fr = f + (long long)s * D * 2 + 4 * pr;
    const float a = x[pr], c = x[half + pr];
    y[pr] = __fadd_rn(__fmul_rn(fr[0], a), __fmul_rn(fr[1], c));
    y[half + pr] = __fadd_rn(__fmul_rn(fr[2], a), __fmul_rn(fr[3], c));
  }
}

// prologue_tokens_kernel: prologue_kernel's arithmetic for calls with few heads (H at most
// half of the HB rows a warp loads per batch: 4 for fp32, 8 for 16-bit input, i.e. the head
// split over 4 or more GPUs).  prologue_kernel's item is one token, so with H = 2 a warp has
// 2 of its 8 row slots (1 KiB) in flight and the pass is latency-bound (measured: 26.5 us
// for 37.7 MB at H = 2, 1.4 TB/s).  Here an item is TG = HB / H consecutive tokens of one
// tensor, so every batch fills its HB rows.  Each pass needs the RoPE row of its own token;
// those rows are prefetched into L1 with the data loads and read when the pass is processed,
// so they hold no registers while the loads are in flight.
template <typename T>
__device__ __forceinline__ T sel3(const T (&a)[3], int t) {  // no runtime index into params
  return t == 0 ? a[0] : t == 1 ? a[1] : a[2];
}

__device__ __forceinline__ void prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

template <typename Tin, int kOp>
__global__ void __launch_bounds__(256, sizeof(Tin) == 4 ? 3 : 2)
    prologue_tokens_kernel(const PrologueParams p, int TG, long long items_q, long long items_k) {
  constexpr int E = 16 / (int)sizeof(Tin);
  constexpr int R = 64 / E;        // lanes per head row
  constexpr int G = 32 / R;        // head rows per pass
  constexpr int kPasses = 4;
  const int lane = threadIdx.x & 31;
  const int gl = lane % R;
  const int grp = lane / R;
  const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  const long long total = items_q + 2 * items_k;
  grid_dependents_launch();  // as in prologue_kernel

  for (long long item = warp0; item < total; item += nwarps) {
    int t;
    long long it, tokens;
    if (item < items_q) {
      t = 0;
      it = item;
      tokens = p.tokens_q;
    } else if (item < items_q + items_k) {
      t = 1;
      it = item - items_q;
      tokens = p.tokens_k;
    } else {
      t = 2;
      it = item - items_q - items_k;
      tokens = p.tokens_k;
    }
    const int S = sel3(p.S, t);
    const long long sb = sel3(p.sb, t), ss_ = sel3(p.ss, t), sh = sel3(p.sh, t);
    const long long tok0 = it * TG;
    const int b0 = (int)(tok0 / S);
    const int s0 = (int)(tok0 - (long long)b0 * S);
    const Tin* base = reinterpret_cast<const Tin*>(sel3(p.in, t)) + E * gl;
    char* dst = reinterpret_cast<char*>(sel3(p.out, t));
    const bool norm = (p.norm_mask >> t) & 1u;
    const bool rope = (p.freqs != nullptr) && t < 2;

    uint4 lo[kPasses], hi[kPasses];
    int rb[kPasses], rs[kPasses], rh[kPasses];
    bool ok[kPasses];
#pragma unroll
    for (int u = 0; u < kPasses; ++u) {
      int tl = 0, h = G * u + grp;  // this lane group's row of the item: token tl, head h
      while (h >= p.H) {
        h -= p.H;
        ++tl;
      }
      int si = s0 + tl, b = b0;
      while (si >= S) {  // the item's tokens may run into the next sample
        si -= S;
        ++b;
      }
      rb[u] = b;
      rs[u] = si;
      rh[u] = h;
      ok[u] = tl < TG && tok0 + tl < tokens;
      if (ok[u]) {
        const Tin* row = base + (long long)b * sb + (long long)si * ss_ + (long long)h * sh;
        lo[u] = load16<Tin>(row);
        hi[u] = load16<Tin>(row + 64);
        if (rope) prefetch_l1(p.freqs + (long long)si * 256 + 4 * E * gl);
      } else {  // no row here: defined values for the norm shuffle, nothing stored
        lo[u] = hi[u] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    float wl[E], wh[E];
    {
      const float* w = t == 0 ? p.w[0] : t == 1 ? p.w[1] : nullptr;
#pragma unroll
      for (int e = 0; e < E; e += 4) {
        const float4 a = (norm && w) ? __ldg(reinterpret_cast<const float4*>(w + E * gl + e))
                                     : make_float4(1.f, 1.f, 1.f, 1.f);
        const float4 c = (norm && w) ? __ldg(reinterpret_cast<const float4*>(w + 64 + E * gl + e))
                                     : make_float4(1.f, 1.f, 1.f, 1.f);
        wl[e] = a.x; wl[e + 1] = a.y; wl[e + 2] = a.z; wl[e + 3] = a.w;
        wh[e] = c.x; wh[e + 1] = c.y; wh[e + 2] = c.z; wh[e + 3] = c.w;
      }
    }
#pragma unroll
    for (int u = 0; u < kPasses; ++u) {
      float a[E], c[E];
      widen<Tin>(lo[u], a);
      widen<Tin>(hi[u], c);
      if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) ss += a[e] * a[e] + c[e] * c[e];
#pragma unroll
        for (int o = R / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = 1.0f / sqrtf(ss / 128.0f + p.eps);
        // x * inv * w with both products rounded (the reference's order)
#pragma unroll
        for (int e = 0; e < E; ++e) {
          a[e] = __fmul_rn(__fmul_rn(a[e], inv), wl[e]);
          c[e] = __fmul_rn(__fmul_rn(c[e], inv), wh[e]);
        }
      }
      if (rope && ok[u]) {
        const float4* fr = reinterpret_cast<const float4*>(p.freqs + (long long)rs[u] * 256) + E * gl;
#pragma unroll
        for (int e = 0; e < E; ++e) rot(a[e], c[e], __ldg(fr + e));
      }
      if (ok[u]) {
        char* orow = dst + ((((long long)rb[u] * p.H + rh[u]) * S + rs[u]) * 128 + E * gl) * 2;
        store_op<E, kOp>(orow, a);
        store_op<E, kOp>(orow + 128, c);
      }
    }
  }
}

// ---------------------------------------------------------------- launchers
static int grid_for(long long warps_needed, int threads, int sm_count) {
  long long blocks = (warps_needed * 32 + threads - 1) / threads;
  const long long cap = (long long)sm_count * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

// Few heads (H <= HB / 2): prologue_tokens_kernel with TG = HB / H tokens per item;
// otherwise prologue_kernel, one token per item.
template <typename Tin, int kOp>
static int prologue_t(const PrologueParams& prm, int sm_count, cudaStream_t st) {
  constexpr int HB = (32 / (64 / (16 / (int)sizeof(Tin)))) * 4;  // rows per batch: 8 or 16
  if (2 * prm.H <= HB) {
    const int TG = HB / prm.H;
    const long long items_q = (prm.tokens_q + TG - 1) / TG;
    const long long items_k = (prm.tokens_k + TG - 1) / TG;
    prologue_tokens_kernel<Tin, kOp><<<grid_for(items_q + 2 * items_k, 256, sm_count), 256, 0, st>>>(
        prm, TG, items_q, items_k);
    return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
  }
  const long long items = prm.tokens_q + 2 * prm.tokens_k;
  prologue_kernel<Tin, kOp><<<grid_for(items, 256, sm_count), 256, 0, st>>>(prm);
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

int prologue_launch(const AnimaPrologueArgs* a, int sm_count, cudaStream_t st) {
  if (a->D != 128) return ANIMA_ERR_SHAPE;
  // S_q == 0 or S_kv == 0 skips that side; its pointers may then be null.
  if (a->B <= 0 || a->H <= 0 || a->S_q < 0 || a->S_kv < 0 || (a->S_q == 0 && a->S_kv == 0))
    return ANIMA_ERR_SHAPE;
  const bool has[3] = {a->S_q > 0, a->S_kv > 0, a->S_kv > 0};
  if ((has[0] && (!a->q || !a->q_out)) || (has[1] && (!a->k || !a->v || !a->k_out || !a->v_out)))
    return ANIMA_ERR_ARG;
  if ((a->flags & ANIMA_FLAG_ROPE) && (!a->rope_freqs || a->S_q != a->S_kv))
    return ANIMA_ERR_ARG;
  const int esz = a->in_dtype == ANIMA_DTYPE_F32 ? 4 : 2;
  const int64_t* st3[3] = {a->q_stride, a->k_stride, a->v_stride};
  const void* in3[3] = {a->q, a->k, a->v};
  void* out3[3] = {a->q_out, a->k_out, a->v_out};
  PrologueParams prm;
  for (int t = 0; t < 3; ++t) {
    prm.in[t] = nullptr;
    prm.sb[t] = prm.ss[t] = prm.sh[t] = 0;
    if (!has[t]) continue;
    const int vec = 16 / esz;  // elements per 16-byte load
    for (int d = 0; d < 3; ++d)
      if (st3[t][d] < 0 || (st3[t][d] % vec) != 0) return ANIMA_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(in3[t]) & 15u) != 0) return ANIMA_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(out3[t]) & 15u) != 0) return ANIMA_ERR_ARG;
    prm.in[t] = in3[t];
    prm.sb[t] = st3[t][0];
    prm.ss[t] = st3[t][1];
    prm.sh[t] = st3[t][2];
  }
  if ((reinterpret_cast<uintptr_t>(a->rope_freqs) & 15u) != 0) return ANIMA_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(a->q_norm_w) & 15u) || (reinterpret_cast<uintptr_t>(a->k_norm_w) & 15u))
    return ANIMA_ERR_ARG;
  prm.out[0] = a->q_out;
  prm.out[1] = a->k_out;
  prm.out[2] = a->v_out;
  prm.S[0] = a->S_q;
  prm.S[1] = a->S_kv;
  prm.S[2] = a->S_kv;
  prm.B = a->B;
  prm.H = a->H;
  prm.w[0] = a->q_norm_w;
  prm.w[1] = a->k_norm_w;
  prm.norm_mask = ((a->flags & ANIMA_FLAG_QNORM) ? 1u : 0u) | ((a->flags & ANIMA_FLAG_KNORM) ? 2u : 0u);
  prm.freqs = (a->flags & ANIMA_FLAG_ROPE) ? a->rope_freqs : nullptr;
  prm.eps = a->eps;
  prm.tokens_q = (long long)a->B * a->S_q;
  prm.tokens_k = (long long)a->B * a->S_kv;
  const bool bf = a->op_dtype == ANIMA_DTYPE_BF16;
  if (a->op_dtype != ANIMA_DTYPE_BF16 && a->op_dtype != ANIMA_DTYPE_F16) return ANIMA_ERR_ARG;
  switch (a->in_dtype) {
    case ANIMA_DTYPE_F32:
      return bf ? prologue_t<float, ANIMA_DTYPE_BF16>(prm, sm_count, st)
                : prologue_t<float, ANIMA_DTYPE_F16>(prm, sm_count, st);
    case ANIMA_DTYPE_BF16:
      return bf ? prologue_t<__nv_bfloat16, ANIMA_DTYPE_BF16>(prm, sm_count, st)
                : prologue_t<__nv_bfloat16, ANIMA_DTYPE_F16>(prm, sm_count, st);
    case ANIMA_DTYPE_F16:
      return bf ? prologue_t<__half, ANIMA_DTYPE_BF16>(prm, sm_count, st)
                : prologue_t<__half, ANIMA_DTYPE_F16>(prm, sm_count, st);
  }
  return ANIMA_ERR_ARG;
}

int rmsnorm_launch(const float* x, const float* w, float* y, long long m, int d, float eps,
                   int sm_count, cudaStream_t st) {
  rmsnorm_kernel<<<grid_for(m, 256, sm_count), 256, 0, st>>>(x, w, y, m, d, eps);
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

int rope_launch(const float* t, const float* f, float* out, int N, int S, int D, int sm_count,
                cudaStream_t st) {
  const long long total = (long long)N * S * (D / 2);
  long long blocks = (total + 255) / 256;
  if (blocks > (long long)sm_count * 16) blocks = (long long)sm_count * 16;
  if (blocks < 1) blocks = 1;
  rope_kernel<<<(int)blocks, 256, 0, st>>>(t, f, out, N, S, D);
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

}  // namespace anima

namespace anima {
int rope_strided_launch(const float* t, const long long* ts, const float* f, float* out,
                        const long long* os, int O, int S, int Hn, int D, int sm_count,
                        cudaStream_t st) {
  const long long total = (long long)O * S * Hn * (D / 2);
  if (total == 0) return ANIMA_OK;
  long long blocks = (total + 255) / 256;
  if (blocks > (long long)sm_count * 8) blocks = (long long)sm_count * 8;
  rope_strided_kernel<<<(int)blocks, 256, 0, st>>>(t, ts[0], ts[1], ts[2], f, out, os[0], os[1],
                                                    os[2], O, S, Hn, D);
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}
}  // namespace anima
