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
// row of that token is read once and reused for every head (layout in prologue_kernel).
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

// Four consecutive elements of a row as fp32.
template <typename T>
__device__ __forceinline__ float4 load4(const T* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
template <>
__device__ __forceinline__ float4 load4<__half>(const __half* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

template <int kOp>
__device__ __forceinline__ uint32_t pack_op(float lo, float hi) {
  return kOp == ANIMA_DTYPE_BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}

// x * inv * w with both products rounded (the reference's order), for 4 lanes of a row.
__device__ __forceinline__ float4 scale4(float4 x, float inv, float4 w) {
  return make_float4(__fmul_rn(__fmul_rn(x.x, inv), w.x), __fmul_rn(__fmul_rn(x.y, inv), w.y),
                     __fmul_rn(__fmul_rn(x.z, inv), w.z), __fmul_rn(__fmul_rn(x.w, inv), w.w));
}

// One RoPE pair (a, c) with table entry f = [cos, -sin, sin, cos]; products and sums
// rounded separately as in the reference (no FMA contraction).
__device__ __forceinline__ void rot(float& a, float& c, float4 f) {
  const float x = __fadd_rn(__fmul_rn(f.x, a), __fmul_rn(f.y, c));
  const float y = __fadd_rn(__fmul_rn(f.z, a), __fmul_rn(f.w, c));
  a = x;
  c = y;
}

// Work item = one token (b, s) of one tensor.  A half-warp owns one head row: lane
// l = lane & 15 holds elements [4l, 4l+4) and [64+4l, 64+4l+4), i.e. RoPE pairs
// p = 4l..4l+3, so the rotation needs no shuffles and the norm reduces over 16 lanes.
// The two half-warps take heads h and h+1; 2*kPairsInFlight heads are loaded before any
// is processed to keep enough bytes in flight per SM.
template <typename Tin, int kOp>
__global__ void __launch_bounds__(256) prologue_kernel(const PrologueParams p) {
  constexpr int kPairsInFlight = 4;  // 8 heads per batch of loads
  const int lane = threadIdx.x & 31;
  const int hl = lane & 15;
  const int half = lane >> 4;
  const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  const long long total = p.tokens_q + 2 * p.tokens_k;

  float4 wlo[2], whi[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const float* w = p.w[t];
    wlo[t] = w ? *reinterpret_cast<const float4*>(w + 4 * hl) : make_float4(1.f, 1.f, 1.f, 1.f);
    whi[t] = w ? *reinterpret_cast<const float4*>(w + 64 + 4 * hl) : make_float4(1.f, 1.f, 1.f, 1.f);
  }

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
                     (long long)s * p.ss[t];
    const long long sh = p.sh[t];
    uint2* dst = reinterpret_cast<uint2*>(p.out[t]);
    const bool norm = (p.norm_mask >> t) & 1u;
    const bool rope = (p.freqs != nullptr) && t < 2;
    const float4 w_lo = t == 1 ? wlo[1] : wlo[0];
    const float4 w_hi = t == 1 ? whi[1] : whi[0];

    float4 f[4];
    if (rope) {
      const float4* fr = reinterpret_cast<const float4*>(p.freqs + (long long)s * 256) + 4 * hl;
#pragma unroll
      for (int k = 0; k < 4; ++k) f[k] = __ldg(fr + k);
    }

    for (int h0 = 0; h0 < p.H; h0 += 2 * kPairsInFlight) {
      float4 lo[kPairsInFlight], hi[kPairsInFlight];
#pragma unroll
      for (int u = 0; u < kPairsInFlight; ++u) {
        const int h = h0 + 2 * u + half;
        if (h < p.H) {
          const Tin* row = src + (long long)h * sh;
          lo[u] = load4<Tin>(row + 4 * hl);
          hi[u] = load4<Tin>(row + 64 + 4 * hl);
        } else {
          lo[u] = hi[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int u = 0; u < kPairsInFlight; ++u) {
        const int h = h0 + 2 * u + half;
        float4 a = lo[u], c = hi[u];
        if (norm) {
          float ss = a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w + c.x * c.x + c.y * c.y +
                     c.z * c.z + c.w * c.w;
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          const float inv = 1.0f / sqrtf(ss / 128.0f + p.eps);
          a = scale4(a, inv, w_lo);
          c = scale4(c, inv, w_hi);
        }
        if (rope) {
          rot(a.x, c.x, f[0]);
          rot(a.y, c.y, f[1]);
          rot(a.z, c.z, f[2]);
          rot(a.w, c.w, f[3]);
        }
        if (h < p.H) {
          const long long orow = (((long long)b * p.H + h) * S + s) * 32;  // 8-byte units
          dst[orow + hl] = make_uint2(pack_op<kOp>(a.x, a.y), pack_op<kOp>(a.z, a.w));
          dst[orow + 16 + hl] = make_uint2(pack_op<kOp>(c.x, c.y), pack_op<kOp>(c.z, c.w));
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

// ---------------------------------------------------------------- launchers
static int grid_for(long long warps_needed, int threads, int sm_count) {
  long long blocks = (warps_needed * 32 + threads - 1) / threads;
  const long long cap = (long long)sm_count * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

template <typename Tin, int kOp>
static int prologue_t(const PrologueParams& prm, int sm_count, cudaStream_t st) {
  const long long items = prm.tokens_q + 2 * prm.tokens_k;
  prologue_kernel<Tin, kOp><<<grid_for(items, 256, sm_count), 256, 0, st>>>(prm);
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

int prologue_launch(const AnimaPrologueArgs* a, int sm_count, cudaStream_t st) {
  if (a->D != 128) return ANIMA_ERR_SHAPE;
  if (a->B <= 0 || a->H <= 0 || a->S_q <= 0 || a->S_kv <= 0) return ANIMA_ERR_SHAPE;
  if (!a->q || !a->k || !a->v || !a->q_out || !a->k_out || !a->v_out) return ANIMA_ERR_ARG;
  if ((a->flags & ANIMA_FLAG_ROPE) && (!a->rope_freqs || a->S_q != a->S_kv))
    return ANIMA_ERR_ARG;
  const int esz = a->in_dtype == ANIMA_DTYPE_F32 ? 4 : 2;
  const int64_t* st3[3] = {a->q_stride, a->k_stride, a->v_stride};
  const void* in3[3] = {a->q, a->k, a->v};
  PrologueParams prm;
  for (int t = 0; t < 3; ++t) {
    for (int d = 0; d < 3; ++d)
      if (st3[t][d] < 0 || (st3[t][d] % 4) != 0) return ANIMA_ERR_ARG;  // 4-element loads
    if ((reinterpret_cast<uintptr_t>(in3[t]) % (4 * esz)) != 0) return ANIMA_ERR_ARG;
    prm.in[t] = in3[t];
    prm.sb[t] = st3[t][0];
    prm.ss[t] = st3[t][1];
    prm.sh[t] = st3[t][2];
  }
  if ((reinterpret_cast<uintptr_t>(a->rope_freqs) & 15u) != 0) return ANIMA_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(a->q_norm_w) & 15u) || (reinterpret_cast<uintptr_t>(a->k_norm_w) & 15u))
    return ANIMA_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(a->q_out) | reinterpret_cast<uintptr_t>(a->k_out) |
       reinterpret_cast<uintptr_t>(a->v_out)) & 15u)
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
