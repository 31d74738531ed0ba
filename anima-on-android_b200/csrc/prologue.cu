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
// row of that token is read once and reused for every head.  Lane t holds elements
// {2t, 2t+1} and {64+2t, 64+2t+1} of a row: exactly the RoPE pairs p = 2t, 2t+1.
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

template <typename T>
__device__ __forceinline__ float2 load2(const T* p);
template <>
__device__ __forceinline__ float2 load2<float>(const float* p) {
  return *reinterpret_cast<const float2*>(p);
}
template <>
__device__ __forceinline__ float2 load2<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
template <>
__device__ __forceinline__ float2 load2<__half>(const __half* p) {
  return __half22float2(*reinterpret_cast<const __half2*>(p));
}

template <int kOp>
__device__ __forceinline__ uint32_t pack_op(float lo, float hi) {
  return kOp == ANIMA_DTYPE_BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}

template <typename Tin, int kOp>
__global__ void __launch_bounds__(256) prologue_kernel(const PrologueParams p) {
  const int lane = threadIdx.x & 31;
  const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  const long long total = p.tokens_q + 2 * p.tokens_k;

  float wq[4], wk[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int col = (e < 2) ? 2 * lane + e : 64 + 2 * lane + (e - 2);
    wq[e] = p.w[0] ? p.w[0][col] : 1.f;
    wk[e] = p.w[1] ? p.w[1][col] : 1.f;
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
    uint32_t* dst = reinterpret_cast<uint32_t*>(p.out[t]);
    const bool norm = (p.norm_mask >> t) & 1u;
    const bool rope = (p.freqs != nullptr) && t < 2;
    const float* w = t == 0 ? wq : wk;

    float4 f0 = make_float4(1.f, 0.f, 0.f, 1.f), f1 = f0;
    if (rope) {
      const float4* fr = reinterpret_cast<const float4*>(p.freqs + (long long)s * 256) + 2 * lane;
      f0 = __ldg(fr);
      f1 = __ldg(fr + 1);
    }

#pragma unroll 4
    for (int h = 0; h < p.H; ++h) {
      const Tin* row = src + (long long)h * p.sh[t];
      float2 a = load2<Tin>(row + 2 * lane);
      float2 c = load2<Tin>(row + 64 + 2 * lane);
      if (norm) {
        float ss = a.x * a.x + a.y * a.y + c.x * c.x + c.y * c.y;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = 1.0f / sqrtf(ss / 128.0f + p.eps);
        a.x = __fmul_rn(__fmul_rn(a.x, inv), w[0]);
        a.y = __fmul_rn(__fmul_rn(a.y, inv), w[1]);
        c.x = __fmul_rn(__fmul_rn(c.x, inv), w[2]);
        c.y = __fmul_rn(__fmul_rn(c.y, inv), w[3]);
      }
      if (rope) {
        // pair p = 2*lane uses f0 = [cos, -sin, sin, cos], pair 2*lane+1 uses f1
        const float x0 = __fadd_rn(__fmul_rn(f0.x, a.x), __fmul_rn(f0.y, c.x));
        const float y0 = __fadd_rn(__fmul_rn(f0.z, a.x), __fmul_rn(f0.w, c.x));
        const float x1 = __fadd_rn(__fmul_rn(f1.x, a.y), __fmul_rn(f1.y, c.y));
        const float y1 = __fadd_rn(__fmul_rn(f1.z, a.y), __fmul_rn(f1.w, c.y));
        a = make_float2(x0, x1);
        c = make_float2(y0, y1);
      }
      const long long orow = (((long long)b * p.H + h) * S + s) * 64;  // in 32-bit words
      dst[orow + lane] = pack_op<kOp>(a.x, a.y);
      dst[orow + 32 + lane] = pack_op<kOp>(c.x, c.y);
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
      if (st3[t][d] < 0 || (st3[t][d] % 2) != 0) return ANIMA_ERR_ARG;  // pair loads
    if ((reinterpret_cast<uintptr_t>(in3[t]) % (2 * esz)) != 0) return ANIMA_ERR_ARG;
    prm.in[t] = in3[t];
    prm.sb[t] = st3[t][0];
    prm.ss[t] = st3[t][1];
    prm.sh[t] = st3[t][2];
  }
  if ((reinterpret_cast<uintptr_t>(a->rope_freqs) & 15u) != 0) return ANIMA_ERR_ARG;
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
