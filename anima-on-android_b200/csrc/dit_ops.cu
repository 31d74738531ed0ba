// dit_ops.cu -- fused HBM-bound passes of the DiT block around the attention.
//
// The block (src/predict2.py:469-583) applies, three times per block,
//   h = LayerNorm(x) * (1 + scale) + shift        (predict2.py:512-513, eps 1e-6, no affine)
// followed by a GEMM on h, and the gated residual
//   x = x + gate * y                              (predict2.py:536, 563, 582)
// on the GEMM's output y.  Unfused, each is 3-5 separate elementwise passes over the
// fp32 residual stream [B, L, 2048]; here each is one pass:
//   ln_modulate_kernel    x fp32 -> h 16-bit (the GEMM's operand type), one warp per row
//   gate_residual_kernel  x += gate[b] * y, fp32, in place, float4-vectorised
//   gate_residual_ln_modulate_kernel  the two back to back (every gated residual is
//                         followed by the next sub-block's LayerNorm + modulation)
//   gelu16_kernel         exact GELU on the 16-bit MLP hidden layer
// scale / shift / gate are per-sample rows [B, D] (adaLN-LoRA outputs), addressed with a
// batch stride so the chunks of one [B, 3D] tensor can be passed without copies.
#include "common.cuh"

namespace anima {

template <int kOut>
__device__ __forceinline__ void store4(void* base, long long idx, float a, float b, float c,
                                       float d) {
  uint2 v = kOut == ANIMA_DTYPE_BF16 ? make_uint2(pack_bf16x2(a, b), pack_bf16x2(c, d))
                                     : make_uint2(pack_f16x2(a, b), pack_f16x2(c, d));
  reinterpret_cast<uint2*>(base)[idx] = v;
}

// One warp per row of kD floats (kD / 128 float4 per lane).  Two-pass mean / variance
// on the row held in registers.
template <int kD, int kOut>
__global__ void __launch_bounds__(256)
    ln_modulate_kernel(const float* __restrict__ x, const float* __restrict__ scale,
                       const float* __restrict__ shift, long long mod_stride, void* y,
                       long long rows, int rows_per_b, float eps) {
  constexpr int kV = kD / 128;  // float4 per lane
  const int lane = threadIdx.x & 31;
  const long long w0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long r = w0; r < rows; r += nw) {
    const float4* xr = reinterpret_cast<const float4*>(x + r * kD);
    float4 v[kV];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kV; ++k) {
      v[k] = xr[lane + 32 * k];
      s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / (float)kD;
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < kV; ++k) {
      const float a = v[k].x - mean, b = v[k].y - mean, c = v[k].z - mean, d = v[k].w - mean;
      q += (a * a + b * b) + (c * c + d * d);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float rstd = 1.0f / sqrtf(q / (float)kD + eps);
    const long long b = r / rows_per_b;
    const float4* sc = reinterpret_cast<const float4*>(scale + b * mod_stride);
    const float4* sh = reinterpret_cast<const float4*>(shift + b * mod_stride);
#pragma unroll
    for (int k = 0; k < kV; ++k) {
      const float4 a = __ldg(sc + lane + 32 * k), c = __ldg(sh + lane + 32 * k);
      store4<kOut>(y, r * (kD / 4) + lane + 32 * k,
                   (v[k].x - mean) * rstd * (1.f + a.x) + c.x, (v[k].y - mean) * rstd * (1.f + a.y) + c.y,
                   (v[k].z - mean) * rstd * (1.f + a.z) + c.z, (v[k].w - mean) * rstd * (1.f + a.w) + c.w);
    }
  }
}

// x[r, :] += gate[r / rows_per_b, :] * y[r, :]; D a multiple of 4.
__global__ void __launch_bounds__(256)
    gate_residual_kernel(float* __restrict__ x, const float* __restrict__ gate, long long gate_stride,
                         const float* __restrict__ y, long long rows, int rows_per_b, int D) {
  const int d4 = D / 4;
  const long long total = rows * d4;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / d4;
    const int c = (int)(i - r * d4);
    const long long b = r / rows_per_b;
    const float4 g = __ldg(reinterpret_cast<const float4*>(gate + b * gate_stride) + c);
    const float4 yy = reinterpret_cast<const float4*>(y)[i];
    float4 xx = reinterpret_cast<float4*>(x)[i];
    xx.x += g.x * yy.x;
    xx.y += g.y * yy.y;
    xx.z += g.z * yy.z;
    xx.w += g.w * yy.w;
    reinterpret_cast<float4*>(x)[i] = xx;
  }
}

// Four consecutive elements of y as fp32 (y fp32, fp16 or bf16).
template <int kY>
__device__ __forceinline__ float4 load_y4(const void* y, long long idx4) {
  if constexpr (kY == ANIMA_DTYPE_F32) {
    return reinterpret_cast<const float4*>(y)[idx4];
  } else {
    const uint2 u = reinterpret_cast<const uint2*>(y)[idx4];
    float2 a, b;
    if constexpr (kY == ANIMA_DTYPE_F16) {
      a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    } else {
      a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
      b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    }
    return make_float4(a.x, a.y, b.x, b.y);
  }
}

// Fused: x[r] += gate[b] * y[r] (fp32, in place), then h[r] = LayerNorm(x[r]) * (1 +
// scale[b]) + shift[b] as 16-bit -- the gated residual of one sub-block followed by the
// LayerNorm + modulation that opens the next.  One warp per row; the updated row stays in
// registers for the norm, so x is read once instead of twice.  y (the GEMM output being
// added) may be fp32 or the 16-bit operand type.
template <int kD, int kOut, int kY>
__global__ void __launch_bounds__(256)
    gate_residual_ln_modulate_kernel(float* __restrict__ x, const float* __restrict__ gate,
                                     long long gate_stride, const void* __restrict__ y,
                                     const float* __restrict__ scale,
                                     const float* __restrict__ shift, long long mod_stride,
                                     void* h, long long rows, int rows_per_b, float eps) {
  constexpr int kV = kD / 128;  // float4 per lane
  const int lane = threadIdx.x & 31;
  const long long w0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long r = w0; r < rows; r += nw) {
    const long long b = r / rows_per_b;
    float4* xr = reinterpret_cast<float4*>(x + r * kD);
    const float4* gr = reinterpret_cast<const float4*>(gate + b * gate_stride);
    float4 v[kV];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kV; ++k) {
      const float4 a = xr[lane + 32 * k], g = __ldg(gr + lane + 32 * k);
      const float4 c = load_y4<kY>(y, r * (kD / 4) + lane + 32 * k);
      v[k] = make_float4(a.x + g.x * c.x, a.y + g.y * c.y, a.z + g.z * c.z, a.w + g.w * c.w);
      xr[lane + 32 * k] = v[k];
      s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / (float)kD;
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < kV; ++k) {
      const float a = v[k].x - mean, bb = v[k].y - mean, c = v[k].z - mean, d = v[k].w - mean;
      q += (a * a + bb * bb) + (c * c + d * d);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float rstd = 1.0f / sqrtf(q / (float)kD + eps);
    const float4* sc = reinterpret_cast<const float4*>(scale + b * mod_stride);
    const float4* sh = reinterpret_cast<const float4*>(shift + b * mod_stride);
#pragma unroll
    for (int k = 0; k < kV; ++k) {
      const float4 a = __ldg(sc + lane + 32 * k), c = __ldg(sh + lane + 32 * k);
      store4<kOut>(h, r * (kD / 4) + lane + 32 * k,
                   (v[k].x - mean) * rstd * (1.f + a.x) + c.x, (v[k].y - mean) * rstd * (1.f + a.y) + c.y,
                   (v[k].z - mean) * rstd * (1.f + a.z) + c.z, (v[k].w - mean) * rstd * (1.f + a.w) + c.w);
    }
  }
}

// Exact GELU, y = x * (1 + erf(x / sqrt(2))) / 2 (torch.nn.GELU(), predict2.py:45), on
// 16-bit tensors in fp32 arithmetic; 8 elements (16 bytes) per thread and iteration.
template <int kDt>
__global__ void __launch_bounds__(256) gelu16_kernel(const uint4* __restrict__ x, uint4* y,
                                                     long long n8) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
    const uint4 u = x[i];
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f;
      if (kDt == ANIMA_DTYPE_BF16)
        f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
      else
        f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      const float a = 0.5f * f.x * (1.f + erff(f.x * 0.70710678118654752f));
      const float b = 0.5f * f.y * (1.f + erff(f.y * 0.70710678118654752f));
      w[j] = kDt == ANIMA_DTYPE_BF16 ? pack_bf16x2(a, b) : pack_f16x2(a, b);
    }
    y[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

static int grid_cap(long long work, int per_block, int sm_count, int waves) {
  long long g = (work + per_block - 1) / per_block;
  const long long cap = (long long)sm_count * waves;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

int ln_modulate_launch(const float* x, const float* scale, const float* shift, long long mod_stride,
                       void* y, int out_dtype, long long rows, int rows_per_b, int D, float eps,
                       int sm_count, cudaStream_t st) {
  if (D != 2048) return ANIMA_ERR_SHAPE;
  const int grid = grid_cap(rows, 8, sm_count, 16);
  if (out_dtype == ANIMA_DTYPE_F16)
    ln_modulate_kernel<2048, ANIMA_DTYPE_F16><<<grid, 256, 0, st>>>(x, scale, shift, mod_stride, y,
                                                                   rows, rows_per_b, eps);
  else if (out_dtype == ANIMA_DTYPE_BF16)
    ln_modulate_kernel<2048, ANIMA_DTYPE_BF16><<<grid, 256, 0, st>>>(x, scale, shift, mod_stride, y,
                                                                    rows, rows_per_b, eps);
  else
    return ANIMA_ERR_ARG;
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

int gate_residual_launch(float* x, const float* gate, long long gate_stride, const float* y,
                         long long rows, int rows_per_b, int D, int sm_count, cudaStream_t st) {
  if (D % 4) return ANIMA_ERR_SHAPE;
  const int grid = grid_cap(rows * (D / 4), 256, sm_count, 16);
  gate_residual_kernel<<<grid, 256, 0, st>>>(x, gate, gate_stride, y, rows, rows_per_b, D);
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

template <int kOut>
static int grlm_t(float* x, const float* gate, long long gate_stride, const void* y, int y_dtype,
                  const float* scale, const float* shift, long long mod_stride, void* h,
                  long long rows, int rows_per_b, float eps, int grid, cudaStream_t st) {
  switch (y_dtype) {
    case ANIMA_DTYPE_F32:
      gate_residual_ln_modulate_kernel<2048, kOut, ANIMA_DTYPE_F32><<<grid, 256, 0, st>>>(
          x, gate, gate_stride, y, scale, shift, mod_stride, h, rows, rows_per_b, eps);
      break;
    case ANIMA_DTYPE_F16:
      gate_residual_ln_modulate_kernel<2048, kOut, ANIMA_DTYPE_F16><<<grid, 256, 0, st>>>(
          x, gate, gate_stride, y, scale, shift, mod_stride, h, rows, rows_per_b, eps);
      break;
    case ANIMA_DTYPE_BF16:
      gate_residual_ln_modulate_kernel<2048, kOut, ANIMA_DTYPE_BF16><<<grid, 256, 0, st>>>(
          x, gate, gate_stride, y, scale, shift, mod_stride, h, rows, rows_per_b, eps);
      break;
    default:
      return ANIMA_ERR_ARG;
  }
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

int gate_residual_ln_modulate_launch(float* x, const float* gate, long long gate_stride,
                                     const void* y, int y_dtype, const float* scale,
                                     const float* shift, long long mod_stride, void* h,
                                     int out_dtype, long long rows, int rows_per_b, int D,
                                     float eps, int sm_count, cudaStream_t st) {
  if (D != 2048) return ANIMA_ERR_SHAPE;
  const int grid = grid_cap(rows, 8, sm_count, 16);
  if (out_dtype == ANIMA_DTYPE_F16)
    return grlm_t<ANIMA_DTYPE_F16>(x, gate, gate_stride, y, y_dtype, scale, shift, mod_stride, h,
                                   rows, rows_per_b, eps, grid, st);
  if (out_dtype == ANIMA_DTYPE_BF16)
    return grlm_t<ANIMA_DTYPE_BF16>(x, gate, gate_stride, y, y_dtype, scale, shift, mod_stride, h,
                                    rows, rows_per_b, eps, grid, st);
  return ANIMA_ERR_ARG;
}

int gelu16_launch(const void* x, void* y, int dtype, long long n, int sm_count, cudaStream_t st) {
  if (n % 8) return ANIMA_ERR_SHAPE;
  const long long n8 = n / 8;
  const int grid = grid_cap(n8, 256, sm_count, 16);
  if (dtype == ANIMA_DTYPE_F16)
    gelu16_kernel<ANIMA_DTYPE_F16><<<grid, 256, 0, st>>>(static_cast<const uint4*>(x),
                                                         static_cast<uint4*>(y), n8);
  else if (dtype == ANIMA_DTYPE_BF16)
    gelu16_kernel<ANIMA_DTYPE_BF16><<<grid, 256, 0, st>>>(static_cast<const uint4*>(x),
                                                          static_cast<uint4*>(y), n8);
  else
    return ANIMA_ERR_ARG;
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

}  // namespace anima
