// rt_ops.cu -- device kernels behind the rest of the reference runtime's host ABI.
//
// The reference's Python binding (anima_rt/scripts/anima_rt_ops.py:11-34) binds, besides
// the attention entries, six more symbols of libanima_rt (anima_rt/src/anima_rt.cpp:24-57,
// anima_rt/src/gemm_backend.cpp:140-171).  For that binding to load this library those
// symbols must exist, and they compute on the B200 like the rest:
//   elementwise_kernel  GELU (exact erf form, cpu/gelu_kernel.h:14-17) and SiLU
//                       (x / (1 + exp(-x)), cpu/silu_kernel.h), float4 per thread
//   layernorm_kernel    y = (x - mean) * rsqrt(var + eps), no affine (the binding's
//                       elementwise_affine=False case, anima_rt.cpp:37-43), warp per row
//   softmax_kernel      y = exp(x - max) / sum, per row of `dim` (cpu/softmax_kernel.h),
//                       warp per row
//   gemm_nt_kernel      C[M,N] = A[M,K] * B[N,K]^T in fp32, B fp32 or bf16 (widened
//                       exactly, as gemm_backend.cpp's fallbacks do); fp32 CUDA-core tiles
// None of these is on the attention path; they serve the host-pointer compatibility ABI,
// where the PCIe copies around each call dominate its cost.
#include "common.cuh"

namespace anima {

// ---------------------------------------------------------------- elementwise
enum { kActGelu = 0, kActSilu = 1 };

template <int kAct>
__device__ __forceinline__ float act(float x) {
  if (kAct == kActGelu) return x * 0.5f * (1.0f + erff(x * 0.70710678118654752f));
  return x / (1.0f + expf(-x));
}

template <int kAct>
__global__ void __launch_bounds__(256)
    elementwise_kernel(const float* __restrict__ x, float* __restrict__ y, long long n) {
  const long long n4 = n >> 2;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long t0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  for (long long i = t0; i < n4; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    reinterpret_cast<float4*>(y)[i] = make_float4(act<kAct>(v.x), act<kAct>(v.y),
                                                  act<kAct>(v.z), act<kAct>(v.w));
  }
  for (long long i = (n4 << 2) + t0; i < n; i += stride) y[i] = act<kAct>(x[i]);
}

// ---------------------------------------------------------------- row kernels
// One warp per row of d floats, rows strided over the grid's warps.
__global__ void __launch_bounds__(256)
    layernorm_kernel(const float* __restrict__ x, float* __restrict__ y, long long m, int d,
                     float eps) {
  const int lane = threadIdx.x & 31;
  const long long w0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long r = w0; r < m; r += nw) {
    const float* xr = x + r * d;
    float s = 0.f;
    for (int j = lane; j < d; j += 32) s += xr[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / (float)d;
    float q = 0.f;
    for (int j = lane; j < d; j += 32) {
      const float t = xr[j] - mean;
      q += t * t;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float rstd = 1.0f / sqrtf(q / (float)d + eps);
    float* yr = y + r * d;
    for (int j = lane; j < d; j += 32) yr[j] = (xr[j] - mean) * rstd;
  }
}

__global__ void __launch_bounds__(256)
    softmax_kernel(const float* __restrict__ x, float* __restrict__ y, long long outer, int dim) {
  const int lane = threadIdx.x & 31;
  const long long w0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long r = w0; r < outer; r += nw) {
    const float* xr = x + r * dim;
    float mx = -INFINITY;
    for (int j = lane; j < dim; j += 32) mx = fmaxf(mx, xr[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float s = 0.f;
    float* yr = y + r * dim;
    for (int j = lane; j < dim; j += 32) {
      const float e = expf(xr[j] - mx);
      yr[j] = e;
      s += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float inv = 1.0f / s;
    __syncwarp();
    for (int j = lane; j < dim; j += 32) yr[j] *= inv;
  }
}

// ---------------------------------------------------------------- fp32 GEMM, C = A B^T
// 128 x 128 output tile per 256-thread block, 8 x 8 outputs per thread, K in steps of 8.
// A [M, K] and B [N, K] are both K-contiguous; each step stages an 8-deep slice of both
// tiles transposed in shared memory ([k][row]), so a thread's 8 A and 8 B values of one k
// are two 32-byte runs.  Out-of-range rows and k read as zero.
constexpr int kGT = 128, kGK = 8;

__device__ __forceinline__ float widen(float v) { return v; }
__device__ __forceinline__ float widen(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }

template <typename TB>
__global__ void __launch_bounds__(256)
    gemm_nt_kernel(const float* __restrict__ A, const TB* __restrict__ Bm, float* __restrict__ C,
                   int M, int N, int K) {
  __shared__ float sa[kGK][kGT], sb[kGK][kGT];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * kGT, n0 = blockIdx.x * kGT;
  const int ty = tid >> 4, tx = tid & 15;  // 16 x 16 threads, 8 x 8 outputs each
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  // loader: thread -> (row lr, k-pair lk): 128 rows x 8 k = 1024 values = 4 per thread
  for (int k0 = 0; k0 < K; k0 += kGK) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int idx = tid + e * 256;  // 0..1023
      const int r = idx >> 3, kk = idx & 7;
      const int gk = k0 + kk;
      const int gm = m0 + r, gn = n0 + r;
      sa[kk][r] = (gm < M && gk < K) ? A[(long long)gm * K + gk] : 0.f;
      sb[kk][r] = (gn < N && gk < K) ? widen(Bm[(long long)gn * K + gk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kGK; ++kk) {
      float a[8], b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = sa[kk][ty * 8 + i];
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = sb[kk][tx * 8 + j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + ty * 8 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + tx * 8 + j;
      if (gn < N) C[(long long)gm * N + gn] = acc[i][j];
    }
  }
}

// ---------------------------------------------------------------- launchers
static int grid_for(long long work, int per_block, int sm_count) {
  const long long g = (work + per_block - 1) / per_block;
  const long long cap = (long long)sm_count * 8;
  return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

int act_launch(int which, const float* x, float* y, long long n, int sm_count, cudaStream_t st) {
  if (n <= 0) return ANIMA_OK;
  const int grid = grid_for((n + 3) / 4, 256, sm_count);
  if (which == kActGelu)
    elementwise_kernel<kActGelu><<<grid, 256, 0, st>>>(x, y, n);
  else
    elementwise_kernel<kActSilu><<<grid, 256, 0, st>>>(x, y, n);
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

int layernorm_launch(const float* x, float* y, long long m, int d, float eps, int sm_count,
                     cudaStream_t st) {
  if (m <= 0) return ANIMA_OK;
  layernorm_kernel<<<grid_for(m, 8, sm_count), 256, 0, st>>>(x, y, m, d, eps);
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

int softmax_launch(const float* x, float* y, long long outer, int dim, int sm_count,
                   cudaStream_t st) {
  if (outer <= 0) return ANIMA_OK;
  softmax_kernel<<<grid_for(outer, 8, sm_count), 256, 0, st>>>(x, y, outer, dim);
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

// b_bf16: B holds bf16 bit patterns (uint16), else fp32.
int gemm_nt_launch(const float* A, const void* Bm, bool b_bf16, float* C, int M, int N, int K,
                   cudaStream_t st) {
  if (M <= 0 || N <= 0) return ANIMA_OK;
  const dim3 grid((N + kGT - 1) / kGT, (M + kGT - 1) / kGT);
  if (grid.y > 65535u) return ANIMA_ERR_SHAPE;
  if (b_bf16)
    gemm_nt_kernel<uint16_t><<<grid, 256, 0, st>>>(A, static_cast<const uint16_t*>(Bm), C, M, N, K);
  else
    gemm_nt_kernel<float><<<grid, 256, 0, st>>>(A, static_cast<const float*>(Bm), C, M, N, K);
  return cudaGetLastError() == cudaSuccess ? ANIMA_OK : ANIMA_ERR_CUDA;
}

}  // namespace anima
