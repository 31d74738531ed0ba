/*
 * anima_rt.h -- drop-in replacement for the reference runtime's attention entry points.
 *
 * libanima_attn.so exports these symbols with the exact signatures, argument meaning,
 * ownership and bool-return convention of riorgord/Anima-on-Android's
 * anima_rt/src/anima_rt.cpp, so the reference's ctypes bindings
 * (anima_rt/scripts/anima_rt_ops.py:11-34, scripts/phone_pipeline_nd.py:46-68) load it
 * unchanged.  All pointers are caller-owned, contiguous fp32 HOST memory; each call
 * copies its inputs to the current CUDA device, runs the B200 kernels, copies the
 * result back and returns.  A call returns false (never aborts) on any CUDA error or
 * unsupported shape; anima_rt_last_error() then describes why.
 *
 * Calls are serialised inside the library (one device workspace); concurrent callers
 * are safe but do not overlap on the GPU.
 */
#ifndef ANIMA_RT_H_
#define ANIMA_RT_H_

#include <stdbool.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Replaces anima_rt_init (anima_rt/src/anima_rt.cpp:13-20).  Idempotent.  Selects the
 * current CUDA device and creates the library's stream and workspace.  false when no
 * CUDA device is usable. */
bool anima_rt_init(void);

/* Replaces anima_rt_destroy (anima_rt/src/anima_rt.cpp:166-171).  Frees the workspace;
 * later calls that need init (rmsnorm, math sdpa) return false until anima_rt_init. */
void anima_rt_destroy(void);

/* Replaces anima_rt_run_sdpa_flash (anima_rt/src/anima_rt.cpp:147-156,
 * anima_rt/include/cpu/flash_attention.h:55-208).
 * Q [BH, S_q, D], K/V [BH, S_kv, D], output [BH, S_q, D], fp32.  Computes
 * softmax(Q K^T * scale) V per head, top-left causal mask when is_causal.  Operands
 * are rounded to bf16 for the tensor cores, accumulation and softmax are fp32.
 * Supports D == 128 (the Anima head size); other D return false.  Like the reference
 * it does not require anima_rt_init. */
bool anima_rt_run_sdpa_flash(const float* Q, const float* K, const float* V, float* output,
                             int BH, int S_q, int S_kv, int D, float scale, bool is_causal);

/* Replaces anima_rt_run_sdpa (anima_rt/src/anima_rt.cpp:78-140).  The reference's math
 * path scales both Q and K by `scale` (effective scale^2); this library computes the
 * correct SDPA with `scale` applied once, identical to anima_rt_run_sdpa_flash.
 * Returns false before anima_rt_init, as the reference does. */
bool anima_rt_run_sdpa(const float* Q, const float* K, const float* V, float* output,
                       int BH, int S_q, int S_kv, int D, float scale, bool is_causal);

/* Replaces anima_rt_run_rmsnorm (anima_rt/src/anima_rt.cpp:45-50,
 * anima_rt/include/cpu/rmsnorm_kernel.h:11-33): y = x / sqrt(mean(x^2) + eps) * w
 * per row of x [m, d]; w may be NULL.  Returns false before anima_rt_init. */
bool anima_rt_run_rmsnorm(const float* x, const float* w, float* out, int m, int d,
                          float eps);

/* Replaces anima_rt_run_rope (anima_rt/src/anima_rt.cpp:160-164,
 * anima_rt/include/cpu/rope_kernel.h:30-62): t [N, S, D], freqs [S, D/2, 2, 2]
 * ([cos, -sin, sin, cos] per pair), pairs (p, D/2 + p).  Bit-identical to the
 * reference (no fused multiply-add). */
bool anima_rt_run_rope(const float* t, const float* freqs, float* out, int N, int S, int D);

/* The rest of the symbols the reference's binding sets argtypes on
 * (anima_rt/scripts/anima_rt_ops.py:12-27), so that binding loads this library.  They
 * run on the device like the entries above (copy in, one kernel, copy back) and keep the
 * reference's semantics; none of them is on the attention path.
 *
 * Replace anima_rt_run_gelu / anima_rt_run_silu (anima_rt/src/anima_rt.cpp:24-32;
 * cpu/gelu_kernel.h:14-17, cpu/silu_kernel.h): out[i] = x*0.5*(1+erf(x/sqrt(2))) and
 * x/(1+exp(-x)) over n fp32 values.  false before anima_rt_init, as in the reference. */
bool anima_rt_run_gelu(const float* x, float* out, int n);
bool anima_rt_run_silu(const float* x, float* out, int n);

/* Replaces anima_rt_run_layernorm (anima_rt/src/anima_rt.cpp:36-43,
 * cpu/layernorm_kernel.h): y = (x - mean) / sqrt(var + eps) per row of x [m, d], no
 * affine (the reference passes null gamma/beta).  false before anima_rt_init. */
bool anima_rt_run_layernorm(const float* x, float* out, int m, int d, float eps);

/* Replaces anima_rt_run_softmax (anima_rt/src/anima_rt.cpp:52-57, cpu/softmax_kernel.h):
 * y = exp(x - max) / sum(exp(x - max)) per row of x [outer, dim].  false before
 * anima_rt_init. */
bool anima_rt_run_softmax(const float* x, float* out, int outer, int dim);

/* Replace anima_rt_run_gemm_fp32 / anima_rt_run_gemm_bf16
 * (anima_rt/src/gemm_backend.cpp:140-171): C[M,N] = A[M,K] * B[N,K]^T with fp32 A and C;
 * B fp32, or bf16 bit patterns (uint16) widened exactly to fp32.  fp32 arithmetic; the
 * summation order differs from the reference's sequential loop.  Like the reference they
 * do not require anima_rt_init. */
bool anima_rt_run_gemm_fp32(const float* A, const float* B, float* C, int M, int N, int K);
bool anima_rt_run_gemm_bf16(const float* A, const uint16_t* W, float* C, int M, int N, int K);

/* Extension (no single reference counterpart): the whole per-block attention sequence
 * of NumpyAttention.forward (anima_rt/scripts/numpy_dit.py:285-294) in one call --
 * q/k RMSNorm (q_w / k_w may be NULL: weight 1; flags select which are applied),
 * RoPE on q and k with freqs [S_q, D/2, 2, 2] (self-attention, S_q == S_kv), flash
 * SDPA and the transposes.  q [B, S_q, H, D], k/v [B, S_kv, H, D], out [B, S_q, H, D],
 * all fp32 host memory.  kv_valid (host int32 [B], may be NULL) masks keys >= kv_valid[b].
 * flags: 1 = q norm, 2 = k norm, 4 = RoPE, 16 = causal (bit values of ANIMA_FLAG_*).
 * Host buffers in page-locked memory are copied by the copy engine directly (full PCIe
 * speed).  Ordinary pageable arrays above 1 MiB are copied through the library's own
 * page-locked ring by up to 16 host threads (the process's CPUs, divided by torchrun's
 * LOCAL_WORLD_SIZE when set; ANIMA_RT_COPY_THREADS overrides; ANIMA_RT_STAGE=0
 * leaves them to the CUDA driver's single-threaded copies); the same holds for the
 * other host entries above. */
bool anima_rt_run_attention(const float* q, const float* k, const float* v, const float* q_w,
                            const float* k_w, const float* freqs, const int* kv_valid,
                            float* out, int B, int S_q, int S_kv, int H, int D, float eps,
                            float scale, unsigned flags);

/* Extension: text of the last failure on this thread ("" if none). */
const char* anima_rt_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* ANIMA_RT_H_ */
