/*
 * anima_attn.h -- device-pointer C ABI of the B200 attention library.
 *
 * These entries serve PyTorch / CUDA callers that already hold the projections on the
 * GPU.  They replace, as one fused pipeline, the per-block attention sequence of the
 * reference DiT:
 *
 *   q/k RMSNorm (D = 128, eps 1e-6)   anima_rt/scripts/numpy_dit.py:285-286,
 *                                     src/predict2.py:185-186
 *   3D RoPE, self-attention only      anima_rt/scripts/numpy_dit.py:288-289,
 *                                     src/predict2.py:187-189, 31-38
 *   [B,S,H,D] -> [B,H,S,D] transpose  anima_rt/scripts/numpy_dit.py:291
 *   flash SDPA                        anima_rt/src/anima_rt.cpp:147-156
 *   transpose back to [B,S,H*D]       anima_rt/scripts/numpy_dit.py:294
 *
 * No torch types cross this boundary: plain device pointers, element strides, sizes
 * and a cudaStream_t passed as void*.  Every entry is asynchronous on that stream and
 * returns ANIMA_OK or a negative code; none aborts.  Device-side waits are bounded
 * (about one second); a kernel that gives up records ANIMA_ERR_TIMEOUT in the
 * library's per-device status word (anima_attn_status) and returns.
 */
#ifndef ANIMA_ATTN_H_
#define ANIMA_ATTN_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  ANIMA_OK = 0,
  ANIMA_ERR_ARG = -1,         /* null pointer, bad dtype, bad stride */
  ANIMA_ERR_SHAPE = -2,       /* unsupported or inconsistent shape */
  ANIMA_ERR_CUDA = -3,        /* a CUDA runtime/driver call failed */
  ANIMA_ERR_TIMEOUT = -4,     /* a device-side wait ran out (see anima_attn_status) */
  ANIMA_ERR_UNSUPPORTED = -5, /* device is not sm_100 */
  ANIMA_ERR_NOMEM = -6
};

enum { ANIMA_DTYPE_F32 = 0, ANIMA_DTYPE_BF16 = 1, ANIMA_DTYPE_F16 = 2 };

/* flags */
#define ANIMA_FLAG_QNORM 0x1u  /* RMSNorm q rows with q_norm_w            */
#define ANIMA_FLAG_KNORM 0x2u  /* RMSNorm k rows with k_norm_w            */
#define ANIMA_FLAG_ROPE 0x4u   /* rotate q and k with rope_freqs          */
#define ANIMA_FLAG_MASK 0x8u   /* key-padding mask from kv_valid_len[B]   */
#define ANIMA_FLAG_CAUSAL 0x10u /* top-left causal mask (col <= row)      */
#define ANIMA_FLAG_PAIR 0x20u  /* anima_attn_fwd: run on CTA pairs (2-SM MMA), one pair per
                                  512-row unit                             */
/* Schedule overrides of anima_attn_fwd(_noalloc) for calls that span more than one wave of
 * 256-row units (the library's own choice is described at `workspace` below).  A call of
 * one wave runs one CTA per unit, or, when most SMs would idle (e.g. B=2 with 2 heads at
 * 4096 tokens: 64 units), the cut schedule over all SMs; ANIMA_FLAG_UNIT / WHOLE keep it at
 * one CTA per unit:                                                                      */
#define ANIMA_FLAG_SPLIT 0x40u /* persistent grid with the last round cut into key-tile slices
                                  (needs the workspace; anima_attn_workspace_size takes the
                                  same flag)                                               */
#define ANIMA_FLAG_UNIT 0x80u  /* one CTA per 256-row unit                                */
#define ANIMA_FLAG_WHOLE 0x100u /* persistent grid, whole units only (no workspace)       */
/* Kernel choice of anima_attn_fwd(_noalloc): */
#define ANIMA_FLAG_KV64 0x200u /* 64-key tiles with P in tensor-memory columns of its own,
                                  so a query tile's next QK^T overlaps its softmax (the
                                  default kernel uses 128-key tiles with P over S)       */

/*
 * Prologue: per-head RMSNorm + RoPE + cast, one HBM pass.
 * Inputs q [B, S_q, H, D], k/v [B, S_kv, H, D] of dtype in_dtype, addressed by element
 * strides (stride_b, stride_s, stride_h; the D axis must be contiguous).
 * Outputs q_out [B*H, S_q, D], k_out/v_out [B*H, S_kv, D], contiguous, dtype op_dtype
 * (BF16 or F16) -- the layout anima_attn_fwd reads.
 * rope_freqs: fp32 [S_q, D/2, 2, 2] table (VideoRopePosition3DEmb layout); with
 * ANIMA_FLAG_ROPE it rotates q and k (requires S_q == S_kv).
 * q_norm_w / k_norm_w: fp32 [D]; NULL means weight 1.
 * S_q = 0 or S_kv = 0 skips that side (its input and output pointers may be NULL), for
 * callers that keep one side's operands across calls, such as the cross-attention K/V of
 * a text context that stays the same over a sampling run.
 */
typedef struct AnimaPrologueArgs {
  const void* q;
  const void* k;
  const void* v;
  int in_dtype;
  int64_t q_stride[3];
  int64_t k_stride[3];
  int64_t v_stride[3];
  int B, H, S_q, S_kv, D;
  const float* q_norm_w;
  const float* k_norm_w;
  float eps;
  const float* rope_freqs;
  unsigned flags;
  void* q_out;
  void* k_out;
  void* v_out;
  int op_dtype;
} AnimaPrologueArgs;

/*
 * Attention core (tcgen05 / TMEM flash forward, sm_100a).
 * q [B*H, S_q, D], k/v [B*H, S_kv, D] contiguous, dtype op_dtype (BF16 or F16), D = 128.
 * out: element strides out_stride = {b, h, s}, D contiguous, dtype out_dtype (F32, BF16, F16).
 *   [B*H, S_q, D] (the anima_rt layout):   {H*S_q*D, S_q*D, D}
 *   [B, S_q, H, D] (feeds the o-proj):     {S_q*H*D, D, H*D}
 * kv_valid_len: device int32 [B], used with ANIMA_FLAG_MASK (keys >= valid are masked;
 * a sample with 0 valid keys gets a zero output).
 * Schedule: a call of at most one wave of 256-row units, or a causal call, launches one
 * CTA per unit.  Otherwise the kernel runs persistently, one CTA per SM taking whole units
 * round-robin, which saves the per-CTA start-up and pipeline drain of every unit; where it
 * measured faster, the last partial round is also cut into equal slices of key tiles whose
 * fp32 partials are merged in-kernel, which needs the workspace.  Masked calls run whole
 * units persistently when their units have at most 16 key tiles (cross-attention into a
 * padded text context), else one CTA per unit; they are never cut.
 * workspace: optional device scratch of workspace_bytes, 256-byte aligned, ZERO-FILLED
 * before its first use; anima_attn_workspace_size() gives the size the cut needs (0 when
 * the call does not cut).  Without it the call runs whole units only.  The kernel leaves
 * the workspace's counters (its first 4 KiB) at zero, so a zero-filled workspace can be
 * reused; after an ANIMA_ERR_TIMEOUT, zero it again.  Calls that share a workspace must be
 * ordered on one stream.
 */
typedef struct AnimaAttnArgs {
  const void* q;
  const void* k;
  const void* v;
  int op_dtype;
  void* out;
  int out_dtype;
  int64_t out_stride[3];
  int B, H, S_q, S_kv, D;
  float scale;
  unsigned flags;
  const int* kv_valid_len;
  void* workspace;
  uint64_t workspace_bytes;
} AnimaAttnArgs;

/* Replaces the norm/RoPE/transpose steps listed above (numpy_dit.py:285-291). */
int anima_attn_prologue(const AnimaPrologueArgs* args, void* stream);

/* Replaces anima::cpu::flash_attention (anima_rt/include/cpu/flash_attention.h:55-208)
 * for device-resident operands. */
int anima_attn_fwd(const AnimaAttnArgs* args, void* stream);

/* anima_attn_fwd for callers that cannot allocate device memory.  No counterpart in the
 * reference.  Some hosts cannot let a library allocate: a host that owns the whole device
 * budget through its own allocator (a cudaMalloc behind its back breaks its accounting),
 * and C plugins that are handed only device pointers and sizes, with no allocator to
 * call; cudaMalloc and cudaFree also stall the device, which a caller in a tight loop
 * cannot afford.  This entry takes the same arguments as anima_attn_fwd, ignores
 * args->workspace, and allocates nothing: the scratch of the split schedule lives in a
 * static device array of about 40.6 MB (4 KiB of counters plus two partial slots for
 * each of up to 160 SMs), which every GPU that loads the library holds until the process
 * exits.  The first call on each device looks the array up with that device current;
 * make that first call before any stream capture.  Each call clears the array's counters
 * on `stream` before its kernel; all calls on a device share the array, so calls that
 * overlap on the GPU (different streams, no ordering) race and must not be issued.
 * A call whose schedule would need more scratch than the array holds returns
 * ANIMA_ERR_SHAPE (see anima_rt_last_error).  ANIMA_FLAG_PAIR calls run the CTA-pair
 * kernel, as in anima_attn_fwd; it uses no scratch.  No entry of this header allocates
 * device memory: the status word below is a static device variable too. */
int anima_attn_fwd_noalloc(const AnimaAttnArgs* args, void* stream);

/* Workspace bytes anima_attn_fwd can use for this shape on the current device
 * (0 when the call does not cut its last round; see anima_attn_schedule). */
uint64_t anima_attn_workspace_size(int B, int H, int S_q, int S_kv, unsigned flags);

/* Attention whose output is all-gathered over NVLink inside its epilogue (replaces the
 * NCCL all-gather of per-head outputs before the output projection of the head-parallel
 * DiT step; the reference's step runs on one device and has no counterpart).  Same
 * arguments as anima_attn_fwd except args->out, which is not used: every output block is
 * stored to each of peer_out[0 .. n_peers) (1 <= n_peers <= 8, 16-byte aligned, all with
 * args->out_stride and args->out_dtype).  A rank passes the bases of every rank's gather
 * buffer [B, S, H_total, 128], its own included, each already offset to the columns of its
 * heads; the other ranks' bases are peer mappings (anima_ipc_open).  The kernel only
 * stores; the caller orders the ranks afterwards (e.g. a one-element NCCL all-reduce on
 * the stream) before anyone reads the gathered buffer, and alternates between two buffers
 * so that no rank writes one that another is still reading.  ANIMA_FLAG_PAIR is rejected.
 * Asynchronous on `stream`. */
int anima_attn_fwd_gather(const AnimaAttnArgs* args, void* const* peer_out, int n_peers,
                          void* stream);

/* CUDA IPC for the gather buffers (no counterpart in the reference): anima_ipc_export writes
 * the ANIMA_IPC_HANDLE_BYTES-byte handle of the allocation holding `ptr` and ptr's offset in
 * it; another process of the node opens it with anima_ipc_open (peer access enabled) and
 * releases the mapping with anima_ipc_close(ptr, offset). */
#define ANIMA_IPC_HANDLE_BYTES 64
int anima_ipc_export(const void* ptr, void* handle, uint64_t* offset);
int anima_ipc_open(const void* handle, uint64_t offset, void** ptr);
int anima_ipc_close(void* ptr, uint64_t offset);

/* The schedule anima_attn_fwd(_noalloc) runs for this call when it is given the workspace
 * it asks for: ANIMA_SCHED_UNIT (one CTA per 256-row unit), ANIMA_SCHED_WHOLE (persistent
 * grid of whole units) or ANIMA_SCHED_CUT (persistent grid, last round cut into key-tile
 * slices; without the workspace such a call runs ANIMA_SCHED_WHOLE for units of at most
 * 4096 keys, else ANIMA_SCHED_UNIT).  ANIMA_FLAG_PAIR calls run the CTA-pair kernel and
 * report ANIMA_SCHED_UNIT.  sm_count <= 0 takes the current device's SM count; a positive
 * one needs no GPU.  Negative ANIMA_ERR_* on bad arguments.  Host arithmetic only; it has
 * no counterpart in the reference, whose CPU attention has a single schedule. */
enum { ANIMA_SCHED_UNIT = 0, ANIMA_SCHED_WHOLE = 1, ANIMA_SCHED_CUT = 2 };
int anima_attn_schedule(int B, int H, int S_q, int S_kv, unsigned flags, int sm_count);

/* Device status word of the current device: 0, or the first ANIMA_ERR_* a kernel
 * recorded.  Synchronises `stream`; clears the word when reset != 0. */
int anima_attn_status(void* stream, int reset);

/*
 * Q/K/V projection with the prologue in its epilogue (tcgen05 GEMM, sm_100a).  Replaces,
 * in one kernel, the projection GEMMs and the norm / RoPE / transpose passes that follow
 * them (anima_rt/scripts/numpy_dit.py:276-291; src/predict2.py:174-193):
 *   C = x W^T (x [B*L, K], W [N, K], both row-major 16-bit, fp32 accumulation); the N
 *   columns are n_tensors blocks of H heads x 128, tensors in the order q, k, v starting at
 *   first_tensor.  Per 128-column head block of q and k, RMSNorm over the fp32 accumulator
 *   (ANIMA_FLAG_QNORM / KNORM; weights [128] fp32, NULL = 1) and RoPE with rope_freqs
 *   [L, 64, 2, 2] (ANIMA_FLAG_ROPE); v is stored as is.  Outputs: head-major
 *   [B*H, L, 128] of dtype per tensor (the layout anima_attn_fwd reads), 16-byte aligned.
 * L must be a multiple of 32 and K of 8.  Asynchronous on `stream`.
 */
typedef struct AnimaQkvProjArgs {
  const void* x;
  const void* w;
  int dtype;              /* ANIMA_DTYPE_F16 or BF16: x, w and the outputs */
  int B, L, H, K;
  int n_tensors;          /* 1 .. 3 */
  int first_tensor;       /* 0 = q, 1 = k, 2 = v */
  const float* q_norm_w;
  const float* k_norm_w;
  float eps;
  const float* rope_freqs;
  unsigned flags;         /* ANIMA_FLAG_QNORM | ANIMA_FLAG_KNORM | ANIMA_FLAG_ROPE */
  void* q_out;
  void* k_out;
  void* v_out;
} AnimaQkvProjArgs;

int anima_qkv_projection(const AnimaQkvProjArgs* args, void* stream);

/* The two all-to-alls of a sequence-parallel attention, each folded into the kernel before
 * it (the reference's step runs on one device and has no counterpart).  A rank owns token
 * rows [r * rows, (r + 1) * rows) of the B x L grid for everything outside the attention and
 * heads [r * H, (r + 1) * H) inside it; the other ranks' buffers are peer mappings
 * (anima_ipc_open); the caller orders the ranks between the two kernels and after the
 * second (e.g. a one-element NCCL all-reduce on the stream).
 * anima_qkv_projection_scatter: args as for anima_qkv_projection with args->H the heads
 *   per rank and args->B, args->L the whole token grid; x holds `rows` token rows starting
 *   at global row `row0` (a multiple of 32), W all n_dest * H heads of each tensor.  The
 *   operand rows of head g go to rank g / H: dest[d * 3 + c] is rank d's head-major
 *   [B * H, L, 128] buffer of tensor c (q, k, v; only the computed tensors are read).
 * anima_attn_fwd_scatter_rows: args as for anima_attn_fwd (args->out and out_stride unused;
 *   S_q a multiple of 32); output row s of sample b is global row g = b * S_q + s and goes to
 *   dest[g / rows_per_dest] at local row g % rows_per_dest (a multiple of 32), as the
 *   columns of heads head0 .. head0 + H - 1 of a row-major buffer with dest_row_stride
 *   elements per row.
 * Asynchronous on `stream`. */
int anima_qkv_projection_scatter(const AnimaQkvProjArgs* args, int rows, int row0,
                                 void* const* dest, int n_dest, void* stream);
int anima_attn_fwd_scatter_rows(const AnimaAttnArgs* args, void* const* dest, int n_dest,
                                int rows_per_dest, int64_t dest_row_stride, int head0,
                                void* stream);

/* RoPE on device memory, for callers that apply it outside the fused prologue (replaces
 * predict2.apply_rotary_pos_emb, src/predict2.py:31-38, and the device side of
 * anima_rt_run_rope, anima_rt/include/cpu/rope_kernel.h:30-62, with the same arithmetic).
 * t and out are fp32 views [O, S, Hn, D] with element strides {o, s, h} and D contiguous
 * ([N, S, D]: O = N, Hn = 1; [B, S, H, D]: O = B, Hn = H); freqs [S, D/2, 2, 2] fp32
 * ([cos, -sin, sin, cos] per pair), pairs (p, D/2 + p).  out may equal t.  Asynchronous on
 * `stream`. */
int anima_attn_rope(const float* t, const int64_t t_stride[3], const float* freqs, float* out,
                    const int64_t out_stride[3], int O, int S, int Hn, int D, void* stream);

/* DiT block helpers around the attention (fused HBM passes; no single reference
 * counterpart, they replace chains of elementwise ops of src/predict2.py:469-583).
 * anima_dit_ln_modulate: y = LayerNorm(x) * (1 + scale[b]) + shift[b] over rows of D = 2048
 *   (eps, no affine; predict2.py:512-513), written as out_dtype (F16 or BF16) for the next
 *   GEMM; b = row / rows_per_b; scale/shift rows are mod_stride_b floats apart.
 * anima_dit_gate_residual: x += gate[b] * y, fp32, in place (predict2.py:536, 563, 582).
 * Pointers 16-byte aligned, strides multiples of 4.  Asynchronous on `stream`. */
int anima_dit_ln_modulate(const float* x, const float* scale, const float* shift,
                          int64_t mod_stride_b, void* y, int out_dtype, int64_t rows,
                          int rows_per_b, int D, float eps, void* stream);
int anima_dit_gate_residual(float* x, const float* gate, int64_t gate_stride_b, const float* y,
                            int64_t rows, int rows_per_b, int D, void* stream);
/* anima_gemm_gelu: y [M, N] = GELU(x [M, K] W[N, K]^T), the first layer of the DiT block's
 *   MLP with its exact GELU (x (1 + erf(x / sqrt 2)) / 2, src/predict2.py:45) applied to the
 *   fp32 accumulator in the epilogue of one tcgen05 GEMM; x, W and y row-major 16-bit of
 *   dtype (ANIMA_DTYPE_F16 or BF16), 16-byte aligned, N a multiple of 16 and K of 8.
 *   Asynchronous on `stream`. */
int anima_gemm_gelu(const void* x, const void* w, void* y, int M, int N, int K, int dtype,
                    void* stream);
/* anima_dit_gate_residual_ln_modulate: the two above back to back in one pass -- x += gate[b]*y
 *   in place, then h = LayerNorm(x) * (1 + scale[b]) + shift[b] as out_dtype (a sub-block's
 *   gated residual followed by the next sub-block's modulated LayerNorm, predict2.py:536-563);
 *   y of y_dtype (F32, F16 or BF16).
 * anima_dit_gelu: exact GELU (predict2.py:45, nn.GELU) on n 16-bit values (dtype F16 or BF16),
 *   n a multiple of 8, x and y 16-byte aligned (y may equal x). */
int anima_dit_gate_residual_ln_modulate(float* x, const float* gate, int64_t gate_stride_b,
                                        const void* y, int y_dtype, const float* scale,
                                        const float* shift, int64_t mod_stride_b, void* h,
                                        int out_dtype, int64_t rows, int rows_per_b, int D,
                                        float eps, void* stream);
int anima_dit_gelu(const void* x, void* y, int dtype, int64_t n, void* stream);

/* Self-test of the bounded-wait path (no reference counterpart): launches one block
 * whose mbarrier wait can never complete and gives up after timeout_us microseconds
 * (1..1000000), recording ANIMA_ERR_TIMEOUT in the status word exactly as a stalled
 * attention kernel would.  The kernel returns normally and the context stays usable;
 * read and clear the result with anima_attn_status. */
int anima_attn_selftest_timeout(unsigned timeout_us, void* stream);

/* Number of streaming multiprocessors and compute capability of the current device
 * (major*10 + minor); returns ANIMA_ERR_CUDA without a device. */
int anima_attn_device_info(int* sm_count, int* cc);

/* Library build identifier (kernel configuration), for logs. */
const char* anima_attn_version(void);

#ifdef __cplusplus
}
#endif

#endif /* ANIMA_ATTN_H_ */
