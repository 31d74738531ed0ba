/*
 * anima_oracle.c -- CPU restatement of the reference's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the B200 kernels:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it.
 * Nothing in the product path links, calls or falls back to it.
 *
 * Each function restates one reference routine of riorgord/Anima-on-Android, in the
 * same arithmetic order so that results are bit-identical to the reference library
 * compiled by oracle/Makefile (the tests check exactly that):
 *
 *   oracle_flash_attention  anima_rt/include/cpu/flash_attention.h:55-208
 *                           (entered from anima_rt/src/anima_rt.cpp:147-156)
 *   oracle_rmsnorm          anima_rt/include/cpu/rmsnorm_kernel.h:11-33
 *                           (entered from anima_rt/src/anima_rt.cpp:45-50)
 *   oracle_rope             anima_rt/include/cpu/rope_kernel.h:30-62
 *                           (entered from anima_rt/src/anima_rt.cpp:160-164)
 *   oracle_rope_freqs_3d    src/position_embedding.py:80-98 and 100-163
 *                           (VideoRopePosition3DEmb.__init__ / generate_embeddings)
 *
 * One extension has no reference counterpart: oracle_flash_attention_varlen runs the
 * reference algorithm per sample with S_kv = valid_len[b], which is exactly a
 * key-padding mask (the reference has no mask on the DiT path; context is
 * zero-padded and attended).  valid_len == 0 yields a zero output row (the reference
 * would divide by zero computing its kv split count for S_kv == 0).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* Query/key split sizes of the reference tiling (flash_attention.h:62-67).  The
 * online-softmax rounding depends on them, so they are kept. */
static int q_split_for(int s_q) { return s_q >= 768 ? 256 : (s_q >= 192 ? 64 : 32); }
#define KV_SPLIT 512

/* One head: q [s_q, d], k/v [s_kv, d], o [s_q, d]; scratch sized q_split*kv_split. */
static void flash_one_head(const float* q, const float* k, const float* v, float* o,
                           int s_q, int s_kv, int d, float scale, int causal,
                           float* sc, float* mx, float* sm) {
  int qs = q_split_for(s_q);
  int ks = KV_SPLIT;
  if (qs > s_q) qs = s_q;
  if (ks > s_kv) ks = s_kv;
  for (int q0 = 0; q0 < s_q; q0 += qs) {
    const int qn = (q0 + qs <= s_q) ? qs : s_q - q0;
    for (int r = 0; r < qn; ++r) {
      mx[r] = -INFINITY;
      sm[r] = 0.0f;
      memset(o + (size_t)(q0 + r) * d, 0, sizeof(float) * (size_t)d);
    }
    const int keys = causal ? (q0 + qn < s_kv ? q0 + qn : s_kv) : s_kv;
    for (int k0 = 0; k0 < s_kv; k0 += ks) {
      const int kn = (k0 + ks <= s_kv) ? ks : s_kv - k0;
      if (k0 >= keys) break;
      int kv_eff = kn;
      if (causal) {
        if (keys - k0 < kn) kv_eff = keys - k0;
        if (kv_eff <= 0) break;
      }
      /* scores = (Q_blk . K_blk^T) * scale, padded columns = -inf */
      for (int i = 0; i < qn; ++i) {
        const float* qr = q + (size_t)(q0 + i) * d;
        float* srow = sc + (size_t)i * kn;
        for (int j = 0; j < kv_eff; ++j) {
          const float* kr = k + (size_t)(k0 + j) * d;
          float acc = 0.0f;
          for (int e = 0; e < d; ++e) acc += qr[e] * kr[e];
          srow[j] = acc * scale;
        }
        for (int j = kv_eff; j < kn; ++j) srow[j] = -INFINITY;
      }
      if (causal) {
        for (int i = 0; i < qn; ++i)
          for (int j = 0; j < kn; ++j)
            if (k0 + j > q0 + i) sc[(size_t)i * kn + j] = -INFINITY;
      }
      /* online softmax, one row at a time */
      for (int i = 0; i < qn; ++i) {
        float* srow = sc + (size_t)i * kn;
        float* orow = o + (size_t)(q0 + i) * d;
        float bmax = -INFINITY;
        for (int j = 0; j < kn; ++j)
          if (srow[j] > bmax) bmax = srow[j];
        if (bmax == -INFINITY) continue;
        const float m_new = mx[i] > bmax ? mx[i] : bmax;
        const float corr = (mx[i] == -INFINITY) ? 0.0f : expf(mx[i] - m_new);
        if (k0 > 0)
          for (int e = 0; e < d; ++e) orow[e] *= corr;
        sm[i] = sm[i] * corr;
        float rsum = 0.0f;
        for (int j = 0; j < kn; ++j) {
          const float p = expf(srow[j] - m_new);
          srow[j] = p;
          rsum += p;
        }
        sm[i] += rsum;
        for (int j = 0; j < kn; ++j) {
          const float p = srow[j];
          if (p == 0.0f) continue;
          const float* vr = v + (size_t)(k0 + j) * d;
          for (int e = 0; e < d; ++e) orow[e] += p * vr[e];
        }
        mx[i] = m_new;
      }
    }
    for (int i = 0; i < qn; ++i) {
      if (sm[i] > 0.0f) {
        const float inv = 1.0f / sm[i];
        float* orow = o + (size_t)(q0 + i) * d;
        for (int e = 0; e < d; ++e) orow[e] *= inv;
      }
    }
  }
}

/* Q [bh, s_q, d], K/V [bh, s_kv, d], O [bh, s_q, d]; returns 0 on success. */
int oracle_flash_attention(const float* Q, const float* K, const float* V, float* O,
                           int bh, int s_q, int s_kv, int d, float scale, int causal) {
  if (bh < 0 || s_q < 0 || s_kv <= 0 || d <= 0) return -1;
  int qs = q_split_for(s_q);
  if (qs > s_q) qs = s_q;
  const int ks = s_kv < KV_SPLIT ? s_kv : KV_SPLIT;
  float* sc = (float*)malloc(sizeof(float) * (size_t)(qs > 0 ? qs : 1) * (size_t)ks);
  float* mx = (float*)malloc(sizeof(float) * (size_t)(qs > 0 ? qs : 1));
  float* sm = (float*)malloc(sizeof(float) * (size_t)(qs > 0 ? qs : 1));
  if (!sc || !mx || !sm) { free(sc); free(mx); free(sm); return -2; }
  for (int h = 0; h < bh; ++h)
    flash_one_head(Q + (size_t)h * s_q * d, K + (size_t)h * s_kv * d,
                   V + (size_t)h * s_kv * d, O + (size_t)h * s_q * d, s_q, s_kv, d,
                   scale, causal, sc, mx, sm);
  free(sc); free(mx); free(sm);
  return 0;
}

/* Key-padding-masked attention: heads [b*n_heads + h], sample b attends to its first
 * valid[b] keys only (the reference algorithm run with S_kv = valid[b]).  Heads
 * h0..h1-1 of the flattened b*n_heads range are processed (for thread slicing). */
int oracle_flash_attention_varlen(const float* Q, const float* K, const float* V,
                                  float* O, int n_heads, int s_q, int s_kv, int d,
                                  float scale, const int* valid, int h0, int h1) {
  for (int bh = h0; bh < h1; ++bh) {
    const int b = bh / n_heads;
    const int nv = valid[b] < s_kv ? valid[b] : s_kv;
    float* o = O + (size_t)bh * s_q * d;
    if (nv <= 0) {
      memset(o, 0, sizeof(float) * (size_t)s_q * d);
      continue;
    }
    int rc = oracle_flash_attention(Q + (size_t)bh * s_q * d, K + (size_t)bh * s_kv * d,
                                    V + (size_t)bh * s_kv * d, o, 1, s_q, nv, d, scale, 0);
    if (rc) return rc;
  }
  return 0;
}

/* y[m, :] = x[m, :] * (1/sqrt(sum(x^2)/D + eps)) (* w) -- sequential fp32 sum. */
void oracle_rmsnorm(const float* X, const float* w, float* Y, int64_t M, int64_t D,
                    float eps) {
  for (int64_t r = 0; r < M; ++r) {
    const float* x = X + r * D;
    float* y = Y + r * D;
    float ss = 0.0f;
    for (int64_t j = 0; j < D; ++j) {
      const float t = x[j];
      ss += t * t;
    }
    const float ms = ss / (float)D;
    const float inv = 1.0f / sqrtf(ms + eps);
    for (int64_t j = 0; j < D; ++j) {
      float t = x[j] * inv;
      if (w) t *= w[j];
      y[j] = t;
    }
  }
}

/* Half-split RoPE: pair (p, D/2+p); freqs [S, D/2, 2, 2] = [cos, -sin, sin, cos]. */
void oracle_rope(const float* t, const float* freqs, float* out, int N, int S, int D) {
  const int half = D / 2;
  for (int n = 0; n < N; ++n)
    for (int s = 0; s < S; ++s) {
      const float* x = t + ((size_t)n * S + s) * D;
      float* y = out + ((size_t)n * S + s) * D;
      const float* f = freqs + (size_t)s * D * 2;
      for (int p = 0; p < half; ++p) {
        const float a = x[p], b = x[half + p];
        y[p] = f[4 * p + 0] * a + f[4 * p + 1] * b;
        y[half + p] = f[4 * p + 2] * a + f[4 * p + 3] * b;
      }
    }
}

/* 3D (t, h, w) RoPE table, out [(T*H*W), head_dim/2, 2, 2] fp32, token order
 * (t h w) with w fastest; pair blocks [t | h | w] of sizes dim_t/2, dim_h/2, dim_w/2.
 * dim_h = dim_w = head_dim/6*2, dim_t = head_dim - 2*dim_h; NTK factor
 * ratio^(dim/(dim-2)); theta_axis = theta * ntk_axis; freq_p = 1/theta_axis^(2p/dim). */
int oracle_rope_freqs_3d(float* out, int T, int H, int W, int head_dim, double h_ratio,
                         double w_ratio, double t_ratio, double theta) {
  const int dim_h = head_dim / 6 * 2, dim_w = dim_h, dim_t = head_dim - 2 * dim_h;
  const int ph = dim_h / 2, pw = dim_w / 2, pt = dim_t / 2, half = head_dim / 2;
  if (pt + ph + pw != half) return -1;
  const double h_ntk = pow(h_ratio, (double)dim_h / (double)(dim_h - 2));
  const double w_ntk = pow(w_ratio, (double)dim_w / (double)(dim_w - 2));
  const double t_ntk = pow(t_ratio, (double)dim_t / (double)(dim_t - 2));
  const float h_theta = (float)(theta * h_ntk), w_theta = (float)(theta * w_ntk),
              t_theta = (float)(theta * t_ntk);
  float* fh = (float*)malloc(sizeof(float) * (size_t)(ph + pw + pt));
  if (!fh) return -2;
  float* fw = fh + ph;
  float* ft = fw + pw;
  for (int i = 0; i < ph; ++i) fh[i] = 1.0f / powf(h_theta, (float)(2 * i) / (float)dim_h);
  for (int i = 0; i < pw; ++i) fw[i] = 1.0f / powf(w_theta, (float)(2 * i) / (float)dim_w);
  for (int i = 0; i < pt; ++i) ft[i] = 1.0f / powf(t_theta, (float)(2 * i) / (float)dim_t);
  for (int t = 0; t < T; ++t)
    for (int h = 0; h < H; ++h)
      for (int w = 0; w < W; ++w) {
        float* row = out + ((size_t)(t * H + h) * W + w) * half * 4;
        for (int p = 0; p < half; ++p) {
          float ang;
          if (p < pt) ang = (float)t * ft[p];
          else if (p < pt + ph) ang = (float)h * fh[p - pt];
          else ang = (float)w * fw[p - pt - ph];
          const float c = cosf(ang), s = sinf(ang);
          row[4 * p + 0] = c;
          row[4 * p + 1] = -s;
          row[4 * p + 2] = s;
          row[4 * p + 3] = c;
        }
      }
  free(fh);
  return 0;
}
