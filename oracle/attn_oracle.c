/* TEST INFRASTRUCTURE ONLY — see attn_oracle.h.
 *
 * Compiled with -fno-fast-math -ffp-contract=off: every fused multiply-add
 * below is an explicit fmaf() standing for an FMA the reference issues
 * (_mm512_fmadd_ps / _mm512_fnmadd_ps); every other operation is a single
 * IEEE float operation.
 */
#include "attn_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* Pairwise reduction of 16 lanes in _mm512_reduce_add_ps order: halves of
 * 8, then 4, then 2, then 1. */
static float reduce16(float v[16]) {
  for (int l = 0; l < 8; ++l) v[l] = v[l] + v[l + 8];
  for (int l = 0; l < 4; ++l) v[l] = v[l] + v[l + 4];
  v[0] = v[0] + v[2];
  v[1] = v[1] + v[3];
  return v[0] + v[1];
}

/* gemm.h:17-28 */
float oracle_dot(const float* a, const float* b, int n) {
  float acc[16] = {0};
  int i = 0;
  for (; i + 16 <= n; i += 16)
    for (int l = 0; l < 16; ++l) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
  float tail = 0.0f;
  for (; i < n; ++i) tail = fmaf(a[i], b[i], tail);
  return reduce16(acc) + tail;
}

/* norm.h:35-47: clamp to [-88, 88], n = rint(x*log2e), r = x - n*ln2 (one
 * fused op), Horner Taylor-5, scale by 2^n. */
float oracle_exp_taylor(float x) {
  x = fminf(fmaxf(x, -88.0f), 88.0f);
  float n = rintf(x * 1.4426950409f);
  float r = fmaf(-n, 0.6931471806f, x);
  float p = 1.0f / 120;
  p = fmaf(p, r, 1.0f / 24);
  p = fmaf(p, r, 1.0f / 6);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  return ldexpf(p, (int)n);
}

/* attn.h:19-28, NEOX half-split pairs (x[i], x[i+d/2]). */
void oracle_rope_apply(float* x, int d, int pos, const float* inv_freq) {
  int h = d / 2;
  for (int i = 0; i < h; ++i) {
    float ang = (float)pos * inv_freq[i];
    float c = cosf(ang), s = sinf(ang);
    float x0 = x[i], x1 = x[i + h];
    x[i] = x0 * c - x1 * s;
    x[i + h] = x0 * s + x1 * c;
  }
}

/* attn.h:31-33 */
void oracle_rope_inv_freq(float base, int d, float* out) {
  for (int i = 0; i < d / 2; ++i) out[i] = 1.0f / powf(base, (2.0f * (float)i) / (float)d);
}

static float sumsq16(const float* x, int n) {
  float acc[16] = {0};
  int i = 0;
  for (; i + 16 <= n; i += 16)
    for (int l = 0; l < 16; ++l) acc[l] = fmaf(x[i + l], x[i + l], acc[l]);
  float tail = 0.0f;
  for (; i < n; ++i) tail = fmaf(x[i], x[i], tail);
  return reduce16(acc) + tail;
}

/* norm.h:9-28 */
void oracle_rmsnorm(const float* x, const float* w, float* y, int n, float eps) {
  float mean = sumsq16(x, n) / (float)n;
  float inv = 1.0f / sqrtf(mean + eps);
  for (int i = 0; i < n; ++i) y[i] = (x[i] * inv) * w[i];
}

/* norm.h:82-96 */
void oracle_rmsnorm_plain(const float* x, float* y, int n, float eps) {
  float inv = 1.0f / sqrtf(sumsq16(x, n) / (float)n + eps);
  for (int i = 0; i < n; ++i) y[i] = x[i] * inv;
}

static int window_start(int pos_cur, int window) {
  return (window > 0 && pos_cur - window + 1 > 0) ? pos_cur - window + 1 : 0;
}

/* attn.h:57-101 / the per-head body of attn.h:130-176. */
void oracle_attn_decode_head_strided(const float* q, const float* K, const float* V, float* out,
                                     int n, int d, long row_stride, float scale, int pos_cur,
                                     int window, float* scores) {
  int t0 = window_start(pos_cur, window);
  float m = -1e30f;
  for (int t = t0; t < n; ++t) {
    float s = oracle_dot(q, K + (long)t * row_stride, d) * scale;
    scores[t] = s;
    if (s > m) m = s;
  }
  float den = 0.0f;
  int t = t0;
  for (; t + 16 <= n; t += 16) {
    float e[16];
    for (int l = 0; l < 16; ++l) {
      e[l] = oracle_exp_taylor(scores[t + l] - m);
      scores[t + l] = e[l];
    }
    den += reduce16(e);
  }
  for (; t < n; ++t) {
    scores[t] = expf(scores[t] - m);
    den += scores[t];
  }
  float inv = 1.0f / den;
  for (int j = 0; j < d; ++j) out[j] = 0.0f;
  for (int tt = t0; tt < n; ++tt) {
    float w = scores[tt] * inv;
    const float* vv = V + (long)tt * row_stride;
    for (int j = 0; j < d; ++j) out[j] = fmaf(vv[j], w, out[j]);
  }
}

void oracle_attn_decode_gqa_cache(const float* Q, const float* K, const float* V, float* O,
                                  int nq, int nkv, int n, int qhd, float scale, int pos_cur,
                                  int window) {
  int groups = nq / nkv;
  long S = (long)nkv * qhd;
  float* scores = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
  for (int h = 0; h < nq; ++h) {
    int kv = h / groups;
    oracle_attn_decode_head_strided(Q + (long)h * qhd, K + (long)kv * qhd, V + (long)kv * qhd,
                                    O + (long)h * qhd, n, qhd, S, scale, pos_cur, window, scores);
  }
  free(scores);
}

void oracle_attn_decode_gqa_win(const float* Q, const float* K, const float* V, float* O,
                                int nq, int nkv, int n, int d, float scale, int pos_cur,
                                int window) {
  int groups = nq / nkv;
  float* scores = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
  for (int h = 0; h < nq; ++h) {
    int kv = h / groups;
    oracle_attn_decode_head_strided(Q + (long)h * d, K + (long)kv * n * d, V + (long)kv * n * d,
                                    O + (long)h * d, n, d, d, scale, pos_cur, window, scores);
  }
  free(scores);
}

void oracle_attn_decode_gqa_cache_f64(const float* Q, const float* K, const float* V, double* O,
                                      int nq, int nkv, int n, int qhd, double scale,
                                      int pos_cur, int window) {
  int groups = nq / nkv;
  long S = (long)nkv * qhd;
  int t0 = window_start(pos_cur, window);
  double* s = (double*)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
  for (int h = 0; h < nq; ++h) {
    int kv = h / groups;
    const float* q = Q + (long)h * qhd;
    double m = -INFINITY;
    for (int t = t0; t < n; ++t) {
      const float* k = K + (long)t * S + (long)kv * qhd;
      double acc = 0.0;
      for (int j = 0; j < qhd; ++j) acc += (double)q[j] * (double)k[j];
      s[t] = acc * scale;
      if (s[t] > m) m = s[t];
    }
    double den = 0.0;
    for (int t = t0; t < n; ++t) {
      s[t] = exp(s[t] - m);
      den += s[t];
    }
    double* o = O + (long)h * qhd;
    for (int j = 0; j < qhd; ++j) o[j] = 0.0;
    for (int t = t0; t < n; ++t) {
      const float* v = V + (long)t * S + (long)kv * qhd;
      double w = s[t] / den;
      for (int j = 0; j < qhd; ++j) o[j] += w * (double)v[j];
    }
  }
  free(s);
}

int oracle_attn_layer_step(float* q, float* k, float* v, const float* q_norm,
                           const float* k_norm, int v_norm, float eps, const float* freq, int pos,
                           float* kc, float* vc, int* n, int cap, float* out, int nq, int nkv,
                           int hd, float scale, int window) {
  /* forward.h:554-568 */
  if (q_norm)
    for (int h = 0; h < nq; ++h) oracle_rmsnorm(q + (long)h * hd, q_norm, q + (long)h * hd, hd, eps);
  if (freq)
    for (int h = 0; h < nq; ++h) oracle_rope_apply(q + (long)h * hd, hd, pos, freq);
  if (k_norm)
    for (int h = 0; h < nkv; ++h) oracle_rmsnorm(k + (long)h * hd, k_norm, k + (long)h * hd, hd, eps);
  if (v_norm) oracle_rmsnorm_plain(v, v, nkv * hd, eps);
  if (freq)
    for (int h = 0; h < nkv; ++h) oracle_rope_apply(k + (long)h * hd, hd, pos, freq);
  /* forward.h:570-575 */
  if (*n >= cap) return -1;
  memcpy(kc + (long)(*n) * nkv * hd, k, sizeof(float) * (size_t)nkv * hd);
  memcpy(vc + (long)(*n) * nkv * hd, v, sizeof(float) * (size_t)nkv * hd);
  (*n)++;
  /* forward.h:589-590 */
  oracle_attn_decode_gqa_cache(q, kc, vc, out, nq, nkv, *n, hd, scale, pos, window);
  return 0;
}

void oracle_attn_decode_paged(const float* Q, const float* Kpool, const float* Vpool, float* O,
                              const int* block_table, int max_pages, const int* seq_lens,
                              const int* positions, int B, int nq, int nkv, int d, int page_size,
                              float scale, int window) {
  long row = (long)nkv * d;
  for (int b = 0; b < B; ++b) {
    int n = seq_lens[b];
    float* kc = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1) * row);
    float* vc = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1) * row);
    for (int t = 0; t < n; ++t) {
      long page = block_table[(long)b * max_pages + t / page_size];
      int off = t % page_size;
      for (int g = 0; g < nkv; ++g) {
        long src = ((page * nkv + g) * page_size + off) * (long)d;
        memcpy(kc + t * row + (long)g * d, Kpool + src, sizeof(float) * (size_t)d);
        memcpy(vc + t * row + (long)g * d, Vpool + src, sizeof(float) * (size_t)d);
      }
    }
    int pos = positions ? positions[b] : n - 1;
    oracle_attn_decode_gqa_cache(Q + (long)b * nq * d, kc, vc, O + (long)b * nq * d, nq, nkv, n,
                                 d, scale, pos, window);
    free(kc);
    free(vc);
  }
}

/* gemm.h:409-446 attn_prefill_gqa: causal prefill of M queries (positions
 * pos0+m) against a filled [N][nkv*d] cache.  Per (head, query): slots
 * [t0, nn) with nn = min(pos+1, N) and t0 = max(0, pos-window+1) capped at N;
 * scores = dot*scale; two-pass softmax with expf and a double denominator;
 * inv = (float)(1/den); o[j] accumulated over t in order with w = s*inv. */
void oracle_attn_prefill_gqa(const float* Qm, const float* K, const float* V, float* Om, int nq,
                             int nkv, int M, int N, int d, float scale, int pos0, int window) {
  int groups = nq / nkv;
  long S = (long)nkv * d;
  float* scores = (float*)malloc(sizeof(float) * (size_t)(N > 0 ? N : 1));
  for (int h = 0; h < nq; ++h) {
    int kv = h / groups;
    for (int m = 0; m < M; ++m) {
      int pos = pos0 + m;
      int t0 = 0;
      if (window > 0 && pos - window + 1 > t0) t0 = pos - window + 1;
      if (t0 > N) t0 = N;
      int nn = pos + 1 < N ? pos + 1 : N;
      const float* qh = Qm + ((long)m * nq + h) * d;
      float* oh = Om + ((long)m * nq + h) * d;
      float mx = -1e30f;
      for (int t = t0; t < nn; ++t) {
        float s = oracle_dot(qh, K + (long)t * S + (long)kv * d, d) * scale;
        scores[t] = s;
        if (s > mx) mx = s;
      }
      double den = 0;
      for (int t = t0; t < nn; ++t) {
        scores[t] = expf(scores[t] - mx);
        den += scores[t];
      }
      float inv = (float)(1.0 / den);
      for (int j = 0; j < d; ++j) oh[j] = 0;
      for (int t = t0; t < nn; ++t) {
        float w = scores[t] * inv;
        const float* vv = V + (long)t * S + (long)kv * d;
        for (int j = 0; j < d; ++j) oh[j] = fmaf(vv[j], w, oh[j]);
      }
    }
  }
  free(scores);
}

/* ---- Q4 GEMV (gemm.h:36-70, 174-254; quant.h:70-123) ------------------ */

/* quant.h:84-110 quantize_q4_row for every row: per 32-group min/max, scale
 * (max-min)/15 (1 when not positive), zero nearbyint(-min/s) in [0,15],
 * nibbles nearbyint(x/s)+zero in [0,15], element 2j in the low nibble of
 * byte j, wsums = sum(nibble - zero). */
void oracle_quantize_q4(const float* W, int rows, int cols, float* scales, int8_t* zeros,
                        uint8_t* data, int16_t* wsums) {
  int ng = cols / 32;
  for (int r = 0; r < rows; ++r)
    for (int g = 0; g < ng; ++g) {
      const float* grp = W + (long)r * cols + (long)g * 32;
      float mn = grp[0], mx = grp[0];
      for (int k = 0; k < 32; ++k) {
        if (grp[k] < mn) mn = grp[k];
        if (grp[k] > mx) mx = grp[k];
      }
      /* the reference's -ffast-math build multiplies by the reciprocal of
       * the constant: (mx - mn) / 15 becomes (mx - mn) * (1/15) */
      float s = (mx - mn) * (1.0f / 15.0f);
      if (!(s > 0)) s = 1.0f;
      int z = (int)nearbyintf(-mn / s);
      z = z < 0 ? 0 : (z > 15 ? 15 : z);
      scales[(long)r * ng + g] = s;
      zeros[(long)r * ng + g] = (int8_t)z;
      int wsum = 0;
      for (int k = 0; k < 32; k += 2) {
        int v0 = (int)nearbyintf(grp[k] / s) + z;
        int v1 = (int)nearbyintf(grp[k + 1] / s) + z;
        v0 = v0 < 0 ? 0 : (v0 > 15 ? 15 : v0);
        v1 = v1 < 0 ? 0 : (v1 > 15 ? 15 : v1);
        data[(long)r * cols / 2 + (long)g * 16 + k / 2] = (uint8_t)(v0 | (v1 << 4));
        wsum += (v0 - z) + (v1 - z);
      }
      wsums[(long)r * ng + g] = (int16_t)wsum;
    }
}

/* gemm.h:44-70 quantize_act_q8: per 32 values, xs = amax/127 (1 when not
 * positive) rounded to fp16 (nearest even, as F16C's _cvtss_sh); q =
 * round-half-away(x/xs) clamped to [-127, 127]. */
void oracle_quantize_act_q8(const float* x, int n, int8_t* q, float* scales) {
  for (int s = 0; s < n; s += 32) {
    int e = s + 32 < n ? s + 32 : n;
    float amax = 0;
    for (int i = s; i < e; ++i) {
      float v = fabsf(x[i]);
      if (v > amax) amax = v;
    }
    float xs = amax / 127.0f;
    if (!(xs > 0)) xs = 1.0f;
    xs = (float)(_Float16)xs;
    scales[s / 32] = xs;
    for (int i = s; i < e; ++i) {
      int v = (int)roundf(x[i] / xs);
      v = v > 127 ? 127 : (v < -127 ? -127 : v);
      q[i] = (int8_t)v;
    }
  }
}

/* The Q8 KV row format: quant.h:33-43 quantize_q8_row applied to each
 * 32-value block of x on its own (n a multiple of 32): s = amax/127 (1 when
 * not positive), q = nearbyint(x/s) clamped to [-127, 127].  The reference's
 * -ffast-math build evaluates s as amax * (1/127) and x/s as x * (127/amax);
 * those are the operations spelled out here (checked bit for bit against the
 * compiled reference). */
void oracle_quantize_q8_blocks(const float* x, long n, int8_t* q, float* scales) {
  for (long b = 0; b < n / 32; ++b) {
    const float* blk = x + 32 * b;
    float amax = 0;
    for (int i = 0; i < 32; ++i) {
      float v = fabsf(blk[i]);
      if (v > amax) amax = v;
    }
    const float s = amax * (1.0f / 127.0f);
    const float inv = 127.0f / amax;
    scales[b] = s > 0 ? s : 1.0f;
    for (int i = 0; i < 32; ++i) {
      int v = s > 0 ? (int)nearbyintf(blk[i] * inv) : 0;
      q[32 * b + i] = (int8_t)(v > 127 ? 127 : (v < -127 ? -127 : v));
    }
  }
}

/* gemm.h:174-254 gemv_q4: activations quantized once; per row and group
 * the exact integer sum G = sum((nibble - zero) * q); y = sum over groups,
 * in group order, of (float)G * scale_w * scale_x. */
void oracle_gemv_q4(const float* scales, const int8_t* zeros, const uint8_t* data, int rows,
                    int cols, const float* x, float* y) {
  int ng = cols / 32;
  int8_t* q = (int8_t*)malloc((size_t)cols);
  float* xs = (float*)malloc(sizeof(float) * (size_t)ng);
  oracle_quantize_act_q8(x, cols, q, xs);
  for (int r = 0; r < rows; ++r) {
    float acc = 0.0f;
    for (int g = 0; g < ng; ++g) {
      const uint8_t* pp = data + (long)r * cols / 2 + (long)g * 16;
      int z = zeros[(long)r * ng + g];
      int isum = 0;
      for (int k = 0; k < 32; ++k) {
        int w = ((k & 1) ? (pp[k / 2] >> 4) : (pp[k / 2] & 15)) - z;
        isum += w * q[g * 32 + k];
      }
      acc += (float)isum * scales[(long)r * ng + g] * xs[g];
    }
    y[r] = acc;
  }
  free(q);
  free(xs);
}
