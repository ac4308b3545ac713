/* TEST INFRASTRUCTURE ONLY — the CPU checker for the molot_b200 kernels.
 *
 * A plain-C restatement of the reference decode-attention path
 * (include/molot/attn.h, norm.h, gemm.h and the attention segment of
 * forward.h).  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may load it, and only to check or time; the product
 * library never links it.
 *
 * Arithmetic follows the reference operation by operation:
 *   - dot products keep 16 fused-multiply-add accumulators, lane l owning
 *     elements j with j % 16 == l, reduced by the same pairwise tree as
 *     _mm512_reduce_add_ps (l+8, then l+4, then l+2, then l+1), plus the
 *     scalar tail (gemm.h:17-28);
 *   - exp is the reference's clamped Taylor-5 range reduction
 *     (norm.h:35-47), with libm expf for the <16 tail (attn.h:158-161);
 *   - softmax is the reference's three passes over [t0, n): scores and max,
 *     exp and a sequential denominator, then weighted V accumulation with
 *     the normalised weight (attn.h:137-175).
 * The f64 entry points evaluate the same maths in double precision and are
 * the accuracy yardstick.
 */
#ifndef MOLOT_ATTN_ORACLE_H
#define MOLOT_ATTN_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* gemm.h:17-28 */
float oracle_dot(const float* a, const float* b, int n);
/* norm.h:35-47, one lane */
float oracle_exp_taylor(float x);
/* attn.h:19-28 */
void oracle_rope_apply(float* x, int d, int pos, const float* inv_freq);
/* attn.h:31-33 */
void oracle_rope_inv_freq(float base, int d, float* out);
/* norm.h:9-28 */
void oracle_rmsnorm(const float* x, const float* w, float* y, int n, float eps);
/* norm.h:82-96 */
void oracle_rmsnorm_plain(const float* x, float* y, int n, float eps);

/* attn.h:57-101 for one query head over rows t*row_stride of K and V. */
void oracle_attn_decode_head_strided(const float* q, const float* K, const float* V, float* out,
                                     int n, int d, long row_stride, float scale, int pos_cur,
                                     int window, float* scratch /* >= n floats */);

/* attn.h:125-177: Q [nq][qhd], K/V [n][nkv*qhd], O [nq][qhd]. */
void oracle_attn_decode_gqa_cache(const float* Q, const float* K, const float* V, float* O,
                                  int nq, int nkv, int n, int qhd, float scale, int pos_cur,
                                  int window);

/* attn.h:111-120 / 178-187: K/V [nkv][n][d]. */
void oracle_attn_decode_gqa_win(const float* Q, const float* K, const float* V, float* O,
                                int nq, int nkv, int n, int d, float scale, int pos_cur,
                                int window);

/* Double-precision attention over the [n][nkv*qhd] layout (same masking). */
void oracle_attn_decode_gqa_cache_f64(const float* Q, const float* K, const float* V, double* O,
                                      int nq, int nkv, int n, int qhd, double scale,
                                      int pos_cur, int window);

/* Attention segment of forward.h:554-590 for one KV-owning layer (see
 * oracle/ref_shim.cc for the argument contract).  Returns 0 or -1 (full). */
int oracle_attn_layer_step(float* q, float* k, float* v, const float* q_norm,
                           const float* k_norm, int v_norm, float eps, const float* freq, int pos,
                           float* kc, float* vc, int* n, int cap, float* out, int nq, int nkv,
                           int hd, float scale, int window);

/* Paged batch: sequence b has seq_lens[b] slots in pages block_table[b][*]
 * of a pool laid out [page][nkv][page_size][d] (K and V pools separately).
 * Each sequence is gathered into the [n][nkv*d] layout and passed to
 * oracle_attn_decode_gqa_cache with pos_cur = positions[b] (or n-1 when
 * positions is null).  Q, O are [B][nq][d]. */
void oracle_attn_decode_paged(const float* Q, const float* Kpool, const float* Vpool, float* O,
                              const int* block_table, int max_pages, const int* seq_lens,
                              const int* positions, int B, int nq, int nkv, int d, int page_size,
                              float scale, int window);

/* Causal prefill attention, gemm.h:409-446: Qm, Om [M][nq][d], K/V
 * [N][nkv*d]; query m sits at position pos0+m. */
void oracle_attn_prefill_gqa(const float* Qm, const float* K, const float* V, float* Om, int nq,
                             int nkv, int M, int N, int d, float scale, int pos0, int window);

/* Q4 weights (quant.h:70-123) and the Q4 GEMV of gemm.h:174-254. */
void oracle_quantize_q4(const float* W, int rows, int cols, float* scales, int8_t* zeros,
                        uint8_t* data, int16_t* wsums);
void oracle_quantize_act_q8(const float* x, int n, int8_t* q, float* scales);
/* The Q8 KV row format's block rule (quant.h:33-43 per 32 values). */
void oracle_quantize_q8_blocks(const float* x, long n, int8_t* q, float* scales);
void oracle_gemv_q4(const float* scales, const int8_t* zeros, const uint8_t* data, int rows,
                    int cols, const float* x, float* y);

#ifdef __cplusplus
}
#endif
#endif
