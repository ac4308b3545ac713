// TEST INFRASTRUCTURE ONLY — never linked into the product library.
//
// C ABI over the reference's own decode-attention headers, compiled unchanged
// from the reference source tree (include/molot/attn.h, norm.h, gemm.h,
// thread_pool.h) with the reference's Makefile flags.  Tests and the CPU
// baseline arm of bench.py load the resulting oracle/_ref/libmolot_ref.so to
// (a) pin the C restatement in attn_oracle.c and (b) time the reference's
// AVX-512 path on the host cores.
//
// Every wrapper forwards to exactly one reference function, except
// ref_attn_layer_step, which replays the attention segment of
// Runner::forward_token (include/molot/forward.h:554-590) on caller-owned
// host buffers: per-head QK RMSNorm, NEOX RoPE on q and k, V plain norm,
// append into a [cap][nkv*hd] cache, then attn_decode_gqa_cache.
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>

#include "molot/attn.h"
#include "molot/norm.h"
#include "molot/quant.h"
#include "molot/thread_pool.h"

namespace {

// One persistent pool per requested width (the reference's ThreadPool is
// not re-entrant, thread_pool.h:62-69, so callers serialise on the mutex).
std::mutex g_mu;
std::map<int, std::unique_ptr<molot::ThreadPool>> g_pools;

molot::ThreadPool& pool_for(int nthreads) {
  auto it = g_pools.find(nthreads);
  if (it == g_pools.end())
    it = g_pools.emplace(nthreads, std::make_unique<molot::ThreadPool>(nthreads)).first;
  return *it->second;
}

}  // namespace

extern "C" {

int ref_pool_size(int nthreads) {
  std::lock_guard<std::mutex> lk(g_mu);
  return pool_for(nthreads).size();
}

// attn.h:125-177
void ref_attn_decode_gqa_cache(const float* Q, const float* K, const float* V, float* O, int nq,
                               int nkv, int n, int qhd, float scale, int pos_cur, int window,
                               int nthreads) {
  std::lock_guard<std::mutex> lk(g_mu);
  molot::attn_decode_gqa_cache(Q, K, V, O, nq, nkv, n, qhd, scale, pos_cur, window,
                               pool_for(nthreads));
}

// attn.h:111-120 ([nkv][n][d] layout, full prefix)
void ref_attn_decode_gqa(const float* Q, const float* K, const float* V, float* O, int nq,
                         int nkv, int n, int d, float scale, int nthreads) {
  std::lock_guard<std::mutex> lk(g_mu);
  molot::attn_decode_gqa(Q, K, V, O, nq, nkv, n, d, scale, pool_for(nthreads));
}

// attn.h:178-187 ([nkv][n][d] layout, windowed)
void ref_attn_decode_gqa_win(const float* Q, const float* K, const float* V, float* O, int nq,
                             int nkv, int n, int d, float scale, int pos_cur, int window,
                             int nthreads) {
  std::lock_guard<std::mutex> lk(g_mu);
  molot::attn_decode_gqa_win(Q, K, V, O, nq, nkv, n, d, scale, pos_cur, window,
                             pool_for(nthreads));
}

// attn.h:57-101
void ref_attn_decode_head_win(const float* Q, const float* K, const float* V, float* out, int n,
                              int d, float scale, int pos_cur, int window) {
  molot::attn_decode_head_win(Q, K, V, out, n, d, scale, pos_cur, window);
}

// attn.h:104-107
void ref_attn_decode_head(const float* Q, const float* K, const float* V, float* out, int n,
                          int d, float scale) {
  molot::attn_decode_head(Q, K, V, out, n, d, scale);
}

// attn.h:19-28
void ref_rope_apply(float* x, int d, int pos, const float* inv_freq) {
  molot::rope_apply(x, d, pos, inv_freq);
}

// attn.h:31-33
void ref_rope_inv_freq(float base, int d, float* out) { molot::rope_inv_freq(base, d, out); }

// norm.h:9-28
void ref_rmsnorm(const float* x, const float* w, float* y, int n, float eps) {
  molot::rmsnorm(x, w, y, n, eps);
}

// norm.h:82-96
void ref_rmsnorm_plain(const float* x, float* y, int n, float eps) {
  molot::rmsnorm_plain(x, y, n, eps);
}

// norm.h:35-47 on 16 lanes
void ref_exp16(const float* in, float* out) {
  _mm512_storeu_ps(out, molot::exp_avx512_ps(_mm512_loadu_ps(in)));
}

// gemm.h:17-28
float ref_dot(const float* a, const float* b, int n) { return molot::dot_fp32_avx512(a, b, n); }

// Attention segment of forward.h:554-590 for one layer that owns its KV.
//   q [nq*hd] and k, v [nkv*hd] are the raw projections; they are normalised
//   and rotated in place.  kc, vc are [cap][nkv*hd]; *n is the slot count,
//   incremented on append.  q_norm / k_norm may be null (no QK-norm); freq
//   null means NoPE (forward.h:556,566).  Returns 0, or -1 when the cache is
//   full (forward.h:570 throws there).
int ref_attn_layer_step(float* q, float* k, float* v, const float* q_norm, const float* k_norm,
                        int v_norm, float eps, const float* freq, int pos, float* kc, float* vc,
                        int* n, int cap, float* out, int nq, int nkv, int hd, float scale,
                        int window, int nthreads) {
  std::lock_guard<std::mutex> lk(g_mu);
  // forward.h:138-140 rms_per_head; the reference always applies the norm
  // weights it loaded, a null pointer here stands for "layer has none".
  if (q_norm)
    for (int h = 0; h < nq; ++h) molot::rmsnorm(q + (size_t)h * hd, q_norm, q + (size_t)h * hd, hd, eps);
  if (freq)
    for (int h = 0; h < nq; ++h) molot::rope_apply(q + (size_t)h * hd, hd, pos, freq);
  if (k_norm)
    for (int h = 0; h < nkv; ++h) molot::rmsnorm(k + (size_t)h * hd, k_norm, k + (size_t)h * hd, hd, eps);
  if (v_norm) molot::rmsnorm_plain(v, v, nkv * hd, eps);
  if (freq)
    for (int h = 0; h < nkv; ++h) molot::rope_apply(k + (size_t)h * hd, hd, pos, freq);
  if (*n >= cap) return -1;
  std::memcpy(kc + (size_t)(*n) * nkv * hd, k, (size_t)nkv * hd * 4);
  std::memcpy(vc + (size_t)(*n) * nkv * hd, v, (size_t)nkv * hd * 4);
  (*n)++;
  molot::attn_decode_gqa_cache(q, kc, vc, out, nq, nkv, *n, hd, scale, pos, window,
                               pool_for(nthreads));
  return 0;
}

// gemm.h:409-446 (causal prefill attention over a filled cache)
void ref_attn_prefill_gqa(const float* Qm, const float* K, const float* V, float* Om, int nq,
                          int nkv, int M, int N, int d, float scale, int pos0, int window,
                          int nthreads) {
  std::lock_guard<std::mutex> lk(g_mu);
  molot::attn_prefill_gqa(Qm, K, V, Om, nq, nkv, M, N, d, scale, pos0, window,
                          pool_for(nthreads));
}

}  // extern "C"

extern "C" {

// quant.h:112-123 quantize_q4: rows x cols FP32 -> the Q4Matrix arrays.
void ref_quantize_q4(const float* W, int rows, int cols, float* scales, int8_t* zeros,
                     uint8_t* data, int16_t* wsums) {
  molot::Q4Matrix m = molot::quantize_q4(W, rows, cols);
  std::memcpy(scales, m.scales.data(), m.scales.size() * sizeof(float));
  std::memcpy(zeros, m.zeros.data(), m.zeros.size());
  std::memcpy(data, m.data.data(), m.data.size());
  std::memcpy(wsums, m.wsums.data(), m.wsums.size() * sizeof(int16_t));
}

// gemm.h:44-70 quantize_act_q8: per-32 absmax/127 scales (fp16-rounded), q.
void ref_quantize_act_q8(const float* x, int n, int8_t* q, float* scales) {
  molot::QAct8 a = molot::quantize_act_q8(x, n);
  std::memcpy(q, a.q.data(), a.q.size());
  std::memcpy(scales, a.scales.data(), a.scales.size() * sizeof(float));
}

// quant.h:33-50 quantize_q8_row applied to each 32-value block of x on its
// own (n a multiple of 32): the block rule of the Q8 KV row format.
void ref_quantize_q8_blocks(const float* x, long n, int8_t* q, float* scales) {
  for (long b = 0; b < n / 32; ++b) {
    int32_t bsum = 0;
    molot::quantize_q8_row(x + 32 * b, 32, 1, scales + b, q + 32 * b, &bsum);
  }
}

// gemm.h:223-254 gemv_q4 on a Q4Matrix given as its arrays.
void ref_gemv_q4(const float* scales, const int8_t* zeros, const uint8_t* data,
                 const int16_t* wsums, int rows, int cols, const float* x, float* y,
                 int nthreads) {
  std::lock_guard<std::mutex> lk(g_mu);
  molot::Q4Matrix m;
  m.rows = rows;
  m.cols = cols;
  m.ngroups = cols / molot::Q4Matrix::GS;
  m.scales.assign(scales, scales + (size_t)rows * m.ngroups);
  m.zeros.assign(zeros, zeros + (size_t)rows * m.ngroups);
  m.data.assign(data, data + (size_t)rows * cols / 2);
  m.wsums.assign(wsums, wsums + (size_t)rows * m.ngroups);
  molot::gemv_q4(m, x, y, pool_for(nthreads));
}

}  // extern "C"
