// The C++ drop-in (include/molot_b200/attn.hpp) used the way the reference's
// own callers use attn.h (bench/bench.cc, forward.h), checked against the CPU
// oracle (oracle/attn_oracle.c, test infrastructure).  Exits non-zero on any
// failed CHECK, like the reference's bench.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <random>
#include <stdexcept>
#include <vector>

#include "../../oracle/attn_oracle.h"
#include "molot_b200/attn.hpp"

static int failures = 0;
#define CHECK(cond, ...)                   \
  do {                                     \
    if (!(cond)) {                         \
      ++failures;                          \
      std::printf("FAIL %d: ", __LINE__);  \
      std::printf(__VA_ARGS__);            \
      std::printf("\n");                   \
    }                                      \
  } while (0)

static double rel_err(const std::vector<float>& got, const std::vector<float>& want) {
  double num = 0, den = 0;
  for (size_t i = 0; i < got.size(); ++i) {
    num = std::fmax(num, std::fabs((double)got[i] - want[i]));
    den = std::fmax(den, std::fabs((double)want[i]));
  }
  return den > 0 ? num / den : num;
}

static std::mt19937 rng(1234);
static float frand() {
  static std::normal_distribution<float> d(0, 1);
  return d(rng);
}

int main() {
  // ---- attn_decode_gqa_cache on host buffers (attn.h:125), cfg1 shape
  {
    const int nq = 32, nkv = 8, d = 128, n = 4097;
    std::vector<float> Q(nq * d), K((size_t)n * nkv * d), V(K.size()), O(nq * d), R(nq * d);
    for (auto& x : Q) x = frand();
    for (auto& x : K) x = frand();
    for (auto& x : V) x = frand();
    const float scale = 1.0f / std::sqrt((float)d);
    molot_b200::attn_decode_gqa_cache(Q.data(), K.data(), V.data(), O.data(), nq, nkv, n, d, scale,
                                      n - 1, 0);
    oracle_attn_decode_gqa_cache(Q.data(), K.data(), V.data(), R.data(), nq, nkv, n, d, scale,
                                 n - 1, 0);
    const double e = rel_err(O, R);
    CHECK(e <= 1e-5, "attn_decode_gqa_cache rel err %g", e);
    std::printf("[ok] attn_decode_gqa_cache n=%d rel_err=%.2e\n", n, e);
  }
  // ---- attn_decode_head vs double softmax (bench.cc:186-218)
  {
    const int n = 512, d = 128;
    std::vector<float> Q(d), K(n * d), V(n * d), O(d);
    for (auto& x : Q) x = frand() * 0.2f;
    for (auto& x : K) x = frand() * 0.2f;
    for (auto& x : V) x = frand() * 0.2f;
    molot_b200::attn_decode_head(Q.data(), K.data(), V.data(), O.data(), n, d,
                                 1.0f / std::sqrt((float)d));
    std::vector<double> s(n);
    double m = -1e300, den = 0, err = 0;
    for (int t = 0; t < n; ++t) {
      double dot = 0;
      for (int j = 0; j < d; ++j) dot += (double)Q[j] * K[t * d + j];
      s[t] = dot / std::sqrt((double)d);
      m = std::fmax(m, s[t]);
    }
    for (auto& v : s) den += (v = std::exp(v - m));
    for (int j = 0; j < d; ++j) {
      double a = 0;
      for (int t = 0; t < n; ++t) a += s[t] / den * V[t * d + j];
      err = std::fmax(err, std::fabs(O[j] - a));
    }
    CHECK(err < 1e-3, "attn_decode_head err %g", err);
    std::printf("[ok] attn_decode_head maxerr=%.2e\n", err);
  }
  // ---- KVCache: forward.h:554-590 for a gemma-style layer, several tokens
  {
    const int nq = 8, nkv = 4, hd = 256, n0 = 300, cap = 320, window = 64;
    std::vector<float> kc((size_t)cap * nkv * hd, 0.f), vc(kc.size(), 0.f);
    for (size_t i = 0; i < (size_t)n0 * nkv * hd; ++i) {
      kc[i] = frand();
      vc[i] = frand();
    }
    std::vector<float> qn(hd), kn(hd), freq(hd / 2);
    for (auto& x : qn) x = 1.0f + 0.1f * frand();
    for (auto& x : kn) x = 1.0f + 0.1f * frand();
    molot_b200::rope_inv_freq(1e4f, hd, freq.data());
    float *dq, *dk, *dv, *dqr, *dout, *dqn, *dkn, *dfreq;
    cudaMalloc(&dq, nq * hd * 4);
    cudaMalloc(&dk, nkv * hd * 4);
    cudaMalloc(&dv, nkv * hd * 4);
    cudaMalloc(&dqr, nq * hd * 4);
    cudaMalloc(&dout, nq * hd * 4);
    cudaMalloc(&dqn, hd * 4);
    cudaMalloc(&dkn, hd * 4);
    cudaMalloc(&dfreq, hd / 2 * 4);
    cudaMemcpy(dqn, qn.data(), hd * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dkn, kn.data(), hd * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dfreq, freq.data(), hd / 2 * 4, cudaMemcpyHostToDevice);
    molot_b200::KVCache cache(2, nkv, hd, cap);
    cache.write(0, 0, n0, kc.data(), vc.data());
    cache.set_n(0, n0);
    int n_host = n0;
    double worst = 0;
    for (int step = 0; step < 5; ++step) {
      const int pos = n0 + step;
      std::vector<float> q(nq * hd), k(nkv * hd), v(nkv * hd), out(nq * hd), ref(nq * hd);
      for (auto& x : q) x = frand();
      for (auto& x : k) x = frand();
      for (auto& x : v) x = frand();
      cudaMemcpy(dq, q.data(), q.size() * 4, cudaMemcpyHostToDevice);
      cudaMemcpy(dk, k.data(), k.size() * 4, cudaMemcpyHostToDevice);
      cudaMemcpy(dv, v.data(), v.size() * 4, cudaMemcpyHostToDevice);
      if (step % 2 == 0) {  // two launches
        cache.append_rope(0, dq, dk, dv, dqr, dqn, dkn, true, 1e-6f, dfreq, pos, nq);
        cache.decode(0, dqr, dout, nq, 1.0f, pos, window);
      } else {  // one launch
        cache.step(0, dq, dk, dv, dqn, dkn, true, 1e-6f, dfreq, pos, dout, nq, 1.0f, window);
      }
      cache.sync();
      cudaMemcpy(out.data(), dout, out.size() * 4, cudaMemcpyDeviceToHost);
      int st = oracle_attn_layer_step(q.data(), k.data(), v.data(), qn.data(), kn.data(), 1, 1e-6f,
                                      freq.data(), pos, kc.data(), vc.data(), &n_host, cap,
                                      ref.data(), nq, nkv, hd, 1.0f, window);
      CHECK(st == 0, "oracle layer step status %d", st);
      worst = std::fmax(worst, rel_err(out, ref));
    }
    CHECK(cache.n(0) == n0 + 5, "cache length %d", cache.n(0));
    CHECK(worst <= 1e-5, "KVCache layer step rel err %g", worst);
    std::printf("[ok] KVCache append_rope+decode / step x5 rel_err=%.2e\n", worst);
    // a shared-KV layer (model.h:565-583): its own q, normalised and rotated
    // alone, attends to layer 0's cache
    {
      const int pos = n0 + 5;
      std::vector<float> q(nq * hd), out(nq * hd), ref(nq * hd), qr(nq * hd);
      for (auto& x : q) x = frand();
      cudaMemcpy(dq, q.data(), q.size() * 4, cudaMemcpyHostToDevice);
      molot_b200::norm_rope_q_dev(dq, dqr, dqn, 1e-6f, dfreq, pos, nq, hd);
      cache.decode(0, dqr, dout, nq, 1.0f, pos, window);
      cache.sync();
      cudaMemcpy(out.data(), dout, out.size() * 4, cudaMemcpyDeviceToHost);
      for (int h = 0; h < nq; ++h) {
        oracle_rmsnorm(q.data() + h * hd, qn.data(), qr.data() + h * hd, hd, 1e-6f);
        oracle_rope_apply(qr.data() + h * hd, hd, pos, freq.data());
      }
      oracle_attn_decode_gqa_cache(qr.data(), kc.data(), vc.data(), ref.data(), nq, nkv, n_host,
                                   hd, 1.0f, pos, window);
      const double e = rel_err(out, ref);
      CHECK(e <= 1e-5, "shared-KV reader rel err %g", e);
      std::printf("[ok] norm_rope_q_dev + shared-KV decode rel_err=%.2e\n", e);
    }
    // forward.h:580: a shared-KV layer reading an empty cache throws
    bool threw = false;
    try {
      cache.decode(1, dqr, dout, nq, 1.0f, 0, 0);
    } catch (const std::runtime_error&) {
      threw = true;
    }
    CHECK(threw, "empty shared KV did not throw");
    cudaFree(dq);
    cudaFree(dk);
    cudaFree(dv);
    cudaFree(dqr);
    cudaFree(dout);
    cudaFree(dqn);
    cudaFree(dkn);
    cudaFree(dfreq);
  }
  // ---- attn_prefill_gqa on host buffers (gemm.h:409-446)
  {
    const int nq = 16, nkv = 4, d = 128, M = 50, pos0 = 30, N = pos0 + M;
    std::vector<float> Q((size_t)M * nq * d), K((size_t)N * nkv * d), V(K.size()),
        O(Q.size()), R(Q.size());
    for (auto& x : Q) x = frand();
    for (auto& x : K) x = frand();
    for (auto& x : V) x = frand();
    molot_b200::attn_prefill_gqa(Q.data(), K.data(), V.data(), O.data(), nq, nkv, M, N, d, 0.0884f,
                                 pos0, 24);
    oracle_attn_prefill_gqa(Q.data(), K.data(), V.data(), R.data(), nq, nkv, M, N, d, 0.0884f,
                            pos0, 24);
    const double e = rel_err(O, R);
    CHECK(e <= 1e-5, "attn_prefill_gqa rel err %g", e);
    std::printf("[ok] attn_prefill_gqa M=%d rel_err=%.2e\n", M, e);
  }
  // ---- gemv_q4 on host buffers (gemm.h:223-254)
  {
    const int rows = 512, cols = 2048, ng = cols / 32;
    std::vector<float> W((size_t)rows * cols), x(cols), y(rows), r(rows), sc((size_t)rows * ng);
    std::vector<int8_t> z((size_t)rows * ng);
    std::vector<uint8_t> data((size_t)rows * cols / 2);
    std::vector<int16_t> ws((size_t)rows * ng);
    for (auto& v : W) v = 0.02f * frand();
    for (auto& v : x) v = frand();
    oracle_quantize_q4(W.data(), rows, cols, sc.data(), z.data(), data.data(), ws.data());
    molot_b200::gemv_q4(sc.data(), z.data(), data.data(), ws.data(), rows, cols, x.data(),
                        y.data());
    oracle_gemv_q4(sc.data(), z.data(), data.data(), rows, cols, x.data(), r.data());
    const double e = rel_err(y, r);
    CHECK(e <= 1e-6, "gemv_q4 rel err %g", e);
    std::printf("[ok] gemv_q4 %dx%d rel_err=%.2e\n", rows, cols, e);
  }
  // ---- continuous batching through Pager + PagedPlan (FP32 pools)
  {
    const int nq = 8, nkv = 2, d = 128, ps = 16, B = 2;
    molot_b200::Pager pager(1, nkv, d, ps, 16, 4, 8);
    const int s0 = pager.add(30), s1 = pager.add(9);
    const int seqs[B] = {s0, s1};
    float *kp, *vp;
    pager.layer_pools(0, &kp, &vp);
    std::vector<int> bt((size_t)B * pager.max_pages()), lens(B);
    pager.tables(seqs, B, bt.data(), lens.data());
    // host mirrors of each sequence's cache ([n][nkv*d]), prompt rows scattered into pages
    std::vector<std::vector<float>> hk(B), hv(B);
    for (int b = 0; b < B; ++b) {
      hk[b].resize((size_t)lens[b] * nkv * d);
      hv[b].resize(hk[b].size());
      for (auto& x : hk[b]) x = frand();
      for (auto& x : hv[b]) x = frand();
      for (int t = 0; t < lens[b]; ++t)
        for (int g = 0; g < nkv; ++g) {
          const size_t dst = (((size_t)bt[b * pager.max_pages() + t / ps] * nkv + g) * ps +
                              t % ps) * d;
          cudaMemcpy(kp + dst, hk[b].data() + ((size_t)t * nkv + g) * d, d * 4,
                     cudaMemcpyHostToDevice);
          cudaMemcpy(vp + dst, hv[b].data() + ((size_t)t * nkv + g) * d, d * 4,
                     cudaMemcpyHostToDevice);
        }
    }
    for (int b = 0; b < B; ++b) pager.grow(seqs[b]);
    pager.tables(seqs, B, bt.data(), lens.data());
    std::vector<float> q((size_t)B * nq * d), k((size_t)B * nkv * d), v(k.size()),
        o(q.size()), ref((size_t)nq * d);
    for (auto& x : q) x = frand();
    for (auto& x : k) x = frand();
    for (auto& x : v) x = frand();
    float *dq, *dk, *dv, *dqr, *dout;
    int* dbt;
    cudaMalloc(&dq, q.size() * 4);
    cudaMalloc(&dk, k.size() * 4);
    cudaMalloc(&dv, v.size() * 4);
    cudaMalloc(&dqr, q.size() * 4);
    cudaMalloc(&dout, q.size() * 4);
    cudaMalloc(&dbt, bt.size() * 4);
    cudaMemcpy(dq, q.data(), q.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dk, k.data(), k.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dv, v.data(), v.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dbt, bt.data(), bt.size() * 4, cudaMemcpyHostToDevice);
    molot_b200::PagedPlan plan;
    plan.build(B, nq, nkv, d, lens.data());
    const float scale = 1.f / std::sqrt((float)d);
    plan.append(dq, dk, dv, dqr, nullptr, nullptr, false, 1e-6f, nullptr, kp, vp, dbt,
                pager.max_pages(), ps);
    plan.decode(dqr, dout, kp, vp, dbt, pager.max_pages(), ps, scale);
    plan.sync();
    cudaMemcpy(o.data(), dout, o.size() * 4, cudaMemcpyDeviceToHost);
    double worst = 0;
    for (int b = 0; b < B; ++b) {
      hk[b].insert(hk[b].end(), k.begin() + (size_t)b * nkv * d, k.begin() + (size_t)(b + 1) * nkv * d);
      hv[b].insert(hv[b].end(), v.begin() + (size_t)b * nkv * d, v.begin() + (size_t)(b + 1) * nkv * d);
      oracle_attn_decode_gqa_cache(q.data() + (size_t)b * nq * d, hk[b].data(), hv[b].data(),
                                   ref.data(), nq, nkv, lens[b], d, scale, lens[b] - 1, 0);
      std::vector<float> got(o.begin() + (size_t)b * nq * d, o.begin() + (size_t)(b + 1) * nq * d);
      worst = std::max(worst, rel_err(got, ref));
    }
    CHECK(worst <= 1e-5, "paged decode rel err %g", worst);
    CHECK(pager.length(s0) == 31 && pager.length(s1) == 10, "pager lengths");
    cudaFree(dq);
    cudaFree(dk);
    cudaFree(dv);
    cudaFree(dqr);
    cudaFree(dout);
    cudaFree(dbt);
    std::printf("[ok] Pager + PagedPlan append/decode B=%d rel_err=%.2e\n", B, worst);
  }
  if (failures) {
    std::printf("CORRECTNESS: %d FAILURES\n", failures);
    return 1;
  }
  std::printf("all checks passed\n");
  return 0;
}
