// C++ drop-in for the reference's decode-attention header
// (include/molot/attn.h) and its KV cache (Runner::KVC, forward.h:48-51),
// backed by the molot_b200 C ABI (include/molot_b200.h).
//
// Same function names and argument meaning as the reference, in namespace
// molot_b200.  The reference's trailing ThreadPool& becomes the CUDA device
// current on the calling thread; results are ready on return, as in the
// reference.  Errors throw std::runtime_error, matching the places where the
// reference's forward pass throws (forward.h:570, 580); bad arguments, which
// the reference does not check, throw too instead of reading out of bounds.
#pragma once

#include <stdexcept>
#include <string>

#include "molot_b200.h"

namespace molot_b200 {

inline void check(int status) {
  if (status != MOLOT_OK)
    throw std::runtime_error(std::string("molot_b200: ") + molot_status_string(status) + ": " +
                             molot_last_error());
}

// attn.h:19-28
inline void rope_apply(float* x, int d, int pos, const float* inv_freq) {
  check(molot_rope_apply(x, d, pos, inv_freq));
}

// attn.h:31-33
inline void rope_inv_freq(float base, int d, float* out) {
  check(molot_rope_inv_freq(base, d, out));
}

// attn.h:57-101
inline void attn_decode_head_win(const float* Q, const float* K, const float* V, float* out,
                                 int n, int d, float scale, int pos_cur, int window) {
  check(molot_attn_decode_head_win(Q, K, V, out, n, d, scale, pos_cur, window));
}

// attn.h:104-107
inline void attn_decode_head(const float* Q, const float* K, const float* V, float* out, int n,
                             int d, float scale) {
  check(molot_attn_decode_head(Q, K, V, out, n, d, scale));
}

// attn.h:111-120
inline void attn_decode_gqa(const float* Q, const float* K, const float* V, float* O, int nq,
                            int nkv, int n, int d, float scale) {
  check(molot_attn_decode_gqa(Q, K, V, O, nq, nkv, n, d, scale));
}

// attn.h:125-177
inline void attn_decode_gqa_cache(const float* Q, const float* K, const float* V, float* O,
                                  int nq, int nkv, int n, int qhd, float scale, int pos_cur,
                                  int window) {
  check(molot_attn_decode_gqa_cache(Q, K, V, O, nq, nkv, n, qhd, scale, pos_cur, window));
}

// attn.h:178-187
inline void attn_decode_gqa_win(const float* Q, const float* K, const float* V, float* O, int nq,
                                int nkv, int n, int d, float scale, int pos_cur, int window) {
  check(molot_attn_decode_gqa_win(Q, K, V, O, nq, nkv, n, d, scale, pos_cur, window));
}

// gemm.h:409-446 (causal prefill attention), host buffers, ready on return
inline void attn_prefill_gqa(const float* Qm, const float* K, const float* V, float* Om, int nq,
                             int nkv, int M, int N, int d, float scale, int pos0, int window) {
  check(molot_attn_prefill_gqa(Qm, K, V, Om, nq, nkv, M, N, d, scale, pos0, window));
}

// gemm.h:223-254 (Q4 GEMV) on a Q4Matrix given as its arrays, host buffers
inline void gemv_q4(const float* scales, const int8_t* zeros, const uint8_t* data,
                    const int16_t* wsums, int rows, int cols, const float* x, float* y) {
  check(molot_gemv_q4(scales, zeros, data, wsums, rows, cols, x, y));
}

// forward.h:554-558 for a shared-KV layer's query only: per-head RMSNorm
// (q_norm may be null) and NEOX RoPE (freq may be null: NoPE), device
// buffers, stream-ordered.
inline void norm_rope_q_dev(const float* q, float* q_out, const float* q_norm, float eps,
                            const float* freq, int pos, int nq, int d, void* stream = nullptr) {
  check(molot_norm_rope_append_dev(q, nullptr, nullptr, q_out, q_norm, nullptr, 0, eps, freq, pos,
                                   nullptr, nullptr, 0, nq, 1, d, stream));
}

// HBM-resident replacement for Runner::KVC: one handle for all layers.
// Device pointers in, device pointers out; stream-ordered (stream = a
// cudaStream_t, nullptr = legacy default stream).
class KVCache {
 public:
  KVCache(int n_layers, int nkv, int hd, int cap, int kv_dtype = MOLOT_KV_F32)
      : nkv_(nkv), hd_(hd), cap_(cap) {
    check(molot_kv_create_ex(n_layers, nkv, hd, cap, kv_dtype, &h_));
  }
  ~KVCache() { molot_kv_destroy(h_); }
  KVCache(const KVCache&) = delete;
  KVCache& operator=(const KVCache&) = delete;

  int n(int layer) const {
    int r = molot_kv_length(h_, layer);
    if (r < 0) check(r);
    return r;
  }
  int cap() const { return cap_; }
  void set_n(int layer, int n) { check(molot_kv_set_length(h_, layer, n)); }
  // Prefill-style bulk write of rows [slot0, slot0+nrows) ([nrows][nkv*hd]).
  void write(int layer, int slot0, int nrows, const float* k, const float* v,
             void* stream = nullptr) {
    check(molot_kv_write(h_, layer, slot0, nrows, k, v, stream));
  }
  // forward.h:554-575: norms + RoPE on the new token, append at slot n.
  void append_rope(int layer, const float* q, const float* k, const float* v, float* q_out,
                   const float* q_norm, const float* k_norm, bool v_norm, float eps,
                   const float* freq, int pos, int nq, void* stream = nullptr) {
    check(molot_attn_append_rope(h_, layer, q, k, v, q_out, q_norm, k_norm, v_norm ? 1 : 0, eps,
                                 freq, pos, nq, stream));
  }
  // forward.h:578-590: attention over the cache of src_layer.
  // forward.h:554-590 for a KV-owning layer in one launch: QK-norm / V-norm /
  // RoPE of the raw q, k, v, append at slot n, attention into o.
  void step(int layer, const float* q, const float* k, const float* v, const float* q_norm,
            const float* k_norm, bool v_norm, float eps, const float* freq, int pos, float* o,
            int nq, float scale, int window, void* stream = nullptr) {
    check(molot_attn_step(h_, layer, q, k, v, q_norm, k_norm, v_norm ? 1 : 0, eps, freq, pos, o,
                          nq, scale, window, stream));
  }
  // forward.h:368-392: prologue of M tokens, rows appended at n..n+M-1
  void append_rope_tokens(int layer, const float* q, const float* k, const float* v,
                          float* q_out, const float* q_norm, const float* k_norm, bool v_norm,
                          float eps, const float* freq, int pos0, int M, int nq,
                          void* stream = nullptr) {
    check(molot_attn_append_rope_tokens(h_, layer, q, k, v, q_out, q_norm, k_norm, v_norm ? 1 : 0,
                                        eps, freq, pos0, M, nq, stream));
  }
  // forward.h:394-398: prefill attention over src_layer's cache
  void prefill(int src_layer, const float* q, float* o, int nq, int M, float scale, int pos0,
               int window, void* stream = nullptr) {
    check(molot_attn_prefill(h_, src_layer, q, o, nq, M, scale, pos0, window, stream));
  }
  void decode(int src_layer, const float* q, float* o, int nq, float scale, int pos_cur,
              int window, void* stream = nullptr) {
    check(molot_attn_decode(h_, src_layer, q, o, nq, scale, pos_cur, window, stream));
  }
  // Synchronise and surface device-side wait timeouts.
  void sync(void* stream = nullptr) { check(molot_kv_check(h_, stream)); }
  molot_kv_cache* handle() { return h_; }

 private:
  molot_kv_cache* h_ = nullptr;
  int nkv_, hd_, cap_;
};

// Continuous-batching page manager (molot_pager_*): sequences, their pages
// and lengths, block tables for a batch, and optionally the per-layer K/V
// page pools in HBM ([num_pages][nkv][page_size][d] of the storage type).
class Pager {
 public:
  Pager(int n_layers, int nkv, int d, int page_size, int num_pages, int max_seqs,
        int max_pages_per_seq, int kv_dtype = MOLOT_KV_F32)
      : max_pages_(max_pages_per_seq) {
    check(molot_pager_create_ex(n_layers, nkv, d, page_size, num_pages, max_seqs,
                                max_pages_per_seq, kv_dtype, &h_));
  }
  ~Pager() { molot_pager_destroy(h_); }
  Pager(const Pager&) = delete;
  Pager& operator=(const Pager&) = delete;

  int add(int slots) {
    int s = -1;
    check(molot_pager_add(h_, slots, &s));
    return s;
  }
  void grow(int seq, int n_new = 1) { check(molot_pager_grow(h_, seq, n_new)); }
  void free(int seq) { check(molot_pager_free(h_, seq)); }
  int length(int seq) const {
    int r = molot_pager_length(h_, seq);
    if (r < 0) check(r);
    return r;
  }
  int free_pages() const { return molot_pager_free_pages(h_); }
  int max_pages() const { return max_pages_; }
  // Host block table [B][max_pages()] and lengths of the batch `seqs`.
  void tables(const int* seqs, int B, int* block_table, int* seq_lens) {
    check(molot_pager_tables(h_, seqs, B, block_table, seq_lens));
  }
  // Device K/V pools of one layer (raw bases for BF16 / Q8 pools).
  void layer_pools(int layer, float** k_pool, float** v_pool) {
    check(molot_pager_layer_pools(h_, layer, k_pool, v_pool));
  }

 private:
  molot_pager* h_ = nullptr;
  int max_pages_;
};

// Batch shape of one paged decode step (molot_paged_*): build once per step,
// then append + decode per layer over that layer's pools.
class PagedPlan {
 public:
  explicit PagedPlan(int kv_dtype = MOLOT_KV_F32) {
    check(molot_paged_plan_create(&h_));
    check(molot_paged_plan_set_kv_dtype(h_, kv_dtype));
  }
  ~PagedPlan() { molot_paged_plan_destroy(h_); }
  PagedPlan(const PagedPlan&) = delete;
  PagedPlan& operator=(const PagedPlan&) = delete;

  // seq_lens (host): slots per sequence, the new token's included.
  void build(int B, int nq, int nkv, int d, const int* seq_lens, const int* positions = nullptr,
             int window = 0, void* stream = nullptr) {
    check(molot_paged_plan_build(h_, B, nq, nkv, d, seq_lens, positions, window, stream));
  }
  // forward.h:554-575 for the batch: the new rows go to slot seq_lens[b]-1.
  void append(const float* q, const float* k, const float* v, float* q_out, const float* q_norm,
              const float* k_norm, bool v_norm, float eps, const float* freq, float* k_pool,
              float* v_pool, const int* block_table, int max_pages, int page_size,
              void* stream = nullptr) {
    check(molot_paged_append(h_, q, k, v, q_out, q_norm, k_norm, v_norm ? 1 : 0, eps, freq, k_pool,
                             v_pool, block_table, max_pages, page_size, stream));
  }
  void decode(const float* Q, float* O, const float* k_pool, const float* v_pool,
              const int* block_table, int max_pages, int page_size, float scale,
              void* stream = nullptr) {
    check(molot_paged_decode(h_, Q, O, k_pool, v_pool, block_table, max_pages, page_size, scale,
                             stream));
  }
  // Synchronise and surface device-side wait timeouts.
  void sync(void* stream = nullptr) { check(molot_paged_check(h_, stream)); }

  molot_paged_plan* handle() const { return h_; }

 private:
  molot_paged_plan* h_ = nullptr;
};

// Peer-gather group for kv-head sharding over the GPUs of one node
// (molot_comm_*): construct on every rank, exchange handle() bytes with the
// job's own transport (MPI_Allgather, a socket, ...), then open().  Each
// rank's decode_gather writes its heads' outputs into every rank's
// gathered buffer; wait() orders later work on a stream after all of them.
class PeerGather {
 public:
  PeerGather(int nranks, int rank, size_t buf_bytes) {
    check(molot_comm_create(nranks, rank, buf_bytes, &h_));
  }
  ~PeerGather() { molot_comm_destroy(h_); }
  PeerGather(const PeerGather&) = delete;
  PeerGather& operator=(const PeerGather&) = delete;

  // MOLOT_COMM_HANDLE_BYTES bytes for the other ranks.
  void handle(void* out) const { check(molot_comm_handle(h_, out)); }
  // nranks handles in rank order.
  void open(const void* handles) { check(molot_comm_open(h_, handles)); }
  // This rank's gathered buffer (device floats).
  float* buffer() const {
    float* p = nullptr;
    check(molot_comm_buffer(h_, &p));
    return p;
  }
  // Paged decode of this rank's kv heads, outputs into every rank's buffer
  // at float offset out_offset ([B][nranks*nq][d], this rank's heads at
  // [rank*nq, (rank+1)*nq)).
  void decode_gather(PagedPlan& plan, const float* Q, size_t out_offset, const float* k_pool,
                     const float* v_pool, const int* block_table, int max_pages, int page_size,
                     float scale, void* stream = nullptr) {
    check(molot_paged_decode_gather(plan.handle(), h_, Q, out_offset, k_pool, v_pool, block_table,
                                    max_pages, page_size, scale, stream));
  }
  void wait(void* stream = nullptr) { check(molot_comm_wait(h_, stream)); }
  // Synchronise and surface a wait for a peer that gave up.
  void sync(void* stream = nullptr) { check(molot_comm_check(h_, stream)); }

 private:
  molot_comm* h_ = nullptr;
};

}  // namespace molot_b200
