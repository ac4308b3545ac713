// Continuous-batching page manager: the block-table side of a paged KV cache
// (the reference specifies 16-token pages and continuous batching, its
// DESIGN.md:47-48,101-105, and implements neither).  Host logic -- a free
// list of page ids, each sequence's page list and length, block tables for a
// batch -- plus, optionally, the per-layer K/V page pools in HBM that
// molot_paged_decode / molot_paged_append read and write.
//
// Pages are handed out lowest id first from a LIFO free list, so a freed
// sequence's pages are reused before untouched ones (warm in L2) and the
// tables of a fresh pager are deterministic.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "molot_b200.h"

namespace molot {
int set_last_error(int code, const char* msg);
}

struct molot_pager {
  int n_layers = 0, nkv = 0, d = 0, page_size = 0, num_pages = 0, max_seqs = 0;
  int max_pages_per_seq = 0;
  std::vector<int> free_pages;            // stack: back() is handed out next
  std::vector<std::vector<int>> pages;    // per sequence slot
  std::vector<int> len;                   // slots in use per sequence
  std::vector<char> live;
  unsigned char* pools = nullptr;  // [n_layers][2][num_pages][nkv][page_size][row], may be null
  size_t pool_bytes = 0;           // per K (or V) pool of one layer
  int kvt = MOLOT_KV_F32;
  int device = -1;
  mutable std::mutex mu;  // every call, queries included
};

namespace {

int pager_fail(int code, const std::string& msg) { return molot::set_last_error(code, msg.c_str()); }

int pages_for(const molot_pager* p, int slots) {
  return (slots + p->page_size - 1) / p->page_size;
}

// Grows sequence s to `slots` slots, taking pages from the free list.
int reserve(molot_pager* p, int s, int slots) {
  const int need = pages_for(p, slots);
  if (need > p->max_pages_per_seq)
    return pager_fail(MOLOT_ERR_CACHE_FULL, "sequence exceeds max_pages_per_seq");
  const int more = need - (int)p->pages[s].size();
  if (more > (int)p->free_pages.size())
    return pager_fail(MOLOT_ERR_CACHE_FULL, "page pool exhausted");
  for (int i = 0; i < more; ++i) {
    p->pages[s].push_back(p->free_pages.back());
    p->free_pages.pop_back();
  }
  return MOLOT_OK;
}

}  // namespace

extern "C" {

int molot_pager_create(int n_layers, int nkv, int d, int page_size, int num_pages, int max_seqs,
                       int max_pages_per_seq, molot_pager** out) {
  return molot_pager_create_ex(n_layers, nkv, d, page_size, num_pages, max_seqs,
                               max_pages_per_seq, MOLOT_KV_F32, out);
}

int molot_pager_create_ex(int n_layers, int nkv, int d, int page_size, int num_pages,
                          int max_seqs, int max_pages_per_seq, int kv_dtype, molot_pager** out) {
  if (!out) return pager_fail(MOLOT_ERR_INVALID, "null out");
  if (kv_dtype != MOLOT_KV_F32 && kv_dtype != MOLOT_KV_BF16 && kv_dtype != MOLOT_KV_Q8)
    return pager_fail(MOLOT_ERR_INVALID, "kv_dtype must be MOLOT_KV_F32, MOLOT_KV_BF16 or MOLOT_KV_Q8");
  if (kv_dtype == MOLOT_KV_Q8 && d % 64)
    return pager_fail(MOLOT_ERR_INVALID, "Q8 pools need d a multiple of 64");
  *out = nullptr;
  if (n_layers < 0 || nkv <= 0 || d <= 0 || page_size <= 0 || page_size % 16 || num_pages <= 0 ||
      max_seqs <= 0 || max_pages_per_seq <= 0)
    return pager_fail(MOLOT_ERR_INVALID, "bad pager sizes (page_size a multiple of 16)");
  auto* p = new molot_pager();
  p->n_layers = n_layers;
  p->nkv = nkv;
  p->d = d;
  p->page_size = page_size;
  p->num_pages = num_pages;
  p->max_seqs = max_seqs;
  p->max_pages_per_seq = max_pages_per_seq;
  p->kvt = kv_dtype;
  p->free_pages.resize(num_pages);
  for (int i = 0; i < num_pages; ++i) p->free_pages[i] = num_pages - 1 - i;  // 0 handed out first
  p->pages.assign(max_seqs, {});
  p->len.assign(max_seqs, 0);
  p->live.assign(max_seqs, 0);
  if (n_layers > 0) {
    cudaGetDevice(&p->device);
    // bytes of one row of one kv head: d floats, d bf16, or a Q8 row
    const size_t row = kv_dtype == MOLOT_KV_Q8 ? (size_t)((d + d / 8 + 15) & ~15)
                                               : (size_t)d * (kv_dtype == MOLOT_KV_BF16 ? 2 : 4);
    p->pool_bytes = ((size_t)num_pages * nkv * page_size * row + 255) & ~size_t(255);
    const cudaError_t e = cudaMalloc(&p->pools, p->pool_bytes * 2 * (size_t)n_layers);
    if (e != cudaSuccess) {
      delete p;
      return pager_fail(MOLOT_ERR_NOMEM, std::string("cudaMalloc(page pools): ") +
                                             cudaGetErrorString(e));
    }
  }
  *out = p;
  return MOLOT_OK;
}

void molot_pager_destroy(molot_pager* p) {
  if (!p) return;
  if (p->pools) {
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(p->device);
    cudaDeviceSynchronize();
    cudaFree(p->pools);
    if (prev >= 0) cudaSetDevice(prev);
  }
  delete p;
}

int molot_pager_add(molot_pager* p, int slots, int* seq) {
  if (!p || !seq || slots < 0) return pager_fail(MOLOT_ERR_INVALID, "bad arguments");
  std::lock_guard<std::mutex> lk(p->mu);
  int s = -1;
  for (int i = 0; i < p->max_seqs; ++i)
    if (!p->live[i]) {
      s = i;
      break;
    }
  if (s < 0) return pager_fail(MOLOT_ERR_CACHE_FULL, "no free sequence slot");
  p->pages[s].clear();
  int rc = reserve(p, s, slots);
  if (rc) {
    for (int pg : p->pages[s]) p->free_pages.push_back(pg);
    p->pages[s].clear();
    return rc;
  }
  p->live[s] = 1;
  p->len[s] = slots;
  *seq = s;
  return MOLOT_OK;
}

int molot_pager_grow(molot_pager* p, int seq, int n_new) {
  if (!p || seq < 0 || seq >= (p ? p->max_seqs : 0) || n_new < 0)
    return pager_fail(MOLOT_ERR_INVALID, "bad arguments");
  std::lock_guard<std::mutex> lk(p->mu);
  if (!p->live[seq]) return pager_fail(MOLOT_ERR_INVALID, "sequence not live");
  int rc = reserve(p, seq, p->len[seq] + n_new);
  if (rc) return rc;  // pages taken by a failed reserve stay with the sequence
  p->len[seq] += n_new;
  return MOLOT_OK;
}

int molot_pager_free(molot_pager* p, int seq) {
  if (!p || seq < 0 || seq >= p->max_seqs) return pager_fail(MOLOT_ERR_INVALID, "bad sequence");
  std::lock_guard<std::mutex> lk(p->mu);
  if (!p->live[seq]) return pager_fail(MOLOT_ERR_INVALID, "sequence not live");
  // reverse so the sequence's first page is handed out first again
  for (auto it = p->pages[seq].rbegin(); it != p->pages[seq].rend(); ++it)
    p->free_pages.push_back(*it);
  p->pages[seq].clear();
  p->len[seq] = 0;
  p->live[seq] = 0;
  return MOLOT_OK;
}

int molot_pager_length(const molot_pager* p, int seq) {
  if (!p) return pager_fail(MOLOT_ERR_INVALID, "null pager");
  std::lock_guard<std::mutex> lk(p->mu);
  if (seq < 0 || seq >= p->max_seqs || !p->live[seq])
    return pager_fail(MOLOT_ERR_INVALID, "bad sequence");
  return p->len[seq];
}

int molot_pager_free_pages(const molot_pager* p) {
  if (!p) return pager_fail(MOLOT_ERR_INVALID, "null pager");
  std::lock_guard<std::mutex> lk(p->mu);
  return (int)p->free_pages.size();
}

int molot_pager_tables(molot_pager* p, const int* seqs, int B, int* block_table, int* seq_lens) {
  if (!p || !seqs || B <= 0 || !block_table) return pager_fail(MOLOT_ERR_INVALID, "bad arguments");
  std::lock_guard<std::mutex> lk(p->mu);
  for (int b = 0; b < B; ++b) {
    const int s = seqs[b];
    if (s < 0 || s >= p->max_seqs || !p->live[s])
      return pager_fail(MOLOT_ERR_INVALID, "sequence not live");
    int* row = block_table + (size_t)b * p->max_pages_per_seq;
    const auto& pg = p->pages[s];
    std::copy(pg.begin(), pg.end(), row);
    std::fill(row + pg.size(), row + p->max_pages_per_seq, 0);  // never read (beyond n)
    if (seq_lens) seq_lens[b] = p->len[s];
  }
  return MOLOT_OK;
}

int molot_pager_layer_pools(molot_pager* p, int layer, float** k_pool, float** v_pool) {
  if (!p || layer < 0 || layer >= p->n_layers || !p->pools)
    return pager_fail(MOLOT_ERR_INVALID, "bad layer (or a pager without pools)");
  if (k_pool) *k_pool = reinterpret_cast<float*>(p->pools + (size_t)(2 * layer) * p->pool_bytes);
  if (v_pool) *v_pool = reinterpret_cast<float*>(p->pools + (size_t)(2 * layer + 1) * p->pool_bytes);
  return MOLOT_OK;
}

}  // extern "C"
