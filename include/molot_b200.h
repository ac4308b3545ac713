/* molot_b200 — B200 (sm_100a) decode attention behind a plain C ABI.
 *
 * Drop-in replacement for the decode-attention path of Molot
 * (include/molot/attn.h and its call site in include/molot/forward.h).  All
 * arithmetic is FP32.  Every entry point returns an int status (MOLOT_OK or
 * a negative MOLOT_ERR_*) and never throws across the ABI.
 *
 * Conventions
 *   - "host" entry points take host pointers, copy to the current CUDA
 *     device, run, copy back and synchronise: outputs are ready on return,
 *     as with the reference's functions.
 *   - "_dev" / handle entry points take device pointers and a cudaStream_t
 *     (passed as void*, NULL = legacy default stream); they are
 *     stream-ordered and return once the work is enqueued.
 *   - Calls that share a scratch workspace (the per-device default one, or a
 *     handle's own) must be ordered on one stream.
 *   - K/V base pointers must be 16-byte aligned and K/V strides multiples of
 *     4 floats (the kernels stream rows with TMA bulk copies); head_dim must
 *     be 64, 128 or 256 and nq/nkv in {1,2,4,8,16,32} (256: up to 16).
 */
#ifndef MOLOT_B200_H
#define MOLOT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOLOT_B200_ABI_VERSION 1

enum molot_status {
  MOLOT_OK = 0,
  MOLOT_ERR_INVALID = -1,     /* bad argument (sizes, null, alignment) */
  MOLOT_ERR_CUDA = -2,        /* CUDA runtime error; see molot_last_error() */
  MOLOT_ERR_NOMEM = -3,       /* device allocation failed */
  MOLOT_ERR_CACHE_FULL = -4,  /* forward.h:570 "KV cache full" */
  MOLOT_ERR_CACHE_EMPTY = -5, /* forward.h:580 "shared KV empty" */
  MOLOT_ERR_UNSUPPORTED = -6, /* head_dim / group size not instantiated */
  MOLOT_ERR_TIMEOUT = -7,     /* a bounded device-side wait expired */
  MOLOT_ERR_NO_DEVICE = -8    /* no CUDA device */
};

/* Human-readable text for a status code. */
const char* molot_status_string(int status);
/* Detail of the last error on the calling thread (CUDA error text etc.). */
const char* molot_last_error(void);
/* Reads (and clears when `clear` != 0) the device-side status words of the
 * current device's default workspace and of its no-alloc scratch (see
 * molot_attn_decode_strided_noalloc); synchronises the device.  Returns
 * MOLOT_OK or MOLOT_ERR_TIMEOUT. */
int molot_device_status(int clear);

/* Failure-detection test hook (no counterpart in the reference).  The next
 * decode-kernel launch made by the calling host thread, through any entry
 * point, runs with its producer withholding every copy and with its stage
 * waits bounded by wait_limit_ns: the consumers' first wait runs out with no
 * copy in flight, the launch records MOLOT_ERR_TIMEOUT in the status word of
 * the workspace it used and its outputs are garbage.  Nothing faults, traps
 * or hangs.  wait_limit_ns = 0 cancels a pending request.  For tests of the
 * status path (molot_kv_check, molot_paged_check, molot_device_status,
 * molot_noalloc_status); never set in production. */
int molot_debug_withhold_next(unsigned long long wait_limit_ns);

/* ------------------------------------------------------------------------
 * attn.h drop-ins: host buffers, synchronous ("ready on return").
 * The ThreadPool& parameter of the reference is replaced by the current
 * CUDA device.
 * ---------------------------------------------------------------------- */

/* Replaces molot::attn_decode_gqa_cache (attn.h:125-177): Q [nq][qhd],
 * K/V [n][nkv*qhd] slot-major (attn.h:122-124), O [nq][qhd].  Slots
 * [max(0, pos_cur-window+1), n) are attended when window > 0, all n
 * otherwise (attn.h:137); an empty range yields zeros, as the reference. */
int molot_attn_decode_gqa_cache(const float* Q, const float* K, const float* V, float* O, int nq,
                                int nkv, int n, int qhd, float scale, int pos_cur, int window);

/* Replaces molot::attn_decode_gqa (attn.h:111-120): K/V [nkv][n][d]. */
int molot_attn_decode_gqa(const float* Q, const float* K, const float* V, float* O, int nq,
                          int nkv, int n, int d, float scale);

/* Replaces molot::attn_decode_gqa_win (attn.h:178-187): K/V [nkv][n][d]. */
int molot_attn_decode_gqa_win(const float* Q, const float* K, const float* V, float* O, int nq,
                              int nkv, int n, int d, float scale, int pos_cur, int window);

/* Replaces molot::attn_decode_head_win (attn.h:57-101): one head, K/V [n][d]. */
int molot_attn_decode_head_win(const float* Q, const float* K, const float* V, float* out, int n,
                               int d, float scale, int pos_cur, int window);

/* Replaces molot::attn_decode_head (attn.h:104-107). */
int molot_attn_decode_head(const float* Q, const float* K, const float* V, float* out, int n,
                           int d, float scale);

/* Replaces molot::rope_apply (attn.h:19-28) on a host vector of `d` floats
 * (NEOX half-split pairs), computed on the device. */
int molot_rope_apply(float* x, int d, int pos, const float* inv_freq);

/* Replaces molot::rope_inv_freq (attn.h:31-33): out[i] = 1/base^(2i/d).
 * Host-side table set-up (not on the per-token path). */
int molot_rope_inv_freq(float base, int d, float* out);

/* ------------------------------------------------------------------------
 * Device-pointer, stream-ordered forms.
 * ---------------------------------------------------------------------- */

/* Decode attention over any strided contiguous cache: slot t of kv head g at
 * K + t*stride_t + g*stride_h (elements).  [n][nkv*d] (attn.h:125) is
 * stride_t = nkv*d, stride_h = d; [nkv][n][d] (attn.h:111) is stride_t = d,
 * stride_h = n*d.  Uses the current device's default workspace. */
int molot_attn_decode_strided_dev(const float* Q, const float* K, const float* V, float* O,
                                  int nq, int nkv, int n, int d, long long stride_t,
                                  long long stride_h, float scale, int pos_cur, int window,
                                  void* stream);

/* No counterpart in the reference: molot_attn_decode_strided_dev for callers
 * that cannot allocate device memory (their host runtime owns every device
 * allocation, or a cudaMalloc on first use would synchronise the device).
 * Same arguments and results, but the split-KV scratch is a fixed ~1.4 MB
 * array inside the library (held by every GPU that loads it) instead of a
 * workspace allocated on first use.  Limits: head_dim 64/128/256, group
 * nq/nkv 1/2/4/8 with group*head_dim <= 1024, nkv <= 256; larger requests
 * return MOLOT_ERR_UNSUPPORTED.  The first call on a device sets up the
 * scratch address (make it before any stream capture).  All calls share the
 * scratch: calls that overlap on the GPU race, so order them on one stream. */
int molot_attn_decode_strided_noalloc(const float* Q, const float* K, const float* V, float* O,
                                      int nq, int nkv, int n, int d, long long stride_t,
                                      long long stride_h, float scale, int pos_cur, int window,
                                      void* stream);

/* Status word of the no-alloc scratch on the current device: synchronises
 * `stream`, returns MOLOT_OK, or MOLOT_ERR_TIMEOUT when a no-alloc decode
 * gave up on a bounded wait since the word was last cleared (its outputs are
 * then garbage); clears the word when `clear` != 0.  The word stays set
 * until read with clear (no-alloc calls do not reset it).  Allocates
 * nothing. */
int molot_noalloc_status(void* stream, int clear);

/* Replaces molot::attn_prefill_gqa (gemm.h:409-446) on host buffers: Qm, Om
 * [M][nq][d], K/V [N][nkv*d] (attn.h:122-124 layout); query m sits at
 * position pos0+m and attends slots [max(0, pos-window+1), min(pos+1, N)).
 * nq/nkv must divide 64; d 64, 128 or 256. */
int molot_attn_prefill_gqa(const float* Qm, const float* K, const float* V, float* Om, int nq,
                           int nkv, int M, int N, int d, float scale, int pos0, int window);

/* molot_attn_prefill_gqa on device buffers with any cache strides (slot t of
 * kv head g at K + t*stride_t + g*stride_h), stream-ordered. */
int molot_attn_prefill_strided_dev(const float* Q, const float* K, const float* V, float* O,
                                   int nq, int nkv, int M, int N, int d, long long stride_t,
                                   long long stride_h, float scale, int pos0, int window,
                                   void* stream);

/* ------------------------------------------------------------------------
 * Q4 GEMV (the projections either side of attention, forward.h:543-553,600)
 * ---------------------------------------------------------------------- */

/* Replaces molot::gemv_q4 (gemm.h:223-254) on host buffers: a Q4Matrix
 * (quant.h:70-80) given as its arrays -- scales [rows][cols/32] FP32, zeros
 * [rows][cols/32] int8, data [rows][cols/2] packed nibbles (element 2j in
 * the low nibble of byte j), wsums (accepted, unused) -- times x [cols];
 * y [rows].  Activations are quantized to int8 per 32 values as
 * quantize_act_q8 does (gemm.h:44-70).  cols must be a multiple of 32. */
int molot_gemv_q4(const float* scales, const int8_t* zeros, const uint8_t* data,
                  const int16_t* wsums, int rows, int cols, const float* x, float* y);

/* molot_gemv_q4 on device buffers (data and x 16-byte aligned),
 * stream-ordered, one launch.  The launch fetches weights before it waits
 * for its predecessor on the stream: do not write W in a kernel that
 * releases its dependents early (programmatic dependent launch) right
 * before this call. */
int molot_gemv_q4_dev(const float* scales, const int8_t* zeros, const uint8_t* data, int rows,
                      int cols, const float* x, float* y, void* stream);

/* forward.h:554-575 on device buffers for a [cap][nkv*d] cache: q (nq heads)
 * and k (nkv heads) get per-head weighted RMSNorm when q_norm / k_norm are
 * non-null, then NEOX RoPE at `pos` when freq ([d/2]) is non-null; v gets a
 * plain RMSNorm over all nkv*d values when v_norm != 0.  The rotated q goes
 * to q_out; k and v are written to slot `slot` of kc / vc.  With k, v, kc and
 * vc all NULL only q is processed (a shared-KV layer's query, forward.h:554-558,
 * before molot_attn_decode on its source layer). */
int molot_norm_rope_append_dev(const float* q, const float* k, const float* v, float* q_out,
                               const float* q_norm, const float* k_norm, int v_norm, float eps,
                               const float* freq, int pos, float* kc, float* vc, int slot,
                               int nq, int nkv, int d, void* stream);

/* ------------------------------------------------------------------------
 * KV cache handle: replaces Runner::KVC (forward.h:48-51) and its up-front
 * allocation (forward.h:103-110).  Per layer, K and V are FP32 in HBM,
 * 256-byte aligned, laid out head-major [nkv][cap][hd] (each kv head's slots
 * contiguous, so the decode kernel streams whole 16-slot blocks with single
 * TMA copies), with a host-side slot count n.  Rows enter in the
 * reference's [slot][nkv*hd] order through molot_kv_write / append.
 * ---------------------------------------------------------------------- */
typedef struct molot_kv_cache molot_kv_cache;

/* KV element types of the handle. */
enum molot_kv_dtype {
  MOLOT_KV_F32 = 0, /* the reference's format (bit-exact QK scores) */
  MOLOT_KV_BF16 = 1, /* half the bytes; the reference specifies but does not
                        implement it: results match the reference run on the
                        bf16-rounded cache */
  MOLOT_KV_Q8 = 2 /* ~0.28x the bytes (the Q8 KV of the reference's design,
                     DESIGN.md:48,87-88, deferred at exp/README.md:36-39): a
                     row is hd int8 codes then hd/32 FP32 scales, padded to
                     16 bytes; each 32-value block quantized by the rule of
                     quant.h:33-43 (s = absmax/127, q = nearbyint(x/s)).
                     Results match the reference run on the dequantized
                     cache (q*s) within the parity tolerance.  All handle
                     calls accept it (write, append, step, decode,
                     prefill). */
};

int molot_kv_create(int n_layers, int nkv, int hd, int cap, molot_kv_cache** out);
/* molot_kv_create with a storage type.  With MOLOT_KV_BF16 every row that
 * enters the cache (write, append, step, prefill prologue) is rounded to
 * bf16 (nearest even), with MOLOT_KV_Q8 quantized per 32 values; attention
 * math stays FP32. */
int molot_kv_create_ex(int n_layers, int nkv, int hd, int cap, int kv_dtype,
                       molot_kv_cache** out);
/* MOLOT_KV_F32, MOLOT_KV_BF16 or MOLOT_KV_Q8 (or a negative status). */
int molot_kv_dtype(const molot_kv_cache* kv);
void molot_kv_destroy(molot_kv_cache* kv);
int molot_kv_length(const molot_kv_cache* kv, int layer);
int molot_kv_set_length(molot_kv_cache* kv, int layer, int n);
/* Device base of a layer's K and V ([nkv][cap][hd]); the elements are
 * uint16 bf16 bit patterns for MOLOT_KV_BF16 handles despite the type, and
 * a MOLOT_KV_Q8 layer is bytes, [nkv][cap][row] with row = hd codes, hd/32
 * float scales, padding to a multiple of 16 bytes. */
int molot_kv_layer_data(molot_kv_cache* kv, int layer, float** k, float** v);

/* Copies nrows rows of K and V (each [nrows][nkv*hd] FP32, host or device
 * memory) into slots [slot0, slot0+nrows) of `layer`, stream-ordered; the
 * bulk write a prefill performs (forward.h:370-392).  Does not change n.
 * BF16 handles convert on the device (host rows are staged in a buffer the
 * handle owns: order such writes on one stream). */
int molot_kv_write(molot_kv_cache* kv, int layer, int slot0, int nrows, const float* k,
                   const float* v, void* stream);

/* forward.h:554-575 for a KV-owning layer: normalise/rotate q into q_out,
 * normalise/rotate k and (v_norm) v and append them at slot n, n++.
 * MOLOT_ERR_CACHE_FULL when n == cap (forward.h:570). */
int molot_attn_append_rope(molot_kv_cache* kv, int layer, const float* q, const float* k,
                           const float* v, float* q_out, const float* q_norm,
                           const float* k_norm, int v_norm, float eps, const float* freq,
                           int pos, int nq, void* stream);

/* forward.h:578-590: attention of q (already rotated) over the cache of
 * `src_layer` (the layer itself, or its shared-KV source, model.h:565-583)
 * with its current length.  MOLOT_ERR_CACHE_EMPTY when that length is 0
 * (forward.h:580). */
int molot_attn_decode(molot_kv_cache* kv, int src_layer, const float* q, float* o, int nq,
                      float scale, int pos_cur, int window, void* stream);

/* forward.h:554-590 for a KV-owning layer in one launch: the raw q (nq
 * heads) and the new k, v rows get the QK-norm / V-norm / RoPE of
 * molot_attn_append_rope, the new row is appended at slot n (n++), and the
 * attention over slots [max(0, pos-window+1), n] is written to o ([nq][hd]).
 * Same results as molot_attn_append_rope + molot_attn_decode(layer), without
 * the rotated-q round trip or a second launch.  MOLOT_ERR_CACHE_FULL when
 * n == cap (forward.h:570).  The launch may start while the preceding
 * kernel on the stream drains (programmatic dependent launch): q, k and v
 * are read after it completes, but freq, q_norm and k_norm (the layer's
 * constants) are read before, so they must not be written by the kernel
 * immediately preceding this call. */
int molot_attn_step(molot_kv_cache* kv, int layer, const float* q, const float* k,
                    const float* v, const float* q_norm, const float* k_norm, int v_norm,
                    float eps, const float* freq, int pos, float* o, int nq, float scale,
                    int window, void* stream);

/* forward.h:368-392 (prefill prologue) for M tokens of a KV-owning layer:
 * q [M][nq][hd], k, v [M][nkv][hd] raw projections of tokens at positions
 * pos0..pos0+M-1 get the QK-norm / V-norm / RoPE of molot_attn_append_rope;
 * rotated q goes to q_out [M][nq][hd], k/v rows to slots n..n+M-1, n += M.
 * MOLOT_ERR_CACHE_FULL when n + M > cap (forward.h:385).  M <= 65535. */
int molot_attn_append_rope_tokens(molot_kv_cache* kv, int layer, const float* q, const float* k,
                                  const float* v, float* q_out, const float* q_norm,
                                  const float* k_norm, int v_norm, float eps, const float* freq,
                                  int pos0, int M, int nq, void* stream);

/* Replaces molot::attn_prefill_gqa at forward.h:396 (gemm.h:409-446):
 * causal / sliding-window attention of M rotated queries q [M][nq][hd]
 * (query m at position pos0+m) over the cache of `src_layer` with its
 * current length N; o [M][nq][hd].  nq/nkv must divide 64. */
int molot_attn_prefill(molot_kv_cache* kv, int src_layer, const float* q, float* o, int nq, int M,
                       float scale, int pos0, int window, void* stream);

/* Synchronises the handle's stream work and reports device-side timeouts. */
int molot_kv_check(molot_kv_cache* kv, void* stream);

/* ------------------------------------------------------------------------
 * Paged, batched decode (continuous batching; no counterpart in the
 * reference, which specifies but does not implement paging,
 * DESIGN.md:47-48,103 / README.md:113-114 of the reference).
 * Pools: K and V each [num_pages][nkv][page_size][d] FP32 (or BF16, or Q8
 * rows of bytes, per molot_paged_plan_set_kv_dtype; the pool pointers are
 * then raw bases despite their type); page_size a multiple of 16.
 * block_table [B][max_pages] int32 (device).
 * ---------------------------------------------------------------------- */
typedef struct molot_paged_plan molot_paged_plan;

/* A plan fixes the batch shape for one decode step (all layers): sequence
 * lengths (host array, slots already containing the new token), optional
 * positions (host, NULL = length-1) and the window.  It owns its scratch. */
int molot_paged_plan_create(molot_paged_plan** out);
void molot_paged_plan_destroy(molot_paged_plan* plan);
int molot_paged_plan_build(molot_paged_plan* plan, int B, int nq, int nkv, int d,
                           const int* seq_lens, const int* positions, int window, void* stream);
/* Element type of the pools the plan's appends and decodes use: a
 * molot_kv_dtype (MOLOT_KV_F32 when never set).  The same storage options
 * as the KV handle; no counterpart in the reference (see molot_kv_dtype). */
int molot_paged_plan_set_kv_dtype(molot_paged_plan* plan, int kv_dtype);

/* Attention for every sequence of the plan: Q, O [B][nq][d] device. */
int molot_paged_decode(molot_paged_plan* plan, const float* Q, float* O, const float* k_pool,
                       const float* v_pool, const int* block_table, int max_pages,
                       int page_size, float scale, void* stream);

/* forward.h:554-575 for a batch: each sequence's new k/v go to slot
 * seq_lens[b]-1 of its pages; q is normalised/rotated into q_out. */
int molot_paged_append(molot_paged_plan* plan, const float* q, const float* k, const float* v,
                       float* q_out, const float* q_norm, const float* k_norm, int v_norm,
                       float eps, const float* freq, float* k_pool, float* v_pool,
                       const int* block_table, int max_pages, int page_size, void* stream);

/* Synchronises and reports device-side timeouts of the plan's launches. */
int molot_paged_check(molot_paged_plan* plan, void* stream);

/* ------------------------------------------------------------------------
 * Peer gather for kv-head sharding over several GPUs (no counterpart in the
 * reference, which runs on one CPU; it serves forward.h:589-600, where the
 * attention of every head feeds the output projection).  One process per
 * GPU of one node.  Rank r owns kv heads [r*nkv/N, (r+1)*nkv/N) and their
 * grouped q heads, for every sequence.  Its paged decode writes each final
 * output value straight into the gathered buffer of every rank over NVLink
 * / NVSwitch (plain stores to peer memory mapped by CUDA IPC; no
 * multicast), so the gather costs no separate collective and overlaps the
 * attention itself.  Set-up:
 *   molot_comm_create(N, r, bytes, &c);            every rank, its own GPU
 *   molot_comm_handle(c, h[r]);                    64 bytes per rank
 *   (exchange the N handles: MPI_Allgather, sockets, a torch store ...)
 *   molot_comm_open(c, h);                         maps the peers' buffers
 * Per layer: molot_paged_decode_gather(plan, c, ...) then, on the stream of
 * whatever reads the gathered outputs, molot_comm_wait(c, stream).  Every
 * rank makes the same sequence of decode_gather / wait calls on one comm
 * (each wait matches the decode_gather of the same index).  An offset of the
 * buffer may be rewritten once every rank has consumed it: alternating two
 * offsets by layer parity is safe when each rank consumes layer l's outputs
 * in stream order before its decode of layer l+1.
 * ---------------------------------------------------------------------- */
typedef struct molot_comm molot_comm;

#define MOLOT_COMM_HANDLE_BYTES 64
#define MOLOT_COMM_MAX_RANKS 8

/* This rank's end of an nranks-way group on the current device, with a
 * gathered-output buffer of buf_bytes (a multiple of 16) plus a small
 * control block.  nranks 1..8; with nranks == 1 no open is needed. */
int molot_comm_create(int nranks, int rank, size_t buf_bytes, molot_comm** out);
/* The IPC handle of this rank's buffer (MOLOT_COMM_HANDLE_BYTES bytes). */
int molot_comm_handle(const molot_comm* c, void* handle);
/* Maps every peer's buffer: `handles` holds nranks handles in rank order
 * (this rank's own entry is ignored). */
int molot_comm_open(molot_comm* c, const void* handles);
/* Device address of this rank's gathered buffer (floats). */
int molot_comm_buffer(const molot_comm* c, float** buf);
/* molot_paged_decode whose outputs land in every rank's gathered buffer at
 * float offset out_offset, laid out [B][nranks*nq][d] with this rank's nq
 * heads (the plan's) at [rank*nq, (rank+1)*nq).  Every sequence of the plan
 * must attend at least one slot.  Q [B][nq][d] as for molot_paged_decode. */
int molot_paged_decode_gather(molot_paged_plan* plan, molot_comm* c, const float* Q,
                              size_t out_offset, const float* k_pool, const float* v_pool,
                              const int* block_table, int max_pages, int page_size, float scale,
                              void* stream);
/* Stream-ordered: work after it on `stream` sees every rank's outputs of
 * the matching molot_paged_decode_gather.  The wait is bounded (5 s); one
 * that gives up records MOLOT_ERR_TIMEOUT for molot_comm_check. */
int molot_comm_wait(molot_comm* c, void* stream);
/* Synchronises `stream` and reports (then clears) a wait that gave up. */
int molot_comm_check(molot_comm* c, void* stream);
void molot_comm_destroy(molot_comm* c);

/* ------------------------------------------------------------------------
 * Continuous-batching page manager: page ids, per-sequence page lists and
 * lengths, block tables for a batch; optionally the per-layer K/V page pools
 * ([num_pages][nkv][page_size][d] FP32 each) in HBM.  The reference
 * specifies this (its DESIGN.md:47-48,101-105) and implements none of it.
 * Pages come from a LIFO free list, lowest id first in a fresh pager.  One
 * host thread at a time per call (internally locked).
 * ---------------------------------------------------------------------- */
typedef struct molot_pager molot_pager;

/* n_layers = 0: tables only, no device memory (and no CUDA call). */
int molot_pager_create(int n_layers, int nkv, int d, int page_size, int num_pages, int max_seqs,
                       int max_pages_per_seq, molot_pager** out);
/* molot_pager_create with pools of a molot_kv_dtype (rows of d floats, d
 * bf16, or Q8 rows of q8 bytes: d codes, d/32 float scales, padded to 16). */
int molot_pager_create_ex(int n_layers, int nkv, int d, int page_size, int num_pages,
                          int max_seqs, int max_pages_per_seq, int kv_dtype, molot_pager** out);
void molot_pager_destroy(molot_pager* p);
/* A new sequence with `slots` slots reserved (its prompt); id in *seq.
 * MOLOT_ERR_CACHE_FULL when no sequence slot or not enough pages. */
int molot_pager_add(molot_pager* p, int slots, int* seq);
/* Reserves n_new more slots (the tokens of the next step); length += n_new. */
int molot_pager_grow(molot_pager* p, int seq, int n_new);
/* Returns the sequence's pages to the pool. */
int molot_pager_free(molot_pager* p, int seq);
int molot_pager_length(const molot_pager* p, int seq);
int molot_pager_free_pages(const molot_pager* p);
/* Host block table [B][max_pages_per_seq] (unused entries 0) and lengths of
 * the batch `seqs`, ready for molot_paged_plan_build / molot_paged_decode. */
int molot_pager_tables(molot_pager* p, const int* seqs, int B, int* block_table, int* seq_lens);
/* Device K/V pools of one layer. */
int molot_pager_layer_pools(molot_pager* p, int layer, float** k_pool, float** v_pool);

#ifdef __cplusplus
}
#endif
#endif /* MOLOT_B200_H */
