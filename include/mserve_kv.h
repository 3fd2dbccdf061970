/*
 * mserve_kv.h — C ABI of the B200 (sm_100a) KV-cache selection-and-offload library
 * (libmserve_kv.so).
 *
 * Every entry point takes plain pointers, sizes and byte strides and a CUDA stream passed
 * as `void*` (NULL = legacy default stream).  Nothing here allocates device memory; the
 * caller owns every buffer.  Kernels are enqueued asynchronously on the given stream and
 * never synchronize the device.
 *
 * Return value: MSKV_OK (0) or one of the MSKV_ERR_* codes; the text of the last failure on
 * the calling thread is available from mskv_last_error().
 *
 * Device-side faults that depend on data (an index outside the valid token range, a page
 * table entry that is negative) are not fatal: the offending row is skipped (a gathered row
 * is zero-filled), and the corresponding MSKV_STATUS_* bit is OR-ed into the optional
 * `status` word (device memory or mapped pinned host memory) so the host can raise after
 * the stream completes.
 *
 * "Device-accessible" below means device memory of the current device or pinned host memory
 * that is mapped into the device address space (cudaHostAlloc / cudaHostRegister under
 * unified addressing).  Host KV stores are read and written in place over PCIe ("UVA",
 * zero-copy); they are never staged through a bounce buffer.
 *
 * Reference interfaces replaced are cited as file:line within the MServe project
 * (qwen-eljrte/...).
 */
#ifndef MSERVE_KV_H
#define MSERVE_KV_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MSKV_ABI_VERSION 2

/* ---- return codes ---------------------------------------------------------------------- */
#define MSKV_OK 0
#define MSKV_ERR_ARG 1         /* invalid argument: null pointer, size, stride or alignment  */
#define MSKV_ERR_NOT_MAPPED 2  /* a host pointer is not pinned + mapped for device access    */
#define MSKV_ERR_DTYPE 3       /* unsupported element type                                    */
#define MSKV_ERR_CUDA 4        /* CUDA runtime error (launch failure, bad device, ...)        */
#define MSKV_ERR_RANGE 5       /* a size exceeds what the entry point supports                */

/* ---- device status bits (OR-ed into the optional `status` word) ------------------------ */
#define MSKV_STATUS_INDEX_OOB 0x1u   /* a source token index was outside [0, len)            */
#define MSKV_STATUS_BAD_PAGE 0x2u    /* a page-table entry needed by a row was negative      */
#define MSKV_STATUS_DST_OOB 0x4u     /* a destination token was outside [0, len)             */
#define MSKV_STATUS_TIMEOUT 0x8u     /* a bounded wait (mskv_flag_wait) reached its time limit */

/* ---- element types ---------------------------------------------------------------------- */
#define MSKV_DT_F32 0
#define MSKV_DT_F16 1
#define MSKV_DT_BF16 2
#define MSKV_DT_F64 3
#define MSKV_DT_FP8_E4M3 4
#define MSKV_DT_FP8_E5M2 5

/* ---- library ---------------------------------------------------------------------------- */
int mskv_abi_version(void);
const char* mskv_last_error(void);
/* Number of kernels this library has launched in this process (all threads, all devices). */
uint64_t mskv_launch_count(void);

/* ---- pinned, mapped host memory (the offload store) --------------------------------------
 * Replaces the `.pin_memory()` host tensors of CPUKVCache
 * (qwen-eljrte/Qwen_Transformer/kv_cache.py:727-728, 756-759) with one allocation per layer
 * that is pinned, mapped and portable, so every GPU of the process can read it in place.   */
int mskv_host_alloc(void** host_ptr, uint64_t bytes);
int mskv_host_free(void* host_ptr);
/* Pin + map an existing host range (cudaHostRegister, mapped | portable). */
int mskv_host_register(void* ptr, uint64_t bytes);
int mskv_host_unregister(void* ptr);
/* Device-accessible address of `ptr` (host-mapped or device memory).  Returns
 * MSKV_ERR_NOT_MAPPED for pageable host memory. */
int mskv_device_view(const void* ptr, void** dev_ptr);

/* ---- (a1) UVA gather, reference layout ----------------------------------------------------
 * Replaces uva_gather_cuda / uva_gather (qwen-eljrte/cuda_uva_kernel.cpp:48-108,
 * qwen-eljrte/cuda_uva_kernel_v2.cpp:86-129).
 *   k_out[b,h,s,:] = k_in[b,h,indices[s],:]   (same for v), one index list shared by all (b,h)
 * k_in, v_in : contiguous [B,H,T,D], pinned mapped host memory (or device memory)
 * indices    : device-accessible int64 [S]
 * k_out,v_out: device memory, contiguous [B,H,S,D]
 * elem_bytes : 1, 2, 4 or 8 (the copy is bit-exact for any element type of that size)
 * Indices outside [0,T) are skipped: the output row is zero-filled and
 * MSKV_STATUS_INDEX_OOB is set in `status` (may be NULL). */
int mskv_uva_gather(const void* k_in, const void* v_in, const int64_t* indices,
                    int64_t num_selected, int64_t batch_size, int64_t num_heads,
                    int64_t seq_len, int64_t head_dim, int32_t elem_bytes,
                    void* k_out, void* v_out, uint32_t* status, void* stream);

/* ---- generic row addressing ----------------------------------------------------------------
 * A "segment" is one (b, h) pair; a "row" is the head_dim vector of one token of one segment.
 * The address of logical token t of segment (b, h) on one side of a move is
 *   paged  (page_table != NULL): base + page_table[b*pt_stride_b + t/page_size]*stride_page
 *                                     + h*stride_h + (t % page_size)*stride_t
 *                                (a page id outside [0, num_pages) skips the row)
 *   strided (page_table == NULL): base + b*stride_b + h*stride_h + p*stride_t,
 *                                 p = t, or (ring_start[b] + t) mod ring_cap when ring_start
 * and t is valid when 0 <= t < len[b] (len == NULL: len_scalar).  All strides in bytes. */
typedef struct mskv_rows {
  const void* base_k;
  const void* base_v;           /* NULL: the move has no V half                       */
  int64_t stride_b;
  int64_t stride_h;
  int64_t stride_t;
  int64_t stride_page;
  int64_t pt_stride_b;          /* elements                                           */
  int64_t len_scalar;
  int64_t num_pages;            /* paged: page ids must lie in [0, num_pages)         */
  const int32_t* page_table;
  const int32_t* ring_start;    /* per batch; physical slot of logical token 0        */
  const int32_t* tok0;          /* per batch; logical token of row 0 (NULL: 0)        */
  const int32_t* len;           /* per batch; valid logical tokens (NULL: len_scalar) */
  int32_t page_size;
  int32_t ring_cap;
} mskv_rows;

/* ---- (a1/a2/a3) selected-row gather: per-segment indices ----------------------------------
 * Replaces CPUKVCache.get_sparse_async_uva / get_sparse_async
 * (qwen-eljrte/Qwen_Transformer/kv_cache.py:493-543, 545-629) and generalises the reference
 * kernel to per-(b, KV head) index lists, ring-buffer host stores, paged sources and ragged
 * selections.  Row s of segment (b,h) copies source token
 *   idx[b*idx_stride_b + h*idx_stride_h + s]            (index list, int32 or int64)
 * for s < count, count = counts ? counts[b*cnt_stride_b + h*cnt_stride_h] : num_selected,
 * into destination token (dst.tok0 ? dst.tok0[b] : 0) + s. */
typedef struct mskv_gather_desc {
  mskv_rows src;
  mskv_rows dst;
  const void* indices;
  int64_t idx_stride_b;         /* elements; 0 with idx_stride_h 0 = one shared list  */
  int64_t idx_stride_h;
  const int32_t* counts;        /* NULL: every segment has num_selected rows          */
  int64_t cnt_stride_b;
  int64_t cnt_stride_h;
  int64_t row_bytes;            /* head_dim * element size                            */
  uint32_t* status;
  int32_t index_bits;           /* 32 or 64                                           */
  int32_t batch;
  int32_t heads;
  int32_t num_selected;         /* rows per segment (upper bound when counts != NULL) */
  int32_t max_ctas;             /* grid bound; 0: library default (bounded when either
                                   side is host memory, the full grid otherwise)       */
  int32_t pad_;
} mskv_gather_desc;
int mskv_gather(const mskv_gather_desc* d, void* stream);

/* ---- (c) contiguous row moves: paged append, host write-back, page write-back ------------
 * Row i (0 <= i < n, n = counts ? counts[b] : num_tokens) of segment (b,h) copies
 * source token (src.tok0 ? src.tok0[b] : 0) + i to destination token
 * (dst.tok0 ? dst.tok0[b] : 0) + i.  With a paged destination this is the paged append of
 * new KV into HBM pages; with a ring-strided host destination it is the write-back that
 * replaces CPUKVCache.append_new's torch.cat + keep-last-max_len
 * (qwen-eljrte/Qwen_Transformer/kv_cache.py:718-765; kv_cache_optimized.py:54-149); with a
 * paged source and host destination it is the write-back of evicted pages. */
typedef struct mskv_copy_desc {
  mskv_rows src;
  mskv_rows dst;
  const int32_t* counts;        /* per batch; NULL: num_tokens                        */
  int64_t row_bytes;
  uint32_t* status;
  int32_t batch;
  int32_t heads;
  int32_t num_tokens;
  int32_t max_ctas;             /* grid bound; 0: library default, as mskv_gather     */
} mskv_copy_desc;
int mskv_copy_rows(const mskv_copy_desc* d, void* stream);

/* ---- (b) importance scores ----------------------------------------------------------------
 * Replaces the scoring half of compute_token_importance
 * (qwen-eljrte/Qwen_Transformer/attention.py:532-565 for "attention_score", 574 for "norm").
 * method 0 (attention_score): scores[b,hk,t] = sum_d qsum[b,hk,d] * k[b,hk,t,d] in fp32,
 *          qsum[b,hk,:] = sum_{g<G} q[b, hk*G+g, :]  (G = q_heads / kv_heads; the GQA group
 *          sum, equal to the reference's per-head products summed over repeat_kv'd heads)
 * method 1 (norm):            scores[b,hk,t] = sqrt(sum_d k[b,hk,t,d]^2) in fp32
 * k rows are addressed by `k` (mskv_rows, base_v unused); q row (b, hq) is at
 * q + b*q_stride_b + hq*q_stride_h (bytes); scores row (b,hk) at
 * scores + (b*kv_heads + hk)*scores_stride (elements); tokens t >= len[b] are not written
 * (len[b] above max_tokens is clamped to it); tokens whose page is unmapped score -inf
 * (MSKV_STATUS_BAD_PAGE).
 * Fast path (16-bit K, head_dim in {64,128,256}, 16-byte aligned rows, page_size a multiple
 * of 8): register streaming, 8 rows per group of head_dim/8 lanes with 16-byte loads, 24
 * warps per SM each with one slice's loads in flight; warps share the slices that hold tokens
 * equally however ragged len[] is.  Other shapes use a 32-row register kernel or a generic
 * one. */
typedef struct mskv_score_desc {
  mskv_rows k;
  const void* q;
  int64_t q_stride_b;
  int64_t q_stride_h;
  float* scores;
  int64_t scores_stride;
  int64_t max_tokens;           /* upper bound of len[b] (< 2^31), <= scores_stride   */
  uint32_t* status;             /* optional device status word                        */
  int32_t dtype;                /* MSKV_DT_BF16 / F16 / F32, same for q and k         */
  int32_t method;               /* 0 attention_score, 1 norm                          */
  int32_t batch;
  int32_t q_heads;
  int32_t kv_heads;
  int32_t head_dim;
} mskv_score_desc;
int mskv_score(const mskv_score_desc* d, void* stream);
/* mskv_score that also stores every score into npeers (0..7) other copies of d->scores, at
 * the same offsets: the score rows of this rank's KV heads written straight into the other
 * ranks' gathered buffers through CUDA IPC mappings (mskv_ipc_open), over NVLink.  The
 * kernel makes its stores system-visible before it exits; signal the peers afterwards with
 * mskv_flag_signal on the same stream. */
int mskv_score_fanout(const mskv_score_desc* d, float* const* peer_scores, int32_t npeers, void* stream);

/* ---- (b) top-k with recent window ---------------------------------------------------------
 * Replaces the selection half of compute_token_importance
 * (qwen-eljrte/Qwen_Transformer/attention.py:567-572, torch.topk) and adds the recent window.
 * Selection j (b = j / sel_per_batch) ranks the key
 *   key(t) = scale * sum_{r<rows_per_sel} scores[row(j, r) + t],
 *   row(j, r) = j*sel_stride + (r / row_block)*block_stride + (r % row_block)*scores_stride
 * (fp32, summed in r order; sel_stride 0 means rows_per_sel*scores_stride and row_block 0
 * means rows_per_sel, i.e. the rows of a selection are consecutive at scores_stride), over
 * the candidates t in [0, n), n = max(L - recent, 0),
 * L = len[b] (NULL: len_scalar), keeps the top k = min(top_k[b] or top_k_scalar, n) by key
 * (ties broken toward the lower token index, NaN ranks highest), and appends the window
 * [n, L).  The output row idx[j*out_stride ...] is sorted ascending and holds
 * count = k + (L - n) entries; counts[j] receives it (may be NULL).  Scores of the
 * candidates only are read.  When len != NULL, len_scalar bounds every len[b] (larger values
 * are clamped to it) and sizes the kernel: up to 8 x 49152 candidates the keys of a selection
 * live in shared memory (one 1024-thread CTA up to 49152, else a cluster of 2, 4 or 8 CTAs);
 * beyond that one CTA per selection re-reads them from L2. */
typedef struct mskv_topk_desc {
  const float* scores;
  int64_t scores_stride;
  void* out_idx;
  int64_t out_stride;           /* elements                                           */
  int32_t* counts;
  const int32_t* len;
  const int32_t* top_k;         /* per batch, NULL: top_k_scalar                      */
  uint32_t* status;
  float scale;
  int32_t len_scalar;
  int32_t top_k_scalar;
  int32_t recent;
  int32_t num_sel;
  int32_t rows_per_sel;
  int32_t sel_per_batch;
  int32_t out_bits;             /* 32 or 64                                           */
  int32_t row_block;            /* rows per block (0: rows_per_sel)                   */
  int64_t sel_stride;           /* elements (0: rows_per_sel * scores_stride)         */
  int64_t block_stride;         /* elements between row blocks                        */
} mskv_topk_desc;
/* The blocked row layout serves selections shared by KV heads that are sharded over
 * ranks: each rank's per-head score rows [B, Hl, T] all-gathered into [ranks, B, Hl, T]
 * are summed in global head order with sel_stride = Hl*T, row_block = Hl,
 * scores_stride = T, block_stride = B*Hl*T and rows_per_sel = ranks*Hl. */
int mskv_topk(const mskv_topk_desc* d, void* stream);

/* ---- sparse decode attention over the selected rows ---------------------------------------
 * Replaces sparse_sdpa_attention (qwen-eljrte/Qwen_Transformer/attention.py:591-641):
 *   out[b,hq,i,:] = softmax(scale * q[b,hq,i,:] . K_sel[b,hk,s,:]) V_sel[b,hk,s,:],
 *   hk = hq / G, s < count(b,hk)
 * in fp32, output in `dtype`.  K_sel/V_sel row s of (b,hk) at
 *   base + (b*kv_heads + hk)*kv_stride_seg + s*kv_stride_s (bytes).
 * q row (b,hq,i) at q + b*q_stride_b + hq*q_stride_h + i*q_stride_q (bytes), likewise out.
 * `workspace` must hold mskv_attention_workspace_bytes(d) bytes of device memory.  That is 0
 * for the fast path's selections of up to 32768 rows (16-bit q/K/V, head_dim 64 or 128, at
 * most 16 query rows per KV head, 16-byte aligned rows and strides): one kernel whose CTAs of a
 * (b,hk) segment merge through distributed shared memory.  Wider selections use the
 * split-sequence kernels, whose partial results live in the workspace (every launch writes all
 * it reads, so no initialisation is needed; launches that share a workspace must be ordered on
 * one stream).  A segment's rows are split the same way whatever the batch and the number of
 * segments in the call, so a segment's output does not depend on the rest of the call. */
typedef struct mskv_attn_desc {
  const void* q;
  int64_t q_stride_b;
  int64_t q_stride_h;
  int64_t q_stride_q;
  const void* k;
  const void* v;
  int64_t kv_stride_seg;
  int64_t kv_stride_s;
  const int32_t* counts;        /* per (b,hk) segment; NULL: num_selected             */
  void* out;
  int64_t out_stride_b;
  int64_t out_stride_h;
  int64_t out_stride_q;
  void* workspace;
  uint64_t workspace_bytes;
  uint32_t* status;             /* optional device status word                        */
  float scale;
  int32_t dtype;                /* MSKV_DT_BF16 / F16 / F32 for q, K, V and out       */
  int32_t batch;
  int32_t q_heads;
  int32_t kv_heads;
  int32_t head_dim;
  int32_t q_len;
  int32_t num_selected;
} mskv_attn_desc;
uint64_t mskv_attention_workspace_bytes(const mskv_attn_desc* d);
int mskv_sparse_attention(const mskv_attn_desc* d, void* stream);

/* ---- sparse decode attention without any allocation -----------------------------------------
 * No counterpart in the reference: an addition for callers that cannot allocate device memory
 * where they run attention (code under an allocator lock or inside another library's memory
 * pool, host frameworks that forbid cudaMalloc on the decode path, callers with no allocator
 * to hand out a workspace).  Same computation and arguments as mskv_sparse_attention, but
 * d->workspace / d->workspace_bytes are ignored: shapes that need a workspace (selections
 * wider than 32768 rows) get a device array of MSKV_NOALLOC_ATTN_SCRATCH_BYTES built into the
 * library, which each GPU that loads the library holds until the process exits.  Shapes whose
 * mskv_attention_workspace_bytes() exceeds that size are rejected with MSKV_ERR_RANGE.  The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress) with that device current, and looks it up
 * again when the device's context has been re-created since (cudaDeviceReset); make that
 * first call before any stream capture.  Every call on a device shares the array and
 * rewrites every part of it that it reads, so calls that overlap on the GPU -- on streams
 * not ordered with each other -- race and give wrong results.  Calls no cudaMalloc or
 * cudaFree. */
#define MSKV_NOALLOC_ATTN_SCRATCH_BYTES (8u << 20)
int mskv_sparse_attention_noalloc(const mskv_attn_desc* d, void* stream);

/* ---- prefill image-token filter ------------------------------------------------------------
 * Replaces dual_attention_filter (qwen-eljrte/Qwen_Transformer/dual_attention_filter.py:6-103).
 * attn: the attention probabilities of batch 0, element (h, query r, key c) at
 *   attn + h*stride_h + r*stride_q + c*stride_k (elements), dtype F32 / F16 / BF16.
 * Image tokens are the keys [img_start, img_start + img_seq); text tokens are the query rows
 * [text_start, text_start + text_seq) (the reference: img_start = v_token_start, text_start =
 * v_token_start + img_seq, text_seq = T - text_start).  Over the block [heads, text, img], with
 * stage() the rounding to the stage dtype (the input dtype; F16 for F32 input when round_f16,
 * which first rounds every element to f16 as the reference's use_fp16 does) and fp32 sums:
 *   hm[i,j] = stage((sum_h attn[h, text_i, img_j]) / heads)      (heads in order)
 *   sum_j   = stage(sum_i hm[i,j]),  max_j = max_i hm[i,j],  total = stage(sum_j sum_j)
 * (text rows in blocks of 32, each summed in order, block sums in order; the total over tiles
 * of 32 columns the same way).  Image token j is dropped when sum_j < stage(total*global_thr)
 * and max_j < stage(individual_thr) (the threshold rounded to the stage dtype, as torch casts a
 * Python scalar to the tensor's dtype before comparing); the kept ones are written to out_idx
 * (int64, ascending; img_seq entries of room) and their number to *out_count (device int32).
 * workspace: mskv_image_filter_workspace_bytes(img_seq, text_seq) bytes of device memory
 * (row-block partials, column sums and maxima, tile totals), 4-byte aligned. */
typedef struct mskv_filter_desc {
  const void* attn;
  int64_t stride_h;
  int64_t stride_q;
  int64_t stride_k;
  int64_t* out_idx;
  int32_t* out_count;
  void* workspace;
  uint64_t workspace_bytes;
  float global_thr;
  float individual_thr;
  int32_t dtype;
  int32_t heads;
  int32_t img_start;
  int32_t img_seq;
  int32_t text_start;
  int32_t text_seq;
  int32_t round_f16;
  int32_t pad_;
} mskv_filter_desc;
uint64_t mskv_image_filter_workspace_bytes(int32_t img_seq, int32_t text_seq);
int mskv_image_filter(const mskv_filter_desc* d, void* stream);

/* ---- peer memory and flags (score-row exchange between the GPUs of one node) --------------
 * The shared selection's exchange of score rows (attention.py:558-572 with the KV heads on
 * several GPUs) without a collective library: device memory from mskv_ipc_alloc (zeroed;
 * `handle` receives mskv_ipc_handle_bytes() bytes, a cudaIpcMemHandle_t) is mapped by the
 * other processes with mskv_ipc_open and released with mskv_ipc_close / mskv_ipc_free.
 * mskv_flag_signal stores `value` at flags[r][index] for r < nranks (int64 elements, release
 * at system scope) once the stream's earlier work is complete; mskv_flag_wait makes the
 * stream wait until each of flags[0..count) equals `value` (at_least: is >= value), for at
 * most timeout_ns (0 < timeout <= 60 s), after which it sets MSKV_STATUS_TIMEOUT in `status`
 * and lets the stream continue.  Neither uses multicast. */
uint64_t mskv_ipc_handle_bytes(void);
int mskv_ipc_alloc(uint64_t bytes, void** ptr, void* handle);
int mskv_ipc_open(const void* handle, void** ptr);
int mskv_ipc_close(void* ptr);
int mskv_ipc_free(void* ptr);
int mskv_flag_signal(int64_t* const* flags, int32_t nranks, int32_t index, int64_t value, void* stream);
int mskv_flag_wait(const int64_t* flags, int32_t count, int64_t value, int32_t at_least, uint64_t timeout_ns,
                   uint32_t* status, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MSERVE_KV_H */
