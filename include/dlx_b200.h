/*
 * dlx_b200.h - C ABI of the B200 (sm_100a) kernels for Diffulex's decode hot path.
 *
 * The operators, each the device body of one Python entry point of the reference's
 * diffulex_kernel package or of a host loop of its model runner:
 *
 *   dlx_store_kvcache_unified  <- store_kvcache_unified_layout
 *                                 (diffulex_kernel/python/kv_cache_kernels.py:110-124, kernel :11-32)
 *   dlx_load_kvcache           <- load_kvcache (kv_cache_kernels.py:230-279, kernel :127-227)
 *   dlx_decode_attn            <- dllm_flash_attn_decode
 *                                 (diffulex_kernel/python/dllm_flash_attn.py:599-637, kernels :163-536)
 *                                 and, without a cache, dllm_flash_attn_prefill (:539-596, kernel :23-160)
 *   dlx_store_kvcache_distinct <- store_kvcache_distinct_layout (kv_cache_kernels.py:86-107, kernel :35-83)
 *   dlx_decode_attn_prepare    <- the per-step lengths and offsets the runner derives for the kernels
 *                                 (diffulex/strategy/block_diffusion/engine/model_runner.py:125-158)
 *   dlx_build_slot_mapping     <- the runner's slot-mapping loop (model_runner.py:141-151)
 *
 * Conventions: every pointer is a DEVICE pointer unless stated; strides are in ELEMENTS; all
 * functions only enqueue work on `stream` (a cudaStream_t passed as void*), never synchronise,
 * never allocate, never throw; they return 0 or a dlx_status code and leave a message retrievable
 * with dlx_last_error() (thread local).  Nothing is retained after return.  All launches are
 * legal inside CUDA stream capture.
 */
#ifndef DLX_B200_H
#define DLX_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    DLX_OK = 0,
    DLX_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, inconsistent counts            */
    DLX_ERR_UNSUPPORTED = 2,      /* geometry or dtype with no kernel (e.g. head_dim not 64/128) */
    DLX_ERR_ALIGNMENT = 3,        /* a base pointer or stride breaks the 16-byte vector rule     */
    DLX_ERR_WORKSPACE = 4,        /* split-K workspace missing or too small                      */
    DLX_ERR_CUDA = 5              /* a CUDA runtime call failed; see dlx_last_error()            */
} dlx_status;

enum { DLX_DTYPE_BF16 = 0, DLX_DTYPE_FP16 = 1 };

/* Which keys a query row sees.  Cached keys (positions < context_len) are always visible.
 * FULL: every in-flight key (the static block-diffusion kernel, dllm_flash_attn.py:300-307, and
 *       the non-causal varlen call, :634-637).
 * BLOCK_CAUSAL: in-flight key j is visible to query row i iff j < (i / dbs + 1) * dbs
 *       (diffulex_legacy/engine/sequence.py:477-490; dllm_flash_attn.py:109-116). */
enum { DLX_MASK_FULL = 0, DLX_MASK_BLOCK_CAUSAL = 1 };

/* Library version: major * 10000 + minor * 100 + patch. */
int dlx_version(void);
const char* dlx_status_string(int status);
/* Message of the last non-zero status returned on the calling thread ("" if none). */
const char* dlx_last_error(void);

/*
 * Slot-mapped KV store, unified layout.  For every token t in [0, num_tokens) with
 * slot[t] >= 0:  k_cache_rows[slot[t]] = key[t],  v_cache_rows[slot[t]] = value[t], where a cache
 * row is `row_elems` = Hkv*head_dim contiguous elements and caches are [num_slots, row_elems].
 * Tokens with slot < 0 are skipped (kv_cache_kernels.py:24-25).  Slots >= num_slots are skipped
 * too (the reference would write out of bounds).  Offsets are 64-bit (the reference multiplies
 * slot * D in int32, :30).  Bit-exact copy.
 *   key/value       [num_tokens rows, row stride key_row_stride/value_row_stride elements]
 *   slot_mapping    int32 (slot_is_int64 == 0) or int64 (!= 0), num_tokens entries
 *   elem_bytes      size of one element (2 for bf16/fp16)
 */
int dlx_store_kvcache_unified(const void* key, int64_t key_row_stride, const void* value, int64_t value_row_stride,
                              void* k_cache, void* v_cache, const void* slot_mapping, int slot_is_int64,
                              int64_t num_tokens, int64_t row_elems, int elem_bytes, int64_t num_slots,
                              void* stream);

/*
 * Slot-mapped KV store, split ("distinct") layout: K cache [NB, H, hd/x, PAGE, x],
 * V cache [NB, H, hd, PAGE], both contiguous (kv_cache_kernels.py:35-107).
 */
int dlx_store_kvcache_distinct(const void* key, int64_t key_row_stride, const void* value, int64_t value_row_stride,
                               void* k_cache, void* v_cache, const void* slot_mapping, int slot_is_int64,
                               int64_t num_tokens, int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                               int32_t x, int64_t num_pages, int elem_bytes, void* stream);

/*
 * Paged KV gather.  For sequence s (rows o = cu_seqlens_k[s] ...):
 *   out[o + p]         = cache[block_tables[s][p / page] , p % page]   for p < context_lens[s]
 *   out[o + ctx + j]   = kv_new[cu_seqlens_q[s] + j]                   for j < seq_lens[s]
 * cu_seqlens_k cumulates ctx+new (kv_cache_kernels.py:245-248).  Writes every such row, including
 * the last full page of a page-aligned context and a ragged in-flight tail, which the reference
 * kernel leaves unwritten (:167, :204).  Bit-exact copy.  out_rows = rows of k_out/v_out;
 * rows >= cu_seqlens_k[num_seqs] are left untouched.
 *   cache_page_stride / cache_token_stride: elements between pages / between tokens of a page
 *   block_tables [num_seqs, max_blocks] int32, row stride block_table_stride; -1 padded
 */
int dlx_load_kvcache(const void* k_cache, const void* v_cache, int64_t cache_page_stride, int64_t cache_token_stride,
                     const void* k_new, int64_t k_new_row_stride, const void* v_new, int64_t v_new_row_stride,
                     const int32_t* block_tables, int64_t block_table_stride, int32_t max_blocks,
                     const int32_t* context_lens, const int32_t* seq_lens, const int32_t* cu_seqlens_q,
                     const int32_t* cu_seqlens_k, void* k_out, void* v_out, int64_t out_rows, int32_t num_seqs,
                     int32_t page_size, int64_t num_pages, int64_t row_elems, int elem_bytes, void* stream);

/*
 * The slot mapping of a decode step, built on the device: what the reference's model runner builds in a Python
 * loop and copies over every step (diffulex/strategy/block_diffusion/engine/model_runner.py:118, 141-151, 156).
 * Row t of the step's in-flight K/V belongs to the sequence s with cu_seqlens_q[s] <= t < cu_seqlens_q[s+1] and is
 * position pos = context_lens[s] + (t - cu_seqlens_q[s]) of it:
 *     slot[t] = block_tables[s][pos / page_size] * page_size + pos % page_size
 * and -1 (store nothing) when store_flags[s] == 0 (the sequence's block is still being denoised, :141-142), when the
 * position has no page (table entry -1 or pos / page_size >= max_blocks), or when t belongs to no sequence
 * (padding).  store_flags == NULL: every sequence stores.  For page sizes that divide the diffusion block this is
 * the reference's list of whole pages (:143-151).  slot_mapping: int32 or int64, total_rows entries.
 */
int dlx_build_slot_mapping(const int32_t* block_tables, int64_t block_table_stride, int32_t max_blocks,
                           const int32_t* context_lens, const int32_t* cu_seqlens_q, const int32_t* store_flags,
                           int32_t num_seqs, int32_t page_size, int64_t total_rows, int64_t num_pages,
                           void* slot_mapping, int slots_are_int64, void* stream);

/*
 * Paged block-diffusion decode attention.  For sequence s, query rows
 * q[cu_seqlens_q[s] .. cu_seqlens_q[s+1]) of every query head attend to
 * [cached keys 0..context_lens[s]-1 (through block_tables) ; in-flight keys k/v[kv0 .. kv0+new)]
 * with  out = softmax(scale * q k^T + mask) v,  fp32 accumulation, output in the input dtype.
 * kv0/new come from cu_seqlens_kv (which cumulates IN-FLIGHT lengths only, the static decode
 * convention, diffulex/strategy/block_diffusion/engine/model_runner.py:135-139); pass
 * cu_seqlens_kv == NULL to address the in-flight rows with cu_seqlens_q (varlen convention, where
 * the caller's cu_seqlens_k cumulates ctx+new).  Query head h reads KV head h / (Hq/Hkv)
 * (dllm_flash_attn.py:236).  Sequences with a non-positive query length are skipped.
 *
 * Prefill (dllm_flash_attn_prefill, dllm_flash_attn.py:539-596) is the same call without a cache:
 * max_blocks == 0 (caches, block_tables and context_lens may be NULL), cu_seqlens_kv = the prompt's
 * cu_seqlens_k, mask_mode DLX_MASK_FULL for attn_type "full_attention" (:546-552) and
 * DLX_MASK_BLOCK_CAUSAL for "block_attention" (key j visible to query i when
 * j < (i / diffusion_block_size + 1) * diffusion_block_size, :109-116).
 */
typedef struct dlx_decode_attn_params {
    uint32_t struct_bytes;       /* = sizeof(dlx_decode_attn_params), checked                          */
    int32_t dtype;               /* DLX_DTYPE_BF16 | DLX_DTYPE_FP16                                    */
    const void* q;               /* [total_q, Hq, hd], head stride hd, row stride q_row_stride         */
    const void* k;               /* [total_kv_new, Hkv, hd]                                            */
    const void* v;
    const void* k_cache;         /* [num_pages, page_size, Hkv, hd], head stride hd                    */
    const void* v_cache;
    void* out;                   /* [total_q, Hq, hd], row stride out_row_stride                       */
    const int32_t* block_tables; /* [num_seqs, max_blocks], -1 padded                                  */
    const int32_t* context_lens; /* [num_seqs]; ignored (may be NULL) when max_blocks == 0             */
    const int32_t* cu_seqlens_q; /* [num_seqs + 1]                                                     */
    const int32_t* cu_seqlens_kv;/* [num_seqs + 1] in-flight offsets, or NULL (= cu_seqlens_q)         */
    const void* schedule;        /* optional: a schedule written by dlx_decode_attn_prepare for THESE
                                    parameters and the current contents of context_lens / cu_seqlens_* /
                                    block_tables.  NULL: the call plans itself (one more small launch) into
                                    the tail of `workspace`                                            */
    int64_t schedule_bytes;
    void* workspace;             /* scratch, >= dlx_decode_attn_workspace_bytes(): split-K partials and, when
                                    `schedule` is NULL, the schedule.  May be NULL when nothing is needed */
    int64_t workspace_bytes;
    int64_t q_row_stride, k_row_stride, v_row_stride, out_row_stride;
    int64_t cache_page_stride, cache_token_stride;
    int64_t block_table_stride;
    int64_t num_pages;
    int32_t total_q;             /* rows of q / out                                                    */
    int32_t num_seqs, max_blocks;
    int32_t num_q_heads, num_kv_heads, head_dim, page_size;
    int32_t max_q_len;           /* host upper bound on rows per sequence (sizes the M tile)           */
    int32_t max_kv_len;          /* host upper bound on ctx+new per sequence; 0 = max_blocks*page_size
                                    + max_q_len.  Only steers the split-K choice                       */
    int32_t mask_mode;           /* DLX_MASK_*                                                         */
    int32_t diffusion_block_size;
    int32_t num_splits;          /* 0 = choose; >= 1 forces that many key-range splits per sequence    */
    int32_t kernel;              /* 0 = choose; 1 = mma.sync kernel; 2 = tcgen05 kernel, one CTA per item;
                                    3 = tcgen05 kernel, one CTA pair per item (if eligible)            */
    float scale;                 /* softmax scale, hd^-1/2 in every shipped model                      */
    int32_t total_kv;            /* rows of k / v; 0 = total_q.  Bounds the tcgen05 kernels' copies of
                                    in-flight rows: rows past it read as zero                           */
    const void* slot_mapping;    /* optional, [rows of k / v] int32 or int64: the call ALSO stores the in-flight
                                    K / V rows into the caches at these flat slots (negative = skip), i.e. it does
                                    the work of dlx_store_kvcache_unified + dlx_decode_attn (attn_impl.py:54-57 and
                                    :66-67) in one call: the store kernel is launched first on the same stream
                                    (needs contiguous cache pages).  NULL: attention only                       */
    int32_t slots_are_int64;
    int32_t reserved0;
} dlx_decode_attn_params;

/* Bytes of scratch dlx_decode_attn needs for these parameters when it plans itself (split-K partials
 * + schedule; 0 when neither is used), or a negative dlx_status.  Depends only on host-known sizes,
 * never on device contents. */
int64_t dlx_decode_attn_workspace_bytes(const dlx_decode_attn_params* p);
/* Number of splits dlx_decode_attn will use for these parameters. */
int32_t dlx_decode_attn_num_splits(const dlx_decode_attn_params* p);
int dlx_decode_attn(const dlx_decode_attn_params* p, void* stream);

/*
 * The per-step half of decode attention: what the reference's model runner computes on the host before
 * every decode step (diffulex/strategy/block_diffusion/engine/model_runner.py:125-158 and
 * diffulex/strategy/d2f/engine/model_runner.py:150-243: per-sequence lengths and offsets for the kernels),
 * done on the device.  dlx_decode_attn_prepare launches one small kernel that reads context_lens,
 * cu_seqlens_q / cu_seqlens_kv and block_tables and writes a schedule: one packed record per (sequence,
 * KV head, query-token block, key-range split) with its lengths, offsets and first page ids, placed on the
 * persistent CTAs longest first.  Every layer of the step then passes that buffer as `schedule`.  The launch
 * can be captured: a replayed graph re-plans from the refilled metadata buffers.  Only the pointers and sizes
 * named above are read; q / k / v / caches / out may be NULL here.
 * dlx_decode_attn_schedule_bytes: bytes of the buffer (0: the kernel chosen for these parameters takes no
 * schedule, prepare is a no-op), or a negative dlx_status.
 */
int64_t dlx_decode_attn_schedule_bytes(const dlx_decode_attn_params* p);
int dlx_decode_attn_prepare(const dlx_decode_attn_params* p, void* schedule, int64_t schedule_bytes, void* stream);
/* Library plumbing: *id = the capture sequence id of `stream` while it is being captured, else 0 (lets a
 * caller keep one prepared schedule per captured graph). */
int dlx_stream_capture_id(void* stream, uint64_t* id);

/*
 * Decode attention for callers that cannot hand over scratch memory.  No counterpart in the reference.
 *
 * Same operator, same parameters and same results as dlx_decode_attn, but the scratch (partial
 * outputs and log-sum-exps of the key-range splits, the launch's schedule) is a fixed array inside the library's device image
 * instead of `p->workspace` (which is ignored here).  Meant for hosts that own no allocator on the device
 * side of the call: a serving loop whose memory pool is sized and frozen at start-up, a plugin that is
 * handed tensors but may not call cudaMalloc (or torch's allocator) from its callback, code running
 * under a memory budget where a late allocation failure is not an option.  The function calls no
 * allocating routine of CUDA or of any library; q, k, v, caches, tables and `out` still come from the caller.
 *
 *  - Capacity: dlx_static_scratch_bytes() (32 MiB).  A call that would need more (see
 *    dlx_decode_attn_workspace_bytes) returns DLX_ERR_WORKSPACE with a message and launches nothing; lower
 *    num_splits or use dlx_decode_attn.
 *  - The first call on a device looks the array's device address up (with that device current) and keeps
 *    it.  That look-up is also what makes the CUDA runtime load this part of the library, the 32 MiB array
 *    included, on that device, so it is the one call here that can still fail for lack of device memory:
 *    make it at start-up, outside of any stream capture.  From then on the GPU holds the array until the
 *    process exits.  The kept address does not survive a cudaDeviceReset; devices 0..63 are tracked.
 *  - All calls on a device share the one array, which keeps whatever the last call left in it.  Nothing in
 *    it has to start at zero: every entry a call reads was written by that call.  Two calls whose kernels
 *    may overlap on the GPU (different streams, no dependency) race on it; order them.
 */
int64_t dlx_static_scratch_bytes(void);
int dlx_decode_attn_static_scratch(const dlx_decode_attn_params* p, void* stream);

/*
 * Debug aid with no counterpart in the reference.  out[0] bit 0 = a bounded wait inside a tcgen05 kernel
 * expired (every wait there is bounded; the CTA then stops early instead of trapping, and out[1..3] hold
 * the wait site, the tile and the CTA that gave up first).  This call synchronises the device, copies the
 * word to the HOST array `out` and clears it.  out[0] == 0: it did not happen since the last call.
 */
int dlx_debug_device_status(int32_t out[4]);

#ifdef __cplusplus
}
#endif
#endif /* DLX_B200_H */
