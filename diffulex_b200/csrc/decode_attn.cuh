// Device-side argument block and launch plans shared by the decode-attention kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace dlx {

// One record of a decode schedule: a (sequence, KV head, block of query tokens, key-range split) work item with every
// length and offset a kernel needs already resolved, plus the ids of the last pages of its key range (tiles are
// walked from the end of the range towards its start, so these are the first ids a kernel asks for).  Written by
// decode_sched_kernel once per metadata state, read by the persistent tcgen05 kernels.  128 bytes.
struct alignas(16) SchedRec {
    int32_t seq, kvh, mb, split;
    int32_t q0, qn, ctx, kv0;      // first query row and query tokens of the sequence; cached tokens; first in-flight row
    int32_t nnew, t0, n, flags;    // in-flight tokens; first 128-key tile and tile count of this split; SCHED_* bits
    int32_t first_page, n_pages;   // pages[j] is the id of page first_page + j of the sequence, j < n_pages
    int32_t limit, reserved;       // keys [0, limit) are visible to at least one row of the item
    int32_t pages[16];
};
static_assert(sizeof(SchedRec) == 128, "schedule record size");
enum { SCHED_VALID = 1, SCHED_EMPTY_SPLIT = 2 };
constexpr int kSchedPages = 16;
constexpr int kSchedMaxBins = 160;

// A schedule buffer: int32 offsets[bins + 1] (records of bin b are recs[offsets[b] .. offsets[b + 1])), padded to
// 1 KiB, then the records.  `bins` is the number of persistent CTAs (or CTA pairs) of the kernel it is made for.
constexpr int64_t kSchedHeaderBytes = 1024;
inline int64_t sched_bytes(int64_t items) { return kSchedHeaderBytes + items * (int64_t)sizeof(SchedRec); }

struct DecodeArgs {
    const void *q, *k, *v, *k_cache, *v_cache;
    void* out;
    const int32_t *block_tables, *context_lens, *cu_q, *cu_kv;  // cu_kv == nullptr: in-flight rows follow cu_q
    const int32_t* sched_off;     // tcgen05 kernels: offsets[bins + 1] of the schedule
    const SchedRec* sched_recs;   // tcgen05 kernels: records of the schedule
    float* ws_o;    // [num_splits, total_q, Hq, hd] normalised fp32 partial outputs
    float* ws_lse;  // [num_splits, total_q, Hq]     log2-sum-exp of each partial (-inf: nothing seen)
    int64_t q_rs, k_rs, v_rs, o_rs;     // row strides, elements
    int64_t page_stride, token_stride;  // cache strides, elements
    int64_t bt_stride, num_pages;
    int total_q, num_seqs, max_blocks, max_q_len;
    int total_kv;   // rows of k / v
    int hq, hkv, group, page_size;
    int mask_mode, dbs;
    int num_splits, m_blocks;
    int tma_box_rows;  // tcgen05 kernel: rows per TMA box (0 = cached tiles are not fetched by TMA)
    int tma_lvl0;      // tcgen05 kernel: level of the largest usable box (rows = 128 >> level)
    int q_tokens;      // tcgen05 kernel: whole tokens per 128-row block (128 / group)
    int q_by_tma;      // tcgen05 kernel: Q blocks are fetched by TMA (else by 16-byte cp.async)
    int items_total;   // tcgen05 kernels: num_seqs * hkv * m_blocks * num_splits work items, walked by persistent CTAs
    int bins;          // tcgen05 kernels: persistent CTAs (single-CTA kernel) or CTA pairs (pair kernel) of the launch
    int tokens_per_item;  // tcgen05 kernels: query tokens of one work item (two blocks of q_tokens when two CTAs share an item)
    int group_ctas;       // tcgen05 kernels: CTAs that work on the same schedule bin (1, or 2: each takes one block of q_tokens)
    float scale_log2;  // softmax scale * log2(e)
};

// Tile plan of the mma.sync kernel for `rows` = G * max_q_len packed query rows.
struct MmaPlan {
    int id;
    int block_m, block_n;
    int m_blocks;
    int ctas_per_sm;
};
MmaPlan plan_mma(int rows, int head_dim);
int launch_decode_mma(const DecodeArgs& a, const MmaPlan& plan, int head_dim, cudaStream_t st);
int launch_combine(const DecodeArgs& a, int head_dim, cudaStream_t st);

// tcgen05 kernels: head_dim 128, up to 128 query heads per KV head, bf16.  The pair kernel runs an item of up to
// 2 x 128 packed rows on two CTAs of a cluster (tcgen05 cta_group::2), each fetching half of every K / V tile.
bool tc5_eligible(int group, int head_dim);
int launch_decode_tc5(const DecodeArgs& a, cudaStream_t st);
int launch_decode_tc5_pair(const DecodeArgs& a, cudaStream_t st);
// Fills a.bins / a.tokens_per_item / a.group_ctas / a.m_blocks / a.items_total for the chosen tcgen05 kernel.  `two_ctas`:
// an item is 2 x (128 / group) query tokens taken by two CTAs (the CTA-pair kernel, or two neighbouring CTAs of the
// single-CTA kernel that walk the same record list, so that the second reader of a K / V tile finds it in L2).
void tc5_plan_items(DecodeArgs& a, bool two_ctas, int sm_count);
// Builds the schedule of a launch (a.sched_off / a.sched_recs must point into a buffer of sched_bytes(a.items_total)).
int launch_decode_sched(const DecodeArgs& a, cudaStream_t st);
int device_sm_count();
// Copy out and clear the device status word of the single-CTA / CTA-pair tcgen05 kernel (synchronises the device).
int read_tc5_status(int out[4]);
int read_tc5_pair_status(int out[4]);

}  // namespace dlx
