// Device-side argument block and launch plans shared by the decode-attention kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace dlx {

struct DecodeArgs {
    const void *q, *k, *v, *k_cache, *v_cache;
    void* out;
    const int32_t *block_tables, *context_lens, *cu_q, *cu_kv;  // cu_kv == nullptr: in-flight rows follow cu_q
    const int32_t* seq_order;  // optional [num_seqs]: sequence handled by grid slot z (longest first balances SMs)
    float* ws_o;    // [num_splits, total_q, Hq, hd] normalised fp32 partial outputs
    float* ws_lse;  // [num_splits, total_q, Hq]     log2-sum-exp of each partial (-inf: nothing seen)
    int64_t q_rs, k_rs, v_rs, o_rs;     // row strides, elements
    int64_t page_stride, token_stride;  // cache strides, elements
    int64_t bt_stride, num_pages;
    int total_q, num_seqs, max_blocks, max_q_len;
    int hq, hkv, group, page_size;
    int mask_mode, dbs;
    int num_splits, m_blocks;
    int tma_box_rows;  // tcgen05 kernel: rows per TMA box (0 = cached tiles are not fetched by TMA)
    int tma_lvl0;      // tcgen05 kernel: level of the largest usable box (rows = 128 >> level)
    int q_tokens;      // tcgen05 kernel: whole tokens per 128-row block (128 / group)
    int q_by_tma;      // tcgen05 kernel: Q blocks are fetched by TMA (else by 16-byte cp.async)
    int items_total;   // tcgen05 kernel: num_seqs * hkv * m_blocks * num_splits work items, walked by persistent CTAs
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

// tcgen05 kernel: head_dim 128, up to 128 query heads per KV head, bf16.
bool tc5_eligible(int group, int head_dim);
int launch_decode_tc5(const DecodeArgs& a, cudaStream_t st);
// Copies out and clears the device status word of the tcgen05 kernel (synchronises the device).
int read_tc5_status(int out[4]);
// Cycle accounting of CTA (0,0,0) of the tcgen05 kernel: copy out (if out != null), clear, and switch on/off.
int tc5_profile(int enable, unsigned long long out[24]);

}  // namespace dlx
