// Device-side schedule of one decode-attention launch of the persistent tcgen05 kernels.
//
// One small kernel turns the per-step metadata (context_lens, cu_seqlens, block tables: what the reference's model
// runner fills on the host, diffulex/strategy/block_diffusion/engine/model_runner.py:125-158) into packed work-item
// records: every (sequence, KV head, query-token block, key-range split) with its lengths and offsets resolved and
// the ids of its last pages attached, assigned to the persistent CTAs (bins) by a longest-processing-time greedy
// over the items sorted by key-tile count.  It runs once per metadata state (all layers of a step share it), on the
// stream, with no host involvement, so a captured step re-plans itself when its static buffers are refilled.
#include "dlx_common.cuh"
#include "decode_attn.cuh"

namespace dlx {

namespace {

constexpr int SORT_MAX = 4096;      // items sorted and placed greedily; larger launches are dealt round-robin
constexpr int SCHED_THREADS = 1024;
constexpr int TILE_N = 128;

struct ItemShape {
    int seq, kvh, mb, split;
    int q0, qn, ctx, kv0, nnew, t0, n, flags, limit;
};

// Everything about work item `item` that follows from the metadata.  flags == 0: the item has no query rows (a
// token block past the end of a short sequence, a padded sequence): it gets no record.
__device__ ItemShape item_shape(const DecodeArgs& a, int item) {
    ItemShape it{};
    const int per_seq = a.hkv * a.m_blocks * a.num_splits;
    it.seq = item / per_seq;
    const int rem = item - it.seq * per_seq;
    const int y = rem / a.num_splits;
    it.split = rem - y * a.num_splits;
    it.kvh = y / a.m_blocks;
    it.mb = y - it.kvh * a.m_blocks;
    if (it.seq >= a.num_seqs) return it;
    it.q0 = a.cu_q[it.seq];
    it.qn = a.cu_q[it.seq + 1] - it.q0;
    if (it.qn <= 0 || it.q0 < 0 || it.q0 + it.qn > a.total_q) return it;
    it.ctx = a.context_lens != nullptr ? max(a.context_lens[it.seq], 0) : 0;
    it.kv0 = it.q0; it.nnew = it.qn;
    if (a.cu_kv != nullptr) {
        it.kv0 = a.cu_kv[it.seq];
        it.nnew = max(a.cu_kv[it.seq + 1] - it.kv0, 0);
    }
    const int tok0 = it.mb * a.tokens_per_item;
    if (tok0 >= it.qn) return it;
    const int tok_last = min(it.qn, tok0 + a.tokens_per_item) - 1;
    it.limit = it.ctx + it.nnew;
    if (a.mask_mode == DLX_MASK_BLOCK_CAUSAL) it.limit = it.ctx + min(it.nnew, (tok_last / a.dbs + 1) * a.dbs);
    const int n_tiles = (it.limit + TILE_N - 1) / TILE_N;
    const int per_split = (n_tiles + a.num_splits - 1) / a.num_splits;
    it.t0 = it.split * per_split;
    const int t1 = min(n_tiles, it.t0 + per_split);
    if (it.t0 >= t1) { it.flags = SCHED_EMPTY_SPLIT; it.n = 0; return it; }
    it.n = t1 - it.t0;
    it.flags = SCHED_VALID;
    return it;
}

__device__ void write_record(const DecodeArgs& a, const ItemShape& it, SchedRec* out) {
    int first_page = 0, n_pages = 0;
    const int32_t* bt = nullptr;
    if ((it.flags & SCHED_VALID) && a.max_blocks > 0 && it.ctx > 0) {
        const int last_key = min((it.t0 + it.n) * TILE_N, it.ctx) - 1;   // last cached key of the range
        if (last_key >= it.t0 * TILE_N) {
            const int last_page = min(last_key / a.page_size, a.max_blocks - 1);
            first_page = max(0, last_page - (kSchedPages - 1));
            n_pages = last_page - first_page + 1;
            bt = a.block_tables + (int64_t)it.seq * a.bt_stride + first_page;
        }
    }
    // four 16-byte stores of scalars, then the page ids four at a time (all loads of a group in flight together)
    int4* dst = reinterpret_cast<int4*>(out);
    dst[0] = make_int4(it.seq, it.kvh, it.mb, it.split);
    dst[1] = make_int4(it.q0, it.qn, it.ctx, it.kv0);
    dst[2] = make_int4(it.nnew, it.t0, it.n, it.flags);
    dst[3] = make_int4(first_page, n_pages, it.limit, 0);
    static_assert(offsetof(SchedRec, pages) == 64 && kSchedPages % 4 == 0, "record layout");
#pragma unroll
    for (int j = 0; j < kSchedPages; j += 4) {
        int4 v;
        v.x = j + 0 < n_pages ? bt[j + 0] : -1;
        v.y = j + 1 < n_pages ? bt[j + 1] : -1;
        v.z = j + 2 < n_pages ? bt[j + 2] : -1;
        v.w = j + 3 < n_pages ? bt[j + 3] : -1;
        dst[4 + j / 4] = v;
    }
}

// cost of an item for the placement: its key tiles plus one tile's worth of per-item overhead
__device__ __forceinline__ uint32_t item_cost(const ItemShape& it) {
    return it.flags == 0 ? 0u : (uint32_t)it.n + 1u;
}

__global__ void __launch_bounds__(SCHED_THREADS) decode_sched_kernel(const DecodeArgs a) {
    // (~cost << 32) | item: ascending = longest first, ties by index.  The placement overwrites the upper half with
    // bin << 16 | position inside the bin.
    __shared__ unsigned long long keys[SORT_MAX];
    __shared__ int offs[kSchedMaxBins + 1];
    __shared__ int n_live_s;   // items with rows
    const int tid = threadIdx.x, lane = tid & 31, nthreads = blockDim.x;
    const int n_items = a.items_total, bins = a.bins;
    int32_t* off_out = const_cast<int32_t*>(a.sched_off);
    SchedRec* recs = const_cast<SchedRec*>(a.sched_recs);

    if (n_items > SORT_MAX) {
        // Too many items to sort in shared memory: deal them round-robin in natural order (every item gets a
        // record, rows or not; kernels skip records without the VALID / EMPTY_SPLIT bits).
        for (int b = tid; b <= bins; b += nthreads) {
            // bin b holds items b, b + bins, ...: offsets are the running counts
            int64_t before = 0;
            if (b > 0) {
                const int full = n_items / bins, extra = n_items % bins;
                before = (int64_t)full * b + min(b, extra);
            }
            off_out[b] = (int)before;
        }
        for (int i = tid; i < n_items; i += nthreads) {
            const int b = i % bins, pos = i / bins;
            const int full = n_items / bins, extra = n_items % bins;
            const int64_t base = (int64_t)full * b + min(b, extra);
            write_record(a, item_shape(a, i), recs + base + pos);
        }
        return;
    }

    int n_pad = 1;
    while (n_pad < n_items) n_pad <<= 1;
    if (tid == 0) n_live_s = 0;
    __syncthreads();
    int live_here = 0;
    for (int i = tid; i < n_pad; i += nthreads) {
        unsigned long long key = ~0ull;
        if (i < n_items) {
            const uint32_t c = item_cost(item_shape(a, i));
            key = ((unsigned long long)(0xffffffffu - c) << 32) | (uint32_t)i;
            live_here += c != 0;
        }
        keys[i] = key;
    }
    live_here = __reduce_add_sync(0xffffffffu, live_here);
    if (lane == 0 && live_here) atomicAdd(&n_live_s, live_here);
    __syncthreads();
    // bitonic sort, ascending
    for (int k = 2; k <= n_pad; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < n_pad; i += nthreads) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long x = keys[i], y = keys[ixj];
                    const bool up = (i & k) == 0;
                    if ((x > y) == up) { keys[i] = y; keys[ixj] = x; }
                }
            }
            __syncthreads();
        }
    }
    // Longest-processing-time greedy by one warp: every lane keeps the loads of bins lane, lane + 32, ... as packed
    // words (load << 8 | bin), so that one warp minimum finds the least loaded bin, lowest index on ties; that bin's
    // lane takes the item.  The first `bins` items meet empty bins: item i goes to bin i, with no search.
    if (tid < 32) {
        static_assert(kSchedMaxBins == 160, "five bins per lane, written out below");
        static_assert(kSchedMaxBins <= 256, "bin index is packed into 8 bits");
        // bins lane, lane + 32, ..., lane + 128 in five scalars each (indexed arrays would live in local memory)
        uint32_t l0, l1, l2, l3, l4, c0 = 0, c1 = 0, c2 = 0, c3 = 0, c4 = 0;
        auto first = [&](int j, uint32_t& l, uint32_t& cnt) {
            const int b = lane + 32 * j;
            l = 0xffffffffu;
            if (b < bins) {
                uint32_t c = 0;
                if (b < n_items) {
                    const unsigned long long key = keys[b];
                    c = 0xffffffffu - (uint32_t)(key >> 32);
                    if (c != 0) { keys[b] = ((unsigned long long)((uint32_t)b << 16) << 32) | (uint32_t)key; cnt = 1; }
                }
                l = (c << 8) | (uint32_t)b;
            }
        };
        first(0, l0, c0); first(1, l1, c1); first(2, l2, c2); first(3, l3, c3); first(4, l4, c4);
        __syncwarp();
        // The rest of the items, several independent greedy placements side by side: bins and lanes fall into `nsets`
        // sets by index modulo nsets (a lane's bins lane, lane + 32, ... all lie in set lane % nsets), and the sorted
        // item i belongs to set (i % bins) % nsets, so that every run of `bins` consecutive items gives each set as
        // many items as it has bins.  A few butterfly exchanges per step give every set its minimum: a step places
        // nsets items (warp exchanges are what a step costs; within 1 % of one global placement for sets of ten
        // bins).  With few bins one set holds them all: the plain greedy placement.
        const int nsets = bins >= 32 ? 8 : bins >= 16 ? 4 : 1;
        const int s4 = lane & (nsets - 1);
        const int n_live = n_live_s;               // the first n_live sorted items have rows
        const int blocks = (n_live + bins - 1) / bins - 1;              // runs of `bins` items after the first
        const int max_steps = blocks > 0 ? blocks * ((bins + nsets - 1) / nsets) : 0;
        int blk = 1, pp = s4;                      // the set's next item is blk * bins + pp
        unsigned long long key = ~0ull;
        if (s4 < bins && bins + pp < n_live) key = keys[bins + pp];
        for (int step = 0; step < max_steps; ++step) {
            const int i = blk * bins + pp;
            const bool active = s4 < bins && i < n_live;
            // the set's least loaded bin (all lanes take part in the exchanges, sets that are done included)
            uint32_t win = min(min(min(l0, l1), min(l2, l3)), l4);
            if (nsets == 1) {
                win = __reduce_min_sync(0xffffffffu, win);
            } else {
                for (int off = nsets; off < 32; off <<= 1) win = min(win, __shfl_xor_sync(0xffffffffu, win, off));
            }
            if (active) {
                const unsigned long long cur = key;
                const uint32_t c = 0xffffffffu - (uint32_t)(cur >> 32);
                int p2 = pp + nsets, blk2 = blk;
                if (p2 >= bins) { p2 = s4; ++blk2; }
                if (blk2 * bins + p2 < n_live) key = keys[blk2 * bins + p2];   // next item's key, off the critical path
                const uint32_t wb = win & 0xffu, sel = wb >> 5;
                const bool mine = (wb & 31u) == (uint32_t)lane;
                const uint32_t inc = mine ? c << 8 : 0u, one = mine ? 1u : 0u;
                const uint32_t pos = sel == 0 ? c0 : sel == 1 ? c1 : sel == 2 ? c2 : sel == 3 ? c3 : c4;
                if (mine) keys[i] = ((unsigned long long)((wb << 16) | pos) << 32) | (uint32_t)cur;
                l0 += sel == 0 ? inc : 0u; c0 += sel == 0 ? one : 0u;
                l1 += sel == 1 ? inc : 0u; c1 += sel == 1 ? one : 0u;
                l2 += sel == 2 ? inc : 0u; c2 += sel == 2 ? one : 0u;
                l3 += sel == 3 ? inc : 0u; c3 += sel == 3 ? one : 0u;
                l4 += sel == 4 ? inc : 0u; c4 += sel == 4 ? one : 0u;
                pp = p2; blk = blk2;
            }
        }
        __syncwarp();
        if (lane < bins) offs[lane + 1] = (int)c0;
        if (lane + 32 < bins) offs[lane + 33] = (int)c1;
        if (lane + 64 < bins) offs[lane + 65] = (int)c2;
        if (lane + 96 < bins) offs[lane + 97] = (int)c3;
        if (lane + 128 < bins) offs[lane + 129] = (int)c4;
        // offsets = exclusive prefix of the counts, in bin order
        __syncwarp();
        if (lane == 0) {
            offs[0] = 0;
            for (int b = 0; b < bins; ++b) offs[b + 1] += offs[b];
        }
        __syncwarp();
    }
    __syncthreads();
    for (int b = tid; b <= bins; b += nthreads) off_out[b] = offs[b];
    const int placed = offs[bins];
    for (int i = tid; i < placed; i += nthreads) {
        const int item = (int)(uint32_t)keys[i];
        const uint32_t pl = (uint32_t)(keys[i] >> 32);
        write_record(a, item_shape(a, item), recs + offs[pl >> 16] + (pl & 0xffffu));
    }
}

}  // namespace

int device_sm_count() {
    static int sm_count[16] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = (dev >= 0 && dev < 16) ? sm_count[dev] : 0;
    if (sms == 0) {
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = kNumSMs;
        if (dev >= 0 && dev < 16) sm_count[dev] = sms;
    }
    return sms;
}

void tc5_plan_items(DecodeArgs& a, bool two_ctas, int sm_count) {
    const bool pair = two_ctas;
    a.group_ctas = two_ctas ? 2 : 1;
    a.q_tokens = 128 / a.group;
    a.tokens_per_item = pair ? 2 * a.q_tokens : a.q_tokens;
    const int q_len = a.max_q_len > (1 << 20) ? (1 << 20) : a.max_q_len;
    a.m_blocks = (q_len + a.tokens_per_item - 1) / a.tokens_per_item;
    const int64_t items = (int64_t)a.num_seqs * a.hkv * a.m_blocks * a.num_splits;
    a.items_total = (int)(items > (1ll << 30) ? (1ll << 30) : items);
    int slots = pair ? sm_count / 2 : sm_count;
    if (slots > kSchedMaxBins) slots = kSchedMaxBins;
    if (slots < 1) slots = 1;
    a.bins = (int)(items < slots ? (items < 1 ? 1 : items) : slots);
}

int launch_decode_sched(const DecodeArgs& a, cudaStream_t st) {
    if (a.sched_off == nullptr || a.sched_recs == nullptr) return fail(DLX_ERR_WORKSPACE, "decode schedule: no buffer");
    if (a.bins < 1 || a.bins > kSchedMaxBins) return fail(DLX_ERR_INVALID_ARGUMENT, "decode schedule: %d bins", a.bins);
    // one block; as many threads as items (a power of two, 128..1024): fewer warps make the sort's barriers cheaper
    int threads = 128;
    while (threads < SCHED_THREADS && threads < a.items_total) threads <<= 1;
    decode_sched_kernel<<<1, threads, 0, st>>>(a);
    return check_launch("decode_sched_kernel");
}

}  // namespace dlx
