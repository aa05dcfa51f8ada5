// Slot-mapped KV-cache store (scatter) and paged KV-cache load (gather) for sm_100a.
//
// Both are pure HBM-bound row copies: a cache row is Hkv*head_dim contiguous elements (1-8 KiB
// in bf16).  One warp moves one row with 16-byte vectors (coalesced: 32 lanes x 16 B = 512 B per
// instruction), K and V rows of the same token in flight together, several independent loads
// issued before the first store.  Offsets are 64-bit throughout.
//
// Reference semantics: diffulex_kernel/python/kv_cache_kernels.py:11-32 (store, unified),
// :35-83 (store, distinct), :127-227 (load).
#include "dlx_common.cuh"

namespace dlx {

template <int BYTES> struct VecOf;
template <> struct VecOf<16> { using type = uint4; };
template <> struct VecOf<8> { using type = uint2; };
template <> struct VecOf<4> { using type = uint32_t; };
template <> struct VecOf<2> { using type = uint16_t; };

// Streaming read: the source row is consumed once.
template <typename V>
__device__ __forceinline__ V ld_stream(const V* p) { return __ldcs(p); }

// One warp copies two rows (K and V of one token / output row) of `nvec` vectors each.
template <typename V>
__device__ __forceinline__ void warp_copy_pair(V* __restrict__ dst_a, const V* __restrict__ src_a,
                                               V* __restrict__ dst_b, const V* __restrict__ src_b, int nvec,
                                               int lane) {
    int i = lane;
    // 2 x 2 loads in flight per lane before the first store
    for (; i + 32 < nvec; i += 64) {
        V a0 = ld_stream(src_a + i), a1 = ld_stream(src_a + i + 32);
        V b0 = ld_stream(src_b + i), b1 = ld_stream(src_b + i + 32);
        dst_a[i] = a0; dst_a[i + 32] = a1;
        dst_b[i] = b0; dst_b[i + 32] = b1;
    }
    for (; i < nvec; i += 32) {
        V a0 = ld_stream(src_a + i);
        V b0 = ld_stream(src_b + i);
        dst_a[i] = a0;
        dst_b[i] = b0;
    }
}

// ---- store, unified layout ------------------------------------------------------------------
template <typename SlotT, int VB>
__global__ void __launch_bounds__(256)
store_unified_kernel(const char* __restrict__ key, int64_t key_row_bytes, const char* __restrict__ value,
                     int64_t value_row_bytes, char* __restrict__ k_cache, char* __restrict__ v_cache,
                     const SlotT* __restrict__ slots, int64_t num_tokens, int64_t row_bytes, int64_t num_slots) {
    using V = typename VecOf<VB>::type;
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int nvec = (int)(row_bytes / VB);
    for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < num_tokens; t += warps) {
        const int64_t slot = (int64_t)slots[t];
        if (slot < 0 || slot >= num_slots) continue;  // negative = row of a still-active block: not cached
        warp_copy_pair<V>(reinterpret_cast<V*>(k_cache + slot * row_bytes),
                          reinterpret_cast<const V*>(key + t * key_row_bytes),
                          reinterpret_cast<V*>(v_cache + slot * row_bytes),
                          reinterpret_cast<const V*>(value + t * value_row_bytes), nvec, lane);
    }
}

static int pick_vec(int64_t row_bytes, std::initializer_list<const void*> ptrs, std::initializer_list<int64_t> strides) {
    for (int vb : {16, 8, 4, 2}) {
        bool ok = row_bytes % vb == 0;
        for (const void* p : ptrs) ok = ok && (reinterpret_cast<uintptr_t>(p) % vb == 0);
        for (int64_t s : strides) ok = ok && (s % vb == 0);
        if (ok) return vb;
    }
    return 0;
}

template <typename SlotT>
static int launch_store_unified(int vb, const char* key, int64_t krb, const char* value, int64_t vrb, char* kc,
                                char* vc, const void* slots, int64_t n, int64_t row_bytes, int64_t num_slots,
                                cudaStream_t st) {
    const int warps_per_cta = 8;
    int64_t ctas = (n + warps_per_cta - 1) / warps_per_cta;
    const int64_t cap = (int64_t)kNumSMs * 16;  // 8 resident CTAs of 256 threads per SM, two waves
    if (ctas > cap) ctas = cap;
    dim3 grid((unsigned)ctas), block(32 * warps_per_cta);
    const SlotT* s = static_cast<const SlotT*>(slots);
    switch (vb) {
        case 16: store_unified_kernel<SlotT, 16><<<grid, block, 0, st>>>(key, krb, value, vrb, kc, vc, s, n, row_bytes, num_slots); break;
        case 8: store_unified_kernel<SlotT, 8><<<grid, block, 0, st>>>(key, krb, value, vrb, kc, vc, s, n, row_bytes, num_slots); break;
        case 4: store_unified_kernel<SlotT, 4><<<grid, block, 0, st>>>(key, krb, value, vrb, kc, vc, s, n, row_bytes, num_slots); break;
        default: store_unified_kernel<SlotT, 2><<<grid, block, 0, st>>>(key, krb, value, vrb, kc, vc, s, n, row_bytes, num_slots); break;
    }
    return check_launch("store_unified_kernel");
}

// ---- store, distinct layout -----------------------------------------------------------------
// K cache [NB, H, hd/x, PAGE, x]: x contiguous elements per (head, dx, token).  V cache
// [NB, H, hd, PAGE]: one element per (head, d, token).  One CTA per token; each thread moves one
// x-element group of K and x single elements of V.
template <typename SlotT, typename E>
__global__ void __launch_bounds__(256)
store_distinct_kernel(const E* __restrict__ key, int64_t key_row_stride, const E* __restrict__ value,
                      int64_t value_row_stride, E* __restrict__ k_cache, E* __restrict__ v_cache,
                      const SlotT* __restrict__ slots, int64_t num_tokens, int heads, int hd, int page, int x,
                      int64_t num_pages) {
    const int64_t t = blockIdx.x;
    const int64_t slot = (int64_t)slots[t];
    if (slot < 0 || slot >= num_pages * page) return;
    const int64_t b = slot / page;
    const int off = (int)(slot % page);
    const int groups = heads * hd / x;
    const E* krow = key + t * key_row_stride;
    const E* vrow = value + t * value_row_stride;
    for (int g = threadIdx.x; g < groups; g += blockDim.x) {
        const int h = (g * x) / hd;
        const int dx = ((g * x) % hd) / x;
        E* kd = k_cache + ((((b * heads + h) * (hd / x) + dx) * page + off) * (int64_t)x);
        E* vd = v_cache + (((b * heads + h) * hd + (int64_t)dx * x) * page + off);
        for (int e = 0; e < x; ++e) {
            kd[e] = krow[g * x + e];
            vd[(int64_t)e * page] = vrow[g * x + e];
        }
    }
}

// Fast form for x = 8 two-byte elements (one 16-byte vector per (head, dx, token)) and 16-byte aligned rows: a CTA
// takes 32 consecutive tokens and walks the row in chunks of 512 elements through shared memory.  Lanes are TOKENS:
// for a fixed (head, dx) the K vectors of tokens that sit in consecutive slots of one page are 32 x 16 contiguous
// bytes, and for a fixed (head, d) their V elements are 32 x 2 contiguous bytes, so a block of tokens stored to
// consecutive slots leaves as whole lines instead of 2-byte pieces strided by the page size.
constexpr int kDistTokens = 32, kDistChunk = 512;
template <typename SlotT>
__global__ void __launch_bounds__(256)
store_distinct_x8_kernel(const uint16_t* __restrict__ key, int64_t key_row_stride, const uint16_t* __restrict__ value,
                         int64_t value_row_stride, uint16_t* __restrict__ k_cache, uint16_t* __restrict__ v_cache,
                         const SlotT* __restrict__ slots, int64_t num_tokens, int heads, int hd, int page,
                         int64_t num_pages) {
    constexpr int KROW = kDistChunk * 2 + 16;   // bytes per token in the K tile: vectors stay aligned, quarter-warps conflict-free
    constexpr int VROW = kDistChunk * 2 + 4;    // bytes per token in the V tile: an odd number of words, columns conflict-free
    __shared__ __align__(16) unsigned char tile[kDistTokens * KROW];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t t0 = (int64_t)blockIdx.x * kDistTokens;
    const int D = heads * hd;
    // this lane's token
    const int64_t t = t0 + lane;
    int64_t slot = -1;
    if (t < num_tokens) slot = (int64_t)slots[t];
    const bool live = slot >= 0 && slot < num_pages * page;
    const int64_t b = live ? slot / page : 0;
    const int off = live ? (int)(slot - b * page) : 0;
    for (int c0 = 0; c0 < D; c0 += kDistChunk) {
        const int cw = min(kDistChunk, D - c0);           // elements of this chunk (a multiple of 8)
        // ---- K: rows -> shared (16-byte vectors, coalesced), then one vector per (token, head, dx) ----
        __syncthreads();
        for (int i = tid; i < kDistTokens * (cw >> 3); i += 256) {
            const int r = i / (cw >> 3), v = i - r * (cw >> 3);
            uint4 x = make_uint4(0, 0, 0, 0);
            if (t0 + r < num_tokens) x = *reinterpret_cast<const uint4*>(key + (t0 + r) * key_row_stride + c0 + v * 8);
            *reinterpret_cast<uint4*>(tile + r * KROW + v * 16) = x;
        }
        __syncthreads();
        if (live)
            for (int g = warp; g < (cw >> 3); g += 8) {
                const int e = c0 + g * 8, h = e / hd, dx = (e - h * hd) >> 3;
                const uint4 x = *reinterpret_cast<const uint4*>(tile + lane * KROW + g * 16);
                *reinterpret_cast<uint4*>(k_cache + ((((b * heads + h) * (hd >> 3) + dx) * page + off) << 3)) = x;
            }
        // ---- V: rows -> shared (4-byte words), then one element per (token, head, d) ----
        __syncthreads();
        for (int i = tid; i < kDistTokens * (cw >> 1); i += 256) {
            const int r = i / (cw >> 1), v = i - r * (cw >> 1);
            uint32_t x = 0;
            if (t0 + r < num_tokens) x = *reinterpret_cast<const uint32_t*>(value + (t0 + r) * value_row_stride + c0 + v * 2);
            *reinterpret_cast<uint32_t*>(tile + r * VROW + v * 4) = x;
        }
        __syncthreads();
        if (live)
            for (int c = warp; c < cw; c += 8) {
                const int e = c0 + c, h = e / hd, d = e - h * hd;
                v_cache[((b * heads + h) * hd + d) * page + off] = *reinterpret_cast<const uint16_t*>(tile + lane * VROW + c * 2);
            }
    }
}

// ---- load (gather) --------------------------------------------------------------------------
// A CTA owns ROWS consecutive output rows.  The first ROWS threads resolve, per row, the owning
// sequence (binary search in cu_seqlens_k) and the source row (cache page through the block table,
// or an in-flight row); then each warp streams whole rows.  Work is uniform per output row, so
// ragged sequence lengths cost nothing.
constexpr int kLoadRows = 64;

template <int VB>
__global__ void __launch_bounds__(256)
load_kvcache_kernel(const char* __restrict__ k_cache, const char* __restrict__ v_cache, int64_t page_bytes,
                    int64_t token_bytes, const char* __restrict__ k_new, int64_t k_new_row_bytes,
                    const char* __restrict__ v_new, int64_t v_new_row_bytes, const int32_t* __restrict__ block_tables,
                    int64_t bt_stride, int max_blocks, const int32_t* __restrict__ context_lens,
                    const int32_t* __restrict__ seq_lens, const int32_t* __restrict__ cu_q,
                    const int32_t* __restrict__ cu_k, char* __restrict__ k_out, char* __restrict__ v_out,
                    int64_t out_rows, int num_seqs, int page_size, int64_t num_pages, int64_t row_bytes) {
    using V = typename VecOf<VB>::type;
    __shared__ const char* src_k[kLoadRows];
    __shared__ const char* src_v[kLoadRows];
    const int nvec = (int)(row_bytes / VB);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int64_t total = min((int64_t)cu_k[num_seqs], out_rows);
    for (int64_t base = (int64_t)blockIdx.x * kLoadRows; base < total; base += (int64_t)gridDim.x * kLoadRows) {
        if (threadIdx.x < kLoadRows) {
            const int64_t r = base + threadIdx.x;
            const char *sk = nullptr, *sv = nullptr;
            if (r < total) {
                int lo = 0, hi = num_seqs;  // largest s with cu_k[s] <= r
                while (hi - lo > 1) {
                    const int mid = (lo + hi) >> 1;
                    if ((int64_t)cu_k[mid] <= r) lo = mid; else hi = mid;
                }
                const int s = lo;
                const int64_t p = r - cu_k[s];
                const int ctx = context_lens[s];
                if (p < ctx) {
                    const int j = (int)(p / page_size);
                    const int64_t pid = j < max_blocks ? (int64_t)block_tables[s * bt_stride + j] : -1;
                    if (pid >= 0 && pid < num_pages) {
                        const int64_t o = pid * page_bytes + (p - (int64_t)j * page_size) * token_bytes;
                        sk = k_cache + o;
                        sv = v_cache + o;
                    }
                } else if (p - ctx < seq_lens[s]) {
                    const int64_t n = (int64_t)cu_q[s] + (p - ctx);
                    sk = k_new + n * k_new_row_bytes;
                    sv = v_new + n * v_new_row_bytes;
                }
            }
            src_k[threadIdx.x] = sk;
            src_v[threadIdx.x] = sv;
        }
        __syncthreads();
        for (int i = warp; i < kLoadRows; i += nwarps) {
            const char* sk = src_k[i];
            if (sk == nullptr) continue;
            const int64_t r = base + i;
            warp_copy_pair<V>(reinterpret_cast<V*>(k_out + r * row_bytes), reinterpret_cast<const V*>(sk),
                              reinterpret_cast<V*>(v_out + r * row_bytes), reinterpret_cast<const V*>(src_v[i]), nvec,
                              lane);
        }
        __syncthreads();
    }
}

}  // namespace dlx

using namespace dlx;

extern "C" int dlx_store_kvcache_unified(const void* key, int64_t key_row_stride, const void* value,
                                         int64_t value_row_stride, void* k_cache, void* v_cache,
                                         const void* slot_mapping, int slot_is_int64, int64_t num_tokens,
                                         int64_t row_elems, int elem_bytes, int64_t num_slots, void* stream) {
    if (num_tokens < 0 || row_elems <= 0 || elem_bytes <= 0 || num_slots < 0)
        return fail(DLX_ERR_INVALID_ARGUMENT, "store: negative or zero size (tokens=%lld row_elems=%lld)",
                    (long long)num_tokens, (long long)row_elems);
    if (num_tokens == 0) return DLX_OK;
    if (!key || !value || !k_cache || !v_cache || !slot_mapping)
        return fail(DLX_ERR_INVALID_ARGUMENT, "store: null pointer");
    if (key_row_stride < row_elems || value_row_stride < row_elems)
        return fail(DLX_ERR_INVALID_ARGUMENT, "store: key/value row stride smaller than a row");
    const int64_t rb = row_elems * elem_bytes;
    const int64_t krb = key_row_stride * elem_bytes, vrb = value_row_stride * elem_bytes;
    const int vb = pick_vec(rb, {key, value, k_cache, v_cache}, {krb, vrb});
    if (vb == 0) return fail(DLX_ERR_ALIGNMENT, "store: rows are not even 2-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (slot_is_int64)
        return launch_store_unified<int64_t>(vb, (const char*)key, krb, (const char*)value, vrb, (char*)k_cache,
                                             (char*)v_cache, slot_mapping, num_tokens, rb, num_slots, st);
    return launch_store_unified<int32_t>(vb, (const char*)key, krb, (const char*)value, vrb, (char*)k_cache,
                                         (char*)v_cache, slot_mapping, num_tokens, rb, num_slots, st);
}

extern "C" int dlx_store_kvcache_distinct(const void* key, int64_t key_row_stride, const void* value,
                                          int64_t value_row_stride, void* k_cache, void* v_cache,
                                          const void* slot_mapping, int slot_is_int64, int64_t num_tokens,
                                          int32_t num_kv_heads, int32_t head_dim, int32_t page_size, int32_t x,
                                          int64_t num_pages, int elem_bytes, void* stream) {
    if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || page_size <= 0 || x <= 0 || num_pages < 0)
        return fail(DLX_ERR_INVALID_ARGUMENT, "store_distinct: negative or zero size");
    if (head_dim % x != 0) return fail(DLX_ERR_INVALID_ARGUMENT, "store_distinct: head_dim %% x != 0");
    if (elem_bytes != 2) return fail(DLX_ERR_UNSUPPORTED, "store_distinct: only 2-byte elements");
    if (num_tokens == 0) return DLX_OK;
    if (!key || !value || !k_cache || !v_cache || !slot_mapping)
        return fail(DLX_ERR_INVALID_ARGUMENT, "store_distinct: null pointer");
    if (num_tokens > 0x7fffffffLL) return fail(DLX_ERR_UNSUPPORTED, "store_distinct: more than 2^31-1 tokens");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    using E = uint16_t;
    if (x == 8 && aligned16(key) && aligned16(value) && aligned16(k_cache) && key_row_stride % 8 == 0 &&
        value_row_stride % 8 == 0) {
        dim3 grid((unsigned)((num_tokens + kDistTokens - 1) / kDistTokens)), block(256);
        if (slot_is_int64)
            store_distinct_x8_kernel<int64_t><<<grid, block, 0, st>>>(
                (const E*)key, key_row_stride, (const E*)value, value_row_stride, (E*)k_cache, (E*)v_cache,
                (const int64_t*)slot_mapping, num_tokens, num_kv_heads, head_dim, page_size, num_pages);
        else
            store_distinct_x8_kernel<int32_t><<<grid, block, 0, st>>>(
                (const E*)key, key_row_stride, (const E*)value, value_row_stride, (E*)k_cache, (E*)v_cache,
                (const int32_t*)slot_mapping, num_tokens, num_kv_heads, head_dim, page_size, num_pages);
        return check_launch("store_distinct_x8_kernel");
    }
    dim3 grid((unsigned)num_tokens), block(128);
    if (slot_is_int64)
        store_distinct_kernel<int64_t, E><<<grid, block, 0, st>>>(
            (const E*)key, key_row_stride, (const E*)value, value_row_stride, (E*)k_cache, (E*)v_cache,
            (const int64_t*)slot_mapping, num_tokens, num_kv_heads, head_dim, page_size, x, num_pages);
    else
        store_distinct_kernel<int32_t, E><<<grid, block, 0, st>>>(
            (const E*)key, key_row_stride, (const E*)value, value_row_stride, (E*)k_cache, (E*)v_cache,
            (const int32_t*)slot_mapping, num_tokens, num_kv_heads, head_dim, page_size, x, num_pages);
    return check_launch("store_distinct_kernel");
}

extern "C" int dlx_load_kvcache(const void* k_cache, const void* v_cache, int64_t cache_page_stride,
                                int64_t cache_token_stride, const void* k_new, int64_t k_new_row_stride,
                                const void* v_new, int64_t v_new_row_stride, const int32_t* block_tables,
                                int64_t block_table_stride, int32_t max_blocks, const int32_t* context_lens,
                                const int32_t* seq_lens, const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                                void* k_out, void* v_out, int64_t out_rows, int32_t num_seqs, int32_t page_size,
                                int64_t num_pages, int64_t row_elems, int elem_bytes, void* stream) {
    if (num_seqs < 0 || out_rows < 0 || page_size <= 0 || row_elems <= 0 || elem_bytes <= 0 || max_blocks < 0 ||
        num_pages < 0)
        return fail(DLX_ERR_INVALID_ARGUMENT, "load: negative or zero size");
    if (num_seqs == 0 || out_rows == 0) return DLX_OK;
    if (!k_cache || !v_cache || !block_tables || !context_lens || !seq_lens || !cu_seqlens_q || !cu_seqlens_k ||
        !k_out || !v_out)
        return fail(DLX_ERR_INVALID_ARGUMENT, "load: null pointer");
    if (!k_new || !v_new) return fail(DLX_ERR_INVALID_ARGUMENT, "load: null in-flight K/V");
    if (cache_token_stride < row_elems || k_new_row_stride < row_elems || v_new_row_stride < row_elems)
        return fail(DLX_ERR_INVALID_ARGUMENT, "load: a row stride is smaller than a row");
    const int64_t rb = row_elems * elem_bytes;
    const int64_t pb = cache_page_stride * elem_bytes, tb = cache_token_stride * elem_bytes;
    const int64_t knb = k_new_row_stride * elem_bytes, vnb = v_new_row_stride * elem_bytes;
    const int vb = pick_vec(rb, {k_cache, v_cache, k_new, v_new, k_out, v_out}, {pb, tb, knb, vnb});
    if (vb == 0) return fail(DLX_ERR_ALIGNMENT, "load: rows are not even 2-byte aligned");
    int64_t ctas = (out_rows + kLoadRows - 1) / kLoadRows;
    const int64_t cap = (int64_t)kNumSMs * 32;
    if (ctas > cap) ctas = cap;
    dim3 grid((unsigned)ctas), block(256);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
#define DLX_LOAD_ARGS                                                                                              \
    (const char*)k_cache, (const char*)v_cache, pb, tb, (const char*)k_new, knb, (const char*)v_new, vnb,         \
        block_tables, block_table_stride, max_blocks, context_lens, seq_lens, cu_seqlens_q, cu_seqlens_k,         \
        (char*)k_out, (char*)v_out, out_rows, num_seqs, page_size, num_pages, rb
    switch (vb) {
        case 16: load_kvcache_kernel<16><<<grid, block, 0, st>>>(DLX_LOAD_ARGS); break;
        case 8: load_kvcache_kernel<8><<<grid, block, 0, st>>>(DLX_LOAD_ARGS); break;
        case 4: load_kvcache_kernel<4><<<grid, block, 0, st>>>(DLX_LOAD_ARGS); break;
        default: load_kvcache_kernel<2><<<grid, block, 0, st>>>(DLX_LOAD_ARGS); break;
    }
#undef DLX_LOAD_ARGS
    return check_launch("load_kvcache_kernel");
}

// ---- slot mapping of a decode step, built on the device ----------------------------------------
// Row t of the step's in-flight K / V belongs to sequence s (cu_seqlens_q[s] <= t < cu_seqlens_q[s + 1]) and sits at
// position ctx_s + (t - cu_seqlens_q[s]) of it; its cache slot is page_table[s][pos / PAGE] * PAGE + pos % PAGE.
// Sequences whose block is still being denoised store nothing (-1), as do positions without a page.
namespace dlx {
__global__ void __launch_bounds__(256) build_slot_mapping_kernel(
    const int32_t* __restrict__ block_tables, int64_t bt_stride, int max_blocks, const int32_t* __restrict__ context_lens,
    const int32_t* __restrict__ cu_q, const int32_t* __restrict__ store_flags, int num_seqs, int page_size,
    int64_t total_rows, int32_t* __restrict__ slots32, int64_t* __restrict__ slots64) {
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total_rows; t += (int64_t)gridDim.x * blockDim.x) {
        // The sequence that owns row t: binary search over the offsets.  A captured step's static buffers are
        // zero-filled behind the live sequences (model_runner.py:183-186), so the offsets are not monotone there: when
        // the search ends on a sequence that does not hold t, every sequence is tried in turn.
        int lo = 0, hi = num_seqs;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if ((int64_t)cu_q[mid] <= t) lo = mid; else hi = mid;
        }
        int64_t q0 = cu_q[lo], q1 = cu_q[lo + 1];
        if (!(t >= q0 && t < q1)) {
            for (int s = 0; s < num_seqs; ++s) {
                const int64_t a0 = cu_q[s], a1 = cu_q[s + 1];
                if (t >= a0 && t < a1) { lo = s; q0 = a0; q1 = a1; break; }
            }
        }
        int64_t slot = -1;
        if (t >= q0 && t < q1 && (store_flags == nullptr || store_flags[lo] != 0)) {
            const int64_t pos = (int64_t)max(context_lens[lo], 0) + (t - q0);
            const int64_t j = pos / page_size;
            if (j < max_blocks) {
                const int32_t pid = block_tables[(int64_t)lo * bt_stride + j];
                if (pid >= 0) slot = (int64_t)pid * page_size + (pos - j * page_size);
            }
        }
        if (slots32 != nullptr) slots32[t] = (int32_t)slot; else slots64[t] = slot;
    }
}
}  // namespace dlx

extern "C" int dlx_build_slot_mapping(const int32_t* block_tables, int64_t block_table_stride, int32_t max_blocks,
                                      const int32_t* context_lens, const int32_t* cu_seqlens_q,
                                      const int32_t* store_flags, int32_t num_seqs, int32_t page_size,
                                      int64_t total_rows, int64_t num_pages, void* slot_mapping, int slots_are_int64,
                                      void* stream) {
    using namespace dlx;
    if (num_seqs < 0 || total_rows < 0 || page_size <= 0 || max_blocks < 0 || num_pages < 0)
        return fail(DLX_ERR_INVALID_ARGUMENT, "slot mapping: negative or zero size");
    if (total_rows == 0) return DLX_OK;
    if (!slot_mapping || !cu_seqlens_q || !context_lens || (max_blocks > 0 && !block_tables))
        return fail(DLX_ERR_INVALID_ARGUMENT, "slot mapping: null pointer");
    if (num_seqs == 0) return fail(DLX_ERR_INVALID_ARGUMENT, "slot mapping: rows without sequences");
    if (!slots_are_int64 && num_pages * (int64_t)page_size > 0x7fffffffll)
        return fail(DLX_ERR_UNSUPPORTED, "slot mapping: %lld slots do not fit int32", (long long)(num_pages * page_size));
    int64_t ctas = (total_rows + 255) / 256;
    if (ctas > (int64_t)kNumSMs * 8) ctas = (int64_t)kNumSMs * 8;
    build_slot_mapping_kernel<<<(unsigned)ctas, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        block_tables, block_table_stride, max_blocks, context_lens, cu_seqlens_q, store_flags, num_seqs, page_size,
        total_rows, slots_are_int64 ? nullptr : static_cast<int32_t*>(slot_mapping),
        slots_are_int64 ? static_cast<int64_t*>(slot_mapping) : nullptr);
    return check_launch("build_slot_mapping_kernel");
}
