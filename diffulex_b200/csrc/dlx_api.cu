// C-ABI entry points that are not tied to one kernel file: version / errors, and the planning and
// validation front of dlx_decode_attn (include/dlx_b200.h).
#include <math.h>
#include <string.h>

#include "dlx_common.cuh"
#include "decode_attn.cuh"

namespace dlx {

char* last_error_buffer() {
    static thread_local char buf[512] = {0};
    return buf;
}

struct DecodePlan {
    MmaPlan mma;
    bool use_tc5;    // one of the persistent tcgen05 kernels
    bool use_pair;   // ... the CTA-pair kernel
    int num_splits;
    int64_t ws_o_bytes, ws_lse_bytes, sched_bytes;
    DecodeArgs args; // sizes, strides and pointers of the call; split / schedule pointers are set by the caller
};

static int validate_decode(const dlx_decode_attn_params* p) {
    if (p == nullptr) return fail(DLX_ERR_INVALID_ARGUMENT, "decode: null params");
    if (p->struct_bytes != sizeof(dlx_decode_attn_params))
        return fail(DLX_ERR_INVALID_ARGUMENT, "decode: struct_bytes %u != %zu (header mismatch)", p->struct_bytes,
                    sizeof(dlx_decode_attn_params));
    if (p->dtype != DLX_DTYPE_BF16) return fail(DLX_ERR_UNSUPPORTED, "decode: only bf16 is built");
    if (p->head_dim != 64 && p->head_dim != 128)
        return fail(DLX_ERR_UNSUPPORTED, "decode: head_dim %d (64 and 128 are built)", p->head_dim);
    if (p->num_seqs < 0 || p->total_q < 0 || p->total_kv < 0 || p->max_blocks < 0 || p->num_pages < 0)
        return fail(DLX_ERR_INVALID_ARGUMENT, "decode: negative count");
    if (p->num_q_heads <= 0 || p->num_kv_heads <= 0 || p->num_q_heads % p->num_kv_heads != 0)
        return fail(DLX_ERR_INVALID_ARGUMENT, "decode: %d query heads over %d KV heads", p->num_q_heads,
                    p->num_kv_heads);
    if (p->page_size <= 0 || p->max_q_len <= 0)
        return fail(DLX_ERR_INVALID_ARGUMENT, "decode: page_size %d, max_q_len %d", p->page_size, p->max_q_len);
    if (p->mask_mode != DLX_MASK_FULL && p->mask_mode != DLX_MASK_BLOCK_CAUSAL)
        return fail(DLX_ERR_INVALID_ARGUMENT, "decode: mask_mode %d", p->mask_mode);
    if (p->mask_mode == DLX_MASK_BLOCK_CAUSAL && p->diffusion_block_size <= 0)
        return fail(DLX_ERR_INVALID_ARGUMENT, "decode: block-causal mask needs diffusion_block_size > 0");
    if (p->num_splits < 0 || p->num_splits > 256) return fail(DLX_ERR_INVALID_ARGUMENT, "decode: num_splits %d", p->num_splits);
    if (!(p->scale > 0.f) || !isfinite(p->scale)) return fail(DLX_ERR_INVALID_ARGUMENT, "decode: scale must be positive and finite");
    if (p->kernel < 0 || p->kernel > 3) return fail(DLX_ERR_INVALID_ARGUMENT, "decode: kernel %d", p->kernel);
    if (p->kernel >= 2 && !tc5_eligible(p->num_q_heads / p->num_kv_heads, p->head_dim))
        return fail(DLX_ERR_UNSUPPORTED, "decode: the tcgen05 kernels serve head_dim 128 with up to 128 query heads per KV head");
    if (p->num_seqs > 65535) return fail(DLX_ERR_UNSUPPORTED, "decode: more than 65535 sequences per call");
    return DLX_OK;
}

// The tcgen05 kernels fetch every tile by TMA: page sizes that tile into boxes of 8..128 rows, 16-byte strides below
// 2^40 bytes.  Without a cache (max_blocks == 0) only q / k / v count.
static bool tma_supported(const dlx_decode_attn_params* p) {
    const int ps = p->page_size;
    const bool fits = p->num_pages > 0 && ps > 0 && ((ps % 128 == 0) || (128 % ps == 0 && ps % 8 == 0));
    const bool strides_ok = p->cache_token_stride * 2 % 16 == 0 && p->cache_page_stride * 2 % 16 == 0 &&
                            p->cache_page_stride * 2 < (1ll << 40) && p->num_pages < (1ll << 31);
    const bool rows_ok = p->q_row_stride * 2 % 16 == 0 && p->q_row_stride * 2 < (1ll << 40) &&
                         p->k_row_stride * 2 % 16 == 0 && p->k_row_stride * 2 < (1ll << 40) &&
                         p->v_row_stride * 2 % 16 == 0 && p->v_row_stride * 2 < (1ll << 40);
    return (p->max_blocks == 0 || (fits && strides_ok)) && p->total_q > 0 && rows_ok;
}

static DecodePlan plan_decode(const dlx_decode_attn_params* p) {
    DecodePlan d{};
    DecodeArgs& a = d.args;
    a.q = p->q; a.k = p->k; a.v = p->v; a.k_cache = p->k_cache; a.v_cache = p->v_cache; a.out = p->out;
    a.block_tables = p->block_tables;
    a.context_lens = p->max_blocks > 0 ? p->context_lens : nullptr;   // no cache: every context is empty
    a.cu_q = p->cu_seqlens_q; a.cu_kv = p->cu_seqlens_kv;
    a.q_rs = p->q_row_stride; a.k_rs = p->k_row_stride; a.v_rs = p->v_row_stride; a.o_rs = p->out_row_stride;
    a.page_stride = p->cache_page_stride; a.token_stride = p->cache_token_stride;
    a.bt_stride = p->block_table_stride; a.num_pages = p->num_pages;
    a.total_kv = p->total_kv > 0 ? p->total_kv : p->total_q;
    a.total_q = p->total_q; a.num_seqs = p->num_seqs; a.max_blocks = p->max_blocks; a.max_q_len = p->max_q_len;
    a.hq = p->num_q_heads; a.hkv = p->num_kv_heads; a.group = a.hq / a.hkv; a.page_size = p->page_size;
    a.mask_mode = p->mask_mode; a.dbs = p->diffusion_block_size > 0 ? p->diffusion_block_size : 1;
    a.scale_log2 = p->scale * 1.4426950408889634f;

    const int group = a.group;
    const int64_t rows = (int64_t)group * p->max_q_len;
    d.mma = plan_mma((int)(rows > 1 << 20 ? 1 << 20 : rows), p->head_dim);
    d.use_tc5 = p->kernel != 1 && tc5_eligible(group, p->head_dim) && tma_supported(p);
    // More than 128 packed rows per (sequence, KV head): an item is two row blocks on two CTAs.  The CTA-pair kernel
    // (cta_group::2: each CTA fetches half of every K / V tile) is taken on request only: measured, both kernels spend
    // the same time per key tile (the hand-offs between the tensor pipe and the softmax warps bound it, not the
    // L2 -> SM traffic the pair halves), and the pair pays for its cross-CTA signalling.
    d.use_pair = d.use_tc5 && p->kernel == 3 && p->max_blocks > 0;
    const bool two_ctas = d.use_pair || rows > 128;
    const int sms = kNumSMs;
    if (d.use_tc5) {  // persistent CTAs (or CTA pairs) over 128-key tiles
        a.num_splits = 1;
        tc5_plan_items(a, two_ctas, sms);
        d.mma.block_m = two_ctas ? 256 : 128; d.mma.block_n = 128; d.mma.ctas_per_sm = 1;
        d.mma.m_blocks = a.m_blocks;
    }
    const int64_t max_len = p->max_kv_len > 0 ? p->max_kv_len : (int64_t)p->max_blocks * p->page_size + p->max_q_len;
    const int64_t max_tiles = (max_len + d.mma.block_n - 1) / d.mma.block_n;
    int splits = p->num_splits;
    if (splits == 0) {
        // (1) fill the machine when there are fewer work items than resident slots; (2) cut very long
        // contexts so ragged batches balance.  A split costs one fp32 partial (write + read) of
        // block_m x hd per item, i.e. 2*M/chunk of the chunk's KV bytes: keep chunks >= 40*M keys.
        const int64_t units = (int64_t)p->num_seqs * p->num_kv_heads * d.mma.m_blocks;
        const int64_t slots = (d.use_tc5 && two_ctas) ? sms / 2 : (int64_t)sms * d.mma.ctas_per_sm;
        int64_t want = 1;
        if (units > 0 && units < slots) want = (slots + units - 1) / units;
        const int64_t chunk = 40 * (int64_t)d.mma.block_m > 512 ? 40 * (int64_t)d.mma.block_m : 512;
        // The tcgen05 kernels are persistent and their items are placed longest first: from about 1.6 items per
        // slot on the placement balances by itself (the short items fill up the slots of the medium ones) and a split
        // would only add partial writes and the combine.  Measured on 32 sequences of 4096 ... 32768 keys (128 items
        // on 74 slots): 283 us in one pass, 311 us in four key ranges.
        const int64_t by_len = (d.use_tc5 && units * 5 >= slots * 8) ? 1 : (max_len + chunk - 1) / chunk;
        int64_t s = want > by_len ? want : by_len;
        const int64_t cap = max_tiles / 2 > 1 ? max_tiles / 2 : 1;  // at least two key tiles per split
        if (s > cap) s = cap;
        if (s > 32) s = 32;
        splits = (int)(s < 1 ? 1 : s);
    }
    d.num_splits = splits;
    a.num_splits = splits;
    a.m_blocks = d.mma.m_blocks;
    if (d.use_tc5) {
        tc5_plan_items(a, two_ctas, sms);
        d.sched_bytes = sched_bytes(a.items_total);
    }
    if (splits > 1) {
        const int64_t rows_total = (int64_t)p->total_q * p->num_q_heads;
        d.ws_lse_bytes = ((splits * rows_total * 4 + 255) / 256) * 256;
        d.ws_o_bytes = ((splits * rows_total * p->head_dim * 4 + 255) / 256) * 256;
    }
    return d;
}

static void point_schedule(DecodeArgs& a, void* buffer) {
    a.sched_off = static_cast<const int32_t*>(buffer);
    a.sched_recs = reinterpret_cast<const SchedRec*>(static_cast<char*>(buffer) + kSchedHeaderBytes);
}

}  // namespace dlx

using namespace dlx;

extern "C" int dlx_version(void) { return 100; }

extern "C" const char* dlx_status_string(int status) {
    switch (status) {
        case DLX_OK: return "ok";
        case DLX_ERR_INVALID_ARGUMENT: return "invalid argument";
        case DLX_ERR_UNSUPPORTED: return "unsupported geometry or dtype";
        case DLX_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
        case DLX_ERR_WORKSPACE: return "split-K workspace missing or too small";
        case DLX_ERR_CUDA: return "CUDA runtime error";
        default: return "unknown status";
    }
}

extern "C" const char* dlx_last_error(void) { return last_error_buffer(); }

extern "C" int dlx_debug_device_status(int32_t out[4]) {
    if (out == nullptr) return fail(DLX_ERR_INVALID_ARGUMENT, "device_status: null output");
    int one[4], two[4];
    int rc = read_tc5_status(one);
    if (rc == DLX_OK) rc = read_tc5_pair_status(two);
    if (rc != DLX_OK) return rc;
    const int* first = one[0] != 0 ? one : two;   // the word of whichever kernel reported
    for (int i = 0; i < 4; ++i) out[i] = first[i];
    out[0] = one[0] | two[0];
    return DLX_OK;
}

extern "C" int64_t dlx_decode_attn_workspace_bytes(const dlx_decode_attn_params* p) {
    const int rc = validate_decode(p);
    if (rc != DLX_OK) return -(int64_t)rc;
    const DecodePlan d = plan_decode(p);
    return d.ws_o_bytes + d.ws_lse_bytes + d.sched_bytes;
}

extern "C" int32_t dlx_decode_attn_num_splits(const dlx_decode_attn_params* p) {
    const int rc = validate_decode(p);
    if (rc != DLX_OK) return -rc;
    return plan_decode(p).num_splits;
}

extern "C" int64_t dlx_decode_attn_schedule_bytes(const dlx_decode_attn_params* p) {
    const int rc = validate_decode(p);
    if (rc != DLX_OK) return -(int64_t)rc;
    return plan_decode(p).sched_bytes;
}

static int check_decode_pointers(const dlx_decode_attn_params* p, bool need_io) {
    if ((!p->context_lens && p->max_blocks > 0) || !p->cu_seqlens_q) return fail(DLX_ERR_INVALID_ARGUMENT, "decode: null pointer");
    if (need_io && (!p->q || !p->k || !p->v || !p->out)) return fail(DLX_ERR_INVALID_ARGUMENT, "decode: null pointer");
    if (p->max_blocks > 0 && (!p->block_tables || (need_io && (!p->k_cache || !p->v_cache))))
        return fail(DLX_ERR_INVALID_ARGUMENT, "decode: null cache or block table");
    return DLX_OK;
}

extern "C" int dlx_decode_attn_prepare(const dlx_decode_attn_params* p, void* schedule, int64_t schedule_bytes,
                                       void* stream) {
    int rc = validate_decode(p);
    if (rc != DLX_OK) return rc;
    DecodePlan d = plan_decode(p);
    if (d.sched_bytes == 0 || p->num_seqs == 0 || p->total_q == 0) return DLX_OK;   // this call's kernel takes no schedule
    rc = check_decode_pointers(p, false);
    if (rc != DLX_OK) return rc;
    if (schedule == nullptr || schedule_bytes < d.sched_bytes)
        return fail(DLX_ERR_WORKSPACE, "decode schedule: %lld bytes needed, got %lld", (long long)d.sched_bytes,
                    (long long)schedule_bytes);
    if (!aligned16(schedule)) return fail(DLX_ERR_ALIGNMENT, "decode schedule: buffer must be 16-byte aligned");
    point_schedule(d.args, schedule);
    return launch_decode_sched(d.args, static_cast<cudaStream_t>(stream));
}

extern "C" int dlx_stream_capture_id(void* stream, uint64_t* id) {
    if (id == nullptr) return fail(DLX_ERR_INVALID_ARGUMENT, "capture id: null output");
    cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
    unsigned long long cid = 0;
    const cudaError_t e = cudaStreamGetCaptureInfo(static_cast<cudaStream_t>(stream), &status, &cid);
    if (e != cudaSuccess) return fail(DLX_ERR_CUDA, "cudaStreamGetCaptureInfo: %s", cudaGetErrorString(e));
    *id = status == cudaStreamCaptureStatusActive ? (uint64_t)cid : 0;
    return DLX_OK;
}

extern "C" int dlx_decode_attn(const dlx_decode_attn_params* p, void* stream) {
    int rc = validate_decode(p);
    if (rc != DLX_OK) return rc;
    if (p->num_seqs == 0 || p->total_q == 0) return DLX_OK;
    rc = check_decode_pointers(p, true);
    if (rc != DLX_OK) return rc;
    const int hd = p->head_dim;
    if (p->q_row_stride < (int64_t)p->num_q_heads * hd || p->out_row_stride < (int64_t)p->num_q_heads * hd ||
        p->k_row_stride < (int64_t)p->num_kv_heads * hd || p->v_row_stride < (int64_t)p->num_kv_heads * hd)
        return fail(DLX_ERR_INVALID_ARGUMENT, "decode: a row stride is smaller than a row");
    if (p->max_blocks > 0 && p->cache_token_stride < (int64_t)p->num_kv_heads * hd)
        return fail(DLX_ERR_INVALID_ARGUMENT, "decode: cache token stride smaller than a row");
    // 16-byte vectors everywhere: bases 16-byte aligned, strides multiples of 8 elements
    const bool al = aligned16(p->q) && aligned16(p->k) && aligned16(p->v) && aligned16(p->out) &&
                    (p->max_blocks == 0 || (aligned16(p->k_cache) && aligned16(p->v_cache))) &&
                    p->q_row_stride % 8 == 0 && p->k_row_stride % 8 == 0 && p->v_row_stride % 8 == 0 &&
                    p->out_row_stride % 8 == 0 && p->cache_page_stride % 8 == 0 && p->cache_token_stride % 8 == 0;
    if (!al) return fail(DLX_ERR_ALIGNMENT, "decode: base pointers must be 16-byte aligned and strides multiples of 8 elements");
    if (p->kernel >= 2 && !tma_supported(p))
        return fail(DLX_ERR_UNSUPPORTED, "decode: the tcgen05 kernels need a page size that tiles into boxes of 8..128 rows");
    if (p->kernel == 3 && p->max_blocks == 0)
        return fail(DLX_ERR_UNSUPPORTED, "decode: the CTA-pair kernel needs a cache");

    DecodePlan d = plan_decode(p);
    DecodeArgs& a = d.args;
    if ((int64_t)a.hkv * d.mma.m_blocks > 65535) return fail(DLX_ERR_UNSUPPORTED, "decode: too many (KV head, M block) pairs");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool own_schedule = d.use_tc5 && p->schedule == nullptr;
    const int64_t need = d.ws_o_bytes + d.ws_lse_bytes + (own_schedule ? d.sched_bytes : 0);
    if (need > 0) {
        if (p->workspace == nullptr || p->workspace_bytes < need)
            return fail(DLX_ERR_WORKSPACE, "decode: %d splits%s need %lld workspace bytes, got %lld", d.num_splits,
                        own_schedule ? " and the schedule" : "", (long long)need, (long long)p->workspace_bytes);
        if (!aligned16(p->workspace)) return fail(DLX_ERR_ALIGNMENT, "decode: workspace must be 16-byte aligned");
    }
    if (d.num_splits > 1) {
        a.ws_lse = static_cast<float*>(p->workspace);
        a.ws_o = reinterpret_cast<float*>(static_cast<char*>(p->workspace) + d.ws_lse_bytes);
    }
    if (p->slot_mapping != nullptr && p->max_blocks > 0) {
        // The call also stores: the store kernel runs first, on the same stream.  (Storing from inside the attention
        // kernel was measured slower than this 3 us launch: it held up the epilogue warps of the items that did it.)
        if (p->cache_token_stride != (int64_t)p->num_kv_heads * hd || p->cache_page_stride != p->cache_token_stride * p->page_size)
            return fail(DLX_ERR_UNSUPPORTED, "decode with store: the flat-slot store kernel needs contiguous cache pages");
        rc = dlx_store_kvcache_unified(p->k, p->k_row_stride, p->v, p->v_row_stride, const_cast<void*>(p->k_cache),
                                       const_cast<void*>(p->v_cache), p->slot_mapping, p->slots_are_int64, a.total_kv,
                                       (int64_t)p->num_kv_heads * hd, 2, p->num_pages * (int64_t)p->page_size, stream);
        if (rc != DLX_OK) return rc;
    }
    if (d.use_tc5) {
        if (own_schedule) {
            // no prepared schedule: plan this launch now, into the tail of the workspace
            point_schedule(a, static_cast<char*>(p->workspace) + d.ws_lse_bytes + d.ws_o_bytes);
            rc = launch_decode_sched(a, st);
            if (rc != DLX_OK) return rc;
        } else {
            if (p->schedule_bytes < d.sched_bytes || !aligned16(p->schedule))
                return fail(DLX_ERR_WORKSPACE, "decode: schedule of %lld bytes needed (16-byte aligned), got %lld",
                            (long long)d.sched_bytes, (long long)p->schedule_bytes);
            point_schedule(a, const_cast<void*>(p->schedule));
        }
        rc = d.use_pair ? launch_decode_tc5_pair(a, st) : launch_decode_tc5(a, st);
    } else {
        rc = launch_decode_mma(a, d.mma, hd, st);
    }
    if (rc != DLX_OK) return rc;
    if (d.num_splits > 1) rc = launch_combine(a, hd, st);
    return rc;
}

// ---- decode attention without any allocation by anyone ---------------------------------------------
// Scratch (split-K partials and the launch's schedule) lives in a file-scope device array instead of caller
// memory.  The array's name is only a host-side handle: the device address is looked up once per device with
// cudaGetSymbolAddress (with that device current) and it is that pointer which the kernels receive.  The
// look-up is what makes the CUDA runtime load this file's device module, array included, on that device; the
// pointer table is written without a lock (every writer stores the same value) and is not refreshed after a
// cudaDeviceReset.
namespace {
constexpr int64_t kStaticScratchBytes = 32ll << 20;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];
void* g_static_scratch_ptr[64] = {};
}  // namespace

extern "C" int64_t dlx_static_scratch_bytes(void) { return kStaticScratchBytes; }

extern "C" int dlx_decode_attn_static_scratch(const dlx_decode_attn_params* p, void* stream) {
    int rc = validate_decode(p);
    if (rc != DLX_OK) return rc;
    const DecodePlan d = plan_decode(p);
    const int64_t need = d.ws_o_bytes + d.ws_lse_bytes + (p->schedule == nullptr ? d.sched_bytes : 0);
    if (need > kStaticScratchBytes)
        return fail(DLX_ERR_WORKSPACE,
                    "decode (static scratch): this call needs %lld scratch bytes, the built-in array holds %lld; "
                    "lower num_splits or use dlx_decode_attn with caller memory",
                    (long long)need, (long long)kStaticScratchBytes);
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(DLX_ERR_CUDA, "decode (static scratch): cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64)
        return fail(DLX_ERR_UNSUPPORTED, "decode (static scratch): device ordinal %d is outside the 64 this entry point tracks", dev);
    if (g_static_scratch_ptr[dev] == nullptr) {  // first call on this device: resolve the array's device address
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_static_scratch);
        if (e != cudaSuccess || ptr == nullptr)
            return fail(DLX_ERR_CUDA, "decode (static scratch): cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        g_static_scratch_ptr[dev] = ptr;
    }
    dlx_decode_attn_params q = *p;
    q.workspace = need > 0 ? g_static_scratch_ptr[dev] : nullptr;
    q.workspace_bytes = need > 0 ? kStaticScratchBytes : 0;
    return dlx_decode_attn(&q, stream);
}
