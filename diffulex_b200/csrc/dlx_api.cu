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
    bool use_tc5;
    int num_splits;
    int64_t ws_o_bytes, ws_lse_bytes;
};

static int validate_decode(const dlx_decode_attn_params* p) {
    if (p == nullptr) return fail(DLX_ERR_INVALID_ARGUMENT, "decode: null params");
    if (p->struct_bytes != sizeof(dlx_decode_attn_params))
        return fail(DLX_ERR_INVALID_ARGUMENT, "decode: struct_bytes %u != %zu (header mismatch)", p->struct_bytes,
                    sizeof(dlx_decode_attn_params));
    if (p->dtype != DLX_DTYPE_BF16) return fail(DLX_ERR_UNSUPPORTED, "decode: only bf16 is built");
    if (p->head_dim != 64 && p->head_dim != 128)
        return fail(DLX_ERR_UNSUPPORTED, "decode: head_dim %d (64 and 128 are built)", p->head_dim);
    if (p->num_seqs < 0 || p->total_q < 0 || p->max_blocks < 0 || p->num_pages < 0)
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
    if (p->kernel < 0 || p->kernel > 2) return fail(DLX_ERR_INVALID_ARGUMENT, "decode: kernel %d", p->kernel);
    if (p->kernel == 2 && !tc5_eligible(p->num_q_heads / p->num_kv_heads, p->head_dim))
        return fail(DLX_ERR_UNSUPPORTED, "decode: the tcgen05 kernel serves head_dim 128 with up to 128 query heads per KV head");
    if (p->num_seqs > 65535) return fail(DLX_ERR_UNSUPPORTED, "decode: more than 65535 sequences per call");
    return DLX_OK;
}

static DecodePlan plan_decode(const dlx_decode_attn_params* p) {
    DecodePlan d{};
    const int group = p->num_q_heads / p->num_kv_heads;
    const int64_t rows = (int64_t)group * p->max_q_len;
    d.mma = plan_mma((int)(rows > 1 << 20 ? 1 << 20 : rows), p->head_dim);
    d.use_tc5 = p->kernel != 1 && tc5_eligible(group, p->head_dim);
    if (d.use_tc5) {  // work item = (sequence, KV head, block of 128 / group whole tokens, split): 128-key tiles, 1 CTA/SM
        d.mma.block_m = 128; d.mma.block_n = 128; d.mma.ctas_per_sm = 1;
        const int tokens_per_block = 128 / group;
        const int q_len = p->max_q_len > 1 << 20 ? 1 << 20 : p->max_q_len;
        d.mma.m_blocks = (q_len + tokens_per_block - 1) / tokens_per_block;
    }
    const int64_t max_len = p->max_kv_len > 0 ? p->max_kv_len : (int64_t)p->max_blocks * p->page_size + p->max_q_len;
    const int64_t max_tiles = (max_len + d.mma.block_n - 1) / d.mma.block_n;
    int splits = p->num_splits;
    if (splits == 0) {
        // (1) fill the machine when there are fewer CTAs than resident slots; (2) cut very long
        // contexts so ragged batches balance.  A split costs one fp32 partial (write + read) of
        // block_m x hd per CTA, i.e. 2*M/chunk of the chunk's KV bytes: keep chunks >= 40*M keys.
        const int64_t units = (int64_t)p->num_seqs * p->num_kv_heads * d.mma.m_blocks;
        const int64_t slots = (int64_t)kNumSMs * d.mma.ctas_per_sm;
        int64_t want = 1;
        if (units > 0 && units < slots) want = (slots + units - 1) / units;
        const int64_t chunk = 40 * (int64_t)d.mma.block_m > 512 ? 40 * (int64_t)d.mma.block_m : 512;
        // The tcgen05 kernel is persistent (one CTA per SM walks a longest-first item list): with two or more
        // items per SM the list balances by itself and a split would only add partial writes and the combine.
        const int64_t by_len = (d.use_tc5 && units >= 2 * slots) ? 1 : (max_len + chunk - 1) / chunk;
        int64_t s = want > by_len ? want : by_len;
        const int64_t cap = max_tiles / 2 > 1 ? max_tiles / 2 : 1;  // at least two key tiles per split
        if (s > cap) s = cap;
        if (s > 32) s = 32;
        splits = (int)(s < 1 ? 1 : s);
    }
    d.num_splits = splits;
    if (splits > 1) {
        const int64_t rows_total = (int64_t)p->total_q * p->num_q_heads;
        d.ws_lse_bytes = ((splits * rows_total * 4 + 255) / 256) * 256;
        d.ws_o_bytes = splits * rows_total * p->head_dim * 4;
    }
    return d;
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
    int tmp[4];
    const int rc = read_tc5_status(tmp);
    if (rc != DLX_OK) return rc;
    for (int i = 0; i < 4; ++i) out[i] = tmp[i];
    return DLX_OK;
}

extern "C" int dlx_debug_profile(int enable, uint64_t out[24]) {
    return tc5_profile(enable, reinterpret_cast<unsigned long long*>(out));
}

extern "C" int64_t dlx_decode_attn_workspace_bytes(const dlx_decode_attn_params* p) {
    const int rc = validate_decode(p);
    if (rc != DLX_OK) return -(int64_t)rc;
    const DecodePlan d = plan_decode(p);
    return d.ws_o_bytes + d.ws_lse_bytes;
}

extern "C" int32_t dlx_decode_attn_num_splits(const dlx_decode_attn_params* p) {
    const int rc = validate_decode(p);
    if (rc != DLX_OK) return -rc;
    return plan_decode(p).num_splits;
}

extern "C" int dlx_decode_attn(const dlx_decode_attn_params* p, void* stream) {
    int rc = validate_decode(p);
    if (rc != DLX_OK) return rc;
    if (p->num_seqs == 0 || p->total_q == 0) return DLX_OK;
    if (!p->q || !p->k || !p->v || !p->out || !p->context_lens || !p->cu_seqlens_q)
        return fail(DLX_ERR_INVALID_ARGUMENT, "decode: null pointer");
    if (p->max_blocks > 0 && (!p->k_cache || !p->v_cache || !p->block_tables))
        return fail(DLX_ERR_INVALID_ARGUMENT, "decode: null cache or block table");
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

    const DecodePlan d = plan_decode(p);
    DecodeArgs a{};
    a.q = p->q; a.k = p->k; a.v = p->v; a.k_cache = p->k_cache; a.v_cache = p->v_cache; a.out = p->out;
    a.block_tables = p->block_tables; a.context_lens = p->context_lens;
    a.cu_q = p->cu_seqlens_q; a.cu_kv = p->cu_seqlens_kv; a.seq_order = p->seq_order;
    a.q_rs = p->q_row_stride; a.k_rs = p->k_row_stride; a.v_rs = p->v_row_stride; a.o_rs = p->out_row_stride;
    a.page_stride = p->cache_page_stride; a.token_stride = p->cache_token_stride;
    a.bt_stride = p->block_table_stride; a.num_pages = p->num_pages;
    a.total_q = p->total_q; a.num_seqs = p->num_seqs; a.max_blocks = p->max_blocks; a.max_q_len = p->max_q_len;
    a.hq = p->num_q_heads; a.hkv = p->num_kv_heads; a.group = a.hq / a.hkv; a.page_size = p->page_size;
    a.mask_mode = p->mask_mode; a.dbs = p->diffusion_block_size > 0 ? p->diffusion_block_size : 1;
    a.num_splits = d.num_splits; a.m_blocks = d.mma.m_blocks;
    a.scale_log2 = p->scale * 1.4426950408889634f;
    if ((int64_t)a.hkv * a.m_blocks > 65535) return fail(DLX_ERR_UNSUPPORTED, "decode: too many (KV head, M block) pairs");
    if (d.num_splits > 1) {
        if (p->workspace == nullptr || p->workspace_bytes < d.ws_o_bytes + d.ws_lse_bytes)
            return fail(DLX_ERR_WORKSPACE, "decode: %d splits need %lld workspace bytes, got %lld", d.num_splits,
                        (long long)(d.ws_o_bytes + d.ws_lse_bytes), (long long)p->workspace_bytes);
        if (!aligned16(p->workspace)) return fail(DLX_ERR_ALIGNMENT, "decode: workspace must be 16-byte aligned");
        a.ws_lse = static_cast<float*>(p->workspace);
        a.ws_o = reinterpret_cast<float*>(static_cast<char*>(p->workspace) + d.ws_lse_bytes);
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    rc = d.use_tc5 ? launch_decode_tc5(a, st) : launch_decode_mma(a, d.mma, hd, st);
    if (rc != DLX_OK) return rc;
    if (d.num_splits > 1) rc = launch_combine(a, hd, st);
    return rc;
}

// ---- decode attention without any allocation by anyone ---------------------------------------------
// Split-K scratch lives in a file-scope device array instead of caller memory.  The array's name is only
// a host-side handle: the device address is looked up once per device with cudaGetSymbolAddress (with
// that device current) and it is that pointer which the kernels receive.
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
    const int64_t need = d.ws_o_bytes + d.ws_lse_bytes;
    if (need > kStaticScratchBytes)
        return fail(DLX_ERR_WORKSPACE,
                    "decode (static scratch): this call needs %lld scratch bytes, the built-in array holds %lld; "
                    "lower num_splits or use dlx_decode_attn with caller memory",
                    (long long)need, (long long)kStaticScratchBytes);
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64)
        return fail(DLX_ERR_CUDA, "decode (static scratch): cudaGetDevice: %s", cudaGetErrorString(e));
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
