// Paged block-diffusion decode attention on a PAIR of CTAs (tcgen05 cta_group::2 + TMEM + TMA).
//
// Shape served: head_dim 128, bf16, G <= 128 query heads per KV head, more than 128 packed query rows per
// (sequence, KV head) -- e.g. 28 query heads over 4 KV heads with a 32-token block: 224 rows.  A work item is a
// (sequence, KV head, 2 x (128 / G) query tokens, key-range split); the two CTAs of a cluster take 128 / G whole
// tokens each (their own 128 accumulator rows), and every tcgen05.mma is issued once, by one thread of the even CTA,
// for both: M = 256.  Each CTA fetches only HALF of every K / V tile -- 64 of the 128 keys for S = Q K^T, 64 of the
// 128 head_dim columns for O += P V -- with ordinary per-CTA TMA boxes; the tensor cores read the other half from the
// peer's shared memory.  Against two independent CTAs on the same item this halves the L2 -> SM traffic and the
// shared-memory bytes written and read per tile, and the freed shared memory holds deeper K / V rings and a second
// Q buffer.  Measured, it is not faster than two independent CTAs (the hand-offs between the tensor pipe and the
// softmax warps bound a tile, not the traffic), so it is taken on request only (kernel = 3).
//
// Work comes from a schedule built on the device once per metadata state (decode_sched.cu): records with every length
// resolved and the first page ids attached, placed on the pairs by a longest-processing-time greedy.
//
// Warp roles per CTA (512 threads; register files resized after the split):
//   warps 0-7    two softmax warpgroups over the CTA's 128 rows, alternate key tiles (as in decode_attn_tc5.cu).
//                P = exp2(s * scale - m_ref) with m_ref fixed by the item's first tile; later tiles compute no row
//                maximum at all.  An exponent that leaves the safe range (tile row sum above 2^90, final row sum
//                below 2^-80) marks the item, and the CTA recomputes its rows of that item exactly (plain fp32,
//                two passes) before it retires: results never depend on the fixed reference
//   warp 8, 9    K loader (this CTA's 64 keys of each tile), V loader (all 128 keys, this CTA's 64 head_dim columns)
//   warp 10      even CTA: one thread issues S = Q K^T for the pair; odd CTA: one thread forwards "my K half / my Q
//                landed" to the even CTA's barriers.  Both fetch their own Q block (TMA), one item ahead
//   warp 11      even CTA: one thread issues O += P V; odd CTA: forwards "my V half landed"
//   warps 12-15  epilogue warpgroup: O / l -> global through a swizzled staging buffer
// Barriers that the issuing threads wait on live in the even CTA and count arrivals of both CTAs (one elected lane per
// warp); barriers that announce MMA completion are signalled in both CTAs by one multicast tcgen05.commit.
// TMEM (512 columns per CTA): three score buffers of 128 fp32 columns, P (bf16) written over the first 64 columns of
// its own score buffer once the scores are in registers | O (128).
//
// Every wait is bounded; on expiry the CTA raises an abort word, everyone drains, the place goes to a device status
// word, both CTAs meet at a cluster barrier, TMEM is freed and the CTA returns (no trap).
//
// Reference semantics: diffulex_kernel/python/dllm_flash_attn.py:163-347 and :632-637.
#include <cuda.h>

#include <string.h>

#include "dlx_common.cuh"
#include "decode_attn.cuh"
#include "tc5_common.cuh"

namespace dlx {
namespace tc5 {
// defined in decode_attn_tc5.cu: encodes (and memoises) a tiled tensor map
int tc5_cache_map(const void* ptr, int64_t page_stride, int64_t token_stride, int64_t num_pages, int hkv, int page_size,
                  int rows, int rank, CUtensorMap* out);
}  // namespace tc5

namespace tc5p {
using namespace tc5;

constexpr int HD = 128;
constexpr int TILE_M = 128;                  // packed query rows per CTA (TMEM lanes)
constexpr int TILE_N = 128;                  // keys per K/V tile
constexpr int Q_REGION = 128 * 128;          // [128 rows][64 bf16], 128-byte swizzle: 16 KiB
constexpr int Q_BYTES = 2 * Q_REGION;        // one Q block: two head_dim halves
constexpr int K_ROWS = 64;                   // keys of a tile held by this CTA
constexpr int K_REGION = K_ROWS * 128;       // [64 keys][64 bf16]: 8 KiB
constexpr int K_STAGE = 2 * K_REGION;        // two head_dim halves
constexpr int V_STAGE = TILE_N * 128;        // [128 keys][this CTA's 64 head_dim columns]: 16 KiB
#ifndef DLX_PAIR_KSTAGES
#define DLX_PAIR_KSTAGES 3
#define DLX_PAIR_VSTAGES 4
#endif
constexpr int KSTAGES = DLX_PAIR_KSTAGES, VSTAGES = DLX_PAIR_VSTAGES;
static_assert(KSTAGES >= 2 && KSTAGES <= 4 && VSTAGES >= 2 && VSTAGES <= 4, "ring depth");
constexpr int OFF_K = 2 * Q_BYTES;
constexpr int OFF_V = OFF_K + KSTAGES * K_STAGE;
constexpr int OFF_BAR = OFF_V + VSTAGES * V_STAGE;
constexpr int BT_SLOTS = 512;                      // page ids of a long item that its record does not hold
constexpr int OFF_BT = OFF_BAR + 512;
constexpr int OFF_XCH = OFF_BT + 2 * BT_SLOTS * 4; // 8 x 128 floats: row references and row sums between the warpgroups
constexpr int OFF_STAGE = OFF_XCH + 8 * 128 * 4;   // output staging: 2 halves x 4 epilogue warps x (32 rows x 128 bytes)
constexpr int STAGE_WARP_BYTES = 32 * 128;
constexpr int OFF_ROWMAP = OFF_STAGE + 8 * STAGE_WARP_BYTES;   // int2[128]: (row / group, row % group)
constexpr int MAX_ROUNDS = 32;                     // records kept in shared memory; later rounds are read from global
constexpr int OFF_ITEMS = OFF_ROWMAP + 128 * 8;
constexpr int OFF_FLAGS = OFF_ITEMS + MAX_ROUNDS * (int)sizeof(SchedRec);   // redo bit per round
constexpr int FLAG_WORDS = 128;                    // 4096 rounds
constexpr int OFF_ARGS = OFF_FLAGS + FLAG_WORDS * 4;
constexpr int SMEM_BYTES = OFF_ARGS + 320 + 1024;  // + slack for 1024-byte alignment
static_assert(sizeof(DecodeArgs) <= 320, "argument block copy");
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

constexpr int NUM_THREADS = 512;
constexpr int SOFTMAX_REGS = 184, HELPER_REGS = 56, EPI_REGS = 88;
static_assert(2 * SOFTMAX_REGS + HELPER_REGS + EPI_REGS <= 512, "register budget");
constexpr int EPI_WARP0 = 12;
constexpr int KLOAD_WARP = 8, VLOAD_WARP = 9, QK_WARP = 10, PV_WARP = 11;
// TMEM columns (512 per CTA): three score buffers of 128 fp32 columns, then O.  P of a tile (128 bf16 = 64 columns)
// overwrites the first half of the tile's own score buffer once the scores are in registers, so a buffer is busy from
// the tile's Q K^T until its P V has run, and three tiles are in flight at any time: the chain Q K^T -> scores to
// registers -> exponentials -> P -> P V is about three tile times long.
constexpr int NBUF = 3;
constexpr uint32_t TM_S = 0, TM_O = 384;

// barrier slots (8 bytes each) at OFF_BAR
enum {
    B_QFULL = 0,     // [Q buffer] local: this CTA's Q block has landed
    B_QFULLP = 2,    // [Q buffer] even CTA: the odd CTA's Q block has landed
    B_QEMPTY = 4,    // [Q buffer] both (commit): every Q K^T of the item has read Q
    B_KFULL = 6,     // [stage] local: one arrival (lane 0 of the loader) + the bytes of its boxes + its lanes' row copies
    B_KFULLP = 10,   // [stage] even CTA: the odd CTA's half has landed
    B_KEMPTY = 14,   // [stage] both (commit)
    B_VFULL = 18, B_VFULLP = 22, B_VEMPTY = 26,
    B_SFULL = 30,    // [buffer] both (commit): the tile's scores are in TMEM
    B_PFULL = 33,    // [buffer] even CTA, 8 arrivals: both CTAs' P is in TMEM (over the scores)
    B_BUFFREE = 36,  // [buffer] even CTA (commit): the tile's P V has run, the next Q K^T may overwrite the buffer
    B_OFULL = 39,    // both (commit)
    B_OFREE = 40,    // even CTA, 8 arrivals: both epilogue warpgroups hold O in registers
    B_MRFULL = 41, B_MREMPTY = 43, B_LSFULL = 45, B_LSEMPTY = 47,   // local rings between the warpgroups
    B_EPIDONE = 49,  // local, 128 arrivals: the epilogue warpgroup has written its last output row
    B_COUNT = 50
};
static_assert(8 * B_COUNT + 16 <= 512, "barrier block");

__device__ int g_status_pair[4];  // [0] bit 0: a bounded wait expired; [1] wait site, [2] tile, [3] CTA

// Tensor maps of one launch, by level l = 0..7: boxes of 128 >> l rows x 64 head_dim columns.  kc / vc: the caches as
// {head_dim, Hkv, page row, page}; kn / vn: the in-flight rows as {head_dim, Hkv, token}.  Levels whose box exceeds a
// page (caches) are unused.  Any run of rows is a few boxes of falling size; a box may start at any row of a tile:
// the 128-byte swizzle of a copy follows the shared-memory address it writes.
constexpr int LEVELS = 8;
struct TmaMapsPair {
    CUtensorMap kc[LEVELS], vc[LEVELS], kn[LEVELS], vn[LEVELS];
    CUtensorMap q;
};

// A record as this CTA sees it.
struct Item {
    bool valid, empty_split;
    int seq, kvh, split;
    int q0, ctx, kv0, nnew, total;
    int tok0, rows_here;      // first token of this CTA's block, its valid packed rows (0: this CTA only helps its peer)
    int full_until;           // keys below this are visible to every row of the CTA
    int t0, n;
    int first_page, n_pages;
};

__device__ __forceinline__ Item view_item(const DecodeArgs& a, const SchedRec* r, int rank) {
    Item it;
    const int4 w0 = *reinterpret_cast<const int4*>(&r->seq);
    const int4 w1 = *reinterpret_cast<const int4*>(&r->q0);
    const int4 w2 = *reinterpret_cast<const int4*>(&r->nnew);
    const int2 w3 = *reinterpret_cast<const int2*>(&r->first_page);
    it.seq = w0.x; it.kvh = w0.y; it.split = w0.w;
    it.q0 = w1.x; it.ctx = w1.z; it.kv0 = w1.w;
    it.nnew = w2.x; it.t0 = w2.y; it.n = w2.z;
    it.valid = (w2.w & SCHED_VALID) != 0;
    it.empty_split = (w2.w & SCHED_EMPTY_SPLIT) != 0;
    it.first_page = w3.x; it.n_pages = w3.y;
    it.total = it.ctx + it.nnew;
    const int qn = w1.y;
    it.tok0 = w0.z * a.tokens_per_item + rank * a.q_tokens;
    it.rows_here = max(min(qn - it.tok0, a.q_tokens), 0) * a.group;
    it.full_until = it.total;
    if (a.mask_mode == DLX_MASK_BLOCK_CAUSAL) it.full_until = it.ctx + min(it.nnew, (it.tok0 / a.dbs + 1) * a.dbs);
    return it;
}

__device__ __forceinline__ int tile_of(int jj, int n) { return n - 1 - ((jj < 2 && n >= 2) ? (jj ^ 1) : jj); }

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
decode_attn_tc5_pair_kernel(const DecodeArgs a_param, const __grid_constant__ TmaMapsPair maps) {
    extern __shared__ unsigned char smem_raw[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rank = (int)cluster_cta_rank();          // 0: issues the MMAs of the pair
    const int pair = (int)blockIdx.x >> 1;

    const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
    unsigned char* gbase = smem_raw + (sbase - smem_u32(smem_raw));
    const uint32_t sQ = sbase, sK = sbase + OFF_K, sV = sbase + OFF_V, sBar = sbase + OFF_BAR;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + OFF_BAR + 8 * B_COUNT);
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + OFF_BAR + 8 * B_COUNT + 8);
    auto bar = [&](int slot) { return sBar + 8u * slot; };
    // the same barrier in the even CTA (a shared::cluster address; the even CTA's own for rank 0)
    const uint32_t sBar0 = map_to_cta(sBar, 0);
    auto bar0 = [&](int slot) { return sBar0 + 8u * slot; };
    {
        const uint32_t* src = reinterpret_cast<const uint32_t*>(&a_param);
        uint32_t* dst = reinterpret_cast<uint32_t*>(gbase + OFF_ARGS);
        if (tid < (int)(sizeof(DecodeArgs) / 4)) dst[tid] = src[tid];
    }
    const DecodeArgs& a = *reinterpret_cast<const DecodeArgs*>(gbase + OFF_ARGS);   // for use AFTER the set-up barrier
    const int G = a_param.group;

    // this pair's records: the offsets are requested first, the barriers are set up while they travel
    const int rec0 = a_param.sched_off[pair];
    const int n_rounds = a_param.sched_off[pair + 1] - rec0;
    if (tid < B_COUNT) {
        // one barrier per thread; arrival counts: 8 = one elected lane per warp of a warpgroup in both CTAs, 128 / 256 =
        // every thread of one / two warpgroups of this CTA, 1 = one thread, a tcgen05.commit or a loader's lane 0
        const int b = tid;
        int count = 1;
        if ((b >= B_PFULL && b < B_PFULL + NBUF) || b == B_OFREE) count = 8;
        else if (b == B_LSFULL || b == B_LSFULL + 1) count = 256;
        else if (b >= B_MRFULL) count = 128;   // MRFULL, MREMPTY, LSEMPTY, EPIDONE
        mbar_init(bar(b), count);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (tid == 0) *abort_flag = 0;
    if (warp == QK_WARP) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;\n" ::"r"(sBar + 8u * B_COUNT + 8u) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    // This CTA's barriers and TMEM are ready: tell the peer now, and wait for the peer (cluster_wait, inside the roles)
    // only where something first crosses the pair.  Loads into this CTA's own shared memory start before that.
    cluster_arrive();
    const SchedRec* recs_g = a_param.sched_recs + rec0;
    SchedRec* recs_s = reinterpret_cast<SchedRec*>(gbase + OFF_ITEMS);
    {
        const int n_tab = min(n_rounds, MAX_ROUNDS);
        const uint4* src = reinterpret_cast<const uint4*>(recs_g);
        uint4* dst = reinterpret_cast<uint4*>(recs_s);
        for (int i = tid; i < n_tab * (int)(sizeof(SchedRec) / 16); i += NUM_THREADS) dst[i] = src[i];
    }
    auto rec_of = [&](int k) -> const SchedRec* { return k < MAX_ROUNDS ? recs_s + k : recs_g + k; };
    int2* rowmap = reinterpret_cast<int2*>(gbase + OFF_ROWMAP);
    if (tid >= 128 && tid < 256) rowmap[tid - 128] = make_int2((tid - 128) / G, (tid - 128) % G);
    uint32_t* redo_flags = reinterpret_cast<uint32_t*>(gbase + OFF_FLAGS);
    if (tid >= 256 && tid < 256 + FLAG_WORDS) redo_flags[tid - 256] = 0;
    {
        // Q rows past the last whole token of a block are never written by a Q box: zero them once in both buffers.
        const int rows_used = a_param.q_tokens * G;
        for (int i = tid; i < 2 * (TILE_M - rows_used) * 16; i += NUM_THREADS) {
            const int buf = i / ((TILE_M - rows_used) * 16), j = i - buf * (TILE_M - rows_used) * 16;
            const int row = rows_used + (j >> 4), chunk = j & 15;
            *reinterpret_cast<uint4*>(gbase + buf * Q_BYTES + (chunk >> 3) * Q_REGION + row * 128 + ((chunk & 7) << 4)) = make_uint4(0, 0, 0, 0);
        }
        // The K and V rings start out as zeros: rows that no copy writes must hold finite values.
        for (int i = tid; i < (KSTAGES * K_STAGE + VSTAGES * V_STAGE) / 16; i += NUM_THREADS)
            *reinterpret_cast<uint4*>(gbase + OFF_K + i * 16) = make_uint4(0, 0, 0, 0);
        fence_async_proxy();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    int done = 0, ck = 0;   // valid items finished, key tiles finished (identical in every role of both CTAs)

    if (warp < 8) {
        reg_inc<SOFTMAX_REGS>();
        cluster_wait();   // before the first signal to the even CTA
        // =========================== softmax warpgroups ===========================
        const int w = warp >> 2;
        const int L = tid & 127;
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        float* xm = reinterpret_cast<float*>(gbase + OFF_XCH);    // [2][128] row references
        float* xs = xm + 256;                                     // [2][3][128] row sums of each warpgroup, reference
        const float sl2 = a.scale_log2;
        int mr = 0;
        bool alive = true;
#pragma unroll 1
        for (int round = 0; round < n_rounds && alive; ++round) {
            const Item it = view_item(a, rec_of(round), rank);
            const int64_t head0 = (int64_t)it.kvh * G;
            if (it.empty_split) {
                if (a.num_splits > 1)
                    for (int r = tid; r < it.rows_here; r += 256) {
                        const int2 dm = rowmap[r];
                        a.ws_lse[((int64_t)it.split * a.total_q + it.q0 + it.tok0 + dm.x) * a.hq + head0 + dm.y] = -INFINITY;
                    }
                continue;
            }
            if (!it.valid) continue;
            const int n = it.n, rows_here = it.rows_here;
            const int2 my_row = rowmap[L];
            const bool warp_valid = (warp & 3) * 32 < rows_here;
            const bool row_valid = L < rows_here;
            const int jj_first = (w ^ ck) & 1;
            const bool multi = n >= 2;
            const int slot = mr & 1;
            const uint32_t ring_par = (mr >> 1) & 1;
            int limit = it.total;
            if (a.mask_mode == DLX_MASK_BLOCK_CAUSAL && row_valid) limit = it.ctx + min(it.nnew, ((it.tok0 + my_row.x) / a.dbs + 1) * a.dbs);
            float m_ref = 0.f, l_run = 0.f;
            bool out_of_range = false;
#pragma unroll 1
            for (int jj = jj_first; jj < n && alive; jj += 2) {
                const int buf = (ck + jj) % NBUF, u = (ck + jj) / NBUF;   // score buffer of the tile and its use count
                const uint32_t tS = lane_base + TM_S + buf * 128;
                bool ok = mbar_wait(bar(B_SFULL + buf), u & 1, abort_flag, 1 + w, jj);
                if (!__all_sync(0xffffffffu, ok)) { alive = false; break; }
                tc_fence_after();
                if (multi && jj == 0 && mr >= 2) {
                    bool oke = mbar_wait(bar(B_MREMPTY + slot), ring_par ^ 1, abort_flag, 4, -3);
                    if (!__all_sync(0xffffffffu, oke)) { alive = false; break; }
                }
                if (warp_valid) {
                    const int key0 = (it.t0 + tile_of(jj, n)) * TILE_N;
                    uint32_t v[4][32];
                    tmem_ld32(tS, v[0]); tmem_ld32(tS + 32, v[1]); tmem_ld32(tS + 64, v[2]); tmem_ld32(tS + 96, v[3]);
                    tmem_ld_wait();
                    float mx_any = -INFINITY;
                    if (key0 + TILE_N > it.full_until) {
                        // The tile touches a mask boundary (warp-uniform; one or two tiles per item): hidden scores become
                        // -inf in registers.  Only an item's first tile needs the maximum over its hidden keys as well.
                        const int rel = limit - key0, rel_any = it.total - key0;
                        if (jj == 0) {
#pragma unroll
                            for (int c = 0; c < 4; ++c)
#pragma unroll
                                for (int e = 0; e < 32; ++e)
                                    if (c * 32 + e < rel_any) mx_any = fmaxf(mx_any, __uint_as_float(v[c][e]));
                        }
#pragma unroll
                        for (int c = 0; c < 4; ++c)
#pragma unroll
                            for (int e = 0; e < 32; ++e)
                                if (c * 32 + e >= rel) v[c][e] = 0xff800000u;
                    }
                    if (jj == 0) {
                        // First tile of the item: its row maximum becomes the fixed reference of the row.
                        float mx4[4];
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            mx4[c] = -INFINITY;
#pragma unroll
                            for (int e = 0; e < 32; e += 2)
                                mx4[c] = max3(mx4[c], __uint_as_float(v[c][e]), __uint_as_float(v[c][e + 1]));
                        }
                        const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2;
                        m_ref = (mx != -INFINITY) ? mx : (mx_any != -INFINITY ? mx_any * sl2 : 0.f);
                        if (multi) {
                            xm[slot * 128 + L] = m_ref;
                            mbar_arrive(bar(B_MRFULL + slot));
                        }
                    } else if (jj == 1) {
                        bool okm = mbar_wait(bar(B_MRFULL + slot), ring_par, abort_flag, 4, 0);
                        if (!__all_sync(0xffffffffu, okm)) { alive = false; break; }
                        m_ref = xm[slot * 128 + L];
                        mbar_arrive(bar(B_MREMPTY + slot));
                    }
                    // P = exp2(s * scale - m_ref) as bf16, written over the first half of the tile's own score buffer (the
                    // scores are all in registers by now)
                    float2 lacc0 = make_float2(0.f, 0.f), lacc1 = make_float2(0.f, 0.f);
                    const float2 sl2v = make_float2(sl2, sl2), negm = make_float2(-m_ref, -m_ref);
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        uint32_t pk[16];
#pragma unroll
                        for (int e = 0; e < 32; e += 2) {
                            const float2 x = __ffma2_rn(make_float2(__uint_as_float(v[c][e]), __uint_as_float(v[c][e + 1])), sl2v, negm);
                            const float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
                            if ((e >> 1) & 1) lacc1 = __fadd2_rn(lacc1, p); else lacc0 = __fadd2_rn(lacc0, p);
                            pk[e >> 1] = pack2<__nv_bfloat16>(p.x, p.y);
                        }
                        tmem_st16(tS + c * 16, pk);
                    }
                    lacc0 = __fadd2_rn(lacc0, lacc1);
                    const float tsum = lacc0.x + lacc0.y;
                    out_of_range |= !(tsum <= DLX_SUM_HIGH);   // also catches NaN
                    l_run += tsum;
                    tmem_st_wait();
                } else {
                    if (multi && jj == 0) mbar_arrive(bar(B_MRFULL + slot));
                    if (jj == 1) {
                        bool okm = mbar_wait(bar(B_MRFULL + slot), ring_par, abort_flag, 4, 0);
                        if (!__all_sync(0xffffffffu, okm)) { alive = false; break; }
                        mbar_arrive(bar(B_MREMPTY + slot));
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(bar0(B_PFULL + buf));
            }
            if (!alive) break;
            if (__any_sync(0xffffffffu, out_of_range && row_valid) && lane == 0)
                atomicOr(&redo_flags[(round >> 5) & (FLAG_WORDS - 1)], 1u << (round & 31));
            {
                const int ls = done & 1;
                if (done >= 2) {
                    bool oke = mbar_wait(bar(B_LSEMPTY + ls), ((done >> 1) & 1) ^ 1, abort_flag, 4, -4);
                    if (!__all_sync(0xffffffffu, oke)) { alive = false; break; }
                }
                xs[ls * 384 + w * 128 + L] = l_run;
                if (jj_first == 0) xs[ls * 384 + 256 + L] = m_ref;
                mbar_arrive(bar(B_LSFULL + ls));
            }
            ++done; ck += n; mr += multi ? 1 : 0;
        }
        // ---- items that left the fixed reference's range: this CTA's rows again, exactly ----
        // The epilogue warpgroup signals its last output row (and its last flag); by then every
        // MMA of the pair has completed (its last O_full), so the K / V rings are idle and serve as scratch.
        const bool epi_done = mbar_wait(bar(B_EPIDONE), 0, abort_flag, 15, -7);
        if (alive && epi_done && *abort_flag == 0) {
            float* scratch = reinterpret_cast<float*>(gbase + OFF_K);
            static_assert(8 * (REDO_CHUNK + HD) * 4 <= KSTAGES * K_STAGE + VSTAGES * V_STAGE, "redo scratch");
#pragma unroll 1
            const int flag_words = min((n_rounds + 31) >> 5, FLAG_WORDS);
#pragma unroll 1
            for (int wd = 0; wd < flag_words; ++wd) {
                uint32_t bits = redo_flags[wd];
                while (bits) {
                    const int b = __ffs(bits) - 1;
                    bits &= bits - 1;
                    // rounds beyond the flag words share their bits: every round that maps to a set bit is redone
                    for (int round = wd * 32 + b; round < n_rounds; round += 32 * FLAG_WORDS) {
                        const Item it = view_item(a, rec_of(round), rank);
                        if (it.valid && it.rows_here > 0) redo_item_exact(a, it, warp, lane, scratch);
                    }
                }
            }
        }
    } else if (warp >= EPI_WARP0) {
        // =========================== epilogue warpgroup: O / l -> global ===========================
        reg_dec<EPI_REGS>();
        cluster_wait();   // before the first signal to the even CTA
        const int L = tid & 127, wq = warp & 3;
        const uint32_t tO = tmem + ((uint32_t)(wq * 32) << 16) + TM_O;
        const float* xs = reinterpret_cast<const float*>(gbase + OFF_XCH) + 256;
        unsigned char* stage = gbase + OFF_STAGE + wq * STAGE_WARP_BYTES;
        bool alive = true;
#pragma unroll 1
        for (int round = 0; round < n_rounds && alive; ++round) {
            const Item it = view_item(a, rec_of(round), rank);
            if (!it.valid) continue;
            const int ls = done & 1;
            bool ok = mbar_wait(bar(B_LSFULL + ls), (done >> 1) & 1, abort_flag, 12, -5);
            if (!__all_sync(0xffffffffu, ok)) break;
            const float l_run = xs[ls * 384 + L] + xs[ls * 384 + 128 + L];
            const float m_ref = xs[ls * 384 + 256 + L];
            mbar_arrive(bar(B_LSEMPTY + ls));
            ok = mbar_wait(bar(B_OFULL), done & 1, abort_flag, 3, it.n);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const int rows_here = it.rows_here;
            const int head0 = it.kvh * G;
            const bool row_valid = L < rows_here;
            if (wq * 32 < rows_here) {
                // a row that sees at least one key of this range must have a row sum well inside fp32's range
                bool low = false;
                if (row_valid && !(l_run >= DLX_SUM_LOW)) {
                    int limit = it.total;
                    if (a.mask_mode == DLX_MASK_BLOCK_CAUSAL) limit = it.ctx + min(it.nnew, ((it.tok0 + rowmap[L].x) / a.dbs + 1) * a.dbs);
                    low = limit > it.t0 * TILE_N;
                }
                if (__any_sync(0xffffffffu, low) && lane == 0)
                    atomicOr(&redo_flags[(round >> 5) & (FLAG_WORDS - 1)], 1u << (round & 31));
                const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
                if (a.num_splits == 1) {
                    // bf16 output.  Both halves of O (64 head_dim columns each) go to a swizzled staging buffer first, and O is
                    // released to the next item's P V right after the second load; the rows then leave as 4 rows x 128
                    // contiguous bytes per store instruction (a thread holds a ROW: direct stores would touch 32 lines).
#pragma unroll 1
                    for (int c = 0; c < 2; ++c) {
                        uint32_t v[2][32];
                        tmem_ld32(tO + c * 64, v[0]);
                        tmem_ld32(tO + c * 64 + 32, v[1]);
                        tmem_ld_wait();
                        if (c == 1) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive_cluster(bar0(B_OFREE));   // the next item's P V may overwrite O
                        }
                        unsigned char* st = stage + c * (4 * STAGE_WARP_BYTES);
#pragma unroll
                        for (int q4 = 0; q4 < 8; ++q4) {
                            const uint32_t* x = &v[q4 >> 2][(q4 & 3) * 8];
                            uint4 o;
                            o.x = pack2<__nv_bfloat16>(__uint_as_float(x[0]) * inv, __uint_as_float(x[1]) * inv);
                            o.y = pack2<__nv_bfloat16>(__uint_as_float(x[2]) * inv, __uint_as_float(x[3]) * inv);
                            o.z = pack2<__nv_bfloat16>(__uint_as_float(x[4]) * inv, __uint_as_float(x[5]) * inv);
                            o.w = pack2<__nv_bfloat16>(__uint_as_float(x[6]) * inv, __uint_as_float(x[7]) * inv);
                            *reinterpret_cast<uint4*>(st + lane * 128 + ((q4 ^ (lane & 7)) << 4)) = o;
                        }
                    }
                    __syncwarp();
#pragma unroll 1
                    for (int i = 0; i < 8; ++i) {
                        const int row = 4 * i + (lane >> 3);
                        const int R = wq * 32 + row;
                        if (R < rows_here) {
                            const int2 dm = rowmap[R];
                            char* dst = static_cast<char*>(a.out) + (((int64_t)(it.q0 + it.tok0 + dm.x) * a.o_rs + (int64_t)(head0 + dm.y) * HD) << 1);
                            const uint32_t so = row * 128 + (((lane & 7) ^ (row & 7)) << 4);
                            const uint4 o0 = *reinterpret_cast<const uint4*>(stage + so);
                            const uint4 o1 = *reinterpret_cast<const uint4*>(stage + 4 * STAGE_WARP_BYTES + so);
                            *reinterpret_cast<uint4*>(dst + (lane & 7) * 16) = o0;
                            *reinterpret_cast<uint4*>(dst + 128 + (lane & 7) * 16) = o1;
                        }
                    }
                    __syncwarp();
                } else {
                    const int2 my_row = rowmap[L];
                    const int64_t tok = it.q0 + it.tok0 + (row_valid ? my_row.x : 0);
                    const int64_t head = head0 + (row_valid ? my_row.y : 0);
                    const int64_t e = ((int64_t)it.split * a.total_q + tok) * a.hq + head;
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        uint32_t v[32];
                        tmem_ld32(tO + c * 32, v);
                        tmem_ld_wait();
                        if (c == 3) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive_cluster(bar0(B_OFREE));
                        }
                        if (!row_valid) continue;
                        float4* dst = reinterpret_cast<float4*>(a.ws_o + e * HD + c * 32);
#pragma unroll
                        for (int q4 = 0; q4 < 8; ++q4)
                            dst[q4] = make_float4(__uint_as_float(v[q4 * 4 + 0]) * inv, __uint_as_float(v[q4 * 4 + 1]) * inv,
                                                  __uint_as_float(v[q4 * 4 + 2]) * inv, __uint_as_float(v[q4 * 4 + 3]) * inv);
                    }
                    if (row_valid) a.ws_lse[e] = l_run > 0.f ? m_ref + log2f(l_run) : -INFINITY;
                }
            } else {
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(bar0(B_OFREE));
            }
            ++done;
        }
        mbar_arrive(bar(B_EPIDONE));   // (release: output rows and flags are written)
    } else {
    reg_dec<HELPER_REGS>();
    if (warp == KLOAD_WARP || warp == VLOAD_WARP) {
        // =========================== loaders ===========================
        // K loader: rows [64 rank, 64 rank + 64) of every tile, all 128 head_dim columns (two swizzled regions of
        // [64][64]).  V loader: all 128 rows, head_dim columns [64 rank, 64 rank + 64) (one region of [128][64]).
        // The common tile (inside the cached prefix, one box per region) is lane 0's business alone and kept short:
        // ring position and page are tracked incrementally, the page id comes from the record.  Every other tile
        // (the end of the prefix, in-flight rows, small pages) takes the general path with the whole warp.
        const int which = warp == VLOAD_WARP;
        int32_t* bt_base = reinterpret_cast<int32_t*>(gbase + OFF_BT) + which * BT_SLOTS;
        const int stages = which ? VSTAGES : KSTAGES;
        const int row_lo = which ? 0 : K_ROWS * rank;          // first tile row this loader fetches
        const int rows_mine = which ? TILE_N : K_ROWS;
        const int c0_tma = which ? 64 * rank : 0;              // first head_dim column of its boxes
        const int box_rows0 = which ? a.tma_box_rows : min(a.tma_box_rows, K_ROWS);
        const int lvl0 = which ? a.tma_lvl0 : max(a.tma_lvl0, 1);   // level of the largest cache box this loader uses
        const CUtensorMap* lvl_maps = which ? maps.vc : maps.kc;
        const int page_size = a.page_size;
        const bool one_box_geom = box_rows0 == rows_mine && page_size % TILE_N == 0;   // a whole tile part is one box (pair)
        const int tiles_per_page = page_size / TILE_N;         // used only with one_box_geom
        const uint32_t bar_full0 = bar(which ? B_VFULL : B_KFULL), bar_empty0 = bar(which ? B_VEMPTY : B_KEMPTY);
        const uint32_t ring0 = which ? sV : sK;
        const uint32_t stage_bytes = which ? V_STAGE : K_STAGE;
        int stage = 0;            // ring position of the next tile
        uint32_t par_empty = 1;   // parity of "this slot is free" for the next tile (the first pass finds every slot free)
        bool alive = true;
#pragma unroll 1
        for (int round = 0; round < n_rounds && alive; ++round) {
            const SchedRec* rec = rec_of(round);
            const Item it = view_item(a, rec, rank);
            if (!it.valid) continue;
            const int n = it.n, ctx = it.ctx, kvh = it.kvh;
            const int32_t* bt_g = a.block_tables + (int64_t)it.seq * a.bt_stride;
            // Page ids: the record holds the last n_pages of the range; a longer item's earlier ids are copied to shared
            // memory in the background (4-byte cp.async) and first read many tiles later.
            const int early = min(it.first_page, BT_SLOTS);
            bool early_ready = early == 0;
            __syncwarp();
            for (int j = lane; j < early; j += 32)
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(bt_base + j)), "l"(bt_g + j) : "memory");
            const int first_page = it.first_page, n_pages = it.n_pages;
            auto page_id = [&](int j) -> int {
                if ((unsigned)(j - first_page) < (unsigned)n_pages) return rec->pages[j - first_page];
                if (j >= a.max_blocks) return -1;
                if (j < early) return bt_base[j];
                return bt_g[j];
            };
            // (page, tile inside the page) of the item's last tile; the walk goes n-2, n-1, n-3, n-4, ..., 0
            int pj_hi = 0, sub_hi = 0;
            if (one_box_geom) { pj_hi = (it.t0 + n - 1) / tiles_per_page; sub_hi = (it.t0 + n - 1) - pj_hi * tiles_per_page; }
            int pj_w = pj_hi, sub_w = sub_hi;     // walking position
#pragma unroll 1
            for (int jj = 0; jj < n && alive; ++jj) {
                const int tl = tile_of(jj, n);
                // walking position -> tile tl: jj = 0 steps back from the last tile (unless it is the only one), jj = 1
                // is the last tile itself, from jj = 2 on every tile is one step before the previous walking position
                int pj = pj_hi, sub = sub_hi;
                if (jj != 1 && n >= 2) {
                    if (--sub_w < 0) { sub_w = tiles_per_page - 1; --pj_w; }
                    pj = pj_w; sub = sub_w;
                }
                const int p0 = (it.t0 + tl) * TILE_N + row_lo;   // first key this loader fetches
                const uint32_t full = bar_full0 + 8u * stage;
                const uint32_t d0 = ring0 + stage * stage_bytes;
                if (one_box_geom && p0 + rows_mine <= ctx) {
                    // ---- the common tile: lane 0 alone ----
                    bool ok = true;
                    if (lane == 0) {
                        if (!early_ready && pj < early) {
                            asm volatile("cp.async.wait_all;\n" ::: "memory");
                            early_ready = true;
                        }
                        const int pid0 = page_id(pj);
                        const int prow = sub * TILE_N + row_lo;
                        ok = mbar_wait(bar_empty0 + 8u * stage, par_empty, abort_flag, 5 + which, jj);
                        if (ok) {
                            mbar_arrive_expect_tx(full, stage_bytes);
                            if (which) {
                                tma_load_4d(d0, &lvl_maps[lvl0], c0_tma, kvh, prow, pid0, full);
                            } else {
                                tma_load_4d(d0, &lvl_maps[lvl0], 0, kvh, prow, pid0, full);
                                tma_load_4d(d0 + K_REGION, &lvl_maps[lvl0], 64, kvh, prow, pid0, full);
                            }
                        }
                    }
                    early_ready = __shfl_sync(0xffffffffu, (int)early_ready, 0) != 0;
                    alive = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
                } else {
                    // ---- general path: the tile with the end of the prefix, in-flight rows, small pages.  Lane 0 cuts the
                    // cached rows and the in-flight rows of its part into boxes of falling size (128 >> level rows) ----
                    bool ok = true;
                    if (lane == 0) {
                        const int cr = max(min(ctx - p0, rows_mine), 0);        // cached rows of this part
                        const int ce = max(min(it.total - p0, rows_mine), 0);   // ... plus in-flight rows; the rest stays as it is
                        int pjg = p0 / page_size, prow = p0 - pjg * page_size;
                        if (!early_ready && pjg < early && cr > 0) {
                            asm volatile("cp.async.wait_all;\n" ::: "memory");
                            early_ready = true;
                        }
                        ok = mbar_wait(bar_empty0 + 8u * stage, par_empty, abort_flag, 5 + which, jj);
                        if (ok) {
                            if (ce == 0) {
                                mbar_arrive(full);
                            } else {
                                mbar_arrive_expect_tx(full, (uint32_t)ce * (which ? 128u : 256u));
                                int r = 0;
                                int lvl = lvl0;
#pragma unroll 1
                                for (int sz = box_rows0; sz >= 1; sz >>= 1, ++lvl) {
                                    while (cr - r >= sz) {
                                        const int pid = page_id(pjg);   // a bad id is out of bounds: zero fill
                                        if (which) {
                                            tma_load_4d(d0 + r * 128, &maps.vc[lvl], c0_tma, kvh, prow, pid, full);
                                        } else {
                                            tma_load_4d(d0 + r * 128, &maps.kc[lvl], 0, kvh, prow, pid, full);
                                            tma_load_4d(d0 + K_REGION + r * 128, &maps.kc[lvl], 64, kvh, prow, pid, full);
                                        }
                                        r += sz; prow += sz;
                                        if (prow >= page_size) { prow = 0; ++pjg; }   // boxes never straddle a page
                                    }
                                }
                                int tok = it.kv0 + (p0 + cr - ctx);   // first in-flight row of this part
                                lvl = which ? 0 : 1;
#pragma unroll 1
                                for (int sz = rows_mine; sz >= 1; sz >>= 1, ++lvl) {
                                    while (ce - r >= sz) {
                                        if (which) {
                                            tma_load_3d(d0 + r * 128, &maps.vn[lvl], c0_tma, kvh, tok, full);
                                        } else {
                                            tma_load_3d(d0 + r * 128, &maps.kn[lvl], 0, kvh, tok, full);
                                            tma_load_3d(d0 + K_REGION + r * 128, &maps.kn[lvl], 64, kvh, tok, full);
                                        }
                                        r += sz; tok += sz;
                                    }
                                }
                            }
                        }
                    }
                    early_ready = __shfl_sync(0xffffffffu, (int)early_ready, 0) != 0;
                    alive = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
                }
                if (++stage == stages) { stage = 0; par_empty ^= 1u; }
            }
            ++done; ck += n;
        }
        asm volatile("cp.async.wait_all;\n" ::: "memory");
        cluster_wait();   // the loaders touch nothing of the peer: they only complete the barrier phase they arrived on
    } else if (warp == QK_WARP) {
      // the first item's Q is requested before this warp waits for the peer
      int next_round = 0;    // first round not yet looked at by the Q prefetch
      int fetched = 0;       // valid items whose Q has been requested
      bool ok = true;
      auto fetch_q = [&](const Item& it, int i) {
          // Q of item i goes to buffer i & 1 and is requested one item ahead: as soon as the item that used the buffer
          // before (i - 2) has finished its Q K^T.
          const int qb = i & 1;
          if (i >= 2) ok = mbar_wait(bar(B_QEMPTY + qb), ((i - 2) >> 1) & 1, abort_flag, 6, -2);
          if (!ok) return;
          mbar_arrive_expect_tx(bar(B_QFULL + qb), 2u * (uint32_t)(a.q_tokens * G) * 128u);
          tma_load_3d(sQ + qb * Q_BYTES, &maps.q, 0, it.kvh * G, it.q0 + it.tok0, bar(B_QFULL + qb));
          tma_load_3d(sQ + qb * Q_BYTES + Q_REGION, &maps.q, 64, it.kvh * G, it.q0 + it.tok0, bar(B_QFULL + qb));
      };
      auto prefetch_upto = [&](int want) {   // request Q of valid items until `want` of them are requested
          while (ok && fetched < want && next_round < n_rounds) {
              const Item nx = view_item(a, rec_of(next_round), rank);
              ++next_round;
              if (!nx.valid) continue;
              fetch_q(nx, fetched);
              ++fetched;
          }
      };
      if (lane == 0) prefetch_upto(1);
      __syncwarp();
      cluster_wait();
      if (lane == 0) {
        // =========================== Q fetch; S = Q K^T issue (even CTA) or forwarding (odd CTA) ==================
        constexpr uint32_t ID_QK = instr_desc_pair(false);
#pragma unroll 1
        for (int round = 0; round < n_rounds && ok; ++round) {
            const Item it = view_item(a, rec_of(round), rank);
            if (!it.valid) continue;
            const int n = it.n;
            const int qb = done & 1;
            prefetch_upto(done + 1);   // this item's Q, unless the previous item already asked for it
            if (!ok) break;
            ok = mbar_wait(bar(B_QFULL + qb), (done >> 1) & 1, abort_flag, 7, -1);
            if (!ok) break;
            if (rank != 0) {
                mbar_arrive_cluster(bar0(B_QFULLP + qb));
#pragma unroll 1
                for (int k = 0; k < n && ok; ++k) {
                    const int idx = ck + k;
                    ok = mbar_wait(bar(B_KFULL + idx % KSTAGES), (idx / KSTAGES) & 1, abort_flag, 10, k);
                    if (!ok) break;
                    mbar_arrive_cluster(bar0(B_KFULLP + idx % KSTAGES));   // (TMA wrote the half: no proxy fence needed)
                    if (k == 0) prefetch_upto(done + 2);   // the next item's Q, into the other buffer
                }
            } else {
                ok = mbar_wait(bar(B_QFULLP + qb), (done >> 1) & 1, abort_flag, 7, -6);
                if (!ok) break;
                const uint32_t qaddr = sQ + qb * Q_BYTES;
#pragma unroll 1
                for (int k = 0; k < n && ok; ++k) {
                    const int idx = ck + k;
                    const int b = idx % NBUF, u = idx / NBUF;   // score buffer and its use count
                    const int st = idx % KSTAGES;
                    const uint32_t par = (idx / KSTAGES) & 1;
                    if (u >= 1) {   // the P V of the tile that used the buffer before must have run
                        ok = mbar_wait(bar(B_BUFFREE + b), (u - 1) & 1, abort_flag, 11, k);
                        if (!ok) break;
                    }
                    ok = mbar_wait(bar(B_KFULL + st), par, abort_flag, 10, k);
                    ok = ok && mbar_wait(bar(B_KFULLP + st), par, abort_flag, 13, k);
                    if (!ok) break;
                    tc_fence_after();   // K, V and Q were written by TMA copies: the async proxy already sees them
                    const uint32_t kb = sK + st * K_STAGE;
                    const uint32_t d = tmem + TM_S + b * 128;
                    const uint64_t dq = smem_desc(qaddr, 16, 1024), dk = smem_desc(kb, 16, 1024);
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks) {
                        const uint64_t oq = ((ks >> 2) * Q_REGION + (ks & 3) * 32) / 16;
                        const uint64_t okk = ((ks >> 2) * K_REGION + (ks & 3) * 32) / 16;
                        mma_ss_pair(d, dq + oq, dk + okk, ID_QK, ks > 0);
                    }
                    tc_commit_pair(bar(B_SFULL + b));
                    tc_commit_pair(bar(B_KEMPTY + st));
                    if (k == 0) prefetch_upto(done + 2);   // the next item's Q, into the other buffer
                }
                if (ok) tc_commit_pair(bar(B_QEMPTY + qb));
            }
            ++done; ck += n;
        }
      }
    } else if (warp == PV_WARP) {
      cluster_wait();
      if (lane == 0) {
        // =========================== O += P V issue (even CTA) or forwarding (odd CTA) ===========================
        constexpr uint32_t ID_PV = instr_desc_pair(true);
        bool ok = true;
#pragma unroll 1
        for (int round = 0; round < n_rounds && ok; ++round) {
            const Item it = view_item(a, rec_of(round), rank);
            if (!it.valid) continue;
            const int n = it.n;
            if (rank != 0) {
#pragma unroll 1
                for (int k = 0; k < n && ok; ++k) {
                    const int idx = ck + k;
                    ok = mbar_wait(bar(B_VFULL + idx % VSTAGES), (idx / VSTAGES) & 1, abort_flag, 8, k);
                    if (!ok) break;
                    mbar_arrive_cluster(bar0(B_VFULLP + idx % VSTAGES));
                }
            } else {
                if (done > 0) ok = mbar_wait(bar(B_OFREE), (done - 1) & 1, abort_flag, 8, -2);
#pragma unroll 1
                for (int k = 0; k < n && ok; ++k) {
                    const int idx = ck + k;
                    const int b = idx % NBUF, u = idx / NBUF;
                    const int st = idx % VSTAGES;
                    const uint32_t par = (idx / VSTAGES) & 1;
                    ok = mbar_wait(bar(B_VFULL + st), par, abort_flag, 8, k);
                    ok = ok && mbar_wait(bar(B_VFULLP + st), par, abort_flag, 14, k);
                    ok = ok && mbar_wait(bar(B_PFULL + b), u & 1, abort_flag, 9, k);
                    if (!ok) break;
                    tc_fence_after();   // K, V and Q were written by TMA copies: the async proxy already sees them
                    const uint32_t vb = sV + st * V_STAGE;
                    const uint32_t pa = tmem + TM_S + b * 128;   // P lies over the first 64 columns of the score buffer
                    const uint64_t dv = smem_desc(vb, V_STAGE, 1024);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        mma_ts_pair(tmem + TM_O, pa + kk * 8, dv + (uint64_t)(kk * 2048 / 16), ID_PV, (k > 0 || kk > 0) ? 1u : 0u);
                    tc_commit_local(bar(B_BUFFREE + b));
                    tc_commit_pair(bar(B_VEMPTY + st));
                }
                if (ok) tc_commit_pair(bar(B_OFULL));
            }
            ++done; ck += n;
        }
      }
    }
    }
    tc_fence_before();
    // ---- teardown ----
    __syncthreads();
    if (tid == 0 && *abort_flag != 0) {
        const int word = *abort_flag;
        if (atomicCAS(&g_status_pair[0], 0, 1) == 0) {
            g_status_pair[1] = (word >> 24) & 0xff; g_status_pair[2] = (int)(short)((word >> 8) & 0xffff);
            g_status_pair[3] = blockIdx.x;
        }
    }
    // neither CTA may retire (or free TMEM) while its peer's MMAs, commits or arrivals can still touch it
    cluster_arrive();
    cluster_wait();
    if (warp == QK_WARP) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;\n" ::"r"(tmem) : "memory");
    }
}

}  // namespace tc5p

int read_tc5_pair_status(int out[4]) {
    cudaError_t e = cudaMemcpyFromSymbol(out, tc5p::g_status_pair, sizeof(int) * 4);
    if (e != cudaSuccess) return fail(DLX_ERR_CUDA, "cudaMemcpyFromSymbol(g_status_pair): %s", cudaGetErrorString(e));
    int zero[4] = {0, 0, 0, 0};
    e = cudaMemcpyToSymbol(tc5p::g_status_pair, zero, sizeof(zero));
    if (e != cudaSuccess) return fail(DLX_ERR_CUDA, "cudaMemcpyToSymbol(g_status_pair): %s", cudaGetErrorString(e));
    return DLX_OK;
}

int launch_decode_tc5_pair(const DecodeArgs& a_in, cudaStream_t st) {
    static bool attr_done[16] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 16 || !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(tc5p::decode_attn_tc5_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             tc5p::SMEM_BYTES);
        if (e != cudaSuccess) return fail(DLX_ERR_CUDA, "cudaFuncSetAttribute(tc5 pair smem=%d): %s", tc5p::SMEM_BYTES, cudaGetErrorString(e));
        if (dev >= 0 && dev < 16) attr_done[dev] = true;
    }
    DecodeArgs a = a_in;
    tc5p::TmaMapsPair maps;
    memset(&maps, 0, sizeof(maps));
    const int ps = a.page_size;
    const bool fits = a.max_blocks > 0 && a.num_pages > 0 && ((ps % 128 == 0) || (128 % ps == 0 && ps % 8 == 0));
    const bool strides_ok = a.token_stride * 2 % 16 == 0 && a.page_stride * 2 % 16 == 0 &&
                            a.page_stride * 2 < (1ll << 40) && a.num_pages < (1ll << 31);
    if (!fits || !strides_ok || a.total_q <= 0 || a.q_rs * 2 % 16 != 0 || a.q_rs * 2 >= (1ll << 40) ||
        a.k_rs * 2 % 16 != 0 || a.v_rs * 2 % 16 != 0 || a.k_rs * 2 >= (1ll << 40) || a.v_rs * 2 >= (1ll << 40))
        return fail(DLX_ERR_UNSUPPORTED, "decode (pair kernel): page size %d or strides not served", ps);
    a.tma_box_rows = ps < 128 ? ps : 128;
    a.tma_lvl0 = 0;
    while ((128 >> a.tma_lvl0) > a.tma_box_rows) ++a.tma_lvl0;
    for (int lvl = 0; lvl < tc5p::LEVELS; ++lvl) {
        const int rows = 128 >> lvl;
        int rc = DLX_OK;
        if (rows <= ps) {   // caches: a box lies inside one page
            rc = tc5::tc5_cache_map(a.k_cache, a.page_stride, a.token_stride, a.num_pages, a.hkv, ps, rows, 4, &maps.kc[lvl]);
            if (rc == DLX_OK) rc = tc5::tc5_cache_map(a.v_cache, a.page_stride, a.token_stride, a.num_pages, a.hkv, ps, rows, 4, &maps.vc[lvl]);
        }
        // in-flight rows: {head_dim, Hkv, token}, box {64, 1, rows}
        if (rc == DLX_OK) rc = tc5::tc5_cache_map(a.k, a.k_rs, 0, a.total_kv, a.hkv, 1, rows, 3, &maps.kn[lvl]);
        if (rc == DLX_OK) rc = tc5::tc5_cache_map(a.v, a.v_rs, 0, a.total_kv, a.hkv, 1, rows, 3, &maps.vn[lvl]);
        if (rc != DLX_OK) return rc;
    }
    {
        const int rc = tc5::tc5_cache_map(a.q, a.q_rs, 0, a.total_q, a.hq, a.group, a.q_tokens, 3, &maps.q);
        if (rc != DLX_OK) return rc;
    }
    a.q_by_tma = 1;
    dim3 grid(2u * (unsigned)a.bins), block(tc5p::NUM_THREADS);
    tc5p::decode_attn_tc5_pair_kernel<<<grid, block, tc5p::SMEM_BYTES, st>>>(a, maps);
    return check_launch("decode_attn_tc5_pair_kernel");
}

}  // namespace dlx
