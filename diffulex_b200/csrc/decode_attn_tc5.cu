// Paged block-diffusion decode attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Shape served: head_dim 128, bf16, any number G <= 128 of query heads per KV head.  All G heads of a KV head are
// packed into the M dimension, so every K/V byte is read once per GROUP of heads.
//
// Work item = (sequence, KV head, block of query tokens, key-range split); a CTA takes 128 / G whole tokens of it
// (with more than 128 packed rows per KV head an item is two row blocks, run by the two neighbouring CTAs of a
// schedule bin).  The kernel is persistent: a CTA walks the records the schedule kernel placed in its bin
// (decode_sched.cu) and keeps every ring and barrier phase running across items, so the next item's Q/K/V land while
// the current one is finished.  Prefill attention is the same kernel with an empty context.
//
// Warp roles (512 threads; after the split the warpgroups resize their register files with setmaxnreg):
//   warps 0-7    two softmax warpgroups over the SAME 128 rows (thread <-> TMEM lane <-> query row), taking
//                alternate key tiles: S -> registers, P = exp2(s * scale - m_ref) as bf16 -> TMEM.  m_ref is the row
//                maximum of the item's first tile: later tiles compute no maximum and no accumulator rescale ever
//                runs.  An item whose exponents leave the safe range (tile row sum above 2^90, final row sum below
//                2^-80) is marked and recomputed exactly before the CTA retires
//   warp 8, 9    K loader, V loader: one lane each, everything by TMA.  Tiles (128 keys) inside the cached prefix:
//                cp.async.bulk.tensor, 4-D map {hd, Hkv, page row, page}, 128-byte swizzle, plain per-CTA loads.
//                The tile with the end of the prefix and the in-flight rows: boxes of 128 >> level rows from
//                per-level maps, starting at any row of the tile
//   warp 10      one thread issues S = Q K^T (tcgen05.mma, SS form) and fetches Q (TMA, one box per head_dim half);
//                the warp also allocates and frees TMEM
//   warp 11      one thread issues O += P V (TS form: P from TMEM, V as MN-major B operand from the [key][hd] tile)
//   warps 12-15  epilogue warpgroup: O / l -> global through a swizzled staging buffer (coalesced rows)
// TMEM (512 columns): S[2] (128 fp32 columns each) | P[2] (64 columns = 128 bf16 each) | O (128).
//
// Every mbarrier wait is bounded; on expiry the CTA raises an abort word, everyone drains, the place is copied to a
// device status word, TMEM is freed and the CTA returns (no trap, the context stays usable).
//
// Reference semantics: diffulex_kernel/python/dllm_flash_attn.py:163-347 and :632-637.
#include <cuda.h>  // CUtensorMap and the cuTensorMapEncodeTiled prototype (resolved at run time, no libcuda link)

#include <string.h>

#include <mutex>
#include <vector>

#include "dlx_common.cuh"
#include "decode_attn.cuh"
#include "tc5_common.cuh"

namespace dlx {
namespace tc5 {

constexpr int HD = 128;
constexpr int TILE_M = 128;               // packed query rows per work item (TMEM lanes)
constexpr int TILE_N = 128;               // keys per K/V tile
constexpr int REGION = 128 * 128;         // [128 rows][64 bf16] 128B-swizzled block: 16 KiB
constexpr int Q_BYTES = 2 * REGION;       // one Q tile, 2 head_dim halves
constexpr int ITEM_BYTES = 2 * REGION;    // one K tile or one V tile
#ifndef DLX_KSTAGES
#define DLX_KSTAGES 2
#define DLX_VSTAGES 2
#endif
// A ring slot is refilled when its tile has been consumed.  Two stages each, measured: one stage serialises copy and
// MMA (+30 % run time), a third K or V stage is slower than two (more copies in flight at the item switches, where the
// memory system is the contended resource).
constexpr int KSTAGES = DLX_KSTAGES, VSTAGES = DLX_VSTAGES;
constexpr int OFF_K = Q_BYTES;
constexpr int OFF_V = OFF_K + KSTAGES * ITEM_BYTES;
constexpr int OFF_BAR = OFF_V + VSTAGES * ITEM_BYTES;
constexpr int OFF_BT = OFF_BAR + 512;              // page ids of a long item that its record does not hold, one copy per loader warp
constexpr int BT_SLOTS = 512;                      // 2 KiB per loader warp
constexpr int OFF_XCH = OFF_BT + 2 * BT_SLOTS * 4; // 8 x 128 floats: two slots of row references; two slots of (row sums x 2, reference)
constexpr int OFF_STAGE = OFF_XCH + 8 * 128 * 4;   // output staging: 32 rows x 128 bytes per epilogue warp
constexpr int STAGE_WARP_BYTES = 32 * 128;
constexpr int OFF_ROWMAP = OFF_STAGE + 4 * STAGE_WARP_BYTES;   // int2[128]: (row / group, row % group) of a block's rows
constexpr int OFF_ITEMS = OFF_ROWMAP + 128 * 8;   // this CTA's schedule records, one per round
constexpr int MAX_ROUNDS = 48;                     // records kept in shared memory; later rounds are read from global
constexpr int OFF_FLAGS = OFF_ITEMS + MAX_ROUNDS * (int)sizeof(SchedRec);  // one bit per round: the item has to be computed again, exactly
constexpr int FLAG_WORDS = 128;                    // 4096 rounds; later rounds share the bits
constexpr int OFF_ARGS = OFF_FLAGS + FLAG_WORDS * 4;   // a copy of the argument block (256 bytes)
constexpr int SMEM_BYTES = OFF_ARGS + 320 + 1024;  // + slack for 1024-byte alignment
static_assert(sizeof(DecodeArgs) <= 320, "argument block copy");
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
// P = 2^(s*scale*log2e - m_ref) with m_ref fixed by the first tile.  Floating point keeps full relative
// precision however far later scores lie from m_ref, until 2^x leaves the bf16/fp32 range: an item in which a tile's
// row sum of P exceeds DLX_SUM_HIGH, or whose final row sum falls below DLX_SUM_LOW although the row sees keys, is
// flagged and computed again with a running maximum (tc5_common.cuh) before the CTA retires.
constexpr int NUM_THREADS = 512;
// Registers per thread after the roles split (the kernel starts with 65536 / 512 = 128 each): the four helper warps
// and the epilogue warpgroup give registers back, the two softmax warpgroups (a row of 128 scores each) take them.
#ifndef DLX_SOFTMAX_REGS
#define DLX_SOFTMAX_REGS 176
#define DLX_HELPER_REGS 56
#define DLX_EPI_REGS 104
#endif
constexpr int SOFTMAX_REGS = DLX_SOFTMAX_REGS, HELPER_REGS = DLX_HELPER_REGS, EPI_REGS = DLX_EPI_REGS;
static_assert(2 * SOFTMAX_REGS + HELPER_REGS + EPI_REGS <= 512, "register budget");
constexpr int EPI_WARP0 = 12;
constexpr int KLOAD_WARP = 8, VLOAD_WARP = 9, QK_WARP = 10, PV_WARP = 11;
// TMEM columns (512): two S buffers of 128 fp32 columns, two P buffers of 64 columns (128 bf16 keys), O
constexpr uint32_t TM_S = 0, TM_P = 256, TM_O = 384;

// barrier slots (8 bytes each) at OFF_BAR
enum {
    B_QFULL = 0, B_KFULL = 1, B_VFULL = 4, B_KEMPTY = 7, B_VEMPTY = 10,   // K and V: up to 3 stages each
    B_SFULL = 13,   // [S buffer]
    B_PFULL = 15,   // [P buffer]: the softmax may be two tiles ahead of the P V that consumes its output and an
                    // mbarrier can only be one phase ahead of its waiter, hence one barrier per buffer
    B_OFULL = 17,
    B_OFREE = 18,   // the epilogue has O in registers: the next item's P V may overwrite the accumulator
    B_QEMPTY = 19,  // every Q K^T of the item has run: the next item's Q may be loaded
    B_SFREE = 20,   // [S buffer]: its scores are in the softmax warpgroup's registers, Q K^T may overwrite it
    B_PFREE = 22,   // [P buffer]: the P V that read it has run, the warpgroup may write the next P into it
    // Rings of two slots between the warpgroups, one use per item with two or more tiles:
    B_MRFULL = 24,  // [slot] the row references of the item's first tile are in shared memory
    B_MREMPTY = 26, // [slot] ... and have been read by the owner of the item's second tile
    B_LSFULL = 28,  // [slot] both warpgroups' partial row sums of an item are in shared memory (one use per item)
    B_LSEMPTY = 30, // [slot] ... and the epilogue warpgroup has read them
    B_EPIDONE = 32, // the epilogue warpgroup has written its last output row (128 arrivals, once per launch)
    B_COUNT = 33
};

__device__ int g_status[4];  // [0] bit 0: a bounded wait expired; [1] wait site, [2] tile, [3] CTA


// One unit of work of a CTA: (sequence, KV head, block of 128 / group query tokens, key-range split), read from a
// record of the launch's schedule (decode_sched.cu).
struct alignas(8) Item {
    bool valid;        // has rows and at least one key tile
    bool empty_split;  // has rows but this split's key range is empty: only -inf log-sum-exps are written
    int seq, kvh, split;
    int q0, ctx, kv0, nnew, total;
    int row0, rows_here, tok0;   // first packed row (= tok0 * group), valid rows, first token of the block
    int cta_limit, full_until;
    int t0, n;
    int first_page, n_pages;     // the record holds the ids of pages [first_page, first_page + n_pages)
};

__device__ __forceinline__ Item load_item(const DecodeArgs& a, const SchedRec* r, int rank) {
    Item it;
    const int4 w0 = *reinterpret_cast<const int4*>(&r->seq);
    const int4 w1 = *reinterpret_cast<const int4*>(&r->q0);
    const int4 w2 = *reinterpret_cast<const int4*>(&r->nnew);
    it.seq = w0.x; it.kvh = w0.y; it.split = w0.w;
    it.q0 = w1.x; it.ctx = w1.z; it.kv0 = w1.w;
    it.nnew = w2.x; it.t0 = w2.y; it.n = w2.z;
    it.valid = (w2.w & SCHED_VALID) != 0;
    it.empty_split = (w2.w & SCHED_EMPTY_SPLIT) != 0;
    it.total = it.ctx + it.nnew;
    it.first_page = r->first_page; it.n_pages = r->n_pages;
    // A block holds q_tokens = 128 / group whole tokens (all `group` heads of each), so that its Q rows are one box
    // of the [token][head][head_dim] tensor; packed row r of the (sequence, KV head) is token r / group, head r % group.
    // With two CTAs per schedule bin an item is two such blocks and CTA `rank` of the bin takes the rank-th one; a
    // CTA whose block lies past the end of a short sequence has nothing to do for the item.
    it.tok0 = w0.z * a.tokens_per_item + rank * a.q_tokens;
    it.row0 = it.tok0 * a.group;
    it.rows_here = max(min(w1.y - it.tok0, a.q_tokens), 0) * a.group;
    if (it.rows_here == 0) { it.valid = false; it.empty_split = false; }
    it.cta_limit = r->limit;
    it.full_until = it.total;
    if (a.mask_mode == DLX_MASK_BLOCK_CAUSAL) it.full_until = it.ctx + min(it.nnew, (it.tok0 / a.dbs + 1) * a.dbs);
    return it;
}

// Order of an item's n key tiles: n-2, n-1, n-3, n-4, ..., 0.  The last tile (end of the cached prefix plus the
// in-flight rows) is the slow one to fetch (row-wise copies) and needs the mask pre-pass: near the front, its fetch
// overlaps the previous item's last tiles instead of sitting at the item's end with nothing behind it to hide it.
// It is not the very first, because the first tile's row maxima become the softmax reference that the other
// warpgroup waits for: a full tile delivers them sooner, while the other warpgroup masks the last tile.
__device__ __forceinline__ int tile_of(int jj, int n) { return n - 1 - ((jj < 2 && n >= 2) ? (jj ^ 1) : jj); }

// Tensor maps of one launch, by level l = 0..7: boxes of 128 >> l rows x 64 head_dim columns.  kc / vc: the caches as
// {head_dim, Hkv, page row, page}; kn / vn: the in-flight rows as {head_dim, Hkv, token}.  Levels whose box exceeds a
// page (caches) are unused.  Any run of rows is a few boxes of falling size; a box may start at any row of a tile:
// the 128-byte swizzle of a copy follows the shared-memory address it writes.
constexpr int LEVELS = 8;
struct TmaMaps {
    CUtensorMap kc[LEVELS], vc[LEVELS], kn[LEVELS], vn[LEVELS];
    CUtensorMap q;
};

// Persistent kernel: one CTA per SM walks its rounds of the (longest-first) item list.  Every role keeps running
// counters for the rings and buffers, so the pipeline never drains between items: while the softmax warpgroups
// finish item i the loaders already fetch K / V of item i + 1 and the Q K^T issuer fills its first two S buffers.
// The CTA's first MAX_ROUNDS records are decoded once into a shared-memory table; later rounds (rare) are decoded from
// the global records by every role.
__global__ void __launch_bounds__(NUM_THREADS, 1)
decode_attn_tc5_kernel(const DecodeArgs a_param, const __grid_constant__ TmaMaps maps) {
    extern __shared__ unsigned char smem_raw[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // This CTA's records: placed by the schedule kernel (longest-processing-time greedy, longest item first).  Two
    // neighbouring CTAs walk the same list when an item is two row blocks: they run side by side, and the second
    // reader of a K / V tile finds it in L2.  The offsets are asked for first: their trip to memory overlaps the set-up.
    const int bin = (int)blockIdx.x / a_param.group_ctas, rank = (int)blockIdx.x - bin * a_param.group_ctas;
    const int rec0 = a_param.sched_off[bin];
    const int n_rounds = a_param.sched_off[bin + 1] - rec0;

    const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
    unsigned char* gbase = smem_raw + (sbase - smem_u32(smem_raw));
    const uint32_t sQ = sbase, sK = sbase + OFF_K, sV = sbase + OFF_V, sBar = sbase + OFF_BAR;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + OFF_BAR + 8 * B_COUNT);
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + OFF_BAR + 8 * B_COUNT + 8);
    auto bar = [&](int slot) { return sBar + 8u * slot; };
    // The argument block is read from a shared-memory copy: fields that only the per-item code touches (output
    // pointer, strides, mask mode ...) fall out of the constant cache between items, and every such miss was a trip
    // to L2 in the middle of an item switch.
    {
        const uint32_t* src = reinterpret_cast<const uint32_t*>(&a_param);
        uint32_t* dst = reinterpret_cast<uint32_t*>(gbase + OFF_ARGS);
        if (tid < (int)(sizeof(DecodeArgs) / 4)) dst[tid] = src[tid];   // visible after the set-up barrier below
    }
    const DecodeArgs& a = *reinterpret_cast<const DecodeArgs*>(gbase + OFF_ARGS);   // for use AFTER the set-up barrier
    const int G = a_param.group;

    if (tid < B_COUNT) {   // one barrier per thread; expected arrivals by slot
        uint32_t count = 1;
        if (tid >= B_PFULL && tid < B_PFULL + 2) count = 128;
        else if (tid >= B_SFREE && tid < B_SFREE + 2) count = 128;
        else if (tid == B_OFREE || tid == B_EPIDONE) count = 128;
        else if (tid >= B_MRFULL && tid < B_MRFULL + 2) count = 128;
        else if (tid >= B_MREMPTY && tid < B_MREMPTY + 2) count = 128;
        else if (tid >= B_LSFULL && tid < B_LSFULL + 2) count = 256;
        else if (tid >= B_LSEMPTY && tid < B_LSEMPTY + 2) count = 128;
        mbar_init(bar(tid), count);
        if (tid == 0) *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    const SchedRec* recs_g = a_param.sched_recs + rec0;
    SchedRec* recs_s = reinterpret_cast<SchedRec*>(gbase + OFF_ITEMS);
    auto rec_of = [&](int k) -> const SchedRec* { return k < MAX_ROUNDS ? recs_s + k : recs_g + k; };
    // Division by the (runtime) group size is slow; a block's rows always start at a whole token, so the split of a
    // row index into (token, head) is the same for every item and is tabulated once.
    int2* rowmap = reinterpret_cast<int2*>(gbase + OFF_ROWMAP);
    if (tid >= 128 && tid < 256) rowmap[tid - 128] = make_int2((tid - 128) / G, (tid - 128) % G);
    uint32_t* redo_flags = reinterpret_cast<uint32_t*>(gbase + OFF_FLAGS);
    if (tid >= 256 && tid < 256 + FLAG_WORDS) redo_flags[tid - 256] = 0;
    auto get_item = [&](int k) { return load_item(a, rec_of(k), rank); };
    {
        // Q rows past the last whole token of a block (e.g. rows 126, 127 for 7 heads per KV head) are never written
        // by a Q box: zero them once, so that the unused TMEM lanes only ever see finite scores.
        const int rows_used = a_param.q_tokens * G;
        for (int i = tid; i < (TILE_M - rows_used) * 16; i += NUM_THREADS) {
            const int row = rows_used + (i >> 4), chunk = i & 15;
            *reinterpret_cast<uint4*>(gbase + (chunk >> 3) * REGION + row * 128 + ((chunk & 7) << 4)) = make_uint4(0, 0, 0, 0);
        }
        // The K and V rings start out as zeros: rows that no copy writes (past the last key of a tail tile) must hold
        // finite values, because 0 x NaN would poison the P V product.
        for (int i = tid; i < (KSTAGES + VSTAGES) * ITEM_BYTES / 16; i += NUM_THREADS)
            *reinterpret_cast<uint4*>(gbase + OFF_K + i * 16) = make_uint4(0, 0, 0, 0);
        fence_async_proxy();
    }
    {   // the records, after everything that does not need them (the offsets have had time to arrive)
        const int n_tab = min(n_rounds, MAX_ROUNDS);
        const uint4* src = reinterpret_cast<const uint4*>(recs_g);
        uint4* dst = reinterpret_cast<uint4*>(recs_s);
        for (int i = tid; i < n_tab * (int)(sizeof(SchedRec) / 16); i += NUM_THREADS) dst[i] = src[i];
    }
    if (warp == QK_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;\n" ::"r"(sBar + 8u * B_COUNT + 8u) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Running totals over the valid items this CTA has finished (identical in every role):
    //   done = items, ck = key tiles.  Tile k of an item has running index ck + k: S/P buffer (ck + k) & 1, and
    //   (ck + k) >> 1 earlier uses of that buffer.
    int done = 0, ck = 0;

    if (warp < 8) {
        reg_inc<SOFTMAX_REGS>();
        // =========================== softmax warpgroups ===========================
        // Two warpgroups own the same 128 rows (thread = row = TMEM lane) and take alternate key tiles, counted ACROSS
        // items: the tile with running index g belongs to warpgroup g & 1, which always works on S buffer / P buffer
        // g & 1.  One warp per SM sub-partition cannot issue fast enough to keep the MUFU unit busy; two can, and
        // while one waits for its S the other works.  Both scale their P by the SAME per-row reference m_ref = scaled
        // row maximum of the item's first tile (a fixed reference is exact as long as exponents stay in range; items
        // that leave it are recomputed), so their outputs add up in the one O accumulator and their row sums add up at the end.
        // Neither waits for an item's output to be written: that is the epilogue warpgroup's job.
        const int w = warp >> 2;                       // warpgroup = parity of the running tile index
        const int L = tid & 127;                       // TMEM lane == row inside the tile
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const uint32_t tS = lane_base + TM_S + w * 128, tP = lane_base + TM_P + w * 64;
        float* xm = reinterpret_cast<float*>(gbase + OFF_XCH);    // [2][128] row references, ring of two items
        float* xs = xm + 256;                                     // [2][3][128] per item: row sums of each warpgroup, reference
        const float sl2 = a.scale_log2;
        int mr = 0;                                    // items with two or more tiles so far: position in the m_ref ring
        bool alive = true;
#pragma unroll 1
        for (int round = 0; round < n_rounds && alive; ++round) {
            const Item it = get_item(round);
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
            const int2 my_row = rowmap[L];                 // packed row L of the block: token tok0 + x, head head0 + y
            const bool warp_valid = (warp & 3) * 32 < rows_here;  // any valid row in this warp?
            const bool row_valid = L < rows_here;
            const int jj_first = (w ^ ck) & 1;             // this warpgroup's first tile of the item (0 or 1)
            const bool multi = n >= 2;                     // both warpgroups have tiles: reference and sums are exchanged
            const int slot = mr & 1;
            const uint32_t ring_par = (mr >> 1) & 1;
            int limit = it.total;
            if (a.mask_mode == DLX_MASK_BLOCK_CAUSAL && row_valid) limit = it.ctx + min(it.nnew, ((it.tok0 + my_row.x) / a.dbs + 1) * a.dbs);
            float m_ref = 0.f, l_run = 0.f;
            bool out_of_range = false;
#pragma unroll 1
            for (int jj = jj_first; jj < n && alive; jj += 2) {
                const int u = (ck + jj) >> 1;              // use count of this warpgroup's buffers: phase of their barriers
                bool ok = mbar_wait(bar(B_SFULL + w), u & 1, abort_flag, 1 + w, jj);
                if (!__all_sync(0xffffffffu, ok)) { alive = false; break; }
                tc_fence_after();
                // Ring bookkeeping of the row reference (all warps, valid rows or not, keep the barrier counts whole):
                // the owner of tile 0 fills the slot, the owner of tile 1 drains it.
                if (multi && jj == 0 && mr >= 2) {
                    bool oke = mbar_wait(bar(B_MREMPTY + slot), ring_par ^ 1, abort_flag, 4, -3);
                    if (!__all_sync(0xffffffffu, oke)) { alive = false; break; }
                }
                if (warp_valid) {
                    const int key0 = (it.t0 + tile_of(jj, n)) * TILE_N;
                    // the whole S row of this thread: 128 fp32 scores in registers, one TMEM round trip
                    uint32_t v[4][32];
                    tmem_ld32(tS, v[0]); tmem_ld32(tS + 32, v[1]); tmem_ld32(tS + 64, v[2]); tmem_ld32(tS + 96, v[3]);
                    tmem_ld_wait();
                    tc_fence_before();
                    mbar_arrive(bar(B_SFREE + w));   // S is in registers: the next Q K^T into this buffer may start now
                    float mx_any = -INFINITY;   // first tile only: row maximum over every real key, hidden ones included
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
                        // First tile: its row maximum fixes the reference (later tiles compute no maximum at all).  A row
                        // that sees none of this tile's keys (block-causal rows of an early block; the first tile is a
                        // late key tile) takes the maximum over the tile's hidden keys instead.  0 for a padding row.
                        float mx4[4];  // four independent chains: the max is latency-, not issue-bound
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
                            mbar_arrive(bar(B_MRFULL + slot));   // the other warpgroup needs it before its first exponential
                        }
                    } else if (jj == 1) {  // the other warpgroup's first tile set the reference
                        bool okm = mbar_wait(bar(B_MRFULL + slot), ring_par, abort_flag, 4, 0);
                        if (!__all_sync(0xffffffffu, okm)) { alive = false; break; }
                        m_ref = xm[slot * 128 + L];
                        mbar_arrive(bar(B_MREMPTY + slot));
                    }
                    // P = exp2(s*scale - m_ref) as bf16 into this warpgroup's P buffer
                    // P = exp2(s * scale - m_ref) as bf16.  The first half of the row is kept in registers: the exponentials
                    // do not need the P buffer, only the stores do, and half a row later the P V that last read the
                    // buffer has run (waiting for it up front would stall here, a whole row in registers costs too many)
                    float2 lacc0 = make_float2(0.f, 0.f), lacc1 = make_float2(0.f, 0.f);
                    const float2 sl2v = make_float2(sl2, sl2), negm = make_float2(-m_ref, -m_ref);
                    uint32_t pk[2][16];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        uint32_t pc[16];
#pragma unroll
                        for (int e = 0; e < 32; e += 2) {
                            const float2 x = __ffma2_rn(make_float2(__uint_as_float(v[c][e]), __uint_as_float(v[c][e + 1])), sl2v, negm);
                            const float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
                            if ((e >> 1) & 1) lacc1 = __fadd2_rn(lacc1, p); else lacc0 = __fadd2_rn(lacc0, p);
                            if (c < 2) pk[c][e >> 1] = pack2<__nv_bfloat16>(p.x, p.y); else pc[e >> 1] = pack2<__nv_bfloat16>(p.x, p.y);
                        }
                        if (c == 1) {
                            if (u >= 1) {
                                // Q K^T does not wait for P V, so this warpgroup could lap the tensor pipe: the previous P in
                                // this buffer must have been consumed before the next one goes in
                                bool okp = mbar_wait(bar(B_PFREE + w), (u - 1) & 1, abort_flag, 4, jj);
                                if (!__all_sync(0xffffffffu, okp)) { alive = false; break; }
                                tc_fence_after();
                            }
                            tmem_st16(tP, pk[0]);
                            tmem_st16(tP + 16, pk[1]);
                        } else if (c >= 2) {
                            tmem_st16(tP + c * 16, pc);
                        }
                    }
                    if (!alive) break;
                    lacc0 = __fadd2_rn(lacc0, lacc1);
                    const float tsum = lacc0.x + lacc0.y;
                    out_of_range |= !(tsum <= DLX_SUM_HIGH);   // exponent range left (also catches NaN): redo the item
                    l_run += tsum;
                    tmem_st_wait();
                } else {
                    // A warp without valid rows only keeps the barrier counts whole.  It must not run ahead either: its
                    // arrival for a later tile landing in the phase of this one would complete that phase early.
                    if (multi && jj == 0) mbar_arrive(bar(B_MRFULL + slot));
                    if (jj == 1) {
                        bool okm = mbar_wait(bar(B_MRFULL + slot), ring_par, abort_flag, 4, 0);
                        if (!__all_sync(0xffffffffu, okm)) { alive = false; break; }
                        mbar_arrive(bar(B_MREMPTY + slot));
                    }
                    mbar_arrive(bar(B_SFREE + w));
                    if (u >= 1) {
                        bool okp = mbar_wait(bar(B_PFREE + w), (u - 1) & 1, abort_flag, 4, jj);
                        if (!__all_sync(0xffffffffu, okp)) { alive = false; break; }
                    }
                }
                tc_fence_before();
                mbar_arrive(bar(B_PFULL + w));
            }
            if (!alive) break;
            if (__any_sync(0xffffffffu, out_of_range && row_valid) && lane == 0)
                atomicOr(&redo_flags[(round >> 5) & (FLAG_WORDS - 1)], 1u << (round & 31));
            // ---- hand the item over to the epilogue warpgroup: partial row sums (and the reference) through a ring of
            // two slots, one use per item.  A warpgroup without a tile in the item (one-tile items) hands over a zero.
            {
                const int ls = done & 1;
                if (done >= 2) {
                    bool oke = mbar_wait(bar(B_LSEMPTY + ls), ((done >> 1) & 1) ^ 1, abort_flag, 4, -4);
                    if (!__all_sync(0xffffffffu, oke)) { alive = false; break; }
                }
                xs[ls * 384 + w * 128 + L] = l_run;
                if (jj_first == 0) xs[ls * 384 + 256 + L] = m_ref;   // the owner of tile 0 set it
                mbar_arrive(bar(B_LSFULL + ls));
            }
            ++done; ck += n; mr += multi ? 1 : 0;
        }
        // ---- items that left the fixed reference's range: their rows again, exactly ----
        // The epilogue warpgroup signals its last output row (and its last flag); by then every
        // MMA has completed (its last O_full), so the K / V rings are idle and serve as scratch.
        const bool epi_done = mbar_wait(bar(B_EPIDONE), 0, abort_flag, 15, -7);
        if (alive && epi_done && *abort_flag == 0) {
            float* scratch = reinterpret_cast<float*>(gbase + OFF_K);
            static_assert(8 * (REDO_CHUNK + HD) * 4 <= (KSTAGES + VSTAGES) * ITEM_BYTES, "redo scratch");
#pragma unroll 1
            const int flag_words = min((n_rounds + 31) >> 5, FLAG_WORDS);
#pragma unroll 1
            for (int wd = 0; wd < flag_words; ++wd) {
                uint32_t bits = redo_flags[wd];
                while (bits) {
                    const int b = __ffs(bits) - 1;
                    bits &= bits - 1;
                    for (int round = wd * 32 + b; round < n_rounds; round += 32 * FLAG_WORDS) {
                        const Item it = get_item(round);
                        if (it.valid && it.rows_here > 0) redo_item_exact(a, it, warp, lane, scratch);
                    }
                }
            }
        }
    } else if (warp >= EPI_WARP0) {
        // =========================== epilogue warpgroup: O / l -> global ===========================
        // Its own four warps (TMEM lanes 32 (warp % 4) ..), so that the softmax warpgroups go from an item's last
        // tile straight to the next item's first: the output of item i is written while item i + 1 is computed.
        reg_dec<EPI_REGS>();
        const int L = tid & 127, wq = warp & 3;
        const uint32_t tO = tmem + ((uint32_t)(wq * 32) << 16) + TM_O;
        const float* xs = reinterpret_cast<const float*>(gbase + OFF_XCH) + 256;
        unsigned char* stage = gbase + OFF_STAGE + wq * STAGE_WARP_BYTES;   // 32 rows x 128 bytes of this warp
        bool alive = true;
#pragma unroll 1
        for (int round = 0; round < n_rounds && alive; ++round) {
            const Item it = get_item(round);
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
                    // bf16 output, 64 head_dim columns (128 bytes of each row) per pass.  A thread holds one ROW, so direct
                    // stores would touch 32 different lines per instruction; the pass goes through a swizzled staging
                    // buffer instead and leaves as 4 rows x 128 contiguous bytes per instruction.
                    // Both halves are pulled out of TMEM before anything is written (the first one waits as 32 packed
                    // registers): the next item's first P V is held up by O_free, not by the stores.
                    uint32_t pk[2][32];
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        uint32_t v[2][32];
                        tmem_ld32(tO + c * 64, v[0]);
                        tmem_ld32(tO + c * 64 + 32, v[1]);
                        tmem_ld_wait();
                        if (c == 1) {
                            tc_fence_before();
                            mbar_arrive(bar(B_OFREE));   // O is in registers: the next item's P V may overwrite it
                        }
#pragma unroll
                        for (int e = 0; e < 64; e += 2)
                            pk[c][e >> 1] = pack2<__nv_bfloat16>(__uint_as_float(v[e >> 5][e & 31]) * inv, __uint_as_float(v[e >> 5][(e & 31) + 1]) * inv);
                    }
#pragma unroll 1
                    for (int c = 0; c < 2; ++c) {
#pragma unroll
                        for (int q4 = 0; q4 < 8; ++q4) {
                            uint4 o;
                            if (c == 0) o = make_uint4(pk[0][q4 * 4], pk[0][q4 * 4 + 1], pk[0][q4 * 4 + 2], pk[0][q4 * 4 + 3]);
                            else o = make_uint4(pk[1][q4 * 4], pk[1][q4 * 4 + 1], pk[1][q4 * 4 + 2], pk[1][q4 * 4 + 3]);
                            *reinterpret_cast<uint4*>(stage + lane * 128 + ((q4 ^ (lane & 7)) << 4)) = o;
                        }
                        __syncwarp();
#pragma unroll 2
                        for (int i = 0; i < 8; ++i) {
                            const int row = 4 * i + (lane >> 3);
                            const int R = wq * 32 + row;
                            const uint4 o = *reinterpret_cast<const uint4*>(stage + row * 128 + (((lane & 7) ^ (row & 7)) << 4));
                            if (R < rows_here) {
                                const int2 dm = rowmap[R];
                                char* dst = static_cast<char*>(a.out) + (((int64_t)(it.q0 + it.tok0 + dm.x) * a.o_rs + (int64_t)(head0 + dm.y) * HD) << 1);
                                *reinterpret_cast<uint4*>(dst + c * 128 + (lane & 7) * 16) = o;
                            }
                        }
                        __syncwarp();
                    }
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
                            mbar_arrive(bar(B_OFREE));
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
                mbar_arrive(bar(B_OFREE));
            }
            ++done;
        }
        mbar_arrive(bar(B_EPIDONE));   // (release: output rows and flags are written)
    } else {
    reg_dec<HELPER_REGS>();   // one site for the whole helper warpgroup (warps 8..11)
    if (warp == KLOAD_WARP || warp == VLOAD_WARP) {
        // =========================== loaders: one warp for K tiles, one for V tiles ===========================
        // Separate warps so that K (needed two tiles ahead by Q K^T) never queues behind a V tile that is still
        // waiting for its ring slot.  The rings run across items.  Every tile comes by TMA, issued by lane 0: the
        // common tile (inside the cached prefix, one box per head_dim half) on a short path with ring position and
        // page tracked incrementally and the page id taken from the record; the tile with the end of the prefix and
        // the in-flight rows as a few boxes of falling size (128 >> level rows), cached rows from the cache maps,
        // in-flight rows from the maps over k / v.
        const int which = warp == VLOAD_WARP;          // 0: K, 1: V
        int32_t* bt_base = reinterpret_cast<int32_t*>(gbase + OFF_BT) + which * BT_SLOTS;
        const int stages = which ? VSTAGES : KSTAGES;
        const int box_rows0 = a.tma_box_rows, lvl0 = a.tma_lvl0;   // largest cache box: min(128, page size) rows
        const CUtensorMap* cmaps = which ? maps.vc : maps.kc;
        const CUtensorMap* nmaps = which ? maps.vn : maps.kn;
        const int page_size = a.page_size;
        const bool one_box_geom = box_rows0 == TILE_N && page_size % TILE_N == 0;   // a whole tile is one box per half
        const int tiles_per_page = page_size / TILE_N;         // used only with one_box_geom
        const uint32_t bar_full0 = bar(which ? B_VFULL : B_KFULL), bar_empty0 = bar(which ? B_VEMPTY : B_KEMPTY);
        const uint32_t ring0 = which ? sV : sK;
        int stage = 0;            // ring position of the next tile
        uint32_t par_empty = 1;   // parity of "this slot is free" for the next tile (the first pass finds every slot free)
        int issued = 0;           // tiles whose copies were issued (lane 0)
        bool alive = true;
#pragma unroll 1
        for (int round = 0; round < n_rounds && alive; ++round) {
            const SchedRec* rec = rec_of(round);
            const Item it = load_item(a, rec, rank);
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
                int pj = pj_hi, sub = sub_hi;
                if (jj != 1 && n >= 2) {
                    if (--sub_w < 0) { sub_w = tiles_per_page - 1; --pj_w; }
                    pj = pj_w; sub = sub_w;
                }
                const int p0 = (it.t0 + tl) * TILE_N;   // first key of the tile
                const uint32_t full = bar_full0 + 8u * stage;
                const uint32_t d0 = ring0 + stage * ITEM_BYTES;
                bool ok = true;
                if (lane == 0) {
                    if (one_box_geom && p0 + TILE_N <= ctx) {
                        // ---- the common tile ----
                        if (!early_ready && pj < early) {
                            asm volatile("cp.async.wait_all;\n" ::: "memory");
                            early_ready = true;
                        }
                        const int pid0 = page_id(pj);
                        const int prow = sub * TILE_N;
                        ok = mbar_wait(bar_empty0 + 8u * stage, par_empty, abort_flag, 5 + which, jj);
                        if (ok) {
                            mbar_arrive_expect_tx(full, ITEM_BYTES);
                            tma_load_4d(d0, &cmaps[lvl0], 0, kvh, prow, pid0, full);
                            tma_load_4d(d0 + REGION, &cmaps[lvl0], 64, kvh, prow, pid0, full);
                            ++issued;
                        }
                    } else {
                        // ---- the tile with the end of the prefix, in-flight rows, small pages ----
                        const int cr = max(min(ctx - p0, TILE_N), 0);        // cached rows of the tile
                        const int ce = max(min(it.total - p0, TILE_N), 0);   // ... plus in-flight rows; the rest stays as it is
                        int pjg = p0 / page_size, prow = p0 - pjg * page_size;
                        if (!early_ready && pjg < early && cr > 0) {
                            asm volatile("cp.async.wait_all;\n" ::: "memory");
                            early_ready = true;
                        }
                        ok = mbar_wait(bar_empty0 + 8u * stage, par_empty, abort_flag, 5 + which, jj);
                        if (ok) {
                            ++issued;
                            if (ce == 0) {
                                mbar_arrive(full);
                            } else {
                                mbar_arrive_expect_tx(full, (uint32_t)ce * 256u);
                                int r = 0;
                                int lvl = lvl0;
#pragma unroll 1
                                for (int sz = box_rows0; sz >= 1; sz >>= 1, ++lvl) {
                                    while (cr - r >= sz) {
                                        const int pid = page_id(pjg);   // a bad id is out of bounds: zero fill
                                        tma_load_4d(d0 + r * 128, &cmaps[lvl], 0, kvh, prow, pid, full);
                                        tma_load_4d(d0 + REGION + r * 128, &cmaps[lvl], 64, kvh, prow, pid, full);
                                        r += sz; prow += sz;
                                        if (prow >= page_size) { prow = 0; ++pjg; }   // boxes never straddle a page
                                    }
                                }
                                int tok = it.kv0 + (p0 + cr - ctx);   // first in-flight row of the tile
                                lvl = 0;
#pragma unroll 1
                                for (int sz = TILE_N; sz >= 1; sz >>= 1, ++lvl) {
                                    while (ce - r >= sz) {
                                        tma_load_3d(d0 + r * 128, &nmaps[lvl], 0, kvh, tok, full);
                                        tma_load_3d(d0 + REGION + r * 128, &nmaps[lvl], 64, kvh, tok, full);
                                        r += sz; tok += sz;
                                    }
                                }
                            }
                        }
                    }
                }
                early_ready = __shfl_sync(0xffffffffu, (int)early_ready, 0) != 0;
                alive = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
                if (++stage == stages) { stage = 0; par_empty ^= 1u; }
            }
            ++done; ck += n;
        }
        asm volatile("cp.async.wait_all;\n" ::: "memory");  // nothing may still be landing when the CTA retires
        if (lane == 0 && *abort_flag != 0) {
            // A wait gave up somewhere in the CTA: boxes this lane has issued may still be in flight.  Each stage's
            // "full" barrier completes when the bytes of its last copy have landed, whether or not anybody consumes
            // them; wait for those phases (bounded) before the CTA hands its shared memory back.
            for (int st = 0; st < stages; ++st) {
                const int uses = (issued - st + stages - 1) / stages;   // tiles issued into stage st
                if (uses < 1) continue;
                for (uint32_t it = 0; it < (1u << 16); ++it)
                    if (mbar_try(bar_full0 + 8u * st, (uint32_t)(uses - 1) & 1u)) break;
            }
        }
    } else if (warp == QK_WARP) {
      if (lane == 0) {
        // =========================== Q K^T issuer (one thread) ===========================
        // S[g & 1] = Q K(k)^T for the tile with running index g.  The first two tiles of an item start as soon as Q and K are in and the S buffers
        // are free; tile k + 2 starts when the softmax warpgroup has pulled S(k) into registers (S_free), i.e.
        // while tile k's exponentials are still running.
        constexpr uint32_t ID_QK = instr_desc(false);
        bool ok = true;
#pragma unroll 1
        for (int round = 0; round < n_rounds && ok; ++round) {
            const Item it = get_item(round);
            if (!it.valid) continue;
            const int n = it.n;
            {
                // Q of this item: one box per head_dim half, as soon as the last Q K^T of the previous item has run
                // (this thread's own commit).  Tokens past the end of the tensor read as zero; tokens of the next
                // sequence are loaded but their rows are never stored.
                if (done > 0) ok = mbar_wait(bar(B_QEMPTY), (done - 1) & 1, abort_flag, 6, -2);
                if (!ok) break;
                mbar_arrive_expect_tx(bar(B_QFULL), 2u * (uint32_t)(a.q_tokens * G) * 128u);
                tma_load_3d(sQ, &maps.q, 0, it.kvh * G, it.q0 + it.tok0, bar(B_QFULL));
                tma_load_3d(sQ + REGION, &maps.q, 64, it.kvh * G, it.q0 + it.tok0, bar(B_QFULL));
            }
            ok = mbar_wait(bar(B_QFULL), done & 1, abort_flag, 7, -1);
#pragma unroll 1
            for (int k = 0; k < n && ok; ++k) {
                const int idx = ck + k;
                const int b = idx & 1, u = idx >> 1;   // S buffer and its use count
                if (u >= 1) {
                    ok = mbar_wait(bar(B_SFREE + b), (u - 1) & 1, abort_flag, 11, k);
                    if (!ok) break;
                }
                ok = mbar_wait(bar(B_KFULL + idx % KSTAGES), (idx / KSTAGES) & 1, abort_flag, 10, k);
                if (!ok) break;
                tc_fence_after();
                const uint32_t kb = sK + (idx % KSTAGES) * ITEM_BYTES;
                const uint32_t d = tmem + TM_S + b * 128;
                // the 8 k-steps differ only in the start-address field of the two descriptors (16-byte units)
                const uint64_t dq = smem_desc(sQ, 16, 1024), dk = smem_desc(kb, 16, 1024);
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    constexpr uint32_t unit = 16;
                    const uint64_t o = ((ks >> 2) * REGION + (ks & 3) * 32) / unit;
                    mma_ss(d, dq + o, dk + o, ID_QK, ks > 0);
                }
                tc_commit(bar(B_SFULL + b));
                tc_commit(bar(B_KEMPTY + idx % KSTAGES));
            }
            if (ok) tc_commit(bar(B_QEMPTY));   // every Q K^T of this item has read Q
            else {
                // giving up with this item's Q copy possibly in flight: let it land first (bounded)
                for (uint32_t it = 0; it < (1u << 16); ++it)
                    if (mbar_try(bar(B_QFULL), done & 1)) break;
            }
            ++done; ck += n;
        }
      }
    } else if (warp == PV_WARP) {
      if (lane == 0) {
        // =========================== P V issuer (one thread) ===========================
        // O += P(k) V(k), in tile order (one thread, so the accumulation order is fixed).  A second issuing
        // thread, because tcgen05.mma issue blocks while the pipe is busy: with one thread the waits for P, K
        // and V would line up behind each other's MMAs.
        constexpr uint32_t ID_PV = instr_desc(true);
        bool ok = true;
#pragma unroll 1
        for (int round = 0; round < n_rounds && ok; ++round) {
            const Item it = get_item(round);
            if (!it.valid) continue;
            const int n = it.n;
            if (done > 0) ok = mbar_wait(bar(B_OFREE), (done - 1) & 1, abort_flag, 8, -2);  // the epilogue has read O
#pragma unroll 1
            for (int k = 0; k < n && ok; ++k) {
                const int idx = ck + k;
                const int b = idx & 1, u = idx >> 1;   // P buffer and its use count
                ok = mbar_wait(bar(B_VFULL + idx % VSTAGES), (idx / VSTAGES) & 1, abort_flag, 8, k);
                ok = ok && mbar_wait(bar(B_PFULL + b), u & 1, abort_flag, 9, k);
                if (!ok) break;
                tc_fence_after();   // V arrived by TMA (async proxy): no proxy fence is needed before the MMA reads it
                const uint32_t vb = sV + (idx % VSTAGES) * ITEM_BYTES;
                const uint32_t pa = tmem + TM_P + b * 64;
                const uint64_t dv = smem_desc(vb, REGION, 1024);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    mma_ts(tmem + TM_O, pa + kk * 8, dv + (uint64_t)(kk * 2048 / 16), ID_PV, (k > 0 || kk > 0) ? 1u : 0u);
                tc_commit(bar(B_PFREE + b));
                tc_commit(bar(B_VEMPTY + idx % VSTAGES));
            }
            if (ok) tc_commit(bar(B_OFULL));
            ++done; ck += n;
        }
      }
    }
    }
    // ---- teardown: everyone arrives (all waits above are bounded), then TMEM is returned ----
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && *abort_flag != 0) {   // a wait ran out: record where (the first CTA to report wins)
        const int word = *abort_flag;
        if (atomicCAS(&g_status[0], 0, 1) == 0) {
            g_status[1] = (word >> 24) & 0xff; g_status[2] = (int)(short)((word >> 8) & 0xffff);
            g_status[3] = blockIdx.x;
        }
    }
    if (warp == QK_WARP) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;\n" ::"r"(tmem) : "memory");
    }
}

}  // namespace tc5

bool tc5_eligible(int group, int head_dim) { return head_dim == 128 && group >= 1 && group <= 128; }

// ---- TMA descriptors for the caches -----------------------------------------------------------
// A 4-D map {head_dim, Hkv, page row, page} of one cache tensor; box {64, 1, rows, 1}, 128-byte swizzle.
// Encoding is a host-only computation on (pointer, sizes, strides); results are memoised.
namespace {
struct MapKey {   // cache map: as named; Q map: (q, row stride, 0, total_q, Hq, group, tokens per block), rank 3
    const void* ptr; int64_t page_stride, token_stride, num_pages; int hkv, page_size, rows; int rank = 4;
    bool operator==(const MapKey& o) const {
        return ptr == o.ptr && page_stride == o.page_stride && token_stride == o.token_stride &&
               num_pages == o.num_pages && hkv == o.hkv && page_size == o.page_size && rows == o.rows && rank == o.rank;
    }
};
struct MapEntry { MapKey key; CUtensorMap map; bool used = false; };
// Memo: a hashed table with short probe runs; a launch looks up a few dozen maps, so a lookup has to cost
// nanoseconds however many layers' caches are in it.  A full run of probes replaces one of its entries.
constexpr size_t MAP_SLOTS = 4096, MAP_PROBES = 8;
std::mutex g_map_mutex;
std::vector<MapEntry> g_maps;
size_t g_map_next = 0;
inline size_t map_hash(const MapKey& k) {
    uint64_t h = 0x9e3779b97f4a7c15ull;
    auto mix = [&h](uint64_t v) { h ^= v + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2); };
    mix(reinterpret_cast<uint64_t>(k.ptr) >> 4); mix((uint64_t)k.page_stride); mix((uint64_t)k.token_stride);
    mix((uint64_t)k.num_pages); mix(((uint64_t)(uint32_t)k.hkv << 32) | (uint32_t)k.page_size);
    mix(((uint64_t)(uint32_t)k.rows << 8) | (uint32_t)k.rank);
    return (size_t)(h ^ (h >> 29));
}
typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                             const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                             CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn encode_fn() {
    static EncodeFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<EncodeFn>(f);
    }();
    return fn;
}
int cache_map(const MapKey& k, CUtensorMap* out) {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    if (g_maps.empty()) g_maps.resize(MAP_SLOTS);
    const size_t h = map_hash(k);
    size_t slot = MAP_SLOTS;
    for (size_t i = 0; i < MAP_PROBES; ++i) {
        MapEntry& e = g_maps[(h + i) & (MAP_SLOTS - 1)];
        if (e.used && e.key == k) { *out = e.map; return DLX_OK; }
        if (!e.used && slot == MAP_SLOTS) slot = (h + i) & (MAP_SLOTS - 1);
    }
    if (slot == MAP_SLOTS) slot = (h + (g_map_next++ % MAP_PROBES)) & (MAP_SLOTS - 1);
    EncodeFn enc = encode_fn();
    if (enc == nullptr) return fail(DLX_ERR_CUDA, "cuTensorMapEncodeTiled is not available from this driver");
    cuuint64_t gdim[4] = {(cuuint64_t)tc5::HD, (cuuint64_t)k.hkv, (cuuint64_t)k.page_size, (cuuint64_t)k.num_pages};
    cuuint64_t gstr[3] = {(cuuint64_t)tc5::HD * 2, (cuuint64_t)k.token_stride * 2, (cuuint64_t)k.page_stride * 2};
    cuuint32_t box[4] = {64, 1, (cuuint32_t)k.rows, 1};
    if (k.rank == 3) {   // Q and in-flight rows: {head_dim, heads, token}, box {64, heads per box, tokens per box}
        gdim[2] = (cuuint64_t)k.num_pages;
        gstr[1] = (cuuint64_t)k.page_stride * 2;
        box[1] = (cuuint32_t)k.page_size; box[2] = (cuuint32_t)k.rows;
    }
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    MapEntry e;
    e.key = k;
    e.used = true;
    const CUresult r = enc(&e.map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)k.rank, const_cast<void*>(k.ptr), gdim, gstr, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(DLX_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult %d", (int)r);
    g_maps[slot] = e;
    *out = e.map;
    return DLX_OK;
}
}  // namespace

namespace tc5 {
int tc5_cache_map(const void* ptr, int64_t page_stride, int64_t token_stride, int64_t num_pages, int hkv, int page_size,
                  int rows, int rank, CUtensorMap* out) {
    MapKey k{ptr, page_stride, token_stride, num_pages, hkv, page_size, rows, rank};
    return cache_map(k, out);
}
}  // namespace tc5

int launch_decode_tc5(const DecodeArgs& a_in, cudaStream_t st) {
    static bool attr_done[16] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 16 && !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(tc5::decode_attn_tc5_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             tc5::SMEM_BYTES);
        if (e != cudaSuccess) return fail(DLX_ERR_CUDA, "cudaFuncSetAttribute(tc5 smem=%d): %s", tc5::SMEM_BYTES, cudaGetErrorString(e));
        attr_done[dev] = true;
    }
    DecodeArgs a = a_in;
    tc5::TmaMaps maps;
    memset(&maps, 0, sizeof(maps));
    // Every tile comes by TMA (the caller has checked that page size and strides allow it).  Largest cache box:
    // min(128, page size) rows.  Without a cache no cache box is ever issued.
    if (a.max_blocks == 0) a.page_size = 128;
    const int ps = a.page_size;
    a.tma_box_rows = ps < 128 ? ps : 128;
    a.tma_lvl0 = 0;
    while ((128 >> a.tma_lvl0) > a.tma_box_rows) ++a.tma_lvl0;
    a.q_tokens = 128 / a.group;
    for (int lvl = 0; lvl < tc5::LEVELS; ++lvl) {
        const int rows = 128 >> lvl;
        int rc = DLX_OK;
        if (rows <= ps && a.max_blocks > 0) {   // caches: a box lies inside one page
            rc = tc5::tc5_cache_map(a.k_cache, a.page_stride, a.token_stride, a.num_pages, a.hkv, ps, rows, 4, &maps.kc[lvl]);
            if (rc == DLX_OK) rc = tc5::tc5_cache_map(a.v_cache, a.page_stride, a.token_stride, a.num_pages, a.hkv, ps, rows, 4, &maps.vc[lvl]);
        }
        // in-flight rows: {head_dim, Hkv, token}, box {64, 1, rows}
        if (rc == DLX_OK) rc = tc5::tc5_cache_map(a.k, a.k_rs, 0, a.total_kv, a.hkv, 1, rows, 3, &maps.kn[lvl]);
        if (rc == DLX_OK) rc = tc5::tc5_cache_map(a.v, a.v_rs, 0, a.total_kv, a.hkv, 1, rows, 3, &maps.vn[lvl]);
        if (rc != DLX_OK) return rc;
    }
    {   // Q blocks of 128 / group whole tokens: one box {64, group, tokens} per head_dim half
        const int rc = tc5::tc5_cache_map(a.q, a.q_rs, 0, a.total_q, a.hq, a.group, a.q_tokens, 3, &maps.q);
        if (rc != DLX_OK) return rc;
    }
    a.q_by_tma = 1;
    // Persistent CTAs: one per bin of the schedule (one per SM, fewer when there is less work).
    dim3 grid((unsigned)(a.bins * a.group_ctas)), block(tc5::NUM_THREADS);
    tc5::decode_attn_tc5_kernel<<<grid, block, tc5::SMEM_BYTES, st>>>(a, maps);
    return check_launch("decode_attn_tc5_kernel");
}

int read_tc5_status(int out[4]) {
    cudaError_t e = cudaMemcpyFromSymbol(out, tc5::g_status, sizeof(int) * 4);
    if (e != cudaSuccess) return fail(DLX_ERR_CUDA, "cudaMemcpyFromSymbol(g_status): %s", cudaGetErrorString(e));
    int zero[4] = {0, 0, 0, 0};
    e = cudaMemcpyToSymbol(tc5::g_status, zero, sizeof(zero));
    if (e != cudaSuccess) return fail(DLX_ERR_CUDA, "cudaMemcpyToSymbol(g_status): %s", cudaGetErrorString(e));
    return DLX_OK;
}


}  // namespace dlx
