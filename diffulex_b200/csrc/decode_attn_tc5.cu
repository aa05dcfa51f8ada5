// Paged block-diffusion decode attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Shape served: head_dim 128, bf16, 128 < G * q_len <= 256 packed query rows per KV head (e.g.
// 28 query heads over 4 KV heads with a 32-token diffusion block: 224 rows).  One CTA owns
// (sequence, KV head, key-range split) and keeps TWO 128-row Q tiles resident, so every K/V tile
// is fetched from HBM once and used by both: at ~224 flop per KV byte the legacy mma.sync pipe is
// the limiter, the tcgen05 pipe is not.
//
// Warp roles (352 threads, up to 184 registers each so a softmax thread holds its whole S row):
//   warps 0-3   softmax warpgroup of Q tile 0: thread <-> TMEM lane <-> query row
//   warps 4-7   softmax warpgroup of Q tile 1
//   warps 8-9   loaders: 16-byte cp.async of Q and of K/V tiles (128 keys) into 128B-swizzled
//               shared memory (the canonical K-major / MN-major UMMA layouts), any page size, the
//               cached prefix and the in-flight rows as ONE key axis, rows past the end zero-filled;
//               completion is signalled by cp.async.mbarrier.arrive, so loads run as far ahead as
//               the two-stage K and V rings allow
//   warp 10     one elected thread issues tcgen05.mma: S_t = Q_t K^T (SS form) into TMEM, and
//               O_t += P_t V (TS form: P is read from TMEM, V^T from shared memory), and
//               tcgen05.commit to the mbarriers that hand tiles back and forth
// TMEM (512 columns): S_0 | S_1 | O_0 | O_1, 128 fp32 columns each; P_t (bf16) overwrites the first
// 64 columns of S_t in place.  The two Q tiles ping-pong: while a softmax warpgroup works on S_t
// the tensor pipe runs the other tile's MMAs.  The running maximum is only raised when it grows by
// more than 2^8 (the accumulator then is rescaled in TMEM), so most tiles skip the rescale.
//
// Every mbarrier wait is bounded; on expiry the CTA raises an abort flag, records where it gave up
// in a device status word, drains, frees TMEM and returns (no trap, the context stays usable).
//
// Reference semantics: diffulex_kernel/python/dllm_flash_attn.py:163-347 and :632-637.
#include "dlx_common.cuh"
#include "decode_attn.cuh"

namespace dlx {
namespace tc5 {

constexpr int HD = 128;
constexpr int TILE_N = 128;               // keys per K/V tile
constexpr int REGION = 128 * 128;         // [128 rows][64 bf16] 128B-swizzled block: 16 KiB
constexpr int Q_BYTES = 4 * REGION;       // 2 Q tiles x 2 head_dim halves
constexpr int ITEM_BYTES = 2 * REGION;    // one K tile or one V tile
constexpr int STAGES = 2;
constexpr int OFF_K = Q_BYTES;
constexpr int OFF_V = OFF_K + STAGES * ITEM_BYTES;
constexpr int OFF_BAR = OFF_V + STAGES * ITEM_BYTES;
constexpr int OFF_TAB = OFF_BAR + 256;             // row-source pointer tables: K and V, 2 stages x 128 rows
constexpr int SMEM_BYTES = OFF_TAB + 4 * TILE_N * 8 + 1024;  // + slack for 1024-byte alignment
constexpr int NUM_THREADS = 352;
constexpr int LOADER_WARP0 = 8, MMA_WARP = 10;
constexpr int NUM_LOADERS = 64;
constexpr uint32_t WAIT_LIMIT = 1u << 21;

// barrier slots (8 bytes each) at OFF_BAR
enum { B_QFULL = 0, B_KFULL = 1, B_VFULL = 3, B_KEMPTY = 5, B_VEMPTY = 7, B_SFULL = 9, B_PFULL = 11, B_OFULL = 13, B_COUNT = 14 };

__device__ int g_status[4];  // [0] first failure code, [1] role, [2] tile, [3] CTA linear id
// Optional cycle accounting of CTA (0,0,0): [0] CTA lifetime, [role] cycles spent in that wait site,
// [12..14] softmax pass 1 / rescale / pass 2 of Q tile 0.  Off unless g_prof_on is set by the host.
__device__ unsigned long long g_prof[16];
__device__ int g_prof_on;
__device__ __forceinline__ bool prof_thread() {
    return g_prof_on && (blockIdx.x | blockIdx.y | blockIdx.z) == 0 && ((threadIdx.x & 127) == 0 || threadIdx.x == 320);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.b32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait.  Returns false when the limit ran out or another thread of the CTA gave up.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int role, int tile) {
    const bool rec = prof_thread();
    const long long c0 = rec ? clock64() : 0;
    for (uint32_t it = 0; it < WAIT_LIMIT; ++it) {
        if (mbar_try(bar, parity)) {
            if (rec) atomicAdd(&g_prof[role], (unsigned long long)(clock64() - c0));
            return true;
        }
        if ((it & 255u) == 255u && *abort_flag) return false;
    }
    *abort_flag = 1;
    if (atomicCAS(&g_status[0], 0, 1) == 0) {
        g_status[1] = role; g_status[2] = tile;
        g_status[3] = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    }
    return false;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void fence_async_proxy() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// The mbarrier gets one arrival (of its expected count) once every cp.async this thread issued so far has landed.
__device__ __forceinline__ void cp_async_arrive(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;\n" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}

// 64-bit shared-memory matrix descriptor, 128-byte swizzle, descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
    d |= (uint64_t)(lbo_bytes >> 4) << 16;
    d |= (uint64_t)(sbo_bytes >> 4) << 32;
    d |= 1ull << 46;
    d |= 2ull << 61;
    return d;
}
// kind::f16 instruction descriptor: fp32 accumulate, bf16 x bf16, M=128, N=128; b_mn: B is MN-major.
__host__ __device__ constexpr uint32_t instr_desc(bool b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn ? 1u : 0u) << 16) | ((128u >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc) : "memory");
}
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc) : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr) : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]) : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]) : "memory");
}

__global__ void __launch_bounds__(NUM_THREADS, 1) decode_attn_tc5_kernel(const DecodeArgs a) {
    extern __shared__ unsigned char smem_raw[];
    const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = a.group;

    // ---- CTA-uniform problem setup (before any TMEM / barrier state exists) ----
    const int q0 = a.cu_q[seq];
    const int qn = a.cu_q[seq + 1] - q0;
    if (qn <= 0 || q0 < 0 || q0 + qn > a.total_q) return;
    const int ctx = max(a.context_lens[seq], 0);
    int kv0 = q0, nnew = qn;
    if (a.cu_kv != nullptr) {
        kv0 = a.cu_kv[seq];
        nnew = max(a.cu_kv[seq + 1] - kv0, 0);
    }
    const int total = ctx + nnew;
    const int M = min(qn * G, 256);
    int cta_limit = total, full_until = total;
    if (a.mask_mode == DLX_MASK_BLOCK_CAUSAL) {
        const int i_last = (M - 1) / G;
        cta_limit = ctx + min(nnew, (i_last / a.dbs + 1) * a.dbs);
        full_until = ctx + min(nnew, a.dbs);
    }
    const int n_tiles = (cta_limit + TILE_N - 1) / TILE_N;
    const int tiles_per_split = (n_tiles + a.num_splits - 1) / a.num_splits;
    const int t0 = split * tiles_per_split;
    const int t1 = min(n_tiles, t0 + tiles_per_split);
    const int64_t head0 = (int64_t)kvh * G;
    if (t0 >= t1) {
        if (a.num_splits > 1)
            for (int r = tid; r < M; r += NUM_THREADS)
                a.ws_lse[((int64_t)split * a.total_q + q0 + r / G) * a.hq + head0 + r % G] = -INFINITY;
        return;
    }
    const int n = t1 - t0;

    const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
    unsigned char* gbase = smem_raw + (sbase - smem_u32(smem_raw));
    const uint32_t sQ = sbase, sK = sbase + OFF_K, sV = sbase + OFF_V, sBar = sbase + OFF_BAR;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + OFF_BAR + 8 * B_COUNT);
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + OFF_BAR + 8 * B_COUNT + 8);
    auto bar = [&](int slot) { return sBar + 8u * slot; };

    if (tid == 0) {
        mbar_init(bar(B_QFULL), NUM_LOADERS);
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar(B_KFULL + s), NUM_LOADERS);
            mbar_init(bar(B_VFULL + s), NUM_LOADERS);
            mbar_init(bar(B_KEMPTY + s), 1);
            mbar_init(bar(B_VEMPTY + s), 1);
            mbar_init(bar(B_SFULL + s), 1);
            mbar_init(bar(B_PFULL + s), 128);
        }
        mbar_init(bar(B_OFULL), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;\n" ::"r"(sBar + 8u * B_COUNT + 8u) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const long long cta_c0 = (tid == 0 && prof_thread()) ? clock64() : 0;

    if (warp < 8) {
        // =========================== softmax warpgroups ===========================
        const int t = warp >> 2;                       // Q tile
        const int L = tid & 127;                       // TMEM lane == row inside the tile
        const int r = t * 128 + L;                     // packed row: token r / G, head r % G
        const bool warp_valid = (t * 128 + (warp & 3) * 32) < M;   // any valid row in this warp?
        const bool row_valid = r < M;
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const uint32_t tS = lane_base + t * 128, tO = lane_base + 256 + t * 128;
        int limit = total;
        if (a.mask_mode == DLX_MASK_BLOCK_CAUSAL && row_valid) limit = ctx + min(nnew, ((r / G) / a.dbs + 1) * a.dbs);
        const float sl2 = a.scale_log2;
        float m_used = -INFINITY, l_run = 0.f;
        bool alive = true;
        for (int jj = 0; jj < n; ++jj) {
            bool ok = mbar_wait(bar(B_SFULL + t), jj & 1, abort_flag, 1 + t, jj);
            if (!__all_sync(0xffffffffu, ok)) { alive = false; break; }
            tc_fence_after();
            if (warp_valid) {
                const int key0 = (t0 + jj) * TILE_N;
                const bool rec = prof_thread();
                long long c0 = rec ? clock64() : 0;
                // the whole S row of this thread: 128 fp32 scores in registers, one TMEM round trip
                uint32_t v[4][32];
                tmem_ld32(tS, v[0]); tmem_ld32(tS + 32, v[1]); tmem_ld32(tS + 64, v[2]); tmem_ld32(tS + 96, v[3]);
                tmem_ld_wait();
                if (key0 + TILE_N > full_until) {  // tile touches a mask boundary (warp-uniform)
#pragma unroll
                    for (int c = 0; c < 4; ++c)
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            if (key0 + c * 32 + e >= limit) v[c][e] = 0xff800000u;  // -inf
                }
                float mx = -INFINITY;
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int e = 0; e < 32; e += 2)
                        mx = max3(mx, __uint_as_float(v[c][e]), __uint_as_float(v[c][e + 1]));
                if (rec) { const long long c1 = clock64(); atomicAdd(&g_prof[12], (unsigned long long)(c1 - c0)); c0 = c1; }
                const float m_new = fmaxf(m_used, mx * sl2);
                const bool need = (m_new > m_used) && (m_used == -INFINITY || m_new - m_used > 8.f);
                if (__any_sync(0xffffffffu, need)) {
                    const float alpha = (m_used == -INFINITY) ? 0.f : fast_exp2(m_used - m_new);
                    if (jj > 0) {  // O_t holds the sum over earlier tiles: rescale it in TMEM
#pragma unroll 1
                        for (int c = 0; c < 4; ++c) {
                            uint32_t w[32];
                            tmem_ld32(tO + c * 32, w);
                            tmem_ld_wait();
#pragma unroll
                            for (int e = 0; e < 32; ++e) w[e] = __float_as_uint(__uint_as_float(w[e]) * alpha);
                            tmem_st32(tO + c * 32, w);
                        }
                    }
                    l_run *= alpha;
                    m_used = m_new;
                }
                if (rec) { const long long c1 = clock64(); atomicAdd(&g_prof[13], (unsigned long long)(c1 - c0)); c0 = c1; }
                const float m_use = (m_used == -INFINITY) ? 0.f : m_used;
                // P = exp2(s*scale - m) as bf16, written over S in place (32 keys -> 16 columns)
                float l0 = 0.f, l1 = 0.f;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t pk[16];
#pragma unroll
                    for (int e = 0; e < 32; e += 2) {
                        const float p0 = fast_exp2(fmaf(__uint_as_float(v[c][e]), sl2, -m_use));
                        const float p1 = fast_exp2(fmaf(__uint_as_float(v[c][e + 1]), sl2, -m_use));
                        l0 += p0; l1 += p1;
                        pk[e >> 1] = pack2<__nv_bfloat16>(p0, p1);
                    }
                    tmem_st16(tS + c * 16, pk);
                }
                l_run += l0 + l1;
                tmem_st_wait();
                if (rec) atomicAdd(&g_prof[14], (unsigned long long)(clock64() - c0));
            }
            tc_fence_before();
            mbar_arrive(bar(B_PFULL + t));
        }
        // ---- epilogue: O_t / l -> global ----
        if (alive) {
            bool ok = mbar_wait(bar(B_OFULL), 0, abort_flag, 3 + t, n);
            alive = __all_sync(0xffffffffu, ok);
        }
        if (alive && warp_valid) {
            tc_fence_after();
            const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
            const int64_t tok = q0 + (row_valid ? r / G : 0);
            const int64_t head = head0 + (row_valid ? r % G : 0);
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                uint32_t v[32];
                tmem_ld32(tO + c * 32, v);
                tmem_ld_wait();
                if (!row_valid) continue;
                if (a.num_splits == 1) {
                    uint4* dst = reinterpret_cast<uint4*>(static_cast<char*>(a.out) + ((tok * a.o_rs + head * HD + c * 32) << 1));
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        uint4 o;
                        o.x = pack2<__nv_bfloat16>(__uint_as_float(v[q4 * 8 + 0]) * inv, __uint_as_float(v[q4 * 8 + 1]) * inv);
                        o.y = pack2<__nv_bfloat16>(__uint_as_float(v[q4 * 8 + 2]) * inv, __uint_as_float(v[q4 * 8 + 3]) * inv);
                        o.z = pack2<__nv_bfloat16>(__uint_as_float(v[q4 * 8 + 4]) * inv, __uint_as_float(v[q4 * 8 + 5]) * inv);
                        o.w = pack2<__nv_bfloat16>(__uint_as_float(v[q4 * 8 + 6]) * inv, __uint_as_float(v[q4 * 8 + 7]) * inv);
                        dst[q4] = o;
                    }
                } else {
                    const int64_t e = ((int64_t)split * a.total_q + tok) * a.hq + head;
                    float4* dst = reinterpret_cast<float4*>(a.ws_o + e * HD + c * 32);
#pragma unroll
                    for (int q4 = 0; q4 < 8; ++q4)
                        dst[q4] = make_float4(__uint_as_float(v[q4 * 4 + 0]) * inv, __uint_as_float(v[q4 * 4 + 1]) * inv,
                                              __uint_as_float(v[q4 * 4 + 2]) * inv, __uint_as_float(v[q4 * 4 + 3]) * inv);
                    if (c == 0) a.ws_lse[e] = l_run > 0.f ? m_used + log2f(l_run) : -INFINITY;
                }
            }
        }
    } else if (warp < MMA_WARP) {
        // =========================== loaders ===========================
        const int lt = tid - LOADER_WARP0 * 32;        // 0..63
        const int col = lt & 15, rbase = lt >> 4;      // 16-byte chunk of the row; rows rbase + 4 i
        const uint32_t half_off = (col >> 3) * REGION;
        const int c8 = col & 7;
        const char* qp = static_cast<const char*>(a.q);
        const char* kp = static_cast<const char*>(a.k);
        const char* vp = static_cast<const char*>(a.v);
        const char* kcp = static_cast<const char*>(a.k_cache);
        const char* vcp = static_cast<const char*>(a.v_cache);
        const int32_t* bt = a.block_tables + (int64_t)seq * a.bt_stride;
        // Q: 256 rows (two tiles), rows >= M zero-filled
#pragma unroll 4
        for (int i = 0; i < 64; ++i) {
            const int row = rbase + 4 * i;
            const bool okr = row < M;
            const int qi = okr ? row / G : 0, qg = okr ? row % G : 0;
            const char* src = qp + (((int64_t)(q0 + qi) * a.q_rs + (head0 + qg) * HD + col * 8) << 1);
            const uint32_t dst = sQ + (row >> 7) * (2 * REGION) + half_off + (row & 127) * 128 + ((c8 ^ (row & 7)) << 4);
            cp_async_16(dst, src, okr ? 16 : 0);
        }
        cp_async_arrive(bar(B_QFULL));
        // Row-source tables: for every key row of a tile, where its K and V bytes start (nullptr = row
        // past the end, zero-filled).  Each loader thread resolves two rows (page-table lookup), the
        // table of the NEXT tile is built while this tile's copies are issued.
        const char** tabK = reinterpret_cast<const char**>(gbase + OFF_TAB);   // [2][128]
        const char** tabV = tabK + 2 * TILE_N;                                   // [2][128]
        auto build_table = [&](int jj) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int row = lt + 64 * h;
                const int p = (t0 + jj) * TILE_N + row;
                const char *pk = nullptr, *pv = nullptr;
                if (p < ctx) {
                    const int j = p / a.page_size;
                    const int64_t pid = j < a.max_blocks ? (int64_t)bt[j] : -1;
                    if (pid >= 0 && pid < a.num_pages) {
                        const int64_t o = (pid * a.page_stride + (int64_t)(p - j * a.page_size) * a.token_stride + kvh * HD) << 1;
                        pk = kcp + o; pv = vcp + o;
                    }
                } else if (p < total) {
                    const int64_t r = kv0 + (p - ctx);
                    pk = kp + ((r * a.k_rs + kvh * HD) << 1);
                    pv = vp + ((r * a.v_rs + kvh * HD) << 1);
                }
                tabK[(jj & 1) * TILE_N + row] = pk;
                tabV[(jj & 1) * TILE_N + row] = pv;
            }
        };
        auto loaders_sync = [&]() { asm volatile("bar.sync 1, 64;\n" ::: "memory"); };
        build_table(0);
        loaders_sync();
        bool alive = true;
        for (int jj = 0; jj < n && alive; ++jj) {
            const int stage = jj & 1;
            const uint32_t par_empty = ((jj >> 1) & 1) ^ 1;
            if (jj + 1 < n) build_table(jj + 1);
#pragma unroll
            for (int which = 0; which < 2; ++which) {  // 0: K tile, 1: V tile
                bool ok = mbar_wait(bar((which ? B_VEMPTY : B_KEMPTY) + stage), par_empty, abort_flag, 5 + which, jj);
                if (!__all_sync(0xffffffffu, ok)) { alive = false; break; }
                const uint32_t dbase = (which ? sV : sK) + stage * ITEM_BYTES + half_off;
                const char* const* tab = (which ? tabV : tabK) + stage * TILE_N;
#pragma unroll 8
                for (int i = 0; i < 32; ++i) {
                    const int row = rbase + 4 * i;
                    const char* rp = tab[row];
                    cp_async_16(dbase + row * 128 + ((c8 ^ (row & 7)) << 4), rp ? rp + col * 16 : qp, rp ? 16 : 0);
                }
                cp_async_arrive(bar((which ? B_VFULL : B_KFULL) + stage));
            }
            loaders_sync();  // next tile's table is complete; this tile's table may be overwritten after the next sync
        }
        asm volatile("cp.async.wait_all;\n" ::: "memory");  // nothing may still be landing when the CTA retires
    } else if (lane == 0) {
        // =========================== MMA issuer (one thread) ===========================
        constexpr uint32_t ID_QK = instr_desc(false), ID_PV = instr_desc(true);
        auto issue_qk = [&](int t, int jj) {
            const uint32_t kb = sK + (jj & 1) * ITEM_BYTES;
            const uint32_t qb = sQ + t * (2 * REGION);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t o = (ks >> 2) * REGION + (ks & 3) * 32;
                mma_ss(tmem + t * 128, smem_desc(qb + o, 16, 1024), smem_desc(kb + o, 16, 1024), ID_QK, ks > 0);
            }
        };
        auto issue_pv = [&](int t, int jj) {
            const uint32_t vb = sV + (jj & 1) * ITEM_BYTES;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
                mma_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8, smem_desc(vb + kk * 2048, REGION, 1024), ID_PV,
                       (jj > 0 || kk > 0) ? 1u : 0u);
        };
        bool ok = mbar_wait(bar(B_QFULL), 0, abort_flag, 7, -1) && mbar_wait(bar(B_KFULL), 0, abort_flag, 7, 0);
        if (ok) {
            fence_async_proxy();  // the cp.async writes (generic proxy) must be visible to the tensor pipe's reads
            tc_fence_after();
            issue_qk(0, 0); tc_commit(bar(B_SFULL + 0));
            issue_qk(1, 0); tc_commit(bar(B_SFULL + 1));
            tc_commit(bar(B_KEMPTY + 0));
        }
        for (int jj = 0; jj < n && ok; ++jj) {
            const int st = jj & 1;
            const bool more = jj + 1 < n;
            ok = mbar_wait(bar(B_VFULL + st), (jj >> 1) & 1, abort_flag, 8, jj) &&
                 mbar_wait(bar(B_PFULL + 0), jj & 1, abort_flag, 9, jj);
            if (!ok) break;
            fence_async_proxy();
            tc_fence_after();
            issue_pv(0, jj);
            if (more) {
                ok = mbar_wait(bar(B_KFULL + (st ^ 1)), ((jj + 1) >> 1) & 1, abort_flag, 10, jj + 1);
                if (!ok) break;
                fence_async_proxy();
                tc_fence_after();
                issue_qk(0, jj + 1); tc_commit(bar(B_SFULL + 0));
            }
            ok = mbar_wait(bar(B_PFULL + 1), jj & 1, abort_flag, 11, jj);
            if (!ok) break;
            tc_fence_after();
            issue_pv(1, jj);
            tc_commit(bar(B_VEMPTY + st));
            if (more) {
                issue_qk(1, jj + 1); tc_commit(bar(B_SFULL + 1));
                tc_commit(bar(B_KEMPTY + (st ^ 1)));
            }
        }
        if (ok) tc_commit(bar(B_OFULL));
    }

    if (tid == 0 && prof_thread()) atomicAdd(&g_prof[0], (unsigned long long)(clock64() - cta_c0));
    // ---- teardown: everyone arrives (all waits above are bounded), then TMEM is returned ----
    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;\n" ::"r"(tmem) : "memory");
    }
}

}  // namespace tc5

bool tc5_eligible(int rows, int head_dim) { return head_dim == 128 && rows > 128 && rows <= 256; }

int launch_decode_tc5(const DecodeArgs& a, cudaStream_t st) {
    static bool attr_done[16] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 16 && !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(tc5::decode_attn_tc5_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             tc5::SMEM_BYTES);
        if (e != cudaSuccess) return fail(DLX_ERR_CUDA, "cudaFuncSetAttribute(tc5 smem=%d): %s", tc5::SMEM_BYTES, cudaGetErrorString(e));
        attr_done[dev] = true;
    }
    dim3 grid(a.num_splits, a.hkv, a.num_seqs), block(tc5::NUM_THREADS);
    tc5::decode_attn_tc5_kernel<<<grid, block, tc5::SMEM_BYTES, st>>>(a);
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

int tc5_profile(int enable, unsigned long long out[16]) {
    cudaError_t e = cudaSuccess;
    if (out != nullptr) e = cudaMemcpyFromSymbol(out, tc5::g_prof, sizeof(unsigned long long) * 16);
    unsigned long long zero[16] = {};
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(tc5::g_prof, zero, sizeof(zero));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(tc5::g_prof_on, &enable, sizeof(int));
    if (e != cudaSuccess) return fail(DLX_ERR_CUDA, "tc5_profile: %s", cudaGetErrorString(e));
    return DLX_OK;
}

}  // namespace dlx
