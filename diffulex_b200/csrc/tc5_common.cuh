// PTX helpers shared by the tcgen05 decode-attention kernels: mbarriers (CTA-local and cluster-wide), TMA box loads,
// tcgen05 MMA / commit / TMEM load-store wrappers, shared-memory matrix descriptors.
#pragma once
#include <cuda.h>  // CUtensorMap

#include "dlx_common.cuh"
#include "decode_attn.cuh"

namespace dlx {
namespace tc5 {

constexpr uint32_t WAIT_LIMIT = 1u << 21;   // polls of a bounded mbarrier wait before the CTA gives up

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
// Bounded wait.  Returns false when the limit ran out or another thread of the CTA gave up.  Kept tiny, because it
// is inlined at some forty sites (a called function cannot be used once the warps have resized their register
// files): on expiry the site and tile go into the CTA's abort word, which one thread copies to the device status
// word when the CTA retires.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int role, int tile) {
    if (mbar_try(bar, parity)) return true;
#pragma unroll 1
    for (uint32_t it = 0; it < WAIT_LIMIT; ++it) {
        if (mbar_try(bar, parity)) return true;
        if ((it & 255u) == 255u && *abort_flag) return false;
    }
    *abort_flag = 1 | ((tile & 0xffff) << 8) | (role << 24);
    return false;
}

template <int N> __device__ __forceinline__ void reg_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(N)); }
template <int N> __device__ __forceinline__ void reg_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(N)); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void fence_async_proxy() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// The mbarrier gets one arrival (of its expected count) once every cp.async this thread issued so far has landed.
__device__ __forceinline__ void cp_async_arrive(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(bar) : "memory");
}
// Adds to the barrier's pending byte count without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
// One TMA box global -> shared, completion counted in bytes on `bar`.  Coordinates innermost first; c0 (elements of
// 2 bytes) is 0 or 64, i.e. a multiple of 16 bytes as the copy engine requires.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];\n"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar) : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];\n"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar) : "memory");
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


// ---- cluster (CTA pair) forms ----------------------------------------------------------------------------------
// Address of the same shared-memory offset in CTA `rank` of the cluster (a shared::cluster address).
__device__ __forceinline__ uint32_t map_to_cta(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ uint32_t cluster_cta_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
    return r;
}
// Arrive on a barrier of any CTA of the cluster.  The plain form orders only this CTA's view (what crosses the pair
// with it is tcgen05 / TMEM state, fenced by tcgen05.fence, or data a TMA copy wrote): it costs nothing.  The release
// form makes everything this thread observed or wrote visible cluster-wide first, which on this part takes well over a
// microsecond: it is used only where rows written by ordinary copies must be seen by the peer's tensor core.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];\n" ::"r"(cluster_bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster_release(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];\n" ::"r"(cluster_bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\n"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        "selp.b32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait on a barrier that CTAs of the cluster arrive on (acquire at cluster scope).
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag, int role, int tile) {
    if (mbar_try_cluster(bar, parity)) return true;
#pragma unroll 1
    for (uint32_t it = 0; it < WAIT_LIMIT; ++it) {
        if (mbar_try_cluster(bar, parity)) return true;
        if ((it & 255u) == 255u && *abort_flag) return false;
    }
    *abort_flag = 1 | ((tile & 0xffff) << 8) | (role << 24);
    return false;
}
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void fence_async_proxy_all() { asm volatile("fence.proxy.async;\n" ::: "memory"); }

// tcgen05 over a CTA pair (cta_group::2): one thread of the even CTA issues; both CTAs' tensor cores run, each on
// its own 128 accumulator rows, each supplying half of the B operand from its own shared memory.
// The commit signals the barrier at the same offset in both CTAs once every MMA issued so far has completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n"
                 ::"r"(bar), "h"((uint16_t)3) : "memory");
}
// ... or only this CTA's barrier.
__device__ __forceinline__ void tc_commit_local(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}
// kind::f16 instruction descriptor of the pair: fp32 accumulate, bf16 x bf16, M = 256 (128 per CTA), N = 128.
__host__ __device__ constexpr uint32_t instr_desc_pair(bool b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn ? 1u : 0u) << 16) | ((128u >> 3) << 17) | ((256u >> 4) << 24);
}
__device__ __forceinline__ void mma_ss_pair(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc) : "memory");
}
__device__ __forceinline__ void mma_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc) : "memory");
}

// ---- exact recomputation of flagged items ----------------------------------------------------------------------
// The tcgen05 kernels scale every P of an item by one fixed per-row reference (the row maximum of the item's first key
// tile) and never rescale their accumulator.  That is exact while the exponents stay inside fp32 / bf16 range; an item
// in which they do not (a tile row sum above DLX_SUM_HIGH, a final row sum below DLX_SUM_LOW) is flagged and its rows
// are computed again by the function below before the CTA retires, so results never depend on the fixed reference.
#define DLX_SUM_HIGH 1.2379400392853803e27f   // 2^90
#define DLX_SUM_LOW 8.271806125530277e-25f    // 2^-80
// Exact recomputation of this CTA's rows of one item (fp32, running maximum with rescale), by the eight softmax
// warps: a warp takes every eighth packed row.  Scores of up to CHUNK keys at a time sit in the warp's slice of
// `scratch` (the K / V rings, idle by now); lanes own keys for Q K^T and head_dim columns for P V.
constexpr int REDO_CHUNK = 1024;
template <class ItemT>
__device__ __forceinline__ void redo_item_exact(const DecodeArgs& a, const ItemT& it, int warp, int lane, float* scratch) {
    constexpr int HD = 128, TILE_N = 128;
    float* sc = scratch + warp * (REDO_CHUNK + HD);   // scores of the chunk, then the scaled query row
    float* qrow = sc + REDO_CHUNK;
    const int G = a.group;
    const char* kc = static_cast<const char*>(a.k_cache);
    const char* vc = static_cast<const char*>(a.v_cache);
    const char* kn = static_cast<const char*>(a.k);
    const char* vn = static_cast<const char*>(a.v);
    const int32_t* bt = a.block_tables + (int64_t)it.seq * a.bt_stride;
    for (int r = warp; r < it.rows_here; r += 8) {
        const int tok = it.tok0 + r / G, head = it.kvh * G + r % G;
        int limit = it.total;
        if (a.mask_mode == DLX_MASK_BLOCK_CAUSAL) limit = it.ctx + min(it.nnew, (tok / a.dbs + 1) * a.dbs);
        const int k_begin = it.t0 * TILE_N, k_end = min((it.t0 + it.n) * TILE_N, limit);
        const __nv_bfloat16* qg = static_cast<const __nv_bfloat16*>(a.q) + (int64_t)(it.q0 + tok) * a.q_rs + (int64_t)head * HD;
        __syncwarp();
        for (int d = lane; d < HD; d += 32) qrow[d] = __bfloat162float(qg[d]) * a.scale_log2;
        __syncwarp();
        float m_run = -INFINITY, l_run = 0.f;
        float o[4] = {0.f, 0.f, 0.f, 0.f};
        for (int c0 = k_begin; c0 < k_end; c0 += REDO_CHUNK) {
            const int c1 = min(c0 + REDO_CHUNK, k_end);
            float mx = -INFINITY;
            for (int key = c0 + lane; key < c1; key += 32) {
                const char* row = nullptr;
                if (key < it.ctx) {
                    const int j = key / a.page_size;
                    const int64_t pid = j < a.max_blocks ? (int64_t)bt[j] : -1;
                    if (pid >= 0 && pid < a.num_pages)
                        row = kc + ((pid * a.page_stride + (int64_t)(key - j * a.page_size) * a.token_stride + it.kvh * HD) << 1);
                } else {
                    row = kn + (((int64_t)(it.kv0 + key - it.ctx) * a.k_rs + it.kvh * HD) << 1);
                }
                float s = 0.f;
                if (row != nullptr) {
#pragma unroll 4
                    for (int c = 0; c < 16; ++c) {
                        const uint4 u = *reinterpret_cast<const uint4*>(row + c * 16);
                        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 f = __bfloat1622float2(h[e]);
                            s = fmaf(f.x, qrow[c * 8 + 2 * e], s);
                            s = fmaf(f.y, qrow[c * 8 + 2 * e + 1], s);
                        }
                    }
                }
                sc[key - c0] = s;
                mx = fmaxf(mx, s);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m_run, mx);
            const float f = (m_run == -INFINITY) ? 0.f : exp2f(m_run - m_new);
            l_run *= f;
#pragma unroll
            for (int e = 0; e < 4; ++e) o[e] *= f;
            m_run = m_new;
            __syncwarp();
            for (int key = c0; key < c1; ++key) {
                const float p = exp2f(sc[key - c0] - m_run);
                const char* row = nullptr;
                if (key < it.ctx) {
                    const int j = key / a.page_size;
                    const int64_t pid = j < a.max_blocks ? (int64_t)bt[j] : -1;
                    if (pid >= 0 && pid < a.num_pages)
                        row = vc + ((pid * a.page_stride + (int64_t)(key - j * a.page_size) * a.token_stride + it.kvh * HD) << 1);
                } else {
                    row = vn + (((int64_t)(it.kv0 + key - it.ctx) * a.v_rs + it.kvh * HD) << 1);
                }
                l_run += p;
                if (row != nullptr) {
                    const uint2 u = *reinterpret_cast<const uint2*>(row + lane * 8);
                    const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
                    const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
                    o[0] = fmaf(p, f0.x, o[0]); o[1] = fmaf(p, f0.y, o[1]);
                    o[2] = fmaf(p, f1.x, o[2]); o[3] = fmaf(p, f1.y, o[3]);
                }
            }
            __syncwarp();
        }
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        if (a.num_splits == 1) {
            uint2 pk;
            pk.x = pack2<__nv_bfloat16>(o[0] * inv, o[1] * inv);
            pk.y = pack2<__nv_bfloat16>(o[2] * inv, o[3] * inv);
            char* dst = static_cast<char*>(a.out) + (((int64_t)(it.q0 + tok) * a.o_rs + (int64_t)head * HD) << 1);
            *reinterpret_cast<uint2*>(dst + lane * 8) = pk;
        } else {
            const int64_t e = ((int64_t)it.split * a.total_q + it.q0 + tok) * a.hq + head;
            *reinterpret_cast<float4*>(a.ws_o + e * HD + lane * 4) = make_float4(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv);
            if (lane == 0) a.ws_lse[e] = l_run > 0.f ? m_run + log2f(l_run) : -INFINITY;
        }
    }
}


}  // namespace tc5
}  // namespace dlx
