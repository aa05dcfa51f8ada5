// Paged block-diffusion decode attention, warp-level tensor-core kernel (mma.sync m16n8k16).
//
// This is the general kernel: any Hq/Hkv ratio, query block length, page size, head_dim 64/128,
// both mask modes.  One CTA owns (sequence, KV head, key-range split, M block).  All G = Hq/Hkv
// query heads that share the KV head are packed into the M dimension: row r = i*G + g is query
// token i, head kvh*G + g, so a CTA reads each K/V byte once for the whole GQA group (the
// reference launches one CTA per QUERY head, dllm_flash_attn.py:209, and re-reads KV G times).
//
// Data movement: K/V tiles of BLOCK_N keys are staged by 16-byte cp.async (coalesced: a key row of
// one KV head is head_dim*2 contiguous bytes) into XOR-swizzled shared memory, STAGES deep.  The
// cached prefix and the in-flight rows form ONE key axis (position p < ctx comes from the page the
// block table names, p >= ctx from the fresh k/v tensors), so no separate "fresh" stage exists and
// tiles never straddle an if.  Fragments come from ldmatrix; the online softmax runs in registers
// in the exp2 domain with quad shuffles; P is re-packed from the S accumulators as the A operand
// of P*V.  WN > 1 splits a tile's keys across warps (small M); their partial (m, l, O) are merged
// through shared memory.  With num_splits > 1 each split writes a normalised fp32 partial and its
// log2-sum-exp to the workspace and combine_splits_kernel merges them in fixed split order
// (deterministic).
//
// Reference semantics: diffulex_kernel/python/dllm_flash_attn.py:163-347 (static decode kernel),
// :632-637 (varlen decode = gather + non-causal attention).
#include "dlx_common.cuh"
#include "decode_attn.cuh"

namespace dlx {

template <typename T_, int HD_, int MT_, int WM_, int WN_, int KT_, int STAGES_, int MINB_>
struct MmaCfg {
    using T = T_;
    static constexpr int HD = HD_, MT = MT_, WM = WM_, WN = WN_, KT = KT_, STAGES = STAGES_, MINB = MINB_;
    static constexpr int BLOCK_M = 16 * MT * WM;
    static constexpr int BLOCK_N = KT * WN;
    static constexpr int NT = 32 * WM * WN;
    static constexpr int ROW_BYTES = HD * 2;
    static constexpr int CHUNKS = HD / 8;  // 16-byte chunks per row
    static constexpr int Q_BYTES = BLOCK_M * ROW_BYTES;
    static constexpr int KV_HALF_BYTES = BLOCK_N * ROW_BYTES;
    static constexpr int STAGE_BYTES = 2 * KV_HALF_BYTES;
    static constexpr int PIPE_BYTES = Q_BYTES + STAGES * STAGE_BYTES;
    // epilogue staging (aliases the pipeline buffers once the key loop is done)
    static constexpr int O_LD = HD + 4;  // floats per staged row; +4 spreads quad rows over all banks
    static constexpr int EPI_BYTES = (WN * BLOCK_M * O_LD + 2 * WN * BLOCK_M + 2 * BLOCK_M) * 4;
    static constexpr int SMEM_BYTES = PIPE_BYTES > EPI_BYTES ? PIPE_BYTES : EPI_BYTES;
    static_assert(KT % 16 == 0, "a warp's key tile is a whole number of k16 steps");
    static_assert(HD % 16 == 0 && (HD / 8) % 2 == 0, "head_dim");
};

template <class C>
__global__ void __launch_bounds__(C::NT, C::MINB) decode_attn_mma_kernel(const DecodeArgs a) {
    using T = typename C::T;
    constexpr int HD = C::HD, MT = C::MT, WM = C::WM, WN = C::WN, KT = C::KT, STAGES = C::STAGES;
    constexpr int BLOCK_M = C::BLOCK_M, BLOCK_N = C::BLOCK_N, NT = C::NT, ROW_BYTES = C::ROW_BYTES;
    constexpr int CHUNKS = C::CHUNKS;
    extern __shared__ __align__(128) unsigned char smem[];

    const int split = blockIdx.x;
    const int kvh = blockIdx.y / a.m_blocks, mb = blockIdx.y % a.m_blocks;
    const int seq = (int)blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wm = warp % WM, wn = warp / WM;
    const int G = a.group;
    if (seq < 0 || seq >= a.num_seqs) return;

    const int q0 = a.cu_q[seq];
    const int qn = a.cu_q[seq + 1] - q0;
    if (qn <= 0 || q0 < 0 || q0 + qn > a.total_q) return;  // padded or inconsistent sequence: no rows
    const int ctx = a.context_lens != nullptr ? max(a.context_lens[seq], 0) : 0;
    int kv0 = q0, nnew = qn;
    if (a.cu_kv != nullptr) {
        kv0 = a.cu_kv[seq];
        nnew = max(a.cu_kv[seq + 1] - kv0, 0);
    }
    const int total = ctx + nnew;
    const int M = qn * G;
    const int row0 = mb * BLOCK_M;
    if (row0 >= M) return;
    const int rows_here = min(M - row0, BLOCK_M);

    // Key limits.  cta_limit: no row of this CTA sees a key at or beyond it.  full_until: every
    // row sees every key below it (tiles wholly below need no masking).
    int cta_limit = total, full_until = total;
    if (a.mask_mode == DLX_MASK_BLOCK_CAUSAL) {
        const int i_first = row0 / G, i_last = (row0 + rows_here - 1) / G;
        cta_limit = ctx + min(nnew, (i_last / a.dbs + 1) * a.dbs);
        full_until = ctx + min(nnew, (i_first / a.dbs + 1) * a.dbs);
    }
    const int n_tiles = (cta_limit + BLOCK_N - 1) / BLOCK_N;
    const int tiles_per_split = (n_tiles + a.num_splits - 1) / a.num_splits;
    const int t0 = split * tiles_per_split;
    const int t1 = min(n_tiles, t0 + tiles_per_split);

    const int64_t head0 = (int64_t)kvh * G;
    if (t0 >= t1) {
        // Empty key range: tell the combine pass to ignore this split for these rows.
        if (a.num_splits > 1) {
            for (int r = tid; r < rows_here; r += NT) {
                const int rr = row0 + r;
                const int64_t tok = q0 + rr / G;
                a.ws_lse[((int64_t)split * a.total_q + tok) * a.hq + head0 + rr % G] = -INFINITY;
            }
        }
        return;
    }

    const uint32_t sQ = smem_u32(smem);
    const uint32_t sKV = sQ + C::Q_BYTES;
    const char* qp = static_cast<const char*>(a.q);
    const char* kp = static_cast<const char*>(a.k);
    const char* vp = static_cast<const char*>(a.v);
    const char* kcp = static_cast<const char*>(a.k_cache);
    const char* vcp = static_cast<const char*>(a.v_cache);
    const int32_t* bt = a.block_tables + (int64_t)seq * a.bt_stride;

    // ---- Q tile -> shared (rows >= M zero-filled) ----
    for (int c = tid; c < BLOCK_M * CHUNKS; c += NT) {
        const int row = c / CHUNKS, col = c % CHUNKS;
        const int rr = row0 + row;
        const bool ok = rr < M;
        const int i = ok ? rr / G : 0, g = ok ? rr % G : 0;
        const char* src = qp + (((int64_t)(q0 + i) * a.q_rs + (head0 + g) * HD + col * 8) << 1);
        cp_async_16(sQ + row * ROW_BYTES + ((col ^ (row & 7)) << 4), src, ok ? 16 : 0);
    }

    auto load_tile = [&](int tile, int stage) {
        const int base = tile * BLOCK_N;
        const uint32_t dK = sKV + stage * C::STAGE_BYTES;
        for (int c = tid; c < BLOCK_N * CHUNKS; c += NT) {
            const int row = c / CHUNKS, col = c % CHUNKS;
            const int p = base + row;
            const char *sk = qp, *sv = qp;
            int bytes = 0;
            if (p < ctx) {
                const int j = p / a.page_size;
                const int64_t pid = j < a.max_blocks ? (int64_t)bt[j] : -1;
                if (pid >= 0 && pid < a.num_pages) {
                    const int64_t off =
                        (pid * a.page_stride + (int64_t)(p - j * a.page_size) * a.token_stride + kvh * HD + col * 8) << 1;
                    sk = kcp + off;
                    sv = vcp + off;
                    bytes = 16;
                }
            } else if (p < total) {
                const int64_t n = kv0 + (p - ctx);
                sk = kp + ((n * a.k_rs + kvh * HD + col * 8) << 1);
                sv = vp + ((n * a.v_rs + kvh * HD + col * 8) << 1);
                bytes = 16;
            }
            const uint32_t d = dK + row * ROW_BYTES + ((col ^ (row & 7)) << 4);
            cp_async_16(d, sk, bytes);
            cp_async_16(d + C::KV_HALF_BYTES, sv, bytes);
        }
    };

    // ---- prologue: STAGES-1 tiles in flight (the Q tile rides in the first group) ----
#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) {
        if (t0 + s < t1) load_tile(t0 + s, s);
        cp_async_commit();
    }

    // ---- per-thread row bookkeeping ----
    const int gq = lane >> 2, tq = lane & 3;
    int limit[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int rr = row0 + (wm * MT + mt) * 16 + gq + 8 * h;
            int lim = total;
            if (a.mask_mode == DLX_MASK_BLOCK_CAUSAL && rr < M) lim = ctx + min(nnew, ((rr / G) / a.dbs + 1) * a.dbs);
            limit[mt][h] = lim;
        }

    float o[MT][HD / 8][4];
    float m_run[MT][2], l_run[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        m_run[mt][0] = m_run[mt][1] = -INFINITY;
        l_run[mt][0] = l_run[mt][1] = 0.f;
#pragma unroll
        for (int j = 0; j < HD / 8; ++j) o[mt][j][0] = o[mt][j][1] = o[mt][j][2] = o[mt][j][3] = 0.f;
    }

    const int mi = lane >> 3, r8 = lane & 7;  // ldmatrix: lane supplies row r8 of 8x8 matrix mi
    const float sl2 = a.scale_log2;

    for (int tile = t0; tile < t1; ++tile) {
        cp_async_wait<STAGES - 2>();
        __syncthreads();
        {
            const int nxt = tile + STAGES - 1;
            if (nxt < t1) load_tile(nxt, (nxt - t0) % STAGES);
            cp_async_commit();
        }
        const int stage = (tile - t0) % STAGES;
        const uint32_t sK = sKV + stage * C::STAGE_BYTES;
        const uint32_t sV = sK + C::KV_HALF_BYTES;
        const int key0 = tile * BLOCK_N + wn * KT;  // first key of this warp's slice
        if (key0 >= cta_limit) continue;             // warp-uniform; the barrier is at the loop top

        // ---- S = Q K^T ----
        float s[MT][KT / 8][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int nt = 0; nt < KT / 8; ++nt) s[mt][nt][0] = s[mt][nt][1] = s[mt][nt][2] = s[mt][nt][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
            uint32_t aq[MT][4];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const int row = (wm * MT + mt) * 16 + r8 + 8 * (mi & 1);
                const int chunk = ks * 2 + (mi >> 1);
                ldmatrix_x4(aq[mt][0], aq[mt][1], aq[mt][2], aq[mt][3],
                            sQ + row * ROW_BYTES + ((chunk ^ (row & 7)) << 4));
            }
#pragma unroll
            for (int np = 0; np < KT / 16; ++np) {
                uint32_t b0, b1, b2, b3;
                const int row = wn * KT + (np * 2 + (mi >> 1)) * 8 + r8;
                const int chunk = ks * 2 + (mi & 1);
                ldmatrix_x4(b0, b1, b2, b3, sK + row * ROW_BYTES + ((chunk ^ (row & 7)) << 4));
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    mma_16816<T>(s[mt][np * 2], aq[mt], b0, b1);
                    mma_16816<T>(s[mt][np * 2 + 1], aq[mt], b2, b3);
                }
            }
        }

        // ---- mask + online softmax (exp2 domain) ----
        const bool need_mask = key0 + KT > full_until;
        uint32_t pa[MT][KT / 16][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float mx = -INFINITY;
#pragma unroll
                for (int nt = 0; nt < KT / 8; ++nt)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        float x = s[mt][nt][2 * h + e];
                        if (need_mask && key0 + nt * 8 + 2 * tq + e >= limit[mt][h]) x = -INFINITY;
                        s[mt][nt][2 * h + e] = x;
                        mx = fmaxf(mx, x);
                    }
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                const float m_new = fmaxf(m_run[mt][h], mx * sl2);
                const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
                const float alpha = fast_exp2(m_run[mt][h] - m_use);
                m_run[mt][h] = m_new;
                float sum = 0.f;
#pragma unroll
                for (int nt = 0; nt < KT / 8; ++nt)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const float p = fast_exp2(fmaf(s[mt][nt][2 * h + e], sl2, -m_use));
                        s[mt][nt][2 * h + e] = p;
                        sum += p;
                    }
                l_run[mt][h] = l_run[mt][h] * alpha + sum;
#pragma unroll
                for (int j = 0; j < HD / 8; ++j) {
                    o[mt][j][2 * h] *= alpha;
                    o[mt][j][2 * h + 1] *= alpha;
                }
            }
#pragma unroll
            for (int kk = 0; kk < KT / 16; ++kk) {
                pa[mt][kk][0] = pack2<T>(s[mt][2 * kk][0], s[mt][2 * kk][1]);
                pa[mt][kk][1] = pack2<T>(s[mt][2 * kk][2], s[mt][2 * kk][3]);
                pa[mt][kk][2] = pack2<T>(s[mt][2 * kk + 1][0], s[mt][2 * kk + 1][1]);
                pa[mt][kk][3] = pack2<T>(s[mt][2 * kk + 1][2], s[mt][2 * kk + 1][3]);
            }
        }

        // ---- O += P V ----
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk) {
#pragma unroll
            for (int jp = 0; jp < HD / 16; ++jp) {
                uint32_t b0, b1, b2, b3;
                const int row = wn * KT + kk * 16 + r8 + 8 * (mi & 1);
                const int chunk = jp * 2 + (mi >> 1);
                ldmatrix_x4_trans(b0, b1, b2, b3, sV + row * ROW_BYTES + ((chunk ^ (row & 7)) << 4));
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    mma_16816<T>(o[mt][jp * 2], pa[mt][kk], b0, b1);
                    mma_16816<T>(o[mt][jp * 2 + 1], pa[mt][kk], b2, b3);
                }
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();  // pipeline buffers are dead from here; the epilogue staging aliases them

    // ---- epilogue: quad-reduce l, merge key-warps, normalise, write ----
    float* sO = reinterpret_cast<float*>(smem);                 // [WN][BLOCK_M][O_LD]
    float* sM = sO + WN * BLOCK_M * C::O_LD;                    // [WN][BLOCK_M]
    float* sL = sM + WN * BLOCK_M;                              // [WN][BLOCK_M]
    float* sMf = sL + WN * BLOCK_M;                             // [BLOCK_M] final max (log2 domain)
    float* sLf = sMf + BLOCK_M;                                 // [BLOCK_M] final sum
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float l = l_run[mt][h];
            l += __shfl_xor_sync(0xffffffffu, l, 1);
            l += __shfl_xor_sync(0xffffffffu, l, 2);
            l_run[mt][h] = l;
            const int row = (wm * MT + mt) * 16 + gq + 8 * h;
            if (tq == 0) {
                sM[wn * BLOCK_M + row] = m_run[mt][h];
                sL[wn * BLOCK_M + row] = l;
            }
        }
    if (WN > 1) __syncthreads();
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int row = (wm * MT + mt) * 16 + gq + 8 * h;
            float f = 1.f;
            if (WN > 1) {
                float mstar = -INFINITY;
#pragma unroll
                for (int w = 0; w < WN; ++w) mstar = fmaxf(mstar, sM[w * BLOCK_M + row]);
                const float muse = (mstar == -INFINITY) ? 0.f : mstar;
                float lsum = 0.f;
#pragma unroll
                for (int w = 0; w < WN; ++w) lsum += sL[w * BLOCK_M + row] * fast_exp2(sM[w * BLOCK_M + row] - muse);
                f = fast_exp2(m_run[mt][h] - muse);
                if (wn == 0 && tq == 0) { sMf[row] = mstar; sLf[row] = lsum; }
            } else if (tq == 0) {
                sMf[row] = m_run[mt][h];
                sLf[row] = l_run[mt][h];
            }
            float* dst = sO + ((size_t)wn * BLOCK_M + row) * C::O_LD + 2 * tq;
#pragma unroll
            for (int j = 0; j < HD / 8; ++j)
                *reinterpret_cast<float2*>(dst + j * 8) = make_float2(o[mt][j][2 * h] * f, o[mt][j][2 * h + 1] * f);
        }
    __syncthreads();

    constexpr int C4 = HD / 4;
    for (int idx = tid; idx < rows_here * C4; idx += NT) {
        const int row = idx / C4, c4 = idx % C4;
        float4 acc = *reinterpret_cast<const float4*>(sO + (size_t)row * C::O_LD + c4 * 4);
#pragma unroll
        for (int w = 1; w < WN; ++w) {
            const float4 x = *reinterpret_cast<const float4*>(sO + ((size_t)w * BLOCK_M + row) * C::O_LD + c4 * 4);
            acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
        }
        const float l = sLf[row];
        const float inv = l > 0.f ? 1.f / l : 0.f;
        acc.x *= inv; acc.y *= inv; acc.z *= inv; acc.w *= inv;
        const int rr = row0 + row;
        const int64_t tok = q0 + rr / G;
        const int64_t head = head0 + rr % G;
        if (a.num_splits == 1) {
            uint2 pk;
            pk.x = pack2<T>(acc.x, acc.y);
            pk.y = pack2<T>(acc.z, acc.w);
            *reinterpret_cast<uint2*>(static_cast<char*>(a.out) + ((tok * a.o_rs + head * HD + c4 * 4) << 1)) = pk;
        } else {
            const int64_t e = ((int64_t)split * a.total_q + tok) * a.hq + head;
            *reinterpret_cast<float4*>(a.ws_o + e * HD + c4 * 4) = acc;
            if (c4 == 0) a.ws_lse[e] = l > 0.f ? sMf[row] + log2f(l) : -INFINITY;
        }
    }
}

// Merge the per-split partials: out = sum_i w_i O_i / sum_i w_i with w_i = 2^(lse_i - max lse), in
// split order.  One warp per (token, head); grid.y walks sequences like the main kernel.
template <typename T, int HD>
__global__ void __launch_bounds__(256) combine_splits_kernel(const DecodeArgs a) {
    const int lane = threadIdx.x & 31;
    const int seq = blockIdx.y;
    const int q0 = a.cu_q[seq];
    const int qn = a.cu_q[seq + 1] - q0;  // non-positive for padded sequences: nothing to merge
    const int64_t local = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (qn <= 0 || q0 < 0 || q0 + qn > a.total_q || local >= (int64_t)qn * a.hq) return;   // same guard as the main kernels
    const int64_t tok = q0 + local / a.hq, head = local % a.hq;
    if (tok >= a.total_q) return;
    const int64_t wid = tok * a.hq + head;
    const int64_t stride = (int64_t)a.total_q * a.hq;
    float mx = -INFINITY;
    for (int s = 0; s < a.num_splits; ++s) mx = fmaxf(mx, a.ws_lse[s * stride + wid]);
    constexpr int PER = HD / 32;
    float acc[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) acc[e] = 0.f;
    float wsum = 0.f;
    if (mx != -INFINITY) {
        for (int s = 0; s < a.num_splits; ++s) {
            const float lse = a.ws_lse[s * stride + wid];
            if (lse == -INFINITY) continue;  // that split wrote no O for this row
            const float w = fast_exp2(lse - mx);
            wsum += w;
            const float* src = a.ws_o + (s * stride + wid) * HD + lane * PER;
#pragma unroll
            for (int e = 0; e < PER; ++e) acc[e] += w * src[e];
        }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    T* dst = static_cast<T*>(a.out) + tok * a.o_rs + head * HD + lane * PER;
#pragma unroll
    for (int e = 0; e < PER; e += 2)
        *reinterpret_cast<uint32_t*>(dst + e) = pack2<T>(acc[e] * inv, acc[e + 1] * inv);
}

// ---- launch plumbing --------------------------------------------------------------------------
template <class C>
static int launch_cfg(const DecodeArgs& a, cudaStream_t st) {
    static bool attr_done[16] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 16 && !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(decode_attn_mma_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::SMEM_BYTES);
        if (e != cudaSuccess) return fail(DLX_ERR_CUDA, "cudaFuncSetAttribute(smem=%d): %s", C::SMEM_BYTES, cudaGetErrorString(e));
        attr_done[dev] = true;
    }
    dim3 grid(a.num_splits, a.hkv * a.m_blocks, a.num_seqs), block(C::NT);
    decode_attn_mma_kernel<C><<<grid, block, C::SMEM_BYTES, st>>>(a);
    return check_launch("decode_attn_mma_kernel");
}

//                              T            HD  MT WM WN KT ST MINB
#define DLX_MMA_CFGS(T, HD)                                                   \
    using C16_##HD = MmaCfg<T, HD, 1, 1, 4, 16, 3, 2>;                        \
    using C32_##HD = MmaCfg<T, HD, 2, 1, 4, 16, 3, 2>;                        \
    using C64_##HD = MmaCfg<T, HD, 2, 2, 2, 32, 3, 2>;                        \
    using C128_##HD = MmaCfg<T, HD, 2, 4, 1, 64, 2, 2>;                       \
    using C224_##HD = MmaCfg<T, HD, 2, 7, 1, 64, 3, 1>;                       \
    using C256_##HD = MmaCfg<T, HD, 2, 8, 1, 64, 3, 1>;
DLX_MMA_CFGS(__nv_bfloat16, 128)
DLX_MMA_CFGS(__nv_bfloat16, 64)

MmaPlan plan_mma(int rows, int head_dim) {
    MmaPlan p{};
    if (rows <= 16) { p.id = 0; p.block_m = 16; p.block_n = 64; p.ctas_per_sm = 2; }
    else if (rows <= 32) { p.id = 1; p.block_m = 32; p.block_n = 64; p.ctas_per_sm = 2; }
    else if (rows <= 64) { p.id = 2; p.block_m = 64; p.block_n = 64; p.ctas_per_sm = 2; }
    else if (rows <= 128) { p.id = 3; p.block_m = 128; p.block_n = 64; p.ctas_per_sm = head_dim == 64 ? 2 : 2; }
    else if (rows <= 224) { p.id = 4; p.block_m = 224; p.block_n = 64; p.ctas_per_sm = 1; }
    else { p.id = 5; p.block_m = 256; p.block_n = 64; p.ctas_per_sm = 1; }
    p.m_blocks = (rows + p.block_m - 1) / p.block_m;
    return p;
}

int launch_decode_mma(const DecodeArgs& a, const MmaPlan& plan, int head_dim, cudaStream_t st) {
    int rc;
#define DLX_DISPATCH(HD)                                     \
    switch (plan.id) {                                       \
        case 0: rc = launch_cfg<C16_##HD>(a, st); break;     \
        case 1: rc = launch_cfg<C32_##HD>(a, st); break;     \
        case 2: rc = launch_cfg<C64_##HD>(a, st); break;     \
        case 3: rc = launch_cfg<C128_##HD>(a, st); break;    \
        case 4: rc = launch_cfg<C224_##HD>(a, st); break;    \
        default: rc = launch_cfg<C256_##HD>(a, st); break;   \
    }
    if (head_dim == 128) { DLX_DISPATCH(128) } else { DLX_DISPATCH(64) }
#undef DLX_DISPATCH
    return rc;
}

int launch_combine(const DecodeArgs& a, int head_dim, cudaStream_t st) {
    const int64_t warps = (int64_t)a.max_q_len * a.hq;
    dim3 grid((unsigned)((warps + 7) / 8), a.num_seqs), block(256);
    if (head_dim == 128) combine_splits_kernel<__nv_bfloat16, 128><<<grid, block, 0, st>>>(a);
    else combine_splits_kernel<__nv_bfloat16, 64><<<grid, block, 0, st>>>(a);
    return check_launch("combine_splits_kernel");
}

}  // namespace dlx
