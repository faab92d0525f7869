// Prefill attention on the tensor cores (tensor mode): the split-K decomposition of
// k_attn_partial + k_attn_merge (kernels.cu, Kernels.metal:301-562), with the scores and P.V of a
// split as tcgen05 MMAs instead of one CUDA-core pass per query row.
//
// A CTA takes 8 query tokens of one forward call and one key split (up to `span` keys of the
// window). With one KV head (MQA) the 8 tokens x 16 heads are 128 MMA rows that share every key:
// row r = token * 16 + head, one tensor-memory lane each. Per 256-key chunk of the split:
//   - the chunk's keys are staged in shared memory (local layers re-rotated with the window-relative
//     RoPE coordinates, Kernels.metal:277-285) and the values transposed, both in the K-major
//     128-byte-swizzle layout that the MMA's shared-memory descriptors read;
//   - S = Q.K^T for up to 4 tiles of 64 keys (M 128, N 64, K 128) lands in tensor memory;
//   - two threads own a row, each half of its columns: they read the scores (tcgen05.ld), apply
//     the window / causal mask, agree on the running max through shared memory (rescaling the O
//     row in tensor memory when the max grows) and write P = 2^(score log2 e - max) as a bf16
//     hi/lo pair, so P keeps 16 significant bits like the reference's fp32 softmax output
//     (Kernels.metal:400-437), not bf16's 8;
//   - O += P_hi.V + P_lo.V (M 128, N 128, K 64 per tile) accumulates in tensor memory, each tile's
//     MMAs running while the next tile's P is computed.
// At the end each row stores its split's (max, sum) and unnormalised O in the layout k_attn_merge
// reads, and that merge runs unchanged.
//
// The results follow the tensor core's summation order and P's 16-bit split, so they match the
// order-exact path within rounding, not bit for bit; the runtime uses this kernel only in tensor
// mode. Every mbarrier wait is bounded (2 s) and reports through the tiled-GEMM error word.
#include "common.cuh"
#include "kernels.h"
#include "mbarrier.cuh"
#include "tcgen05.cuh"

namespace plamo {

namespace {

constexpr int ATC_TOK = 8;        // query tokens per CTA (x 16 heads = 128 MMA rows)
constexpr int ATC_H = 16;         // query heads (one KV head)
constexpr int ATC_CH = 256;       // keys per staged chunk
constexpr int ATC_KT = 64;        // keys per S tile (MMA N) and per P.V step (MMA K)
constexpr int ATC_THREADS = 256;  // two threads per MMA row / tensor-memory lane (column halves)
constexpr int ATC_SPLITS = 8;     // target key splits per row (span = cache / 8, >= one chunk)

// shared-memory layout (offsets from a 1024-byte aligned base)
constexpr uint32_t OFF_Q = 0;                        // 2 k-blocks x [128 rows][64] bf16
constexpr uint32_t OFF_K = OFF_Q + 2 * 16384;        // 2 k-blocks x [256 keys][64] bf16
constexpr uint32_t OFF_VT = OFF_K + 2 * 32768;       // 4 key-blocks x [128 dims][64 keys] bf16
constexpr uint32_t OFF_PH = OFF_VT + 4 * 16384;      // [128 rows][64 keys] bf16, P high part
constexpr uint32_t OFF_PL = OFF_PH + 16384;          // P low part
constexpr uint32_t OFF_CTL = OFF_PL + 16384;         // barriers, tensor-memory slot, token table
constexpr uint32_t OFF_XCH = OFF_CTL + 512;          // [2][128] floats: the halves' row maxima / sums
constexpr uint32_t ATC_SMEM = OFF_XCH + 1024 + 1024;  // + alignment slack
constexpr uint32_t TMEM_COLS = 512;                  // S: columns [0, 256), O: [256, 384)
constexpr uint32_t TM_O = 256;

struct TokenInfo {
    int first, count, begin, end, lane, pad;
};

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// 2^x on the multi-function unit (relative error about 2^-22, far below P's 16-bit hi/lo split)
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// Two floats to a bf16 pair (lo in the low half), round to nearest even in one instruction: the
// same bits as f2bf for every finite value, which is all this kernel converts.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
__device__ __forceinline__ float round_bf16(float x) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r << 16);
}
// Rotate-half RoPE of one element as rope_rotate (Kernels.metal:261-274) with the hardware
// rounding: rbf(rbf(x c) + rbf(+-other s)).
__device__ __forceinline__ float rope_fast(float x, float other, bool low, uint32_t cs) {
    const float c = lo_bf(cs), sn = hi_bf(cs);
    return round_bf16(round_bf16(x * c) + round_bf16((low ? -other : other) * sn));
}
constexpr float ATC_LOG2E = 1.4426950408889634f;
constexpr float ATC_LN2 = 0.6931471805599453f;

__global__ void __launch_bounds__(ATC_THREADS, 1) k_attn_tc(AttnArgs a, int span, int* error) {
    pdl_enter();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint64_t* bar_s = reinterpret_cast<uint64_t*>(smem + OFF_CTL);
    uint64_t* bar_pv = bar_s + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_s + 2);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
    TokenInfo* tok = reinterpret_cast<TokenInfo*>(smem + OFF_CTL + 64);
    float* xchg = reinterpret_cast<float*>(smem + OFF_XCH);  // [2 halves][128 rows] row maxima / sums

    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    // warps w and w + 4 share tensor-memory lanes 32 (w % 4) ..: the row is the lane, the two warps
    // take the two halves of every tile's columns
    const int quarter = warp & 3, half = warp >> 2, row = quarter * 32 + lane;
    const int s = blockIdx.x, row0 = blockIdx.y * ATC_TOK;
    const int ntok = min(ATC_TOK, a.rows - row0);
    if (t < ntok) {
        const RowGeo g = a.geo[row0 + t];
        tok[t] = TokenInfo{g.first, g.count, g.begin, g.end, a.desc[row0 + t].lane, 0};
    }
    if (t == 0) {
        bar_init(bar_s, 1);
        bar_init(bar_pv, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    if (warp == 0) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = uint32_t(quarter * 32) << 16;
    const uint32_t sbase = smem_addr(smem);
    const float qscale = PLAMO_ATTN_SCALE * ATC_LOG2E;  // scores in the log2 domain
    uint32_t ps = 0, ppv = 0;  // barrier parities

    const int my_tok = row >> 4, my_head = row & 15;
    unsigned done = 0;
    const unsigned all = (1u << ntok) - 1u;
    while (done != all) {
        // the next run: the pending tokens that share the first one's lane slab and window
        const TokenInfo L = tok[__ffs(~done & all) - 1];
        unsigned run = 0;
        for (int i = 0; i < ntok; i++) {
            const TokenInfo& o = tok[i];
            if (!((done >> i) & 1u) && o.lane == L.lane && o.first == L.first && o.count == L.count) run |= 1u << i;
        }
        done |= run;
        const int k_lo = s * span, k_hi = min(k_lo + span, L.count);
        int klo = 1 << 30, khi = 0;
        for (int i = 0; i < ntok; i++)
            if ((run >> i) & 1u) {
                const int lo = max(tok[i].begin, k_lo), hi = min(tok[i].end, k_hi);
                if (lo < hi) { klo = min(klo, lo); khi = max(khi, hi); }
            }
        const bool mine = (run >> my_tok) & 1u;
        const int vis_lo = mine ? max(tok[my_tok].begin, k_lo) : 0;
        const int vis_hi = mine ? min(tok[my_tok].end, k_hi) : 0;
        float m_run = -INFINITY, l_run = 0.f;  // log2-domain max; this half's share of the sum
        if (klo < khi) {
            // queries of the run's tokens (other rows zero); every load of a thread in flight at once
            {
                uint4 v[8];
#pragma unroll
                for (int b = 0; b < 8; b++) {
                    const int u = t + b * ATC_THREADS, r = u >> 4, c = u & 15, i = r >> 4;
                    v[b] = (run >> i) & 1u
                               ? __ldg(reinterpret_cast<const uint4*>(a.q + size_t(row0 + i) * ATC_H * 128 + (r & 15) * 128) + c)
                               : make_uint4(0u, 0u, 0u, 0u);
                }
#pragma unroll
                for (int b = 0; b < 8; b++) {
                    const int u = t + b * ATC_THREADS, r = u >> 4, c = u & 15;
                    *reinterpret_cast<uint4*>(smem + OFF_Q + (c >> 3) * 16384 + sw128_offset(uint32_t(r), uint32_t(c & 7) * 8)) = v[b];
                }
            }
            const uint16_t* kbase = a.keys + size_t(L.lane) * a.lane_stride;
            const uint16_t* vbase = a.values + size_t(L.lane) * a.lane_stride;
            bool o_init = false;
            for (int kc = klo; kc < khi; kc += ATC_CH) {
                const int nk = min(ATC_CH, khi - kc), ntile = (nk + ATC_KT - 1) / ATC_KT, nrow = ntile * ATC_KT;
                // keys: row j = key kc + j; dims d and d + 64 rotate together (local layers). Four
                // units per thread at a time, their loads issued together.
                for (int b0 = 0; b0 * ATC_THREADS < nrow * 8; b0 += 4) {
                    uint4 x1[4], x2[4], c0[4], c1[4];
#pragma unroll
                    for (int b = 0; b < 4; b++) {
                        const int u = t + (b0 + b) * ATC_THREADS, j = u >> 3, p = u & 7;
                        x1[b] = x2[b] = c0[b] = c1[b] = make_uint4(0u, 0u, 0u, 0u);
                        if (u < nrow * 8 && j < nk) {
                            const int kidx = kc + j, slot = (L.first + kidx) % a.cap;
                            const uint4* src = reinterpret_cast<const uint4*>(kbase + size_t(slot) * 128);
                            x1[b] = __ldg(src + p);
                            x2[b] = __ldg(src + 8 + p);
                            if (!a.full) {
                                const uint4* rp = reinterpret_cast<const uint4*>(a.rope_local + size_t(kidx) * 64 + p * 8);
                                c0[b] = __ldg(rp);
                                c1[b] = __ldg(rp + 1);
                            }
                        }
                    }
#pragma unroll
                    for (int b = 0; b < 4; b++) {
                        const int u = t + (b0 + b) * ATC_THREADS, j = u >> 3, p = u & 7;
                        if (u >= nrow * 8) break;
                        uint4 o1 = x1[b], o2 = x2[b];
                        if (!a.full && j < nk) {
                            const uint32_t cs[8] = {c0[b].x, c0[b].y, c0[b].z, c0[b].w, c1[b].x, c1[b].y, c1[b].z, c1[b].w};
                            const uint32_t a1[4] = {x1[b].x, x1[b].y, x1[b].z, x1[b].w}, a2[4] = {x2[b].x, x2[b].y, x2[b].z, x2[b].w};
                            uint32_t r1[4], r2[4];
#pragma unroll
                            for (int e = 0; e < 4; e++) {
                                const float l1 = lo_bf(a1[e]), h1 = hi_bf(a1[e]), l2 = lo_bf(a2[e]), h2 = hi_bf(a2[e]);
                                const int d = p * 8 + 2 * e;
                                (void)d;
                                r1[e] = pack_bf16x2(rope_fast(l1, l2, true, cs[2 * e]), rope_fast(h1, h2, true, cs[2 * e + 1]));
                                r2[e] = pack_bf16x2(rope_fast(l2, l1, false, cs[2 * e]), rope_fast(h2, h1, false, cs[2 * e + 1]));
                            }
                            o1 = make_uint4(r1[0], r1[1], r1[2], r1[3]);
                            o2 = make_uint4(r2[0], r2[1], r2[2], r2[3]);
                        }
                        *reinterpret_cast<uint4*>(smem + OFF_K + sw128_offset(uint32_t(j), uint32_t(p) * 8)) = o1;
                        *reinterpret_cast<uint4*>(smem + OFF_K + 32768 + sw128_offset(uint32_t(j), uint32_t(p) * 8)) = o2;
                    }
                }
                // values, transposed: V^T[d][j] in blocks of 64 keys (consecutive threads take
                // consecutive keys of one 8-dim group); eight units per thread at a time
                for (int b0 = 0; b0 * ATC_THREADS < nrow * 16; b0 += 8) {
                    uint4 v[8];
#pragma unroll
                    for (int b = 0; b < 8; b++) {
                        const int u = t + (b0 + b) * ATC_THREADS, p = u / nrow, j = u - p * nrow;
                        v[b] = make_uint4(0u, 0u, 0u, 0u);
                        if (u < nrow * 16 && j < nk) {
                            const int slot = (L.first + kc + j) % a.cap;
                            v[b] = __ldg(reinterpret_cast<const uint4*>(vbase + size_t(slot) * 128) + p);
                        }
                    }
#pragma unroll
                    for (int b = 0; b < 8; b++) {
                        const int u = t + (b0 + b) * ATC_THREADS, p = u / nrow, j = u - p * nrow;
                        if (u >= nrow * 16) break;
                        const uint32_t w[4] = {v[b].x, v[b].y, v[b].z, v[b].w};
                        // element (dim 8p + e, key j): rows 8p..8p+7 are one 1024-byte swizzle group
                        uint8_t* blk = smem + OFF_VT + (j >> 6) * 16384 + p * 1024 + (j & 7) * 2;
                        const uint32_t jc = uint32_t(j & 63) >> 3;
#pragma unroll
                        for (int e = 0; e < 8; e++)
                            *reinterpret_cast<uint16_t*>(blk + e * 128 + ((jc ^ uint32_t(e)) << 4)) =
                                uint16_t(w[e >> 1] >> (16 * (e & 1)));
                    }
                }
                fence_async_smem();
                __syncthreads();
                // S = Q.K^T, one 64-key tile per 64 tensor-memory columns
                if (t == 0) {
                    tc_fence_after();
                    const uint32_t idesc = tc_idesc(ATC_KT);
                    for (int jt = 0; jt < ntile; jt++)
#pragma unroll
                        for (int kk = 0; kk < 8; kk++)
                            umma_bf16(tmem + uint32_t(jt * ATC_KT), sw128_desc(sbase + OFF_Q + (kk >> 2) * 16384 + (kk & 3) * 32),
                                      sw128_desc(sbase + OFF_K + (kk >> 2) * 32768 + jt * 8192 + (kk & 3) * 32), idesc,
                                      uint32_t(kk));
                    umma_commit(bar_s);
                }
                if (!__syncthreads_and(bar_wait(bar_s, ps))) {
                    if (t == 0) { atomicCAS(error, 0, 21); *abort_flag = 1; }
                    break;
                }
                ps ^= 1u;
                tc_fence_after();
                // the row's max over its visible keys of the chunk: each half over its columns,
                // then the two halves meet in shared memory
                const int lo_r = vis_lo - kc, hi_r = vis_hi - kc;
                float mc = -INFINITY;
                for (int jt = 0; jt < ntile; jt += 2) {  // two tiles' loads in flight per wait
                    uint32_t va[32], vb[32];
                    const int ca = jt * ATC_KT + half * 32, cb = ca + ATC_KT;
                    tmem_ld32_async(tmem + lane_base + uint32_t(ca), va);
                    if (jt + 1 < ntile) tmem_ld32_async(tmem + lane_base + uint32_t(cb), vb);
                    tmem_wait_ld(va);
                    tmem_wait_ld(vb);
#pragma unroll
                    for (int e = 0; e < 32; e++)
                        if (ca + e >= lo_r && ca + e < hi_r) mc = fmaxf(mc, __uint_as_float(va[e]) * qscale);
                    if (jt + 1 < ntile)
#pragma unroll
                        for (int e = 0; e < 32; e++)
                            if (cb + e >= lo_r && cb + e < hi_r) mc = fmaxf(mc, __uint_as_float(vb[e]) * qscale);
                }
                xchg[half * 128 + row] = mc;
                __syncthreads();
                mc = fmaxf(xchg[row], xchg[128 + row]);
                const float m_new = fmaxf(m_run, mc);
                const float factor = (m_run > -INFINITY && m_new > m_run) ? fast_exp2(m_run - m_new) : 1.0f;
                if (o_init && !__all_sync(FULL_MASK, factor == 1.0f)) {  // this half's 64 columns of O
                    uint32_t va[32], vb[32];
                    const uint32_t col = lane_base + TM_O + uint32_t(half * 64);
                    tmem_ld32_async(tmem + col, va);
                    tmem_ld32_async(tmem + col + 32, vb);
                    tmem_wait_ld(va);
                    tmem_wait_ld(vb);
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        va[e] = __float_as_uint(__uint_as_float(va[e]) * factor);
                        vb[e] = __float_as_uint(__uint_as_float(vb[e]) * factor);
                    }
                    tmem_st32_async(tmem + col, va);
                    tmem_st32_async(tmem + col + 32, vb);
                    tmem_wait_st();
                }
                l_run *= factor;
                m_run = m_new;
                // P tile by tile: each tile's P is computed while the previous tile's P.V runs
                bool pending = false, ok = true;
                for (int jt = 0; jt < ntile && ok; jt++) {
                    uint32_t ph[16], pl[16];
                    {
                        uint32_t v[32];
                        const int c0 = jt * ATC_KT + half * 32;
                        tmem_ld32_async(tmem + lane_base + uint32_t(c0), v);
                        tmem_wait_ld(v);
                        // columns outside [lo_r, hi_r) get P = 0; the tile is wholly visible for most rows
                        const bool whole = c0 >= lo_r && c0 + 32 <= hi_r;
                        const float nm = -m_run;
#pragma unroll
                        for (int e = 0; e < 32; e += 2) {
                            float p0 = fast_exp2(fmaf(__uint_as_float(v[e]), qscale, nm));
                            float p1 = fast_exp2(fmaf(__uint_as_float(v[e + 1]), qscale, nm));
                            if (!whole) {
                                p0 = (c0 + e >= lo_r && c0 + e < hi_r) ? p0 : 0.f;
                                p1 = (c0 + e + 1 >= lo_r && c0 + e + 1 < hi_r) ? p1 : 0.f;
                            }
                            l_run += p0;
                            l_run += p1;
                            const uint32_t hp = pack_bf16x2(p0, p1);
                            ph[e >> 1] = hp;
                            pl[e >> 1] = pack_bf16x2(p0 - lo_bf(hp), p1 - hi_bf(hp));
                        }
                    }
                    if (pending) {  // the previous tile's P.V has read the P buffer
                        ok = __syncthreads_and(bar_wait(bar_pv, ppv)) != 0;
                        ppv ^= 1u;
                        if (!ok) break;
                    }
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        const uint32_t off = sw128_offset(uint32_t(row), uint32_t(half * 4 + c) * 8);
                        *reinterpret_cast<uint4*>(smem + OFF_PH + off) = make_uint4(ph[4 * c], ph[4 * c + 1], ph[4 * c + 2], ph[4 * c + 3]);
                        *reinterpret_cast<uint4*>(smem + OFF_PL + off) = make_uint4(pl[4 * c], pl[4 * c + 1], pl[4 * c + 2], pl[4 * c + 3]);
                    }
                    fence_async_smem();
                    tc_fence_before();
                    __syncthreads();
                    if (t == 0) {
                        tc_fence_after();
                        const uint32_t idesc = tc_idesc(128);
                        const uint32_t vt = sbase + OFF_VT + uint32_t(jt) * 16384;
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)
                            umma_bf16(tmem + TM_O, sw128_desc(sbase + OFF_PH + kk * 32), sw128_desc(vt + kk * 32), idesc,
                                      uint32_t(o_init || kk > 0));
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)
                            umma_bf16(tmem + TM_O, sw128_desc(sbase + OFF_PL + kk * 32), sw128_desc(vt + kk * 32), idesc, 1u);
                        umma_commit(bar_pv);
                    }
                    o_init = true;
                    pending = true;
                }
                if (ok && pending) {
                    ok = __syncthreads_and(bar_wait(bar_pv, ppv)) != 0;
                    ppv ^= 1u;
                }
                if (!ok) {
                    if (t == 0) { atomicCAS(error, 0, 22); *abort_flag = 1; }
                    break;
                }
                tc_fence_after();
                tc_fence_before();
                __syncthreads();  // every MMA of the chunk is complete: the staging buffers are free
            }
        }
        __syncthreads();
        if (*abort_flag) break;
        // this run's rows: the split's (max, sum) in the natural-log domain and unnormalised O
        xchg[half * 128 + row] = l_run;
        __syncthreads();
        const float l_all = xchg[row] + xchg[128 + row];
        const bool keys_seen = mine && l_all > 0.f;
        if (klo < khi) {
            uint32_t va[32], vb[32];
            const int col = half * 64;
            tmem_ld32_async(tmem + lane_base + TM_O + uint32_t(col), va);
            tmem_ld32_async(tmem + lane_base + TM_O + uint32_t(col + 32), vb);
            tmem_wait_ld(va);
            tmem_wait_ld(vb);
            if (keys_seen) {
                float* po = a.part_o + ((size_t(row0 + my_tok) * a.splits + s) * ATC_H + my_head) * 128 + col;
#pragma unroll
                for (int e = 0; e < 32; e += 4) {
                    *reinterpret_cast<float4*>(po + e) = make_float4(__uint_as_float(va[e]), __uint_as_float(va[e + 1]),
                                                                      __uint_as_float(va[e + 2]), __uint_as_float(va[e + 3]));
                    *reinterpret_cast<float4*>(po + 32 + e) = make_float4(__uint_as_float(vb[e]), __uint_as_float(vb[e + 1]),
                                                                           __uint_as_float(vb[e + 2]), __uint_as_float(vb[e + 3]));
                }
            }
        }
        if (mine && half == 0)
            a.part_ml[(size_t(row0 + my_tok) * a.splits + s) * ATC_H + my_head] =
                keys_seen ? make_float2(m_run * ATC_LN2, l_all) : make_float2(-INFINITY, 0.f);
        tc_fence_before();
        __syncthreads();  // the O rows and sums are read before the next run overwrites them
        tc_fence_after();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace

bool attention_tc_supported(const AttnArgs& a) {
    return a.H == ATC_H && a.KV == 1 && a.rows >= 1 && (reinterpret_cast<uintptr_t>(a.q) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(a.keys) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.values) & 15) == 0 &&
           (a.full || (reinterpret_cast<uintptr_t>(a.rope_local) & 15) == 0);
}

// Keys per split: about an eighth of the cache, in whole 256-key chunks, so short prompts spread
// over more CTAs and long ones keep the partials (and the merge's reads) few.
static int attention_tc_span(int cap) {
    const int span = ((cap + ATC_SPLITS - 1) / ATC_SPLITS + ATC_CH - 1) / ATC_CH * ATC_CH;
    return span < ATC_CH ? ATC_CH : span;
}

int attention_tc_splits(int cap) {
    const int span = attention_tc_span(cap);
    return (cap + span - 1) / span;
}

cudaError_t configure_attention_tc() {
    return cudaFuncSetAttribute(k_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, int(ATC_SMEM));
}

// a.splits must be attention_tc_splits(keys), keys = a.key_bound (or a.cap when 0): the partial
// buffers hold that many splits per row.
cudaError_t launch_attention_tc(const AttnArgs& a, cudaStream_t s) {
    const int keys = a.key_bound > 0 && a.key_bound < a.cap ? a.key_bound : a.cap;
    if (!attention_tc_supported(a) || a.splits != attention_tc_splits(keys)) return cudaErrorInvalidValue;
    int* error = gemm_error_word(true);
    if (!error) return cudaErrorInvalidDevice;
    cudaError_t e = pdl_launch(k_attn_tc, dim3(a.splits, (a.rows + ATC_TOK - 1) / ATC_TOK), dim3(ATC_THREADS), ATC_SMEM, s,
                               a, attention_tc_span(keys), error);
    if (e != cudaSuccess) return e;
    return launch_attention_merge(a, s);
}

}  // namespace plamo
