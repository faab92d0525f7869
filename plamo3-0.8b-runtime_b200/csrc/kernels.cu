// sm_100a kernels for the PLaMo-3 decoder hot path (CUDA-core path: batch-1 / few-row decode
// GEMVs, norms, QK-norm + RoPE + KV append, split-K attention, argmax).
//
// Reference counterparts (mikuteto-dev/plamo3-0.8b-runtime, Sources/Plamo/):
//   k_gemv         Kernels.metal:92-114 (linear), :149-200 (matrix), Batch.metal:171-221
//                  (project3/4), :202-210 (swiglu, fused here), :704-729 (argmax, fused here)
//   load16<true>   Kernels.metal:23-44 (packed_bits / packed_four)
//   k_norm         Kernels.metal:46-90
//   k_embed_norm   Runtime.swift:104-110 + :377
//   k_qkv          Kernels.metal:223-274, Batch.metal:1-39
//   k_attn_*       Kernels.metal:277-285, :301-345, :358-437, :440-562, Batch.metal:42-168
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cfloat>

namespace plamo {

// --------------------------------------------------------------------------------------------
// streaming loads (weights are read once per token: keep them out of L1)
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ld_stream2(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

// 16 consecutive weights starting at flat element `el` (multiple of 16) as bf16 pairs.
template <bool PACKED>
__device__ __forceinline__ void load16(const Linear& lin, size_t el, uint32_t (&wp)[8]) {
    if (!PACKED) {
        const uint8_t* p = lin.w + el * 2;
        const uint4 a = ld_stream(p), b = ld_stream(p + 16);
        wp[0] = a.x; wp[1] = a.y; wp[2] = a.z; wp[3] = a.w;
        wp[4] = b.x; wp[5] = b.y; wp[6] = b.z; wp[7] = b.w;
    } else {
        const uint32_t entry = __ldg(lin.offsets + (el >> 7));
        const uint32_t i0 = uint32_t(el & 127);
        const uint8_t* blk = lin.w + (entry & ~63u);
        const uint32_t tag = entry & 63u;
        if (tag) {
            const uint4 sm = ld_stream(blk + i0);
            const uint2 cd = ld_stream2(blk + 128 + (i0 >> 1));
            decode16(sm, cd, tag + 107u, wp);
        } else {
            const uint4 a = ld_stream(blk + 2 * i0), b = ld_stream(blk + 2 * i0 + 16);
            wp[0] = a.x; wp[1] = a.y; wp[2] = a.z; wp[3] = a.w;
            wp[4] = b.x; wp[5] = b.y; wp[6] = b.z; wp[7] = b.w;
        }
    }
}

// --------------------------------------------------------------------------------------------
// GEMV over R activation rows. One warp per output row; lane l covers weights
// [g*512 + 16l, +16) of every 512-weight group g, so raw and packed weights are summed in the same
// order (packed == raw bit for bit). x is staged in shared memory, permuted so that each 16-byte
// shared load of a warp is conflict-free.
template <int R, bool PACKED, int MODE>
__global__ void __launch_bounds__(256) k_gemv(GemvArgs a) {
    pdl_enter();
    extern __shared__ uint4 xs[];
    constexpr int NW = MODE == GEMV_SWIGLU ? 2 : 1;
    // Two interleaved accumulators per (weight row, activation row): the per-row summation order
    // is the same for every R and mode, so a batched step equals the batch-1 path bit for bit.
    constexpr int A = 2;
    constexpr int NV = NW * R;
    // One load batch = one 1536-weight segment (3 groups of 512); segment partials are folded into
    // the running total in order (the summation order of the restatement's dot_bf16).
    constexpr int UG = 3;
    const int K = a.lin.K, K8 = K >> 3, KP8 = (K8 + 63) & ~63;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    for (int i = t; i < R * K8; i += 256) {
        const int r = i / K8, c = i - r * K8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < a.rows) v = reinterpret_cast<const uint4*>(a.x + size_t(r) * K)[c];
        const int g = c >> 6, within = c & 63;
        xs[r * KP8 + g * 64 + (within & 1) * 32 + (within >> 1)] = v;
    }
    __syncthreads();
    const int Mout = MODE == GEMV_SWIGLU ? a.lin.M / 2 : a.lin.M;
    const int G = (K + 511) >> 9;
    constexpr int STRIDE = 32 / NV;
    const int idx = lane / STRIDE;
    const bool holder = (lane % STRIDE) == 0;
    unsigned long long best = 0ull;
    for (int m = blockIdx.x * 8 + warp; m < Mout; m += gridDim.x * 8) {
        float acc[NW][R][A], tot[NW][R];
#pragma unroll
        for (int wr = 0; wr < NW; wr++)
#pragma unroll
            for (int r = 0; r < R; r++) {
                tot[wr][r] = 0.f;
#pragma unroll
                for (int q = 0; q < A; q++) acc[wr][r][q] = 0.f;
            }
        for (int g0 = 0; g0 < G; g0 += UG) {
            uint32_t wp[UG][NW][8];
#pragma unroll
            for (int u = 0; u < UG; u++) {
                const int e0 = (g0 + u) * 512 + lane * 16;
#pragma unroll
                for (int wr = 0; wr < NW; wr++) {
                    if (g0 + u < G && e0 < K) {
                        load16<PACKED>(a.lin, size_t(m + wr * Mout) * K + e0, wp[u][wr]);
                    } else {
#pragma unroll
                        for (int k = 0; k < 8; k++) wp[u][wr][k] = 0u;
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < UG; u++) {
                const int g = g0 + u;
                if (g < G && g * 512 + lane * 16 < K) {
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        const uint4 xa = xs[r * KP8 + g * 64 + lane];
                        const uint4 xb = xs[r * KP8 + g * 64 + 32 + lane];
                        const uint32_t xp[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
                        for (int wr = 0; wr < NW; wr++)
#pragma unroll
                            for (int k = 0; k < 8; k++) {
                                acc[wr][r][(2 * k) % A] = fmaf(lo_bf(wp[u][wr][k]), lo_bf(xp[k]), acc[wr][r][(2 * k) % A]);
                                acc[wr][r][(2 * k + 1) % A] = fmaf(hi_bf(wp[u][wr][k]), hi_bf(xp[k]), acc[wr][r][(2 * k + 1) % A]);
                            }
                    }
                }
            }
#pragma unroll
            for (int wr = 0; wr < NW; wr++)
#pragma unroll
                for (int r = 0; r < R; r++) {
                    tot[wr][r] = tot[wr][r] + (acc[wr][r][0] + acc[wr][r][1]);
                    acc[wr][r][0] = 0.f;
                    acc[wr][r][1] = 0.f;
                }
        }
        float v[NV];
#pragma unroll
        for (int wr = 0; wr < NW; wr++)
#pragma unroll
            for (int r = 0; r < R; r++)
                v[wr * R + r] = tot[wr][r];
        const float res = warp_reduce_transposed<NV>(v, lane);
        if (MODE == GEMV_SWIGLU) {
            const float u = __shfl_down_sync(FULL_MASK, res, 16);
            if (holder && idx < R && idx < a.rows) {
                const float gq = rbf(res), uq = rbf(u);
                const float act = rbf(rbf(gq / (1.0f + pexp(-gq))) * uq);
                const int orow = a.out_map ? a.out_map[idx] : idx;
                a.y[size_t(orow) * a.ystride + m] = uint16_t(f2bf(act));
            }
        } else if (holder && idx < a.rows) {
            const int orow = a.out_map ? a.out_map[idx] : idx;
            const uint32_t b = f2bf(res);
            a.y[size_t(orow) * a.ystride + m] = uint16_t(b);
            if (MODE == GEMV_LOGITS) {
                const unsigned long long key = argmax_key(bf2f(b), uint32_t(m));
                best = key > best ? key : best;
            }
        }
    }
    if (MODE == GEMV_LOGITS) {
        __shared__ unsigned long long s_best[8][R];
        if (holder) s_best[warp][idx] = best;
        __syncthreads();
        if (t < R && t < a.rows) {
            unsigned long long b = 0ull;
#pragma unroll
            for (int w = 0; w < 8; w++) b = s_best[w][t] > b ? s_best[w][t] : b;
            const int orow = a.out_map ? a.out_map[t] : t;
            if (b) atomicMax(a.keys + orow, b);
        }
    }
}

// --------------------------------------------------------------------------------------------
// RMSNorm rows (Kernels.metal:46-90). One CTA of 256 threads per row, n <= 4096.
constexpr int NPT = 16;

__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float s = lane < 8 ? red[lane] : 0.f;
        s = warp_sum(s);
        if (lane == 0) red[8] = s;
    }
    __syncthreads();
    return red[8];
}

// The factors bf16(w + offset) of a norm row, read before the row's reduction so their load
// latency overlaps it.
template <int NJ>
__device__ __forceinline__ void norm_factors(const uint16_t* w, int n, float offset, float (&f)[NJ]) {
#pragma unroll
    for (int j = 0; j < NJ; j++) {
        const int i = threadIdx.x + j * 256;
        f[j] = i < n ? rbf(bf2f(w[i]) + offset) : 0.f;
    }
}

// Elements past n are zero in v and add nothing to the thread's chain, so the sum does not depend
// on NJ (elements per thread) once 256 NJ >= n.
template <int NJ>
__device__ __forceinline__ void norm_row(const float (&v)[NJ], int n, const float (&f)[NJ], float* red,
                                         float (&z)[NJ]) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; j++) ss = fmaf(v[j], v[j], ss);
    const float total = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(total / float(n) + PLAMO_EPS);
#pragma unroll
    for (int j = 0; j < NJ; j++) {
        const int i = threadIdx.x + j * 256;
        z[j] = i < n ? rbf(rbf(v[j] * scale) * f[j]) : 0.f;
    }
}

// Source elements of a row given as split-K partials [split][rows][n]: the bf16 rounding of the
// sum in split order, the value k_gemm_tc_finish would have stored. Every partial of a group of
// eight splits is loaded before the group's adds.
template <int NJ>
__device__ __forceinline__ void split_source(const NormArgs& a, size_t row, float (&v)[NJ]) {
    const size_t ss = size_t(a.rows) * a.n;
    float acc[NJ];
    for (int s0 = 0; s0 < a.src_splits; s0 += 8) {
        float pv[8][NJ];
#pragma unroll
        for (int k = 0; k < 8; k++)
#pragma unroll
            for (int j = 0; j < NJ; j++) {
                const int i = threadIdx.x + j * 256;
                pv[k][j] = s0 + k < a.src_splits && i < a.n ? a.src_part[size_t(s0 + k) * ss + row + i] : 0.f;
            }
#pragma unroll
        for (int k = 0; k < 8; k++)
#pragma unroll
            for (int j = 0; j < NJ; j++)
                if (s0 + k < a.src_splits) acc[j] = s0 + k == 0 ? pv[k][j] : acc[j] + pv[k][j];
    }
#pragma unroll
    for (int j = 0; j < NJ; j++) v[j] = threadIdx.x + j * 256 < a.n ? rbf(acc[j]) : 0.f;
}

// Every global read of the row (source, norm weights, residual row, next norm weights) is issued
// before the first reduction, so a row pays one memory latency instead of one per stage; the
// arithmetic and its order are unchanged.
template <int NJ>
__global__ void __launch_bounds__(256) k_norm(NormArgs a) {
    pdl_enter();
    __shared__ float red[9];
    const int r = blockIdx.x;
    const size_t row = size_t(r) * a.n;
    float v[NJ], z[NJ], f[NJ], xr[NJ], g[NJ];
    if (a.src_splits > 0) split_source<NJ>(a, row, v);
#pragma unroll
    for (int j = 0; j < NJ; j++) {
        const int i = threadIdx.x + j * 256;
        if (a.src_splits <= 0) v[j] = i < a.n ? bf2f(a.src[row + i]) : 0.f;
        xr[j] = a.residual && i < a.n ? bf2f(a.x[row + i]) : 0.f;
    }
    norm_factors(a.w, a.n, a.offset, f);
    if (a.next_w) norm_factors(a.next_w, a.n, 1.0f, g);
    norm_row(v, a.n, f, red, z);
    if (!a.residual) {
        const int orow = a.out_map ? a.out_map[r] : r;
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int i = threadIdx.x + j * 256;
            if (i < a.n) {
                const uint16_t b = uint16_t(f2bf(z[j]));
                a.x[row + i] = b;
                if (a.y2) a.y2[size_t(orow) * a.n + i] = b;
            }
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < NJ; j++) {
        const int i = threadIdx.x + j * 256;
        if (i < a.n) {
            const float val = rbf(xr[j] + z[j]);
            a.x[row + i] = uint16_t(f2bf(val));
            v[j] = val;
        } else {
            v[j] = 0.f;
        }
    }
    if (!a.next_w) return;
    norm_row(v, a.n, g, red, z);
#pragma unroll
    for (int j = 0; j < NJ; j++) {
        const int i = threadIdx.x + j * 256;
        if (i < a.n) a.next[row + i] = uint16_t(f2bf(z[j]));
    }
}

// Embedding gather (bf16 rows, exact) + layer-0 pre-mixer norm; clears the argmax keys the head
// of this call will write.
__global__ void __launch_bounds__(256) k_embed_norm(const int* ids, int vocab, const uint16_t* embed, const uint16_t* w,
                                                    int d, uint16_t* x, uint16_t* h, unsigned long long* keys,
                                                    const int* key_map, int nkeys) {
    pdl_enter();
    __shared__ float red[9];
    const int r = blockIdx.x;
    if (r == 0 && keys)
        for (int i = threadIdx.x; i < nkeys; i += 256) keys[key_map ? key_map[i] : i] = 0ull;
    // Host-supplied ids are validated before upload; a device-chained id (an argmax) is always in
    // range unless every logit was NaN, in which case row 0 is read instead of faulting.
    const int id = ids[r];
    const size_t row = size_t(id >= 0 && id < vocab ? id : 0) * d;
    float v[NPT], z[NPT], f[NPT];
#pragma unroll
    for (int j = 0; j < NPT; j++) {
        const int i = threadIdx.x + j * 256;
        uint16_t b = 0;
        if (i < d) { b = embed[row + i]; x[size_t(r) * d + i] = b; }
        v[j] = bf2f(b);
    }
    norm_factors(w, d, 1.0f, f);
    norm_row(v, d, f, red, z);
#pragma unroll
    for (int j = 0; j < NPT; j++) {
        const int i = threadIdx.x + j * 256;
        if (i < d) h[size_t(r) * d + i] = uint16_t(f2bf(z[j]));
    }
}

// --------------------------------------------------------------------------------------------

// Per (row, head) warp: QK RMSNorm (w + 1), RoPE of queries, KV append into the ring slot
// pos % cap of the row's lane slab (global layers store rotated keys, local layers raw keys).
__global__ void __launch_bounds__(128) k_qkv(QkvArgs a) {
    pdl_enter();
    const int gw = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    const int heads = a.H + a.KV;
    if (gw >= a.rows * heads) return;
    const int r = gw / heads, h = gw - r * heads;
    const RowDesc dsc = a.desc[r];
    int first, count, begin, end, qcoord;
    if (a.full) {
        first = 0; count = dsc.cstart + dsc.crows; end = dsc.pos + 1; begin = 0; qcoord = dsc.pos;
    } else {  // Runtime.swift:389-392, Kernels.metal:251,368-369, Batch.metal:31
        first = max(0, dsc.cstart - (a.W - 1));
        count = dsc.cstart + dsc.crows - first;
        end = dsc.pos - first + 1;
        begin = max(0, end - a.W);
        qcoord = dsc.pos - first;
    }
    if (h == 0 && lane == 0) a.geo[r] = RowGeo{first, count, begin, end};
    const int width = (a.H + 2 * a.KV) * 128;
    const uint16_t* src = a.qkv + size_t(r) * width + h * 128;
    // the head's elements (and for a key head its value head's) as bf16 bits; from split-K
    // partials, the bf16 rounding of their sum in split order (k_gemm_tc_finish's value)
    uint32_t hb[4], vb[4];
    if (a.src_splits > 0) {
        const int nv = h < a.H ? 4 : 8;
        const size_t ss_ = size_t(a.rows) * width, base = size_t(r) * width + h * 128;
        float acc[8];
        for (int s0 = 0; s0 < a.src_splits; s0 += 4) {
            float pv[4][8];
#pragma unroll
            for (int k = 0; k < 4; k++)
#pragma unroll
                for (int j = 0; j < 8; j++)
                    pv[k][j] = s0 + k < a.src_splits && j < nv
                                   ? a.src_part[size_t(s0 + k) * ss_ + base + (j >> 2) * a.KV * 128 + lane + 32 * (j & 3)]
                                   : 0.f;
#pragma unroll
            for (int k = 0; k < 4; k++)
#pragma unroll
                for (int j = 0; j < 8; j++)
                    if (s0 + k < a.src_splits) acc[j] = s0 + k == 0 ? pv[k][j] : acc[j] + pv[k][j];
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            hb[j] = f2bf(acc[j]);
            vb[j] = f2bf(acc[4 + j]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            hb[j] = src[lane + 32 * j];
            vb[j] = h < a.H ? 0u : src[a.KV * 128 + lane + 32 * j];  // v head kvh sits KV heads after k head kvh
        }
    }
    float v[4], ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; j++) { v[j] = bf2f(hb[j]); ss = fmaf(v[j], v[j], ss); }
    ss = warp_sum(ss);
    const float scale = 1.0f / sqrtf(ss / 128.0f + PLAMO_EPS);
    const uint16_t* nw = h < a.H ? a.q_norm : a.k_norm;
    float z[4];
#pragma unroll
    for (int j = 0; j < 4; j++) z[j] = rbf(rbf(v[j] * scale) * rbf(bf2f(nw[lane + 32 * j]) + 1.0f));
    if (h < a.H) {
        const uint32_t* table = a.full ? a.rope_global + size_t(qcoord) * 64 : a.rope_local + size_t(qcoord) * 64;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int d = lane + 32 * j;
            a.q[size_t(r) * a.H * 128 + h * 128 + d] = uint16_t(f2bf(rope_rotate(z[j], z[(j + 2) & 3], d, table[d & 63])));
        }
    } else {
        const int kvh = h - a.H;
        const size_t slot = size_t(dsc.lane) * a.lane_stride + (size_t(dsc.pos % a.cap) * a.KV + kvh) * 128;
        const uint32_t* table = a.rope_global + size_t(dsc.pos) * 64;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int d = lane + 32 * j;
            const float k = a.full ? rope_rotate(z[j], z[(j + 2) & 3], d, table[d & 63]) : z[j];
            a.keys[slot + d] = uint16_t(f2bf(k));
            a.values[slot + d] = uint16_t(vb[j]);
        }
    }
}

// --------------------------------------------------------------------------------------------
// Split-K attention. CTA (split s, row r) covers keys [s*per, (s+1)*per) of the row's window
// (clipped to its visible range), computes scores for all heads (MQA/GQA: key tiles shared),
// local softmax statistics and the unnormalised P.V partial; k_attn_merge combines the splits
// (log-sum-exp) and rounds to bf16 (Kernels.metal:440-562).
constexpr int QS = 132;
// Keys per staged K / V tile: 64 with one KV head; with grouped-query attention a tile holds every
// KV head of its keys, so fewer keys keep the fp32 rotated tile and the bf16 staging in shared memory.
__host__ __device__ constexpr int attn_tile_keys(int KV) { return KV == 1 ? 64 : KV == 2 ? 32 : 16; }

int attention_per_max(int cap, int splits) { return ((cap + splits - 1) / splits + 31) & ~31; }
size_t attention_smem(int H, int KV, int per_max) {
    const size_t AT = size_t(attn_tile_keys(KV));
    return sizeof(float) * (size_t(H) * QS + AT * (KV * 128 + 4) + AT * 64 + size_t(H) * per_max) +
           2 * AT * KV * 128 * 2;  // key / value staging, and the first value tile fetched early
}

// Stages rows [k0, k0 + tk) of the key (or value) cache window into shared memory as raw bf16 with
// 16-byte loads: one round trip per tile.
__device__ __forceinline__ void stage_rows(uint4* dst, const uint16_t* base, int first, int k0, int tk, int cap,
                                           int KV) {
    const int rowv = KV * 16;
    for (int i = threadIdx.x; i < tk * rowv; i += blockDim.x) {
        const int j = i / rowv, c = i - j * rowv;
        const int phys = (first + k0 + j) % cap;
        dst[i] = __ldg(reinterpret_cast<const uint4*>(base + size_t(phys) * KV * 128) + c);
    }
}

// The same rows copied with cp.async (16 bytes a thread, L2 to shared memory), so the copy runs
// while the block computes; complete after cp_async_wait_all and a barrier.
__device__ __forceinline__ void stage_rows_async(uint4* dst, const uint16_t* base, int first, int k0, int tk, int cap,
                                                 int KV) {
    const int rowv = KV * 16;
    for (int i = threadIdx.x; i < tk * rowv; i += blockDim.x) {
        const int j = i / rowv, c = i - j * rowv;
        const int phys = (first + k0 + j) % cap;
        const uint4* src = reinterpret_cast<const uint4*>(base + size_t(phys) * KV * 128) + c;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst + i))),
                     "l"(src)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int AT>
__global__ void __launch_bounds__(256) k_attn_partial(AttnArgs a) {
    pdl_enter();
    extern __shared__ __align__(16) float smem[];
    const int r = blockIdx.y, s = blockIdx.x, t = threadIdx.x;
    const RowGeo g = a.geo[r];
    const int lane_id = a.desc[r].lane;
    const int H = a.H, KV = a.KV, group = H / KV, KS = KV * 128 + 4;  // 16-byte rows, rows 4 banks apart
    int per = (g.count + a.splits - 1) / a.splits;
    per = (per + 31) & ~31;
    const int k0 = s * per, k1 = min(k0 + per, g.count);
    const int lo = max(k0, g.begin), hi = min(k1, g.end);
    float2* ml = a.part_ml + (size_t(r) * a.splits + s) * H;
    if (lo >= hi) {
        for (int h = t; h < H; h += 256) ml[h] = make_float2(-INFINITY, 0.f);
        return;
    }
    float* qs = smem;                                   // [H][QS]
    float* kr = qs + H * QS;                            // [AT][KS] rotated keys (fp32)
    uint32_t* rope = reinterpret_cast<uint32_t*>(kr + AT * KS);  // [AT][64]
    float* sc = reinterpret_cast<float*>(rope + AT * 64);        // [H][per_max]
    uint4* raw = reinterpret_cast<uint4*>(sc + H * a.per_max);   // [AT][KV*128] bf16
    uint4* vfirst = raw + AT * KV * 16;                          // [AT][KV*128] bf16: value tile 0
    const uint16_t* raw16 = reinterpret_cast<const uint16_t*>(raw);
    const uint16_t* kbase = a.keys + size_t(lane_id) * a.lane_stride;
    const uint16_t* vbase = a.values + size_t(lane_id) * a.lane_stride;
    const int n = hi - lo;
    // the first value tile streams in while the keys are staged, rotated and scored
    stage_rows_async(vfirst, vbase, g.first, lo, min(AT, n), a.cap, KV);
    const uint16_t* qrow = a.q + size_t(r) * H * 128;
    if ((reinterpret_cast<uintptr_t>(qrow) & 15) == 0) {  // eight values per 16-byte read
        for (int i8 = t; i8 < H * 16; i8 += 256) {
            const uint4 w = reinterpret_cast<const uint4*>(qrow)[i8];
            float* dst = qs + (i8 >> 4) * QS + (i8 & 15) * 8;
            reinterpret_cast<float4*>(dst)[0] = make_float4(bf2f(w.x & 0xffffu), bf2f(w.x >> 16), bf2f(w.y & 0xffffu), bf2f(w.y >> 16));
            reinterpret_cast<float4*>(dst)[1] = make_float4(bf2f(w.z & 0xffffu), bf2f(w.z >> 16), bf2f(w.w & 0xffffu), bf2f(w.w >> 16));
        }
    } else {
        for (int i = t; i < H * 128; i += 256) qs[(i >> 7) * QS + (i & 127)] = bf2f(qrow[i]);
    }
    // pass 1: scores of every visible key of this split
    for (int t0 = 0; t0 < n; t0 += AT) {
        const int tk = min(AT, n - t0);
        __syncthreads();
        stage_rows(raw, kbase, g.first, lo + t0, tk, a.cap, KV);
        if (!a.full)
            for (int i = t; i < tk * 16; i += 256)
                reinterpret_cast<uint4*>(rope)[i] =
                    __ldg(reinterpret_cast<const uint4*>(a.rope_local + size_t(lo + t0 + (i >> 4)) * 64) + (i & 15));
        __syncthreads();
        // eight consecutive elements per thread and pass (16-byte shared-memory reads and writes)
        for (int i8 = t; i8 < tk * KV * 16; i8 += 256) {
            const int j = i8 / (KV * 16), e0 = (i8 - j * (KV * 16)) * 8;
            const uint16_t* kr16 = raw16 + j * KV * 128;
            const uint4 w = *reinterpret_cast<const uint4*>(kr16 + e0);
            const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
            float val[8];
            if (a.full) {
#pragma unroll
                for (int k = 0; k < 8; k++) val[k] = bf2f((wv[k >> 1] >> (16 * (k & 1))) & 0xffffu);
            } else {  // window-relative re-rotation of raw local keys (Kernels.metal:277-285)
                const int d0 = e0 & 127, kvoff = e0 - d0, p0 = d0 < 64 ? d0 + 64 : d0 - 64;
                const uint4 o = *reinterpret_cast<const uint4*>(kr16 + kvoff + p0);
                const uint32_t ov[4] = {o.x, o.y, o.z, o.w};
                const uint4 c0 = *reinterpret_cast<const uint4*>(rope + j * 64 + (d0 & 63));
                const uint4 c1 = *reinterpret_cast<const uint4*>(rope + j * 64 + (d0 & 63) + 4);
                const uint32_t cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
                for (int k = 0; k < 8; k++)
                    val[k] = rope_rotate(bf2f((wv[k >> 1] >> (16 * (k & 1))) & 0xffffu),
                                         bf2f((ov[k >> 1] >> (16 * (k & 1))) & 0xffffu), d0 + k, cs[k]);
            }
            float4* dst = reinterpret_cast<float4*>(kr + j * KS + e0);
            dst[0] = make_float4(val[0], val[1], val[2], val[3]);
            dst[1] = make_float4(val[4], val[5], val[6], val[7]);
        }
        __syncthreads();
        const int j = t & (AT - 1);
        if (j < tk) {
            for (int h = t / AT; h < H; h += 256 / AT) {
                // 16-byte shared-memory reads; the products are still added in d order
                const float4* qh = reinterpret_cast<const float4*>(qs + h * QS);
                const float4* kj = reinterpret_cast<const float4*>(kr + j * KS + (h / group) * 128);
                float acc = 0.f;
#pragma unroll 8
                for (int d4 = 0; d4 < 32; d4++) {
                    const float4 q = qh[d4], k = kj[d4];
                    acc = fmaf(q.x, k.x, acc);
                    acc = fmaf(q.y, k.y, acc);
                    acc = fmaf(q.z, k.z, acc);
                    acc = fmaf(q.w, k.w, acc);
                }
                sc[h * a.per_max + t0 + j] = acc * PLAMO_ATTN_SCALE;
            }
        }
    }
    __syncthreads();
    // pass 2: split-local softmax statistics per head
    const int warp = t >> 5, lane = t & 31;
    for (int h = warp; h < H; h += 8) {
        float* p = sc + h * a.per_max;
        float m = -INFINITY;
        for (int i = lane; i < n; i += 32) m = fmaxf(m, p[i]);
        m = warp_max(m);
        float l = 0.f;
        for (int i = lane; i < n; i += 32) { const float e = pexp(p[i] - m); p[i] = e; l += e; }
        l = warp_sum(l);
        if (lane == 0) ml[h] = make_float2(m, l);
    }
    // pass 3: unnormalised P.V over staged value tiles
    const int d = t & 127, hh = t >> 7;
    float acc[16];
#pragma unroll
    for (int q = 0; q < 16; q++) acc[q] = 0.f;
    for (int t0 = 0; t0 < n; t0 += AT) {
        const int tk = min(AT, n - t0);
        __syncthreads();
        if (t0 == 0) asm volatile("cp.async.wait_all;" ::: "memory");
        else stage_rows(raw, vbase, g.first, lo + t0, tk, a.cap, KV);
        __syncthreads();
        const uint16_t* vtile = t0 == 0 ? reinterpret_cast<const uint16_t*>(vfirst) : raw16;
        int i = 0;
        if (KV == 1) {
            // four keys at a time: one 16-byte read of each head's scores; every output still adds
            // the keys in order
            for (; i + 4 <= tk; i += 4) {
                float v[4];
#pragma unroll
                for (int u = 0; u < 4; u++) v[u] = bf2f(vtile[(i + u) * 128 + d]);
#pragma unroll
                for (int q = 0; q < 16; q++) {
                    const int h = hh + 2 * q;
                    if (h < H) {
                        const float4 pr = *reinterpret_cast<const float4*>(sc + h * a.per_max + t0 + i);
                        acc[q] = fmaf(pr.x, v[0], acc[q]);
                        acc[q] = fmaf(pr.y, v[1], acc[q]);
                        acc[q] = fmaf(pr.z, v[2], acc[q]);
                        acc[q] = fmaf(pr.w, v[3], acc[q]);
                    }
                }
            }
        }
        for (; i < tk; i++) {
            const uint16_t* vr = vtile + i * KV * 128;
            if (KV == 1) {
                const float v = bf2f(vr[d]);
#pragma unroll
                for (int q = 0; q < 16; q++) {
                    const int h = hh + 2 * q;
                    if (h < H) acc[q] = fmaf(sc[h * a.per_max + t0 + i], v, acc[q]);
                }
            } else {
#pragma unroll
                for (int q = 0; q < 16; q++) {
                    const int h = hh + 2 * q;
                    if (h < H) acc[q] = fmaf(sc[h * a.per_max + t0 + i], bf2f(vr[(h / group) * 128 + d]), acc[q]);
                }
            }
        }
    }
    float* po = a.part_o + (size_t(r) * a.splits + s) * H * 128;
#pragma unroll
    for (int q = 0; q < 16; q++) {
        const int h = hh + 2 * q;
        if (h < H) po[h * 128 + d] = acc[q];
    }
}

// One thread per 8 consecutive outputs of one (row, head): split statistics and 16-byte partial
// loads. Up to eight splits are loaded in one round trip and then folded; more splits are taken
// eight at a time (their maxima first, then the sums). Either way the max runs over the splits in
// order and the sum and P.V chains add the splits in order, as the single-pass form did.
constexpr int MERGE_DIMS = 8;

__device__ __forceinline__ void merge_fold(const float2 (&st)[8], const float4 (&pa)[8], const float4 (&pb)[8], int n,
                                           float M, float& L, float (&o)[MERGE_DIMS]) {
#pragma unroll
    for (int j = 0; j < 8; j++) {
        if (j < n && st[j].y > 0.f) {
            const float w = pexp(st[j].x - M);
            L = fmaf(w, st[j].y, L);
            const float pv[MERGE_DIMS] = {pa[j].x, pa[j].y, pa[j].z, pa[j].w, pb[j].x, pb[j].y, pb[j].z, pb[j].w};
#pragma unroll
            for (int k = 0; k < MERGE_DIMS; k++) o[k] = fmaf(pv[k], w, o[k]);
        }
    }
}

__global__ void __launch_bounds__(256) k_attn_merge(AttnArgs a) {
    pdl_enter();
    const int per_row = (a.H * (128 / MERGE_DIMS) + 255) / 256;
    const int r = blockIdx.x / per_row;
    const int idx = (blockIdx.x - r * per_row) * 256 + threadIdx.x;
    if (idx >= a.H * (128 / MERGE_DIMS)) return;
    const int h = idx / (128 / MERGE_DIMS), d0 = (idx % (128 / MERGE_DIMS)) * MERGE_DIMS;
    const float2* ml = a.part_ml + size_t(r) * a.splits * a.H + h;  // split s at ml[s * H]
    const float* po = a.part_o + size_t(r) * a.splits * a.H * 128 + h * 128 + d0;
    const size_t po_split = size_t(a.H) * 128;
    float M = -INFINITY, L = 0.f, o[MERGE_DIMS];
#pragma unroll
    for (int k = 0; k < MERGE_DIMS; k++) o[k] = 0.f;
    float2 st[8];
    float4 pa[8], pb[8];
    auto load = [&](int s0) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            if (s0 + j < a.splits) {
                st[j] = ml[size_t(s0 + j) * a.H];
                // partials are read whether or not the split had keys; only splits with keys use them
                const float4* q = reinterpret_cast<const float4*>(po + (s0 + j) * po_split);
                pa[j] = q[0];
                pb[j] = q[1];
            } else {
                st[j] = make_float2(-INFINITY, 0.f);
            }
        }
    };
    if (a.splits <= 8) {
        load(0);
#pragma unroll
        for (int j = 0; j < 8; j++) M = fmaxf(M, st[j].x);
        merge_fold(st, pa, pb, a.splits, M, L, o);
    } else {
        for (int s0 = 0; s0 < a.splits; s0 += 8) {
            float m[8];
#pragma unroll
            for (int j = 0; j < 8; j++) m[j] = s0 + j < a.splits ? ml[size_t(s0 + j) * a.H].x : -INFINITY;
#pragma unroll
            for (int j = 0; j < 8; j++) M = fmaxf(M, m[j]);
        }
        for (int s0 = 0; s0 < a.splits; s0 += 8) {
            load(s0);
            merge_fold(st, pa, pb, a.splits - s0, M, L, o);
        }
    }
    uint16_t* out = a.out + size_t(r) * a.H * 128 + h * 128 + d0;
    uint32_t packed[MERGE_DIMS / 2];
#pragma unroll
    for (int k = 0; k < MERGE_DIMS / 2; k++)
        packed[k] = f2bf(o[2 * k] / L) | (f2bf(o[2 * k + 1] / L) << 16);
    if ((reinterpret_cast<uintptr_t>(out) & 15) == 0) {
        *reinterpret_cast<uint4*>(out) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    } else {
#pragma unroll
        for (int k = 0; k < MERGE_DIMS; k++) out[k] = uint16_t(packed[k >> 1] >> (16 * (k & 1)));
    }
}

// --------------------------------------------------------------------------------------------
// Converts argmax keys to ids and clears each key after reading it (every forward leaves the keys
// zeroed, whichever decode path runs next). Device-chained decode also feeds the id back as the
// next input, advances the row descriptor and appends the id to a bounded history.
__global__ void k_finalize(unsigned long long* keys, const int* key_map, int rows, int* result,
                           int* chain_ids, RowDesc* advance, int* hist, int* hist_count, int hist_cap) {
    pdl_enter();
    const int r = threadIdx.x;
    if (r >= rows) return;
    const int k = key_map ? key_map[r] : r;
    const uint32_t id = argmax_index(keys[k]);
    keys[k] = 0ull;
    result[k] = int(id);
    if (chain_ids) chain_ids[r] = int(id);
    if (advance) { advance[r].pos += 1; advance[r].cstart += 1; }
    if (hist && r == 0) {
        const int c = *hist_count;
        if (c >= 0 && c < hist_cap) {
            hist[c] = int(id);
            *hist_count = c + 1;
        }
    }
}

// Standalone first-index argmax over bf16 rows (Kernels.metal:704-729).
__global__ void __launch_bounds__(256) k_argmax(const uint16_t* logits, int n, unsigned long long* keys) {
    pdl_enter();
    const int r = blockIdx.y;
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * 256 + threadIdx.x; i < n; i += gridDim.x * 256) {
        const unsigned long long k = argmax_key(bf2f(logits[size_t(r) * n + i]), uint32_t(i));
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(FULL_MASK, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0 && best) atomicMax(keys + r, best);
}

__global__ void k_packed_decode(Linear lin, long long count, uint16_t* out) {
    const long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (c * 16 >= count) return;
    uint32_t wp[8];
    load16<true>(lin, size_t(c) * 16, wp);
#pragma unroll
    for (int k = 0; k < 8; k++) reinterpret_cast<uint32_t*>(out + c * 16)[k] = wp[k];
}

// --------------------------------------------------------------------------------------------
// launchers

// Staged-activation budget per GEMV CTA (below the 227 KB opt-in limit minus static scratch).
constexpr size_t GEMV_SMEM_MAX = 224 * 1024;

template <int R, bool P, int M>
static cudaError_t gemv_launch(const GemvArgs& a, cudaStream_t s) {
    const int K8 = a.lin.K >> 3, KP8 = (K8 + 63) & ~63;
    const size_t smem = size_t(R) * KP8 * 16;
    const int Mout = M == GEMV_SWIGLU ? a.lin.M / 2 : a.lin.M;
    int grid = (Mout + 7) / 8;
    if (M == GEMV_LOGITS) grid = grid < 148 * 4 ? grid : 148 * 4;
    return pdl_launch(k_gemv<R, P, M>, dim3(grid), dim3(256), smem, s, a);
}

template <int R, bool P>
static cudaError_t gemv_mode(const GemvArgs& a, int mode, cudaStream_t s) {
    switch (mode) {
        case GEMV_PLAIN: return gemv_launch<R, P, GEMV_PLAIN>(a, s);
        case GEMV_SWIGLU: return gemv_launch<R, P, GEMV_SWIGLU>(a, s);
        default: return gemv_launch<R, P, GEMV_LOGITS>(a, s);
    }
}

template <bool P>
static cudaError_t gemv_rows(const GemvArgs& a, int mode, cudaStream_t s) {
    if (a.rows <= 1) return gemv_mode<1, P>(a, mode, s);
    if (a.rows <= 2) return gemv_mode<2, P>(a, mode, s);
    if (a.rows <= 4) return gemv_mode<4, P>(a, mode, s);
    if (a.rows <= 8) return gemv_mode<8, P>(a, mode, s);
    return gemv_mode<16, P>(a, mode, s);
}

cudaError_t launch_gemv(const GemvArgs& a, int mode, cudaStream_t s) {
    if (a.lin.K % 128 || a.lin.K > 8192 || a.rows < 1) return cudaErrorInvalidValue;
    if (a.split_out) *a.split_out = 0;
    // dense contraction on the tensor cores, when the caller chose that path
    if (a.tensor && a.rows >= TC_MIN_ROWS && gemm_tc_supported(a)) return launch_gemm_tc(a, GemvMode(mode), s);
    // many rows of raw weights: the tiled GEMM (same sums, weights read once per 32 rows)
    if (gemm_supported(a)) return launch_gemm(a, GemvMode(mode), s);
    // Rows beyond what the staged activations allow (16, fewer for very long K) run in passes;
    // the weights are re-read once per pass.
    const size_t row_bytes = size_t(((a.lin.K >> 3) + 63) & ~63) * 16;
    int pass = 16;
    while (pass > 1 && size_t(pass) * row_bytes > GEMV_SMEM_MAX) pass >>= 1;
    for (int r0 = 0; r0 < a.rows; r0 += pass) {
        GemvArgs b = a;
        b.rows = a.rows - r0 < pass ? a.rows - r0 : pass;
        b.x = a.x + size_t(r0) * a.lin.K;
        if (a.out_map) b.out_map = a.out_map + r0;
        else b.y = a.y + size_t(r0) * a.ystride;
        cudaError_t e = a.lin.offsets ? gemv_rows<true>(b, mode, s) : gemv_rows<false>(b, mode, s);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// The opt-in dynamic shared memory limit leaves room for each instantiation's static shared
// memory (the argmax scratch of the logits mode).
template <int R, bool P, int M>
static cudaError_t gemv_attr() {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, k_gemv<R, P, M>);
    if (e != cudaSuccess) return e;
    const size_t dyn = std::min(GEMV_SMEM_MAX, size_t(optin) - fa.sharedSizeBytes);
    return cudaFuncSetAttribute(k_gemv<R, P, M>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(dyn));
}
template <int R, bool P>
static cudaError_t gemv_attr_modes() {
    cudaError_t e = gemv_attr<R, P, GEMV_PLAIN>();
    if (e == cudaSuccess) e = gemv_attr<R, P, GEMV_SWIGLU>();
    if (e == cudaSuccess) e = gemv_attr<R, P, GEMV_LOGITS>();
    return e;
}

cudaError_t configure_kernels() {
    cudaError_t e = cudaSuccess;
#define PLAMO_ATTR(R)                                                    \
    if (e == cudaSuccess) e = gemv_attr_modes<R, false>();               \
    if (e == cudaSuccess) e = gemv_attr_modes<R, true>();
    PLAMO_ATTR(1) PLAMO_ATTR(2) PLAMO_ATTR(4) PLAMO_ATTR(8) PLAMO_ATTR(16)
#undef PLAMO_ATTR
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_attn_partial<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_attn_partial<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_attn_partial<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess) e = configure_gemm();
    if (e == cudaSuccess) e = configure_gemm_tc();
    if (e == cudaSuccess) e = configure_attention_tc();
    if (e == cudaSuccess) e = configure_attention_mma();
    return e;
}

cudaError_t launch_embed_norm(const int* ids, int rows, int vocab, const uint16_t* embed, const uint16_t* w, int d,
                              uint16_t* x, uint16_t* h, unsigned long long* keys, const int* key_map, int nkeys,
                              cudaStream_t s) {
    if (d > 256 * NPT) return cudaErrorInvalidValue;
    return pdl_launch(k_embed_norm, dim3(rows), dim3(256), 0, s, ids, vocab, embed, w, d, x, h, keys, key_map,
                      nkeys);
}

// One CTA of 256 threads per row, at the fewest elements per thread that cover the row.
static cudaError_t launch_norm_rows(const NormArgs& a, int nc, cudaStream_t s) {
    switch (nc) {
        case 1: return pdl_launch(k_norm<1>, dim3(a.rows), dim3(256), 0, s, a);
        case 2: return pdl_launch(k_norm<2>, dim3(a.rows), dim3(256), 0, s, a);
        case 3:
        case 4: return pdl_launch(k_norm<4>, dim3(a.rows), dim3(256), 0, s, a);
        case 5:
        case 6: return pdl_launch(k_norm<6>, dim3(a.rows), dim3(256), 0, s, a);
        case 7:
        case 8: return pdl_launch(k_norm<8>, dim3(a.rows), dim3(256), 0, s, a);
        default: return pdl_launch(k_norm<NPT>, dim3(a.rows), dim3(256), 0, s, a);
    }
}

cudaError_t launch_norm(const NormArgs& a, cudaStream_t s) {
    if (a.n > 256 * NPT || a.src_splits < 0 || (a.src_splits > 0 && !a.src_part)) return cudaErrorInvalidValue;
    return launch_norm_rows(a, (a.n + 255) / 256, s);
}

cudaError_t launch_qkv(const QkvArgs& a, cudaStream_t s) {
    if (a.src_splits < 0 || (a.src_splits > 0 && !a.src_part)) return cudaErrorInvalidValue;
    const int warps = a.rows * (a.H + a.KV);
    return pdl_launch(k_qkv, dim3((warps + 3) / 4), dim3(128), 0, s, a);
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s) {
    if (a.H > 32 || a.H % a.KV) return cudaErrorInvalidValue;
    const size_t smem = attention_smem(a.H, a.KV, a.per_max);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    const dim3 grid(a.splits, a.rows);
    cudaError_t e;
    switch (attn_tile_keys(a.KV)) {
        case 64: e = pdl_launch(k_attn_partial<64>, grid, dim3(256), smem, s, a); break;
        case 32: e = pdl_launch(k_attn_partial<32>, grid, dim3(256), smem, s, a); break;
        default: e = pdl_launch(k_attn_partial<16>, grid, dim3(256), smem, s, a); break;
    }
    if (e != cudaSuccess) return e;
    return launch_attention_merge(a, s);
}

cudaError_t launch_attention_merge(const AttnArgs& a, cudaStream_t s) {
    return pdl_launch(k_attn_merge, dim3(a.rows * ((a.H * (128 / MERGE_DIMS) + 255) / 256)), dim3(256), 0, s, a);
}

cudaError_t launch_finalize(unsigned long long* keys, const int* key_map, int rows, int* result, int* chain_ids,
                            RowDesc* advance, int* hist, int* hist_count, int hist_cap, cudaStream_t s) {
    return pdl_launch(k_finalize, dim3(1), dim3(64 * ((rows + 63) / 64)), 0, s, keys, key_map, rows, result, chain_ids,
                      advance, hist, hist_count, hist_cap);
}

cudaError_t launch_argmax(const uint16_t* logits, int rows, int n, unsigned long long* keys, uint32_t* out,
                          cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(keys, 0, sizeof(unsigned long long) * rows, s);
    if (e != cudaSuccess) return e;
    int blocks = (n + 255) / 256;
    blocks = blocks < 64 ? blocks : 64;
    e = pdl_launch(k_argmax, dim3(blocks, rows), dim3(256), 0, s, logits, n, keys);
    if (e != cudaSuccess) return e;
    return launch_finalize(keys, nullptr, rows, reinterpret_cast<int*>(out), nullptr, nullptr, nullptr, nullptr, 0, s);
}

cudaError_t launch_packed_decode(const uint8_t* data, const uint32_t* entries, long long count, uint16_t* out,
                                 cudaStream_t s) {
    Linear lin;
    lin.w = data; lin.offsets = entries;
    const long long chunks = (count + 15) / 16;
    k_packed_decode<<<unsigned((chunks + 255) / 256), 256, 0, s>>>(lin, count, out);
    return cudaGetLastError();
}

}  // namespace plamo
