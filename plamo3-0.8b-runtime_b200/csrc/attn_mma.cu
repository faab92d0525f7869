// Tensor-mode attention of decode rows (batched steps): split-K attention of one row's 16 query
// heads over its one KV head (MQA), with Q.K^T and P.V as warp-level bf16 MMAs
// (mma.sync m16n8k16, fp32 accumulate). The 16 heads are the MMA's 16 rows; every row of a batched
// step attends over its own lane's cache, so no two rows share an operand and the 64- and 128-row
// tcgen05 tiles do not apply.
//
// Same split partition, partial layout and (max, sum) statistics as k_attn_partial
// (Kernels.metal:277-285 re-rotation, :358-437 local attention, :440-562 global split-K), so
// k_attn_merge finishes both. Keys are staged as the bf16 values k_attn_partial computes (rotated
// keys are bf16-rounded, Kernels.metal:277-285), so every product is exact; the tensor core adds
// the products in its own order. P is passed as a bf16 hi / lo pair (p = hi + lo to 16 bits of
// mantissa, P.V = P_hi.V + P_lo.V), close to the reference's fp32 P. Results within the tensor
// path's tolerance of the order-exact kernel, not bit for bit.
#include "common.cuh"
#include "kernels.h"

namespace plamo {
namespace {

constexpr int MT = 64;             // keys per staged tile
constexpr int KP = 136;            // bf16 row stride of a staged tile: 272 B, consecutive rows 4 banks apart
constexpr int MMA_THREADS = 128;   // four warps
constexpr int MMA_HEADS = 16;      // the MMA's M

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two 8x8 bf16 matrices of row-major [key][dim] storage, transposed into a B fragment (k = key,
// n = dim): lanes 0-7 address keys kb..kb+7, lanes 8-15 keys kb+8..kb+15, each at column n0.
__device__ __forceinline__ void ldsm_x2_trans(uint32_t& r0, uint32_t& r1, const uint16_t* p) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(a));
}

__device__ __forceinline__ uint32_t pack_bf16(uint32_t lo, uint32_t hi) { return (lo & 0xffffu) | (hi << 16); }

// Rows [k0, k0 + tk) of the row's cache window into a [MT][KP] bf16 tile (rows >= tk zero). Local
// layers: keys are stored unrotated and get the window-coordinate RoPE here, with k_attn_partial's
// bf16 rounding.
__device__ __forceinline__ void stage_tile(uint16_t* dst, const uint16_t* base, const RowGeo& g, int k0, int tk,
                                           int cap, const uint32_t* rope, bool rotate) {
    for (int i = threadIdx.x; i < MT * 16; i += MMA_THREADS) {
        const int j = i >> 4, d0 = (i & 15) * 8;
        uint4 out = make_uint4(0u, 0u, 0u, 0u);
        if (j < tk) {
            const uint16_t* row = base + size_t((g.first + k0 + j) % cap) * 128;
            const uint4 w = __ldg(reinterpret_cast<const uint4*>(row + d0));
            if (!rotate) {
                out = w;
            } else {
                const int p0 = d0 < 64 ? d0 + 64 : d0 - 64;
                const uint4 o = __ldg(reinterpret_cast<const uint4*>(row + p0));
                const uint4* cs4 = reinterpret_cast<const uint4*>(rope + size_t(k0 + j) * 64 + (d0 & 63));
                const uint4 c0 = __ldg(cs4), c1 = __ldg(cs4 + 1);
                const uint32_t wv[4] = {w.x, w.y, w.z, w.w}, ov[4] = {o.x, o.y, o.z, o.w};
                const uint32_t cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                uint32_t rb[8];
#pragma unroll
                for (int k = 0; k < 8; k++)
                    rb[k] = f2bf(rope_rotate(bf2f((wv[k >> 1] >> (16 * (k & 1))) & 0xffffu),
                                             bf2f((ov[k >> 1] >> (16 * (k & 1))) & 0xffffu), d0 + k, cs[k]));
                out = make_uint4(pack_bf16(rb[0], rb[1]), pack_bf16(rb[2], rb[3]), pack_bf16(rb[4], rb[5]),
                                 pack_bf16(rb[6], rb[7]));
            }
        }
        *reinterpret_cast<uint4*>(dst + j * KP + d0) = out;
    }
}

__global__ void __launch_bounds__(MMA_THREADS) k_attn_rows_mma(AttnArgs a) {
    pdl_enter();
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint16_t* tile = reinterpret_cast<uint16_t*>(smem_raw);              // [MT][KP] keys, later value tiles
    uint16_t* vfirst = tile + MT * KP;                                   // [MT][KP] the first value tile
    float* sc = reinterpret_cast<float*>(smem_raw + 2 * MT * KP * 2);    // [16][per_max] scores, then P
    const int r = blockIdx.y, s = blockIdx.x, t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int gq = lane >> 2, tq = lane & 3;  // MMA fragment coordinates (group, thread in group)
    const RowGeo g = a.geo[r];
    const int lane_id = a.desc[r].lane;
    int per = (g.count + a.splits - 1) / a.splits;
    per = (per + 31) & ~31;
    const int k0 = s * per, k1 = min(k0 + per, g.count);
    const int lo = max(k0, g.begin), hi = min(k1, g.end);
    float2* ml = a.part_ml + (size_t(r) * a.splits + s) * MMA_HEADS;
    if (lo >= hi) {
        if (t < MMA_HEADS) ml[t] = make_float2(-INFINITY, 0.f);
        return;
    }
    const int n = hi - lo;
    const uint16_t* kbase = a.keys + size_t(lane_id) * a.lane_stride;
    const uint16_t* vbase = a.values + size_t(lane_id) * a.lane_stride;
    // the first value tile does not depend on the scores: it streams in (cp.async) while they run
    {
        const int tk0 = min(MT, n);
        for (int i = t; i < MT * 16; i += MMA_THREADS) {
            const int j = i >> 4, d0 = (i & 15) * 8;
            uint16_t* dst = vfirst + j * KP + d0;
            if (j < tk0) {
                const uint16_t* src = vbase + size_t((g.first + lo + j) % a.cap) * 128 + d0;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                             ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))), "l"(src)
                             : "memory");
            } else {
                *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    // Q fragments of all eight 16-dim k-steps (rows = heads gq and gq + 8)
    const uint32_t* q32 = reinterpret_cast<const uint32_t*>(a.q + size_t(r) * MMA_HEADS * 128);
    uint32_t qa[8][4];
#pragma unroll
    for (int kk = 0; kk < 8; kk++) {
        qa[kk][0] = __ldg(q32 + (gq * 128 + kk * 16 + 2 * tq) / 2);
        qa[kk][1] = __ldg(q32 + ((gq + 8) * 128 + kk * 16 + 2 * tq) / 2);
        qa[kk][2] = __ldg(q32 + (gq * 128 + kk * 16 + 2 * tq + 8) / 2);
        qa[kk][3] = __ldg(q32 + ((gq + 8) * 128 + kk * 16 + 2 * tq + 8) / 2);
    }
    // pass 1: scaled scores; warp w takes keys [16w, 16w + 16) of each tile
    for (int t0 = 0; t0 < n; t0 += MT) {
        const int tk = min(MT, n - t0);
        __syncthreads();
        stage_tile(tile, kbase, g, lo + t0, tk, a.cap, a.rope_local, !a.full);
        __syncthreads();
#pragma unroll
        for (int nt = 0; nt < 2; nt++) {
            const int nb = warp * 16 + nt * 8;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            const uint32_t* krow = reinterpret_cast<const uint32_t*>(tile + (nb + gq) * KP);
#pragma unroll
            for (int kk = 0; kk < 8; kk++) mma_bf16_16816(acc, qa[kk], krow[kk * 8 + tq], krow[kk * 8 + 4 + tq]);
            const int key = nb + 2 * tq;
#pragma unroll
            for (int u = 0; u < 2; u++) {
                if (key + u < tk) {
                    sc[gq * a.per_max + t0 + key + u] = acc[u] * PLAMO_ATTN_SCALE;
                    sc[(gq + 8) * a.per_max + t0 + key + u] = acc[2 + u] * PLAMO_ATTN_SCALE;
                }
            }
        }
    }
    __syncthreads();
    // pass 2: split-local softmax statistics per head (k_attn_partial's pass 2)
    for (int h = warp; h < MMA_HEADS; h += MMA_THREADS / 32) {
        float* p = sc + h * a.per_max;
        float m = -INFINITY;
        for (int i = lane; i < n; i += 32) m = fmaxf(m, p[i]);
        m = warp_max(m);
        float l = 0.f;
        for (int i = lane; i < n; i += 32) { const float e = pexp(p[i] - m); p[i] = e; l += e; }
        l = warp_sum(l);
        if (lane == 0) ml[h] = make_float2(m, l);
    }
    // pass 3: unnormalised P.V; warp w takes dims [32w, 32w + 32)
    float o[4][4];
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
        for (int u = 0; u < 4; u++) o[j][u] = 0.f;
    for (int t0 = 0; t0 < n; t0 += MT) {
        const int tk = min(MT, n - t0);
        __syncthreads();  // the score pass / previous tile is done with `tile`; P is complete
        if (t0 == 0) asm volatile("cp.async.wait_all;" ::: "memory");
        else stage_tile(tile, vbase, g, lo + t0, tk, a.cap, nullptr, false);
        __syncthreads();
        const uint16_t* vt = t0 == 0 ? vfirst : tile;
#pragma unroll
        for (int kb = 0; kb < MT; kb += 16) {
            if (kb >= tk) break;
            // P fragment (rows = heads, k = keys kb..kb+15 of the tile) as a bf16 hi / lo pair
            uint32_t ph[4], pl[4];
#pragma unroll
            for (int f = 0; f < 4; f++) {
                const int h = gq + (f & 1) * 8, key = kb + 2 * tq + (f >> 1) * 8;
                float p0 = 0.f, p1 = 0.f;
                if (key < tk) p0 = sc[h * a.per_max + t0 + key];
                if (key + 1 < tk) p1 = sc[h * a.per_max + t0 + key + 1];
                const uint32_t h0 = f2bf(p0), h1 = f2bf(p1);
                ph[f] = pack_bf16(h0, h1);
                pl[f] = pack_bf16(f2bf(p0 - bf2f(h0)), f2bf(p1 - bf2f(h1)));
            }
#pragma unroll
            for (int j = 0; j < 4; j++) {
                uint32_t b0, b1;
                ldsm_x2_trans(b0, b1, vt + (kb + (lane & 15)) * KP + warp * 32 + j * 8);
                mma_bf16_16816(o[j], ph, b0, b1);
                mma_bf16_16816(o[j], pl, b0, b1);
            }
        }
    }
    float* po = a.part_o + (size_t(r) * a.splits + s) * MMA_HEADS * 128;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int d = warp * 32 + j * 8 + 2 * tq;
        *reinterpret_cast<float2*>(po + gq * 128 + d) = make_float2(o[j][0], o[j][1]);
        *reinterpret_cast<float2*>(po + (gq + 8) * 128 + d) = make_float2(o[j][2], o[j][3]);
    }
}

size_t attention_mma_smem(int per_max) { return size_t(2) * MT * KP * 2 + size_t(MMA_HEADS) * per_max * sizeof(float); }

}  // namespace

bool attention_mma_supported(const AttnArgs& a) {
    return a.H == MMA_HEADS && a.KV == 1 && a.per_max >= 32 && attention_mma_smem(a.per_max) <= 200 * 1024 &&
           (reinterpret_cast<uintptr_t>(a.q) & 3) == 0 && (reinterpret_cast<uintptr_t>(a.keys) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(a.values) & 15) == 0 && a.lane_stride % 8 == 0 && a.part_o && a.part_ml;
}

cudaError_t configure_attention_mma() {
    return cudaFuncSetAttribute(k_attn_rows_mma, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

cudaError_t launch_attention_mma(const AttnArgs& a, cudaStream_t s) {
    if (!attention_mma_supported(a)) return cudaErrorInvalidValue;
    const size_t smem = attention_mma_smem(a.per_max);
    cudaError_t e = pdl_launch(k_attn_rows_mma, dim3(a.splits, a.rows), dim3(MMA_THREADS), smem, s, a);
    if (e != cudaSuccess) return e;
    return launch_attention_merge(a, s);
}

}  // namespace plamo
