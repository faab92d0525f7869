// Persistent batch-1 decode step for sm_100a: one cooperative launch per token, one CTA per SM.
//
// The step is a list of phases (per layer: QKV, attention, o_proj, gate/up + SwiGLU, down_proj;
// then the head):
//   QKV  (prologue: residual + post-MLP norm of the previous layer, pre-mixer norm)  Runtime.swift:377,450
//   ATT  (QK-norm + RoPE + KV append fused, split-K attention, per-head merge)         Kernels.metal:223-562
//   O    (o_proj)                                                                      Runtime.swift:445
//   GU   (prologue: residual + post-mixer norm, pre-MLP norm; SwiGLU epilogue)         Runtime.swift:446-448
//   DOWN (down_proj)                                                                   Runtime.swift:449
//   HEAD (residual + post-MLP norm, final norm, lm_head, first-index argmax)           Runtime.swift:450-458
//
// Weights. Every CTA owns a contiguous share of the outputs of every projection. Its 8 warps read
// their weight rows straight from HBM with 16-byte non-allocating loads, up to four (row, 1536-
// weight segment) tasks per warp at a time (24 loads of 16 bytes in flight per lane). The loads
// of a warp's next tasks are issued before the current ones are summed, and across phase
// boundaries: a warp's first tasks of the next projection are in flight while it waits for that
// projection's input (and, for o_proj, during the whole attention phase).
//
// Phase boundaries. Phase outputs are exchanged through tagged words (mega.h): a producer stores
// each value with the (step, layer) tag, a consumer polls exactly the words it needs. There is
// no grid-wide barrier, counter or fence between phases. Every poll is bounded in time and
// raises the error flag (read by the host after the step) instead of hanging.
//
// Attention. A task is (split of the key window, group of 4 query heads); tasks are spread over
// the CTAs, each stages its key and value tiles with TMA bulk copies issued before its queries
// are ready. The merge of head h runs on CTA G - 1 - h as soon as the head's split partials land.
//
// Arithmetic. Every output follows the same per-element operation order as kernels.cu (and the
// CPU restatement): 16-weight lane chunks in 1536-weight segments, two fma chains per segment,
// segment sums folded in order, the 32-lane butterfly; the 256-thread norm tree; one fma chain
// per score and per P.V output; split order in the merge. So this path is bit-identical to the
// multi-kernel path.
#include "common.cuh"
#include "mega.h"

#include <algorithm>

namespace plamo {

// ---- PTX helpers -----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t gtime() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// 1-D bulk copy global -> this CTA's shared memory (no multicast), completion on `bar`
__device__ __forceinline__ void tma_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// 16-byte asynchronous copy global -> shared (L2 only), completed by cp_async_wait_all
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_but_newest() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// orders this thread's earlier generic-proxy accesses before its next bulk copies (async proxy)
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async;" ::: "memory"); }

// Weights: read once per step, never written: non-coherent path, no L1 allocation, and marked
// first to evict from L2, so the 1.45 GB stream does not flush the small tensors every step
// re-reads (norm weights, RoPE rows, KV cache, exchange words).
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ uint4 ldw4(const void* p, uint64_t pol) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ uint2 ldw2(const void* p, uint64_t pol) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0,%1}, [%2], %3;" : "=r"(v.x), "=r"(v.y) : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ uint32_t ldw1(const uint32_t* p, uint64_t pol) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(v) : "l"(p), "l"(pol));
    return v;
}
// tagged exchange words: morally strong (relaxed, gpu scope) so a poll always sees the latest store
__device__ __forceinline__ uint32_t ld_tag(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_tag64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_tag(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void st_tag64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint32_t tagged(uint32_t tag, uint32_t bf) { return (tag << 16) | bf; }
__device__ __forceinline__ unsigned long long tagged64(uint32_t tag, float v) {
    return (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
}

constexpr uint64_t WAIT_NS = 2000000000ull;  // every wait gives up after 2 s
enum MegaError { ERR_DATA = 12, ERR_TILE = 13, ERR_DRAIN = 14 };

// Bounded polling. After a miss the clock starts; the error flag (one global word) and the clock
// are checked every 16 polls, with a short sleep between polls to keep the L2 free for producers.
struct Spin {
    uint64_t t0 = 0;
    uint32_t i = 0;
};
__device__ __forceinline__ bool spin_more(Spin& s, int* error, int code, uint64_t limit_ns = WAIT_NS) {
    if (s.i++ == 0) s.t0 = gtime();
    if ((s.i & 15u) == 0) {
        if (*reinterpret_cast<volatile int*>(error)) return false;
        if (gtime() - s.t0 > limit_ns) {
            atomicCAS(error, 0, code);
            return false;
        }
    }
    __nanosleep(20);
    return true;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* error) {
    if (mbar_test(bar, parity)) return true;
    Spin s;
    while (!mbar_test(bar, parity))
        if (!spin_more(s, error, ERR_TILE)) return false;
    return true;
}
// Waits for copies already issued into this CTA's shared memory before it exits; bounded in
// time only (a copy from valid global memory always completes).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity, int* error) {
    const uint64_t t0 = gtime();
    while (!mbar_test(bar, parity)) {
        if (gtime() - t0 > WAIT_NS) {
            atomicCAS(error, 0, ERR_DRAIN);
            return;
        }
    }
}

// Warp 0 polls the n hint words h[i * stride] until all carry `tag` (a few requests per round,
// spaced out); then the whole CTA passes a barrier. Called by every thread of the CTA.
__device__ __forceinline__ bool wait_hints(const uint32_t* h, int n, int stride, uint32_t tag, int* error) {
    bool ok = true;
    if (threadIdx.x < 32) {
        Spin s;
        for (;;) {
            // every word of the round in flight at once, then the check
            uint32_t v[8];
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const int i = threadIdx.x + 32 * k;
                v[k] = i < n ? ld_tag(h + size_t(i) * stride) : tag;
            }
            bool mine = true;
            for (int i = threadIdx.x + 256; i < n; i += 32) mine = mine && ld_tag(h + size_t(i) * stride) == tag;
#pragma unroll
            for (int k = 0; k < 8; k++) mine = mine && v[k] == tag;
            if (__all_sync(FULL_MASK, mine)) break;
            const bool more = __all_sync(FULL_MASK, spin_more(s, error, ERR_DATA));
            if (!more) {
                ok = false;
                break;
            }
            __nanosleep(64);
        }
    }
    return __syncthreads_and(ok);
}

// ---- norms (256 threads; the tree of k_norm) --------------------------------------------------
// Sum over the 256 threads in k_norm's tree: the butterfly within each warp, then the 8 warp sums
// as lanes 0..7 of one butterfly (lanes 8..31 zero). After the single barrier every warp folds the
// 8 sums itself. `red` alternates between two 8-float halves from call to call: a call's writes
// can only meet the reads of the call before the previous one, which every warp finished before
// passing the previous call's barrier.
__device__ __forceinline__ float cblock_sum(float v, float* red, int& parity) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* r = red + 8 * parity;
    parity ^= 1;
    if (lane == 0) r[warp] = v;
    __syncthreads();
    return warp_sum(lane < 8 ? r[lane] : 0.f);
}

// Norm factors rbf(w + offset) of the elements t + 256 j this thread owns.
template <int NPT>
__device__ __forceinline__ void load_norm(const uint16_t* w, float offset, int n, float (&wf)[NPT]) {
#pragma unroll
    for (int j = 0; j < NPT; j++) {
        const int i = threadIdx.x + j * 256;
        wf[j] = i < n ? rbf(bf2f(w[i]) + offset) : 0.f;
    }
}

// RMSNorm over n elements held NPT per thread (thread t: t + 256 j). The sum of squares is the
// 256-thread tree of k_norm; elements past n are zero and leave every partial sum unchanged.
template <int NPT>
__device__ __forceinline__ void cnorm(const float (&v)[NPT], int n, const float (&wf)[NPT], float* red, int& parity,
                                      float (&z)[NPT]) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NPT; j++) ss = fmaf(v[j], v[j], ss);
    const float total = cblock_sum(ss, red, parity);
    const float scale = 1.0f / sqrtf(total / float(n) + PLAMO_EPS);
#pragma unroll
    for (int j = 0; j < NPT; j++) {
        const int i = threadIdx.x + j * 256;
        z[j] = i < n ? rbf(rbf(v[j] * scale) * wf[j]) : 0.f;
    }
}

// bf16 activation element i -> permuted shared layout read by the dot products: lane l's 16
// elements of group g sit at 16-byte chunks g*64 + l and g*64 + 32 + l (conflict-free reads).
__device__ __forceinline__ int xs_index(int i) {
    const int c = i >> 3, g = c >> 6, within = c & 63;
    return ((g * 64 + (within & 1) * 32 + (within >> 1)) << 3) + (i & 7);
}

// Gathers n tagged bf16 words: dst[i] (or dst[xs_index(i)] with PERMUTE) = the payload of src[i]
// once it carries `tag`. All threads: up to 24 loads in flight per thread, then one compact re-poll loop
// over the words not yet visible. The caller passes a barrier before reading dst.
template <bool PERMUTE>
__device__ __forceinline__ bool gather16(uint16_t* dst, const uint32_t* src, int n, uint32_t tag, int* error) {
    const int t = threadIdx.x;
    for (int base = 0; base < n; base += 24 * 256) {
        uint32_t v[24];
#pragma unroll
        for (int j = 0; j < 24; j++) {
            const int i = base + t + j * 256;
            v[j] = i < n ? ld_tag(src + i) : 0u;
        }
        unsigned miss = 0;
#pragma unroll
        for (int j = 0; j < 24; j++) {
            const int i = base + t + j * 256;
            if (i < n) {
                if ((v[j] >> 16) == tag) dst[PERMUTE ? xs_index(i) : i] = uint16_t(v[j] & 0xffffu);
                else miss |= 1u << j;
            }
        }
        Spin s;
        while (miss) {
            const int i = base + t + (__ffs(miss) - 1) * 256;
            const uint32_t w = ld_tag(src + i);
            if ((w >> 16) == tag) {
                dst[PERMUTE ? xs_index(i) : i] = uint16_t(w & 0xffffu);
                miss &= miss - 1;
            } else if (!spin_more(s, error, ERR_DATA)) {
                return false;
            }
        }
    }
    return true;
}

// The same for tagged f32 words laid out in rows: element i is src[(i >> rshift) * rstride +
// (i & (2^rshift - 1))]; dst[i] receives its value.
__device__ __forceinline__ bool gather64(float* dst, const unsigned long long* src, int n, int rshift, size_t rstride,
                                         uint32_t tag, int* error) {
    const int t = threadIdx.x;
    const int rmask = (1 << rshift) - 1;
    for (int base = 0; base < n; base += 8 * 256) {
        unsigned long long v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int i = base + t + j * 256;
            v[j] = i < n ? ld_tag64(src + size_t(i >> rshift) * rstride + (i & rmask)) : 0ull;
        }
        unsigned miss = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int i = base + t + j * 256;
            if (i < n) {
                if (uint32_t(v[j] >> 32) == tag) dst[i] = __uint_as_float(uint32_t(v[j]));
                else miss |= 1u << j;
            }
        }
        Spin s;
        while (miss) {
            const int i = base + t + (__ffs(miss) - 1) * 256;
            const unsigned long long w = ld_tag64(src + size_t(i >> rshift) * rstride + (i & rmask));
            if (uint32_t(w >> 32) == tag) {
                dst[i] = __uint_as_float(uint32_t(w));
                miss &= miss - 1;
            } else if (!spin_more(s, error, ERR_DATA)) {
                return false;
            }
        }
    }
    return true;
}

// Two tagged-f32 gathers with every load of both in flight before the first check: (dst1, src1,
// n1) and (dst2, src2, n2), laid out as in gather64. n1 <= 512 and n2 <= 8 * 256.
__device__ __forceinline__ bool gather64x2(float* dst1, const unsigned long long* src1, int n1, int rs1, size_t rstride1,
                                           float* dst2, const unsigned long long* src2, int n2, int rs2, size_t rstride2,
                                           uint32_t tag, int* error) {
    const int t = threadIdx.x;
    const int m1 = (1 << rs1) - 1, m2 = (1 << rs2) - 1;
    unsigned long long v1[2], v2[8];
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const int i = t + j * 256;
        v1[j] = i < n1 ? ld_tag64(src1 + size_t(i >> rs1) * rstride1 + (i & m1)) : 0ull;
    }
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int i = t + j * 256;
        v2[j] = i < n2 ? ld_tag64(src2 + size_t(i >> rs2) * rstride2 + (i & m2)) : 0ull;
    }
    unsigned miss = 0;
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const int i = t + j * 256;
        if (i < n1) {
            if (uint32_t(v1[j] >> 32) == tag) dst1[i] = __uint_as_float(uint32_t(v1[j]));
            else miss |= 1u << j;
        }
    }
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int i = t + j * 256;
        if (i < n2) {
            if (uint32_t(v2[j] >> 32) == tag) dst2[i] = __uint_as_float(uint32_t(v2[j]));
            else miss |= 1u << (8 + j);
        }
    }
    Spin s;
    while (miss) {
        const int k = __ffs(miss) - 1, second = k >= 8, i = t + (k & 7) * 256;
        const unsigned long long* p = second ? src2 + size_t(i >> rs2) * rstride2 + (i & m2)
                                             : src1 + size_t(i >> rs1) * rstride1 + (i & m1);
        const unsigned long long w = ld_tag64(p);
        if (uint32_t(w >> 32) == tag) {
            (second ? dst2 : dst1)[i] = __uint_as_float(uint32_t(w));
            miss &= miss - 1;
        } else if (!spin_more(s, error, ERR_DATA)) {
            return false;
        }
    }
    return true;
}

// ---- weight phases ---------------------------------------------------------------------------
// A task is (output row, 1536-weight segment of the row): lane l covers weights
// [g*512 + 16l, +16) of the segment's groups g (at most 3). A warp carries up to RB tasks at a time.
constexpr int RB = 3;
constexpr int GB = 3;
constexpr uint64_t MEGA_STAGGER_NS = 400;  // start offset between warp pairs in multi-round phases

struct Batch {
    uint4 w[RB][GB][2];       // raw: 32 weight bytes; .p12 packed block: sign|mantissa bytes, codes
    uint32_t ent[RB][GB];     // .p12 block-table entries (offset | tag)
};

// This CTA's share of one weight phase.
struct PhaseWork {
    int kind, K, G, nseg, R;  // row length, 512-weight groups, segments per row, tasks per chunk
    const uint8_t* w;
    const uint32_t* off;
    int u0, nu;               // this CTA's outputs [u0, u0 + nu)
    int ntask, nchunk;
    int up;                   // SwiGLU: row offset of the up half
    int upc;                  // SwiGLU: outputs per gate/up chunk pair
};

__device__ __forceinline__ PhaseWork phase_work(const MegaPhase& ph, int cta, int G) {
    PhaseWork p;
    p.kind = ph.kind;
    p.K = ph.lin.K;
    p.G = (p.K + 511) >> 9;
    p.nseg = (p.G + 2) / 3;
    p.w = ph.lin.w;
    p.off = ph.lin.offsets;
    const int units = ph.out_rows;
    p.u0 = int((long long)units * cta / G);
    p.nu = int((long long)units * (cta + 1) / G) - p.u0;
    p.up = ph.kind == MK_GU ? ph.out_rows : 0;
    if (ph.kind == MK_GU) {
        // chunk pairs: the gate rows of RB outputs, then their up rows (same warp, in a row)
        p.ntask = 2 * p.nu;
        p.upc = RB;
        p.R = RB;
        p.nchunk = 2 * ((p.nu + RB - 1) / RB);
    } else {
        p.ntask = p.nu * p.nseg;
        p.upc = 0;
        p.R = min(RB, max(1, (p.ntask + 7) / 8));
        p.nchunk = (p.ntask + p.R - 1) / p.R;
    }
    return p;
}

// A warp's chunks: c = warp, warp + 8, ...; SwiGLU phases walk chunk pairs (2j, 2j + 1) for
// j = warp, warp + 8, ..., so a warp sums the gate rows and then the up rows of the same outputs.
__device__ __forceinline__ int first_chunk(const PhaseWork& p, int warp) { return p.kind == MK_GU ? 2 * warp : warp; }
__device__ __forceinline__ int next_chunk(const PhaseWork& p, int c) {
    return p.kind == MK_GU ? ((c & 1) ? c + 15 : c + 1) : c + 8;
}

// Row and segment of task r of chunk c; false when the slot is empty.
__device__ __forceinline__ bool task_of(const PhaseWork& p, int c, int r, int& row, int& seg) {
    if (r >= p.R) return false;
    if (p.kind == MK_GU) {  // chunk 2j: gate rows of outputs [upc j, upc j + upc), chunk 2j + 1: their up rows
        const int u = (c >> 1) * p.upc + r;
        if (u >= p.nu) return false;
        row = p.u0 + u + (c & 1) * p.up;
        seg = 0;
        return true;
    }
    const int i = c * p.R + r;
    if (i >= p.ntask) return false;
    row = p.u0 + i / p.nseg;
    seg = i % p.nseg;
    return true;
}

// Issues the weight loads of chunk c (this warp). .p12: the block-table entries first, then the
// blocks they point at.
template <bool PACKED>
__device__ __forceinline__ void issue_chunk(const PhaseWork& p, int c, Batch& b, uint64_t pol, const uint32_t* tbl) {
    const int lane = threadIdx.x & 31;
    const uint8_t* rp[RB];
    bool ok[RB];
    int sg[RB];
#pragma unroll
    for (int r = 0; r < RB; r++) {
        int row = 0, seg = 0;
        ok[r] = task_of(p, c, r, row, seg);
        sg[r] = seg;
        if (PACKED) {  // the row's block-table entries in this CTA's shared copy (gate rows, then up rows)
            const int half = p.up && row >= p.up;
            rp[r] = reinterpret_cast<const uint8_t*>(tbl + size_t(row - half * p.up - p.u0 + half * p.nu) * (p.K >> 7));
        } else {
            rp[r] = p.w + size_t(row) * p.K * 2;
        }
    }
#pragma unroll
    for (int r = 0; r < RB; r++)
#pragma unroll
        for (int gi = 0; gi < GB; gi++) {
            const int e0 = (3 * sg[r] + gi) * 512 + lane * 16;
            if (ok[r] && e0 < p.K && (3 * sg[r] + gi) < p.G) {
                if (!PACKED) {
                    b.w[r][gi][0] = ldw4(rp[r] + e0 * 2, pol);
                    b.w[r][gi][1] = ldw4(rp[r] + e0 * 2 + 16, pol);
                } else {
                    b.ent[r][gi] = reinterpret_cast<const uint32_t*>(rp[r])[e0 >> 7];
                }
            }
        }
    if (PACKED) {
#pragma unroll
        for (int r = 0; r < RB; r++)
#pragma unroll
            for (int gi = 0; gi < GB; gi++) {
                const int e0 = (3 * sg[r] + gi) * 512 + lane * 16;
                if (ok[r] && e0 < p.K && (3 * sg[r] + gi) < p.G) {
                    const uint32_t entry = b.ent[r][gi], i0 = uint32_t(e0 & 127);
                    const uint8_t* blk = p.w + (entry & ~63u);
                    if (entry & 63u) {
                        b.w[r][gi][0] = ldw4(blk + i0, pol);
                        const uint2 cd = ldw2(blk + 128 + (i0 >> 1), pol);
                        b.w[r][gi][1] = make_uint4(cd.x, cd.y, 0u, 0u);
                    } else {
                        b.w[r][gi][0] = ldw4(blk + 2 * i0, pol);
                        b.w[r][gi][1] = ldw4(blk + 2 * i0 + 16, pol);
                    }
                }
            }
    }
}

// Both halves of a bf16 pair times the matching halves of x, accumulated into the even (lo) and
// odd (hi) chains with sm_100's mixed-precision fma (bf16 x bf16 + f32, one rounding): the same
// result as fmaf on the widened operands (the product of two bf16 values is exact in f32), in
// one instruction per weight.
__device__ __forceinline__ void fma_bf16x2(uint32_t w, uint32_t x, float& lo, float& hi) {
    asm("{\n .reg .b16 wl, wh, xl, xh;\n mov.b32 {wl, wh}, %2;\n mov.b32 {xl, xh}, %3;\n"
        " fma.rn.f32.bf16 %0, wl, xl, %0;\n fma.rn.f32.bf16 %1, wh, xh, %1;\n}"
        : "+f"(lo), "+f"(hi)
        : "r"(w), "r"(x));
}

// The 16 weights of (task r, group gi) as bf16 pairs.
template <bool PACKED>
__device__ __forceinline__ void weights16(const Batch& b, int r, int gi, uint32_t (&wp)[8]) {
    const uint4 A = b.w[r][gi][0], B = b.w[r][gi][1];
    if (PACKED && (b.ent[r][gi] & 63u)) {
        decode16(A, make_uint2(B.x, B.y), (b.ent[r][gi] & 63u) + 107u, wp);
    } else {
        wp[0] = A.x; wp[1] = A.y; wp[2] = A.z; wp[3] = A.w;
        wp[4] = B.x; wp[5] = B.y; wp[6] = B.z; wp[7] = B.w;
    }
}

// Lane partials of the chunk's tasks: per task the segment's two fma chains (even / odd
// elements, groups in order), returned as a0 + a1.
template <bool PACKED>
__device__ __forceinline__ void chunk_partials(const PhaseWork& p, int c, const Batch& b, const uint4* xs4, float (&res)[RB]) {
    const int lane = threadIdx.x & 31;
    float a0[RB], a1[RB];
    bool ok[RB];
    int sg[RB];
#pragma unroll
    for (int r = 0; r < RB; r++) {
        int row = 0, seg = 0;
        ok[r] = task_of(p, c, r, row, seg);
        sg[r] = seg;
        a0[r] = 0.f;
        a1[r] = 0.f;
    }
    if (p.nseg == 1) {
        // every task is its row's only segment: one read of each activation group serves all tasks
#pragma unroll
        for (int gi = 0; gi < GB; gi++) {
            if (gi < p.G) {
                uint32_t xp[8];
                const uint4 xa = xs4[gi * 64 + lane], xb = xs4[gi * 64 + 32 + lane];
                xp[0] = xa.x; xp[1] = xa.y; xp[2] = xa.z; xp[3] = xa.w;
                xp[4] = xb.x; xp[5] = xb.y; xp[6] = xb.z; xp[7] = xb.w;
                const bool lane_in = gi * 512 + lane * 16 < p.K;
#pragma unroll
                for (int r = 0; r < RB; r++) {
                    if (ok[r] && lane_in) {
                        uint32_t wp[8];
                        weights16<PACKED>(b, r, gi, wp);
#pragma unroll
                        for (int k = 0; k < 8; k++) fma_bf16x2(wp[k], xp[k], a0[r], a1[r]);
                    }
                }
            }
        }
    } else {
#pragma unroll
        for (int gi = 0; gi < GB; gi++) {
#pragma unroll
            for (int r = 0; r < RB; r++) {
                const int g = 3 * sg[r] + gi, e0 = g * 512 + lane * 16;
                if (ok[r] && g < p.G && e0 < p.K) {
                    uint32_t xp[8];
                    const uint4 xa = xs4[g * 64 + lane], xb = xs4[g * 64 + 32 + lane];
                    xp[0] = xa.x; xp[1] = xa.y; xp[2] = xa.z; xp[3] = xa.w;
                    xp[4] = xb.x; xp[5] = xb.y; xp[6] = xb.z; xp[7] = xb.w;
                    uint32_t wp[8];
                    weights16<PACKED>(b, r, gi, wp);
#pragma unroll
                    for (int k = 0; k < 8; k++) fma_bf16x2(wp[k], xp[k], a0[r], a1[r]);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < RB; r++) res[r] = a0[r] + a1[r];
}

// ---- attention ---------------------------------------------------------------------------------
// Shared-memory regions of an attention task (inside the work region, 16-byte aligned):
//   qs   [HG][QSM] f32         normed + rotated queries of the task's heads
//   kraw [ATM][128] bf16       key tile as stored in the cache (TMA)
//   vraw [ATM][128] bf16       value tile (TMA)
//   rope [ATM][64] u32         RoPE rows of the key tile's window coordinates (local layers, TMA)
//   kr   [ATM][136] bf16       rotated keys, rows padded so 16-byte loads of 8 rows hit distinct banks
//   sc   [HG][per_max] f32     scores, then exp(score - m)
//   aux  knew, vnew [128] bf16 this step's key (cache format) and value; qkvs [768] bf16 the
//        task's query rows, then this step's key and value rows as produced
// The merge of a head reuses kraw for 16 split partials and kr for the split statistics.
constexpr int QSM = 132;
constexpr int KRS = 136;
constexpr int MERGE_CHUNK = 16;  // split partial rows per merge pass: 16 x 128 = 8 loads per thread
struct AttnSizes {
    size_t qs, kraw, vraw, rope, kr, sc, aux, total;
};
__host__ __device__ inline AttnSizes attn_sizes(int per_max) {
    AttnSizes z;
    z.qs = size_t(MEGA_HG) * QSM * 4;
    z.kraw = size_t(MEGA_ATM) * 256;
    z.vraw = size_t(MEGA_ATM) * 256;
    z.rope = size_t(MEGA_ATM) * 256;
    z.kr = size_t(MEGA_ATM) * KRS * 2;
    z.sc = ((size_t(MEGA_HG) * per_max * 4) + 15) & ~size_t(15);
    z.aux = 2048;
    z.total = z.qs + z.kraw + z.vraw + z.rope + z.kr + z.sc + z.aux;
    return z;
}

struct AttnSmem {
    float* qs;
    uint16_t *kraw, *vraw;
    uint32_t* rope;
    uint16_t* kr;
    float* sc;
    uint16_t *knew, *vnew, *qkvs;
};

__device__ __forceinline__ AttnSmem attn_smem(uint8_t* base, int per_max) {
    const AttnSizes z = attn_sizes(per_max);
    AttnSmem m;
    uint8_t* q = base;
    m.qs = reinterpret_cast<float*>(q); q += z.qs;
    m.kraw = reinterpret_cast<uint16_t*>(q); q += z.kraw;
    m.vraw = reinterpret_cast<uint16_t*>(q); q += z.vraw;
    m.rope = reinterpret_cast<uint32_t*>(q); q += z.rope;
    m.kr = reinterpret_cast<uint16_t*>(q); q += z.kr;
    m.sc = reinterpret_cast<float*>(q); q += z.sc;
    m.knew = reinterpret_cast<uint16_t*>(q);
    m.vnew = m.knew + 128;
    m.qkvs = m.knew + 256;
    return m;
}

// The attention copies complete on two mbarriers (key tile + RoPE rows, value tile). Thread
// ISSUER issues every copy; all threads wait on the barrier, so they all track the same parities.
enum { AB_K = 0, AB_V = 1 };
constexpr int ISSUER = 192;  // warp 6: warp 0 polls the hints meanwhile
struct AttnBars {
    uint64_t* bar;     // [2]
    uint32_t parity;   // bit i: parity of barrier i's next completion
    uint32_t pending;  // bit i: copies issued on barrier i and not yet waited for
};
__device__ __forceinline__ bool ab_wait(AttnBars& b, int i, int* error) {
    const bool ok = mbar_wait(&b.bar[i], (b.parity >> i) & 1u, error);
    if (ok) b.pending &= ~(1u << i);
    b.parity ^= 1u << i;
    return ok;
}

// Window geometry of split s for the step's single row (Runtime.swift:389-395, Kernels.metal:440-470).
struct SplitGeo {
    int first, count, qcoord, pos, lo, hi;
};
__device__ __forceinline__ SplitGeo split_geo(const MegaArgs& a, const MegaLayer& Ly, const RowDesc& dsc, int s) {
    SplitGeo g;
    g.pos = dsc.pos;
    int end, begin;
    if (Ly.full) {
        g.first = 0; g.count = dsc.cstart + dsc.crows; end = dsc.pos + 1; begin = 0; g.qcoord = dsc.pos;
    } else {
        g.first = max(0, dsc.cstart - (a.W - 1));
        g.count = dsc.cstart + dsc.crows - g.first;
        end = dsc.pos - g.first + 1;
        begin = max(0, end - a.W);
        g.qcoord = dsc.pos - g.first;
    }
    int per = (g.count + Ly.splits - 1) / Ly.splits;
    per = (per + 31) & ~31;
    const int k0 = s * per, k1 = min(k0 + per, g.count);
    g.lo = max(k0, begin);
    g.hi = min(k1, end);
    return g;
}
// Splits holding keys form a prefix of the split list (decode rows see their whole window).
__device__ __forceinline__ int active_splits(const MegaArgs& a, const MegaLayer& Ly, const RowDesc& dsc) {
    int n = 0;
    for (int s = 0; s < Ly.splits; s++) {
        const SplitGeo g = split_geo(a, Ly, dsc, s);
        if (g.lo < g.hi) n = s + 1;
    }
    return n;
}

// ISSUER only: rows [t0, t0 + tk) of the split's cache window (a ring buffer: at most two
// contiguous row ranges) and, for local layers, the RoPE rows of their window coordinates.
__device__ __forceinline__ void issue_rows(const MegaArgs& a, void* dst, const uint16_t* cache, const SplitGeo& g, int t0,
                                           int tk, int cap, uint32_t* rope_dst, uint64_t* bar) {
    const uint32_t rb = rope_dst ? uint32_t(tk) * 256u : 0u;
    fence_proxy_async();
    mbar_expect_tx(bar, uint32_t(tk) * 256u + rb);
    const int start = (g.first + g.lo + t0) % cap, n1 = min(tk, cap - start);
    const uint8_t* base = reinterpret_cast<const uint8_t*>(cache);
    tma_load(dst, base + size_t(start) * 256, uint32_t(n1) * 256u, bar);
    if (tk > n1) tma_load(static_cast<uint8_t*>(dst) + size_t(n1) * 256, base, uint32_t(tk - n1) * 256u, bar);
    if (rope_dst) tma_load(rope_dst, a.rope_local + size_t(g.lo + t0) * 64, rb, bar);
}

// One attention task: split s of the layer's key window for query heads [4 hg, 4 hg + 4).
// Same arithmetic as k_qkv + k_attn_partial. Writes the tagged split partials of its heads.
// Returns false when a wait gave up.
__device__ __forceinline__ bool attention_task(const MegaArgs& a, const MegaLayer& Ly, const SplitGeo& g, int s, int hg,
                                            int task, uint32_t tag, const AttnSmem& sm, AttnBars& ab, unsigned long long* dt) {
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int H = a.H, cap = Ly.cap, per_max = Ly.per_max;
    const bool full = Ly.full != 0;
    const int n = g.hi - g.lo, ntiles = (n + MEGA_ATM - 1) / MEGA_ATM;
    const int newest = g.count - 1;
    const bool owner = g.lo <= newest && newest < g.hi;
    const int jnew = owner ? newest - g.lo : -1;  // split-relative row of this step's key
    if (dt && t == 0) dt[0] = gtime();
    // key and value tiles (cache rows written by earlier steps) before the queries are ready
    if (t == ISSUER) {
        issue_rows(a, sm.kraw, Ly.keys, g, 0, min(MEGA_ATM, n), cap, full ? nullptr : sm.rope, &ab.bar[AB_K]);
        issue_rows(a, sm.vraw, Ly.values, g, 0, min(MEGA_ATM, n), cap, nullptr, &ab.bar[AB_V]);
    }
    ab.pending |= (1u << AB_K) | (1u << AB_V);
    // norm weights and RoPE rows of the warp's head (step-independent): in flight during the wait
    const int h0 = MEGA_HG * hg, nq = min(MEGA_HG, H - h0);
    const bool qwarp = warp < nq, kwarp = warp == MEGA_HG && owner;
    const uint16_t* nwp = qwarp ? Ly.q_norm : Ly.k_norm;
    const uint32_t* rrow = qwarp ? (full ? a.rope_global : a.rope_local) + size_t(g.qcoord) * 64
                                 : (full ? a.rope_global + size_t(g.pos) * 64 : nullptr);
    uint16_t nwv[4];
    uint32_t csv[4];
    if (qwarp || kwarp) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            nwv[j] = nwp[lane + 32 * j];
            csv[j] = rrow ? rrow[(lane + 32 * j) & 63] : 0u;
        }
    }
    // every CTA's q/k/v rows are in (their hints); the group's query rows and, for the split that
    // holds this step's key, the key and value rows are read once into shared memory
    bool ok = wait_hints(a.hints, gridDim.x, 1, tag, a.error);
    if (!ok) return false;
    ok = gather16<false>(sm.qkvs, a.qkv + h0 * 128, nq * 128, tag, a.error);
    if (owner && ok) ok = gather16<false>(sm.qkvs + MEGA_HG * 128, a.qkv + H * 128, 256, tag, a.error);
    if (!__syncthreads_and(ok)) return false;
    // per-head RMSNorm with w + 1 and RoPE (Kernels.metal:223-252): warp u < 4 for query head
    // h0 + u; warp 4 for this step's key (rotated at its absolute position on global layers,
    // stored unrotated on local ones), whose value is copied
    if (qwarp || kwarp) {
        const uint16_t* src = sm.qkvs + (qwarp ? warp : MEGA_HG) * 128;
        float v[4], z[4], ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            v[j] = bf2f(src[lane + 32 * j]);
            ss = fmaf(v[j], v[j], ss);
        }
        ss = warp_sum(ss);
        const float scale = 1.0f / sqrtf(ss / 128.0f + PLAMO_EPS);
#pragma unroll
        for (int j = 0; j < 4; j++) z[j] = rbf(rbf(v[j] * scale) * rbf(bf2f(nwv[j]) + 1.0f));
        const size_t slot = size_t(g.pos % cap) * 128;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int d = lane + 32 * j;
            const float r = rrow ? rope_rotate(z[j], z[(j + 2) & 3], d, csv[j]) : z[j];
            if (qwarp) {
                sm.qs[warp * QSM + d] = r;
            } else {
                const uint16_t kb = uint16_t(f2bf(r)), vb = sm.qkvs[(MEGA_HG + 1) * 128 + d];
                sm.knew[d] = kb;
                sm.vnew[d] = vb;
                if (hg == 0) {  // one task of the owning split appends to the cache
                    Ly.keys[slot + d] = kb;
                    Ly.values[slot + d] = vb;
                }
            }
        }
    }
    __syncthreads();
    if (dt && t == 0) dt[1] = gtime();
    const uint16_t* vnew = sm.vnew;
    // pass 1: scores. Thread (key j, head u) runs one fma chain over d = 0..127 (k_attn_partial order).
    for (int tile = 0; tile < ntiles; tile++) {
        const int t0 = tile * MEGA_ATM, tk = min(MEGA_ATM, n - t0);
        if (tile > 0) {
            __syncthreads();
            if (t == ISSUER) issue_rows(a, sm.kraw, Ly.keys, g, t0, tk, cap, full ? nullptr : sm.rope, &ab.bar[AB_K]);
            ab.pending |= 1u << AB_K;
        }
        if (!ab_wait(ab, AB_K, a.error)) ok = false;
        if (!__syncthreads_and(ok)) return false;
        // keys into the padded tile: local keys get the window-relative RoPE (Kernels.metal:277-285),
        // one thread per (d, d + 64) pair; global keys are copied
        if (full) {
            for (int i = t; i < tk * 16; i += 256) {
                const int j = i >> 4, c = i & 15;
                const uint16_t* k16 = t0 + j == jnew ? sm.knew : sm.kraw + j * 128;
                reinterpret_cast<uint4*>(sm.kr + j * KRS)[c] = reinterpret_cast<const uint4*>(k16)[c];
            }
        } else {
            for (int i = t; i < tk * 64; i += 256) {
                const int j = i >> 6, dd = i & 63;
                const uint16_t* k16 = t0 + j == jnew ? sm.knew : sm.kraw + j * 128;
                const uint32_t cs = sm.rope[j * 64 + dd];
                const float x1 = bf2f(k16[dd]), x2 = bf2f(k16[dd + 64]);
                sm.kr[j * KRS + dd] = uint16_t(f2bf(rope_rotate(x1, x2, dd, cs)));
                sm.kr[j * KRS + dd + 64] = uint16_t(f2bf(rope_rotate(x2, x1, dd + 64, cs)));
            }
        }
        __syncthreads();
        const int j = t & (MEGA_ATM - 1), u = t >> 6;
        if (j < tk && MEGA_HG * hg + u < H) {
            const float4* q4 = reinterpret_cast<const float4*>(sm.qs + u * QSM);
            const uint4* k4 = reinterpret_cast<const uint4*>(sm.kr + j * KRS);
            float acc = 0.f;
#pragma unroll 4
            for (int c = 0; c < 16; c++) {
                const uint4 kk = k4[c];
                const float4 qa = q4[2 * c], qb = q4[2 * c + 1];
                acc = fmaf(qa.x, lo_bf(kk.x), acc);
                acc = fmaf(qa.y, hi_bf(kk.x), acc);
                acc = fmaf(qa.z, lo_bf(kk.y), acc);
                acc = fmaf(qa.w, hi_bf(kk.y), acc);
                acc = fmaf(qb.x, lo_bf(kk.z), acc);
                acc = fmaf(qb.y, hi_bf(kk.z), acc);
                acc = fmaf(qb.z, lo_bf(kk.w), acc);
                acc = fmaf(qb.w, hi_bf(kk.w), acc);
            }
            sm.sc[u * per_max + t0 + j] = acc * PLAMO_ATTN_SCALE;
        }
    }
    __syncthreads();
    if (dt && t == 0) dt[2] = gtime();
    // pass 2: split-local softmax statistics, warp u for head u (lane-strided sums, butterfly)
    if (warp < MEGA_HG && MEGA_HG * hg + warp < H) {
        const int h = MEGA_HG * hg + warp;
        float* p0 = sm.sc + warp * per_max;
        float m0 = -INFINITY;
        for (int i = lane; i < n; i += 32) m0 = fmaxf(m0, p0[i]);
        m0 = warp_max(m0);
        float l0 = 0.f;
        for (int i = lane; i < n; i += 32) {
            const float e0 = pexp(p0[i] - m0);
            l0 += e0;
            p0[i] = e0;
        }
        l0 = warp_sum(l0);
        if (lane == 0) {
            st_tag64(a.part_ml + (size_t(s) * H + h) * 2, tagged64(tag, m0));
            st_tag64(a.part_ml + (size_t(s) * H + h) * 2 + 1, tagged64(tag, l0));
        }
    }
    __syncthreads();
    if (dt && t == 0) dt[3] = gtime();
    // pass 3: unnormalised P.V; thread (d, hh) accumulates heads hh and hh + 2 of the group, each
    // one chain over the split's keys in order
    const int d = t & 127, hh = t >> 7;
    float acc0 = 0.f, acc1 = 0.f;
    const float* p0 = sm.sc + hh * per_max;
    const float* p1 = sm.sc + (hh + 2) * per_max;
    for (int tile = 0; tile < ntiles; tile++) {
        const int t0 = tile * MEGA_ATM, tk = min(MEGA_ATM, n - t0);
        if (tile > 0) {
            __syncthreads();
            if (t == ISSUER) issue_rows(a, sm.vraw, Ly.values, g, t0, tk, cap, nullptr, &ab.bar[AB_V]);
            ab.pending |= 1u << AB_V;
        }
        if (!ab_wait(ab, AB_V, a.error)) ok = false;
        if (!__syncthreads_and(ok)) return false;
        int i = 0;
        for (; i + 4 <= tk; i += 4) {
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) v[u] = bf2f((t0 + i + u == jnew ? vnew : sm.vraw + (i + u) * 128)[d]);
            const float4 pa = *reinterpret_cast<const float4*>(p0 + t0 + i);
            const float4 pb = *reinterpret_cast<const float4*>(p1 + t0 + i);
            acc0 = fmaf(pa.x, v[0], acc0);
            acc0 = fmaf(pa.y, v[1], acc0);
            acc0 = fmaf(pa.z, v[2], acc0);
            acc0 = fmaf(pa.w, v[3], acc0);
            acc1 = fmaf(pb.x, v[0], acc1);
            acc1 = fmaf(pb.y, v[1], acc1);
            acc1 = fmaf(pb.z, v[2], acc1);
            acc1 = fmaf(pb.w, v[3], acc1);
        }
        for (; i < tk; i++) {
            const float v = bf2f((t0 + i == jnew ? vnew : sm.vraw + i * 128)[d]);
            acc0 = fmaf(p0[t0 + i], v, acc0);
            acc1 = fmaf(p1[t0 + i], v, acc1);
        }
    }
    const int ha = h0 + hh, hb = ha + 2;
    if (ha < H) st_tag64(a.part_o + (size_t(s) * H + ha) * 128 + d, tagged64(tag, acc0));
    if (hb < H) st_tag64(a.part_o + (size_t(s) * H + hb) * 128 + d, tagged64(tag, acc1));
    __syncthreads();  // the tiles and score rows are free for the next task
    if (t == 0) st_tag(a.hints + 4 * gridDim.x + H + task, tag);
    if (dt && t == 0) dt[4] = gtime();
    return true;
}

// Merge of head h over the layer's first `S` splits (Kernels.metal:530-562): M = max of the split
// maxima, w_q = exp(m_q - M), L = sum of w_q * l_q and o = sum of part_o_q * w_q, both in split
// order; splits without keys are skipped. Polls the tagged partials as they land.
__device__ __forceinline__ bool attention_merge(const MegaArgs& a, int S, int h, uint32_t tag, const AttnSmem& sm, uint32_t out_tag) {
    const int t = threadIdx.x, H = a.H, d = t & 127;
    const int ngroups = (H + MEGA_HG - 1) / MEGA_HG;
    // the head's tasks (s, h / 4) for s < S
    if (!wait_hints(a.hints + 4 * gridDim.x + H + h / MEGA_HG, S, ngroups, tag, a.error)) return false;
    float* pbuf = reinterpret_cast<float*>(sm.kraw);  // [MERGE_CHUNK][128] in kraw
    float* mxy = reinterpret_cast<float*>(sm.kr);      // [S][2] split (max, sum)
    float* mw = mxy + 2 * S;
    // the statistics and the first MERGE_CHUNK partial rows, read once each
    bool ok = gather64x2(mxy, a.part_ml + size_t(h) * 2, 2 * S, 1, size_t(H) * 2, pbuf, a.part_o + size_t(h) * 128,
                         min(MERGE_CHUNK, S) * 128, 7, size_t(H) * 128, tag, a.error);
    if (!__syncthreads_and(ok)) return false;
    // M: a max, exact in any order (every warp computes it); w_q and the split-order chain for L
    // run in every warp with the split statistics in registers, broadcast lane by lane
    const int lane = t & 31;
    float M = -INFINITY;
    for (int q = lane; q < S; q += 32) M = fmaxf(M, mxy[2 * q]);
    M = warp_max(M);
    float L = 0.f, o = 0.f;
    for (int q0 = 0; q0 < S; q0 += 32) {
        const int q = q0 + lane;
        const float l = q < S ? mxy[2 * q + 1] : 0.f;
        const float w = q < S && l > 0.f ? pexp(mxy[2 * q] - M) : -1.f;
        if (t < 32 && q < S) mw[q] = w;
        const int nq = min(32, S - q0);
#pragma unroll 8
        for (int j = 0; j < nq; j++) {
            const float wj = __shfl_sync(FULL_MASK, w, j), lj = __shfl_sync(FULL_MASK, l, j);
            if (wj >= 0.f) L = fmaf(wj, lj, L);
        }
    }
    __syncthreads();
    for (int q0 = 0; q0 < S; q0 += MERGE_CHUNK) {
        const int nq = min(MERGE_CHUNK, S - q0);
        if (q0 > 0) {
            __syncthreads();
            ok = gather64(pbuf, a.part_o + (size_t(q0) * H + h) * 128, nq * 128, 7, size_t(H) * 128, tag, a.error);
            if (!__syncthreads_and(ok)) return false;
        }
        if (t < 128) {
#pragma unroll 8
            for (int q = 0; q < nq; q++) {
                const float w = mw[q0 + q];
                if (w >= 0.f) o = fmaf(pbuf[q * 128 + d], w, o);
            }
        }
    }
    if (t < 128) st_tag(a.att + h * 128 + d, tagged(out_tag, f2bf(o / L)));
    __syncthreads();  // the merge buffers are free, the head's rows are stored: raise its hint
    if (t == 0) st_tag(a.hints + 4 * gridDim.x + h, out_tag);
    return true;
}

size_t mega_xs_bytes(int kmax) { return size_t(((kmax + 511) / 512) * 512) * 2; }
__host__ __device__ inline size_t mega_table_bytes(int nphases, int L) {
    return (size_t(nphases) * sizeof(MegaPhase) + size_t(L) * sizeof(MegaLayer) + 127) & ~size_t(127);
}

// dynamic shared memory: [mbarriers, reduction scratch 256][2 x activations][split-row partials]
// [phase and layer tables][attention]
size_t mega_smem_bytes(int per_max, int splits_max, int kmax, int nphases, int L, int tbl_bytes) {
    const size_t head = 256;
    const size_t fold = size_t(MEGA_FOLD_TASKS) * 32 * 4;
    size_t att = attn_sizes(per_max).total;
    // merge statistics (3 x splits floats) live in the rotated-key region
    if (size_t(3) * splits_max * 4 > attn_sizes(per_max).kr) att = 0;
    const size_t nbuf = size_t(4) * ((kmax + 7) / 8 * 8);  // two norm rows (d <= kmax)
    return att ? head + 2 * mega_xs_bytes(kmax) + fold + mega_table_bytes(nphases, L) + nbuf + size_t(tbl_bytes) + att : 0;
}

// NPT: hidden elements per thread (d <= 256 * NPT).
template <bool PACKED, int NPT>
__global__ void __launch_bounds__(MEGA_THREADS, 1) k_decode_mega(MegaArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* abar = reinterpret_cast<uint64_t*>(smem);  // [2] attention copy barriers
    float* red = reinterpret_cast<float*>(smem + 64);    // [2][8] norm reduction scratch
    int rpar = 0;
    __shared__ int s_flag;
    // two activation buffers, alternating between consecutive weight phases: a phase's staging
    // never overwrites the vector that slower warps of the previous phase are still reading
    uint16_t* const xs_buf = reinterpret_cast<uint16_t*>(smem + 256);
    float* part = reinterpret_cast<float*>(smem + 256 + 2 * a.xs_bytes);  // [MEGA_FOLD_TASKS][32]
    // the phase and layer tables, copied once per step (their global copies are not re-read)
    MegaPhase* const phases = reinterpret_cast<MegaPhase*>(smem + 256 + 2 * a.xs_bytes + MEGA_FOLD_TASKS * 32 * 4);
    MegaLayer* const layers = reinterpret_cast<MegaLayer*>(phases + a.nphases);
    // the two norm-weight rows of the next norm prologue, copied in while the phase before runs
    uint16_t* const nbuf = reinterpret_cast<uint16_t*>(smem + 256 + 2 * a.xs_bytes + MEGA_FOLD_TASKS * 32 * 4 + mega_table_bytes(a.nphases, a.L));
    // .p12: this CTA's block-table entries of the current weight phase, copied at the phase start
    uint32_t* const tbl = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(nbuf) + size_t(4) * a.dpad);
    uint8_t* attn_base = reinterpret_cast<uint8_t*>(tbl) + a.tbl_bytes;
    int wphase = 0;
    const AttnSmem asm_ = attn_smem(attn_base, a.attn_per_max);
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    if (t == 0) {
        for (int i = 0; i < 2; i++) mbar_init(&abar[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    {
        const int nw4 = int(sizeof(MegaPhase) / 4) * a.nphases, lw4 = int(sizeof(MegaLayer) / 4) * a.L;
        for (int i = t; i < nw4; i += MEGA_THREADS) reinterpret_cast<uint32_t*>(phases)[i] = reinterpret_cast<const uint32_t*>(a.phases)[i];
        for (int i = t; i < lw4; i += MEGA_THREADS) reinterpret_cast<uint32_t*>(layers)[i] = reinterpret_cast<const uint32_t*>(a.layers)[i];
    }
    __syncthreads();
    const uint64_t pol = evict_first_policy();
    // rows of the norm table: layer l: 4l pre-mixer, 4l+1 post-mixer, 4l+2 pre-MLP, 4l+3 post-MLP; 4L final
    auto prefetch_norms = [&](int r1, int r2) {
        const int per = a.dpad / 8;
        for (int i = threadIdx.x; i < 2 * per; i += MEGA_THREADS) {
            const int which = i >= per, c = i - which * per, row = which ? r2 : r1;
            if (row >= 0) cp_async16(nbuf + which * a.dpad + c * 8, a.norms + size_t(row) * a.dpad + c * 8);
        }
        cp_async_commit();
    };
    prefetch_norms(-1, 0);
    AttnBars ab{abar, 0u, 0u};
    unsigned long long* trace = a.trace && t == 0 ? a.trace + size_t(cta) * (a.nphases + 1) * MEGA_TRACE_STAMPS : nullptr;
    if (trace) trace[a.nphases * MEGA_TRACE_STAMPS] = gtime();
    const uint32_t step = *reinterpret_cast<volatile unsigned*>(a.step);
    auto tag_of = [&](int layer) -> uint32_t {
        return uint32_t((static_cast<unsigned long long>(step) * unsigned(a.L + 1) + unsigned(layer)) % 65535ull) + 1u;
    };
    const RowDesc dsc0 = a.desc[0];
    const int d = a.d;
    float xres[NPT];  // residual stream (bf16 values), computed identically by every CTA
#pragma unroll
    for (int j = 0; j < NPT; j++) xres[j] = 0.f;
    unsigned long long best = 0ull;
    bool ok = true;

    // the first weight phase's first chunk of this warp
    Batch b;
    bool pref_cur = false, pref_next = false;  // b already holds this / the next phase's first chunk
    PhaseWork pw = phase_work(phases[a.first_weight], cta, G);

    for (int p = 0; p < a.nphases && ok; p++) {
        const MegaPhase ph = phases[p];
        const int l = ph.layer;
        if (trace) trace[p * MEGA_TRACE_STAMPS] = gtime();
        if (ph.kind == MK_ATT) {
            const MegaLayer Ly = layers[l];
            const uint32_t tag = tag_of(l);
            const int S = active_splits(a, Ly, dsc0);
            const int ngroups = (a.H + MEGA_HG - 1) / MEGA_HG, ntask = S * ngroups;
            if (trace) trace[p * MEGA_TRACE_STAMPS + 1] = gtime();
            for (int task = cta; task < ntask && ok; task += G) {
                const int s = task / ngroups, hg = task - s * ngroups;
                const SplitGeo g = split_geo(a, Ly, dsc0, s);
                unsigned long long* dt = a.trace && l == 0 && task == cta
                                             ? a.trace + size_t(G) * (a.nphases + 1) * MEGA_TRACE_STAMPS + size_t(cta) * MEGA_TRACE_DETAIL
                                             : nullptr;
                ok = attention_task(a, Ly, g, s, hg, task, tag, asm_, ab, dt);
            }
            if (ok && cta >= G - a.H) ok = attention_merge(a, S, G - 1 - cta, tag, asm_, tag);
            if (trace) trace[p * MEGA_TRACE_STAMPS + 2] = gtime();
            continue;
        }
        // ---- weight phase p: pw describes it, b holds this warp's first chunk in flight
        // detail stamps (timeline only) of layer 1's weight phases, thread 0: entry, hints seen,
        // input gathered, prologue done, chunk loop done, outputs stored
        unsigned long long* wd = nullptr;
        if (a.trace && t == 0 && l == 1 && ph.kind != MK_HEAD) {
            const int slot = ph.kind == MK_QKV ? 0 : ph.kind == MK_O ? 1 : ph.kind == MK_GU ? 2 : 3;
            wd = a.trace + size_t(G) * (a.nphases + 1) * MEGA_TRACE_STAMPS + size_t(cta) * MEGA_TRACE_DETAIL + 8 + 6 * slot;
            wd[0] = gtime();
        }
        const int nw = ph.next_weight;
        const PhaseWork pn = nw < a.nphases ? phase_work(phases[nw], cta, G) : PhaseWork{};
        const uint32_t tag = tag_of(ph.kind == MK_HEAD ? a.L : l);
        if (PACKED) {  // this CTA's block-table rows of the phase into shared memory (gate rows, then up rows)
            const int bpr = pw.K >> 7, n32 = pw.nu * bpr;
            for (int half = 0; half < (pw.up ? 2 : 1); half++) {
                const uint32_t* src = pw.off + size_t(pw.u0 + half * pw.up) * bpr;
                for (int i = t; i < n32; i += MEGA_THREADS) cp_async4(tbl + half * n32 + i, src + i);
            }
            cp_async_commit();
        }
        uint16_t* const xs = xs_buf + (wphase++ & 1) * (a.xs_bytes / 2);
        const uint4* const xs4 = reinterpret_cast<const uint4*>(xs);
        // prologue: the phase's input vector, staged in the permuted layout. Every prologue passes
        // a CTA barrier, so no warp is still in phase p - 1 when phase p + 1 restages its buffer.
        if (ph.kind == MK_QKV || ph.kind == MK_GU || ph.kind == MK_HEAD) {
            float w1[NPT], w2[NPT], z[NPT];
            const bool first = ph.kind == MK_QKV && l == 0;
            // norm weights: the post-mixer norm (offset 0.2) before the MLP, the post-MLP norm
            // (1/5^1.5) before the next layer / the head (Runtime.swift:446-450), then the pre-norm
            // (offset 1); read from nbuf after the barrier that follows every thread's copy wait
            const float off1 = ph.kind == MK_GU ? 0.2f : a.post_mlp_offset;
            if (PACKED) cp_async_wait_but_newest();  // the norm rows; the table copy may still run
            else cp_async_wait_all();
            if (first) {
                __syncthreads();
                load_norm<NPT>(nbuf + a.dpad, 1.0f, d, w2);
                const int id0 = a.ids[0];
                const size_t row = size_t(id0 >= 0 && id0 < a.V ? id0 : 0) * d;
#pragma unroll
                for (int j = 0; j < NPT; j++) {
                    const int i = t + j * 256;
                    xres[j] = i < d ? bf2f(a.embed[row + i]) : 0.f;
                }
            } else {
                // residual stream + norm of the previous projection (o_proj before the MLP,
                // down_proj before the next layer and the head), as its tagged words land
                const uint32_t* pin = ph.kind == MK_GU ? a.po : a.pd;
                const uint32_t itag = tag_of(ph.kind == MK_HEAD ? a.L - 1 : (ph.kind == MK_GU ? l : l - 1));
                if (!wait_hints(a.hints + (ph.kind == MK_GU ? 1 : 3) * G, G, 1, itag, a.error)) { ok = false; break; }
                if (wd) wd[1] = gtime();
                load_norm<NPT>(nbuf, off1, d, w1);
                load_norm<NPT>(nbuf + a.dpad, 1.0f, d, w2);
                // the vector lands in this phase's activation buffer, which the norm overwrites only
                // after its barriers
                ok = gather16<false>(xs, pin, d, itag, a.error);
                if (!__syncthreads_and(ok)) break;
                float pv[NPT];
#pragma unroll
                for (int j = 0; j < NPT; j++) {
                    const int i = t + j * 256;
                    pv[j] = i < d ? bf2f(xs[i]) : 0.f;
                }
                if (trace) trace[p * MEGA_TRACE_STAMPS + 1] = gtime();
                if (wd) wd[2] = gtime();
                cnorm<NPT>(pv, d, w1, red, rpar, z);
#pragma unroll
                for (int j = 0; j < NPT; j++) {
                    const int i = t + j * 256;
                    xres[j] = i < d ? rbf(xres[j] + z[j]) : 0.f;
                }
            }
            cnorm<NPT>(xres, d, w2, red, rpar, z);
            // every thread has read nbuf (before the norm's barrier): fetch the next prologue's rows
            if (ph.kind == MK_QKV) prefetch_norms(4 * l + 1, 4 * l + 2);
            else if (ph.kind == MK_GU) prefetch_norms(4 * l + 3, l + 1 < a.L ? 4 * (l + 1) : 4 * a.L);
#pragma unroll
            for (int j = 0; j < NPT; j++) {
                const int i = t + j * 256;
                if (i < d) {
                    const uint16_t bv = uint16_t(f2bf(z[j]));
                    xs[xs_index(i)] = bv;
                    if (ph.kind == MK_HEAD && cta == 0) a.hidden[i] = bv;
                }
            }
        } else {
            // o_proj reads the merged attention rows, down_proj the SwiGLU activations
            if (pw.nchunk > 0) {
                ok = ph.kind == MK_O ? wait_hints(a.hints + 4 * G, a.H, 1, tag, a.error)
                                     : wait_hints(a.hints + 2 * G, G, 1, tag, a.error);
                if (wd) wd[1] = gtime();
                if (ok) ok = gather16<true>(xs, ph.kind == MK_O ? a.att : a.act, ph.lin.K, tag, a.error);
            }
            if (!__syncthreads_and(ok)) break;
            if (trace) trace[p * MEGA_TRACE_STAMPS + 1] = gtime();
            if (wd) wd[2] = gtime();
        }
        __syncthreads();
        if (wd) wd[3] = gtime();
        // raw weights: the first chunk's rows were prefetched into L2 one or two phases ago; its
        // loads are issued only now, so no burst of loads sits in front of this phase's exchange
        if (PACKED) {
            cp_async_wait_all();
            __syncthreads();
        }
        // Phases of several chunk rounds: warp pair q starts q x 0.5 us after pair 0 (its first
        // chunk's loads, or the sums of the chunk it prefetched), so the pairs take turns between
        // waiting for HBM and summing and the stream does not pause while all warps compute.
        if (pw.nchunk > 8) {
            const uint64_t t0 = gtime(), dly = uint64_t(warp >> 1) * MEGA_STAGGER_NS;
            while (gtime() - t0 < dly) __nanosleep(128);
        }
        if (first_chunk(pw, warp) < pw.nchunk && !pref_cur) issue_chunk<PACKED>(pw, first_chunk(pw, warp), b, pol, tbl);
        pref_cur = false;
        // ---- the warp's chunks; each chunk's successor (in this phase or the next weight phase)
        // is issued before the chunk's sums are reduced and stored
        float gstash = 0.f;  // SwiGLU: the gate sums of the warp's last gate chunk (lane 8 r: output r)
        for (int c = first_chunk(pw, warp);; c = next_chunk(pw, c)) {
            const bool have = c < pw.nchunk;
            float res[RB];
            if (have) chunk_partials<PACKED>(pw, c, b, xs4, res);
            {  // the successor: the warp's next chunk of this phase, else (raw weights) its first chunk
               // of the next weight phase, in flight across the phase boundary
                const bool inph = next_chunk(pw, c) < pw.nchunk;
                const PhaseWork nx = inph ? pw : pn;
                const int nc = inph ? next_chunk(pw, c) : first_chunk(pn, warp);
                if ((inph || (!PACKED && nw < a.nphases)) && nc < nx.nchunk) issue_chunk<PACKED>(nx, nc, b, pol, tbl);
                if (!inph && !PACKED) pref_next = nw < a.nphases && nc < nx.nchunk;
            }
            if (!have) break;
            if (ph.kind == MK_O || ph.kind == MK_DOWN) {
                // split-row phases: segment partials meet in shared memory, folded below
#pragma unroll
                for (int r = 0; r < RB; r++)
                    if (r < pw.R && c * pw.R + r < pw.ntask) part[(c * pw.R + r) * 32 + lane] = res[r];
                if (next_chunk(pw, c) >= pw.nchunk) break;
                continue;
            }
            // whole-row phases: t = 0 + (a0 + a1) (one segment), then the butterfly; lane 8 r
            // holds task r's sum
            float v4[4];
#pragma unroll
            for (int r = 0; r < 4; r++) v4[r] = r < RB ? 0.f + res[r] : 0.f;
            const float sum = warp_reduce_transposed<4>(v4, lane);
            const int r = lane >> 3;
            int row = 0, seg = 0;
            const bool mine = (lane & 7) == 0 && task_of(pw, c, r, row, seg);
            if (ph.kind == MK_GU) {
                // a gate chunk parks its sums; the up chunk that follows finishes the outputs
                if ((c & 1) == 0) {
                    gstash = sum;
                } else if (mine) {
                    const float gq = rbf(gstash), uq = rbf(sum);
                    st_tag(a.act + (row - pw.up), tagged(tag, f2bf(rbf(rbf(gq / (1.0f + pexp(-gq))) * uq))));
                }
            } else if (mine) {
                const uint32_t bits = f2bf(sum);
                if (ph.kind == MK_QKV) {
                    st_tag(a.qkv + row, tagged(tag, bits));
                } else {
                    a.logits[row] = uint16_t(bits);
                    const unsigned long long key = argmax_key(bf2f(bits), uint32_t(row));
                    best = key > best ? key : best;
                }
            }
            if (next_chunk(pw, c) >= pw.nchunk) break;
        }
        if (wd) wd[4] = gtime();
        if (ph.kind == MK_O || ph.kind == MK_DOWN) {
            // fold each row's segment partials in segment order, then the butterfly (one warp per row)
            __syncthreads();
            uint32_t* out = ph.kind == MK_O ? a.po : a.pd;
            for (int rl = warp; rl < pw.nu; rl += 8) {
                float s = 0.f;
                for (int sg = 0; sg < pw.nseg; sg++) s = s + part[(rl * pw.nseg + sg) * 32 + lane];
                s = warp_sum(s);
                if (lane == 0) st_tag(out + pw.u0 + rl, tagged(tag, f2bf(s)));
            }
        }
        if (ph.kind != MK_HEAD) {  // this CTA's outputs of the phase are stored: raise its hint
            __syncthreads();
            if (t == 0) st_tag(a.hints + (ph.kind == MK_QKV ? 0 : ph.kind == MK_O ? 1 : ph.kind == MK_GU ? 2 : 3) * G + cta, tag);
            if (wd) wd[5] = gtime();
        }
        if (a.trace && lane == 0)  // a phase ends for the CTA when its last warp is done
            atomicMax(a.trace + (size_t(cta) * (a.nphases + 1) + p) * MEGA_TRACE_STAMPS + 2, gtime());
        pw = pn;
        pref_cur = pref_next;
        pref_next = false;
    }
    // no bulk copy may still be writing this CTA's shared memory when its threads exit (only an
    // aborted step can leave one pending)
    __syncthreads();
    if (t == 0)
        for (int i = 0; i < 2; i++)
            if ((ab.pending >> i) & 1u) mbar_drain(&abar[i], (ab.parity >> i) & 1u, a.error);
    if (!__syncthreads_and(ok)) return;
    // head epilogue: CTA argmax -> global key; the last CTA finishes the step
    if (trace) trace[a.nphases * MEGA_TRACE_STAMPS + 1] = gtime();
    __shared__ unsigned long long keys8[8];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {  // the emitting lanes of a warp are 0, 8, 16 and 24
        const unsigned long long other = __shfl_xor_sync(FULL_MASK, best, o);
        best = other > best ? other : best;
    }
    if (lane == 0) keys8[warp] = best;
    __syncthreads();
    if (t == 0) {
        unsigned long long bk = 0ull;
        for (int w = 0; w < 8; w++) bk = keys8[w] > bk ? keys8[w] : bk;
        if (bk) atomicMax(a.amkey, bk);
        __threadfence();
        s_flag = atomicAdd(a.ticket, 1u) == unsigned(G - 1);
        if (trace) trace[a.nphases * MEGA_TRACE_STAMPS + 2] = gtime();
    }
    __syncthreads();
    if (!s_flag || t != 0) return;
    __threadfence();
    const unsigned long long key = atomicAdd(a.amkey, 0ull);
    const int id = int(argmax_index(key));
    a.result[0] = id;
    a.ids[0] = id;
    a.desc[0].pos += 1;
    a.desc[0].cstart += 1;
    const int c = *a.hist_count;
    if (c >= 0 && c < a.hist_cap) {
        a.hist[c] = id;
        *a.hist_count = c + 1;
    }
    *a.amkey = 0ull;
    *a.ticket = 0u;
    *a.step = step + 1u;
    __threadfence();
}

// The persistent kernel's bounded poll on a word that nothing sets, with a caller-chosen limit: the
// failure path of every exchange wait (the poll gives up, raises `error` with ERR_DATA and returns)
// made to run on purpose, for the host's recovery test. One warp polls, as wait_hints does.
__global__ void k_wait_unset(const uint32_t* word, int* error, unsigned long long limit_ns) {
    Spin s;
    for (;;) {
        const bool set = ld_tag(word) != 0u;
        if (__all_sync(FULL_MASK, set)) return;
        if (!__all_sync(FULL_MASK, spin_more(s, error, ERR_DATA, limit_ns))) return;
    }
}

cudaError_t launch_wait_unset(const uint32_t* word, int* error, unsigned long long limit_ns, cudaStream_t s) {
    k_wait_unset<<<1, 32, 0, s>>>(word, error, limit_ns);
    return cudaGetLastError();
}

static const void* mega_kernel(bool packed, int npt) {
    if (packed) {
        if (npt <= 2) return reinterpret_cast<const void*>(k_decode_mega<true, 2>);
        return reinterpret_cast<const void*>(k_decode_mega<true, 6>);
    }
    if (npt <= 2) return reinterpret_cast<const void*>(k_decode_mega<false, 2>);
    return reinterpret_cast<const void*>(k_decode_mega<false, 6>);
}

int mega_npt(int d) { return d <= 512 ? 2 : 6; }

cudaError_t configure_mega(size_t smem, bool packed, int npt) {
    return cudaFuncSetAttribute(mega_kernel(packed, npt), cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
}

int mega_occupancy(size_t smem, bool packed, int npt) {
    int n = 0;
    const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, mega_kernel(packed, npt), MEGA_THREADS, smem);
    return e == cudaSuccess ? n : 0;
}

cudaError_t launch_mega(const MegaArgs& a, int grid, size_t smem, cudaStream_t s) {
    MegaArgs args = a;
    void* params[] = {&args};
    return cudaLaunchCooperativeKernel(mega_kernel(a.phases_packed, mega_npt(a.d)), dim3(grid), dim3(MEGA_THREADS),
                                       params, smem, s);
}

}  // namespace plamo
