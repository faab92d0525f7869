// Persistent batch-1 decode step for sm_100a: one cooperative launch per token, one CTA per SM.
//
// Every CTA owns a contiguous share of the output rows of every projection and streams its weight
// tiles for the whole step (all 16 layers and the lm_head) through a 6-slot shared-memory ring
// with TMA bulk copies (cp.async.bulk + mbarrier complete_tx). The ring runs ahead of the data
// dependencies: the last of the 8 warps to release a slot refills it with the tile six ahead in
// the step's order, so the next phase's first tiles are already resident while the warps wait at
// a phase boundary. (No dedicated producer warp: with 8 warps every thread may hold 255
// registers, with a ninth the register file's per-scheduler split would cap it at 168.) The 8
// warps run the phases of the step:
//   QKV  (prologue: residual + post-MLP norm of the previous layer, pre-mixer norm)  Runtime.swift:377,450
//   ATT  (QK-norm + RoPE + KV append fused, split-K attention, merge by the last split) Kernels.metal:223-562
//   O    (o_proj)                                                                      Runtime.swift:445
//   GU   (prologue: residual + post-mixer norm, pre-MLP norm; SwiGLU epilogue)         Runtime.swift:446-448
//   DOWN (down_proj)                                                                   Runtime.swift:449
//   HEAD (residual + post-MLP norm, final norm, lm_head, first-index argmax)           Runtime.swift:450-458
// Phases are joined by device counters in global memory; every wait is bounded in time and
// raises the error flag (read by the host after the step) instead of hanging.
// The arithmetic of every output follows the same per-element operation order as kernels.cu (and
// the CPU restatement), so this path is bit-identical to the multi-kernel path.
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
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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
// Tiled tensor copy (3-D map, no multicast) global -> this CTA's shared memory, completion on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int c0, int c1, int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            smem_u32(dst)),
        "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// orders this thread's earlier generic-proxy accesses (and the data it acquired) before its next
// bulk copies, which run in the async proxy
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async;" ::: "memory"); }
__device__ __forceinline__ uint16_t ldcg16(const uint16_t* p) { return __ldcg(reinterpret_cast<const unsigned short*>(p)); }

constexpr uint64_t WAIT_NS = 2000000000ull;  // every wait gives up after 2 s
enum MegaError { ERR_CONSUMER = 12, ERR_COUNTER = 13, ERR_DRAIN = 14 };

// The error flag and the clock are checked every 64 polls only: the flag is one global word that
// every waiting warp of the grid would otherwise hammer.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* error, int code) {
    if (mbar_test(bar, parity)) return true;
    const uint64_t t0 = gtime();
    for (uint32_t i = 1;; i++) {
        if (mbar_test(bar, parity)) return true;
        if ((i & 63u) == 0) {
            if (*reinterpret_cast<volatile int*>(error)) return false;
            if (gtime() - t0 > WAIT_NS) {
                atomicCAS(error, 0, code);
                return false;
            }
        }
    }
}

// Waits for the completion of copies already issued into this CTA's shared memory before it
// exits; bounded in time only (a copy from valid global memory always completes).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity, int* error) {
    const uint64_t t0 = gtime();
    while (!mbar_test(bar, parity)) {
        if (gtime() - t0 > WAIT_NS) {
            atomicCAS(error, 0, ERR_DRAIN);
            return;
        }
    }
}

__device__ __forceinline__ bool counter_wait(const unsigned* c, unsigned target, int* error) {
    const uint64_t t0 = gtime();
    for (uint32_t i = 1;; i++) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
        if (v >= target) return true;
        if ((i & 15u) == 0) {
            if (*reinterpret_cast<volatile int*>(error)) return false;
            if (gtime() - t0 > WAIT_NS) {
                atomicCAS(error, 0, ERR_COUNTER);
                return false;
            }
        }
        __nanosleep(32);
    }
}

// ---- tile schedule ---------------------------------------------------------------------------
struct TileSpec {
    const uint8_t* data;
    const uint32_t* table;
    uint32_t data_bytes, table_bytes;
    int row0;  // first weight row (tensor-map tiles)
};

__device__ __forceinline__ void block_range(int out_rows, int tile_rows, int cta, int G, int& b0, int& b1) {
    const int nb = (out_rows + tile_rows - 1) / tile_rows;
    b0 = int((long long)nb * cta / G);
    b1 = int((long long)nb * (cta + 1) / G);
}

__device__ __forceinline__ TileSpec tile_spec(const MegaPhase& ph, int block, int sub) {
    const int K = ph.lin.K;
    int r0 = block * ph.tile_rows;
    const int n = min(ph.tile_rows, ph.out_rows - r0);
    if (sub) r0 += ph.out_rows;  // up rows of the SwiGLU phase
    TileSpec t;
    t.row0 = r0;
    if (!ph.lin.offsets) {
        // raw weights come through the phase's swizzled tensor map as a full box of tile_rows
        // rows (rows past the matrix are zero-filled and still counted)
        t.data = ph.lin.w + size_t(r0) * K * 2;
        t.data_bytes = uint32_t(ph.tile_rows) * K * 2;
        t.table = nullptr;
        t.table_bytes = 0;
    } else {
        const uint32_t a = __ldg(ph.rowoff + r0), b = __ldg(ph.rowoff + r0 + n);
        t.data = ph.lin.w + a;
        t.data_bytes = b - a;
        t.table = ph.lin.offsets + size_t(r0) * (K / 128);
        t.table_bytes = (uint32_t(n) * (K / 128) * 4 + 15u) & ~15u;
    }
    return t;
}

// Walks this CTA's tiles of every weight phase in step order. Holds the current phase
// descriptor and, loaded one phase early (nothing waits for it until the phase ends), the next
// weight phase's, so advancing costs no global read on the critical path.
struct Cursor {
    MegaPhase ph, nxt;
    int p, b, b1, sub;
};

// Enters weight phase q (descriptor phq) or the first later one with blocks for this CTA.
__device__ __forceinline__ bool cursor_enter(const MegaArgs& a, Cursor& c, int q, MegaPhase phq, int cta, int G) {
    while (q < a.nphases) {
        int b0, b1;
        block_range(phq.out_rows, phq.tile_rows, cta, G, b0, b1);
        if (b0 < b1) {
            c.p = q;
            c.ph = phq;
            c.b = b0;
            c.b1 = b1;
            c.sub = 0;
            if (phq.next_weight < a.nphases) c.nxt = a.phases[phq.next_weight];
            return true;
        }
        q = phq.next_weight;
        if (q < a.nphases) phq = a.phases[q];
    }
    return false;
}
__device__ __forceinline__ bool cursor_seek(const MegaArgs& a, Cursor& c, int cta, int G) {
    return a.nphases > 0 && cursor_enter(a, c, a.first_weight, a.phases[a.first_weight], cta, G);
}
__device__ __forceinline__ bool cursor_next(const MegaArgs& a, Cursor& c, int cta, int G) {
    if (c.ph.kind == MK_GU && c.sub == 0) {
        c.sub = 1;
        return true;
    }
    c.sub = 0;
    if (++c.b < c.b1) return true;
    return c.ph.next_weight < a.nphases && cursor_enter(a, c, c.ph.next_weight, c.nxt, cta, G);
}

// ---- consumer building blocks (256 threads; same arithmetic order as kernels.cu) ----------------
constexpr int QSM = 132;  // query row stride (floats) in shared memory
constexpr int ATM = 64;   // keys per staged attention tile

__device__ __forceinline__ float cblock_sum(float v, float* red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    consumers_sync();
    if (lane == 0) red[warp] = v;
    consumers_sync();
    if (warp == 0) {
        float s = lane < 8 ? red[lane] : 0.f;
        s = warp_sum(s);
        if (lane == 0) red[8] = s;
    }
    consumers_sync();
    return red[8];
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
__device__ __forceinline__ void cnorm(const float (&v)[NPT], int n, const float (&wf)[NPT], float* red, float (&z)[NPT]) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NPT; j++) ss = fmaf(v[j], v[j], ss);
    const float total = cblock_sum(ss, red);
    const float scale = 1.0f / sqrtf(total / float(n) + PLAMO_EPS);
#pragma unroll
    for (int j = 0; j < NPT; j++) {
        const int i = threadIdx.x + j * 256;
        z[j] = i < n ? rbf(rbf(v[j] * scale) * wf[j]) : 0.f;
    }
}

// bf16 activation element i -> permuted shared layout used by row_dot (conflict-free 16-B reads)
__device__ __forceinline__ int xs_index(int i) {
    const int c = i >> 3, g = c >> 6, within = c & 63;
    return ((g * 64 + (within & 1) * 32 + (within >> 1)) << 3) + (i & 7);
}

__device__ __forceinline__ void stage_vec(uint16_t* xs, const uint16_t* src, int n) {
    for (int i = threadIdx.x; i < n; i += 256) xs[xs_index(i)] = ldcg16(src + i);
}

// Both halves of a bf16 pair times the matching halves of x, accumulated into the even (lo) and
// odd (hi) chains with sm_100's mixed-precision fma (bf16 x bf16 + f32, one rounding): the same
// result as fmaf on the widened operands, without unpacking either pair.
__device__ __forceinline__ void fma_bf16x2(uint32_t w, uint32_t x, float& lo, float& hi) {
    asm("{\n .reg .b16 wl, wh, xl, xh;\n mov.b32 {wl, wh}, %2;\n mov.b32 {xl, xh}, %3;\n"
        " fma.rn.f32.bf16 %0, wl, xl, %0;\n fma.rn.f32.bf16 %1, wh, xh, %1;\n}"
        : "+f"(lo), "+f"(hi)
        : "r"(w), "r"(x));
}

// The 16 weights of row r at element e0 of a ring tile, as 8 bf16 pairs (raw or .p12 blocks).
// Raw tiles arrive 128-byte swizzled (the tensor map's SWIZZLE_128B on a 1024-byte aligned slot):
// 16-byte chunk c of 128-byte line L sits at chunk c ^ (L & 7), so the two 16-byte reads of the
// 8 lanes of each quarter-warp hit 8 distinct chunk positions (no bank conflict).
template <bool PACKED>
__device__ __forceinline__ void tile_w16(const uint8_t* tile, const uint32_t* tab, int r, int K, int e0, uint32_t (&wp)[8]) {
    if (!PACKED) {
        const uint32_t line = uint32_t(r) * uint32_t(K >> 6) + uint32_t(e0 >> 6), c = uint32_t(e0 & 63) >> 3;
        const uint8_t* lb = tile + size_t(line) * 128;
        const uint4 A = *reinterpret_cast<const uint4*>(lb + ((c ^ (line & 7u)) << 4));
        const uint4 B = *reinterpret_cast<const uint4*>(lb + (((c + 1u) ^ (line & 7u)) << 4));
        wp[0] = A.x; wp[1] = A.y; wp[2] = A.z; wp[3] = A.w;
        wp[4] = B.x; wp[5] = B.y; wp[6] = B.z; wp[7] = B.w;
    } else {
        const uint32_t entry = tab[r * (K >> 7) + (e0 >> 7)];
        const uint8_t* blk = tile + ((entry & ~63u) - (tab[0] & ~63u));
        const uint32_t i0 = uint32_t(e0 & 127), tag = entry & 63u;
        if (tag) {
            decode16(*reinterpret_cast<const uint4*>(blk + i0), *reinterpret_cast<const uint2*>(blk + 128 + (i0 >> 1)),
                     tag + 107u, wp);
        } else {
            const uint4 A = *reinterpret_cast<const uint4*>(blk + 2 * i0);
            const uint4 B = *reinterpret_cast<const uint4*>(blk + 2 * i0 + 16);
            wp[0] = A.x; wp[1] = A.y; wp[2] = A.z; wp[3] = A.w;
            wp[4] = B.x; wp[5] = B.y; wp[6] = B.z; wp[7] = B.w;
        }
    }
}

// Lane partials of two weight rows (row rA of tile A, row rB of tile B; a row is skipped when its
// flag is false) over the groups [gb, ge) of 512 weights (lane l: elements g*512 + 16l .. +16),
// against the activations this lane holds in registers (bf16 pairs xr[g - gb]). The two rows
// are independent chains computed side by side for instruction-level parallelism; each follows
// the GEMV order of kernels.cu: two fma chains (even / odd elements) per 1536-weight segment,
// segment sums folded in order (t = t + (a0 + a1)). With `raw_segment` the single segment's
// a0 + a1 is returned instead (a warp computing one segment of a split row).
template <bool PACKED>
__device__ __forceinline__ void lane_partial2(const uint8_t* tA, const uint32_t* tabA, int rA, bool okA, const uint8_t* tB,
                                              const uint32_t* tabB, int rB, bool okB, int K, int gb, int ge,
                                              const uint32_t (&xr)[4][8], bool raw_segment, float& outA, float& outB) {
    const int lane = threadIdx.x & 31;
    float tA_ = 0.f, a0 = 0.f, a1 = 0.f, sA = 0.f;
    float tB_ = 0.f, b0 = 0.f, b1 = 0.f, sB = 0.f;
#pragma unroll
    for (int gi = 0; gi < 4; gi++) {
        const int g = gb + gi;
        if (g < ge) {
            const int e0 = g * 512 + lane * 16;
            if (e0 < K) {
                uint32_t wa[8], wb[8];
                if (okA) tile_w16<PACKED>(tA, tabA, rA, K, e0, wa);
                if (okB) tile_w16<PACKED>(tB, tabB, rB, K, e0, wb);
                if (okA) {
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        fma_bf16x2(wa[k], xr[gi][k], a0, a1);
                        if (okB) fma_bf16x2(wb[k], xr[gi][k], b0, b1);
                    }
                } else if (okB) {
#pragma unroll
                    for (int k = 0; k < 8; k++) fma_bf16x2(wb[k], xr[gi][k], b0, b1);
                }
            }
            if (gi == 2 || g == ge - 1) {  // end of a 1536-weight segment
                sA = a0 + a1;
                tA_ = tA_ + sA;
                sB = b0 + b1;
                tB_ = tB_ + sB;
                a0 = a1 = b0 = b1 = 0.f;
            }
        }
    }
    outA = raw_segment ? sA : tA_;
    outB = raw_segment ? sB : tB_;
}

// Two independent butterfly sums over the warp, interleaved.
__device__ __forceinline__ void warp_sum2(float& x, float& y) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        x += __shfl_xor_sync(0xffffffffu, x, o);
        y += __shfl_xor_sync(0xffffffffu, y, o);
    }
}

// The CTA's weight ring as seen by one warp. Every warp consumes every tile in step order and
// keeps an identical lead cursor on the tile MEGA_SLOTS ahead; the warp whose release completes
// a slot's count (rel) issues that tile into the slot.
struct ConsumerRing {
    uint64_t* full;    // [MEGA_SLOTS] tile landed (TMA complete_tx)
    unsigned* rel;     // [MEGA_SLOTS] warps done with the slot's current tile
    unsigned* issued;  // [MEGA_SLOTS] tiles issued into the slot so far (for the exit drain)
    uint8_t* ring;     // [MEGA_SLOTS][MEGA_SLOT_DATA], 1024-byte aligned
    uint8_t* tables;   // [MEGA_SLOTS][MEGA_TABLE_BYTES] .p12 block tables of the tiles
    int slot;
    uint32_t parity;  // bit i: phase parity of slot i's next fill
    Cursor lead;      // the tile MEGA_SLOTS ahead of this warp's next one
    bool lead_has;
};

// Issues the weight tile at `c` into ring slot `slot` (one thread). The weights are never
// written, and the slot's previous tile has been read by every warp (each warp's release follows
// its last read of the slot), so no proxy fence is needed.
__device__ __forceinline__ void issue_tile(const Cursor& c, uint8_t* ring, uint8_t* tables, uint64_t* full, int slot) {
    const TileSpec ts = tile_spec(c.ph, c.b, c.sub);
    mbar_expect_tx(&full[slot], ts.data_bytes + ts.table_bytes);
    uint8_t* dst = ring + size_t(slot) * MEGA_SLOT_DATA;
    if (c.ph.tmap) {
        tma_load_3d(dst, c.ph.tmap, 0, 0, ts.row0, &full[slot]);
    } else {
        tma_load(dst, ts.data, ts.data_bytes, &full[slot]);
        if (ts.table_bytes) tma_load(tables + size_t(slot) * MEGA_TABLE_BYTES, ts.table, ts.table_bytes, &full[slot]);
    }
}

// The warp is done reading slot `s`: count the release; the 8th release refills the slot with
// the lead tile. Every lane advances the lead cursor.
__device__ __forceinline__ void release_slot(const MegaArgs& a, ConsumerRing& cr, int s) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) {
        if (atomicAdd(&cr.rel[s], 1u) == 7u) {
            cr.rel[s] = 0u;
            if (cr.lead_has) {
                issue_tile(cr.lead, cr.ring, cr.tables, cr.full, s);
                cr.issued[s] += 1u;
            }
        }
    }
    if (cr.lead_has) cr.lead_has = cursor_next(a, cr.lead, blockIdx.x, gridDim.x);
}

// Output of row `row` (the full dot product v) of a weight phase. SwiGLU rows only park their
// gate / up sums in shared memory (glu[2 * (row - row0) + sub]); the CTA finishes them together
// at the end of the phase (swiglu_rows).
__device__ __forceinline__ void emit_row(const MegaArgs& a, int kind, int row, float v, int sub, float* glu, int row0,
                                         unsigned long long* best) {
    if (kind == MK_GU) {
        glu[2 * (row - row0) + sub] = v;
    } else if (kind == MK_HEAD) {
        const uint32_t bits = f2bf(v);
        a.logits[row] = uint16_t(bits);
        const unsigned long long key = argmax_key(bf2f(bits), uint32_t(row));
        *best = key > *best ? key : *best;
    } else {
        uint16_t* out = kind == MK_QKV ? a.qkv : (kind == MK_O ? a.po : a.pd);
        out[row] = uint16_t(f2bf(v));
    }
}

// One weight phase: every tile of this CTA's blocks, in the producer's order, two tiles at a
// time (a SwiGLU block's gate and up tiles, otherwise consecutive blocks) so that every warp
// carries two independent rows. Rows of up to 2048 weights: warp w computes row w of each tile.
// Longer rows (down_proj) are split into their 1536-weight segments: warp w computes segment
// w % nseg of row w / nseg, the segment sums meet in shared memory (double-buffered by pair) and
// one warp per row folds them in segment order, the same arithmetic as one warp walking the
// whole row. After a timed-out wait the warp stops computing but keeps walking the schedule
// (later waits fail at once, and split pairs still take their barrier), so all consumer warps
// reach the phase end together.
template <bool PACKED>
__device__ __forceinline__ void gemv_phase(const MegaArgs& a, const MegaPhase& ph, ConsumerRing& cr, const uint16_t* xs,
                                           float* part, unsigned long long* best, unsigned long long* dt) {
    int nt = 0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = ph.lin.K, G = (K + 511) >> 9;
    const bool split = G > 4;
    const int nseg = split ? (G + 2) / 3 : 1;
    const int gb = split ? 3 * (warp % nseg) : 0, ge = split ? min(G, gb + 3) : G;
    // this warp's activations in registers for the whole phase
    uint32_t xr[4][8];
    const uint4* xs4 = reinterpret_cast<const uint4*>(xs);
#pragma unroll
    for (int gi = 0; gi < 4; gi++) {
        const int g = gb + gi;
        uint4 xa = make_uint4(0, 0, 0, 0), xb = xa;
        if (g < ge) {
            xa = xs4[g * 64 + lane];
            xb = xs4[g * 64 + 32 + lane];
        }
        xr[gi][0] = xa.x; xr[gi][1] = xa.y; xr[gi][2] = xa.z; xr[gi][3] = xa.w;
        xr[gi][4] = xb.x; xr[gi][5] = xb.y; xr[gi][6] = xb.z; xr[gi][7] = xb.w;
    }
    int b0, b1;
    block_range(ph.out_rows, ph.tile_rows, blockIdx.x, gridDim.x, b0, b1);
    const int nsub = ph.kind == MK_GU ? 2 : 1;
    const int T = (b1 - b0) * nsub;  // tiles of this CTA in this phase
    const int r = split ? warp / nseg : warp;
    const int row0 = b0 * ph.tile_rows;
    float* glu = part + 2 * 512;  // [rows of this CTA][gate, up]
    for (int k = 0, pair = 0; k < T; k += 2, pair++) {
        const bool two = k + 1 < T;
        const int bA = b0 + k / nsub, subA = k % nsub;
        const int bB = b0 + (k + 1) / nsub, subB = (k + 1) % nsub;
        const int nA = min(ph.tile_rows, ph.out_rows - bA * ph.tile_rows);
        const int nB = two ? min(ph.tile_rows, ph.out_rows - bB * ph.tile_rows) : 0;
        const int sA = cr.slot, sB = cr.slot + 1 == MEGA_SLOTS ? 0 : cr.slot + 1;
        const bool readyA = mbar_wait(&cr.full[sA], (cr.parity >> sA) & 1u, a.error, ERR_CONSUMER);
        const bool readyB = two && mbar_wait(&cr.full[sB], (cr.parity >> sB) & 1u, a.error, ERR_CONSUMER);
        const bool stamp = dt && threadIdx.x == 0 && nt < 4;
        if (stamp) dt[nt * 4] = gtime();
        const uint8_t* tA = cr.ring + size_t(sA) * MEGA_SLOT_DATA;
        const uint8_t* tB = cr.ring + size_t(sB) * MEGA_SLOT_DATA;
        const uint32_t* tabA = reinterpret_cast<const uint32_t*>(cr.tables + size_t(sA) * MEGA_TABLE_BYTES);
        const uint32_t* tabB = reinterpret_cast<const uint32_t*>(cr.tables + size_t(sB) * MEGA_TABLE_BYTES);
        float vA = 0.f, vB = 0.f;
        lane_partial2<PACKED>(tA, tabA, r, readyA && r < nA, tB, tabB, r, readyB && r < nB, K, gb, ge, xr, split, vA, vB);
        if (stamp) dt[nt * 4 + 1] = gtime();
        if (readyA) {
            release_slot(a, cr, sA);
            cr.parity ^= 1u << sA;
            cr.slot = sB;
        }
        if (readyB) {
            release_slot(a, cr, sB);
            cr.parity ^= 1u << sB;
            cr.slot = sB + 1 == MEGA_SLOTS ? 0 : sB + 1;
        }
        if (!split) {
            warp_sum2(vA, vB);
            if (stamp) dt[nt * 4 + 2] = gtime();
            if (lane == 0) {
                if (readyA && r < nA) emit_row(a, ph.kind, bA * ph.tile_rows + r, vA, subA, glu, row0, best);
                if (readyB && r < nB) emit_row(a, ph.kind, bB * ph.tile_rows + r, vB, subB, glu, row0, best);
            }
            if (stamp) dt[nt++ * 4 + 3] = gtime();
            continue;
        }
        float* pk = part + (pair & 1) * 512;  // [tile A | tile B][warp][lane]
        pk[warp * 32 + lane] = vA;
        pk[256 + warp * 32 + lane] = vB;
        consumers_sync();
        // warp w folds the pair's row w: rows 0..nA-1 of tile A, then rows of tile B
        const bool inA = warp < nA, inB = !inA && warp < nA + nB;
        if (inA || inB) {
            const int rr = inA ? warp : warp - nA;
            const float* src = pk + (inA ? 0 : 256) + rr * nseg * 32 + lane;
            float t = 0.f;
            for (int sgi = 0; sgi < nseg; sgi++) t = t + src[sgi * 32];
            t = warp_sum(t);
            if (lane == 0) emit_row(a, ph.kind, (inA ? bA : bB) * ph.tile_rows + rr, t, inA ? subA : subB, glu, row0, best);
        }
    }
    if (ph.kind == MK_GU) {  // SwiGLU of this CTA's rows (Kernels.metal:202-210), all threads at once
        consumers_sync();
        const int nrows = min(ph.out_rows, b1 * ph.tile_rows) - row0;
        for (int i = threadIdx.x; i < nrows; i += 256) {
            const float gq = rbf(glu[2 * i]), uq = rbf(glu[2 * i + 1]);
            a.act[row0 + i] = uint16_t(f2bf(rbf(rbf(gq / (1.0f + pexp(-gq))) * uq)));
        }
    }
}

// Weight rows per tile (host and device agree): whole rows up to 2048 weights, one row per warp;
// longer rows take nseg warps each.
int mega_tile_rows(int K) {
    const int G = (K + 511) / 512, byslot = MEGA_SLOT_DATA / (K * 2);
    if (G > 4) return std::min(byslot, 8 / ((G + 2) / 3));
    return std::max(1, std::min(8, byslot));
}

// ---- attention ---------------------------------------------------------------------------------
// Shared-memory regions of the attention phase (inside the union region, all 16-byte aligned):
//   qs   [H][QSM] f32      normed + rotated queries
//   raw  [ATM][KV*128] bf16 key tile as stored in the cache, later the value tile
//   rope [ATM][64] u32     RoPE rows of the tile's window coordinates (local layers)
//   kr   [ATM][KV*128+8]   rotated keys, rows padded to a 16-byte multiple that keeps 16-byte
//                          loads of 8 consecutive rows on distinct banks (first: q/k/v rows)
//   sc   [H][per_max] f32  scores, then exp(score - m)
//   aux  q/k norm weights, the two RoPE rows of this step, this step's key and value
// The merge of one head reuses raw + rope for up to 64 split partials and kr for the statistics.
struct AttnSizes {
    size_t qs, raw, rope, kr, sc, aux, total;
};
__host__ __device__ inline AttnSizes attn_sizes(int H, int KV, int per_max) {
    AttnSizes z;
    z.qs = size_t(H) * QSM * 4;
    z.raw = size_t(ATM) * KV * 256;
    z.rope = size_t(ATM) * 256;
    z.kr = size_t(ATM) * (KV * 128 + 8) * 2;
    z.sc = size_t(H) * per_max * 4;
    z.aux = 1024 + size_t(KV) * 512;
    z.total = z.qs + z.raw + z.rope + z.kr + z.sc + z.aux;
    return z;
}

struct AttnSmem {
    float* qs;
    uint4* raw;
    uint32_t* rope;
    uint16_t* kr;
    float* sc;
    uint16_t *qn, *kn;        // q_norm / k_norm weights [128]
    uint32_t *ropeq, *ropek;  // RoPE rows of the query coordinate and of the key position [64]
    uint16_t *knew, *vnew;    // this step's key (cache format) and value [KV*128]
};

__device__ __forceinline__ AttnSmem attn_smem(uint8_t* uni, const MegaArgs& a) {
    const AttnSizes z = attn_sizes(a.H, a.KV, a.attn_per_max);
    AttnSmem m;
    uint8_t* q = uni;
    m.qs = reinterpret_cast<float*>(q); q += z.qs;
    m.raw = reinterpret_cast<uint4*>(q); q += z.raw;
    m.rope = reinterpret_cast<uint32_t*>(q); q += z.rope;
    m.kr = reinterpret_cast<uint16_t*>(q); q += z.kr;
    m.sc = reinterpret_cast<float*>(q); q += z.sc;
    m.qn = reinterpret_cast<uint16_t*>(q);
    m.kn = m.qn + 128;
    m.ropeq = reinterpret_cast<uint32_t*>(q + 512);
    m.ropek = m.ropeq + 64;
    m.knew = reinterpret_cast<uint16_t*>(q + 1024);
    m.vnew = m.knew + a.KV * 128;
    return m;
}

// Attention copies are TMA bulk copies, one mbarrier per purpose: key tile + its RoPE rows, this
// step's q/k/v rows, value tile, merge partials. Thread ISSUER issues every copy; all consumer
// threads wait on the barrier, so they all track the same phase parities and pending copies.
enum { AB_K = 0, AB_Q = 1, AB_V = 2, AB_M = 3 };
constexpr int ISSUER = 32;  // warp 1, lane 0 (thread 0 is the counter-polling thread)
struct AttnBars {
    uint64_t* bar;     // [4] in the shared-memory header
    uint32_t parity;   // bit i: parity of barrier i's next completion
    uint32_t pending;  // bit i: copies issued on barrier i and not yet waited for
};
__device__ __forceinline__ void ab_wait(const MegaArgs& a, AttnBars& b, int i) {
    if (mbar_wait(&b.bar[i], (b.parity >> i) & 1u, a.error, ERR_CONSUMER)) b.pending &= ~(1u << i);
    b.parity ^= 1u << i;
}

// Window geometry of split s for the step's single row (Runtime.swift:389-395, Kernels.metal:440-470).
struct SplitGeo {
    int first, count, begin, end, qcoord, pos, lo, hi;
};
__device__ __forceinline__ SplitGeo split_geo(const MegaArgs& a, const MegaLayer& Ly, const RowDesc& dsc, int s) {
    SplitGeo g;
    g.pos = dsc.pos;
    if (Ly.full) {
        g.first = 0; g.count = dsc.cstart + dsc.crows; g.end = dsc.pos + 1; g.begin = 0; g.qcoord = dsc.pos;
    } else {
        g.first = max(0, dsc.cstart - (a.W - 1));
        g.count = dsc.cstart + dsc.crows - g.first;
        g.end = dsc.pos - g.first + 1;
        g.begin = max(0, g.end - a.W);
        g.qcoord = dsc.pos - g.first;
    }
    int per = (g.count + Ly.splits - 1) / Ly.splits;
    per = (per + 31) & ~31;
    const int k0 = s * per, k1 = min(k0 + per, g.count);
    g.lo = max(k0, g.begin);
    g.hi = min(k1, g.end);
    return g;
}

// Issuer only: rows [t0, t0 + tk) of the split's cache window (a ring buffer: at most two
// contiguous row ranges) and, for local layers, the RoPE rows of their window coordinates.
__device__ __forceinline__ void issue_tile(const MegaArgs& a, void* dst, const uint16_t* cache, const SplitGeo& g, int t0,
                                           int tk, int cap, uint32_t* rope_dst, uint64_t* bar) {
    const uint32_t row = uint32_t(a.KV) * 256;
    const uint32_t rb = rope_dst ? uint32_t(tk) * 256u : 0u;
    fence_proxy_async();
    mbar_expect_tx(bar, uint32_t(tk) * row + rb);
    const int start = (g.first + g.lo + t0) % cap, n1 = min(tk, cap - start);
    const uint8_t* base = reinterpret_cast<const uint8_t*>(cache);
    tma_load(dst, base + size_t(start) * row, uint32_t(n1) * row, bar);
    if (tk > n1) tma_load(static_cast<uint8_t*>(dst) + size_t(n1) * row, base, uint32_t(tk - n1) * row, bar);
    if (rope_dst) tma_load(rope_dst, a.rope_local + size_t(g.lo + t0) * 64, rb, bar);
}

// Everything a split reads that this step does not write: its first key tile with the tile's
// RoPE rows (bulk copies), the norm weights and this step's RoPE rows (plain loads; the norm
// weights are only 2-byte aligned). Issued before the wait for the QKV phase so the copies
// overlap it; thread 0, the waiting thread, issues nothing. The plain stores are read after the
// next consumer barrier.
__device__ __forceinline__ void attention_prefetch(const MegaArgs& a, const MegaLayer& Ly, const SplitGeo& g, const AttnSmem& sm,
                                   AttnBars& ab) {
    const int t = threadIdx.x;
    if (g.lo >= g.hi) return;
    if (t == ISSUER)
        issue_tile(a, sm.raw, Ly.keys, g, 0, min(ATM, g.hi - g.lo), Ly.cap, Ly.full ? nullptr : sm.rope, &ab.bar[AB_K]);
    ab.pending |= 1u << AB_K;
    if (t >= 64 && t < 192) {
        sm.qn[t - 64] = Ly.q_norm[t - 64];
        sm.kn[t - 64] = Ly.k_norm[t - 64];
    } else if (t >= 192) {
        const uint32_t* qtab = Ly.full ? a.rope_global : a.rope_local;
        sm.ropeq[t - 192] = qtab[size_t(g.qcoord) * 64 + (t - 192)];
        sm.ropek[t - 192] = a.rope_global[size_t(g.pos) * 64 + (t - 192)];
    }
}

// Split-K attention task `s` (same arithmetic as k_qkv + k_attn_partial): QK-norm and RoPE of the
// queries, the append of this step's key/value by the split that holds it, scores, split-local
// softmax statistics and the unnormalised P.V partial. Expects attention_prefetch's copies issued
// and a consumer barrier after it.
__device__ __forceinline__ void attention_split(const MegaArgs& a, const MegaLayer& Ly, const SplitGeo& g, int s, const AttnSmem& sm,
                                AttnBars& ab, unsigned long long* dt) {
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int H = a.H, KV = a.KV, group = H / KV, cap = Ly.cap, per_max = Ly.per_max;
    const bool full = Ly.full != 0;
    float2* ml = a.part_ml + size_t(s) * H;
    float* po = a.part_o + size_t(s) * H * 128;
    if (g.lo >= g.hi) {
        for (int h = t; h < H; h += 256) ml[h] = make_float2(-INFINITY, 0.f);
        return;
    }
    // this step's q/k/v rows, staged in the rotated-key region (free until the first rotation)
    uint16_t* qkvs = sm.kr;
    if (t == ISSUER) {
        const uint32_t bytes = uint32_t(H + 2 * KV) * 256;
        fence_proxy_async();
        mbar_expect_tx(&ab.bar[AB_Q], bytes);
        tma_load(qkvs, a.qkv, bytes, &ab.bar[AB_Q]);
    }
    ab.pending |= 1u << AB_Q;
    if (dt) {
        dt[0] = gtime();
        dt[9] = clock64();
    }
    ab_wait(a, ab, AB_Q);
    if (dt) dt[1] = gtime();
    ab_wait(a, ab, AB_K);
    if (dt) dt[2] = gtime();
    // queries: per-head RMSNorm (w + 1) and RoPE (Kernels.metal:223-252)
    for (int h = warp; h < H; h += 8) {
        const uint16_t* src = qkvs + h * 128;
        float v[4], z[4], ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) { v[j] = bf2f(src[lane + 32 * j]); ss = fmaf(v[j], v[j], ss); }
        ss = warp_sum(ss);
        const float scale = 1.0f / sqrtf(ss / 128.0f + PLAMO_EPS);
#pragma unroll
        for (int j = 0; j < 4; j++) z[j] = rbf(rbf(v[j] * scale) * rbf(bf2f(sm.qn[lane + 32 * j]) + 1.0f));
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int d = lane + 32 * j;
            sm.qs[h * QSM + d] = rope_rotate(z[j], z[(j + 2) & 3], d, sm.ropeq[d & 63]);
        }
    }
    // the split that holds this step's key appends it to the cache (local layers store it
    // unrotated, global layers rotated) and keeps a copy for its own tiles
    const int newest = g.count - 1;
    const bool owner = g.lo <= newest && newest < g.hi;
    if (owner) {
        for (int kvh = warp; kvh < KV; kvh += 8) {
            const uint16_t* src = qkvs + (H + kvh) * 128;
            float v[4], z[4], ss = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++) { v[j] = bf2f(src[lane + 32 * j]); ss = fmaf(v[j], v[j], ss); }
            ss = warp_sum(ss);
            const float scale = 1.0f / sqrtf(ss / 128.0f + PLAMO_EPS);
#pragma unroll
            for (int j = 0; j < 4; j++) z[j] = rbf(rbf(v[j] * scale) * rbf(bf2f(sm.kn[lane + 32 * j]) + 1.0f));
            const size_t slot = (size_t(g.pos % cap) * KV + kvh) * 128;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int d = lane + 32 * j;
                const float k = full ? rope_rotate(z[j], z[(j + 2) & 3], d, sm.ropek[d & 63]) : z[j];
                const uint16_t kb = uint16_t(f2bf(k)), vb = src[KV * 128 + d];
                Ly.keys[slot + d] = kb;
                Ly.values[slot + d] = vb;
                sm.knew[kvh * 128 + d] = kb;
                sm.vnew[kvh * 128 + d] = vb;
            }
        }
    }
    consumers_sync();
    if (dt) dt[3] = gtime();
    const int KS = KV * 128 + 8, kvw = KV * 128;
    const uint16_t* raw16 = reinterpret_cast<const uint16_t*>(sm.raw);
    const int n = g.hi - g.lo;
    const int jnew = owner ? newest - g.lo : -1;  // split-relative row of this step's key
    const int ntiles = (n + ATM - 1) / ATM;
    // pass 1: scores
    for (int tile = 0; tile < ntiles; tile++) {
        const int t0 = tile * ATM, tk = min(ATM, n - t0);
        if (tile > 0) {
            consumers_sync();
            if (t == ISSUER) issue_tile(a, sm.raw, Ly.keys, g, t0, tk, cap, full ? nullptr : sm.rope, &ab.bar[AB_K]);
            ab.pending |= 1u << AB_K;
            ab_wait(a, ab, AB_K);
        }
        // rotated keys into the padded tile: local keys get the window-relative RoPE
        // (Kernels.metal:277-285), one thread per (d, d + 64) pair; global keys are copied
        if (full) {
            for (int i = t; i < tk * KV * 16; i += 256) {
                const int j = i / (KV * 16), c = i - j * (KV * 16);
                const uint16_t* k16 = t0 + j == jnew ? sm.knew : raw16 + j * kvw;
                reinterpret_cast<uint4*>(sm.kr + j * KS)[c] = reinterpret_cast<const uint4*>(k16)[c];
            }
        } else {
            for (int i = t; i < tk * KV * 64; i += 256) {
                const int j = KV == 1 ? i >> 6 : i / (KV * 64), e = i - j * (KV * 64);
                const int d = e & 63, kvoff = (e >> 6) * 128;
                const uint16_t* k16 = (t0 + j == jnew ? sm.knew : raw16 + j * kvw) + kvoff;
                const uint32_t cs = sm.rope[j * 64 + d];
                const float x1 = bf2f(k16[d]), x2 = bf2f(k16[d + 64]);
                sm.kr[j * KS + kvoff + d] = uint16_t(f2bf(rope_rotate(x1, x2, d, cs)));
                sm.kr[j * KS + kvoff + d + 64] = uint16_t(f2bf(rope_rotate(x2, x1, d + 64, cs)));
            }
        }
        consumers_sync();
        if (dt) dt[4] = gtime();
        if (tile == ntiles - 1) {  // the raw tile is free: start the first value tile
            if (t == ISSUER) issue_tile(a, sm.raw, Ly.values, g, 0, min(ATM, n), cap, nullptr, &ab.bar[AB_V]);
            ab.pending |= 1u << AB_V;
        }
        // scores: thread (key j, head quarter hq) computes heads hq, hq + 4, hq + 8, hq + 12 side by
        // side, each one fma chain over d = 0..127 as the multi-kernel path
        const int j = t & (ATM - 1), hq = t >> 6;
        if (j < tk) {
            const float4* q4[4];
            const uint4* k4[4];
            float acc[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int h = min(hq + 4 * u, H - 1);
                q4[u] = reinterpret_cast<const float4*>(sm.qs + h * QSM);
                k4[u] = reinterpret_cast<const uint4*>(sm.kr + j * KS + (h / group) * 128);
                acc[u] = 0.f;
            }
#pragma unroll 2
            for (int c = 0; c < 16; c++) {
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const uint4 kk = KV == 1 ? k4[0][c] : k4[u][c];
                    const float4 qa = q4[u][2 * c], qb = q4[u][2 * c + 1];
                    acc[u] = fmaf(qa.x, lo_bf(kk.x), acc[u]);
                    acc[u] = fmaf(qa.y, hi_bf(kk.x), acc[u]);
                    acc[u] = fmaf(qa.z, lo_bf(kk.y), acc[u]);
                    acc[u] = fmaf(qa.w, hi_bf(kk.y), acc[u]);
                    acc[u] = fmaf(qb.x, lo_bf(kk.z), acc[u]);
                    acc[u] = fmaf(qb.y, hi_bf(kk.z), acc[u]);
                    acc[u] = fmaf(qb.z, lo_bf(kk.w), acc[u]);
                    acc[u] = fmaf(qb.w, hi_bf(kk.w), acc[u]);
                }
            }
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (hq + 4 * u < H) sm.sc[(hq + 4 * u) * per_max + t0 + j] = acc[u] * PLAMO_ATTN_SCALE;
        }
    }
    consumers_sync();
    if (dt) dt[5] = gtime();
    // pass 2: split-local softmax statistics; warp w handles heads w and w + 8 side by side
    {
        const int h0 = warp, h1 = min(warp + 8, H - 1);
        const bool two = warp + 8 < H;
        if (h0 < H) {
            float* p0 = sm.sc + h0 * per_max;
            float* p1 = sm.sc + h1 * per_max;
            float m0 = -INFINITY, m1 = -INFINITY;
            for (int i = lane; i < n; i += 32) {
                m0 = fmaxf(m0, p0[i]);
                m1 = fmaxf(m1, p1[i]);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
                m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
            }
            float l0 = 0.f, l1 = 0.f;
            for (int i = lane; i < n; i += 32) {
                const float e0 = pexp(p0[i] - m0), e1 = pexp(p1[i] - m1);
                l0 += e0;
                l1 += e1;
                p0[i] = e0;
                if (two) p1[i] = e1;
            }
            warp_sum2(l0, l1);
            if (lane == 0) {
                ml[h0] = make_float2(m0, l0);
                if (two) ml[h1] = make_float2(m1, l1);
            }
        }
    }
    consumers_sync();
    if (dt) dt[6] = gtime();
    // pass 3: unnormalised P.V
    // thread (d, hh) accumulates heads hh, hh + 2, ... (at most 8: H <= 16 on this path), each
    // one chain over the split's keys in order
    const int d = t & 127, hh = t >> 7;
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; q++) acc[q] = 0.f;
    for (int tile = 0; tile < ntiles; tile++) {
        const int t0 = tile * ATM, tk = min(ATM, n - t0);
        if (tile > 0) {
            consumers_sync();
            if (t == ISSUER) issue_tile(a, sm.raw, Ly.values, g, t0, tk, cap, nullptr, &ab.bar[AB_V]);
            ab.pending |= 1u << AB_V;
        }
        ab_wait(a, ab, AB_V);
        if (dt) dt[7] = gtime();
        // probability rows of this thread's heads (clamped to a valid row; results of heads >= H
        // are never stored)
        const float* pq[8];
#pragma unroll
        for (int q = 0; q < 8; q++) pq[q] = sm.sc + min(hh + 2 * q, H - 1) * per_max + t0;
        if (KV == 1) {
            int i = 0;
            for (; i + 4 <= tk; i += 4) {  // four keys per round: 16-byte probability loads
                float v[4];
#pragma unroll
                for (int u = 0; u < 4; u++) v[u] = bf2f((t0 + i + u == jnew ? sm.vnew : raw16 + (i + u) * 128)[d]);
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    const float4 pr = *reinterpret_cast<const float4*>(pq[q] + i);
                    acc[q] = fmaf(pr.x, v[0], acc[q]);
                    acc[q] = fmaf(pr.y, v[1], acc[q]);
                    acc[q] = fmaf(pr.z, v[2], acc[q]);
                    acc[q] = fmaf(pr.w, v[3], acc[q]);
                }
            }
            for (; i < tk; i++) {
                const float v = bf2f((t0 + i == jnew ? sm.vnew : raw16 + i * 128)[d]);
#pragma unroll
                for (int q = 0; q < 8; q++) acc[q] = fmaf(pq[q][i], v, acc[q]);
            }
        } else {
            const float* sct = sm.sc + hh * per_max + t0;
            for (int i = 0; i < tk; i++) {
                const uint16_t* vr = t0 + i == jnew ? sm.vnew : raw16 + i * kvw;
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    const int h = hh + 2 * q;
                    if (h < H) acc[q] = fmaf(sct[2 * q * per_max + i], bf2f(vr[(h / group) * 128 + d]), acc[q]);
                }
            }
        }
    }
#pragma unroll
    for (int q = 0; q < 8; q++)
        if (hh + 2 * q < H) po[(hh + 2 * q) * 128 + d] = acc[q];
    if (dt) {
        dt[8] = gtime();
        dt[10] = clock64();
    }
}

// Merge of head h over the layer's S split partials (Kernels.metal:530-562), run by CTA h once
// every split has been counted: M = max of the split maxima, w_q = exp(m_q - M), L = sum of
// w_q * l_q and o = sum of part_o_q * w_q, both in split order; splits without keys are skipped.
// The partial rows of the head (512 bytes per split) are bulk-copied 64 splits at a time, the
// first batch together with the statistics loads. Returns false when the wait for the splits
// gave up.
constexpr int MERGE_CHUNK = 64;
__device__ __forceinline__ bool attention_merge_head(const MegaArgs& a, int S, int l, int h, const AttnSmem& sm, AttnBars& ab) {
    const int t = threadIdx.x, H = a.H, d = t & 127;
    __shared__ int merge_stop;
    if (t == 0) merge_stop = counter_wait(&a.sync[a.nphases + l], unsigned(S), a.error) ? 0 : 1;
    consumers_sync();
    if (merge_stop) return false;
    float* pbuf = reinterpret_cast<float*>(sm.raw);  // [MERGE_CHUNK][128] (raw + rope regions)
    float* mx = reinterpret_cast<float*>(sm.kr);
    float* my = mx + S;
    float* mw = my + S;
    auto stage = [&](int q0) {
        if (t == ISSUER) {
            const int nq = min(MERGE_CHUNK, S - q0);
            fence_proxy_async();
            mbar_expect_tx(&ab.bar[AB_M], uint32_t(nq) * 512u);
            for (int q = 0; q < nq; q++)
                tma_load(pbuf + q * 128, a.part_o + (size_t(q0 + q) * H + h) * 128, 512u, &ab.bar[AB_M]);
        }
        ab.pending |= 1u << AB_M;
    };
    stage(0);
    for (int q = t; q < S; q += 256) {
        const float2 st = __ldcg(&a.part_ml[size_t(q) * H + h]);
        mx[q] = st.x;
        my[q] = st.y;
    }
    consumers_sync();
    float M = -INFINITY;
    for (int q = 0; q < S; q++) M = fmaxf(M, mx[q]);
    for (int q = t; q < S; q += 256) mw[q] = my[q] > 0.f ? pexp(mx[q] - M) : -1.f;
    consumers_sync();
    float L = 0.f, o = 0.f;
    for (int q = 0; q < S; q++) {
        const float w = mw[q];
        if (w >= 0.f) L = fmaf(w, my[q], L);
    }
    for (int q0 = 0; q0 < S; q0 += MERGE_CHUNK) {
        if (q0 > 0) {
            consumers_sync();
            stage(q0);
        }
        ab_wait(a, ab, AB_M);
        if (t < 128) {
            const int nq = min(MERGE_CHUNK, S - q0);
            for (int q = 0; q < nq; q++) {
                const float w = mw[q0 + q];
                if (w >= 0.f) o = fmaf(pbuf[q * 128 + d], w, o);
            }
        }
    }
    if (t < 128) a.att[h * 128 + d] = uint16_t(f2bf(o / L));
    return true;
}

size_t mega_attention_smem(int H, int KV, int per_max) { return attn_sizes(H, KV, per_max).total; }

// The merge keeps 3 x S statistics in the rotated-key region.
bool mega_merge_fits(int H, int KV, int splits) {
    (void)H;
    return size_t(3) * splits * 4 <= attn_sizes(1, KV, 32).kr;
}

size_t mega_xs_bytes(int kmax) { return size_t(((kmax + 511) / 512) * 512) * 2; }

size_t mega_smem_bytes(int H, int KV, int per_max, int kmax) {
    const size_t head = 256;  // mbarriers + reduction scratch
    // ring data 1024-byte aligned (up to 1 KB of padding) + block tables
    const size_t ring = 1024 + size_t(MEGA_SLOTS) * (MEGA_SLOT_DATA + MEGA_TABLE_BYTES);
    // activations + split-row segment sums + SwiGLU gate/up sums of this CTA's rows
    const size_t gemv = mega_xs_bytes(kmax) + 2 * 512 * 4 + size_t(2) * MEGA_GLU_ROWS * 4;
    return head + ring + std::max(gemv, mega_attention_smem(H, KV, per_max));
}

// NPT: hidden elements per consumer thread (d <= 256 * NPT).
template <bool PACKED, int NPT>
__global__ void __launch_bounds__(MEGA_THREADS, 1) k_decode_mega(MegaArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);        // [6] at 0
    uint64_t* abar = full + MEGA_SLOTS;                         // [4] attention copy barriers at 48
    unsigned* rel = reinterpret_cast<unsigned*>(smem + 80);     // [6] slot release counts
    unsigned* issued = reinterpret_cast<unsigned*>(smem + 104); // [6] tiles issued per slot
    float* red = reinterpret_cast<float*>(smem + 128);
    // ring slots on a 1024-byte boundary (the 128-byte swizzle pattern repeats every 1024 bytes)
    uint8_t* ring = smem + 256 + ((1024u - ((smem_u32(smem) + 256u) & 1023u)) & 1023u);
    uint8_t* tables = ring + size_t(MEGA_SLOTS) * MEGA_SLOT_DATA;
    uint8_t* uni = tables + size_t(MEGA_SLOTS) * MEGA_TABLE_BYTES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    // ring: every thread walks the tile order; thread 0 issues the first MEGA_SLOTS tiles
    ConsumerRing cr;
    cr.full = full;
    cr.rel = rel;
    cr.issued = issued;
    cr.ring = ring;
    cr.tables = tables;
    cr.slot = 0;
    cr.parity = 0;
    cr.lead_has = cursor_seek(a, cr.lead, cta, G);
    if (threadIdx.x == 0) {
        for (int i = 0; i < MEGA_SLOTS; i++) {
            mbar_init(&full[i], 1);
            rel[i] = 0u;
            issued[i] = 0u;
        }
        for (int i = 0; i < 4; i++) mbar_init(&abar[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    for (int i = 0; i < MEGA_SLOTS && cr.lead_has; i++) {
        if (threadIdx.x == 0) {
            issue_tile(cr.lead, ring, tables, full, i);
            issued[i] = 1u;
        }
        cr.lead_has = cursor_next(a, cr.lead, cta, G);
    }

    // ----------------------------------------------------------------------------- consumers
    const int t = threadIdx.x;
    unsigned long long* trace = a.trace && t == 0 ? a.trace + size_t(cta) * (a.nphases + 1) * MEGA_TRACE_STAMPS : nullptr;
    if (trace) trace[a.nphases * MEGA_TRACE_STAMPS] = gtime();
    uint16_t* xs = reinterpret_cast<uint16_t*>(uni);
    const AttnSmem asm_ = attn_smem(uni, a);
    AttnBars ab{abar, 0u, 0u};
    const RowDesc dsc0 = a.desc[0];
    unsigned long long best = 0ull;
    const int d = a.d;
    float xres[NPT];    // residual stream (bf16 values), computed identically by every CTA
    float w1[NPT], w2[NPT];  // norm factors of the current prologue
    // Stop decisions are taken by thread 0 and read by all consumers from shared memory after a
    // barrier, so every consumer warp leaves at the same phase (a split decision would leave the
    // others waiting at the next named barrier). Two alternating flags: the flag of phase p is
    // rewritten at phase p + 2, after every consumer passed the barrier of phase p + 1.
    __shared__ int stop_flag[2];
    bool ok = true;
    for (int p = 0; p < a.nphases; p++) {
        const MegaPhase ph = a.phases[p];
        const int l = ph.layer;
        if (trace) trace[p * MEGA_TRACE_STAMPS] = gtime();
        // -- work that does not depend on the previous phase, overlapping the wait
        MegaLayer Ly;
        SplitGeo g0;
        if (ph.kind == MK_ATT) {
            Ly = a.layers[l];
            if (cta < Ly.splits) {
                g0 = split_geo(a, Ly, dsc0, cta);
                attention_prefetch(a, Ly, g0, asm_, ab);
            }
        } else if (ph.kind == MK_QKV || ph.kind == MK_GU || ph.kind == MK_HEAD) {
            if (!(ph.kind == MK_QKV && l == 0)) {
                // post-mixer norm (offset 0.2) before the MLP, post-MLP norm (1/5^1.5) before the
                // next layer / the head (Runtime.swift:446-450)
                const bool mlp_in = ph.kind == MK_GU;
                const MegaLayer& Lp = a.layers[mlp_in ? l : (ph.kind == MK_HEAD ? a.L - 1 : l - 1)];
                load_norm<NPT>(mlp_in ? Lp.post_mixer : Lp.post_mlp, mlp_in ? 0.2f : a.post_mlp_offset, d, w1);
            }
            const uint16_t* nw = ph.kind == MK_HEAD ? a.final_norm
                                 : (ph.kind == MK_GU ? a.layers[l].pre_mlp : a.layers[l].pre_mixer);
            load_norm<NPT>(nw, 1.0f, d, w2);
        }
        // -- wait for the previous phase (attention completes with one count per merged head)
        if (p > 0) {
            const unsigned target = a.phases[p - 1].kind == MK_ATT ? unsigned(a.H) : unsigned(G);
            if (t == 0)
                stop_flag[p & 1] = counter_wait(&a.sync[p - 1], target, a.error) ? *reinterpret_cast<volatile int*>(a.error) : 1;
            consumers_sync();
            if (stop_flag[p & 1]) { ok = false; break; }
        }
        if (trace) trace[p * MEGA_TRACE_STAMPS + 1] = gtime();
        if (ph.kind == MK_ATT) {
            int nspl = 0;
            for (int s = cta; s < Ly.splits; s += G) {
                if (s != cta) {  // further splits of this CTA (more splits than CTAs)
                    consumers_sync();
                    const SplitGeo g = split_geo(a, Ly, dsc0, s);
                    attention_prefetch(a, Ly, g, asm_, ab);
                    consumers_sync();
                    attention_split(a, Ly, g, s, asm_, ab, nullptr);
                } else {
                    // detail timeline of the first attention phase (tracing only)
                    unsigned long long* dt = trace && l == 0 ? a.trace + size_t(G) * (a.nphases + 1) * MEGA_TRACE_STAMPS + size_t(cta) * MEGA_TRACE_DETAIL : nullptr;
                    attention_split(a, Ly, g0, s, asm_, ab, dt);
                }
                nspl++;
            }
            consumers_sync();
            if (t == 0 && nspl) {
                __threadfence();
                atomicAdd(&a.sync[a.nphases + l], unsigned(nspl));
            }
            bool merged = false;
            if (cta < a.H) merged = attention_merge_head(a, Ly.splits, l, cta, asm_, ab);
            consumers_sync();
            if (t == 0 && merged) {
                __threadfence();
                atomicAdd(&a.sync[p], 1u);
            }
            if (trace) trace[p * MEGA_TRACE_STAMPS + 2] = gtime();
            continue;
        }
        // prologue: the phase's input vector, staged in the permuted layout
        if (ph.kind == MK_QKV || ph.kind == MK_GU || ph.kind == MK_HEAD) {
            float z[NPT];
            if (ph.kind == MK_QKV && l == 0) {
                const int id0 = a.ids[0];
                const size_t row = size_t(id0 >= 0 && id0 < a.V ? id0 : 0) * d;
#pragma unroll
                for (int j = 0; j < NPT; j++) {
                    const int i = t + j * 256;
                    xres[j] = i < d ? bf2f(a.embed[row + i]) : 0.f;
                }
            } else {
                // residual stream + norm of the previous projection
                const uint16_t* pin = ph.kind == MK_GU ? a.po : a.pd;
                float pv[NPT];
#pragma unroll
                for (int j = 0; j < NPT; j++) {
                    const int i = t + j * 256;
                    pv[j] = i < d ? bf2f(ldcg16(pin + i)) : 0.f;
                }
                cnorm<NPT>(pv, d, w1, red, z);
#pragma unroll
                for (int j = 0; j < NPT; j++) {
                    const int i = t + j * 256;
                    xres[j] = i < d ? rbf(xres[j] + z[j]) : 0.f;
                }
            }
            cnorm<NPT>(xres, d, w2, red, z);
#pragma unroll
            for (int j = 0; j < NPT; j++) {
                const int i = t + j * 256;
                if (i < d) {
                    const uint16_t b = uint16_t(f2bf(z[j]));
                    xs[xs_index(i)] = b;
                    if (ph.kind == MK_HEAD && cta == 0) a.hidden[i] = b;
                }
            }
        } else {
            stage_vec(xs, ph.kind == MK_O ? a.att : a.act, ph.lin.K);
        }
        consumers_sync();
        unsigned long long* gdt = trace && ph.kind == MK_GU && l == 0
                                      ? a.trace + size_t(G) * (a.nphases + 1) * MEGA_TRACE_STAMPS + size_t(cta) * MEGA_TRACE_DETAIL + 16
                                      : nullptr;
        if (gdt) gdt[-1] = gtime();
        gemv_phase<PACKED>(a, ph, cr, xs, reinterpret_cast<float*>(uni + a.xs_bytes), &best, gdt);
        consumers_sync();
        if (trace) trace[p * MEGA_TRACE_STAMPS + 2] = gtime();
        if (ph.kind != MK_HEAD && t == 0) {
            __threadfence();
            atomicAdd(&a.sync[p], 1u);
        }
    }
    // no bulk copy may still be writing this CTA's shared memory when its threads exit (only an
    // aborted step can leave one pending): wait for the last tile issued into every ring slot and
    // for the attention copies still outstanding
    consumers_sync();
    if (t == 0) {
        for (int i = 0; i < MEGA_SLOTS; i++)
            if (issued[i]) mbar_drain(&full[i], (issued[i] - 1u) & 1u, a.error);
        for (int i = 0; i < 4; i++)
            if ((ab.pending >> i) & 1u) mbar_drain(&abar[i], (ab.parity >> i) & 1u, a.error);
    }
    if (!ok) return;
    // head epilogue: CTA argmax -> global key; the last CTA finishes the step and resets the counters
    if (trace) trace[a.nphases * MEGA_TRACE_STAMPS + 1] = gtime();
    __shared__ unsigned long long keys8[8];
    if (lane == 0) keys8[warp] = best;
    consumers_sync();
    __shared__ unsigned last;
    if (t == 0) {
        unsigned long long b = 0ull;
        for (int w = 0; w < 8; w++) b = keys8[w] > b ? keys8[w] : b;
        if (b) atomicMax(a.amkey, b);
        __threadfence();
        last = atomicAdd(&a.sync[a.nphases + a.L], 1u) == unsigned(G - 1);
        if (trace) trace[a.nphases * MEGA_TRACE_STAMPS + 2] = gtime();
    }
    consumers_sync();
    if (!last || t != 0) return;
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
    for (int i = 0; i <= a.nphases + a.L; i++) a.sync[i] = 0u;
    __threadfence();
}

static const void* mega_kernel(bool packed, int npt) {
    if (packed) {
        if (npt <= 2) return reinterpret_cast<const void*>(k_decode_mega<true, 2>);
        if (npt <= 6) return reinterpret_cast<const void*>(k_decode_mega<true, 6>);
        return reinterpret_cast<const void*>(k_decode_mega<true, 16>);
    }
    if (npt <= 2) return reinterpret_cast<const void*>(k_decode_mega<false, 2>);
    if (npt <= 6) return reinterpret_cast<const void*>(k_decode_mega<false, 6>);
    return reinterpret_cast<const void*>(k_decode_mega<false, 16>);
}

int mega_npt(int d) { return d <= 512 ? 2 : (d <= 1536 ? 6 : 16); }

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
