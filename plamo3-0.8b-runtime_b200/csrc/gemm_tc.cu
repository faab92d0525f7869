// Tensor-core GEMM for the dense contractions of prefill and of batched steps with many rows:
// Y[r][m] = sum_k X[r][k] W[m][k], bf16 operands, fp32 accumulation on the 5th-generation tensor
// cores (tcgen05.mma kind::f16, accumulators in tensor memory), operands staged by TMA.
//
// Unlike the CUDA-core kernels (kernels.cu, gemm.cu) this path does not reproduce the order-exact
// summation of the CPU restatement: the tensor core adds its products in its own order, so an
// output can differ from the exact path by an ulp of the bf16 result. The runtime uses it only when
// asked (plamo_set_tensor_gemm). Its tests hold every output to one bf16 ulp of a float64 product,
// and a model's logits to a small multiple of the drift the restatement itself shows when its sums
// are reordered, instead of bit equality.
//
// Tile: 128 weight rows (the MMA's M, one tensor-memory lane each) x BN activation rows (the MMA's
// N, one fp32 tensor-memory column each). Each stage holds 64 k of both operands, one 128-byte
// line per row in the 128-byte swizzle that TMA writes and the MMA's shared-memory descriptor
// reads (8-row groups 1024 bytes apart); the four K = 16 MMAs of a stage advance the descriptors'
// start address by 32 bytes. SwiGLU tiles take gate rows m0..m0+63 into lanes 0..63 and the
// matching up rows into lanes 64..127, so one tile finishes 64 outputs.
//
// Roles (128 threads): lane 0 of warp 0 issues the TMA copies (STAGES deep, a stage is refilled
// once the MMAs that read it have committed to its `empty` barrier); lane 0 of warp 1 issues the
// MMAs; then all four warps drain tensor memory (warp w reads lanes 32w..32w+31) and write bf16
// outputs, SwiGLU products (gate and up halves exchanged through shared memory, so all four warps
// share that math) or logits with argmax keys. A tile with few weight rows (small M at few
// activation rows) splits K over `splits` CTAs that store fp32 partials; a second kernel adds them
// in split order and applies the same epilogue.
#include "common.cuh"
#include "kernels.h"
#include "mbarrier.cuh"
#include "tcgen05.cuh"

#include <cstdlib>
#include <algorithm>

namespace plamo {

namespace {

constexpr int TC_BM = 128;       // weight rows per tile (MMA M = tensor-memory lanes)
constexpr int TC_BK = 64;        // k per stage: one 128-byte swizzled line per row
constexpr int TC_UK = 16;        // k per tcgen05.mma of kind::f16
constexpr int TC_THREADS = 128;  // four warps: every tensor-memory lane quarter has its warp
constexpr int TC_SPLITS_MAX = 16;

template <int BN>
struct TcTile {
    static constexpr int A_BYTES = TC_BM * 128;
    static constexpr int B_BYTES = BN * 128;
    static constexpr int STAGE = A_BYTES + B_BYTES;  // a multiple of 1024 (swizzle atoms stay aligned)
    static constexpr int STAGES = BN == 256 ? 4 : BN == 128 ? 6 : (BN == 64 ? 4 : 5);
    static constexpr int SMEM = 1024 + STAGES * STAGE + 256;
};

// SwiGLU of the tensor-core epilogues (Kernels.metal:202-210 rounding points): the accumulation
// order already differs from the exact path here, so the sigmoid takes the multi-function unit's
// exponential and reciprocal (a few ulps of fp32, far below the bf16 roundings that follow).
__device__ __forceinline__ float swiglu(float g, float u) {
    const float gq = rbf(g), uq = rbf(u);
    return rbf(rbf(__fdividef(gq, 1.0f + __expf(-gq))) * uq);
}

template <int BN, int MODE>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_gemm_tc(GemvArgs a, const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw, int splits,
              int* error) {
    pdl_enter();
    using T = TcTile<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + T::STAGES * T::STAGE);
    uint64_t* empty = full + T::STAGES;
    uint64_t* done = empty + T::STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    int* stop = reinterpret_cast<int*>(tmem_slot + 1);

    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int M = a.lin.M, Mout = MODE == GEMV_SWIGLU ? M / 2 : M;
    const int per = MODE == GEMV_SWIGLU ? TC_BM / 2 : TC_BM;
    const int nn = (a.rows + BN - 1) / BN, nkb = a.lin.K / TC_BK;
    int idx = int(blockIdx.x);
    const int nt = idx % nn;
    idx /= nn;
    const int ks = idx % splits, mt = idx / splits;
    const int m0 = mt * per, n0 = nt * BN;
    const int kb0 = nkb * ks / splits, nk = nkb * (ks + 1) / splits - kb0;

    if (t == 0) {
        for (int i = 0; i < T::STAGES; i++) {
            bar_init(&full[i], 1);
            bar_init(&empty[i], 1);
        }
        bar_init(done, 1);
        *stop = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    if (warp == 0) tmem_alloc(tmem_slot, BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    int issued = 0;
    if (warp == 0) {
        if (lane == 0) {
            for (int i = 0; i < nk; i++) {
                const int s = i % T::STAGES;
                if (i >= T::STAGES && !bar_wait(&empty[s], uint32_t((i / T::STAGES) & 1) ^ 1u)) {
                    atomicCAS(error, 0, 1);
                    *stop = 1;
                    break;
                }
                uint8_t* st = smem + s * T::STAGE;
                const int kx = (kb0 + i) * TC_BK;
                bar_expect(&full[s], T::STAGE);
                if (MODE == GEMV_SWIGLU) {
                    tma2(st, &tmw, kx, m0, &full[s]);
                    tma2(st + T::A_BYTES / 2, &tmw, kx, Mout + m0, &full[s]);
                } else {
                    tma2(st, &tmw, kx, m0, &full[s]);
                }
                tma2(st + T::A_BYTES, &tmx, kx, n0, &full[s]);
                issued = i + 1;
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = tc_idesc(BN);
            for (int i = 0; i < nk; i++) {
                const int s = i % T::STAGES;
                if (!bar_wait(&full[s], uint32_t(i / T::STAGES) & 1u)) {
                    atomicCAS(error, 0, 2);
                    *stop = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t sa = smem_addr(smem + s * T::STAGE), sb = sa + T::A_BYTES;
#pragma unroll
                for (int kk = 0; kk < TC_BK / TC_UK; kk++)
                    umma_bf16(tmem, sw128_desc(sa + kk * 32), sw128_desc(sb + kk * 32), idesc, uint32_t(i | kk));
                umma_commit(&empty[s]);
            }
            umma_commit(done);  // also after an abort: the MMAs in flight finish before tensor memory is freed
        }
        __syncwarp();
    }
    __syncthreads();  // `stop` is settled
    const bool finished = __syncthreads_and(bar_wait(done, 0)) != 0;  // uniform: the epilogue has barriers
    tc_fence_after();
    if (!finished && t == 0) atomicCAS(error, 0, 3);

    if (finished && !*stop) {
        const int row = warp * 32 + lane;  // tensor-memory lane = weight row of the tile
        const uint32_t lane_base = uint32_t(warp * 32) << 16;
        // SwiGLU exchange (the stages are drained): gate values of columns 8..15 for warps 2-3,
        // up values of columns 0..7 for warps 0-1, [64][9] each
        float* xg = reinterpret_cast<float*>(smem);
        float* xu = xg + 64 * 9;
        for (int c0 = 0; c0 < BN && n0 + c0 < a.rows; c0 += 16) {
            uint32_t v[16];
            tmem_ld16(tmem + lane_base + uint32_t(c0), v);
            if (splits > 1) {
                // fp32 partials [split][row][M], by raw weight row
                int col = m0 + row;
                bool ok = col < Mout;
                if (MODE == GEMV_SWIGLU) {
                    const int i = row & 63;
                    col = (row < 64 ? 0 : Mout) + m0 + i;
                    ok = m0 + i < Mout;
                }
                if (ok) {
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const int r = n0 + c0 + j;
                        if (r < a.rows) a.part[(size_t(ks) * a.rows + r) * M + col] = __uint_as_float(v[j]);
                    }
                }
            } else if (MODE == GEMV_SWIGLU) {
                // warps 0-1 hold the gate sums and finish columns 0..7, warps 2-3 the up sums and
                // finish columns 8..15: each passes the other half of its columns across
                const bool gate = warp < 2;
                const int i = row & 63;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    if (gate) xg[i * 9 + j] = __uint_as_float(v[8 + j]);
                    else xu[i * 9 + j] = __uint_as_float(v[j]);
                }
                __syncthreads();
                if (m0 + i < Mout) {
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int col = gate ? j : 8 + j;
                        const int r = n0 + c0 + col;
                        if (r < a.rows) {
                            const int orow = a.out_map ? a.out_map[r] : r;
                            const float g = gate ? __uint_as_float(v[j]) : xg[i * 9 + j];
                            const float u = gate ? xu[i * 9 + j] : __uint_as_float(v[8 + j]);
                            a.y[size_t(orow) * a.ystride + m0 + i] = uint16_t(f2bf(swiglu(g, u)));
                        }
                    }
                }
                __syncthreads();
            } else {
                const int m = m0 + row;
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int r = n0 + c0 + j;
                    const bool rok = r < a.rows, ok = rok && m < Mout;
                    const int orow = rok ? (a.out_map ? a.out_map[r] : r) : 0;
                    const uint32_t b = f2bf(__uint_as_float(v[j]));
                    if (ok) a.y[size_t(orow) * a.ystride + m] = uint16_t(b);
                    if (MODE == GEMV_LOGITS) {
                        unsigned long long key = ok ? argmax_key(bf2f(b), uint32_t(m)) : 0ull;
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) {
                            const unsigned long long other = __shfl_xor_sync(FULL_MASK, key, o);
                            key = other > key ? other : key;
                        }
                        if (lane == 0 && rok && key) atomicMax(a.keys + orow, key);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, BN);
        // copies issued into this CTA's shared memory land before it exits (only an aborted
        // producer can leave some in flight)
        if (lane == 0)
            for (int i = issued - T::STAGES < 0 ? 0 : issued - T::STAGES; i < issued; i++)
                bar_wait(&full[i % T::STAGES], uint32_t(i / T::STAGES) & 1u);
    }
}

// Persistent form for calls with a tile for every SM and no K split (prefill): one CTA per SM walks
// the tiles (tile = m-tile * n-tiles + n-tile, so the CTAs running together share weight tiles in
// L2) with its roles in separate warps: warp 0 issues the TMA copies into a ring of stages that
// runs on across tiles, warp 1 issues the MMAs into one of two tensor-memory accumulators, and
// warps 2-5 drain the other accumulator (the previous tile) meanwhile, so a tile's epilogue no
// longer sits between two tiles' main loops. Same epilogues and results as k_gemm_tc.
constexpr int TCP_THREADS = 192;

template <int BN, int MODE>
__global__ void __launch_bounds__(TCP_THREADS, 1)
    k_gemm_tcp(GemvArgs a, const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw, int* error) {
    pdl_enter();
    using T = TcTile<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + T::STAGES * T::STAGE);
    uint64_t* empty = full + T::STAGES;
    uint64_t* tfull = empty + T::STAGES;  // [2] accumulator b holds a finished tile
    uint64_t* tempty = tfull + 2;         // [2] accumulator b was drained by the epilogue warps
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* stop = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* ep_abort = reinterpret_cast<volatile int*>(smem + T::STAGES * T::STAGE + 192);  // [2]
    float* xg = reinterpret_cast<float*>(smem + T::STAGES * T::STAGE + 256);  // SwiGLU exchange
    float* xu = xg + 64 * 9;

    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int M = a.lin.M, Mout = MODE == GEMV_SWIGLU ? M / 2 : M;
    const int per = MODE == GEMV_SWIGLU ? TC_BM / 2 : TC_BM;
    const int nn = (a.rows + BN - 1) / BN, nkb = a.lin.K / TC_BK;
    const int ntiles = ((Mout + per - 1) / per) * nn;

    if (t == 0) {
        for (int i = 0; i < T::STAGES; i++) {
            bar_init(&full[i], 1);
            bar_init(&empty[i], 1);
        }
        for (int b = 0; b < 2; b++) {
            bar_init(&tfull[b], 1);
            bar_init(&tempty[b], 4);
        }
        *stop = 0;
        ep_abort[0] = ep_abort[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    if (warp == 1) tmem_alloc(tmem_slot, 2 * BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        int issued = 0;
        if (lane == 0) {
            int g = 0;
            for (int tile = blockIdx.x; tile < ntiles && !*stop; tile += gridDim.x) {
                const int m0 = (tile / nn) * per, n0 = (tile % nn) * BN;
                for (int i = 0; i < nkb; i++, g++) {
                    const int s = g % T::STAGES;
                    if (g >= T::STAGES && !bar_wait(&empty[s], uint32_t((g / T::STAGES) & 1) ^ 1u)) {
                        atomicCAS(error, 0, 4);
                        *stop = 1;
                        break;
                    }
                    uint8_t* st = smem + s * T::STAGE;
                    const int kx = i * TC_BK;
                    bar_expect(&full[s], T::STAGE);
                    if (MODE == GEMV_SWIGLU) {
                        tma2(st, &tmw, kx, m0, &full[s]);
                        tma2(st + T::A_BYTES / 2, &tmw, kx, Mout + m0, &full[s]);
                    } else {
                        tma2(st, &tmw, kx, m0, &full[s]);
                    }
                    tma2(st + T::A_BYTES, &tmx, kx, n0, &full[s]);
                    issued = g + 1;
                }
            }
            // copies issued into this CTA's shared memory land before it exits (only an aborted
            // step leaves some unconsumed)
            for (int i = issued - T::STAGES < 0 ? 0 : issued - T::STAGES; i < issued; i++)
                bar_wait(&full[i % T::STAGES], uint32_t(i / T::STAGES) & 1u);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = tc_idesc(BN);
            int g = 0, local = 0;
            for (int tile = blockIdx.x; tile < ntiles && !*stop; tile += gridDim.x, local++) {
                const int b = local & 1;
                if (local >= 2 && !bar_wait(&tempty[b], uint32_t(((local >> 1) - 1) & 1))) {
                    atomicCAS(error, 0, 5);
                    *stop = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem + uint32_t(b * BN);
                bool ok = true;
                for (int i = 0; i < nkb; i++, g++) {
                    const int s = g % T::STAGES;
                    if (!bar_wait(&full[s], uint32_t(g / T::STAGES) & 1u)) {
                        atomicCAS(error, 0, 6);
                        *stop = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_addr(smem + s * T::STAGE), sb = sa + T::A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < TC_BK / TC_UK; kk++)
                        umma_bf16(acc, sw128_desc(sa + kk * 32), sw128_desc(sb + kk * 32), idesc, uint32_t(i | kk));
                    umma_commit(&empty[s]);
                }
                umma_commit(&tfull[b]);  // also after an abort: the epilogue waits on it, bounded
                if (!ok) break;
            }
        }
        __syncwarp();
    } else {
        // epilogue warps 2-5: tensor-memory lane quarter warp % 4, one weight row per thread
        const int q = warp & 3, row = q * 32 + lane;
        const uint32_t lane_base = uint32_t(q * 32) << 16;
        int local = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, local++) {
            const int b = local & 1;
            const bool ok = bar_wait(&tfull[b], uint32_t(local >> 1) & 1u);
            if (!ok) {
                atomicCAS(error, 0, 7);
                ep_abort[local & 1] = 1;
            }
            // the four epilogue warps take the same decision (they meet at named barriers): a slot
            // per tile parity, only ever set, read by all after the barrier below; a slot is
            // written again two tiles later, after every warp passed the next tile's barrier
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (ep_abort[local & 1]) break;
            tc_fence_after();
            const int m0 = (tile / nn) * per, n0 = (tile % nn) * BN;
            const uint32_t acc = tmem + uint32_t(b * BN);
            for (int c0 = 0; c0 < BN && n0 + c0 < a.rows; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(acc + lane_base + uint32_t(c0), v);
                if (MODE == GEMV_SWIGLU) {
                    // gate rows in lanes 0-63, up rows in 64-127: quarters 0-1 finish columns
                    // 0..7 of the 16, quarters 2-3 columns 8..15, each passing the other half
                    const bool gate = q < 2;
                    const int i = row & 63;
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        if (gate) xg[i * 9 + j] = __uint_as_float(v[8 + j]);
                        else xu[i * 9 + j] = __uint_as_float(v[j]);
                    }
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                    if (m0 + i < Mout) {
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            const int col = gate ? j : 8 + j;
                            const int r = n0 + c0 + col;
                            if (r < a.rows) {
                                const int orow = a.out_map ? a.out_map[r] : r;
                                const float gv = gate ? __uint_as_float(v[j]) : xg[i * 9 + j];
                                const float uv = gate ? xu[i * 9 + j] : __uint_as_float(v[8 + j]);
                                a.y[size_t(orow) * a.ystride + m0 + i] = uint16_t(f2bf(swiglu(gv, uv)));
                            }
                        }
                    }
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                } else {
                    const int m = m0 + row;
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const int r = n0 + c0 + j;
                        const bool rok = r < a.rows, okm = rok && m < Mout;
                        const int orow = rok ? (a.out_map ? a.out_map[r] : r) : 0;
                        const uint32_t bits = f2bf(__uint_as_float(v[j]));
                        if (okm) a.y[size_t(orow) * a.ystride + m] = uint16_t(bits);
                        if (MODE == GEMV_LOGITS) {
                            unsigned long long key = okm ? argmax_key(bf2f(bits), uint32_t(m)) : 0ull;
#pragma unroll
                            for (int o = 16; o > 0; o >>= 1) {
                                const unsigned long long other = __shfl_xor_sync(FULL_MASK, key, o);
                                key = other > key ? other : key;
                            }
                            if (lane == 0 && rok && key) atomicMax(a.keys + orow, key);
                        }
                    }
                }
            }
            // this accumulator is drained: the MMA warp may reuse it (one arrival per warp)
            tc_fence_before();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(&tempty[b])) : "memory");
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * BN);
    }
}

// Adds the split partials of one output in split order and applies the mode's epilogue. Every
// split's partial is loaded before the first add, so the sum costs one memory round trip.
template <int MODE>
__global__ void __launch_bounds__(256) k_gemm_tc_finish(GemvArgs a, int splits) {
    pdl_enter();
    const int r = int(blockIdx.y), m = int(blockIdx.x) * 256 + int(threadIdx.x);
    const int M = a.lin.M, Mout = MODE == GEMV_SWIGLU ? M / 2 : M;
    const size_t sstride = size_t(a.rows) * M;
    const float* p = a.part + size_t(r) * M;
    const int orow = a.out_map ? a.out_map[r] : r;
    unsigned long long key = 0ull;
    if (m < Mout) {
        float pv[TC_SPLITS_MAX], pu[TC_SPLITS_MAX];
#pragma unroll
        for (int s = 0; s < TC_SPLITS_MAX; s++) {
            if (s < splits) {
                pv[s] = p[s * sstride + m];
                if (MODE == GEMV_SWIGLU) pu[s] = p[s * sstride + Mout + m];
            }
        }
        float v = pv[0];
#pragma unroll
        for (int s = 1; s < TC_SPLITS_MAX; s++)
            if (s < splits) v = v + pv[s];
        if (MODE == GEMV_SWIGLU) {
            float u = pu[0];
#pragma unroll
            for (int s = 1; s < TC_SPLITS_MAX; s++)
                if (s < splits) u = u + pu[s];
            a.y[size_t(orow) * a.ystride + m] = uint16_t(f2bf(swiglu(v, u)));
        } else {
            const uint32_t b = f2bf(v);
            a.y[size_t(orow) * a.ystride + m] = uint16_t(b);
            if (MODE == GEMV_LOGITS) key = argmax_key(bf2f(b), uint32_t(m));
        }
    }
    if (MODE == GEMV_LOGITS) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(FULL_MASK, key, o);
            key = other > key ? other : key;
        }
        if ((threadIdx.x & 31) == 0 && key) atomicMax(a.keys + orow, key);
    }
}

// [rows][K] bf16 row-major as a 2-D tensor map: box of 64 k x box_rows rows, 128-byte swizzle,
// rows past the matrix read as zeros.
bool encode_kmajor(CUtensorMap* map, const void* base, int rows, int K, int box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode || K % TC_BK || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
    const cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
    const cuuint64_t strides[1] = {cuuint64_t(K) * 2};
    const cuuint32_t box[2] = {TC_BK, cuuint32_t(box_rows)};
    const cuuint32_t unit[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, unit,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct TcDevice {
    int sms = 0;
    int* error = nullptr;  // the device's tiled-GEMM error word (gemm.cu)
};

TcDevice* tc_device() {
    static TcDevice dev[64];
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 64) return nullptr;
    TcDevice& t = dev[d];
    if (!t.sms) {
        t.error = gemm_error_word(true);
        if (!t.error || cudaDeviceGetAttribute(&t.sms, cudaDevAttrMultiProcessorCount, d) != cudaSuccess) {
            t.sms = 0;
            return nullptr;
        }
    }
    return &t;
}

// PLAMO_TC_PERSISTENT=0 in the environment keeps every call on the one-tile-per-CTA kernel (A/B runs).
bool tcp_enabled() {
    static const bool on = [] {
        const char* e = getenv("PLAMO_TC_PERSISTENT");
        return !(e && e[0] == '0');
    }();
    return on;
}

// PLAMO_TC_BN256=0 in the environment keeps the persistent kernel at 128-row tiles (A/B runs).
bool bn256_enabled() {
    static const bool on = [] {
        const char* e = getenv("PLAMO_TC_BN256");
        return !(e && e[0] == '0');
    }();
    return on;
}

template <int BN, int MODE>
cudaError_t tc_launch(const GemvArgs& a, int splits, int tiles, TcDevice& dev, cudaStream_t s) {
    CUtensorMap tmx, tmw;
    if (!encode_kmajor(&tmx, a.x, a.rows, a.lin.K, BN) ||
        !encode_kmajor(&tmw, a.lin.w, a.lin.M, a.lin.K, MODE == GEMV_SWIGLU ? TC_BM / 2 : TC_BM))
        return cudaErrorInvalidValue;
    if (splits == 1 && tiles > dev.sms && BN >= 128 && tcp_enabled()) {  // persistent: more tiles than SMs
        return pdl_launch(k_gemm_tcp<BN, MODE>, dim3(dev.sms), dim3(TCP_THREADS), TcTile<BN>::SMEM + 5120, s, a, tmx,
                          tmw, dev.error);
    }
    cudaError_t e = pdl_launch(k_gemm_tc<BN, MODE>, dim3(tiles * splits), dim3(TC_THREADS), TcTile<BN>::SMEM, s, a, tmx,
                               tmw, splits, dev.error);
    if (e != cudaSuccess || splits == 1) return e;
    if (MODE == GEMV_PLAIN && a.split_out && !a.out_map) {  // the next kernel adds the partials
        *a.split_out = splits;
        return cudaSuccess;
    }
    const int Mout = MODE == GEMV_SWIGLU ? a.lin.M / 2 : a.lin.M;
    return pdl_launch(k_gemm_tc_finish<MODE>, dim3((Mout + 255) / 256, a.rows), dim3(256), 0, s, a, splits);
}

template <int BN>
cudaError_t tc_mode(const GemvArgs& a, GemvMode mode, int splits, int tiles, TcDevice& dev, cudaStream_t s) {
    switch (mode) {
        case GEMV_PLAIN: return tc_launch<BN, GEMV_PLAIN>(a, splits, tiles, dev, s);
        case GEMV_SWIGLU: return tc_launch<BN, GEMV_SWIGLU>(a, splits, tiles, dev, s);
        default: return tc_launch<BN, GEMV_LOGITS>(a, splits, tiles, dev, s);
    }
}

template <int BN>
cudaError_t tc_attr() {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_tc<BN, GEMV_PLAIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcTile<BN>::SMEM);
    if (BN >= 128) {
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_gemm_tcp<BN, GEMV_PLAIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcTile<BN>::SMEM + 5120);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_gemm_tcp<BN, GEMV_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcTile<BN>::SMEM + 5120);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_gemm_tcp<BN, GEMV_LOGITS>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcTile<BN>::SMEM + 5120);
    }
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_gemm_tc<BN, GEMV_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcTile<BN>::SMEM);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_gemm_tc<BN, GEMV_LOGITS>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcTile<BN>::SMEM);
    return e;
}

}  // namespace

cudaError_t configure_gemm_tc() {
    cudaError_t e = tc_attr<32>();
    if (e == cudaSuccess) e = tc_attr<64>();
    if (e == cudaSuccess) e = tc_attr<128>();
    if (e == cudaSuccess) e = tc_attr<256>();
    return e;
}

// Raw weights, K a multiple of 64, 16-byte aligned operands (tensor maps).
bool gemm_tc_supported(const GemvArgs& a) {
    return a.lin.offsets == nullptr && a.rows >= 1 && a.lin.K >= TC_BK && a.lin.K % TC_BK == 0 && a.lin.M >= 1 &&
           (reinterpret_cast<uintptr_t>(a.lin.w) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 &&
           tensor_map_encoder() != nullptr;
}

int gemm_tc_plan(const GemvArgs& a, GemvMode mode, int sms, int* bn_out, int* tiles_out) {
    const int Mout = mode == GEMV_SWIGLU ? a.lin.M / 2 : a.lin.M;
    const int per = mode == GEMV_SWIGLU ? TC_BM / 2 : TC_BM;
    const int mtiles = (Mout + per - 1) / per, nkb = a.lin.K / TC_BK;
    int bn = a.rows <= 32 ? 32 : 64;
    if (a.rows > 64 && mtiles * ((a.rows + 127) / 128) >= sms) bn = 128;
    // 256-row activation tiles (the persistent kernel) once they too leave no SM idle: each
    // weight tile staged in shared memory then serves twice the rows (measured: down_proj over
    // 4096 rows 105 -> 83 us, qkv 45 -> 36 us)
    if (mode != GEMV_SWIGLU && a.rows >= 256 && mtiles * ((a.rows + 255) / 256) > sms && tcp_enabled() && bn256_enabled())
        bn = 256;  // (SwiGLU tiles stay at 128 rows: their epilogue, not the loads, bounds them)
    const int tiles = mtiles * ((a.rows + bn - 1) / bn);
    // A long reduction (down_proj, K = 6144) over fewer tiles than SMs: 256-row activation tiles
    // with K split over the idle SMs, so each SM streams a third of the operand bytes (measured:
    // 512 x 6144 x 1536, 34.9 -> 24.4 us; shorter K such as qkv and o_proj measured slower split)
    if (mode == GEMV_PLAIN && a.rows >= 256 && nkb >= 64 && tiles < sms && a.part && tcp_enabled() && bn256_enabled()) {
        const int t256 = mtiles * ((a.rows + 255) / 256);
        const int sp = std::min(std::min(sms / t256, TC_SPLITS_MAX), nkb / 8);
        if (sp >= 2 && size_t(sp) * a.rows * a.lin.M <= a.part_cap) {
            *bn_out = 256;
            *tiles_out = t256;
            return sp;
        }
    }
    // split K while the tiles leave SMs idle, each split keeps >= 4 stages of k, and the
    // partials fit the caller's workspace
    int splits = 1;
    while (splits * 2 <= TC_SPLITS_MAX && tiles * splits * 2 <= sms && nkb / (splits * 2) >= 4 && a.part &&
           size_t(splits) * 2 * a.rows * a.lin.M <= a.part_cap)
        splits *= 2;

    *bn_out = bn;
    *tiles_out = tiles;
    return splits;
}

cudaError_t launch_gemm_tc(const GemvArgs& a, GemvMode mode, cudaStream_t s, int splits_override) {
    if (!gemm_tc_supported(a) || (mode == GEMV_SWIGLU && a.lin.M % 2) || (mode == GEMV_LOGITS && !a.keys))
        return cudaErrorInvalidValue;
    TcDevice* dev = tc_device();
    if (!dev) return cudaErrorInvalidDevice;
    int bn = 0, tiles = 0;
    int splits = gemm_tc_plan(a, mode, dev->sms, &bn, &tiles);
    if (splits_override > 0) {
        splits = splits_override;
        if (splits > a.lin.K / TC_BK || splits > TC_SPLITS_MAX ||
            (splits > 1 && (!a.part || size_t(splits) * a.rows * a.lin.M > a.part_cap)))
            return cudaErrorInvalidValue;
    }
    switch (bn) {
        case 32: return tc_mode<32>(a, mode, splits, tiles, *dev, s);
        case 64: return tc_mode<64>(a, mode, splits, tiles, *dev, s);
        case 128: return tc_mode<128>(a, mode, splits, tiles, *dev, s);
        default: return tc_mode<256>(a, mode, splits, tiles, *dev, s);
    }
}


}  // namespace plamo
