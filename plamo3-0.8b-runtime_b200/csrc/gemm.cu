// Order-exact GEMM for many activation rows (batched decode lanes, wide prefill): the same sums
// as k_gemv, bit for bit, with each weight tile read once per 32 activation rows instead of once
// per 16.
//
// The GEMV sums a weight row against an activation row as 32 lane partials. Lane l owns the
// weights [g*512 + 16l, +16) of every 512-weight group g and keeps two fma chains (even / odd
// elements) per 1536-weight segment, folding each segment's sum into its running total in order.
// The lane partials are then combined by the xor butterfly (pairs 16 apart, then 8, 4, 2, 1).
// Here warp lane l plays GEMV lane l for a whole tile of outputs: a tile is 32 activation rows x
// 8 weight rows (SwiGLU: 4 gate + 4 up rows), each warp 4 rows x 8 weights, so every thread keeps
// 32 outputs' chains in registers. One persistent CTA per SM walks its tiles group by group (512
// weights of the tile's rows). Each (tile, group) work item arrives by TMA tensor copies
// (activations [32 rows][8][64], weights [8 rows][8][64], 128-byte swizzle) into one of NSTAGE
// 1024-byte aligned stages, completing on the stage's mbarrier; one thread issues them
// NSTAGE - 1 items ahead. Reads undo the swizzle (16-byte chunk c of 128-byte line L sits at
// c ^ (L & 7)), which keeps every warp's 16-byte reads on distinct banks. At a tile's end the 32
// lane partials of each output meet in shared memory and one thread sums them in the butterfly's
// tree order.
#include "common.cuh"
#include "kernels.h"
#include "mbarrier.cuh"

#include <mutex>

namespace plamo {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    cudaGetLastError();
    return fn;
}

// [rows][K/64][64] bf16 view of a row-major [rows][K] matrix, box (64, lines, box_rows), 128-byte
// swizzle; rows or lines past the matrix read as zeros.
bool encode_rows_map(CUtensorMap* map, const void* base, int rows, int K, int lines, int box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode || K % 64 || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
    const cuuint64_t dims[3] = {64, cuuint64_t(K / 64), cuuint64_t(rows)};
    const cuuint64_t strides[2] = {128, cuuint64_t(K) * 2};
    const cuuint32_t box[3] = {64, cuuint32_t(lines), cuuint32_t(box_rows)};
    const cuuint32_t unit[3] = {1, 1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, unit,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// One error word per device shared by the tiled GEMMs (this file and gemm_tc.cu): a stage wait
// that gives up stores a non-zero code.
int* gemm_error_word(bool create) {
    static std::mutex mu;
    static int* words[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!words[dev] && create) {
        int* w = nullptr;
        if (cudaMalloc(&w, sizeof(int)) != cudaSuccess || cudaMemset(w, 0, sizeof(int)) != cudaSuccess) return nullptr;
        words[dev] = w;
    }
    return words[dev];
}

int gemm_take_error() {
    int* w = gemm_error_word(false);
    if (!w) return 0;
    int v = 0;
    if (cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (v) cudaMemset(w, 0, sizeof(int));
    return v;
}

namespace {

constexpr int TR = 32;  // activation rows per tile (4 per warp)
constexpr int TM = 8;   // weight rows per tile
constexpr int XS_BYTES = TR * 1024;
constexpr int WS_BYTES = TM * 1024;
constexpr int STAGE_BYTES = XS_BYTES + WS_BYTES;  // a multiple of 1024
constexpr int NSTAGE = 4;
constexpr int RED_STRIDE = 33;  // floats per output row of lane partials (conflict-free reads)
constexpr int RED_BYTES = 8 * 32 * RED_STRIDE * 4;
constexpr int GEMM_SMEM = 1024 + NSTAGE * STAGE_BYTES + RED_BYTES + 64;

// bf16 pair x bf16 pair into the even / odd chains (sm_100 mixed-precision fma: the same result
// as fmaf on the widened operands).
__device__ __forceinline__ void fma2(uint32_t w, uint32_t x, float& lo, float& hi) {
    asm("{\n .reg .b16 wl, wh, xl, xh;\n mov.b32 {wl, wh}, %2;\n mov.b32 {xl, xh}, %3;\n"
        " fma.rn.f32.bf16 %0, wl, xl, %0;\n fma.rn.f32.bf16 %1, wh, xh, %1;\n}"
        : "+f"(lo), "+f"(hi)
        : "r"(w), "r"(x));
}

// The 16 bf16 of lane `lane` in row r of a staged group (lines = 128-byte lines per row).
__device__ __forceinline__ void read16(const uint8_t* base, int r, int lines, int lane, uint32_t (&v)[8]) {
    const uint32_t line = uint32_t(r * lines + (lane >> 2)), c = uint32_t(lane & 3) * 2;
    const uint8_t* lb = base + size_t(line) * 128;
    const uint4 A = *reinterpret_cast<const uint4*>(lb + ((c ^ (line & 7u)) << 4));
    const uint4 B = *reinterpret_cast<const uint4*>(lb + (((c + 1u) ^ (line & 7u)) << 4));
    v[0] = A.x; v[1] = A.y; v[2] = A.z; v[3] = A.w;
    v[4] = B.x; v[5] = B.y; v[6] = B.z; v[7] = B.w;
}

template <int MODE>
__global__ void __launch_bounds__(256, 1)
    k_gemm(GemvArgs a, const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw, int* error) {
    pdl_enter();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + NSTAGE * STAGE_BYTES + RED_BYTES);
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int K = a.lin.K, G = (K + 511) >> 9, lines = K / 64 < 8 ? K / 64 : 8;
    const int Mout = MODE == GEMV_SWIGLU ? a.lin.M / 2 : a.lin.M;
    const int per = MODE == GEMV_SWIGLU ? TM / 2 : TM;
    const int nm = (Mout + per - 1) / per, nr = (a.rows + TR - 1) / TR;
    const int ntiles = nm * nr;
    const int my_tiles = int(blockIdx.x) < ntiles ? (ntiles - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;
    const int items = my_tiles * G;
    // full boxes are counted, rows and lines past the matrices included (zero-filled)
    const uint32_t item_bytes = uint32_t(TR + TM) * lines * 128;
    float* red = reinterpret_cast<float*>(smem + NSTAGE * STAGE_BYTES) + warp * 32 * RED_STRIDE;

    auto issue = [&](int item) {  // one thread
        const int tile = int(blockIdx.x) + (item / G) * int(gridDim.x), g = item % G;
        const int m0 = (tile % nm) * per, r0 = (tile / nm) * TR;
        uint8_t* xs = smem + (item % NSTAGE) * STAGE_BYTES;
        uint64_t* bar = &full[item % NSTAGE];
        bar_expect(bar, item_bytes);
        tma3(xs, &tmx, g * 8, r0, bar);
        if (MODE == GEMV_SWIGLU) {  // gate rows m0.., up rows Mout + m0..
            tma3(xs + XS_BYTES, &tmw, g * 8, m0, bar);
            tma3(xs + XS_BYTES + 4 * lines * 128, &tmw, g * 8, Mout + m0, bar);
        } else {
            tma3(xs + XS_BYTES, &tmw, g * 8, m0, bar);
        }
    };

    if (t == 0) {
        for (int i = 0; i < NSTAGE; i++) bar_init(&full[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int k = 0; k < NSTAGE - 1 && k < items; k++) issue(k);
    }
    __syncthreads();

    float a0[4][TM], a1[4][TM], tot[4][TM];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int m = 0; m < TM; m++) a0[i][m] = a1[i][m] = tot[i][m] = 0.f;

    // Stop decisions are uniform: a failed wait is shared through `stop` after the barrier that
    // ends the item, so every thread leaves the loop at the same item.
    __shared__ int stop;
    if (t == 0) stop = 0;
    __syncthreads();
    int k = 0;
    for (; k < items; k++) {
        if (t == 0 && k + NSTAGE - 1 < items) issue(k + NSTAGE - 1);  // its stage was freed at the end of k - 1
        const bool landed = bar_wait(&full[k % NSTAGE], uint32_t(k / NSTAGE) & 1u);
        if (!landed) {
            atomicCAS(error, 0, 1);
            stop = 1;
        }
        const int g = k % G;
        const uint8_t* xs = smem + (k % NSTAGE) * STAGE_BYTES;
        const uint8_t* ws = xs + XS_BYTES;
        if (landed && g * 512 + 16 * lane < K) {
            uint32_t xr[4][8];
#pragma unroll
            for (int i = 0; i < 4; i++) read16(xs, warp * 4 + i, lines, lane, xr[i]);
#pragma unroll
            for (int m = 0; m < TM; m++) {
                uint32_t wp[8];
                read16(ws, m, lines, lane, wp);
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int q = 0; q < 8; q++) fma2(wp[q], xr[i][q], a0[i][m], a1[i][m]);
            }
        }
        if (g % 3 == 2 || g == G - 1) {  // end of a 1536-weight segment
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int m = 0; m < TM; m++) {
                    tot[i][m] = tot[i][m] + (a0[i][m] + a1[i][m]);
                    a0[i][m] = 0.f;
                    a1[i][m] = 0.f;
                }
        }
        if (g == G - 1) {
            // tile done: lane partials -> shared [output (i*8+m)][lane] of this warp; lane o then
            // sums output o in the butterfly's tree order
            const int tile = int(blockIdx.x) + (k / G) * int(gridDim.x);
            const int m0 = (tile % nm) * per, r0 = (tile / nm) * TR;
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int m = 0; m < TM; m++) {
                    red[(i * TM + m) * RED_STRIDE + lane] = tot[i][m];
                    tot[i][m] = 0.f;
                }
            __syncwarp();
            const float* v = red + lane * RED_STRIDE;
            float s[16];
#pragma unroll
            for (int j = 0; j < 16; j++) s[j] = v[j] + v[j + 16];
#pragma unroll
            for (int j = 0; j < 8; j++) s[j] = s[j] + s[j + 8];
#pragma unroll
            for (int j = 0; j < 4; j++) s[j] = s[j] + s[j + 4];
#pragma unroll
            for (int j = 0; j < 2; j++) s[j] = s[j] + s[j + 2];
            const float res = s[0] + s[1];
            __syncwarp();  // the partials are read before the next tile overwrites them
            const int i = lane >> 3, m = lane & 7;
            const int r = r0 + warp * 4 + i;
            const bool rok = r < a.rows;
            const int orow = rok ? (a.out_map ? a.out_map[r] : r) : 0;
            if (MODE == GEMV_SWIGLU) {
                const float u = __shfl_down_sync(FULL_MASK, res, 4);  // up row m + 4 of the same activation row
                if (m < 4 && rok && m0 + m < Mout) {
                    const float gq = rbf(res), uq = rbf(u);
                    a.y[size_t(orow) * a.ystride + m0 + m] = uint16_t(f2bf(rbf(rbf(gq / (1.0f + pexp(-gq))) * uq)));
                }
            } else {
                const bool okm = rok && m0 + m < Mout;
                const uint32_t b = f2bf(res);
                if (okm) a.y[size_t(orow) * a.ystride + m0 + m] = uint16_t(b);
                if (MODE == GEMV_LOGITS) {
                    unsigned long long key = okm ? argmax_key(bf2f(b), uint32_t(m0 + m)) : 0ull;
#pragma unroll
                    for (int o = 1; o < 8; o <<= 1) {
                        const unsigned long long other = __shfl_xor_sync(FULL_MASK, key, o);
                        key = other > key ? other : key;
                    }
                    if (m == 0 && rok && key) atomicMax(a.keys + orow, key);
                }
            }
        }
        __syncthreads();  // stage k % NSTAGE is free for item k + NSTAGE; `stop` is settled
        if (stop) break;
    }
    // every copy issued into this CTA's shared memory lands before the CTA exits (only an aborted
    // kernel can leave some in flight): items up to k + NSTAGE - 1 were issued
    if (stop && t == 0)
        for (int j = k + 1; j < items && j <= k + NSTAGE - 1; j++) bar_wait(&full[j % NSTAGE], uint32_t(j / NSTAGE) & 1u);
}

template <int MODE>
cudaError_t gemm_launch(const GemvArgs& a, cudaStream_t s) {
    const int K = a.lin.K, lines = K / 64 < 8 ? K / 64 : 8;
    const int Mout = MODE == GEMV_SWIGLU ? a.lin.M / 2 : a.lin.M;
    const int per = MODE == GEMV_SWIGLU ? TM / 2 : TM;
    CUtensorMap tmx, tmw;
    if (!encode_rows_map(&tmx, a.x, a.rows, K, lines, TR) || !encode_rows_map(&tmw, a.lin.w, a.lin.M, K, lines, per))
        return cudaErrorInvalidValue;
    const int tiles = ((Mout + per - 1) / per) * ((a.rows + TR - 1) / TR);
    static int sms[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!sms[dev & 63]) cudaDeviceGetAttribute(&sms[dev & 63], cudaDevAttrMultiProcessorCount, dev);
    int* err = gemm_error_word(true);
    if (!err) return cudaErrorMemoryAllocation;
    const int grid = tiles < sms[dev & 63] ? tiles : sms[dev & 63];  // persistent: one CTA per SM
    return pdl_launch(k_gemm<MODE>, dim3(grid), dim3(256), GEMM_SMEM, s, a, tmx, tmw, err);
}

}  // namespace

cudaError_t configure_gemm() {
    cudaError_t e = cudaFuncSetAttribute(k_gemm<GEMV_PLAIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMM_SMEM);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_gemm<GEMV_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMM_SMEM);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k_gemm<GEMV_LOGITS>, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMM_SMEM);
    return e;
}

// Raw weights, more than 16 rows, K a multiple of 128, 16-byte aligned operands (tensor maps).
bool gemm_supported(const GemvArgs& a) {
    return a.lin.offsets == nullptr && a.rows > 16 && a.lin.K % 128 == 0 && a.lin.K <= 8192 &&
           (reinterpret_cast<uintptr_t>(a.lin.w) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 &&
           tensor_map_encoder() != nullptr;
}

cudaError_t launch_gemm(const GemvArgs& a, GemvMode mode, cudaStream_t s) {
    if (!gemm_supported(a) || (mode == GEMV_SWIGLU && a.lin.M % 2)) return cudaErrorInvalidValue;
    switch (mode) {
        case GEMV_PLAIN: return gemm_launch<GEMV_PLAIN>(a, s);
        case GEMV_SWIGLU: return gemm_launch<GEMV_SWIGLU>(a, s);
        default: return gemm_launch<GEMV_LOGITS>(a, s);
    }
}

}  // namespace plamo
