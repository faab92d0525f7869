// Shared device helpers for the sm_100a kernels.
#pragma once
#include <cstdint>
#include <cstdlib>
#include <utility>
#include <cuda_runtime.h>

#define PLAMO_HD 128        // head_dim
#define PLAMO_EPS 1e-6f     // rms_norm_eps
#define PLAMO_ATTN_SCALE 0.08838834764831845f  // 1/sqrt(128), Kernels.metal:372

namespace plamo {

constexpr unsigned FULL_MASK = 0xffffffffu;

// Programmatic dependent launch. The kernels of a forward call are launched with programmatic
// stream serialization, so a kernel's launch and CTA rasterisation overlap the tail of the kernel
// before it in the stream. Each such kernel calls pdl_enter() before it touches global memory:
// the wait returns once the previous kernel has completed and its writes are visible, so the data
// dependencies are those of a plain launch; the trigger then lets the next kernel launch while
// this one runs. Without the launch attribute both instructions are no-ops.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// PLAMO_PDL=0 in the environment launches plainly (for comparison); on by default.
inline bool pdl_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("PLAMO_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

// kernel<<<grid, block, smem, s>>>(args...) with the programmatic-serialization attribute.
template <typename... KArgs, typename... Args>
inline cudaError_t pdl_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// bf16 widening and the reference's round-to-nearest-even narrowing (Kernels.metal:5-10); the
// integer form reproduces its behaviour bit for bit, NaN payloads included.
__device__ __forceinline__ float bf2f(uint32_t b) { return __uint_as_float(b << 16); }
__device__ __forceinline__ uint32_t f2bf(float x) {
    uint32_t u = __float_as_uint(x);
    return ((u + 0x7fffu + ((u >> 16) & 1u)) >> 16) & 0xffffu;
}
__device__ __forceinline__ float rbf(float x) { return bf2f(f2bf(x)); }
__device__ __forceinline__ float lo_bf(uint32_t pair) { return __uint_as_float(pair << 16); }
__device__ __forceinline__ float hi_bf(uint32_t pair) { return __uint_as_float(pair & 0xffff0000u); }

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// e^x in fp32 from IEEE operations only (so the CPU restatement reproduces it bit for bit):
// Cody-Waite reduction x = n*ln2 + r with ln2 split as 355/512 + (ln2 - 355/512), |r| <= ln2/2,
// then the degree-7 Taylor polynomial of e^r in Horner form (truncation < 6e-9 relative), scaled
// by 2^n through the exponent field (two steps at the ends of the range so subnormals round once).
__device__ __forceinline__ float pexp(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
    if (x < -103.972084045410156f) return 0.0f;
    const float n = rintf(__fmul_rn(x, 1.44269502162933349609375f));
    float r = fmaf(-n, 0.693359375f, x);
    r = fmaf(-n, -2.12194440e-4f, r);
    float p = 1.98412698e-4f;          // 1/5040
    p = fmaf(p, r, 1.38888889e-3f);    // 1/720
    p = fmaf(p, r, 8.33333377e-3f);    // 1/120
    p = fmaf(p, r, 4.16666679e-2f);    // 1/24
    p = fmaf(p, r, 1.66666672e-1f);    // 1/6
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int k = int(n);
    if (k > 127) return __fmul_rn(__fmul_rn(p, __int_as_float(254 << 23)), __int_as_float((k - 127 + 127) << 23));
    if (k < -126) return __fmul_rn(__fmul_rn(p, __int_as_float((k + 100 + 127) << 23)), __int_as_float((127 - 100) << 23));
    return __fmul_rn(p, __int_as_float((k + 127) << 23));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL_MASK, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL_MASK, v, o));
    return v;
}

// Reduces NV per-lane values across the warp in 31 shuffles (recursive halving). On return,
// lane L holds in v[0] the warp total of value index L / (32 / NV) (the top log2(NV) lane bits).
template <int NV>
__device__ __forceinline__ float warp_reduce_transposed(float (&v)[NV], int lane) {
    static_assert(NV >= 1 && NV <= 32 && (NV & (NV - 1)) == 0, "NV must be a power of two <= 32");
    int n = NV;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        if (n > 1) {
            const bool upper = lane & off;
#pragma unroll
            for (int j = 0; j < NV / 2; j++) {
                if (j < n / 2) {
                    float send = upper ? v[j] : v[j + n / 2];
                    float keep = upper ? v[j + n / 2] : v[j];
                    v[j] = keep + __shfl_xor_sync(FULL_MASK, send, off);
                }
            }
            n >>= 1;
        } else {
            v[0] += __shfl_xor_sync(FULL_MASK, v[0], off);
        }
    }
    return v[0];
}

// Total-order key for the first-index argmax of Kernels.metal:704-729: larger value wins, ties go
// to the lower index, NaN never wins (no key), -0 == +0. Key 0 means "no candidate".
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t index) {
    if (v != v) return 0ull;
    uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
    uint32_t ordered = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(ordered) << 32) | static_cast<unsigned long long>(0xffffffffu - index);
}
__device__ __forceinline__ uint32_t argmax_index(unsigned long long key) {
    return key == 0ull ? 0xffffffffu : 0xffffffffu - static_cast<uint32_t>(key & 0xffffffffull);
}

// Decodes 16 consecutive weights of one packed block into 8 bf16 pairs.
// sm: 16 sign|mantissa bytes; codes: 16 4-bit exponent codes (low nibble first); minimum: block
// minimum exponent (108..170). bits = (sm & 127) | (sm & 128) << 8 | (code == 15 ? 0 : min+code) << 7.
__device__ __forceinline__ void decode16(uint4 sm, uint2 codes, uint32_t minimum, uint32_t (&wp)[8]) {
    const uint32_t zx = ((codes.x & 0x77777777u) + 0x11111111u) & codes.x & 0x88888888u;
    const uint32_t zy = ((codes.y & 0x77777777u) + 0x11111111u) & codes.y & 0x88888888u;
    const uint32_t s[4] = {sm.x, sm.y, sm.z, sm.w};
    if ((zx | zy) == 0u) {
        // No signed-zero codes: two weights per 32-bit operation.
        const uint32_t min7 = (minimum << 7) * 0x00010001u;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t w = h ? codes.y : codes.x;
            const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                // [code(2k) | 0 | code(2k+1) | 0] as two 16-bit halves (sign-replicate gives 0x00)
                const uint32_t c2 = prmt(lo, hi, uint32_t(k) | (uint32_t(8 | k) << 4) | (uint32_t(4 + k) << 8) |
                                                     (uint32_t(8 | (4 + k)) << 12));
                const uint32_t e7 = c2 * 128u + min7;
                const uint32_t p = 2u * (k & 1);
                const uint32_t dup = prmt(s[2 * h + (k >> 1)], 0u, p | (p << 4) | ((p + 1) << 8) | ((p + 1) << 12));
                wp[4 * h + k] = (dup & 0x807F807Fu) | e7;
            }
        }
    } else {
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
            uint32_t out = 0;
#pragma unroll
            for (int q = 0; q < 2; q++) {
                const uint32_t i = e + q;
                const uint32_t b = (s[i >> 2] >> (8 * (i & 3))) & 255u;
                const uint32_t cw = i < 8 ? codes.x : codes.y;
                const uint32_t code = (cw >> (4 * (i & 7))) & 15u;
                const uint32_t ex = code == 15u ? 0u : minimum + code;
                out |= ((b & 127u) | ((b & 128u) << 8) | (ex << 7)) << (16 * q);
            }
            wp[e >> 1] = out;
        }
    }
}

// Rotate-half RoPE with a bf16 (cos, sin) pair (Kernels.metal:261-274).
__device__ __forceinline__ float rope_rotate(float x, float other, int d, uint32_t cs) {
    const float c = lo_bf(cs), s = hi_bf(cs);
    return rbf(rbf(x * c) + rbf((d < 64 ? -other : other) * s));
}

}  // namespace plamo
