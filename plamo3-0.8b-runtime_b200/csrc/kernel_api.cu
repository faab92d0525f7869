// Kernel-level C ABI (include/plamo_kernels.h): thin launchers over kernels.cu on caller-owned
// device buffers.
#include "../../include/plamo_kernels.h"
#include "common.cuh"
#include "kernels.h"

#include <mutex>
#include <string>

namespace plamo {
extern thread_local std::string g_error;
}
using namespace plamo;

static int kfail(cudaError_t e) {
    g_error = std::string("CUDA error: ") + cudaGetErrorString(e);
    return 1;
}

static bool configured() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    static std::mutex mu;
    static bool done[64] = {false};
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64) return false;
    if (!done[dev]) done[dev] = configure_kernels() == cudaSuccess;
    return done[dev];
}

namespace {
__global__ void k_exp(const float* x, float* y, long long n) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = pexp(x[i]);
}

// Writes the row descriptor and window geometry of a single attention row into device memory;
// they travel as kernel parameters, so no host buffer has to outlive the call.
__global__ void k_set_attention_row(RowDesc* desc, RowGeo* geo, RowDesc d, RowGeo g) {
    *desc = d;
    *geo = g;
}

__global__ void k_keys_to_index(const unsigned long long* keys, int rows, uint32_t* out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < rows) {
        const unsigned long long k = keys[r];
        out[r] = k == 0ull ? 0xffffffffu : 0xffffffffu - uint32_t(k & 0xffffffffull);
    }
}
}  // namespace

extern "C" {

int plamo_k_linear(const void* w, const uint32_t* offsets, const uint16_t* x, int rows, int K, int M, int mode,
                   uint16_t* y, uint64_t* argmax_keys, void* stream) {
    if (!w || !x || !y || rows < 1 || K < 128 || K % 128 || M < 1 || mode < 0 || mode > 2 ||
        (mode == 1 && M % 2) || (mode == 2 && !argmax_keys)) {
        g_error = "Invalid linear arguments";
        return 1;
    }
    if (!configured()) { g_error = "Cannot configure kernels"; return 1; }
    GemvArgs a;
    a.lin.w = static_cast<const uint8_t*>(w);
    a.lin.offsets = offsets;
    a.lin.M = M;
    a.lin.K = K;
    a.x = x;
    a.rows = rows;
    a.y = y;
    a.ystride = mode == 1 ? M / 2 : M;
    a.keys = reinterpret_cast<unsigned long long*>(argmax_keys);
    cudaError_t e = launch_gemv(a, mode, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? 0 : kfail(e);
}

int plamo_k_linear_tc(const void* w, const uint16_t* x, int rows, int K, int M, int mode, uint16_t* y,
                      uint64_t* argmax_keys, int splits, float* workspace, size_t workspace_floats, void* stream) {
    if (!w || !x || !y || rows < 1 || K < 64 || K % 64 || M < 1 || mode < 0 || mode > 2 || (mode == 1 && M % 2) ||
        (mode == 2 && !argmax_keys) || splits < 0 || splits > 16 || splits > K / 64 ||
        (splits > 1 && (!workspace || size_t(splits) * rows * M > workspace_floats))) {
        g_error = "Invalid linear arguments";
        return 1;
    }
    if (!configured()) { g_error = "Cannot configure kernels"; return 1; }
    GemvArgs a;
    a.lin.w = static_cast<const uint8_t*>(w);
    a.lin.M = M;
    a.lin.K = K;
    a.x = x;
    a.rows = rows;
    a.y = y;
    a.ystride = mode == 1 ? M / 2 : M;
    a.keys = reinterpret_cast<unsigned long long*>(argmax_keys);
    a.part = workspace;
    a.part_cap = workspace ? workspace_floats : 0;
    cudaError_t e = launch_gemm_tc(a, GemvMode(mode), static_cast<cudaStream_t>(stream), splits);
    return e == cudaSuccess ? 0 : kfail(e);
}

int plamo_k_select(const uint16_t* logits, int V, const int32_t* history, int n, float penalty, int no_repeat_ngram,
                   float frequency, float presence, int32_t* counts, uint8_t* flags, uint64_t* key_out, void* stream) {
    if (!logits || V < 1 || n < 0 || (n > 0 && !history) || !counts || !flags || !key_out) {
        g_error = "Invalid select arguments";
        return 1;
    }
    cudaError_t e = launch_select(logits, V, history, n, penalty, no_repeat_ngram, frequency, presence, counts, flags,
                                  reinterpret_cast<unsigned long long*>(key_out), static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? 0 : kfail(e);
}

int plamo_k_exp(const float* x, float* y, long long n, void* stream) {
    if (!x || !y || n < 1) { g_error = "Invalid exp arguments"; return 1; }
    k_exp<<<unsigned((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : kfail(e);
}

int plamo_k_argmax_keys(const uint64_t* keys, int rows, uint32_t* out, void* stream) {
    if (!keys || !out || rows < 1) { g_error = "Invalid arguments"; return 1; }
    k_keys_to_index<<<(rows + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const unsigned long long*>(keys), rows, out);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : kfail(e);
}

int plamo_k_norm(const uint16_t* w, const uint16_t* src, uint16_t* x, int rows, int n, float offset, int residual,
                 const uint16_t* next_w, uint16_t* next, void* stream) {
    if (!w || !src || !x || rows < 1 || n < 1 || n > 4096 || (next_w && !next) || (next_w && !residual)) {
        g_error = "Invalid norm arguments";
        return 1;
    }
    NormArgs a;
    a.w = w; a.src = src; a.x = x; a.next_w = next_w; a.next = next; a.rows = rows; a.n = n; a.offset = offset;
    a.residual = residual;
    cudaError_t e = launch_norm(a, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? 0 : kfail(e);
}

int plamo_k_argmax(const uint16_t* logits, int rows, int n, uint64_t* scratch, uint32_t* out, void* stream) {
    if (!logits || !scratch || !out || rows < 1 || n < 1) { g_error = "Invalid argmax arguments"; return 1; }
    cudaError_t e = launch_argmax(logits, rows, n, reinterpret_cast<unsigned long long*>(scratch), out,
                                  static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? 0 : kfail(e);
}

int plamo_k_packed_decode(const uint8_t* data, const uint32_t* entries, long long count, uint16_t* out, void* stream) {
    if (!data || !entries || !out || count < 16 || count % 16) { g_error = "Invalid decode arguments"; return 1; }
    cudaError_t e = launch_packed_decode(data, entries, count, out, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? 0 : kfail(e);
}

int plamo_k_attention_rows(const uint16_t* q, const uint16_t* keys, const uint16_t* values, int heads, int kv_heads,
                           int cap, const int32_t* geo, int rows, int full, const uint32_t* rope_local, int splits,
                           int tensor, uint16_t* out, void* workspace, size_t workspace_bytes, void* stream) {
    if (!q || !keys || !values || !geo || !out || !workspace || rows < 1 || heads < 1 || heads > 32 || kv_heads < 1 ||
        heads % kv_heads || cap < 1 || (!full && !rope_local) || tensor < 0 || tensor > 2 ||
        (tensor != 1 && (splits < 1 || splits > 4096))) {
        g_error = "Invalid attention arguments";
        return 1;
    }
    if (!configured()) { g_error = "Cannot configure kernels"; return 1; }
    AttnArgs a;
    a.q = q; a.keys = keys; a.values = values; a.geo = reinterpret_cast<const RowGeo*>(geo); a.rope_local = rope_local;
    a.out = out; a.lane_stride = 0; a.rows = rows; a.H = heads; a.KV = kv_heads; a.cap = cap; a.full = full;
    a.splits = tensor == 1 ? attention_tc_splits(cap) : splits;
    a.per_max = attention_per_max(cap, a.splits);
    if (tensor == 1 && !attention_tc_supported(a)) {
        g_error = "The tensor-core attention takes 16 query heads over one KV head";
        return 1;
    }
    if (!tensor && attention_smem(heads, kv_heads, a.per_max) > 200 * 1024) { g_error = "Too few attention splits"; return 1; }
    const size_t desc_b = (size_t(rows) * sizeof(RowDesc) + 255) & ~size_t(255);
    const size_t po_b = (size_t(rows) * a.splits * heads * 128 * sizeof(float) + 255) & ~size_t(255);
    const size_t need = desc_b + po_b + size_t(rows) * a.splits * heads * sizeof(float2);
    if (workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255)) {
        g_error = "Attention workspace too small or not 256-byte aligned: " + std::to_string(need) + " bytes needed";
        return 1;
    }
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(ws, 0, desc_b, s);  // every row in lane 0
    if (e != cudaSuccess) return kfail(e);
    a.desc = reinterpret_cast<const RowDesc*>(ws);
    a.part_o = reinterpret_cast<float*>(ws + desc_b);
    a.part_ml = reinterpret_cast<float2*>(ws + desc_b + po_b);
    if (tensor == 2 && !attention_mma_supported(a)) {
        g_error = "The tensor-core decode-row attention takes 16 query heads over one KV head";
        return 1;
    }
    e = tensor == 1 ? launch_attention_tc(a, s) : tensor == 2 ? launch_attention_mma(a, s) : launch_attention(a, s);
    return e == cudaSuccess ? 0 : kfail(e);
}

// Library-owned scratch for plamo_k_attention (per device, grown on demand, freed at exit).
struct AttnScratch {
    void* base = nullptr;
    size_t bytes = 0;
};
static AttnScratch g_attn_scratch[64];
static std::mutex g_attn_mu;

int plamo_k_attention(const uint16_t* q, const uint16_t* keys, const uint16_t* values, int heads, int kv_heads,
                      int cap, int first, int count, int begin, int end, int full, const uint32_t* rope_local,
                      int splits, uint16_t* out, void* stream) {
    if (!q || !keys || !values || !out || heads < 1 || heads > 32 || kv_heads < 1 || heads % kv_heads || cap < 1 ||
        first < 0 || count < 1 || count > cap || begin < 0 || end > count || begin >= end || splits < 1 ||
        splits > 4096 || (!full && !rope_local)) {
        g_error = "Invalid attention arguments";
        return 1;
    }
    if (!configured()) { g_error = "Cannot configure kernels"; return 1; }
    int dev = 0;
    cudaGetDevice(&dev);
    const int per_max = attention_per_max(count, splits);
    if (attention_smem(heads, kv_heads, per_max) > 200 * 1024) { g_error = "Too few attention splits"; return 1; }
    // scratch: RowDesc + RowGeo + partial outputs + (max, sum) statistics
    const size_t part_o = size_t(splits) * heads * 128 * sizeof(float);
    const size_t part_ml = size_t(splits) * heads * sizeof(float2);
    const size_t need = 256 + part_o + part_ml;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    std::lock_guard<std::mutex> lock(g_attn_mu);
    AttnScratch& sc = g_attn_scratch[dev & 63];
    if (sc.bytes < need) {
        if (sc.base) { cudaStreamSynchronize(s); cudaFree(sc.base); sc.base = nullptr; sc.bytes = 0; }
        cudaError_t e = cudaMalloc(&sc.base, need);
        if (e != cudaSuccess) return kfail(e);
        sc.bytes = need;
    }
    uint8_t* base = static_cast<uint8_t*>(sc.base);
    RowDesc* desc = reinterpret_cast<RowDesc*>(base);
    RowGeo* geo = reinterpret_cast<RowGeo*>(base + 64);
    const RowDesc hd{0, 0, 0, 1};
    const RowGeo hg{first, count, begin, end};
    cudaError_t e = cudaMemcpyAsync(desc, &hd, sizeof(hd), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(geo, &hg, sizeof(hg), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return kfail(e);
    AttnArgs a;
    a.q = q; a.keys = keys; a.values = values; a.desc = desc; a.geo = geo; a.rope_local = rope_local;
    a.part_o = reinterpret_cast<float*>(base + 256);
    a.part_ml = reinterpret_cast<float2*>(base + 256 + part_o);
    a.out = out; a.lane_stride = 0; a.rows = 1; a.H = heads; a.KV = kv_heads; a.cap = cap; a.full = full;
    a.splits = splits; a.per_max = per_max;
    e = launch_attention(a, s);
    if (e != cudaSuccess) return kfail(e);
    // the host-side descriptors must outlive the async copies
    e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? 0 : kfail(e);
}

// Fixed device scratch of plamo_k_attention_static: a file-scope device array (every device has
// its own instance), found once per device with cudaGetSymbolAddress, shared by all calls on the
// device. Layout: RowDesc at 0, RowGeo at 64, partial outputs at 256, then the (max, sum) pairs.
// The looked-up address stays valid while the device's primary context lives; a cudaDeviceReset
// would reload the module elsewhere, which is why the header rules out calls after a reset.
constexpr size_t STATIC_ATTN_BYTES = size_t(2) << 20;
static __device__ __align__(256) unsigned char g_attn_static[STATIC_ATTN_BYTES];
static void* g_attn_static_ptr[64];
static std::mutex g_attn_static_mu;

int plamo_k_attention_static(const uint16_t* q, const uint16_t* keys, const uint16_t* values, int heads, int kv_heads,
                             int cap, int first, int count, int begin, int end, int full, const uint32_t* rope_local,
                             int splits, uint16_t* out, void* stream) {
    if (!q || !keys || !values || !out || heads < 1 || heads > 32 || kv_heads < 1 || heads % kv_heads || cap < 1 ||
        first < 0 || count < 1 || count > cap || begin < 0 || end > count || begin >= end || splits < 1 ||
        splits > 4096 || (!full && !rope_local)) {
        g_error = "Invalid attention arguments";
        return 1;
    }
    const int per_max = attention_per_max(count, splits);
    if (attention_smem(heads, kv_heads, per_max) > 200 * 1024) { g_error = "Too few attention splits"; return 1; }
    const size_t part_o = size_t(splits) * heads * 128 * sizeof(float);
    const size_t part_ml = size_t(splits) * heads * sizeof(float2);
    if (256 + part_o + part_ml > STATIC_ATTN_BYTES) {
        g_error = "Attention scratch exceeds the static 2 MiB buffer: splits x heads must be at most " +
                  std::to_string((STATIC_ATTN_BYTES - 256) / (128 * sizeof(float) + sizeof(float2)));
        return 1;
    }
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return kfail(e);
    if (dev < 0 || dev >= 64) { g_error = "Device ordinal out of range"; return 1; }
    if (!configured()) { g_error = "Cannot configure kernels"; return 1; }
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_attn_static_mu);
        if (!g_attn_static_ptr[dev]) {
            void* p = nullptr;
            e = cudaGetSymbolAddress(&p, g_attn_static);
            if (e != cudaSuccess) return kfail(e);
            g_attn_static_ptr[dev] = p;
        }
        scratch = g_attn_static_ptr[dev];
    }
    uint8_t* base = static_cast<uint8_t*>(scratch);
    RowDesc* desc = reinterpret_cast<RowDesc*>(base);
    RowGeo* geo = reinterpret_cast<RowGeo*>(base + 64);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // every statistic the merge reads is written by the partial kernel of the same call (splits
    // without visible keys write (-inf, 0) and their stale partial outputs are skipped), so the
    // previous call's contents need no clearing
    k_set_attention_row<<<1, 1, 0, s>>>(desc, geo, RowDesc{0, 0, 0, 1}, RowGeo{first, count, begin, end});
    e = cudaGetLastError();
    if (e != cudaSuccess) return kfail(e);
    AttnArgs a;
    a.q = q; a.keys = keys; a.values = values; a.desc = desc; a.geo = geo; a.rope_local = rope_local;
    a.part_o = reinterpret_cast<float*>(base + 256);
    a.part_ml = reinterpret_cast<float2*>(base + 256 + part_o);
    a.out = out; a.lane_stride = 0; a.rows = 1; a.H = heads; a.KV = kv_heads; a.cap = cap; a.full = full;
    a.splits = splits; a.per_max = per_max;
    e = launch_attention(a, s);
    return e == cudaSuccess ? 0 : kfail(e);
}

}  // extern "C"
