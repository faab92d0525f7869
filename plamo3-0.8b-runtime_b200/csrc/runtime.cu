// Runtime / Batch orchestration behind the C ABI of include/plamo.h.
//   Runtime.init            Runtime.swift:164-286   -> plamo_open
//   Runtime.encode/forward  Runtime.swift:321-467   -> Runtime::run / plamo_forward
//   Runtime.fill/prefill    Runtime.swift:469-483   -> plamo_prefill
//   Batch.init/prefill/step Batch.swift:33-179      -> plamo_batch_*
//   decodeBatch             BatchDecode.swift:8-47  -> plamo_batch_generate
// Device layout: one weight arena (all projection weights, norms, the input embedding and the
// lm_head, 256-byte aligned; for .p12 the archive payload as is), per-layer KV caches
// ([capacity][kv_heads][128] bf16; batch slabs [lanes][capacity][kv_heads][128]), RoPE tables and
// work buffers sized for one 16-token chunk (or the batch's lane count).
#include "../../include/plamo.h"
#include "kernels.h"
#include "loader.h"
#include "mega.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <dlfcn.h>
#include <nccl.h>  // types and constants only: the library is loaded with dlopen

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <mutex>
#include <thread>
#include <set>
#include <string>
#include <utility>
#include <vector>

namespace plamo {

thread_local std::string g_error;

static int fail(const std::string& m) {
    g_error = m;
    return 1;
}
#define CK(call)                                                                                 \
    do {                                                                                         \
        cudaError_t _e = (call);                                                                 \
        if (_e != cudaSuccess) return fail(std::string("CUDA error: ") + cudaGetErrorString(_e)); \
    } while (0)

static inline uint16_t bits_of(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    return uint16_t((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
static inline float from_bits(uint16_t b) {
    uint32_t u = uint32_t(b) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

struct Layer {
    const uint16_t *pre_mixer, *post_mixer, *pre_mlp, *post_mlp, *q_norm, *k_norm;
    Linear qkv, o, gate_up, down;
    bool full;
    int cap, splits, per_max;
    uint16_t *keys = nullptr, *values = nullptr;
};

struct CacheView {
    std::vector<uint16_t*> keys, values;
    std::vector<long long> stride;
};

struct Work {
    int rows_cap = 0;
    int att_rows = 0;  // rows per attention launch (its split partials hold that many)
    long long att_row_splits = 0;  // (row, split) partial slots the buffers hold
    uint16_t *x, *h, *qkv, *q, *att, *proj, *act;
    RowGeo* geo;
    RowDesc* desc;
    int* ids;
    int* out_map;
    float* part_o;
    float2* part_ml;
    float* part_tc;         // tcgen05 GEMM split-K partials
    size_t part_tc_cap;     // floats
    RowDesc* h_desc;
    int* h_ids;
    int* h_out_map;
};

struct Outputs {
    uint16_t* logits;
    uint16_t* hidden;
    unsigned long long* keys;
    int* result;
    int* h_result;
    int n;
};

}  // namespace plamo

using namespace plamo;

struct plamo_runtime {
    int device = 0;
    cudaStream_t stream = nullptr;
    Config c;
    int context = 0, chunk = 16;
    // Local layers keep a ring of the last keys. The reference's ring holds window + 16 keys
    // (Runtime.swift:240), enough for one 16-token chunk per command buffer; that capacity
    // (local_ref_cap) sets the split-K partitions and the debug view. The physical ring here
    // (local_cap) holds window + PREFILL_CALL_ROWS keys, so one forward call can take up to that
    // many rows of a long prompt without overwriting a key an earlier row of the call still sees.
    int local_cap = 0, local_ref_cap = 0;
    bool packed = false;
    bool tensor = false;       // projections over >= 16 rows on the tcgen05 GEMM (plamo_set_tensor_gemm bit 0)
    bool tensor_attn = false;  // attention of calls over >= 16 rows on the tensor cores (bit 1)
    std::string name;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0, weight_bytes = 0;
    const uint16_t* embed = nullptr;
    const uint16_t* final_norm = nullptr;
    Linear head;
    std::vector<Layer> layers;
    uint32_t *rope_local = nullptr, *rope_global = nullptr;
    Work work{};
    Outputs out{};
    CacheView cache;
    int* chain_hist = nullptr;
    int* chain_count = nullptr;
    int chain_cap = 0;
    int position = 0, last_rows = 0, last_result = -1;
    double gpu_seconds = 0, bcast_seconds = 0;
    size_t device_bytes = 0;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cudaGraphExec_t graph = nullptr;
    int step_launches = 0;
    // persistent decode kernel (decode_mega.cu)
    bool mega = false;
    MegaArgs margs{};
    uint64_t* trace = nullptr;  // phase timeline buffer (plamo_trace_decode), allocated on first use
    int mega_grid = 0;
    size_t mega_smem = 0;
    cudaGraphExec_t mega_graph = nullptr;
    bool mega_graph_tried = false;
    std::vector<std::pair<void*, size_t>> mega_words;  // tagged exchange buffers (pointer, bytes)
    int* h_error = nullptr;
    uint32_t* unset_word = nullptr;  // plamo_debug_wait_timeout: a word nothing writes (zero)
    // plamo_select scratch, allocated on first use: counts [V], flags [V], history [sel_cap] ids
    int* sel_counts = nullptr;
    uint8_t* sel_flags = nullptr;
    int* sel_hist = nullptr;
    int* h_sel_hist = nullptr;
    unsigned long long* sel_key = nullptr;
    unsigned long long* h_sel_key = nullptr;
    int sel_cap = 0;
    std::vector<void*> allocs, host_allocs;

    template <typename T>
    int dalloc(T*& p, size_t count) {
        void* q = nullptr;
        const size_t bytes = std::max<size_t>(count * sizeof(T), 256);
        cudaError_t e = cudaMalloc(&q, bytes);
        if (e != cudaSuccess) return fail("Cannot allocate " + std::to_string(bytes) + " device bytes");
        allocs.push_back(q);
        if (cudaMemset(q, 0, bytes) != cudaSuccess) return fail("Cannot clear device memory");
        device_bytes += bytes;
        p = static_cast<T*>(q);
        return 0;
    }
    template <typename T>
    int halloc(T*& p, size_t count) {
        void* q = nullptr;
        if (cudaMallocHost(&q, std::max<size_t>(count * sizeof(T), 64)) != cudaSuccess) return fail("Cannot allocate pinned memory");
        host_allocs.push_back(q);
        p = static_cast<T*>(q);
        return 0;
    }
    ~plamo_runtime() {
        if (graph) cudaGraphExecDestroy(graph);
        if (mega_graph) cudaGraphExecDestroy(mega_graph);
        for (void* p : allocs) cudaFree(p);
        for (void* p : host_allocs) cudaFreeHost(p);
        if (e0) cudaEventDestroy(e0);
        if (e1) cudaEventDestroy(e1);
        if (stream) cudaStreamDestroy(stream);
    }
};

struct plamo_batch {
    plamo_runtime* rt = nullptr;
    int lanes = 0;
    CacheView cache;
    Work work{};
    Outputs out{};
    std::vector<int> positions;
    bool ready = false;
    double gpu_seconds = 0;
    std::vector<void*> allocs, host_allocs;
    ~plamo_batch() {
        for (void* p : allocs) cudaFree(p);
        for (void* p : host_allocs) cudaFreeHost(p);
    }
};

namespace plamo {

// Live handles: closing is idempotent and a runtime's close also closes its batches.
static std::mutex g_handles_mu;
static std::set<plamo_runtime*> g_runtimes;
static std::set<plamo_batch*> g_batches;

// ------------------------------------------------------------------------------------------------
// allocation helpers shared by runtime and batch

template <typename Owner, typename T>
static int dev_alloc(Owner& o, plamo_runtime& rt, T*& p, size_t count) {
    void* q = nullptr;
    const size_t bytes = std::max<size_t>(count * sizeof(T), 256);
    if (cudaMalloc(&q, bytes) != cudaSuccess) return fail("Cannot allocate " + std::to_string(bytes) + " device bytes");
    o.allocs.push_back(q);
    if (cudaMemset(q, 0, bytes) != cudaSuccess) return fail("Cannot clear device memory");
    rt.device_bytes += bytes;
    p = static_cast<T*>(q);
    return 0;
}
template <typename Owner, typename T>
static int pin_alloc(Owner& o, T*& p, size_t count) {
    void* q = nullptr;
    if (cudaMallocHost(&q, std::max<size_t>(count * sizeof(T), 64)) != cudaSuccess) return fail("Cannot allocate pinned memory");
    o.host_allocs.push_back(q);
    p = static_cast<T*>(q);
    return 0;
}

// Attention runs over a bounded number of rows per launch, so its split partials are sized for
// them (a wide prefill would otherwise need rows x splits x heads x 128 floats at once): as many
// rows as ATT_PART_BYTES of partials hold, and at least ATT_ROWS.
constexpr int ATT_ROWS = 64;
// Rows of one prompt a prefill call may take once the prompt overruns the local ring (the slack
// of the physical ring beyond the window).
constexpr int PREFILL_CALL_ROWS = 512;
constexpr size_t ATT_PART_BYTES = size_t(64) << 20;
// Split-K partials of the tcgen05 GEMM (8 MiB): splits of the small projections at up to a few
// dozen rows; larger calls have tiles enough for every SM and do not split.
constexpr size_t TC_PART_FLOATS = size_t(8) << 20;

template <typename Owner>
static int alloc_work(Owner& o, plamo_runtime& rt, Work& w, int rows) {
    const Config& c = rt.c;
    int max_splits = 1;
    for (const Layer& L : rt.layers) max_splits = std::max(max_splits, L.splits);
    const size_t row_part = size_t(max_splits) * c.heads * (128 * sizeof(float) + sizeof(float2));
    w.att_rows = int(std::min<size_t>(rows, std::max<size_t>(ATT_ROWS, ATT_PART_BYTES / row_part)));
    w.att_row_splits = (long long)w.att_rows * max_splits;
    const size_t R = size_t(rows), RA = size_t(w.att_rows);
    w.rows_cap = rows;
    w.part_tc_cap = TC_PART_FLOATS;
    if (dev_alloc(o, rt, w.x, R * c.d) || dev_alloc(o, rt, w.h, R * c.d) || dev_alloc(o, rt, w.qkv, R * c.qkv_rows()) ||
        dev_alloc(o, rt, w.q, R * c.q_dim()) || dev_alloc(o, rt, w.att, R * c.q_dim()) || dev_alloc(o, rt, w.proj, R * c.d) ||
        dev_alloc(o, rt, w.act, R * c.ffn) || dev_alloc(o, rt, w.geo, R) || dev_alloc(o, rt, w.desc, R) ||
        dev_alloc(o, rt, w.ids, R) || dev_alloc(o, rt, w.out_map, R) ||
        dev_alloc(o, rt, w.part_o, RA * max_splits * c.heads * 128) || dev_alloc(o, rt, w.part_ml, RA * max_splits * c.heads) ||
        dev_alloc(o, rt, w.part_tc, TC_PART_FLOATS) ||
        pin_alloc(o, w.h_desc, R) || pin_alloc(o, w.h_ids, R) || pin_alloc(o, w.h_out_map, R))
        return 1;
    return 0;
}

template <typename Owner>
static int alloc_outputs(Owner& o, plamo_runtime& rt, Outputs& out, int n) {
    out.n = n;
    if (dev_alloc(o, rt, out.logits, size_t(n) * rt.c.vocab) || dev_alloc(o, rt, out.hidden, size_t(n) * rt.c.d) ||
        dev_alloc(o, rt, out.keys, size_t(n)) || dev_alloc(o, rt, out.result, size_t(n)) || pin_alloc(o, out.h_result, size_t(n)))
        return 1;
    CK(cudaMemset(out.logits, 0, size_t(n) * rt.c.vocab * 2));
    CK(cudaMemset(out.hidden, 0, size_t(n) * rt.c.d * 2));
    CK(cudaMemset(out.result, 0, size_t(n) * 4));
    return 0;
}

// ------------------------------------------------------------------------------------------------
// RoPE tables (Kernels.metal:212-219 and :264-267): cos/sin evaluated in double on the fp32 angle,
// rounded once to fp32 and then to bf16 (the CPU restatement builds the same tables).
static void build_rope(const Config& c, const float* inv_local, const float* inv_full, int local_rows, int context,
                       std::vector<uint32_t>& local, std::vector<uint32_t>& global) {
    local.resize(size_t(local_rows) * 64);
    for (int p = 0; p < local_rows; p++)
        for (int i = 0; i < 64; i++) {
            const float phase = float(p) * inv_local[i];
            const uint16_t cb = bits_of(float(std::cos(double(phase)))), sb = bits_of(float(std::sin(double(phase))));
            local[size_t(p) * 64 + i] = uint32_t(cb) | (uint32_t(sb) << 16);
        }
    global.resize(size_t(context) * 64);
    const float mscale = 1.5545177444479562f;
    for (int p = 0; p < context; p++)
        for (int i = 0; i < 64; i++) {
            const float angle = float(p) * inv_full[i];
            const float cr = from_bits(bits_of(float(std::cos(double(angle)))));
            const float sr = from_bits(bits_of(float(std::sin(double(angle)))));
            const uint16_t cb = bits_of(cr * mscale), sb = bits_of(sr * mscale);
            global[size_t(p) * 64 + i] = uint32_t(cb) | (uint32_t(sb) << 16);
        }
    (void)c;
}

// ------------------------------------------------------------------------------------------------
// Optional per-launch timing (plamo_profile_decode): every launch is bracketed by two events and its
// device time is attributed to a kernel class.
enum KClass { K_GEMV = 0, K_QKV = 1, K_ATTN = 2, K_NORM = 3, K_HEAD = 4, K_CLASSES = 5 };
struct Profiler {
    bool on = false;
    std::vector<cudaEvent_t> ev;
    std::vector<int> cls;
    size_t used = 0;
    int launches = 0;
};
static thread_local Profiler* g_prof = nullptr;
static thread_local int g_launches = 0;

static int prof_begin(cudaStream_t s) {
    g_launches++;
    if (!g_prof || !g_prof->on) return 0;
    if (g_prof->used + 2 > g_prof->ev.size()) {
        for (int i = 0; i < 64; i++) {
            cudaEvent_t e;
            if (cudaEventCreate(&e) != cudaSuccess) return fail("Cannot create profiling events");
            g_prof->ev.push_back(e);
        }
    }
    CK(cudaEventRecord(g_prof->ev[g_prof->used], s));
    return 0;
}
static int prof_end(cudaStream_t s, int cls) {
    if (!g_prof || !g_prof->on) return 0;
    CK(cudaEventRecord(g_prof->ev[g_prof->used + 1], s));
    g_prof->cls.push_back(cls);
    g_prof->used += 2;
    return 0;
}
#define LAUNCH(cls, call)                      \
    do {                                       \
        if (prof_begin(s)) return 1;           \
        CK(call);                              \
        if (prof_end(s, cls)) return 1;        \
    } while (0)

// ------------------------------------------------------------------------------------------------
// One decoder pass over `rows` rows whose ids / descriptors / output map are already on the device.
// The head (final norm, lm_head, argmax) runs on the last `nout` rows, output row k going to slot
// out_map[k]: 1 for the scalar runtime (Runtime.swift:453-458), every row for a batched step
// (Batch.swift:163-165), the lanes' last prompt rows for a batched prefill. chain: also feed the
// argmax back as the next step's input id and advance the row descriptors (device-chained decode).
// chunked: the rows are prompt chunks (consecutive rows share a chunk and a lane), the shape the
// tensor-core attention takes; batched decode steps (one row per lane) are not.
// PLAMO_SPLIT_FINISH=1 in the environment keeps the separate split-K finish launch before the
// norms (for comparison; both give the same bits).
static bool fuse_split_sums() {
    static const bool on = [] {
        const char* v = std::getenv("PLAMO_SPLIT_FINISH");
        return !(v && v[0] == '1');
    }();
    return on;
}

// PLAMO_ATTN_MMA=0 in the environment keeps tensor mode's batched decode rows on the CUDA-core
// attention kernel (for comparison).
static bool attention_mma_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("PLAMO_ATTN_MMA");
        return !(v && v[0] == '0');
    }();
    return on;
}

static int enqueue_forward(plamo_runtime& rt, Work& w, int rows, const CacheView& cv, int nout, Outputs& o,
                           bool chain, bool chunked = false) {
    const Config& c = rt.c;
    cudaStream_t s = rt.stream;
    LAUNCH(K_NORM, launch_embed_norm(w.ids, rows, c.vocab, rt.embed, rt.layers[0].pre_mixer, c.d, w.x, w.h, nout ? o.keys : nullptr,
                                     w.out_map, nout, s));
    const float post_mlp_offset = float(1.0 / std::pow(5.0, 1.5));  // Runtime.swift:450
    // chunked calls: no row's window counts more keys than its chunk's end (host descriptors)
    int key_bound = 1;
    if (chunked)
        for (int r = 0; r < rows; r++) key_bound = std::max(key_bound, w.h_desc[r].cstart + w.h_desc[r].crows);
    GemvArgs tc;  // path selection shared by every projection of the pass
    tc.tensor = rt.tensor ? 1 : 0;
    tc.part = w.part_tc;
    tc.part_cap = w.part_tc_cap;
    for (int l = 0; l < c.layers; l++) {
        const Layer& L = rt.layers[l];
        // q/k/v, o_proj and down_proj: a tcgen05 K split leaves its partials to the kernel that
        // follows (k_qkv, the norms), which adds them in split order (the finish kernel's sums)
        // instead of a finish launch
        int qsplits = 0;
        GemvArgs g = tc;
        g.lin = L.qkv; g.x = w.h; g.rows = rows; g.y = w.qkv; g.ystride = c.qkv_rows();
        g.split_out = fuse_split_sums() ? &qsplits : nullptr;
        LAUNCH(K_GEMV, launch_gemv(g, GEMV_PLAIN, s));
        QkvArgs q;
        q.src_part = qsplits ? w.part_tc : nullptr; q.src_splits = qsplits;
        q.qkv = w.qkv; q.q_norm = L.q_norm; q.k_norm = L.k_norm; q.q = w.q; q.keys = cv.keys[l]; q.values = cv.values[l];
        q.desc = w.desc; q.geo = w.geo; q.rope_local = rt.rope_local; q.rope_global = rt.rope_global;
        q.lane_stride = cv.stride[l]; q.rows = rows; q.H = c.heads; q.KV = c.kv_heads; q.cap = L.cap; q.W = c.window;
        q.full = L.full;
        LAUNCH(K_QKV, launch_qkv(q, s));
        AttnArgs a;
        a.q = w.q; a.keys = cv.keys[l]; a.values = cv.values[l]; a.desc = w.desc; a.geo = w.geo; a.rope_local = rt.rope_local;
        a.part_o = w.part_o; a.part_ml = w.part_ml; a.out = w.att; a.lane_stride = cv.stride[l]; a.rows = rows;
        a.H = c.heads; a.KV = c.kv_heads; a.cap = L.cap; a.full = L.full; a.splits = L.splits; a.per_max = L.per_max;
        // tensor mode: rows of a prefill-like call attend on the tensor cores (attn_tc.cu)
        const bool attn_tc = rt.tensor_attn && chunked && rows >= TC_MIN_ROWS && attention_tc_supported(a);
        // tensor mode: decode rows of a batched step attend with warp-level MMAs (attn_mma.cu)
        const bool attn_mma =
            rt.tensor_attn && !chunked && rows >= TC_MIN_ROWS && attention_mma_enabled() && attention_mma_supported(a);
        // the tensor-core kernel splits each row's keys into fewer, wider splits: a launch takes as
        // many rows as the partial buffers hold at that split count
        if (attn_tc) {
            a.key_bound = std::min(L.cap, key_bound);
            a.splits = attention_tc_splits(a.key_bound);
        }
        const int per_launch = attn_tc ? int(std::max<long long>(1, w.att_row_splits / a.splits)) : w.att_rows;
        for (int r0 = 0; r0 < rows; r0 += per_launch) {
            AttnArgs b = a;
            b.rows = std::min(per_launch, rows - r0);
            b.q = w.q + size_t(r0) * c.q_dim(); b.out = w.att + size_t(r0) * c.q_dim();
            b.desc = w.desc + r0; b.geo = w.geo + r0;
            if (attn_tc) LAUNCH(K_ATTN, launch_attention_tc(b, s));
            else if (attn_mma) LAUNCH(K_ATTN, launch_attention_mma(b, s));
            else LAUNCH(K_ATTN, launch_attention(b, s));
        }
        int osplits = 0;
        g = tc;
        g.lin = L.o; g.x = w.att; g.rows = rows; g.y = w.proj; g.ystride = c.d;
        g.split_out = fuse_split_sums() ? &osplits : nullptr;
        LAUNCH(K_GEMV, launch_gemv(g, GEMV_PLAIN, s));
        NormArgs n;
        n.w = L.post_mixer; n.src = w.proj; n.x = w.x; n.next_w = L.pre_mlp; n.next = w.h; n.rows = rows; n.n = c.d;
        n.offset = 0.2f; n.residual = 1;
        n.src_part = osplits ? w.part_tc : nullptr; n.src_splits = osplits;
        LAUNCH(K_NORM, launch_norm(n, s));
        g = tc;
        g.lin = L.gate_up; g.x = w.h; g.rows = rows; g.y = w.act; g.ystride = c.ffn;
        LAUNCH(K_GEMV, launch_gemv(g, GEMV_SWIGLU, s));
        g = tc;
        g.lin = L.down; g.x = w.act; g.rows = rows; g.y = w.proj; g.ystride = c.d;
        g.split_out = fuse_split_sums() ? &osplits : nullptr;
        LAUNCH(K_GEMV, launch_gemv(g, GEMV_PLAIN, s));
        n = NormArgs();
        n.w = L.post_mlp; n.src = w.proj; n.x = w.x; n.rows = rows; n.n = c.d; n.offset = post_mlp_offset; n.residual = 1;
        n.src_part = osplits ? w.part_tc : nullptr; n.src_splits = osplits;
        if (l + 1 < c.layers) { n.next_w = rt.layers[l + 1].pre_mixer; n.next = w.h; }
        LAUNCH(K_NORM, launch_norm(n, s));
    }
    if (!nout) return 0;
    NormArgs n;
    n.w = rt.final_norm; n.src = w.x + size_t(rows - nout) * c.d; n.x = w.h; n.y2 = o.hidden; n.out_map = w.out_map;
    n.rows = nout; n.n = c.d; n.offset = 1.0f; n.residual = 0;
    LAUNCH(K_NORM, launch_norm(n, s));
    GemvArgs g = tc;
    g.lin = rt.head; g.x = w.h; g.rows = nout; g.y = o.logits; g.ystride = c.vocab; g.out_map = w.out_map; g.keys = o.keys;
    LAUNCH(K_GEMV, launch_gemv(g, GEMV_LOGITS, s));
    LAUNCH(K_HEAD, launch_finalize(o.keys, w.out_map, nout, o.result, chain ? w.ids : nullptr, chain ? w.desc : nullptr,
                                   chain ? rt.chain_hist : nullptr, chain ? rt.chain_count : nullptr, rt.chain_cap, s));
    return 0;
}

static int upload_inputs(plamo_runtime& rt, Work& w, int rows) {
    CK(cudaMemcpyAsync(w.ids, w.h_ids, sizeof(int) * rows, cudaMemcpyHostToDevice, rt.stream));
    CK(cudaMemcpyAsync(w.desc, w.h_desc, sizeof(RowDesc) * rows, cudaMemcpyHostToDevice, rt.stream));
    CK(cudaMemcpyAsync(w.out_map, w.h_out_map, sizeof(int) * rows, cudaMemcpyHostToDevice, rt.stream));
    return 0;
}

static int finish(plamo_runtime& rt, double* seconds) {
    CK(cudaEventRecord(rt.e1, rt.stream));
    cudaError_t e = cudaStreamSynchronize(rt.stream);
    if (e != cudaSuccess) return fail(std::string("CUDA execution failed: ") + cudaGetErrorString(e));
    float ms = 0;
    CK(cudaEventElapsedTime(&ms, rt.e0, rt.e1));
    *seconds += ms * 1e-3;
    return 0;
}

// After a call that may have run the tiled GEMMs (more than one row): a stage wait that gave up
// fails the call instead of returning its partial results.
static int check_gemm() {
    const int code = gemm_take_error();
    if (code) return fail("GEMM stage wait timed out (code " + std::to_string(code) + ")");
    return 0;
}

static int capture_decode_graph(plamo_runtime& rt) {
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(rt.stream, cudaStreamCaptureModeThreadLocal));
    g_launches = 0;
    const int rc = enqueue_forward(rt, rt.work, 1, rt.cache, 1, rt.out, true);
    rt.step_launches = g_launches;
    cudaError_t e = cudaStreamEndCapture(rt.stream, &g);
    if (rc) { if (g) cudaGraphDestroy(g); return rc; }
    if (e != cudaSuccess) return fail(std::string("CUDA graph capture failed: ") + cudaGetErrorString(e));
    e = cudaGraphInstantiate(&rt.graph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) { rt.graph = nullptr; return fail(std::string("CUDA graph instantiate failed: ") + cudaGetErrorString(e)); }
    return 0;
}

// Prepares the persistent decode kernel (decode_mega.cu): the phase table, the tagged exchange
// buffers and the step counter. Leaves rt.mega false when the model shape is outside the kernel's
// plan (hidden size <= 1536, one KV head, <= 16 query heads) or cooperative launch is unavailable
// (the multi-kernel path remains).
// The persistent kernel's copy of every norm vector, from the weight arena: [4l + k] = pre-mixer,
// post-mixer, pre-MLP, post-MLP of layer l; [4L] final. Taken again after a broadcast open has
// received the arena (the copy at setup saw the arena before the weights arrived).
static int copy_mega_norms(plamo_runtime& rt, const MegaArgs& a) {
    const Config& c = rt.c;
    uint16_t* tab = const_cast<uint16_t*>(a.norms);
    for (int l = 0; l < c.layers; l++) {
        const Layer& L = rt.layers[l];
        const uint16_t* src[4] = {L.pre_mixer, L.post_mixer, L.pre_mlp, L.post_mlp};
        for (int k = 0; k < 4; k++)
            CK(cudaMemcpy(tab + size_t(4 * l + k) * a.dpad, src[k], size_t(c.d) * 2, cudaMemcpyDeviceToDevice));
    }
    CK(cudaMemcpy(tab + size_t(4 * c.layers) * a.dpad, rt.final_norm, size_t(c.d) * 2, cudaMemcpyDeviceToDevice));
    return 0;
}

static int setup_mega(plamo_runtime& rt) {
    const char* env = getenv("PLAMO_PERSISTENT");
    if (env && env[0] == '0') return 0;
    const Config& c = rt.c;
    int dev = rt.device, sms = 0, coop = 0, optin = 0;
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
    CK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    if (!coop || c.d > 1536 || c.heads > 16 || c.kv_heads != 1 || c.head_dim != 128) return 0;
    if (sms < c.heads + 1) return 0;  // one merging CTA per head
    int per_max = 0, splits_max = 0;
    for (const Layer& L : rt.layers) { per_max = std::max(per_max, L.per_max); splits_max = std::max(splits_max, L.splits); }
    if (splits_max > 256) return 0;  // the merge gathers a head's split statistics in one pass
    const int kmax = std::max(std::max(c.d, c.q_dim()), c.ffn);
    const int nphases = 5 * c.layers + 1;
    int tbl_bytes = 0;  // .p12: the largest per-CTA share of one phase's block table
    if (rt.packed) {
        auto share = [&](int rows, int K, int halves) { return ((rows + sms - 1) / sms) * (K / 128) * 4 * halves; };
        tbl_bytes = std::max({share(c.qkv_rows(), c.d, 1), share(c.d, c.q_dim(), 1), share(c.ffn, c.d, 2),
                              share(c.d, c.ffn, 1), share(c.vocab, c.d, 1)});
        tbl_bytes = (tbl_bytes + 15) & ~15;
    }
    const size_t smem = mega_smem_bytes(per_max, splits_max, kmax, nphases, c.layers, tbl_bytes);
    if (!smem || smem + 2048 > size_t(optin)) return 0;
    // split-row phases (o_proj, down_proj): a CTA's (row, segment) partials fit the fold buffer
    auto fold_ok = [&](int rows, int K) {
        return size_t((rows + sms - 1) / sms) * size_t(((K + 511) / 512 + 2) / 3) <= size_t(MEGA_FOLD_TASKS);
    };
    if (!fold_ok(c.d, c.q_dim()) || !fold_ok(c.d, c.ffn)) return 0;
    if (configure_mega(smem, rt.packed, mega_npt(c.d)) != cudaSuccess) { cudaGetLastError(); return 0; }
    std::vector<MegaPhase> phases;
    std::vector<MegaLayer> layers;
    auto weight_phase = [&](int kind, int l, const Linear& lin, int rows) -> int {
        phases.push_back(MegaPhase{kind, l, lin, rows, 0});
        return 0;
    };
    for (int l = 0; l < c.layers; l++) {
        const Layer& L = rt.layers[l];
        MegaLayer ml{L.pre_mixer, L.post_mixer, L.pre_mlp, L.post_mlp, L.q_norm, L.k_norm,
                     L.keys, L.values, L.cap, L.splits, L.per_max, L.full ? 1 : 0};
        layers.push_back(ml);
        if (weight_phase(MK_QKV, l, L.qkv, c.qkv_rows())) return 1;
        phases.push_back(MegaPhase{MK_ATT, l, Linear{}, 0, 0});
        if (weight_phase(MK_O, l, L.o, c.d) || weight_phase(MK_GU, l, L.gate_up, c.ffn) ||
            weight_phase(MK_DOWN, l, L.down, c.d))
            return 1;
    }
    if (weight_phase(MK_HEAD, c.layers, rt.head, c.vocab)) return 1;
    {  // link every phase to the next weight phase (attention phases have no weights)
        int nextw = int(phases.size());
        for (int i = int(phases.size()) - 1; i >= 0; i--) {
            phases[i].next_weight = nextw;
            if (phases[i].kind != MK_ATT) nextw = i;
        }
        rt.margs.first_weight = nextw;
    }
    MegaArgs& a = rt.margs;
    MegaPhase* dph = nullptr;
    MegaLayer* dly = nullptr;
    if (rt.dalloc(dph, phases.size()) || rt.dalloc(dly, layers.size())) return 1;
    CK(cudaMemcpy(dph, phases.data(), phases.size() * sizeof(MegaPhase), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dly, layers.data(), layers.size() * sizeof(MegaLayer), cudaMemcpyHostToDevice));
    a.phases = dph;
    a.nphases = int(phases.size());
    a.layers = dly;
    a.L = c.layers;
    a.embed = rt.embed;
    a.final_norm = rt.final_norm;
    a.rope_local = rt.rope_local;
    a.rope_global = rt.rope_global;
    a.d = c.d; a.H = c.heads; a.F = c.ffn; a.V = c.vocab; a.W = c.window;
    {  // the norm table (filled from the weight arena by copy_mega_norms)
        a.dpad = (c.d + 7) / 8 * 8;
        uint16_t* tab = nullptr;
        if (rt.dalloc(tab, size_t(4 * c.layers + 1) * a.dpad)) return 1;
        a.norms = tab;
        if (copy_mega_norms(rt, a)) return 1;
    }
    a.post_mlp_offset = float(1.0 / std::pow(5.0, 1.5));
    a.phases_packed = rt.packed;
    a.attn_per_max = per_max;
    a.splits_max = splits_max;
    a.xs_bytes = int(mega_xs_bytes(kmax));
    a.tbl_bytes = tbl_bytes;
    a.ids = rt.work.ids;
    a.desc = rt.work.desc;
    // tagged buffers start at zero: tag 0 is never current
    rt.mega_words = {{(void*)nullptr, size_t(c.qkv_rows()) * 4}, {nullptr, size_t(c.q_dim()) * 4}, {nullptr, size_t(c.d) * 4},
                     {nullptr, size_t(c.d) * 4}, {nullptr, size_t(c.ffn) * 4},
                     {nullptr, size_t(splits_max) * c.heads * 128 * 8}, {nullptr, size_t(splits_max) * c.heads * 2 * 8},
                     {nullptr, (size_t(4) * sms + c.heads + size_t(splits_max) * ((c.heads + MEGA_HG - 1) / MEGA_HG)) * 4}};
    if (rt.dalloc(a.qkv, c.qkv_rows()) || rt.dalloc(a.att, c.q_dim()) ||
        rt.dalloc(a.po, c.d) || rt.dalloc(a.pd, c.d) || rt.dalloc(a.act, c.ffn) ||
        rt.dalloc(a.part_o, size_t(splits_max) * c.heads * 128) || rt.dalloc(a.part_ml, size_t(splits_max) * c.heads * 2) ||
        rt.dalloc(a.hints, size_t(4) * sms + c.heads + size_t(splits_max) * ((c.heads + MEGA_HG - 1) / MEGA_HG)) ||
        rt.dalloc(a.step, 1) || rt.dalloc(a.ticket, 1) || rt.dalloc(a.error, 1) || rt.halloc(rt.h_error, 1))
        return 1;
    {
        void* ptrs[8] = {a.qkv, a.att, a.po, a.pd, a.act, a.part_o, a.part_ml, a.hints};
        for (int i = 0; i < 8; i++) rt.mega_words[i].first = ptrs[i];
    }
    a.logits = rt.out.logits;
    a.hidden = rt.out.hidden;
    a.amkey = rt.out.keys;
    a.result = rt.out.result;
    a.hist = rt.chain_hist;
    a.hist_count = rt.chain_count;
    a.hist_cap = rt.chain_cap;
    *rt.h_error = 0;
    if (mega_occupancy(smem, rt.packed, mega_npt(c.d)) < 1) return 0;  // a cooperative grid needs one CTA on every SM
    rt.mega_grid = sms;
    rt.mega_smem = smem;
    rt.mega = true;
    return 0;
}

// One cooperative launch of the persistent decode kernel; captured in a CUDA graph when the
// driver allows cooperative launches in graphs, launched directly otherwise.
static int mega_launch(plamo_runtime& rt) {
    if (!rt.mega_graph && !rt.mega_graph_tried) {
        rt.mega_graph_tried = true;
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(rt.stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            const cudaError_t le = launch_mega(rt.margs, rt.mega_grid, rt.mega_smem, rt.stream);
            const cudaError_t ce = cudaStreamEndCapture(rt.stream, &g);
            if (le == cudaSuccess && ce == cudaSuccess && g && cudaGraphInstantiate(&rt.mega_graph, g, 0) != cudaSuccess)
                rt.mega_graph = nullptr;
            if (g) cudaGraphDestroy(g);
            cudaGetLastError();  // a refused capture only means direct launches
        }
    }
    if (rt.mega_graph) CK(cudaGraphLaunch(rt.mega_graph, rt.stream));
    else CK(launch_mega(rt.margs, rt.mega_grid, rt.mega_smem, rt.stream));
    return 0;
}

// One batch-1 decode step whose id / descriptor are already on the device.
static int decode_step(plamo_runtime& rt) {
    if (rt.mega) return mega_launch(rt);
    if (!rt.graph && capture_decode_graph(rt)) return 1;
    CK(cudaGraphLaunch(rt.graph, rt.stream));
    return 0;
}

// Clears every tagged exchange word of the persistent kernel (tag 0 is never current). Tags repeat
// after 65535 / (L + 1) steps, and a consumer takes any word whose tag is current: a word that is
// read is normally rewritten in the same step, so a repeat cannot be mistaken for fresh data. Two
// cases break that rule, and both clear the words: an aborted step (some words of that step were
// never written) and a reset (the key splits of a shorter history go unused and become active
// again later, holding words of steps long past).
static int mega_clear_exchange(plamo_runtime& rt) {
    if (!rt.mega) return 0;
    for (const auto& w : rt.mega_words) CK(cudaMemsetAsync(w.first, 0, w.second, rt.stream));
    return 0;
}

// After a synchronised persistent-kernel step: a bounded device wait that timed out aborts the
// call with an error (and re-arms the counters), it never hangs the stream.
static int mega_check(plamo_runtime& rt) {
    if (!rt.mega || *rt.h_error == 0) return 0;
    const int code = *rt.h_error;
    *rt.h_error = 0;
    cudaMemset(rt.margs.error, 0, sizeof(int));
    cudaMemset(rt.margs.ticket, 0, sizeof(unsigned));
    cudaMemset(rt.margs.amkey, 0, sizeof(unsigned long long));
    // the aborted step left some exchange words unwritten: clear them and move every tag past it
    mega_clear_exchange(rt);
    cudaStreamSynchronize(rt.stream);
    unsigned step = 0;
    cudaMemcpy(&step, rt.margs.step, sizeof(unsigned), cudaMemcpyDeviceToHost);
    step += 1u;
    cudaMemcpy(rt.margs.step, &step, sizeof(unsigned), cudaMemcpyHostToDevice);
    return fail("decode step aborted: a bounded device wait timed out (code " + std::to_string(code) + ")");
}

// One lane's prompt for prefill_rows.
struct PrefillLane {
    const int32_t* ids;
    int len;   // prompt tokens
    int pos0;  // position of the first token (lane-relative)
    int lane;  // lane slab (0 for the scalar runtime)
    int slot;  // output slot of the lane's last token
};

// Prefills prompts in as few forward calls as the work buffers allow. Every prompt is cut into
// the reference's 16-token chunks (Runtime.swift:476-479, Batch.swift:86-101): the row
// descriptors carry each chunk's start and length, so window bases and attention partitions are
// those of a chunk-by-chunk prefill. Calls take chunks in chunk-index order across lanes; a call
// holds several chunks of one lane only when that lane's prompt cannot reuse a local ring slot
// (pos0 + len <= ring capacity). Then all of the lane's keys in the call are appended before any
// of its rows attend, and each row masks the keys after its own position, which is exactly the
// chunked computation. The rows whose logits are wanted (each lane's last prompt token) go last
// in their call, where the head runs.
static int prefill_rows(plamo_runtime& rt, Work& w, const CacheView& cv, Outputs& o, const std::vector<PrefillLane>& lanes,
                        double* seconds) {
    const int chunk = rt.chunk;
    int max_chunks = 0;
    for (const PrefillLane& L : lanes) max_chunks = std::max(max_chunks, (L.len + chunk - 1) / chunk);
    std::vector<std::pair<int, int>> units;  // (lane index, chunk start), chunk-index major
    for (int c = 0; c < max_chunks; c++)
        for (int i = 0; i < int(lanes.size()); i++)
            if (c * chunk < lanes[i].len) units.push_back({i, c * chunk});
    std::vector<int> in_call(lanes.size());  // rows of each lane in the call being built
    std::vector<std::pair<int, int>> call;
    size_t u = 0;
    while (u < units.size()) {
        std::fill(in_call.begin(), in_call.end(), 0);
        call.clear();
        int rows = 0;
        while (u < units.size()) {
            const int i = units[u].first, cn = std::min(chunk, lanes[i].len - units[u].second);
            if (rows + cn > w.rows_cap) break;
            // a lane whose prompt overruns the local ring takes at most ring - window rows per call
            if (in_call[i] && lanes[i].pos0 + lanes[i].len > rt.local_cap && in_call[i] + cn > rt.local_cap - rt.c.window)
                break;
            in_call[i] += cn;
            call.push_back(units[u++]);
            rows += cn;
        }
        int k = 0, nout = 0;
        for (int pass = 0; pass < 2; pass++)  // rows without logits first, then the output rows
            for (const auto& cu : call) {
                const PrefillLane& L = lanes[cu.first];
                const int st = cu.second, cn = std::min(chunk, L.len - st);
                for (int j = 0; j < cn; j++) {
                    const bool last = st + j == L.len - 1;
                    if (int(last) != pass) continue;
                    w.h_ids[k] = L.ids[st + j];
                    w.h_desc[k] = RowDesc{L.pos0 + st + j, L.lane, L.pos0 + st, cn};
                    k++;
                    if (last) w.h_out_map[nout++] = L.slot;
                }
            }
        if (upload_inputs(rt, w, rows)) return 1;
        CK(cudaEventRecord(rt.e0, rt.stream));
        if (enqueue_forward(rt, w, rows, cv, nout, o, false, true)) return 1;
        if (finish(rt, seconds)) return 1;
        if (rows > 1 && check_gemm()) return 1;
    }
    return 0;
}

// Runtime.encode (Runtime.swift:327-467) for the scalar cache.
static int forward_impl(plamo_runtime& rt, const int32_t* ids, int n, bool output, int32_t* next) {
    if (n < 1 || n > rt.chunk || rt.position + n > rt.context) return fail("Invalid tokens or context exhausted");
    for (int i = 0; i < n; i++)
        if (ids[i] < 0 || ids[i] >= rt.c.vocab) return fail("Invalid tokens or context exhausted");
    Work& w = rt.work;
    for (int i = 0; i < n; i++) {
        w.h_ids[i] = ids[i];
        w.h_desc[i] = RowDesc{rt.position + i, 0, rt.position, n};
        w.h_out_map[i] = 0;
    }
    if (upload_inputs(rt, w, n)) return 1;
    CK(cudaEventRecord(rt.e0, rt.stream));
    const bool step = n == 1 && output;
    if (step) {
        if (decode_step(rt)) return 1;
        if (rt.mega) CK(cudaMemcpyAsync(rt.h_error, rt.margs.error, sizeof(int), cudaMemcpyDeviceToHost, rt.stream));
    } else {
        if (enqueue_forward(rt, w, n, rt.cache, output ? 1 : 0, rt.out, false, true)) return 1;
    }
    if (output) CK(cudaMemcpyAsync(rt.out.h_result, rt.out.result, sizeof(int), cudaMemcpyDeviceToHost, rt.stream));
    if (finish(rt, &rt.gpu_seconds)) return 1;
    if (step && mega_check(rt)) return 1;
    if (!step && n > 1 && check_gemm()) return 1;
    rt.position += n;
    rt.last_rows = output ? 1 : 0;
    if (output) rt.last_result = rt.out.h_result[0];
    if (next) *next = output ? rt.out.h_result[0] : -1;
    return 0;
}

}  // namespace plamo

// ================================================================================================
// C ABI

extern "C" {

const char* plamo_last_error(void) { return plamo::g_error.c_str(); }

static int setup_runtime(plamo_runtime* rt, const ModelFiles* mf, bool upload, size_t* arena_out);

static int open_common(const char* model_dir, int context, int packed, int device, plamo_runtime** out,
                       const void* nccl_id, int rank, int world);

int plamo_open(const char* model_dir, int context, int packed, int device, plamo_runtime** out) {
    return open_common(model_dir, context, packed, device, out, nullptr, 0, 1);
}

int plamo_open_broadcast(const char* model_dir, int context, int packed, int device, const void* nccl_id, int rank,
                         int world, plamo_runtime** out) {
    if (!nccl_id || world < 1 || rank < 0 || rank >= world) return fail("Invalid broadcast arguments");
    return open_common(model_dir, context, packed, device, out, nccl_id, rank, world);
}

// --- NCCL loaded on demand (no link-time dependency; reuses an already loaded libnccl) --------
// PLAMO_NCCL_LIBRARY names the library to load first (a deployment's own NCCL build). The
// communicator is created non-blocking (ncclCommInitRankConfig, blocking = 0) and every NCCL step
// is polled with a limit (PLAMO_NCCL_TIMEOUT_MS, default 120 s): a rank that never joins, or dies
// mid-broadcast, ends the other ranks' calls with an error after the limit, and the communicator
// is aborted (which also ends its kernels in flight) instead of waiting forever.
typedef int (*nccl_get_uid_fn)(ncclUniqueId*);
typedef int (*nccl_init_rank_fn)(void**, int, ncclUniqueId, int);
typedef int (*nccl_init_config_fn)(void**, int, ncclUniqueId, int, ncclConfig_t*);
typedef int (*nccl_bcast_fn)(const void*, void*, size_t, int, int, void*, cudaStream_t);
typedef int (*nccl_comm_fn)(void*);
typedef int (*nccl_async_fn)(void*, int*);
typedef const char* (*nccl_err_fn)(int);
struct NcclApi {
    void* h = nullptr;
    nccl_get_uid_fn get_uid = nullptr;
    nccl_init_rank_fn init_rank = nullptr;
    nccl_init_config_fn init_config = nullptr;
    nccl_bcast_fn bcast = nullptr;
    nccl_comm_fn destroy = nullptr;
    nccl_comm_fn abort = nullptr;
    nccl_async_fn async_error = nullptr;
    nccl_err_fn err = nullptr;
};
static bool nccl_api(NcclApi& api) {
    static NcclApi cached;
    static bool tried = false;
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    if (!tried) {
        tried = true;
        void* h = nullptr;
        if (const char* path = std::getenv("PLAMO_NCCL_LIBRARY")) h = dlopen(path, RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (h) {
            cached.h = h;
            cached.get_uid = (nccl_get_uid_fn)dlsym(h, "ncclGetUniqueId");
            cached.init_rank = (nccl_init_rank_fn)dlsym(h, "ncclCommInitRank");
            cached.init_config = (nccl_init_config_fn)dlsym(h, "ncclCommInitRankConfig");
            cached.bcast = (nccl_bcast_fn)dlsym(h, "ncclBroadcast");
            cached.destroy = (nccl_comm_fn)dlsym(h, "ncclCommDestroy");
            cached.abort = (nccl_comm_fn)dlsym(h, "ncclCommAbort");
            cached.async_error = (nccl_async_fn)dlsym(h, "ncclCommGetAsyncError");
            cached.err = (nccl_err_fn)dlsym(h, "ncclGetErrorString");
        }
    }
    api = cached;
    return api.h && api.get_uid && api.init_rank && api.bcast && api.destroy;
}

static std::string nccl_message(const NcclApi& api, const char* what, int e) {
    return std::string(what) + " failed: " + (api.err ? api.err(e) : "?");
}

static long long nccl_limit_ms() {
    const char* v = std::getenv("PLAMO_NCCL_TIMEOUT_MS");
    const long long ms = v ? std::atoll(v) : 0;
    return ms > 0 ? ms : 120000;
}

// Polls the communicator (and, when given, the stream its work was enqueued on) until the step
// completes, fails, or the limit passes; aborts the communicator on failure or timeout. Returns 0,
// or 1 with the error set; *comm is null after an abort.
static int nccl_finish(const NcclApi& api, void** comm, cudaStream_t stream, long long limit_ms, const char* what) {
    const auto t0 = std::chrono::steady_clock::now();
    auto elapsed_ms = [&] {
        return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    };
    std::string err;
    if (api.async_error) {
        for (;;) {
            int state = ncclSuccess;
            const int e = api.async_error(*comm, &state);
            if (e != ncclSuccess) { err = nccl_message(api, what, e); break; }
            if (state == ncclSuccess) break;
            if (state != ncclInProgress) { err = nccl_message(api, what, state); break; }
            if (elapsed_ms() > limit_ms) { err = std::string(what) + " timed out after " + std::to_string(limit_ms) + " ms (a rank did not join)"; break; }
            std::this_thread::sleep_for(std::chrono::microseconds(200));
        }
    }
    while (err.empty() && stream) {
        const cudaError_t q = cudaStreamQuery(stream);
        if (q == cudaSuccess) break;
        if (q != cudaErrorNotReady) { err = std::string(what) + ": " + cudaGetErrorString(q); break; }
        if (elapsed_ms() > limit_ms) { err = std::string(what) + " timed out after " + std::to_string(limit_ms) + " ms (a rank stopped)"; break; }
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
    if (err.empty()) return 0;
    if (*comm) (api.abort ? api.abort : api.destroy)(*comm);
    *comm = nullptr;
    return fail(err);
}

// Creates the broadcast communicator: non-blocking when the library has ncclCommInitRankConfig
// (bounded by the limit), else the blocking ncclCommInitRank.
static int nccl_comm_init(const NcclApi& api, const void* nccl_id, int rank, int world, long long limit_ms, void** comm) {
    ncclUniqueId id;
    memcpy(&id, nccl_id, sizeof(id));
    *comm = nullptr;
    if (!api.init_config || !api.async_error) {
        const int e = api.init_rank(comm, world, id, rank);
        if (e) { *comm = nullptr; return fail(nccl_message(api, "ncclCommInitRank", e)); }
        return 0;
    }
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    const int e = api.init_config(comm, world, id, rank, &cfg);
    if (e != ncclSuccess && e != ncclInProgress) {
        if (*comm) (api.abort ? api.abort : api.destroy)(*comm);
        *comm = nullptr;
        return fail(nccl_message(api, "ncclCommInitRankConfig", e));
    }
    if (!*comm) return fail("ncclCommInitRankConfig returned no communicator");
    return nccl_finish(api, comm, nullptr, limit_ms, "NCCL communicator setup");
}

// One broadcast from rank 0 on `stream`, completed (or failed) within the limit.
static int nccl_broadcast(const NcclApi& api, void** comm, void* buf, size_t bytes, cudaStream_t stream, long long limit_ms) {
    const int e = api.bcast(buf, buf, bytes, /*ncclUint8*/ 1, 0, *comm, stream);
    if (e != ncclSuccess && e != ncclInProgress) {
        (api.abort ? api.abort : api.destroy)(*comm);
        *comm = nullptr;
        return fail(nccl_message(api, "ncclBroadcast", e));
    }
    return nccl_finish(api, comm, stream, limit_ms, "ncclBroadcast");
}

int plamo_nccl_unique_id(void* out) {
    NcclApi api;
    if (!out || !nccl_api(api)) return fail("NCCL is not available");
    ncclUniqueId id;
    int e = api.get_uid(&id);
    if (e) return fail(nccl_message(api, "ncclGetUniqueId", e));
    memcpy(out, &id, sizeof(id));
    return 0;
}

int plamo_debug_nccl_init(const void* nccl_id, int rank, int world, long long limit_ms) {
    NcclApi api;
    if (!nccl_id || world < 1 || rank < 0 || rank >= world || limit_ms < 1) return fail("Invalid broadcast arguments");
    if (!nccl_api(api)) return fail("NCCL is not available");
    void* comm = nullptr;
    if (nccl_comm_init(api, nccl_id, rank, world, limit_ms, &comm)) return 1;
    api.destroy(comm);
    return 0;
}

static int open_common(const char* model_dir, int context, int packed, int device, plamo_runtime** out,
                       const void* nccl_id, int rank, int world) {
    if (!out) return fail("Invalid output handle");
    *out = nullptr;
    if (context < 1 || context > 32768) return fail("Context must be 1...32768");
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) return fail("A CUDA device is required");
    CK(cudaSetDevice(device));
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10) return fail("libplamo_cuda requires an sm_100a (B200-class) device");
    auto* mf = new ModelFiles();
    std::string err;
    if (!mf->load(model_dir ? model_dir : "", packed != 0, err)) { delete mf; return fail(err); }
    auto* rt = new plamo_runtime();
    rt->device = device;
    rt->name = prop.name;
    rt->c = mf->cfg;
    rt->context = context;
    rt->packed = packed != 0;
    rt->chunk = std::min(context, 16);                                   // Runtime.swift:173
    rt->local_ref_cap = std::min(context, rt->c.window + rt->chunk);     // Runtime.swift:240
    rt->local_cap = std::min(context, rt->c.window + PREFILL_CALL_ROWS);
    int rc = configure_kernels() == cudaSuccess ? 0 : fail("Cannot configure kernels");
    if (!rc && (cudaStreamCreateWithFlags(&rt->stream, cudaStreamNonBlocking) != cudaSuccess ||
                cudaEventCreate(&rt->e0) != cudaSuccess || cudaEventCreate(&rt->e1) != cudaSuccess))
        rc = fail("Cannot create CUDA stream");
    size_t arena = 0;
    if (!rc) rc = setup_runtime(rt, mf, nccl_id == nullptr || rank == 0, &arena);
    if (!rc && nccl_id) {
        NcclApi api;
        const long long limit = nccl_limit_ms();
        if (!nccl_api(api)) rc = fail("NCCL is not available");
        void* comm = nullptr;
        if (!rc) rc = nccl_comm_init(api, nccl_id, rank, world, limit, &comm);
        // a first small broadcast sets up the communicator's channels (lazily, on first use), so
        // the timed one measures the weight transfer alone
        if (!rc) rc = nccl_broadcast(api, &comm, rt->arena, 256, rt->stream, limit);
        if (!rc) {
            auto t0 = std::chrono::steady_clock::now();
            rc = nccl_broadcast(api, &comm, rt->arena, rt->arena_bytes, rt->stream, limit);
            rt->bcast_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        }
        if (comm) api.destroy(comm);
        // state derived from the arena's contents at setup is taken again from the received weights
        if (!rc && rank > 0 && rt->mega) rc = copy_mega_norms(*rt, rt->margs);
    }
    delete mf;  // weights are resident; the mappings are no longer needed
    if (rc) { delete rt; return rc; }
    {
        std::lock_guard<std::mutex> lock(g_handles_mu);
        g_runtimes.insert(rt);
    }
    *out = rt;
    return 0;
}

// Builds the weight arena (uploading it unless another rank will broadcast it), KV caches, RoPE
// tables and work buffers.
static int setup_runtime(plamo_runtime* rt, const ModelFiles* mf, bool upload, size_t* arena_out) {
    const Config& c = rt->c;
    std::string err;
    struct Item { std::string name; std::vector<long long> shape; bool p12; TensorRef ref; size_t off; };
    std::vector<Item> items;
    auto add = [&](const std::string& name, std::vector<long long> shape, bool p12) { items.push_back({name, shape, p12, {}, 0}); };
    const long long d = c.d, V = c.vocab;
    add("model.embed_tokens.weight", {V, d}, false);
    add("lm_head.weight", {V, d}, rt->packed);
    add("model.norm.weight", {d}, rt->packed);
    for (int i = 0; i < c.layers; i++) {
        const std::string p = "model.layers.layers." + std::to_string(i) + ".";
        add(p + "pre_mixer_norm.weight", {d}, rt->packed);
        add(p + "post_mixer_norm.weight", {d}, rt->packed);
        add(p + "pre_mlp_norm.weight", {d}, rt->packed);
        add(p + "post_mlp_norm.weight", {d}, rt->packed);
        add(p + "mixer.qkv_proj.weight", {c.qkv_rows(), d}, rt->packed);
        add(p + "mixer.o_proj.weight", {d, c.q_dim()}, rt->packed);
        add(p + "mixer.q_norm.weight", {128}, rt->packed);
        add(p + "mixer.k_norm.weight", {128}, rt->packed);
        add(p + "mlp.gate_up_proj.weight", {2LL * c.ffn, d}, rt->packed);
        add(p + "mlp.down_proj.weight", {d, c.ffn}, rt->packed);
    }
    for (auto& it : items)
        if (!mf->tensor(it.name, it.shape, it.p12, it.ref, err)) return fail(err);
    // Arena layout: raw tensors each 256-byte aligned; in packed mode the whole .p12 payload (its
    // regions are already 64-byte aligned) followed by the bf16 input embedding.
    size_t off = 0;
    size_t payload_off = 0;
    if (rt->packed) { payload_off = 0; off = (mf->p12_payload + 255) & ~size_t(255); }
    for (auto& it : items) {
        if (it.p12) continue;
        it.off = off;
        off += (it.ref.bytes + 255) & ~size_t(255);
    }
    rt->arena_bytes = off;
    if (rt->dalloc(rt->arena, off)) return 1;
    if (upload) {
        // staged through a pinned buffer (pageable copies of mmapped files are slow)
        const size_t stage_bytes = size_t(64) << 20;
        uint8_t* stage = nullptr;
        if (cudaMallocHost(&stage, stage_bytes) != cudaSuccess) return fail("Cannot allocate pinned staging");
        auto copy = [&](size_t dst, const uint8_t* src, size_t bytes) -> int {
            for (size_t done = 0; done < bytes; done += stage_bytes) {
                const size_t n = std::min(stage_bytes, bytes - done);
                memcpy(stage, src + done, n);
                if (cudaMemcpy(rt->arena + dst + done, stage, n, cudaMemcpyHostToDevice) != cudaSuccess) return 1;
            }
            return 0;
        };
        int bad = 0;
        if (rt->packed) bad |= copy(payload_off, mf->p12.data + mf->p12_data_start, mf->p12_payload);
        for (auto& it : items)
            if (!it.p12) bad |= copy(it.off, it.ref.data, it.ref.bytes);
        cudaFreeHost(stage);
        if (bad) return fail("Weight upload failed");
    }
    *arena_out = off;
    rt->weight_bytes = off;
    auto ptr = [&](const Item& it) -> const uint8_t* {
        if (!it.p12) return rt->arena + it.off;
        if (it.ref.packed) return rt->arena + payload_off + it.ref.data_off;
        return rt->arena + payload_off + it.ref.raw_off;
    };
    auto lin = [&](const Item& it, int M, int K) {
        Linear l;
        l.M = M; l.K = K;
        l.w = ptr(it);
        l.offsets = it.p12 ? reinterpret_cast<const uint32_t*>(rt->arena + payload_off + it.ref.table_off) : nullptr;
        return l;
    };
    size_t k = 0;
    rt->embed = reinterpret_cast<const uint16_t*>(ptr(items[k++]));
    rt->head = lin(items[k++], c.vocab, c.d);
    rt->final_norm = reinterpret_cast<const uint16_t*>(ptr(items[k++]));
    rt->layers.resize(c.layers);
    int max_splits = 1;
    for (int i = 0; i < c.layers; i++) {
        Layer& L = rt->layers[i];
        L.pre_mixer = reinterpret_cast<const uint16_t*>(ptr(items[k++]));
        L.post_mixer = reinterpret_cast<const uint16_t*>(ptr(items[k++]));
        L.pre_mlp = reinterpret_cast<const uint16_t*>(ptr(items[k++]));
        L.post_mlp = reinterpret_cast<const uint16_t*>(ptr(items[k++]));
        L.qkv = lin(items[k++], c.qkv_rows(), c.d);
        L.o = lin(items[k++], c.d, c.q_dim());
        L.q_norm = reinterpret_cast<const uint16_t*>(ptr(items[k++]));
        L.k_norm = reinterpret_cast<const uint16_t*>(ptr(items[k++]));
        L.gate_up = lin(items[k++], 2 * c.ffn, c.d);
        L.down = lin(items[k++], c.d, c.ffn);
        L.full = c.is_global(i);
        L.cap = L.full ? rt->context : rt->local_cap;
        // split-K width: ~64 keys per split for the local window, <= 256 keys for global history,
        // from the reference's capacities (the partitions set the summation order)
        const int ref_cap = L.full ? rt->context : rt->local_ref_cap;
        L.splits = L.full ? std::max(32, (ref_cap + 255) / 256) : std::max(1, (ref_cap + 63) / 64);
        L.per_max = attention_per_max(ref_cap, L.splits);
        max_splits = std::max(max_splits, L.splits);
        const size_t n = size_t(L.cap) * c.kv_heads * 128;
        if (rt->dalloc(L.keys, n) || rt->dalloc(L.values, n)) return 1;
        CK(cudaMemset(L.keys, 0, n * 2));
        CK(cudaMemset(L.values, 0, n * 2));
        rt->cache.keys.push_back(L.keys);
        rt->cache.values.push_back(L.values);
        rt->cache.stride.push_back(0);
    }
    std::vector<uint32_t> lo, gl;
    const int local_rows = std::min(rt->context, c.window + 16);  // Runtime.swift:266 (window-relative rows)
    build_rope(c, mf->inv_local, mf->inv_full, local_rows, rt->context, lo, gl);
    if (rt->dalloc(rt->rope_local, lo.size()) || rt->dalloc(rt->rope_global, gl.size())) return 1;
    CK(cudaMemcpy(rt->rope_local, lo.data(), lo.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(rt->rope_global, gl.data(), gl.size() * 4, cudaMemcpyHostToDevice));
    // prefill calls take up to 512 rows (a 512-token prompt in one call)
    if (alloc_work(*rt, *rt, rt->work, std::max(16, std::min(rt->context, 512))) || alloc_outputs(*rt, *rt, rt->out, 1)) return 1;
    rt->chain_cap = rt->context;
    if (rt->dalloc(rt->chain_hist, size_t(rt->chain_cap)) || rt->dalloc(rt->chain_count, 1)) return 1;
    CK(cudaMemset(rt->chain_count, 0, sizeof(int)));
    return setup_mega(*rt);
}

void plamo_close(plamo_runtime* rt) {
    // Closing a runtime also closes the batches opened on it; closing an unknown or already
    // closed handle is a no-op (so finalizers may run in any order).
    std::vector<plamo_batch*> batches;
    {
        std::lock_guard<std::mutex> lock(g_handles_mu);
        if (!rt || !g_runtimes.erase(rt)) return;
        for (auto it = g_batches.begin(); it != g_batches.end();) {
            if ((*it)->rt == rt) { batches.push_back(*it); it = g_batches.erase(it); }
            else ++it;
        }
    }
    cudaSetDevice(rt->device);
    if (rt->stream) cudaStreamSynchronize(rt->stream);
    for (plamo_batch* b : batches) delete b;
    delete rt;
}

int plamo_forward(plamo_runtime* rt, const int32_t* ids, int n, int output, int32_t* next_id) {
    if (!rt || (!ids && n)) return fail("Invalid tokens or context exhausted");
    CK(cudaSetDevice(rt->device));
    return forward_impl(*rt, ids, n, output != 0, next_id);
}

int plamo_prefill(plamo_runtime* rt, const int32_t* ids, int n, int32_t* next_id) {
    if (!rt || !ids || n < 1 || rt->position + n > rt->context) return fail("Input exceeds context");  // Runtime.swift:474
    for (int i = 0; i < n; i++)
        if (ids[i] < 0 || ids[i] >= rt->c.vocab) return fail("Invalid tokens or context exhausted");  // Runtime.swift:328-330
    CK(cudaSetDevice(rt->device));
    // the prompt in 16-token chunks (Runtime.swift:476-479), as few calls as the buffers allow
    if (prefill_rows(*rt, rt->work, rt->cache, rt->out, {PrefillLane{ids, n, rt->position, 0, 0}}, &rt->gpu_seconds))
        return 1;
    CK(cudaMemcpy(rt->out.h_result, rt->out.result, sizeof(int), cudaMemcpyDeviceToHost));
    rt->position += n;
    rt->last_rows = 1;
    rt->last_result = rt->out.h_result[0];
    if (next_id) *next_id = rt->last_result;
    return 0;
}

int plamo_decode_chain(plamo_runtime* rt, int steps, int32_t* out_ids) {
    if (!rt || steps < 1 || !out_ids) return fail("Invalid decode chain arguments");
    if (rt->last_rows < 1 || rt->last_result < 0 || rt->last_result >= rt->c.vocab || rt->position + steps > rt->context)
        return fail("Invalid tokens or context exhausted");
    CK(cudaSetDevice(rt->device));
    Work& w = rt->work;
    w.h_ids[0] = rt->last_result;
    w.h_desc[0] = RowDesc{rt->position, 0, rt->position, 1};
    w.h_out_map[0] = 0;
    if (upload_inputs(*rt, w, 1)) return 1;
    CK(cudaMemsetAsync(rt->chain_count, 0, sizeof(int), rt->stream));
    if (!rt->mega && !rt->graph && capture_decode_graph(*rt)) return 1;
    CK(cudaEventRecord(rt->e0, rt->stream));
    for (int i = 0; i < steps; i++)
        if (decode_step(*rt)) return 1;
    if (rt->mega) CK(cudaMemcpyAsync(rt->h_error, rt->margs.error, sizeof(int), cudaMemcpyDeviceToHost, rt->stream));
    CK(cudaMemcpyAsync(out_ids, rt->chain_hist, sizeof(int) * steps, cudaMemcpyDeviceToHost, rt->stream));
    if (finish(*rt, &rt->gpu_seconds)) return 1;
    if (mega_check(*rt)) return 1;
    rt->position += steps;
    rt->last_rows = 1;
    rt->last_result = out_ids[steps - 1];
    rt->out.h_result[0] = rt->last_result;
    return 0;
}

int plamo_step_launches(plamo_runtime* rt) {
    if (!rt) return 0;
    if (rt->mega) return 1;
    cudaSetDevice(rt->device);
    if (!rt->graph && capture_decode_graph(*rt)) return -1;
    return rt->step_launches;
}

int plamo_persistent_decode(const plamo_runtime* rt) { return rt && rt->mega ? 1 : 0; }

// Failure path of the persistent kernel's bounded waits, run on purpose: one poll of a device word
// that nothing sets gives up after limit_ns, raises the kernel's error word, and the call fails
// the way an aborted decode step does (mega_check: message, re-armed counters, cleared exchange
// words, tags moved on). The runtime stays usable.
int plamo_debug_wait_timeout(plamo_runtime* rt, unsigned long long limit_ns) {
    if (!rt) return fail("Invalid runtime");
    if (!rt->mega) return fail("The persistent decode kernel is not active");
    if (limit_ns < 1000ull || limit_ns > 2000000000ull) return fail("Wait limit must be 1 us ... 2 s");
    CK(cudaSetDevice(rt->device));
    if (!rt->unset_word && rt->dalloc(rt->unset_word, 1)) return 1;
    CK(launch_wait_unset(rt->unset_word, rt->margs.error, limit_ns, rt->stream));
    CK(cudaMemcpyAsync(rt->h_error, rt->margs.error, sizeof(int), cudaMemcpyDeviceToHost, rt->stream));
    const cudaError_t e = cudaStreamSynchronize(rt->stream);
    if (e != cudaSuccess) return fail(std::string("CUDA execution failed: ") + cudaGetErrorString(e));
    if (mega_check(*rt)) return 1;
    return fail("The bounded wait did not time out");
}

// One device-chained decode step of the persistent kernel with its phase timeline recorded
// (launched directly, outside the captured graph, with the trace pointer set).
int plamo_trace_decode(plamo_runtime* rt, uint64_t* out, size_t cap, int32_t* shape) {
    if (!rt || !out || !shape) return fail("Invalid trace arguments");
    if (!rt->mega) return fail("The persistent decode kernel is not active");
    if (rt->last_rows < 1 || rt->position + 1 > rt->context) return fail("Invalid tokens or context exhausted");
    const size_t per = size_t(rt->margs.nphases + 1) * MEGA_TRACE_STAMPS + MEGA_TRACE_DETAIL,
                 n = per * size_t(rt->mega_grid);
    shape[0] = rt->mega_grid;
    shape[1] = rt->margs.nphases;
    shape[2] = MEGA_TRACE_STAMPS;
    shape[3] = MEGA_TRACE_DETAIL;
    if (cap < n) return fail("Trace buffer too small: " + std::to_string(n) + " entries needed");
    CK(cudaSetDevice(rt->device));
    if (!rt->trace && rt->dalloc(rt->trace, n)) return 1;
    Work& w = rt->work;
    w.h_ids[0] = rt->last_result;
    w.h_desc[0] = RowDesc{rt->position, 0, rt->position, 1};
    w.h_out_map[0] = 0;
    if (upload_inputs(*rt, w, 1)) return 1;
    CK(cudaMemsetAsync(rt->chain_count, 0, sizeof(int), rt->stream));
    CK(cudaMemsetAsync(rt->trace, 0, n * sizeof(uint64_t), rt->stream));
    MegaArgs a = rt->margs;
    a.trace = reinterpret_cast<unsigned long long*>(rt->trace);
    CK(launch_mega(a, rt->mega_grid, rt->mega_smem, rt->stream));
    CK(cudaMemcpyAsync(rt->h_error, rt->margs.error, sizeof(int), cudaMemcpyDeviceToHost, rt->stream));
    CK(cudaStreamSynchronize(rt->stream));
    if (mega_check(*rt)) return 1;
    CK(cudaMemcpy(out, rt->trace, n * sizeof(uint64_t), cudaMemcpyDeviceToHost));
    int last = 0;
    CK(cudaMemcpy(&last, rt->chain_hist, sizeof(int), cudaMemcpyDeviceToHost));
    rt->position += 1;
    rt->last_result = last;
    return 0;
}

// Runs `steps` batch-1 decode steps (same kernels as the decode graph, launched directly) with
// every launch bracketed by CUDA events; class_ms[c] / launches[c] receive the summed device time
// and launch count per kernel class (0 GEMV, 1 QK-norm/RoPE/KV, 2 attention, 3 norms, 4 argmax).
int plamo_profile_decode(plamo_runtime* rt, int steps, double* class_ms, int32_t* launches) {
    if (!rt || steps < 1 || !class_ms || !launches) return fail("Invalid profile arguments");
    if (rt->last_rows < 1 || rt->position + steps > rt->context) return fail("Invalid tokens or context exhausted");
    CK(cudaSetDevice(rt->device));
    Work& w = rt->work;
    w.h_ids[0] = rt->last_result;
    w.h_desc[0] = RowDesc{rt->position, 0, rt->position, 1};
    w.h_out_map[0] = 0;
    if (upload_inputs(*rt, w, 1)) return 1;
    CK(cudaMemsetAsync(rt->chain_count, 0, sizeof(int), rt->stream));
    for (int c = 0; c <= K_CLASSES; c++) { class_ms[c] = 0; launches[c] = 0; }
    if (rt->mega) {  // the persistent kernel is the whole step: time each launch
        std::vector<cudaEvent_t> ev(2 * size_t(steps));
        for (auto& e : ev) CK(cudaEventCreate(&e));
        int rc = 0;
        for (int i = 0; i < steps && !rc; i++) {
            cudaEventRecord(ev[2 * i], rt->stream);
            rc = mega_launch(*rt);
            cudaEventRecord(ev[2 * i + 1], rt->stream);
        }
        if (!rc) CK(cudaMemcpyAsync(rt->h_error, rt->margs.error, sizeof(int), cudaMemcpyDeviceToHost, rt->stream));
        if (!rc && cudaStreamSynchronize(rt->stream) != cudaSuccess) rc = fail("CUDA execution failed");
        for (int i = 0; i < steps && !rc; i++) {
            float ms = 0;
            cudaEventElapsedTime(&ms, ev[2 * i], ev[2 * i + 1]);
            class_ms[K_CLASSES] += ms;
            launches[K_CLASSES] += 1;
        }
        for (auto& e : ev) cudaEventDestroy(e);
        if (rc || mega_check(*rt)) return 1;
        int last = 0;
        CK(cudaMemcpy(&last, rt->chain_hist + (steps - 1), sizeof(int), cudaMemcpyDeviceToHost));
        rt->position += steps;
        rt->last_result = last;
        return 0;
    }
    Profiler prof;
    prof.on = true;
    g_prof = &prof;
    int rc = 0;
    for (int i = 0; i < steps && !rc; i++) rc = enqueue_forward(*rt, w, 1, rt->cache, 1, rt->out, true);
    g_prof = nullptr;
    if (!rc && cudaStreamSynchronize(rt->stream) != cudaSuccess) rc = fail("CUDA execution failed");
    for (size_t i = 0; !rc && i < prof.cls.size(); i++) {
        float ms = 0;
        cudaEventElapsedTime(&ms, prof.ev[2 * i], prof.ev[2 * i + 1]);
        class_ms[prof.cls[i]] += ms;
        launches[prof.cls[i]] += 1;
    }
    for (cudaEvent_t e : prof.ev) cudaEventDestroy(e);
    if (rc) return rc;
    int last = 0;
    CK(cudaMemcpy(&last, rt->chain_hist + (steps - 1), sizeof(int), cudaMemcpyDeviceToHost));
    rt->position += steps;
    rt->last_result = last;
    return 0;
}

int plamo_logits(plamo_runtime* rt, int slot, float* out) {
    if (!rt || !out || slot < 0 || slot >= std::max(1, rt->last_rows)) return fail("Invalid logits slot");
    CK(cudaSetDevice(rt->device));
    std::vector<uint16_t> tmp(rt->c.vocab);
    CK(cudaMemcpy(tmp.data(), rt->out.logits + size_t(slot) * rt->c.vocab, tmp.size() * 2, cudaMemcpyDeviceToHost));
    for (int i = 0; i < rt->c.vocab; i++) out[i] = from_bits(tmp[i]);
    return 0;
}

int plamo_hidden(plamo_runtime* rt, float* out) {
    if (!rt || !out) return fail("Invalid arguments");
    CK(cudaSetDevice(rt->device));
    std::vector<uint16_t> tmp(rt->c.d);
    CK(cudaMemcpy(tmp.data(), rt->out.hidden, tmp.size() * 2, cudaMemcpyDeviceToHost));
    for (int i = 0; i < rt->c.d; i++) out[i] = from_bits(tmp[i]);
    return 0;
}

void plamo_reset(plamo_runtime* rt) {
    if (!rt) return;
    rt->position = 0; rt->gpu_seconds = 0; rt->last_rows = 0;  // Runtime.swift:319
    if (rt->mega && cudaSetDevice(rt->device) == cudaSuccess) mega_clear_exchange(*rt);
}

int plamo_position(const plamo_runtime* rt) { return rt ? rt->position : 0; }
double plamo_gpu_seconds(const plamo_runtime* rt) { return rt ? rt->gpu_seconds : 0; }
size_t plamo_weight_bytes(const plamo_runtime* rt) { return rt ? rt->weight_bytes : 0; }
size_t plamo_device_bytes(const plamo_runtime* rt) { return rt ? rt->device_bytes : 0; }
const char* plamo_device_name(const plamo_runtime* rt) { return rt ? rt->name.c_str() : ""; }
double plamo_broadcast_seconds(const plamo_runtime* rt) { return rt ? rt->bcast_seconds : 0; }
int plamo_select(plamo_runtime* rt, const int32_t* history, int n, float penalty, int no_repeat_ngram, float frequency,
                 float presence, int32_t* out_id) {
    if (!rt || !out_id || n < 0 || (n > 0 && !history)) return fail("Invalid select arguments");
    CK(cudaSetDevice(rt->device));
    const int V = rt->c.vocab;
    if (!rt->sel_counts) {
        if (rt->dalloc(rt->sel_counts, V) || rt->dalloc(rt->sel_flags, V) || rt->dalloc(rt->sel_key, 1) ||
            rt->halloc(rt->h_sel_key, 1))
            return 1;
    }
    if (n > rt->sel_cap) {  // history buffers grow to the longest history seen (older ones freed at close)
        const int cap = std::max(n, std::max(rt->sel_cap * 2, rt->context));
        if (rt->dalloc(rt->sel_hist, cap) || rt->halloc(rt->h_sel_hist, cap)) return 1;
        rt->sel_cap = cap;
    }
    if (n > 0) {
        std::copy(history, history + n, rt->h_sel_hist);
        CK(cudaMemcpyAsync(rt->sel_hist, rt->h_sel_hist, sizeof(int) * size_t(n), cudaMemcpyHostToDevice, rt->stream));
    }
    CK(launch_select(rt->out.logits, V, rt->sel_hist, n, penalty, no_repeat_ngram, frequency, presence, rt->sel_counts,
                     rt->sel_flags, rt->sel_key, rt->stream));
    CK(cudaMemcpyAsync(rt->h_sel_key, rt->sel_key, sizeof(unsigned long long), cudaMemcpyDeviceToHost, rt->stream));
    const cudaError_t e = cudaStreamSynchronize(rt->stream);
    if (e != cudaSuccess) return fail(std::string("CUDA execution failed: ") + cudaGetErrorString(e));
    *out_id = select_key_to_id(*rt->h_sel_key);
    return 0;
}

int plamo_repetition_period(const int32_t* tokens, int n, int repeats) {
    return tokens && n > 0 ? repetition_period(tokens, n, repeats) : 0;
}

int plamo_set_tensor_gemm(plamo_runtime* rt, int enable) {
    if (!rt) return fail("Invalid runtime");
    rt->tensor = (enable & 1) != 0;
    rt->tensor_attn = (enable & 2) != 0;
    return 0;
}

int plamo_dims(const plamo_runtime* rt, int32_t out[10]) {
    if (!rt || !out) return fail("Invalid arguments");
    const Config& c = rt->c;
    const int32_t v[10] = {c.d, c.layers, c.heads, c.kv_heads, c.head_dim, c.ffn, c.vocab, c.window, c.pattern, rt->context};
    memcpy(out, v, sizeof(v));
    return 0;
}

// Copies one layer's cache of one lane in the reference's ring layout: a local layer's physical
// ring (local_cap slots) is shown as the reference's ring of local_ref_cap slots, key position k of
// the last local_ref_cap positions before `position` at slot k % local_ref_cap (zeros elsewhere).
static int copy_kv_view(const plamo_runtime& rt, const Layer& L, const uint16_t* dk, const uint16_t* dv, int position,
                        uint16_t* keys, uint16_t* values) {
    const size_t row = size_t(rt.c.kv_heads) * 128;
    const int phys = L.cap, ref = L.full ? L.cap : rt.local_ref_cap;
    if (phys == ref) {
        CK(cudaMemcpy(keys, dk, size_t(phys) * row * 2, cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(values, dv, size_t(phys) * row * 2, cudaMemcpyDeviceToHost));
        return 0;
    }
    std::vector<uint16_t> hk(size_t(phys) * row), hv(size_t(phys) * row);
    CK(cudaMemcpy(hk.data(), dk, hk.size() * 2, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(hv.data(), dv, hv.size() * 2, cudaMemcpyDeviceToHost));
    std::fill(keys, keys + size_t(ref) * row, uint16_t(0));
    std::fill(values, values + size_t(ref) * row, uint16_t(0));
    for (int k = std::max(0, position - ref); k < position; k++) {
        std::copy_n(hk.data() + size_t(k % phys) * row, row, keys + size_t(k % ref) * row);
        std::copy_n(hv.data() + size_t(k % phys) * row, row, values + size_t(k % ref) * row);
    }
    return 0;
}

int plamo_debug_kv(plamo_runtime* rt, int layer, uint16_t* keys, uint16_t* values) {
    if (!rt || layer < 0 || layer >= rt->c.layers) return fail("Invalid layer");
    CK(cudaSetDevice(rt->device));
    const Layer& L = rt->layers[layer];
    return copy_kv_view(*rt, L, L.keys, L.values, rt->position, keys, values);
}

// ---- Batch ---------------------------------------------------------------------------------------

int plamo_batch_open(plamo_runtime* rt, int lanes, plamo_batch** out) {
    if (!rt || !out) return fail("Invalid arguments");
    *out = nullptr;
    if (rt->context >= 8192) return fail("Batch requires dense greedy inference with context below 8192");  // Batch.swift:34-35
    if (lanes < 1 || lanes > 64) return fail("Batch lanes must be 1...64");
    CK(cudaSetDevice(rt->device));
    auto* b = new plamo_batch();
    b->rt = rt;
    b->lanes = lanes;
    int rc = 0;
    for (int i = 0; i < rt->c.layers && !rc; i++) {
        const Layer& L = rt->layers[i];
        const long long stride = (long long)L.cap * rt->c.kv_heads * 128;
        uint16_t *k = nullptr, *v = nullptr;
        rc = dev_alloc(*b, *rt, k, size_t(stride) * lanes) || dev_alloc(*b, *rt, v, size_t(stride) * lanes);
        if (!rc) {
            cudaMemset(k, 0, size_t(stride) * lanes * 2);
            cudaMemset(v, 0, size_t(stride) * lanes * 2);
        }
        b->cache.keys.push_back(k);
        b->cache.values.push_back(v);
        b->cache.stride.push_back(stride);
    }
    if (!rc) rc = alloc_work(*b, *rt, b->work, std::max(lanes, std::min(16 * lanes, 1024)));
    if (!rc) rc = alloc_outputs(*b, *rt, b->out, lanes);
    if (rc) { delete b; return rc; }
    {
        std::lock_guard<std::mutex> lock(g_handles_mu);
        g_batches.insert(b);
    }
    *out = b;
    return 0;
}

void plamo_batch_close(plamo_batch* b) {
    {
        std::lock_guard<std::mutex> lock(g_handles_mu);
        if (!b || !g_batches.erase(b)) return;
    }
    cudaSetDevice(b->rt->device);
    cudaStreamSynchronize(b->rt->stream);
    delete b;
}

void plamo_batch_reset(plamo_batch* b) {
    if (!b) return;
    b->ready = false; b->positions.clear(); b->gpu_seconds = 0;  // Batch.swift:182
}

double plamo_batch_gpu_seconds(const plamo_batch* b) { return b ? b->gpu_seconds : 0; }

int plamo_batch_prefill(plamo_batch* b, const int32_t* const* prompts, const int32_t* lens, int n, int32_t* next_ids) {
    if (!b || !prompts || !lens) return fail("Expected one to four valid prompts");
    plamo_runtime& rt = *b->rt;
    if (n < 1 || n > b->lanes) return fail("Expected one to four valid prompts");  // Batch.swift:81-83
    for (int l = 0; l < n; l++) {
        if (!prompts[l] || lens[l] < 1 || lens[l] > rt.context) return fail("Expected one to four valid prompts");
        for (int i = 0; i < lens[l]; i++)
            if (prompts[l][i] < 0 || prompts[l][i] >= rt.c.vocab) return fail("Expected one to four valid prompts");
    }
    CK(cudaSetDevice(rt.device));
    b->ready = false;
    b->gpu_seconds = 0;
    // Every prompt goes in 16-token chunks straight into its lane slab (the reference prefills
    // through the scalar runtime and copies the KV rows, Batch.swift:86-101); the lanes' chunks
    // share forward calls.
    std::vector<PrefillLane> pl;
    for (int l = 0; l < n; l++) pl.push_back(PrefillLane{prompts[l], lens[l], 0, l, l});
    if (prefill_rows(rt, b->work, b->cache, b->out, pl, &b->gpu_seconds)) return 1;
    CK(cudaMemcpy(b->out.h_result, b->out.result, sizeof(int) * n, cudaMemcpyDeviceToHost));
    b->positions.assign(lens, lens + n);
    b->ready = true;
    for (int l = 0; l < n; l++) next_ids[l] = b->out.h_result[l];
    return 0;
}

int plamo_batch_step(plamo_batch* b, const int32_t* tokens, int n, int32_t* next_ids) {
    const char* msg = "Invalid quad step or context exhausted";  // Batch.swift:110-112
    if (!b || !tokens || !b->ready || n != int(b->positions.size())) return fail(msg);
    plamo_runtime& rt = *b->rt;
    Work& w = b->work;
    int rows = 0;
    for (int l = 0; l < n; l++) {
        if (tokens[l] < 0) continue;
        if (tokens[l] >= rt.c.vocab || b->positions[l] >= rt.context) return fail(msg);
        w.h_ids[rows] = tokens[l];
        w.h_desc[rows] = RowDesc{b->positions[l], l, b->positions[l], 1};
        w.h_out_map[rows] = l;
        rows++;
    }
    if (!rows) return fail(msg);
    CK(cudaSetDevice(rt.device));
    if (upload_inputs(rt, w, rows)) return 1;
    CK(cudaEventRecord(rt.e0, rt.stream));
    if (enqueue_forward(rt, w, rows, b->cache, rows, b->out, false)) { b->ready = false; return 1; }
    CK(cudaMemcpyAsync(b->out.h_result, b->out.result, sizeof(int) * n, cudaMemcpyDeviceToHost, rt.stream));
    if (finish(rt, &b->gpu_seconds) || (rows > 1 && check_gemm())) { b->ready = false; return 1; }
    for (int l = 0; l < n; l++)
        if (tokens[l] >= 0) b->positions[l] += 1;
    for (int l = 0; l < n; l++) next_ids[l] = b->out.h_result[l];
    return 0;
}

int plamo_batch_logits(plamo_batch* b, int lane, float* out) {
    if (!b || !out || lane < 0 || lane >= b->lanes) return fail("Invalid lane");
    CK(cudaSetDevice(b->rt->device));
    const int V = b->rt->c.vocab;
    std::vector<uint16_t> tmp(V);
    CK(cudaMemcpy(tmp.data(), b->out.logits + size_t(lane) * V, size_t(V) * 2, cudaMemcpyDeviceToHost));
    for (int i = 0; i < V; i++) out[i] = from_bits(tmp[i]);
    return 0;
}

int plamo_batch_hidden(plamo_batch* b, int lane, float* out) {
    if (!b || !out || lane < 0 || lane >= b->lanes) return fail("Invalid lane");
    CK(cudaSetDevice(b->rt->device));
    const int d = b->rt->c.d;
    std::vector<uint16_t> tmp(d);
    CK(cudaMemcpy(tmp.data(), b->out.hidden + size_t(lane) * d, size_t(d) * 2, cudaMemcpyDeviceToHost));
    for (int i = 0; i < d; i++) out[i] = from_bits(tmp[i]);
    return 0;
}

int plamo_batch_debug_kv(plamo_batch* b, int layer, int lane, uint16_t* keys, uint16_t* values) {
    if (!b || layer < 0 || layer >= b->rt->c.layers || lane < 0 || lane >= b->lanes) return fail("Invalid layer or lane");
    CK(cudaSetDevice(b->rt->device));
    const long long stride = b->cache.stride[layer];
    const int position = lane < int(b->positions.size()) ? b->positions[lane] : 0;
    return copy_kv_view(*b->rt, b->rt->layers[layer], b->cache.keys[layer] + size_t(lane) * stride,
                        b->cache.values[layer] + size_t(lane) * stride, position, keys, values);
}

// decodeBatch + Batch.generate (BatchDecode.swift:8-47)
int plamo_batch_generate(plamo_batch* b, const int32_t* const* prompts, const int32_t* lens, const int32_t* limits, int n,
                         int stop_on_truncation, int32_t* out_ids, int out_stride, int32_t* out_lens, int32_t* reasons,
                         int32_t* out_count) {
    if (!b || !limits || !out_ids || !out_lens || !reasons || !out_count || n < 1 || n > b->lanes)
        return fail("Quad output budget exceeds context");
    for (int i = 0; i < n; i++)
        if (limits[i] < 0 || limits[i] > 8191 || !lens || lens[i] + limits[i] > b->rt->context || limits[i] > out_stride)
            return fail("Quad output budget exceeds context");
    std::vector<int32_t> next(n);
    if (plamo_batch_prefill(b, prompts, lens, n, next.data())) { plamo_batch_reset(b); return 1; }
    std::vector<int> count(n, 0), reason(n, -1);
    int last = n - 1;
    std::vector<int32_t> tokens(n), preds(n);
    for (;;) {
        bool pending = false;
        for (int l = 0; l <= last; l++) pending |= reason[l] < 0;
        if (!pending) break;
        bool any = false;
        for (int l = 0; l < n; l++) {
            tokens[l] = -1;
            if (l > last || reason[l] >= 0) continue;
            if (count[l] == limits[l]) reason[l] = 1;
            else if (next[l] == 1 || next[l] == 16) reason[l] = 0;
            else {
                out_ids[size_t(l) * out_stride + count[l]] = next[l];
                count[l]++;
                if (count[l] == limits[l]) reason[l] = 1;
                else { tokens[l] = next[l]; any = true; }
            }
            if (reason[l] == 1 && stop_on_truncation) last = std::min(last, l);
        }
        if (!any) break;
        if (plamo_batch_step(b, tokens.data(), n, preds.data())) { plamo_batch_reset(b); return 1; }
        for (int l = 0; l < n; l++) next[l] = preds[l];
    }
    for (int l = 0; l <= last; l++) { out_lens[l] = count[l]; reasons[l] = reason[l] < 0 ? 1 : reason[l]; }
    *out_count = last + 1;
    return 0;
}

}  // extern "C"
