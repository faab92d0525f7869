// TEST INFRASTRUCTURE ONLY. CPU restatement ("oracle") of the PLaMo-3 0.8B decoder hot path
// of mikuteto-dev/plamo3-0.8b-runtime (Swift + Metal). Only tests/, __graft_entry__.smoke()
// and bench.py's cpu_baseline / reference arm may load this library; the product library
// (libplamo_cuda.so) never links or calls it.
//
// Every function restates the reference algorithm at the reference's bf16 rounding points.
// Citations are path:line inside the reference project:
//   Sources/Plamo/Kernels.metal   (K:)   GPU kernels
//   Sources/Plamo/Batch.metal     (BM:)  batched kernels
//   Sources/Plamo/Runtime.swift   (R:)   scalar orchestration
//   Sources/Plamo/Batch.swift     (B:)   batched orchestration
// fp32 summation order: the reference sums in Apple simdgroup order, which cannot be reproduced
// here. This restatement instead fixes the order to the summation trees of the CUDA path
// (per-lane chunks and butterfly trees for dot products and norms, 32/64/256-key split-K
// attention with a log-sum-exp merge, and the same software exp), so the CUDA path can be checked
// bit for bit. The random-init test models are chaotic under reordering (RMSE ~0.2 of logits from
// reversing the dot order alone, see noise_floor in oracle.py), so only an order-exact restatement
// can pin them at the north-star tolerance. Build with -ffp-contract=off: every fused multiply-add
// below is an explicit std::fma.
//
// Parity status: the reference forward (Metal, or PFN's MLX module) cannot run on Linux, so the
// model-level restatement is "parity unpinned" against the reference itself. The packed-weight
// codec, argmax rules and kernel-level known-answer tests are pinned by golden vectors generated
// from the reference's own numpy packer and copied from its XCTest expectations (tests/golden).
#include <cstdint>
#include <cstring>
#include <cmath>
#include <cstdio>
#include <string>
#include <vector>
#include <algorithm>
#include <limits>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

thread_local std::string g_error;
// When > 0, every layer's attention uses this many split-K partitions instead of the CUDA path's
// count: the same arithmetic in another fp32 order (noise-floor experiments only).
int g_split_override = 0;

// ---- bf16 helpers: K:5-10 -------------------------------------------------------------
inline float bf(uint16_t x) { uint32_t u = uint32_t(x) << 16; float f; std::memcpy(&f, &u, 4); return f; }
inline uint16_t bits(float x) {
    uint32_t u; std::memcpy(&u, &x, 4);
    return uint16_t((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
inline float roundbf(float x) { return bf(bits(x)); }

struct Config {
    int d, layers, heads, kv_heads, ffn, vocab, window, pattern, context;
};

struct LayerW {
    const uint16_t *pre_mixer, *post_mixer, *pre_mlp, *post_mlp;
    const uint16_t *qkv, *o, *q_norm, *k_norm, *gate_up, *down;
};

constexpr int HD = 128;                      // head_dim (R:182)
constexpr float EPS = 1e-6f;                 // rms_norm_eps (R:188)
constexpr float ATTN_SCALE = 0.08838834764831845f;  // K:372
constexpr float GLOBAL_MSCALE = 1.5545177444479562f; // K:266-267

// ---- GEMV / GEMM rows: K:92-114 (linear), K:149-200 (matrix) --------------------------
// y[t][m] = sum_k W[m][k] * x[t][k], fp32 accumulation, output bf16-rounded (or bf16 bits
// for the lm_head, K:111,196).
// noise-floor experiments: 1 walks segments and each lane's chains backwards, 2 rounds the exact sum once
int g_dot_reverse = 0;

// Sum over 32 "lanes" by the xor-butterfly tree (offsets 16, 8, 4, 2, 1).
inline float butterfly32(float (&v)[32]) {
    for (int off = 16; off >= 1; off >>= 1) {
        float t[32];
        for (int l = 0; l < 32; l++) t[l] = v[l] + v[l ^ off];
        for (int l = 0; l < 32; l++) v[l] = t[l];
    }
    return v[0];
}

// Dot product in the GEMV order. K is cut into segments of 1536 weights (three 512-weight groups;
// the last segment may be shorter). Within a segment, lane l owns weights [g*512 + 16l, +16) of
// each group g and sums even / odd elements into two fma chains; the lane's segment partial
// (even + odd) is added to its running total segment by segment; the 32 lane totals meet in the
// butterfly tree.
inline float dot_bf16(const uint16_t* w, const float* x, int K) {
    if (g_dot_reverse == 2) {  // correctly rounded twin: exact products, double sum, one rounding
        double acc = 0.0;
        for (int k = 0; k < K; k++) acc += double(bf(w[k])) * double(x[k]);
        return float(acc);
    }
    const int G = (K + 511) / 512, S = (G + 2) / 3;
    float lanes[32];
    for (int l = 0; l < 32; l++) {
        float t = 0.f;
        for (int si = 0; si < S; si++) {
            const int seg = g_dot_reverse ? S - 1 - si : si;
            float a0 = 0.f, a1 = 0.f;
            for (int g = 3 * seg; g < std::min(G, 3 * seg + 3); g++) {
                const int e0 = g * 512 + 16 * l;
                if (e0 >= K) continue;
                for (int kk = 0; kk < 8; kk++) {
                    const int k = g_dot_reverse ? 7 - kk : kk;
                    a0 = std::fma(bf(w[e0 + 2 * k]), x[e0 + 2 * k], a0);
                    a1 = std::fma(bf(w[e0 + 2 * k + 1]), x[e0 + 2 * k + 1], a1);
                }
            }
            t = t + (a0 + a1);
        }
        lanes[l] = t;
    }
    return butterfly32(lanes);
}

// e^x from IEEE operations only: Cody-Waite reduction x = n*ln2 + r (ln2 = 355/512 + rest),
// degree-7 Taylor polynomial of e^r in Horner form, scale by 2^n via the exponent field. The CUDA
// path evaluates the same sequence, so both give identical bits.
inline float f_of(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
inline float pexp(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return std::numeric_limits<float>::infinity();
    if (x < -103.972084045410156f) return 0.0f;
    const float n = std::rint(x * 1.44269502162933349609375f);
    float r = std::fma(-n, 0.693359375f, x);
    r = std::fma(-n, -2.12194440e-4f, r);
    float p = 1.98412698e-4f;
    p = std::fma(p, r, 1.38888889e-3f);
    p = std::fma(p, r, 8.33333377e-3f);
    p = std::fma(p, r, 4.16666679e-2f);
    p = std::fma(p, r, 1.66666672e-1f);
    p = std::fma(p, r, 0.5f);
    p = std::fma(p, r, 1.0f);
    p = std::fma(p, r, 1.0f);
    const int k = int(n);
    if (k > 127) return (p * f_of(254u << 23)) * f_of(uint32_t(k - 127 + 127) << 23);
    if (k < -126) return (p * f_of(uint32_t(k + 100 + 127) << 23)) * f_of(uint32_t(127 - 100) << 23);
    return p * f_of(uint32_t(k + 127) << 23);
}

void linear_rows(const uint16_t* w, const float* x, int rows, int K, int M, float* y, uint16_t* y_bits) {
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        const uint16_t* wr = w + size_t(m) * K;
        for (int t = 0; t < rows; t++) {
            float s = dot_bf16(wr, x + size_t(t) * K, K);
            if (y_bits) y_bits[size_t(t) * M + m] = bits(s);
            else y[size_t(t) * M + m] = roundbf(s);
        }
    }
}

// ---- RMSNorm: K:46-90 ------------------------------------------------------------------
// z = bf(bf(x*rsqrt(mean(x^2)+eps)) * bf(w+offset)); optional residual x <- bf(x+z) (K:71)
// and optional fused next norm with offset 1 over the new x (K:75-89).
// Sum of squares in the norm kernel's order: 256 threads, thread t sums x[t + 256j] (j < 16) by
// fma, each warp of 32 threads by the butterfly tree, the 8 warp sums by a second butterfly (the
// other 24 lanes contribute zeros).
inline float rms_scale(const float* x, int n) {
    float warps[8];
    for (int w = 0; w < 8; w++) {
        float lanes[32];
        for (int l = 0; l < 32; l++) {
            const int t = w * 32 + l;
            float ss = 0.f;
            for (int j = 0; j < 16; j++) {
                const int i = t + 256 * j;
                const float v = i < n ? x[i] : 0.f;
                ss = std::fma(v, v, ss);
            }
            lanes[l] = ss;
        }
        warps[w] = butterfly32(lanes);
    }
    float lanes[32];
    for (int l = 0; l < 32; l++) lanes[l] = l < 8 ? warps[l] : 0.f;
    const float total = butterfly32(lanes);
    return 1.0f / std::sqrt(total / float(n) + EPS);
}

void norm_row(const uint16_t* w, const float* x, float* y, int n, float offset,
              float* residual, const uint16_t* next_w, float* next_y) {
    float r = rms_scale(x, n);
    std::vector<float> staged(n);
    for (int i = 0; i < n; i++) {
        float z = roundbf(roundbf(x[i] * r) * roundbf(bf(w[i]) + offset));
        float value = residual ? roundbf(residual[i] + z) : z;
        staged[i] = value;
    }
    for (int i = 0; i < n; i++) y[i] = staged[i];
    if (!next_w) return;
    float r2 = rms_scale(staged.data(), n);
    for (int i = 0; i < n; i++)
        next_y[i] = roundbf(roundbf(staged[i] * r2) * roundbf(bf(next_w[i]) + 1.0f));
}

// ---- SwiGLU: K:202-210 -----------------------------------------------------------------
void swiglu_rows(const float* gates, float* out, int rows, int F) {
    for (int t = 0; t < rows; t++)
        for (int i = 0; i < F; i++) {
            float g = gates[size_t(t) * 2 * F + i];
            float u = gates[size_t(t) * 2 * F + F + i];
            out[size_t(t) * F + i] = roundbf(roundbf(g / (1.0f + pexp(-g))) * u);
        }
}

// ---- argmax: K:704-729 (first index of the maximum; NaN never wins; all-NaN -> UINT32_MAX)
uint32_t argmax_bits(const uint16_t* v, int n) {
    float best = -std::numeric_limits<float>::infinity(); uint32_t idx = 0xffffffffu;
    for (int i = 0; i < n; i++) {
        float x = bf(v[i]);
        if (x > best || (x == best && uint32_t(i) < idx)) { best = x; idx = uint32_t(i); }
    }
    return idx;
}
uint32_t argmax_f32(const float* v, int n) {
    float best = -std::numeric_limits<float>::infinity(); uint32_t idx = 0xffffffffu;
    for (int i = 0; i < n; i++) {
        float x = v[i];
        if (x > best || (x == best && uint32_t(i) < idx)) { best = x; idx = uint32_t(i); }
    }
    return idx;
}

// ---- RoPE tables ------------------------------------------------------------------------
// Local: bf16 (cos, sin) of float(row)*inv_freq_local[i] (K:212-219, R:266-284).
// Global: fp32 cos/sin of float(pos)*inv_freq_full[i], bf16-rounded, times the YaRN mscale,
// bf16-rounded again (K:264-267). cos/sin here are evaluated in double on the fp32 angle and
// rounded once to fp32; the CUDA library uploads tables built by the same formula.
inline uint16_t cos_bits(float a) { return bits(float(std::cos(double(a)))); }
inline uint16_t sin_bits(float a) { return bits(float(std::sin(double(a)))); }

struct Rope {
    std::vector<uint16_t> local;   // [rows][64][2]
    std::vector<uint16_t> global;  // [context][64][2]
    int local_rows = 0;
    void build(const float* inv_local, const float* inv_full, int local_rows_, int context) {
        local_rows = local_rows_;
        local.resize(size_t(local_rows) * 128);
        for (int p = 0; p < local_rows; p++)
            for (int i = 0; i < 64; i++) {
                float phase = float(p) * inv_local[i];
                local[(size_t(p) * 64 + i) * 2] = cos_bits(phase);
                local[(size_t(p) * 64 + i) * 2 + 1] = sin_bits(phase);
            }
        global.resize(size_t(context) * 128);
        for (int p = 0; p < context; p++)
            for (int i = 0; i < 64; i++) {
                float angle = float(p) * inv_full[i];
                float c = roundbf(bf(cos_bits(angle)) * GLOBAL_MSCALE);
                float s = roundbf(bf(sin_bits(angle)) * GLOBAL_MSCALE);
                global[(size_t(p) * 64 + i) * 2] = bits(c);
                global[(size_t(p) * 64 + i) * 2 + 1] = bits(s);
            }
    }
    // K:261-274: rotate-half, bf(bf(x*c) + bf(+-other*s)).
    inline float rotated(float x, float other, int d, int pos, bool full) const {
        const uint16_t* t = full ? &global[(size_t(pos) * 64 + (d % 64)) * 2] : &local[(size_t(pos) * 64 + (d % 64)) * 2];
        float c = bf(t[0]), s = bf(t[1]);
        return roundbf(roundbf(x * c) + roundbf((d < 64 ? -other : other) * s));
    }
};

// Per-query-row attention geometry. Key r in [0, count) of the visible window lives at
// physical slot (first + r) % cap of its cache; local keys are re-rotated with coordinate r
// (K:277-285, K:301-345, BM:42-88); rows see keys r in [begin, end) (K:368-369, BM:101).
struct RowGeo {
    uint16_t* keys; uint16_t* values;   // this row's cache (scalar cache or lane slab)
    int cap, pos, qcoord, first, count, begin, end;
};

struct State {
    Config c;
    std::vector<LayerW> w;
    const uint16_t *embed, *final_norm, *lm_head;
    Rope rope;
    int chunk;          // batchLimit = min(context, 16) (R:129,173)
    int local_cap;      // min(context, window + chunk) (R:240)
    // scalar caches (R:247)
    std::vector<std::vector<uint16_t>> keys, values;
    int position = 0;
    // outputs of the last call
    std::vector<uint16_t> logits;   // [rows][vocab] bf16
    std::vector<float> hidden;      // final-normed hidden of the output rows
    int last_rows = 0;
    std::vector<uint32_t> result;
    bool full_layer(int i) const { return i % c.pattern == c.pattern - 1; }
    int cap_of(int i) const { return full_layer(i) ? c.context : local_cap; }
    // split-K partition count of a layer (the CUDA runtime's choice: ~64 keys per partition of the
    // local window, at most 256 keys per partition of the global history, at least 32 partitions)
    int splits_of(int i) const {
        const int cap = cap_of(i);
        return full_layer(i) ? std::max(32, (cap + 255) / 256) : std::max(1, (cap + 63) / 64);
    }
};

// ---- QK-norm + RoPE + KV append: K:223-259 (qkv), BM:1-39 (qkv_mapped) ------------------
void qkv_row(const State& s, const LayerW& w, bool full, const float* qkv, float* q_out, const RowGeo& g) {
    const int H = s.c.heads, KV = s.c.kv_heads;
    for (int h = 0; h < H + KV; h++) {
        const float* v = qkv + h * HD;
        float lanes[32];  // lane l holds v[l + 32j], j < 4 (Kernels.metal:237-241 layout)
        for (int l = 0; l < 32; l++) {
            float ss = 0.f;
            for (int j = 0; j < 4; j++) ss = std::fma(v[l + 32 * j], v[l + 32 * j], ss);
            lanes[l] = ss;
        }
        float sum = butterfly32(lanes);
        float scale = 1.0f / std::sqrt(sum / 128.0f + EPS);
        const uint16_t* nw = h < H ? w.q_norm : w.k_norm;
        float z[HD];
        for (int d = 0; d < HD; d++) z[d] = roundbf(roundbf(v[d] * scale) * roundbf(bf(nw[d]) + 1.0f));
        for (int d = 0; d < HD; d++) {
            int partner = d < 64 ? d + 64 : d - 64;
            if (h < H) {
                q_out[h * HD + d] = s.rope.rotated(z[d], z[partner], d, g.qcoord, full);
            } else {
                int kvh = h - H;
                size_t dst = (size_t(g.pos % g.cap) * KV + kvh) * HD + d;
                g.keys[dst] = bits(full ? s.rope.rotated(z[d], z[partner], d, g.pos, true) : z[d]);
                g.values[dst] = bits(qkv[(H + KV + kvh) * HD + d]);
            }
        }
    }
}

// ---- attention for one query row: scores (K:301-345 / BM:42-88), scale + mask + softmax
// (K:358-397 / BM:91-129), P.V with bf16-rounded output (K:400-437 / BM:132-168).
void attend_row(const State& s, bool full, const float* q, const RowGeo& g, float* out) {
    const int H = s.c.heads, KV = s.c.kv_heads, group = H / KV;
    std::vector<float> kr(size_t(g.count) * KV * HD);
    for (int r = 0; r < g.count; r++) {
        int phys = (g.first + r) % g.cap;
        for (int kvh = 0; kvh < KV; kvh++) {
            const uint16_t* k = g.keys + (size_t(phys) * KV + kvh) * HD;
            float* dst = &kr[(size_t(r) * KV + kvh) * HD];
            for (int d = 0; d < HD; d++) {
                int partner = d < 64 ? d + 64 : d - 64;
                dst[d] = full ? bf(k[d]) : s.rope.rotated(bf(k[d]), bf(k[partner]), d, r, false);
            }
        }
    }
    std::vector<float> p(g.count);
    for (int h = 0; h < H; h++) {
        int kvh = h / group;
        const float* qh = q + h * HD;
        float m = -INFINITY;
        for (int r = 0; r < g.count; r++) {
            const float* k = &kr[(size_t(r) * KV + kvh) * HD];
            float acc[8] = {0};
            for (int d = 0; d < HD; d += 8) for (int j = 0; j < 8; j++) acc[j] += qh[d + j] * k[d + j];
            for (int st = 4; st > 0; st >>= 1) for (int j = 0; j < st; j++) acc[j] += acc[j + st];
            float v = (r >= g.begin && r < g.end) ? acc[0] * ATTN_SCALE : -INFINITY;
            p[r] = v; m = std::max(m, v);
        }
        float total = 0;
        for (int r = 0; r < g.count; r++) { float e = std::exp(p[r] - m); p[r] = e; total += e; }
        for (int r = 0; r < g.count; r++) p[r] /= total;
        float o[HD] = {0};
        for (int r = 0; r < g.count; r++) {
            if (p[r] == 0.0f) continue;
            int phys = (g.first + r) % g.cap;
            const uint16_t* v = g.values + (size_t(phys) * KV + kvh) * HD;
            for (int d = 0; d < HD; d++) o[d] += p[r] * bf(v[d]);
        }
        for (int d = 0; d < HD; d++) out[h * HD + d] = roundbf(o[d]);
    }
}

// ---- split-K attention + merge (K:440-562) in the CUDA kernel's order ---------------------
// `splits` key partitions of per = roundup32(ceil(count / splits)) window positions, each clipped
// to the row's visible range; per partition and head: scores by an fma chain over d, scaled;
// max; e = exp(score - max) summed per lane (i mod 32, increasing i) then by the butterfly tree;
// P.V by an fma chain over keys. Merge: M = max of partition maxima, weights exp(m_s - M),
// L = fma chain of w_s * l_s, output fma chain of O_s * w_s, bf16-rounded O / L.
void attend_row_splitk(const State& s, bool full, const float* q, const RowGeo& g, float* out, int splits) {
    const int H = s.c.heads, KV = s.c.kv_heads, group = H / KV;
    int per = (g.count + splits - 1) / splits;
    per = (per + 31) & ~31;
    std::vector<float> po(size_t(splits) * H * HD, 0.f), pm(size_t(splits) * H), pl(size_t(splits) * H);
#pragma omp parallel for schedule(dynamic)
    for (int sp = 0; sp < splits; sp++) {
        const int k0 = sp * per, k1 = std::min(k0 + per, g.count);
        const int lo = std::max(k0, g.begin), hi = std::min(k1, g.end);
        if (lo >= hi) {
            for (int h = 0; h < H; h++) { pm[size_t(sp) * H + h] = -INFINITY; pl[size_t(sp) * H + h] = 0.f; }
            continue;
        }
        const int n = hi - lo;
        std::vector<float> kr(size_t(n) * KV * HD), sc(n);
        for (int i = 0; i < n; i++) {
            const int key = lo + i, phys = (g.first + key) % g.cap;
            for (int kvh = 0; kvh < KV; kvh++) {
                const uint16_t* k = g.keys + (size_t(phys) * KV + kvh) * HD;
                for (int d = 0; d < HD; d++) {
                    const int partner = d < 64 ? d + 64 : d - 64;
                    kr[(size_t(i) * KV + kvh) * HD + d] =
                        full ? bf(k[d]) : s.rope.rotated(bf(k[d]), bf(k[partner]), d, key, false);
                }
            }
        }
        for (int h = 0; h < H; h++) {
            const int kvh = h / group;
            const float* qh = q + h * HD;
            float m = -INFINITY;
            for (int i = 0; i < n; i++) {
                const float* kv = &kr[(size_t(i) * KV + kvh) * HD];
                float acc = 0.f;
                for (int d = 0; d < HD; d++) acc = std::fma(qh[d], kv[d], acc);
                sc[i] = acc * ATTN_SCALE;
                m = std::max(m, sc[i]);
            }
            float lanes[32] = {0};
            for (int i = 0; i < n; i++) {
                const float e = pexp(sc[i] - m);
                sc[i] = e;
                lanes[i % 32] += e;
            }
            const float l = butterfly32(lanes);
            float* o = &po[(size_t(sp) * H + h) * HD];
            for (int i = 0; i < n; i++) {
                const int phys = (g.first + lo + i) % g.cap;
                const uint16_t* v = g.values + (size_t(phys) * KV + kvh) * HD;
                for (int d = 0; d < HD; d++) o[d] = std::fma(sc[i], bf(v[d]), o[d]);
            }
            pm[size_t(sp) * H + h] = m;
            pl[size_t(sp) * H + h] = l;
        }
    }
    for (int h = 0; h < H; h++) {
        float M = -INFINITY;
        for (int sp = 0; sp < splits; sp++) M = std::max(M, pm[size_t(sp) * H + h]);
        float L = 0.f, o[HD] = {0};
        for (int sp = 0; sp < splits; sp++) {
            const float l = pl[size_t(sp) * H + h];
            if (!(l > 0.f)) continue;
            const float w = pexp(pm[size_t(sp) * H + h] - M);
            L = std::fma(w, l, L);
            for (int d = 0; d < HD; d++) o[d] = std::fma(po[(size_t(sp) * H + h) * HD + d], w, o[d]);
        }
        for (int d = 0; d < HD; d++) out[h * HD + d] = roundbf(o[d] / L);
    }
}

// ---- one decoder pass over `rows` token rows: R:376-458 / B:147-165 ----------------------
// x: [rows][d] embeddings (fp32 holding bf16 values). geo[i]: per-row geometry for layer i
// (local and full variants chosen by the caller). Writes normalized/logits for out_rows.
struct Work {
    std::vector<float> x, normalized, qkv, q, attended, projected, gates, activated;
    void size(const Config& c, int rows) {
        int qd = c.heads * HD, qkvd = (c.heads + 2 * c.kv_heads) * HD;
        x.resize(size_t(rows) * c.d); normalized.resize(size_t(rows) * c.d);
        qkv.resize(size_t(rows) * qkvd); q.resize(size_t(rows) * qd); attended.resize(size_t(rows) * qd);
        projected.resize(size_t(rows) * c.d); gates.resize(size_t(rows) * 2 * c.ffn);
        activated.resize(size_t(rows) * c.ffn);
    }
};

using GeoFn = RowGeo (*)(void* ctx, int layer, int row);

void decoder(State& s, Work& wk, int rows, GeoFn geo, void* ctx, bool split_ok) {
    const Config& c = s.c;
    const int d = c.d, qd = c.heads * HD, qkvd = (c.heads + 2 * c.kv_heads) * HD;
    const float post_mlp_offset = float(1.0 / std::pow(5.0, 1.5));  // R:450
    for (int li = 0; li < c.layers; li++) {
        const LayerW& w = s.w[li];
        bool full = s.full_layer(li);
        if (li == 0)  // R:377
            for (int t = 0; t < rows; t++)
                norm_row(w.pre_mixer, &wk.x[size_t(t) * d], &wk.normalized[size_t(t) * d], d, 1.0f, nullptr, nullptr, nullptr);
        linear_rows(w.qkv, wk.normalized.data(), rows, d, qkvd, wk.qkv.data(), nullptr);  // R:388
        for (int t = 0; t < rows; t++) {
            RowGeo g = geo(ctx, li, t);
            qkv_row(s, w, full, &wk.qkv[size_t(t) * qkvd], &wk.q[size_t(t) * qd], g);
        }
#pragma omp parallel for schedule(dynamic) if (rows > 1)
        for (int t = 0; t < rows; t++) {
            RowGeo g = geo(ctx, li, t);
            attend_row_splitk(s, full, &wk.q[size_t(t) * qd], g, &wk.attended[size_t(t) * qd],
                              g_split_override > 0 ? g_split_override : s.splits_of(li));
        }
        linear_rows(w.o, wk.attended.data(), rows, qd, d, wk.projected.data(), nullptr);  // R:445
        for (int t = 0; t < rows; t++)  // R:446
            norm_row(w.post_mixer, &wk.projected[size_t(t) * d], &wk.x[size_t(t) * d], d, 0.2f,
                     &wk.x[size_t(t) * d], w.pre_mlp, &wk.normalized[size_t(t) * d]);
        linear_rows(w.gate_up, wk.normalized.data(), rows, d, 2 * c.ffn, wk.gates.data(), nullptr);  // R:447
        swiglu_rows(wk.gates.data(), wk.activated.data(), rows, c.ffn);  // R:448
        linear_rows(w.down, wk.activated.data(), rows, c.ffn, d, wk.projected.data(), nullptr);  // R:449
        const uint16_t* next = li + 1 < c.layers ? s.w[li + 1].pre_mixer : nullptr;
        for (int t = 0; t < rows; t++)  // R:450-451
            norm_row(w.post_mlp, &wk.projected[size_t(t) * d], &wk.x[size_t(t) * d], d, post_mlp_offset,
                     &wk.x[size_t(t) * d], next, &wk.normalized[size_t(t) * d]);
    }
}

void head(State& s, Work& wk, int first_row, int rows) {  // R:453-458
    const int d = s.c.d, V = s.c.vocab;
    std::vector<float> nrm(size_t(rows) * d);
    for (int t = 0; t < rows; t++)
        norm_row(s.final_norm, &wk.x[size_t(first_row + t) * d], &nrm[size_t(t) * d], d, 1.0f, nullptr, nullptr, nullptr);
    s.logits.assign(size_t(rows) * V, 0);
    linear_rows(s.lm_head, nrm.data(), rows, d, V, nullptr, s.logits.data());
    s.hidden = nrm;
    s.result.resize(rows);
    for (int t = 0; t < rows; t++) s.result[t] = argmax_bits(&s.logits[size_t(t) * V], V);
    s.last_rows = rows;
}

void embed_rows(const State& s, const int32_t* ids, int n, float* x) {  // R:104-110
    for (int t = 0; t < n; t++)
        for (int i = 0; i < s.c.d; i++) x[size_t(t) * s.c.d + i] = bf(s.embed[size_t(ids[t]) * s.c.d + i]);
}

struct ScalarCtx { State* s; int start, rows; };

RowGeo scalar_geo(void* p, int li, int t) {  // R:389-395, K:251,368-369
    ScalarCtx& sc = *(ScalarCtx*)p;
    State& s = *sc.s;
    bool full = s.full_layer(li);
    int W = s.c.window;
    RowGeo g;
    g.keys = s.keys[li].data(); g.values = s.values[li].data(); g.cap = s.cap_of(li);
    int base = full ? 0 : std::max(0, sc.start - (W - 1));
    g.pos = sc.start + t;
    g.qcoord = full ? g.pos : g.pos - base;
    g.first = base;
    g.count = sc.start + sc.rows - base;
    g.end = sc.start + t - base + 1;
    g.begin = full ? 0 : (g.end > W ? g.end - W : 0);
    return g;
}

struct Batch {
    State* s;
    int lanes;
    std::vector<std::vector<uint16_t>> keys, values;  // [layer][lane][cap][KV*128]   (B:40)
    std::vector<float> hidden;                        // [lane][d]    (B:48)
    std::vector<uint16_t> logits;                     // [lane][vocab] (B:49)
    std::vector<uint32_t> result;                     // [lane]
    std::vector<int> positions;
    bool ready = false;
};

struct BatchCtx { Batch* b; const int* lanes; };

RowGeo batch_geo(void* p, int li, int q) {  // B:116-128, BM:27-35,55-64
    BatchCtx& bc = *(BatchCtx*)p;
    Batch& b = *bc.b; State& s = *b.s;
    bool full = s.full_layer(li);
    int W = s.c.window, lane = bc.lanes[q];
    RowGeo g;
    g.cap = s.cap_of(li);
    size_t slab = size_t(g.cap) * s.c.kv_heads * HD;
    g.keys = b.keys[li].data() + size_t(lane) * slab;
    g.values = b.values[li].data() + size_t(lane) * slab;
    g.pos = b.positions[lane];
    g.first = full ? 0 : std::max(0, g.pos - (W - 1));
    g.count = g.pos - g.first + 1;
    g.qcoord = full ? g.pos : std::min(g.pos, W - 1);
    g.begin = 0; g.end = g.count;
    return g;
}

int forward_impl(State& s, const int32_t* ids, int n, bool output, int32_t* next) {
    // R:328-330
    if (n <= 0 || n > s.chunk || s.position + n > s.c.context) { g_error = "Invalid tokens or context exhausted"; return 1; }
    for (int i = 0; i < n; i++) if (ids[i] < 0 || ids[i] >= s.c.vocab) { g_error = "Invalid tokens or context exhausted"; return 1; }
    Work wk; wk.size(s.c, n);
    embed_rows(s, ids, n, wk.x.data());
    ScalarCtx sc{&s, s.position, n};
    decoder(s, wk, n, scalar_geo, &sc, true);
    if (output) head(s, wk, n - 1, 1);
    else s.last_rows = 0;
    s.position += n;
    if (next) *next = output ? int32_t(s.result[0]) : -1;
    return 0;
}

}  // namespace

extern "C" {

struct oracle_config { int d, layers, heads, kv_heads, ffn, vocab, window, pattern, context; };
struct oracle_layer { const uint16_t *pre_mixer, *post_mixer, *pre_mlp, *post_mlp, *qkv, *o, *q_norm, *k_norm, *gate_up, *down; };

const char* oracle_last_error() { return g_error.c_str(); }
void oracle_set_split_partition(int splits) { g_split_override = splits; }
void oracle_set_dot_reverse(int on) { g_dot_reverse = on; }

void oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#endif
}
int oracle_threads() {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void* oracle_create(const oracle_config* cfg, const oracle_layer* layers, const uint16_t* embed,
                    const uint16_t* final_norm, const uint16_t* lm_head, const float* inv_local, const float* inv_full) {
    if (cfg->context < 1 || cfg->heads % cfg->kv_heads != 0 || cfg->pattern < 1) { g_error = "invalid config"; return nullptr; }
    State* s = new State();
    s->c = {cfg->d, cfg->layers, cfg->heads, cfg->kv_heads, cfg->ffn, cfg->vocab, cfg->window, cfg->pattern, cfg->context};
    for (int i = 0; i < cfg->layers; i++) {
        const oracle_layer& l = layers[i];
        s->w.push_back({l.pre_mixer, l.post_mixer, l.pre_mlp, l.post_mlp, l.qkv, l.o, l.q_norm, l.k_norm, l.gate_up, l.down});
    }
    s->embed = embed; s->final_norm = final_norm; s->lm_head = lm_head;
    s->chunk = std::min(cfg->context, 16);
    s->local_cap = std::min(cfg->context, cfg->window + s->chunk);
    s->rope.build(inv_local, inv_full, std::min(cfg->context, cfg->window + 16), cfg->context);  // R:266
    s->keys.resize(cfg->layers); s->values.resize(cfg->layers);
    for (int i = 0; i < cfg->layers; i++) {
        size_t n = size_t(s->cap_of(i)) * cfg->kv_heads * HD;
        s->keys[i].assign(n, 0); s->values[i].assign(n, 0);
    }
    return s;
}

void oracle_destroy(void* p) { delete (State*)p; }
void oracle_reset(void* p) { State* s = (State*)p; s->position = 0; s->last_rows = 0; }  // R:319
int oracle_position(void* p) { return ((State*)p)->position; }

int oracle_forward(void* p, const int32_t* ids, int n, int output, int32_t* next) {
    return forward_impl(*(State*)p, ids, n, output != 0, next);
}

// R:469-483: chunks of batchLimit, logits only for the last chunk.
int oracle_prefill(void* p, const int32_t* ids, int n, int32_t* next) {
    State& s = *(State*)p;
    if (n <= 0 || s.position + n > s.c.context) { g_error = "Input exceeds context"; return 1; }
    int32_t nx = -1;
    for (int start = 0; start < n; start += s.chunk) {
        int end = std::min(start + s.chunk, n);
        int rc = forward_impl(s, ids + start, end - start, end == n, &nx);
        if (rc) return rc;
    }
    if (next) *next = nx;
    return 0;
}

// R:540-552: bf16 logits widened to fp32.
int oracle_logits(void* p, int slot, float* out) {
    State& s = *(State*)p;
    if (slot < 0 || slot >= std::max(1, s.last_rows) || s.logits.empty()) { g_error = "invalid logits slot"; return 1; }
    for (int i = 0; i < s.c.vocab; i++) out[i] = bf(s.logits[size_t(slot) * s.c.vocab + i]);
    return 0;
}
int oracle_logits_bits(void* p, int slot, uint16_t* out) {
    State& s = *(State*)p;
    if (slot < 0 || slot >= std::max(1, s.last_rows) || s.logits.empty()) { g_error = "invalid logits slot"; return 1; }
    std::memcpy(out, &s.logits[size_t(slot) * s.c.vocab], size_t(s.c.vocab) * 2);
    return 0;
}
int oracle_hidden(void* p, float* out) {
    State& s = *(State*)p;
    if (s.hidden.empty()) return 1;
    std::memcpy(out, s.hidden.data(), size_t(s.c.d) * 4);
    return 0;
}
// Copies the scalar KV cache of one layer (cap*KV*128 bf16 each) for state comparisons.
int oracle_kv(void* p, int layer, uint16_t* keys, uint16_t* values) {
    State& s = *(State*)p;
    if (layer < 0 || layer >= s.c.layers) return 1;
    std::memcpy(keys, s.keys[layer].data(), s.keys[layer].size() * 2);
    std::memcpy(values, s.values[layer].data(), s.values[layer].size() * 2);
    return 0;
}

// ---- Batch: B:33-186 ---------------------------------------------------------------------
void* oracle_batch_create(void* rt, int lanes) {
    State* s = (State*)rt;
    if (lanes < 1) { g_error = "invalid lanes"; return nullptr; }
    Batch* b = new Batch();
    b->s = s; b->lanes = lanes;
    b->keys.resize(s->c.layers); b->values.resize(s->c.layers);
    for (int i = 0; i < s->c.layers; i++) {
        size_t n = size_t(lanes) * s->cap_of(i) * s->c.kv_heads * HD;
        b->keys[i].assign(n, 0); b->values[i].assign(n, 0);
    }
    b->hidden.assign(size_t(lanes) * s->c.d, 0.0f);
    b->logits.assign(size_t(lanes) * s->c.vocab, 0);
    b->result.assign(lanes, 0);
    return b;
}
void oracle_batch_destroy(void* p) { delete (Batch*)p; }
void oracle_batch_reset(void* p) { Batch* b = (Batch*)p; b->ready = false; b->positions.clear(); }  // B:182

// B:80-106: serial scalar prefill per lane, then copy min(len, cap) cache rows into the slab.
int oracle_batch_prefill(void* p, const int32_t* const* prompts, const int32_t* lens, int n, int32_t* next) {
    Batch& b = *(Batch*)p; State& s = *b.s;
    if (n < 1 || n > b.lanes) { g_error = "Expected one to four valid prompts"; return 1; }
    for (int l = 0; l < n; l++) {
        if (lens[l] < 1 || lens[l] > s.c.context) { g_error = "Expected one to four valid prompts"; return 1; }
        for (int i = 0; i < lens[l]; i++) if (prompts[l][i] < 0 || prompts[l][i] >= s.c.vocab) { g_error = "Expected one to four valid prompts"; return 1; }
    }
    b.ready = false;
    for (int l = 0; l < n; l++) {
        s.position = 0; s.last_rows = 0;
        int32_t nx = -1;
        if (oracle_prefill(&s, prompts[l], lens[l], &nx)) return 1;
        for (int li = 0; li < s.c.layers; li++) {
            int cap = s.cap_of(li);
            size_t row = size_t(s.c.kv_heads) * HD, slab = size_t(cap) * row;
            size_t cnt = size_t(std::min(lens[l], cap)) * row;
            std::memcpy(b.keys[li].data() + l * slab, s.keys[li].data(), cnt * 2);
            std::memcpy(b.values[li].data() + l * slab, s.values[li].data(), cnt * 2);
        }
        std::memcpy(&b.hidden[size_t(l) * s.c.d], s.hidden.data(), size_t(s.c.d) * 4);
        std::memcpy(&b.logits[size_t(l) * s.c.vocab], s.logits.data(), size_t(s.c.vocab) * 2);
        b.result[l] = uint32_t(nx);
    }
    b.positions.assign(lens, lens + n);
    b.ready = true;
    for (int l = 0; l < n; l++) next[l] = int32_t(b.result[l]);
    return 0;
}

// B:109-179: one batched decode step over the active lanes (token < 0 = inactive lane).
int oracle_batch_step(void* p, const int32_t* tokens, int n, int32_t* next) {
    Batch& b = *(Batch*)p; State& s = *b.s;
    if (!b.ready || n != int(b.positions.size())) { g_error = "Invalid quad step or context exhausted"; return 1; }
    std::vector<int> active; std::vector<int32_t> ids;
    for (int l = 0; l < n; l++) {
        if (tokens[l] < 0) continue;
        if (tokens[l] >= s.c.vocab || b.positions[l] >= s.c.context) { g_error = "Invalid quad step or context exhausted"; return 1; }
        active.push_back(l); ids.push_back(tokens[l]);
    }
    if (active.empty()) { g_error = "Invalid quad step or context exhausted"; return 1; }
    int rows = int(active.size());
    Work wk; wk.size(s.c, rows);
    embed_rows(s, ids.data(), rows, wk.x.data());
    BatchCtx bc{&b, active.data()};
    decoder(s, wk, rows, batch_geo, &bc, false);
    head(s, wk, 0, rows);
    for (int q = 0; q < rows; q++) {
        int l = active[q];
        std::memcpy(&b.hidden[size_t(l) * s.c.d], &s.hidden[size_t(q) * s.c.d], size_t(s.c.d) * 4);
        std::memcpy(&b.logits[size_t(l) * s.c.vocab], &s.logits[size_t(q) * s.c.vocab], size_t(s.c.vocab) * 2);
        b.result[l] = s.result[q];
        b.positions[l] += 1;
    }
    for (int l = 0; l < n; l++) next[l] = int32_t(b.result[l]);
    return 0;
}
int oracle_batch_logits_bits(void* p, int lane, uint16_t* out) {
    Batch& b = *(Batch*)p;
    if (lane < 0 || lane >= b.lanes) return 1;
    std::memcpy(out, &b.logits[size_t(lane) * b.s->c.vocab], size_t(b.s->c.vocab) * 2);
    return 0;
}
int oracle_batch_hidden(void* p, int lane, float* out) {
    Batch& b = *(Batch*)p;
    if (lane < 0 || lane >= b.lanes) return 1;
    std::memcpy(out, &b.hidden[size_t(lane) * b.s->c.d], size_t(b.s->c.d) * 4);
    return 0;
}
int oracle_batch_kv(void* p, int layer, int lane, uint16_t* keys, uint16_t* values) {
    Batch& b = *(Batch*)p; State& s = *b.s;
    if (layer < 0 || layer >= s.c.layers || lane < 0 || lane >= b.lanes) return 1;
    size_t slab = size_t(s.cap_of(layer)) * s.c.kv_heads * HD;
    std::memcpy(keys, b.keys[layer].data() + lane * slab, slab * 2);
    std::memcpy(values, b.values[layer].data() + lane * slab, slab * 2);
    return 0;
}

// ---- kernel-level restatements for unit tests ---------------------------------------------
void oracle_linear(const uint16_t* w, const float* x, int rows, int K, int M, int logits, void* y) {
    if (logits) linear_rows(w, x, rows, K, M, nullptr, (uint16_t*)y);
    else linear_rows(w, x, rows, K, M, (float*)y, nullptr);
}
void oracle_norm(const uint16_t* w, const float* x, float* y, int rows, int n, float offset,
                 float* residual, const uint16_t* next_w, float* next_y) {
    for (int t = 0; t < rows; t++)
        norm_row(w, x + size_t(t) * n, y + size_t(t) * n, n, offset, residual ? residual + size_t(t) * n : nullptr,
                 next_w, next_y ? next_y + size_t(t) * n : nullptr);
}
void oracle_swiglu(const float* gates, float* out, int rows, int F) { swiglu_rows(gates, out, rows, F); }
uint32_t oracle_argmax_bits(const uint16_t* v, int n) { return argmax_bits(v, n); }
void oracle_exp(const float* x, float* y, long long n) { for (long long i = 0; i < n; i++) y[i] = pexp(x[i]); }
uint32_t oracle_argmax_f32(const float* v, int n) { return argmax_f32(v, n); }
void oracle_rope_tables(const float* inv_local, const float* inv_full, int local_rows, int context,
                        uint16_t* local_out, uint16_t* global_out) {
    Rope r; r.build(inv_local, inv_full, local_rows, context);
    std::memcpy(local_out, r.local.data(), r.local.size() * 2);
    std::memcpy(global_out, r.global.data(), r.global.size() * 2);
}

// Attention for one query row over an explicit cache, unfused (softmax path) or split-K.
// keys/values: [cap][kv_heads][128] bf16; q: [heads][128] fp32 (bf16-valued).
void oracle_attention(const uint16_t* keys, const uint16_t* values, const float* q, int heads, int kv_heads,
                      int cap, int first, int count, int begin, int end, int full,
                      const float* inv_local, int local_rows, int split, float* out) {
    State s;
    s.c = {0, 0, heads, kv_heads, 0, 0, 0, 1, std::max(1, local_rows)};
    std::vector<float> zeros(64, 0.0f);
    s.rope.build(inv_local, zeros.data(), local_rows, 1);
    RowGeo g{const_cast<uint16_t*>(keys), const_cast<uint16_t*>(values), cap, 0, 0, first, count, begin, end};
    if (split > 0) attend_row_splitk(s, full != 0, q, g, out, split);
    else attend_row(s, full != 0, q, g, out);
}

// Packed block decode (K:23-31): scalar bit reconstruction of element `index`.
void oracle_packed_decode(const uint8_t* data, const uint32_t* offsets, int64_t count, uint16_t* out) {
    for (int64_t index = 0; index < count; index++) {
        uint32_t block = uint32_t(index / 128), i = uint32_t(index % 128), entry = offsets[block], tag = entry & 63u;
        const uint8_t* blk = data + (entry & ~63u);
        uint32_t minimum = tag == 0 ? 0 : tag + 107u;
        if (minimum == 0) { uint16_t v; std::memcpy(&v, blk + 2 * i, 2); out[index] = v; continue; }
        uint32_t sm = blk[i], code = (blk[128 + i / 2] >> ((i % 2) * 4)) & 15u;
        uint32_t exponent = code == 15 ? 0 : minimum + code;
        out[index] = uint16_t((sm & 127u) | ((sm & 128u) << 8) | (exponent << 7));
    }
}

}  // extern "C"
