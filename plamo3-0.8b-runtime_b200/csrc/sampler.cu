// Decoding controls of the reference CLI on the device: Sampler.select (Sampler.swift:9-31) reads
// the next-token logits where the head wrote them, so a controlled step moves the history ids to
// the device (4 bytes each) instead of the 107,520 logits to the host (Runtime.swift:540-552).
//
// Two launches after three small clears:
// - k_select_mark, one thread per history position: counts[id] += 1 for every in-range id, and
//   flags[id] = 1 for each id that would complete an (n-1)-gram equal to the history's tail
//   (Sampler.forbidden, Sampler.swift:54-70);
// - k_select_argmax over the vocabulary: the repetition penalty (divide positive logits, multiply
//   the rest), the presence and the frequency penalty (times the count) for ids in the history,
//   -inf for flagged ids, then the first index of the largest value through 64-bit keys
//   (value order, then lower index; -0 == +0). Values that are NaN or -inf never win, so a vocabulary
//   without a finite or +inf value selects id 0, as the Swift loop does.
// Every step is an exact function of its inputs (integer counts, one IEEE operation each), so the
// result is identical to the CPU restatement.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace plamo {

namespace {

__global__ void k_select_mark(const int* hist, int n, int V, int use_counts, int ngram, int* counts, uint8_t* flags) {
    const int i = int(blockIdx.x) * blockDim.x + threadIdx.x;
    if (use_counts && i < n) {
        const int id = hist[i];
        if (id >= 0 && id < V) atomicAdd(counts + id, 1);
    }
    if (ngram > 1 && n >= ngram) {
        const int span = ngram - 1, last = n - span;
        if (i < last) {
            bool match = true;
            for (int o = 0; o < span; o++)
                if (hist[i + o] != hist[last + o]) {
                    match = false;
                    break;
                }
            if (match) {
                const int id = hist[i + span];
                if (id >= 0 && id < V) flags[id] = 1;
            }
        }
    }
}

__global__ void __launch_bounds__(256) k_select_argmax(const uint16_t* logits, int V, const int* counts,
                                                        const uint8_t* flags, float penalty, float frequency,
                                                        float presence, unsigned long long* key_out) {
    unsigned long long best = 0ull;
    for (int i = int(blockIdx.x) * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) {
        float v = bf2f(logits[i]);
        if (counts) {
            const int c = counts[i];
            if (c > 0) {
                if (penalty != 1.0f) v = v > 0.0f ? v / penalty : v * penalty;
                if (presence != 0.0f) v = v - presence;
                if (frequency != 0.0f) v = v - frequency * float(c);
            }
        }
        if (flags && flags[i]) v = -INFINITY;
        if (v > -INFINITY) {
            const unsigned long long k = argmax_key(v, uint32_t(i));
            best = k > best ? k : best;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(FULL_MASK, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0 && best) atomicMax(key_out, best);
}

}  // namespace

cudaError_t launch_select(const uint16_t* logits, int V, const int* hist, int n, float penalty, int ngram,
                          float frequency, float presence, int* counts, uint8_t* flags, unsigned long long* key,
                          cudaStream_t s) {
    const bool use_counts = penalty != 1.0f || presence != 0.0f || frequency != 0.0f;  // Sampler.swift:11
    const bool use_flags = ngram > 1 && n >= ngram;                                     // Sampler.swift:20,55
    cudaError_t e = cudaMemsetAsync(key, 0, sizeof(unsigned long long), s);
    if (e == cudaSuccess && use_counts) e = cudaMemsetAsync(counts, 0, sizeof(int) * size_t(V), s);
    if (e == cudaSuccess && use_flags) e = cudaMemsetAsync(flags, 0, size_t(V), s);
    if (e != cudaSuccess) return e;
    if ((use_counts || use_flags) && n > 0) {
        k_select_mark<<<(n + 255) / 256, 256, 0, s>>>(hist, n, V, use_counts ? 1 : 0, use_flags ? ngram : 0, counts,
                                                      flags);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    const int blocks = std::min((V + 255) / 256, 296);
    k_select_argmax<<<blocks, 256, 0, s>>>(logits, V, use_counts ? counts : nullptr, use_flags ? flags : nullptr,
                                           penalty, frequency, presence, key);
    return cudaGetLastError();
}

int select_key_to_id(unsigned long long key) { return key ? int(0xffffffffu - uint32_t(key & 0xffffffffull)) : 0; }

// Sampler.repetitionPeriod (Sampler.swift:35-51).
int repetition_period(const int32_t* tokens, int n, int repeats) {
    if (repeats < 2 || n < repeats) return 0;
    for (int period = 1; period <= 32; period++) {
        const int count = std::max(repeats, (24 + period - 1) / period);
        const long long span = static_cast<long long>(period) * count;
        if (n < span) continue;
        const long long start = n - span;
        bool periodic = true;
        for (long long o = 0; o < span; o++)
            if (tokens[start + o] != tokens[start + o % period]) {
                periodic = false;
                break;
            }
        if (periodic) return period;
    }
    return 0;
}

}  // namespace plamo
