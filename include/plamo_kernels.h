/* libplamo_cuda kernel-level entry points: the hot-path kernels on caller-provided DEVICE
 * buffers, enqueued on `stream` (a cudaStream_t, NULL = default stream). They return 0 on a
 * successful launch, non-zero with plamo_last_error() set otherwise; completion is the caller's
 * stream synchronisation. bf16 values are passed as uint16_t bit patterns. Each entry point names
 * the reference Metal kernel it replaces (Sources/Plamo/Kernels.metal, Batch.metal).
 */
#ifndef PLAMO_KERNELS_H
#define PLAMO_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#ifndef PLAMO_API
#define PLAMO_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* linear (Kernels.metal:92-114), matrix (:149-200), project3/4 (Batch.metal:171-221).
 * y[r][m] = bf16(sum_k W[m][k] * x[r][k]) for r < rows, fp32 accumulation.
 * W: raw bf16 [M][K] (offsets == NULL), or a .p12 tensor: `w` = data region, `offsets` = tagged
 * block table (packed_four, Kernels.metal:33-44). K % 128 == 0.
 * mode 0: plain, y is [rows][M]. mode 1: SwiGLU epilogue (Kernels.metal:202-210): W has 2F rows,
 * y is [rows][F] = bf16(bf16(silu(g)) * u). mode 2: logits + first-index argmax
 * (Kernels.metal:704-729): y is [rows][M] bf16 logits and argmax_keys[r] (zeroed by the caller)
 * receives a 64-bit key, decoded by plamo_k_argmax_keys. */
PLAMO_API int plamo_k_linear(const void* w, const uint32_t* offsets, const uint16_t* x, int rows, int K, int M, int mode,
                   uint16_t* y, uint64_t* argmax_keys, void* stream);

/* The same projection on the tensor cores (tcgen05 GEMM, fp32 accumulation in tensor memory):
 * raw bf16 weights only (offsets are not taken), K a multiple of 64, any rows >= 1. The outputs
 * match plamo_k_linear within the rounding of the accumulation order. splits > 0 forces a K split
 * over that many CTAs per tile (<= 16 and <= K / 64), whose fp32 partials need
 * splits * rows * M floats of `workspace`; splits == 0 lets the launcher choose, splitting only
 * into the workspace given (workspace may then be NULL). */
PLAMO_API int plamo_k_linear_tc(const void* w, const uint16_t* x, int rows, int K, int M, int mode, uint16_t* y,
                                uint64_t* argmax_keys, int splits, float* workspace, size_t workspace_floats,
                                void* stream);

/* Sampler.select on caller-owned device buffers: logits [V] bf16, history [n] ids, scratch counts
 * [V] int32 and flags [V] bytes (cleared by the call); key_out receives the winning argmax key
 * (0 when no value is above -inf: the selected id is then 0, else 0xFFFFFFFF - low 32 bits).
 * Same semantics as plamo_select. */
PLAMO_API int plamo_k_select(const uint16_t* logits, int V, const int32_t* history, int n, float penalty,
                             int no_repeat_ngram, float frequency, float presence, int32_t* counts, uint8_t* flags,
                             uint64_t* key_out, void* stream);

/* Converts argmax keys to indices (0xFFFFFFFF when a row had only NaN). */
PLAMO_API int plamo_k_argmax_keys(const uint64_t* keys, int rows, uint32_t* out, void* stream);

/* norm (Kernels.metal:46-90): z = bf(bf(src*rsqrt(mean(src^2)+1e-6)) * bf(w+offset)).
 * residual == 0: x := z. residual != 0: x := bf(x + z) and, when next_w != NULL,
 * next := norm(x, next_w, offset 1). Rows of n <= 4096 values. */
PLAMO_API int plamo_k_norm(const uint16_t* w, const uint16_t* src, uint16_t* x, int rows, int n, float offset, int residual,
                 const uint16_t* next_w, uint16_t* next, void* stream);

/* argmax (Kernels.metal:704-729) over `rows` rows of n bf16 logits: first index of the maximum,
 * NaN never wins, all-NaN rows give 0xFFFFFFFF. `scratch` holds rows 64-bit keys. */
PLAMO_API int plamo_k_argmax(const uint16_t* logits, int rows, int n, uint64_t* scratch, uint32_t* out, void* stream);

/* packed_bits / packed_four (Kernels.metal:23-44): reconstructs `count` bf16 weights (count %
 * 16 == 0) from a .p12 data region and its tagged block table. */
PLAMO_API int plamo_k_packed_decode(const uint8_t* data, const uint32_t* entries, long long count, uint16_t* out, void* stream);

/* Split-K decode attention for one query row (attention + attention_merge, Kernels.metal:440-562;
 * matrix_rotary / softmax / attend, :301-437): q is heads*128 bf16 (already rotated);
 * keys/values are [cap][kv_heads][128] bf16. Keys r in [0,count) sit at slot (first + r) % cap;
 * the row sees r in [begin, end). Local layers (full == 0) re-rotate raw keys with coordinate r
 * using rope_local ([rows][64] u32 = cos bits | sin bits << 16). out: heads*128 bf16.
 * `splits` key partitions; the partial results live in library-owned device scratch that is
 * allocated on the first call and grown as needed (cudaMalloc). */
PLAMO_API int plamo_k_attention(const uint16_t* q, const uint16_t* keys, const uint16_t* values, int heads, int kv_heads,
                      int cap, int first, int count, int begin, int end, int full, const uint32_t* rope_local,
                      int splits, uint16_t* out, void* stream);

/* Attention of `rows` query rows over one cache (the prefill form of the split-K attention above,
 * Kernels.metal:301-562): q is [rows][heads*128] bf16 (already rotated); geo is a DEVICE array of
 * [rows][4] int32 {first, count, begin, end} per row as in plamo_k_attention (keys r in [0,count)
 * at slot (first + r) % cap, the row sees r in [begin, end)). tensor == 0: the CUDA-core kernels
 * with `splits` key partitions (bit-identical to the runtime's default path); tensor == 1: the
 * tcgen05 kernel of tensor mode's prefill (16 query heads over one KV head, splits chosen by the
 * library); tensor == 2: tensor mode's decode-row kernel (16 query heads over one KV head, warp-level
 * MMAs, the same `splits` as tensor == 0). 1 and 2 are within rounding of 0. Rows of one 16-token
 * chunk should be consecutive for tensor == 1; rows with
 * different windows are handled, at a lower rate. `workspace` (device, 256-byte aligned) holds the
 * row descriptors and split partials; a call that finds it too small fails with the bytes needed. */
PLAMO_API int plamo_k_attention_rows(const uint16_t* q, const uint16_t* keys, const uint16_t* values, int heads,
                                     int kv_heads, int cap, const int32_t* geo, int rows, int full,
                                     const uint32_t* rope_local, int splits, int tensor, uint16_t* out, void* workspace,
                                     size_t workspace_bytes, void* stream);

/* plamo_k_attention without any device allocation. No counterpart in the reference (whose Metal
 * encoder owns its buffers); for callers that must not allocate device memory during a call, such
 * as a serving loop that reserved its memory up front and can afford neither an out-of-memory
 * failure mid-stream nor the device-wide wait of the cudaFree with which plamo_k_attention grows
 * its scratch. Same arguments and results as plamo_k_attention. The partial results live in one
 * fixed 2 MiB device array per device (splits x heads at most 4032; larger requests fail with an
 * error and launch nothing). The first call on a device looks the array up (cudaGetSymbolAddress,
 * with that device current): make it before any stream capture. The address is kept for the life
 * of the process, so a device reset (cudaDeviceReset) in between invalidates it: do not call this
 * entry point on a device after resetting that device. Calls are asynchronous on
 * `stream` (they return once enqueued) and all calls on a device share the array, which keeps the
 * last call's contents: calls whose execution may overlap (other streams, other threads) race. */
PLAMO_API int plamo_k_attention_static(const uint16_t* q, const uint16_t* keys, const uint16_t* values, int heads,
                                       int kv_heads, int cap, int first, int count, int begin, int end, int full,
                                       const uint32_t* rope_local, int splits, uint16_t* out, void* stream);

/* The fp32 exponential used by the softmax and SwiGLU kernels (Kernels.metal:209, :386 use exp):
 * y[i] = e^x[i] from IEEE operations only (Cody-Waite reduction, degree-7 Taylor polynomial), so a
 * CPU restatement reproduces it exactly. n floats, device pointers. */
PLAMO_API int plamo_k_exp(const float* x, float* y, long long n, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* PLAMO_KERNELS_H */
