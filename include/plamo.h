/* libplamo_cuda: B200 (sm_100a) backend for the PLaMo-3 0.8B decoder hot path.
 *
 * C ABI that replaces the Metal compute layer of mikuteto-dev/plamo3-0.8b-runtime one to one:
 * the members of `Runtime` (Sources/Plamo/Runtime.swift) and `Batch` (Sources/Plamo/Batch.swift)
 * that the Swift engine calls. Plain pointers and sizes only; every call is synchronous (it returns
 * after the device work and the result copy finished, like the reference's waitUntilCompleted) and
 * reports failure through its status: 0 = success, non-zero = failure with the message available
 * from plamo_last_error() (thread-local). Handles are single-threaded; separate handles on separate
 * devices may be used concurrently. The library owns all device memory; callers own host arrays,
 * which are copied before the call returns.
 */
#ifndef PLAMO_H
#define PLAMO_H

#include <stddef.h>
#include <stdint.h>

#ifndef PLAMO_API
#define PLAMO_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct plamo_runtime plamo_runtime;
typedef struct plamo_batch plamo_batch;

/* Runtime.init(directory:context:packed:) — Runtime.swift:164-286.
 * Loads <model_dir>/config.json, config-mlx.json and model.safetensors (+ model.p12 when packed),
 * validates them (Runtime.swift:181-189, :33-101; Packed.swift:12-91; an archive must name the
 * reference checkpoint's digest, or with PLAMO_P12_LOCAL_SOURCE=1 the model.safetensors beside it)
 * and makes the weights
 * resident on CUDA device `device`. context: 1...32768. */
PLAMO_API int plamo_open(const char* model_dir, int context, int packed, int device, plamo_runtime** out);

/* Same as plamo_open, but the weights are received from rank 0 with one ncclBroadcast of the
 * weight arena over NVLink instead of being read from disk on every rank (ranks > 0 still read
 * config.json/config-mlx.json and the archive headers). `nccl_id` is the 128-byte ncclUniqueId
 * created on rank 0 (plamo_nccl_unique_id) and shared out of band. No reference counterpart: the
 * reference is single-GPU; this is the data-parallel loader. */
PLAMO_API int plamo_open_broadcast(const char* model_dir, int context, int packed, int device,
                         const void* nccl_id, int rank, int world, plamo_runtime** out);
PLAMO_API int plamo_nccl_unique_id(void* out_128_bytes);
/* The communicator setup of plamo_open_broadcast alone (no model, no device memory), for failure
 * tests of the data-parallel open: creates the NCCL communicator non-blocking and polls it until it
 * is ready, fails, or limit_ms passes (plamo_open_broadcast uses PLAMO_NCCL_TIMEOUT_MS, default
 * 120000), aborting it on failure or timeout, then destroys it. A rank whose peers never join gets
 * "NCCL communicator setup timed out ..." instead of waiting forever. PLAMO_NCCL_LIBRARY in the
 * environment names the NCCL library to load first. Returns 0, or 1 with plamo_last_error set. */
PLAMO_API int plamo_debug_nccl_init(const void* nccl_id, int rank, int world, long long limit_ms);
/* Seconds spent in the load-time weight broadcast (0 when loaded from disk). */
PLAMO_API double plamo_broadcast_seconds(const plamo_runtime*);

PLAMO_API void plamo_close(plamo_runtime*);

/* Runtime.prefill(_:) — Runtime.swift:469-483: feeds ids in 16-token chunks; returns the greedy
 * next id of the last position in *next_id. Errors: "Input exceeds context". */
PLAMO_API int plamo_prefill(plamo_runtime*, const int32_t* ids, int n, int32_t* next_id);

/* Runtime.forward(_:output:) — Runtime.swift:321-467: 1...min(context,16) ids at the current
 * position; with output != 0 writes the greedy next id (else -1).
 * Errors: "Invalid tokens or context exhausted". */
PLAMO_API int plamo_forward(plamo_runtime*, const int32_t* ids, int n, int output, int32_t* next_id);

/* Runtime.logits(into:slot:) / logitValues() — Runtime.swift:540-552: the last output row's
 * bf16 logits widened to vocab_size floats. */
PLAMO_API int plamo_logits(plamo_runtime*, int slot, float* out);

/* Final-normed hidden row of the last output (Runtime.normalized after the head), hidden_size floats. */
PLAMO_API int plamo_hidden(plamo_runtime*, float* out);

PLAMO_API void plamo_reset(plamo_runtime*);                    /* Runtime.reset() — Runtime.swift:319 */
PLAMO_API int plamo_position(const plamo_runtime*);            /* Runtime.position */
PLAMO_API double plamo_gpu_seconds(const plamo_runtime*);      /* Runtime.gpuSeconds (device time, events) */
PLAMO_API size_t plamo_weight_bytes(const plamo_runtime*);     /* Weights.gpuBytes — bytes of resident weights */
PLAMO_API size_t plamo_device_bytes(const plamo_runtime*);     /* Runtime.peakMetalBytes — device bytes allocated */
PLAMO_API const char* plamo_device_name(const plamo_runtime*); /* device.name */
/* Model dimensions: hidden, layers, heads, kv_heads, head_dim, ffn, vocab, window, pattern, context. */
PLAMO_API int plamo_dims(const plamo_runtime*, int32_t out[10]);

/* Batch(runtime) — Batch.swift:33-78. lanes: 1...64 (the reference CLI uses 4). Requires
 * context < 8192 (Batch.swift:34-35). */
PLAMO_API int plamo_batch_open(plamo_runtime*, int lanes, plamo_batch** out);

/* Batch.prefill(_:) — Batch.swift:80-106: prompt i goes to lane i (n <= lanes); next_ids[i] is the
 * greedy next id of lane i. Errors: "Expected one to four valid prompts". */
PLAMO_API int plamo_batch_prefill(plamo_batch*, const int32_t* const* prompts, const int32_t* lens, int n, int32_t* next_ids);

/* Batch.step(_:) — Batch.swift:109-179: tokens[i] < 0 marks an inactive lane; n must equal the
 * number of prefilled lanes; next_ids receives every lane's latest prediction.
 * Errors: "Invalid quad step or context exhausted". */
PLAMO_API int plamo_batch_step(plamo_batch*, const int32_t* tokens, int n, int32_t* next_ids);

/* Batch.logits (per-lane bf16 logits, widened) and Batch.hidden rows. */
PLAMO_API int plamo_batch_logits(plamo_batch*, int lane, float* out);
PLAMO_API int plamo_batch_hidden(plamo_batch*, int lane, float* out);

PLAMO_API void plamo_batch_reset(plamo_batch*);                  /* Batch.reset() — Batch.swift:182 */
PLAMO_API double plamo_batch_gpu_seconds(const plamo_batch*);    /* Batch.gpuSeconds */
PLAMO_API void plamo_batch_close(plamo_batch*);

/* decodeBatch — BatchDecode.swift:8-38 (Batch.generate, :41-47): prefill + greedy decode of n
 * prompts with per-lane output limits; stop ids 1 and 16 end a lane ("stop"), reaching its limit
 * ends it ("length"); stop_on_truncation drops lanes after the first truncated one. Outputs:
 * out_ids[i*out_stride ...] (out_lens[i] ids), reasons[i] = 0 stop / 1 length. On error the batch is
 * reset (BatchDecode.swift:45-46). Returns the number of lanes reported in *out_count. */
PLAMO_API int plamo_batch_generate(plamo_batch*, const int32_t* const* prompts, const int32_t* lens, const int32_t* limits,
                         int n, int stop_on_truncation, int32_t* out_ids, int out_stride, int32_t* out_lens,
                         int32_t* reasons, int32_t* out_count);

/* Debug/state access used by the parity tests: copies one layer's KV cache (scalar runtime, or one
 * lane of a batch) as bf16 bits in the reference's ring layout, capacity*kv_heads*128 values each:
 * global layers hold every position (capacity = context); local layers show the reference's ring of
 * min(context, window + 16) slots (Runtime.swift:240), the key of position k of the last
 * `capacity` positions at slot k % capacity (the library's own ring is longer, so a prefill call
 * can take a long prompt's chunks in one pass). */
PLAMO_API int plamo_debug_kv(plamo_runtime*, int layer, uint16_t* keys, uint16_t* values);
PLAMO_API int plamo_batch_debug_kv(plamo_batch*, int layer, int lane, uint16_t* keys, uint16_t* values);

/* Device-chained greedy decode for benchmarking: runs `steps` batch-1 decode steps back to back on
 * the device (each step feeds its argmax to the next, no host round trip), starting from the last
 * prediction. Writes the generated ids to out_ids. Equivalent to `steps` plamo_forward calls. */
PLAMO_API int plamo_decode_chain(plamo_runtime*, int steps, int32_t* out_ids);

/* Number of kernel launches in one batch-1 decode step: 1 with the persistent decode kernel, else
 * the nodes of the captured multi-kernel decode graph. */
PLAMO_API int plamo_step_launches(plamo_runtime*);

/* 1 when batch-1 decode runs as one persistent cooperative kernel per token (the default on
 * sm_100a; PLAMO_PERSISTENT=0 in the environment selects the multi-kernel graph instead). */
PLAMO_API int plamo_persistent_decode(const plamo_runtime*);

/* Failure-path check of the persistent decode kernel (no reference counterpart; the reference's
 * command buffers report errors through their status, Runtime.swift:462): runs the kernel's bounded
 * poll on a device word that nothing ever sets, with a limit of limit_ns (1 us ... 2 s) instead of
 * the 2 s every decode wait uses. The poll gives up, raises the kernel's error word, and the call
 * fails exactly as a timed-out decode step does ("decode step aborted: a bounded device wait timed
 * out (code 12)"); afterwards the runtime is usable and its next steps are exact. Needs the
 * persistent kernel (plamo_persistent_decode). */
PLAMO_API int plamo_debug_wait_timeout(plamo_runtime*, unsigned long long limit_ns);

/* Dense contractions on the tensor cores ("tensor mode"), a bit mask. Bit 0: every projection over
 * 16 or more rows of raw bf16 weights (prefill calls, batched steps and batched prefill of this
 * runtime and its batches) runs as a tcgen05 GEMM with fp32 accumulation. Bit 1: the attention of
 * every call over 16 or more rows runs its scores and P.V on the tensor cores: prefill chunks as
 * tcgen05 MMAs, the decode rows of a batched step as warp-level bf16 MMAs (16 query heads over one
 * KV head; other shapes keep the CUDA-core kernel). 3 selects both. The
 * results then match the default path within the rounding of the accumulation order (next-token
 * logits within the drift the reference's own reordered sums show), not bit for bit; batch-1
 * decode and .p12 weights are unaffected. Off (0) by default. Returns 0, or 1 for a null handle. */
PLAMO_API int plamo_set_tensor_gemm(plamo_runtime*, int enable);

/* Sampler.select (Sampler.swift:9-31) on the device, over the logits of slot 0 as
 * plamo_logits would return them: for ids in history[0..n) (Main.swift passes the generated
 * tokens), the repetition penalty (positive logits divided by `penalty`, others multiplied), then
 * `presence` subtracted, then `frequency` x the id's count subtracted, applied when penalty != 1 or
 * presence != 0 or frequency != 0; with no_repeat_ngram > 1, ids that would complete an n-gram
 * already in the history (Sampler.forbidden, Sampler.swift:54-70) become -inf; then the first
 * index of the largest value (NaN and -inf never win; 0 when nothing is above -inf). Only the
 * history travels to the device; the logits stay where the head wrote them and are not modified.
 * Returns 0 and writes *out_id, or 1 ("Invalid select arguments" / a CUDA error). */
PLAMO_API int plamo_select(plamo_runtime*, const int32_t* history, int n, float penalty, int no_repeat_ngram,
                           float frequency, float presence, int32_t* out_id);

/* Sampler.repetitionPeriod (Sampler.swift:35-51), host code: the shortest period 1...32 such that
 * the tail of tokens[0..n) is that block repeated max(repeats, ceil(24 / period)) times; 0 when
 * there is none (the Swift nil) or repeats < 2. Needs no device. */
PLAMO_API int plamo_repetition_period(const int32_t* tokens, int n, int repeats);

/* Writes model.p12 beside model.safetensors in model_dir: the lossless plamo-bf16-pack-v2 archive
 * of scripts/pack_weights.py:89-135, byte for byte what that packer writes (every 2-D tensor but
 * the input embedding block-packed, 1-D tensors raw, safetensors-header order). source_sha256: the
 * manifest's digest (NULL: the SHA-256 of model.safetensors, which the loader accepts only when
 * PLAMO_P12_LOCAL_SOURCE=1 is set in the environment; by default it accepts the reference
 * checkpoint's digest alone, as Packed.swift:35 does).
 * stats (optional, 5 values): original linear bytes, packed linear bytes, archive bytes, packed
 * blocks, blocks. Returns 0, or 1 with plamo_last_error set ("Packing changed BF16 bits" if a
 * block fails its round trip). Host code; needs no device. */
PLAMO_API int plamo_pack_p12(const char* model_dir, const char* source_sha256, uint64_t* stats);

/* The loader's check of one tensor's .p12 block table (Packed.swift:63-89): entry i's offset is
 * the running end of the blocks before it (192 bytes packed, 256 raw by the entry's tag), every
 * block fits in the data_bytes data region, and the chain ends exactly there. 1 when valid, else 0.
 * Host code; plamo_open applies it to every packed tensor. */
PLAMO_API int plamo_p12_chain_valid(const uint32_t* entries, size_t count, size_t data_bytes);

/* The block codec alone (pack_weights.py:19-74): packs count bf16 values (a multiple of 128) into
 * data (capacity data_cap, at most 2 * count bytes) and one tagged u32 entry per block; data_bytes
 * receives the bytes used. Host code. */
PLAMO_API int plamo_pack_blocks(const uint16_t* values, size_t count, uint8_t* data, size_t data_cap, uint32_t* entries,
                                size_t* data_bytes);

/* Profiling: runs `steps` batch-1 decode steps (as plamo_decode_chain) with every kernel launch
 * bracketed by CUDA events. class_ms[6] / launches[6] receive the summed device milliseconds and
 * launch counts per kernel class: 0 GEMV (projections, lm_head), 1 QK-norm + RoPE + KV append,
 * 2 attention, 3 norms + embedding, 4 argmax finalisation (multi-kernel path), 5 the persistent
 * decode kernel (whole step). */
PLAMO_API int plamo_profile_decode(plamo_runtime*, int steps, double* class_ms, int32_t* launches);

/* Tracing: one batch-1 decode step (as plamo_decode_chain with steps = 1) of the persistent decode
 * kernel with its device timeline recorded. shape = {CTAs, phases, 3, D}; out receives, per CTA, per
 * phase, the %globaltimer nanoseconds at [wait begin, work begin, work end], then one record per CTA
 * [step begin, head epilogue begin, step end] — CTAs x (phases + 1) x 3 entries — followed by D
 * stamps per CTA (0 where unused): [0, 5) inside its first attention split of layer 0, then for
 * layer 1's QKV, o_proj, gate/up and down_proj phases (k = 0..3) six stamps at 8 + 6k: entry,
 * producers' hints seen, input gathered, prologue done, chunk loop done, outputs stored; cap must hold
 * CTAs x ((phases + 1) x 3 + D) entries. Phases per layer: QKV, attention, o_proj, gate/up (SwiGLU),
 * down_proj; then the lm_head. */
PLAMO_API int plamo_trace_decode(plamo_runtime*, uint64_t* out, size_t cap, int32_t* shape);

PLAMO_API const char* plamo_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* PLAMO_H */
