// Persistent batch-1 decode kernel: one launch per token (see decode_mega.cu).
#pragma once
#include "kernels.h"

namespace plamo {

enum MegaKind { MK_QKV = 0, MK_ATT = 1, MK_O = 2, MK_GU = 3, MK_DOWN = 4, MK_HEAD = 5 };

// One phase of the decode step. Weight phases compute `out_rows` outputs of `lin` (the SwiGLU
// phase: F outputs, each from gate row m and up row F + m).
struct MegaPhase {
    int kind, layer;
    Linear lin;
    int out_rows;
    int next_weight;  // index of the next weight (non-attention) phase; nphases after the last
};

struct MegaLayer {
    const uint16_t *pre_mixer, *post_mixer, *pre_mlp, *post_mlp, *q_norm, *k_norm;
    uint16_t *keys, *values;
    int cap, splits, per_max, full;
};

// Exchange vectors between phases carry their own readiness: every 32-bit word is
// (tag << 16) | bf16 value, every 64-bit word (tag << 32) | f32 bits, where the tag names the
// (step, layer) that wrote it. A consumer polls the words it needs until they carry the current
// tag, so a phase boundary costs one store-to-load trip through L2 and no counters or fences.
struct MegaArgs {
    const MegaPhase* phases;
    int nphases;
    int first_weight;  // index of the first weight phase
    const MegaLayer* layers;
    int L;
    const uint16_t* embed;
    const uint16_t* final_norm;
    const uint16_t* norms;  // [4L + 1][dpad] copy of every norm vector, 16-byte aligned rows
    int dpad;               // hidden size rounded up to 8
    const uint32_t* rope_local;
    const uint32_t* rope_global;
    int d, H, F, V, W;
    float post_mlp_offset;  // 1 / 5^1.5 (Runtime.swift:450)
    bool phases_packed;     // weights are .p12 tensors
    int attn_per_max;       // largest split width over the layers (shared-memory layout)
    int splits_max;         // largest split count over the layers
    int xs_bytes;           // staged activations at the start of the work region
    int tbl_bytes;          // .p12: shared copy of one phase's block-table rows of a CTA
    int* ids;          // [1] input token (device-chained: written by the previous step)
    RowDesc* desc;     // [1] position of the token (advanced by the step)
    uint32_t *qkv, *att, *po, *pd, *act;  // tagged phase outputs: q/k/v rows, attention, o_proj, down_proj, SwiGLU
    // Readiness hints, one word per producer (CTA, attention task or merged head) holding the tag
    // of its last finished phase: [0, G) q/k/v, [G, 2G) o_proj, [2G, 3G) SwiGLU, [3G, 4G) down_proj,
    // [4G, 4G + H) merged heads, then one per attention task. A consumer waits for its producers'
    // hints with one warp, then reads the tagged words once (re-polling the rare word whose store
    // is not yet visible), instead of every thread polling the data.
    uint32_t* hints;
    unsigned long long* part_o;   // [splits][H][128] tagged split partials P.V
    unsigned long long* part_ml;  // [splits][H][2] tagged split (max, sum)
    uint16_t* logits;
    uint16_t* hidden;
    unsigned long long* amkey;
    int* result;
    int* hist;
    int* hist_count;
    int hist_cap;
    unsigned* step;    // [1] steps run so far (source of the tags; never reset)
    unsigned* ticket;  // [1] CTAs done with the step (reset by the last one)
    int* error;        // set to a non-zero code when a bounded wait times out
    // Optional timeline (null when off): per CTA, per phase, %globaltimer ns at [wait begin, work
    // begin, work end], then one record [step begin, head epilogue begin, step end], then
    // after all CTAs' records, MEGA_TRACE_DETAIL stamps per CTA: its first attention task of layer 0
    // at [0, 5), layer 1's weight phases (QKV, o_proj, gate/up, down_proj) six each from index 8.
    unsigned long long* trace;
};
constexpr int MEGA_TRACE_STAMPS = 3;
constexpr int MEGA_TRACE_DETAIL = 32;

constexpr int MEGA_THREADS = 256;    // 8 warps
constexpr int MEGA_HG = 4;           // query heads per attention task
constexpr int MEGA_ATM = 64;         // keys per staged attention tile
constexpr int MEGA_FOLD_TASKS = 64;  // (row, segment) partials one CTA may hold in a split-row phase

size_t mega_smem_bytes(int per_max, int splits_max, int kmax, int nphases, int L, int tbl_bytes);
size_t mega_xs_bytes(int kmax);
int mega_npt(int d);
cudaError_t configure_mega(size_t smem, bool packed, int npt);
int mega_occupancy(size_t smem, bool packed, int npt);
cudaError_t launch_mega(const MegaArgs& a, int grid, size_t smem, cudaStream_t s);
// One bounded poll of `word` (which nothing sets) that gives up after limit_ns and raises `error`.
cudaError_t launch_wait_unset(const uint32_t* word, int* error, unsigned long long limit_ns, cudaStream_t s);

}  // namespace plamo
