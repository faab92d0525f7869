// Persistent batch-1 decode kernel: one launch per token (see decode_mega.cu).
#pragma once
#include "kernels.h"

namespace plamo {

enum MegaKind { MK_QKV = 0, MK_ATT = 1, MK_O = 2, MK_GU = 3, MK_DOWN = 4, MK_HEAD = 5 };

// One phase of the decode step. Weight phases stream `lin` in tiles of `tile_rows` whole rows
// (one contiguous byte range per tile; the SwiGLU phase streams a gate tile and an up tile per
// block of outputs).
struct MegaPhase {
    int kind, layer;
    Linear lin;
    const uint32_t* rowoff;  // .p12: byte offset of each row's first block in the data region (M+1)
    int out_rows;            // outputs of the phase (SwiGLU: F)
    int tile_rows;           // weight rows per tile
    int next_weight;         // index of the next weight (non-attention) phase; nphases after the last
    const void* tmap;        // raw weights: 3-D tensor map [rows][K/64][64] bf16, 128-byte swizzle (device memory)
};

struct MegaLayer {
    const uint16_t *pre_mixer, *post_mixer, *pre_mlp, *post_mlp, *q_norm, *k_norm;
    uint16_t *keys, *values;
    int cap, splits, per_max, full;
};

struct MegaArgs {
    const MegaPhase* phases;
    int nphases;
    int first_weight;  // index of the first weight phase
    const MegaLayer* layers;
    int L;
    const uint16_t* embed;
    const uint16_t* final_norm;
    const uint32_t* rope_local;
    const uint32_t* rope_global;
    int d, H, KV, F, V, W;
    float post_mlp_offset;  // 1 / 5^1.5 (Runtime.swift:450)
    bool phases_packed;     // weights are .p12 tensors
    int attn_per_max;       // largest split width over the layers (shared-memory layout)
    int xs_bytes;           // staged activations at the start of the union region; split-row sums follow
    int* ids;          // [1] input token (device-chained: written by the previous step)
    RowDesc* desc;     // [1] position of the token (advanced by the step)
    uint16_t *qkv, *att, *po, *pd, *act;  // phase outputs: q/k/v rows, attention, o_proj, down_proj, SwiGLU
    float* part_o;
    float2* part_ml;
    uint16_t* logits;
    uint16_t* hidden;
    unsigned long long* amkey;
    int* result;
    int* hist;
    int* hist_count;
    int hist_cap;
    unsigned* sync;    // [nphases] phase counters, [L] split tickets, [1] final ticket (all reset by the step)
    int* error;        // set to a non-zero code when a bounded wait times out
    // Optional timeline (null when off): per CTA, per phase, %globaltimer ns at [wait begin, work
    // begin, work end], then one record [step begin, head epilogue begin, step end].
    unsigned long long* trace;
};
constexpr int MEGA_TRACE_STAMPS = 3;
constexpr int MEGA_TRACE_DETAIL = 32;  // per CTA, after the phase records: stamps inside the first attention split,
                                       // then stamps of the first SwiGLU phase's tile pairs

constexpr int MEGA_THREADS = 256;  // 8 warps (2 per scheduler: up to 255 registers each)
constexpr int MEGA_SLOTS = 6;
constexpr int MEGA_SLOT_DATA = 24576;    // weight bytes per ring slot (a multiple of 1024)
constexpr int MEGA_TABLE_BYTES = 512;    // .p12 block-table bytes per ring slot
constexpr int MEGA_GLU_ROWS = 512;  // SwiGLU rows one CTA may own

size_t mega_attention_smem(int H, int KV, int per_max);
size_t mega_smem_bytes(int H, int KV, int per_max, int kmax);
bool mega_merge_fits(int H, int KV, int splits);
size_t mega_xs_bytes(int kmax);
int mega_tile_rows(int K);
int mega_npt(int d);
cudaError_t configure_mega(size_t smem, bool packed, int npt);
int mega_occupancy(size_t smem, bool packed, int npt);
cudaError_t launch_mega(const MegaArgs& a, int grid, size_t smem, cudaStream_t s);

}  // namespace plamo
