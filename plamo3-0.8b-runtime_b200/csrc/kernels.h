// Kernel launch interface shared by the runtime (runtime.cu) and the kernel-level C ABI.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cstdint>
#include <cuda_runtime.h>

namespace plamo {

// One projection weight: raw bf16 [M][K] (offsets == nullptr) or a .p12 tensor (data region +
// tagged u32 block table, one entry per 128 weights).
struct Linear {
    const uint8_t* w = nullptr;
    const uint32_t* offsets = nullptr;
    int M = 0, K = 0;
};

// Per query row: absolute position, lane (batch slab), and the start/length of the forward call
// ("chunk") the row belongs to. The chunk start sets the local window base exactly as the
// reference does for a 16-token chunk (Runtime.swift:389-395).
struct RowDesc { int pos, lane, cstart, crows; };

// Per query row attention geometry (computed on device by the qkv kernel): keys r in [0,count)
// live at slot (first + r) % cap of the row's lane slab; the row sees r in [begin, end).
struct RowGeo { int first, count, begin, end; };

enum GemvMode { GEMV_PLAIN = 0, GEMV_SWIGLU = 1, GEMV_LOGITS = 2 };

struct GemvArgs {
    Linear lin;
    const uint16_t* x = nullptr;   // [rows][K] bf16
    int rows = 1;
    uint16_t* y = nullptr;         // [out_row][ystride]
    int ystride = 0;
    const int* out_map = nullptr;  // optional row -> output row (batch lanes)
    unsigned long long* keys = nullptr;  // GEMV_LOGITS: argmax keys per output row
    int tensor = 0;                // dense rows (>= 16) of raw weights go to the tcgen05 GEMM
    float* part = nullptr;         // tcgen05 split-K partials (optional workspace)
    size_t part_cap = 0;           // floats in `part`
    int* split_out = nullptr;      // plain mode, no out_map: a K split leaves its partials in `part`
                                   // for the next kernel (no finish launch) and stores the split
                                   // count here; 0 when y was written
};

struct AttnArgs {
    const uint16_t* q = nullptr;       // [rows][H*128] rotated queries
    const uint16_t* keys = nullptr;    // cache base; lane slab = lane * lane_stride elements
    const uint16_t* values = nullptr;
    const RowDesc* desc = nullptr;
    const RowGeo* geo = nullptr;
    const uint32_t* rope_local = nullptr;  // [rows][64] (cos | sin << 16) bf16 pairs
    float* part_o = nullptr;           // [rows][splits][H][128]
    float2* part_ml = nullptr;         // [rows][splits][H]
    uint16_t* out = nullptr;           // [rows][H*128]
    long long lane_stride = 0;
    int rows = 1, H = 16, KV = 1, cap = 0, full = 0, splits = 1, per_max = 0;
    int key_bound = 0;  // tensor-core attention: no row sees key index >= key_bound (0: cap)
};

struct QkvArgs {
    const uint16_t* qkv = nullptr;     // [rows][(H+2KV)*128]
    const uint16_t* q_norm = nullptr;
    const uint16_t* k_norm = nullptr;
    uint16_t* q = nullptr;             // [rows][H*128]
    uint16_t* keys = nullptr;
    uint16_t* values = nullptr;
    const RowDesc* desc = nullptr;
    RowGeo* geo = nullptr;             // written (local or global variant for this layer)
    const uint32_t* rope_local = nullptr;
    const uint32_t* rope_global = nullptr;
    long long lane_stride = 0;
    int rows = 1, H = 16, KV = 1, cap = 0, W = 2048, full = 0;
    const float* src_part = nullptr;  // src_splits > 0: qkv is the bf16 rounding of the split sum of
    int src_splits = 0;               // src_part [split][rows][(H+2KV)*128], in split order
};

struct NormArgs {
    const uint16_t* w = nullptr;
    const uint16_t* src = nullptr;     // [rows][n]
    uint16_t* x = nullptr;             // residual stream (in/out) or plain output when !residual
    const uint16_t* next_w = nullptr;  // fused next norm (offset 1) or nullptr
    uint16_t* next = nullptr;
    uint16_t* y2 = nullptr;            // plain mode: optional second copy at row out_map[r]
    const int* out_map = nullptr;
    int rows = 1, n = 0;
    float offset = 0.f;
    int residual = 0;
    const float* src_part = nullptr;  // src_splits > 0: the source rows are the bf16 rounding of
    int src_splits = 0;               // the split sum of src_part [split][rows][n], in split order
};

// Launchers (return cudaError_t of the launch).
cudaError_t launch_embed_norm(const int* ids, int rows, int vocab, const uint16_t* embed, const uint16_t* w, int d,
                              uint16_t* x, uint16_t* h, unsigned long long* keys, const int* key_map,
                              int nkeys, cudaStream_t s);
cudaError_t launch_norm(const NormArgs& a, cudaStream_t s);
cudaError_t launch_gemv(const GemvArgs& a, int mode, cudaStream_t s);
// cuTensorMapEncodeTiled from the driver, found through the runtime (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();
// Tiled order-exact GEMM (gemm.cu) for more than 16 rows of raw weights; launch_gemv uses it.
bool gemm_supported(const GemvArgs& a);
cudaError_t launch_gemm(const GemvArgs& a, GemvMode mode, cudaStream_t s);
cudaError_t configure_gemm();
// tcgen05 GEMM (gemm_tc.cu): bf16 operands, fp32 accumulation on the tensor cores; matches the
// exact path to within the rounding of the accumulation, not bit for bit. splits_override > 0
// forces the K split (tests).
bool gemm_tc_supported(const GemvArgs& a);
cudaError_t launch_gemm_tc(const GemvArgs& a, GemvMode mode, cudaStream_t s, int splits_override = 0);
cudaError_t configure_gemm_tc();
// Error word of the tiled GEMMs on the current device (created on first use when `create`);
// gemm_take_error reads and clears it (0: no stage wait gave up since the last call).
int* gemm_error_word(bool create);
int gemm_take_error();
constexpr int TC_MIN_ROWS = 16;  // fewer rows stay on the order-exact GEMV
cudaError_t launch_qkv(const QkvArgs& a, cudaStream_t s);
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s);
// The split merge alone (k_attn_merge over a.splits partials per row).
cudaError_t launch_attention_merge(const AttnArgs& a, cudaStream_t s);
// Prefill attention on the tensor cores (attn_tc.cu): 16 query heads over one KV head, each row's
// keys in attention_tc_splits(cap) splits; partials and merge as launch_attention, results within
// rounding of it (tensor mode only).
bool attention_tc_supported(const AttnArgs& a);
int attention_tc_splits(int keys);  // keys: the cache capacity or a smaller bound on the rows' key counts
cudaError_t launch_attention_tc(const AttnArgs& a, cudaStream_t s);
cudaError_t configure_attention_tc();
// Decode rows' attention on the tensor cores (attn_mma.cu, tensor mode): 16 query heads over one KV
// head, warp-level bf16 MMAs, k_attn_partial's splits, partials and merge; results within rounding
// of launch_attention.
bool attention_mma_supported(const AttnArgs& a);
cudaError_t launch_attention_mma(const AttnArgs& a, cudaStream_t s);
cudaError_t configure_attention_mma();
cudaError_t launch_finalize(unsigned long long* keys, const int* key_map, int rows, int* result,
                            int* chain_ids, RowDesc* advance, int* hist, int* hist_count, int hist_cap,
                            cudaStream_t s);
cudaError_t launch_argmax(const uint16_t* logits, int rows, int n, unsigned long long* keys, uint32_t* out,
                          cudaStream_t s);
cudaError_t launch_packed_decode(const uint8_t* data, const uint32_t* entries, long long count, uint16_t* out,
                                 cudaStream_t s);
// Sampler.select on the device (sampler.cu): counts [V] ints and flags [V] bytes of scratch, key
// receives the winning 64-bit argmax key (0: no value above -inf, id 0).
cudaError_t launch_select(const uint16_t* logits, int V, const int* hist, int n, float penalty, int ngram,
                          float frequency, float presence, int* counts, uint8_t* flags, unsigned long long* key,
                          cudaStream_t s);
int select_key_to_id(unsigned long long key);
int repetition_period(const int32_t* tokens, int n, int repeats);
cudaError_t configure_kernels();
int attention_per_max(int cap, int splits);
size_t attention_smem(int H, int KV, int per_max);

}  // namespace plamo
