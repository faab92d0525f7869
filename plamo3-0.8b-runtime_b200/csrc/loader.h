// Host-side model loading: config parsing, safetensors and .p12 validation, SHA-256.
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace plamo {

struct Json {
    enum Type { NUL, BOOL, NUM, STR, ARR, OBJ } type = NUL;
    bool b = false;
    double num = 0;
    bool is_int = false;
    long long inum = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;
    const Json* get(const std::string& k) const;
    bool int_value(long long& out) const;
};
bool parse_json(const char* data, size_t len, Json& out, std::string& err);

struct Config {
    int d = 1536, layers = 16, heads = 16, kv_heads = 1, head_dim = 128, ffn = 6144, vocab = 107520,
        window = 2048, pattern = 8;
    bool is_global(int layer) const { return layer % pattern == pattern - 1; }
    int qkv_rows() const { return (heads + 2 * kv_heads) * head_dim; }
    int q_dim() const { return heads * head_dim; }
};

struct MappedFile {
    const uint8_t* data = nullptr;
    size_t size = 0;
    ~MappedFile();
    bool open(const std::string& path, std::string& err);
};

struct TensorRef {
    const uint8_t* data = nullptr;   // host pointer into the mapped file
    size_t bytes = 0;
    std::vector<long long> shape;
    // packed (.p12) 2-D tensors: block table + data region (payload-relative offsets)
    bool packed = false;
    size_t table_off = 0, table_bytes = 0, data_off = 0, data_bytes = 0, raw_off = 0;
};

struct ModelFiles {
    Config cfg;
    float inv_local[64], inv_full[64];
    MappedFile st;       // model.safetensors
    size_t st_data_start = 0;
    std::map<std::string, TensorRef> st_tensors;
    MappedFile p12;      // model.p12 (packed mode)
    size_t p12_data_start = 0, p12_payload = 0;
    std::map<std::string, TensorRef> p12_tensors;
    // Reads config.json + config-mlx.json + model.safetensors (and model.p12 when packed).
    bool load(const std::string& dir, bool packed, std::string& err);
    // Validated view of one tensor of the expected shape (Runtime.swift:87-101 / Packed.swift:49-91).
    bool tensor(const std::string& name, const std::vector<long long>& shape, bool from_p12, TensorRef& out,
                std::string& err) const;
};

std::string sha256_hex(const uint8_t* data, size_t len);

// Validates a .p12 block table chain (Packed.swift:63-89): entry i's offset equals the running
// end, every block fits in the data region, and the chain ends exactly at the region's end.
bool validate_chain(const uint32_t* entries, size_t count, size_t data_bytes);

extern const char* const kReferenceSourceSha;

}  // namespace plamo
