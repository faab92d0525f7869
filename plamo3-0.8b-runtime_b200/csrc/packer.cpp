// `.p12` (plamo-bf16-pack-v2) writer in C++: the block codec of scripts/pack_weights.py:19-74 and
// the archive layout of its main() (:89-135), so packing needs neither Python nor numpy.
//
// Block codec, 128 bf16 values per block:
// - every value whose low 15 bits are non-zero has exponent e = (v >> 7) & 255;
// - the block is packed when min(e) is in [108, 170], max(e) < 255 and max(e) - min(e) < 15
//   (pack_weights.py:26), otherwise it stays raw (256 bytes);
// - a packed block holds 128 sign|mantissa bytes (v & 127) | ((v >> 8) & 128), then 64 bytes of
//   4-bit exponent codes e - min (15 for a signed zero), low nibble first (192 bytes);
// - the u32 block table holds each block's byte offset in the data region (64-aligned, since
//   both block sizes are) with min - 107 in the low six bits (0 = raw).
// Every packed block is decoded again and compared with its source (pack_weights.py:47-49).
//
// Archive: a 65536-byte header (u64 65528, the compact JSON manifest, spaces), then every region
// 64-byte aligned in safetensors-header order: 1-D tensors raw, 2-D tensors block table then
// data, the input embedding skipped. The manifest keys and their order follow the reference's
// json.dumps output, so the archive is byte-identical to the reference packer's.
#include "../../include/plamo.h"
#include "loader.h"

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace plamo {
extern thread_local std::string g_error;
}

namespace {

constexpr int BLOCK = 128;
constexpr int MINIMUM_BASE = 107;
constexpr size_t HEADER = 65536;

// Packs one block; returns its bytes (192 packed, 256 raw) and sets *minimum (0 = raw).
size_t pack_block(const uint16_t* v, uint8_t* out, int* minimum) {
    int low = 255, high = 0;
    for (int i = 0; i < BLOCK; i++) {
        if ((v[i] & 0x7FFF) == 0) continue;
        const int e = (v[i] >> 7) & 255;
        low = e < low ? e : low;
        high = e > high ? e : high;
    }
    if (!(low >= 108 && low <= 170 && high < 255 && high - low < 15)) {
        std::memcpy(out, v, 256);  // little-endian bf16, as stored
        *minimum = 0;
        return 256;
    }
    for (int i = 0; i < BLOCK; i++) out[i] = uint8_t((v[i] & 127) | ((v[i] >> 8) & 128));
    for (int i = 0; i < BLOCK; i += 2) {
        const int c0 = (v[i] & 0x7FFF) == 0 ? 15 : ((v[i] >> 7) & 255) - low;
        const int c1 = (v[i + 1] & 0x7FFF) == 0 ? 15 : ((v[i + 1] >> 7) & 255) - low;
        out[BLOCK + i / 2] = uint8_t(c0 | (c1 << 4));
    }
    *minimum = low;
    return 192;
}

bool round_trips(const uint16_t* v, const uint8_t* packed, int minimum) {
    for (int i = 0; i < BLOCK; i++) {
        const int code = (packed[BLOCK + i / 2] >> ((i & 1) * 4)) & 15;
        const uint16_t sm = packed[i];
        const uint16_t e = code == 15 ? 0 : uint16_t(minimum + code);
        if (uint16_t((sm & 127) | ((sm & 128) << 8) | (e << 7)) != v[i]) return false;
    }
    return true;
}

// Packs `blocks` blocks into data (grown as needed) and entries; false if a round trip fails.
bool pack_tensor(const uint16_t* v, size_t blocks, std::vector<uint8_t>& data, std::vector<uint32_t>& entries,
                 size_t* packed_blocks) {
    data.resize(blocks * 256);
    entries.resize(blocks);
    size_t at = 0, np = 0;
    for (size_t b = 0; b < blocks; b++) {
        int minimum = 0;
        const size_t n = pack_block(v + b * BLOCK, data.data() + at, &minimum);
        if (minimum) {
            if (!round_trips(v + b * BLOCK, data.data() + at, minimum)) return false;
            np++;
        }
        entries[b] = uint32_t(at) | uint32_t(minimum ? minimum - MINIMUM_BASE : 0);
        at += n;
    }
    data.resize(at);
    *packed_blocks = np;
    return true;
}

struct Writer {
    FILE* f = nullptr;
    size_t pos = 0;
    bool ok = true;
    void put(const void* p, size_t n) {
        if (ok && n && std::fwrite(p, 1, n, f) != n) ok = false;
        pos += n;
    }
    // pads to 64 bytes, writes, returns [begin, end) relative to the payload
    std::pair<size_t, size_t> append(const void* p, size_t n) {
        static const uint8_t zeros[64] = {0};
        put(zeros, (64 - pos % 64) % 64);
        const size_t begin = pos - HEADER;
        put(p, n);
        return {begin, pos - HEADER};
    }
};

// Tensor names go into the manifest verbatim: printable ASCII without quotes or backslashes, the
// characters json.dumps would not escape.
bool plain_name(const std::string& s) {
    for (unsigned char c : s)
        if (c < 0x20 || c >= 0x7F || c == '"' || c == '\\') return false;
    return true;
}

std::string span_json(std::pair<size_t, size_t> s) {
    return "[" + std::to_string(s.first) + "," + std::to_string(s.second) + "]";
}

}  // namespace

extern "C" {

int plamo_p12_chain_valid(const uint32_t* entries, size_t count, size_t data_bytes) {
    return (entries || count == 0) && plamo::validate_chain(entries, count, data_bytes) ? 1 : 0;
}

int plamo_pack_blocks(const uint16_t* values, size_t count, uint8_t* data, size_t data_cap, uint32_t* entries,
                      size_t* data_bytes) {
    if (!values || !data || !entries || !data_bytes || count % BLOCK) {
        plamo::g_error = "Invalid pack arguments";
        return 1;
    }
    std::vector<uint8_t> d;
    std::vector<uint32_t> e;
    size_t np = 0;
    if (!pack_tensor(values, count / BLOCK, d, e, &np)) {
        plamo::g_error = "Packing changed BF16 bits";
        return 1;
    }
    if (d.size() > data_cap) {
        plamo::g_error = "Pack output buffer too small";
        return 1;
    }
    std::memcpy(data, d.data(), d.size());
    std::memcpy(entries, e.data(), e.size() * sizeof(uint32_t));
    *data_bytes = d.size();
    return 0;
}

int plamo_pack_p12(const char* model_dir, const char* source_sha256, uint64_t* stats) {
    using namespace plamo;
    if (!model_dir) {
        g_error = "Invalid pack arguments";
        return 1;
    }
    const std::string dir(model_dir);
    MappedFile st;
    std::string err;
    if (!st.open(dir + "/model.safetensors", err)) {
        g_error = err;
        return 1;
    }
    uint64_t hlen = 0;
    if (st.size < 8) {
        g_error = "Invalid safetensors header";
        return 1;
    }
    std::memcpy(&hlen, st.data, 8);
    Json header;
    if (hlen > st.size - 8 || !parse_json(reinterpret_cast<const char*>(st.data) + 8, size_t(hlen), header, err) ||
        header.type != Json::OBJ) {
        g_error = "Invalid safetensors header";
        return 1;
    }
    const uint8_t* payload = st.data + 8 + hlen;
    const size_t payload_size = st.size - 8 - size_t(hlen);
    const std::string sha = source_sha256 ? std::string(source_sha256) : sha256_hex(st.data, st.size);

    const std::string out_path = dir + "/model.p12", part_path = out_path + ".part";
    Writer w;
    w.f = std::fopen(part_path.c_str(), "wb");
    if (!w.f) {
        g_error = "Cannot write " + part_path;
        return 1;
    }
    std::vector<uint8_t> zeros(HEADER, 0);
    w.put(zeros.data(), HEADER);
    std::string tensors;
    uint64_t total_raw = 0, total_packed = 0, compressed = 0, blocks = 0;
    bool failed = false;
    for (const auto& kv : header.obj) {
        const std::string& name = kv.first;
        if (name == "__metadata__" || name == "model.embed_tokens.weight") continue;
        if (!plain_name(name)) {
            g_error = "Unsupported tensor name in the safetensors header";
            failed = true;
            break;
        }
        const Json& info = kv.second;
        const Json* dt = info.get("dtype");
        const Json* shape = info.get("shape");
        const Json* offs = info.get("data_offsets");
        if (!dt || dt->type != Json::STR || dt->str != "BF16") {
            g_error = name + ": only BF16 tensors can be packed";
            failed = true;
            break;
        }
        long long b0 = 0, b1 = 0;
        if (!shape || shape->type != Json::ARR || !offs || offs->type != Json::ARR || offs->arr.size() != 2 ||
            !offs->arr[0].int_value(b0) || !offs->arr[1].int_value(b1) || b0 < 0 || b1 < b0 ||
            size_t(b1) > payload_size) {
            g_error = name + ": invalid tensor entry";
            failed = true;
            break;
        }
        std::string shape_json = "[";
        long long numel = 1;
        for (size_t i = 0; i < shape->arr.size(); i++) {
            long long dim = 0;
            if (!shape->arr[i].int_value(dim) || dim < 0) {
                failed = true;
                break;
            }
            numel *= dim;
            shape_json += (i ? "," : "") + std::to_string(dim);
        }
        shape_json += "]";
        if (failed || size_t(b1 - b0) != size_t(numel) * 2) {
            g_error = name + ": invalid tensor entry";
            failed = true;
            break;
        }
        const uint16_t* values = reinterpret_cast<const uint16_t*>(payload + b0);
        std::string record = "\"" + name + "\":{\"shape\":" + shape_json;
        if (shape->arr.size() == 1) {
            record += ",\"raw\":" + span_json(w.append(values, size_t(b1 - b0)));
        } else {
            if (numel % BLOCK) {
                g_error = name + ": pack expects whole 128-element blocks";
                failed = true;
                break;
            }
            std::vector<uint8_t> data;
            std::vector<uint32_t> entries;
            size_t np = 0;
            if (!pack_tensor(values, size_t(numel) / BLOCK, data, entries, &np)) {
                g_error = "Packing changed BF16 bits";
                failed = true;
                break;
            }
            record += ",\"offsets\":" + span_json(w.append(entries.data(), entries.size() * 4));
            record += ",\"data\":" + span_json(w.append(data.data(), data.size()));
            compressed += np;
            blocks += entries.size();
            total_packed += data.size() + entries.size() * 4;
            total_raw += uint64_t(b1 - b0);
        }
        record += "}";
        tensors += (tensors.empty() ? "" : ",") + record;
    }
    const size_t payload_bytes = w.pos - HEADER;
    const std::string manifest = "{\"format\":\"plamo-bf16-pack-v2\",\"block\":128,\"minimum_base\":107,\"source_sha256\":\"" +
                                 sha + "\",\"tensors\":{" + tensors + "},\"payload_bytes\":" + std::to_string(payload_bytes) +
                                 "}";
    if (!failed && manifest.size() > HEADER - 8) {
        g_error = "Packed header overflow";
        failed = true;
    }
    if (!failed) {
        std::vector<uint8_t> head(HEADER, ' ');
        const uint64_t count = HEADER - 8;
        std::memcpy(head.data(), &count, 8);
        std::memcpy(head.data() + 8, manifest.data(), manifest.size());
        if (std::fseek(w.f, 0, SEEK_SET) != 0 || std::fwrite(head.data(), 1, HEADER, w.f) != HEADER) w.ok = false;
    }
    const bool closed = std::fclose(w.f) == 0;
    if (failed || !w.ok || !closed || std::rename(part_path.c_str(), out_path.c_str()) != 0) {
        if (!failed) g_error = "Cannot write " + out_path;
        std::remove(part_path.c_str());
        return 1;
    }
    if (stats) {
        stats[0] = total_raw;
        stats[1] = total_packed;
        stats[2] = HEADER + payload_bytes;
        stats[3] = compressed;
        stats[4] = blocks;
    }
    return 0;
}

}  // extern "C"
