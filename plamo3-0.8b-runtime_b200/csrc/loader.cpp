// Model directory loading and validation.
//   config.json checks        Runtime.swift:180-190 (dims are parameters here, structure is checked)
//   RoPE frequencies          Runtime.swift:268-274 (config-mlx.json plamo_rope_inv_freq)
//   safetensors checks        Runtime.swift:33-101
//   .p12 manifest and chain   Packed.swift:12-91 (format from scripts/pack_weights.py)
#include "loader.h"

#include <cstdlib>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>

namespace plamo {

const char* const kReferenceSourceSha = "7c9f0066d166c075bdbe83ada3d444e08bd7a6ee3f345f47a1f3c442aa6898c5";

// ------------------------------------------------------------------------------------------------
// JSON (RFC 8259 subset sufficient for model headers: no surrogate-pair decoding beyond \uXXXX BMP)

const Json* Json::get(const std::string& k) const {
    if (type != OBJ) return nullptr;
    for (const auto& kv : obj)
        if (kv.first == k) return &kv.second;
    return nullptr;
}

bool Json::int_value(long long& out) const {
    if (type != NUM || !is_int) return false;
    out = inum;
    return true;
}

namespace {
struct Parser {
    const char* p;
    const char* e;
    std::string err;
    int depth = 0;
    void ws() { while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++; }
    bool fail(const char* m) { if (err.empty()) err = m; return false; }
    bool str(std::string& out) {
        if (p >= e || *p != '"') return fail("expected string");
        p++;
        while (p < e && *p != '"') {
            if (*p == '\\') {
                if (++p >= e) return fail("bad escape");
                switch (*p) {
                    case '"': out += '"'; break;
                    case '\\': out += '\\'; break;
                    case '/': out += '/'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'n': out += '\n'; break;
                    case 'r': out += '\r'; break;
                    case 't': out += '\t'; break;
                    case 'u': {
                        if (e - p < 5) return fail("bad unicode escape");
                        unsigned v = 0;
                        for (int i = 1; i <= 4; i++) {
                            char c = p[i];
                            v <<= 4;
                            if (c >= '0' && c <= '9') v |= c - '0';
                            else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
                            else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
                            else return fail("bad unicode escape");
                        }
                        p += 4;
                        if (v < 0x80) out += char(v);
                        else if (v < 0x800) { out += char(0xC0 | (v >> 6)); out += char(0x80 | (v & 63)); }
                        else { out += char(0xE0 | (v >> 12)); out += char(0x80 | ((v >> 6) & 63)); out += char(0x80 | (v & 63)); }
                        break;
                    }
                    default: return fail("bad escape");
                }
                p++;
            } else {
                out += *p++;
            }
        }
        if (p >= e) return fail("unterminated string");
        p++;
        return true;
    }
    bool value(Json& v) {
        if (++depth > 64) return fail("json too deep");
        ws();
        if (p >= e) return fail("unexpected end");
        bool ok = true;
        if (*p == '{') {
            v.type = Json::OBJ; p++; ws();
            if (p < e && *p == '}') { p++; }
            else for (;;) {
                ws(); std::string k;
                if (!str(k)) return false;
                ws(); if (p >= e || *p != ':') return fail("expected ':'");
                p++;
                Json child;
                if (!value(child)) return false;
                v.obj.emplace_back(std::move(k), std::move(child));
                ws();
                if (p < e && *p == ',') { p++; continue; }
                if (p < e && *p == '}') { p++; break; }
                return fail("expected ',' or '}'");
            }
        } else if (*p == '[') {
            v.type = Json::ARR; p++; ws();
            if (p < e && *p == ']') { p++; }
            else for (;;) {
                Json child;
                if (!value(child)) return false;
                v.arr.push_back(std::move(child));
                ws();
                if (p < e && *p == ',') { p++; continue; }
                if (p < e && *p == ']') { p++; break; }
                return fail("expected ',' or ']'");
            }
        } else if (*p == '"') {
            v.type = Json::STR; ok = str(v.str);
        } else if (e - p >= 4 && !strncmp(p, "true", 4)) { v.type = Json::BOOL; v.b = true; p += 4; }
        else if (e - p >= 5 && !strncmp(p, "false", 5)) { v.type = Json::BOOL; v.b = false; p += 5; }
        else if (e - p >= 4 && !strncmp(p, "null", 4)) { v.type = Json::NUL; p += 4; }
        else {
            const char* s = p;
            if (p < e && (*p == '-' || *p == '+')) p++;
            bool frac = false;
            while (p < e && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' || *p == '-' || *p == '+')) {
                if (*p == '.' || *p == 'e' || *p == 'E') frac = true;
                p++;
            }
            if (p == s) return fail("unexpected character");
            std::string tok(s, p);
            v.type = Json::NUM;
            char* end = nullptr;
            v.num = strtod(tok.c_str(), &end);
            if (!end || *end) return fail("bad number");
            if (!frac) {
                v.is_int = true;
                v.inum = strtoll(tok.c_str(), &end, 10);
            }
        }
        depth--;
        return ok;
    }
};
}  // namespace

bool parse_json(const char* data, size_t len, Json& out, std::string& err) {
    Parser ps{data, data + len, {}};
    if (!ps.value(out)) { err = ps.err; return false; }
    ps.ws();
    if (ps.p != ps.e) { err = "trailing data after JSON"; return false; }
    return true;
}

// ------------------------------------------------------------------------------------------------
// SHA-256 (FIPS 180-4)

namespace {
const uint32_t kSha[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};
inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
void sha_block(uint32_t h[8], const uint8_t* b) {
    uint32_t w[64];
    for (int i = 0; i < 16; i++) w[i] = uint32_t(b[4 * i]) << 24 | uint32_t(b[4 * i + 1]) << 16 | uint32_t(b[4 * i + 2]) << 8 | b[4 * i + 3];
    for (int i = 16; i < 64; i++) {
        uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
        uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
        w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], bb = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; i++) {
        uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
        uint32_t ch = (e & f) ^ (~e & g);
        uint32_t t1 = hh + S1 + ch + kSha[i] + w[i];
        uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
        uint32_t mj = (a & bb) ^ (a & c) ^ (bb & c);
        uint32_t t2 = S0 + mj;
        hh = g; g = f; f = e; e = d + t1; d = c; c = bb; bb = a; a = t1 + t2;
    }
    h[0] += a; h[1] += bb; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}
}  // namespace

std::string sha256_hex(const uint8_t* data, size_t len) {
    uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    size_t i = 0;
    for (; i + 64 <= len; i += 64) sha_block(h, data + i);
    uint8_t tail[128] = {0};
    size_t rem = len - i;
    memcpy(tail, data + i, rem);
    tail[rem] = 0x80;
    size_t tl = rem + 1 + 8 <= 64 ? 64 : 128;
    uint64_t bits = uint64_t(len) * 8;
    for (int k = 0; k < 8; k++) tail[tl - 1 - k] = uint8_t(bits >> (8 * k));
    sha_block(h, tail);
    if (tl == 128) sha_block(h, tail + 64);
    char out[65];
    for (int k = 0; k < 8; k++) snprintf(out + 8 * k, 9, "%08x", h[k]);
    return std::string(out, 64);
}

// ------------------------------------------------------------------------------------------------

MappedFile::~MappedFile() {
    if (data) munmap(const_cast<uint8_t*>(data), size);
}

bool MappedFile::open(const std::string& path, std::string& err) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) { err = "Cannot open " + path; return false; }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 8) { ::close(fd); err = "Invalid file size: " + path; return false; }
    void* p = mmap(nullptr, size_t(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (p == MAP_FAILED) { err = "Cannot map " + path; return false; }
    data = static_cast<const uint8_t*>(p);
    size = size_t(st.st_size);
    return true;
}

static bool read_text(const std::string& path, std::string& out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    std::stringstream ss;
    ss << f.rdbuf();
    out = ss.str();
    return true;
}

static bool shape_of(const Json* j, std::vector<long long>& out) {
    if (!j || j->type != Json::ARR) return false;
    out.clear();
    for (const auto& v : j->arr) {
        long long x;
        if (!v.int_value(x) || x < 0) return false;
        out.push_back(x);
    }
    return true;
}

static bool pair_of(const Json* j, long long& a, long long& b) {
    if (!j || j->type != Json::ARR || j->arr.size() != 2) return false;
    return j->arr[0].int_value(a) && j->arr[1].int_value(b);
}

bool validate_chain(const uint32_t* entries, size_t count, size_t data_bytes) {
    size_t end = 0;
    for (size_t i = 0; i < count; i++) {
        const uint32_t entry = entries[i];
        const size_t offset = entry & ~63u;
        const size_t bytes = (entry & 63u) == 0 ? 256 : 192;
        if (offset != end || bytes > data_bytes || offset > data_bytes - bytes) return false;
        end = offset + bytes;
    }
    return end == data_bytes;
}

bool ModelFiles::load(const std::string& dir, bool packed, std::string& err) {
    std::string text;
    if (!read_text(dir + "/config.json", text)) { err = "Cannot read " + dir + "/config.json"; return false; }
    Json c;
    if (!parse_json(text.data(), text.size(), c, err)) { err = "Invalid config.json: " + err; return false; }
    auto geti = [&](const char* k, int& out) {
        long long v; const Json* j = c.get(k);
        if (!j || !j->int_value(v) || v <= 0 || v > (1 << 24)) return false;
        out = int(v); return true;
    };
    auto getd = [&](const char* k, double& out) {
        const Json* j = c.get(k);
        if (!j || j->type != Json::NUM) return false;
        out = j->num; return true;
    };
    auto getb = [&](const char* k, bool want) { const Json* j = c.get(k); return j && j->type == Json::BOOL && j->b == want; };
    auto gets = [&](const char* k, const char* want) { const Json* j = c.get(k); return j && j->type == Json::STR && j->str == want; };
    double rope_theta, rope_local, rope_factor, eps;
    bool ok = geti("hidden_size", cfg.d) && geti("num_hidden_layers", cfg.layers) && geti("num_attention_heads", cfg.heads) &&
              geti("num_key_value_heads", cfg.kv_heads) && geti("head_dim", cfg.head_dim) &&
              geti("intermediate_size", cfg.ffn) && geti("vocab_size", cfg.vocab) && geti("window_size", cfg.window) &&
              geti("sliding_window_pattern", cfg.pattern) && getb("tie_word_embeddings", false) &&
              getb("scale_embedding", false) && gets("model_type", "plamo3") && gets("dtype", "bfloat16") &&
              getd("rope_theta", rope_theta) && getd("rope_local_theta", rope_local) &&
              getd("rope_scaling_factor", rope_factor) && getd("rms_norm_eps", eps) && eps == 1e-6;
    // Structural requirements of these kernels: head_dim 128, 128-multiple projection widths, d <= 4096.
    ok = ok && cfg.head_dim == 128 && cfg.heads % cfg.kv_heads == 0 && cfg.heads <= 32 && cfg.d % 128 == 0 &&
         cfg.ffn % 128 == 0 && cfg.d <= 4096 && cfg.ffn <= 8192 && cfg.q_dim() <= 8192;
    if (!ok) { err = "Only PLaMo 3 bfloat16 configurations with head_dim 128 are supported"; return false; }
    if (!read_text(dir + "/config-mlx.json", text)) { err = "Missing source-exact RoPE frequencies in config-mlx.json"; return false; }
    Json m;
    const Json *fr = nullptr, *lo = nullptr, *fu = nullptr;
    if (parse_json(text.data(), text.size(), m, err)) fr = m.get("plamo_rope_inv_freq");
    if (fr) { lo = fr->get("local"); fu = fr->get("full"); }
    if (!lo || !fu || lo->type != Json::ARR || fu->type != Json::ARR || lo->arr.size() != 64 || fu->arr.size() != 64) {
        err = "Missing source-exact RoPE frequencies in config-mlx.json"; return false;
    }
    for (int i = 0; i < 64; i++) {
        const Json &a = lo->arr[i], &b = fu->arr[i];
        if (a.type != Json::NUM || b.type != Json::NUM || !std::isfinite(a.num) || !std::isfinite(b.num) || a.num <= 0 || b.num <= 0) {
            err = "Missing source-exact RoPE frequencies in config-mlx.json"; return false;
        }
        inv_local[i] = float(a.num); inv_full[i] = float(b.num);
    }
    // model.safetensors (Runtime.swift:33-66)
    if (!st.open(dir + "/model.safetensors", err)) { err = "Cannot open weights: " + dir + "/model.safetensors"; return false; }
    uint64_t hs;
    memcpy(&hs, st.data, 8);
    if (hs > 1048576 || hs >= st.size - 8) { err = "Invalid safetensors header size"; return false; }
    st_data_start = 8 + size_t(hs);
    if (st_data_start % 8) { err = "Unaligned safetensors header"; return false; }
    Json h;
    if (!parse_json(reinterpret_cast<const char*>(st.data + 8), size_t(hs), h, err) || h.type != Json::OBJ) {
        err = "Invalid safetensors header"; return false;
    }
    for (const auto& kv : h.obj) {
        if (kv.first == "__metadata__") continue;
        const Json* dt = kv.second.get("dtype");
        TensorRef t;
        long long b, e;
        if (!dt || dt->type != Json::STR || dt->str != "BF16" || !shape_of(kv.second.get("shape"), t.shape) ||
            !pair_of(kv.second.get("data_offsets"), b, e) || b < 0 || e < b || size_t(e) > st.size - st_data_start) {
            continue;  // validated on use (Runtime.swift:87-94)
        }
        t.data = st.data + st_data_start + b;
        t.bytes = size_t(e - b);
        st_tensors[kv.first] = t;
    }
    {
        auto it = st_tensors.find("model.embed_tokens.weight");
        if (it == st_tensors.end() || it->second.shape != std::vector<long long>{cfg.vocab, cfg.d} ||
            it->second.bytes != size_t(cfg.vocab) * cfg.d * 2 || (it->second.data - st.data - st_data_start) % 2) {
            err = "Invalid input embedding"; return false;
        }
    }
    if (!packed) return true;
    // model.p12 (Packed.swift:12-47)
    if (!p12.open(dir + "/model.p12", err)) { err = "Packed weights missing; run scripts/pack_weights.py first"; return false; }
    uint64_t count;
    memcpy(&count, p12.data, 8);
    if (count > 1048576 || count >= p12.size - 8 || (count + 8) % 64) { err = "Invalid packed header"; return false; }
    p12_data_start = size_t(count) + 8;
    Json ph;
    const char* incompatible = "Incompatible packed archive; run scripts/pack_weights.py to regenerate";
    if (!parse_json(reinterpret_cast<const char*>(p12.data + 8), size_t(count), ph, err) || ph.type != Json::OBJ) {
        err = incompatible; return false;
    }
    long long block, base, payload;
    const Json* fmt = ph.get("format");
    const Json* sha = ph.get("source_sha256");
    const Json* tensors = ph.get("tensors");
    if (!fmt || fmt->type != Json::STR || fmt->str != "plamo-bf16-pack-v2" || !ph.get("block") ||
        !ph.get("block")->int_value(block) || block != 128 || !ph.get("minimum_base") ||
        !ph.get("minimum_base")->int_value(base) || base != 107 || !sha || sha->type != Json::STR ||
        !ph.get("payload_bytes") || !ph.get("payload_bytes")->int_value(payload) ||
        size_t(payload) != p12.size - p12_data_start || !tensors || tensors->type != Json::OBJ) {
        err = incompatible; return false;
    }
    // The reference binds an archive to the original checkpoint's digest (Packed.swift:35) and so
    // does this loader by default. With PLAMO_P12_LOCAL_SOURCE=1 in the environment it also accepts
    // an archive bound to the safetensors file beside it (the seeded synthetic checkpoints of the
    // tests and benchmarks); an archive of another checkpoint is still refused.
    const char* local = getenv("PLAMO_P12_LOCAL_SOURCE");
    const bool local_ok = local && local[0] == '1' && sha->str == sha256_hex(st.data, st.size);
    if (sha->str != kReferenceSourceSha && !local_ok) { err = incompatible; return false; }
    p12_payload = size_t(payload);
    for (const auto& kv : tensors->obj) {
        TensorRef t;
        if (!shape_of(kv.second.get("shape"), t.shape)) continue;
        long long a, b;
        if (t.shape.size() == 1) {
            if (!pair_of(kv.second.get("raw"), a, b)) continue;
            t.raw_off = size_t(a); t.bytes = size_t(b - a);
            if (a < 0 || a % 64 || b < a || size_t(b) > p12_payload) { t.bytes = size_t(-1); }
        } else {
            long long c0, c1;
            if (!pair_of(kv.second.get("offsets"), a, b) || !pair_of(kv.second.get("data"), c0, c1)) continue;
            t.packed = true;
            if (a < 0 || a % 64 || b < a || size_t(b) > p12_payload || c0 < 0 || c0 % 64 || c1 < c0 || size_t(c1) > p12_payload) {
                t.table_bytes = size_t(-1);
            } else {
                t.table_off = size_t(a); t.table_bytes = size_t(b - a);
                t.data_off = size_t(c0); t.data_bytes = size_t(c1 - c0);
            }
        }
        p12_tensors[kv.first] = t;
    }
    return true;
}

bool ModelFiles::tensor(const std::string& name, const std::vector<long long>& shape, bool from_p12, TensorRef& out,
                        std::string& err) const {
    long long numel = 1;
    for (long long s : shape) numel *= s;
    auto it = st_tensors.find(name);
    if (it == st_tensors.end() || it->second.shape != shape || it->second.bytes != size_t(numel) * 2 ||
        (it->second.data - st.data - st_data_start) % 4) {
        err = "Missing or incompatible BF16 tensor: " + name;
        return false;
    }
    if (!from_p12) { out = it->second; return true; }
    auto pt = p12_tensors.find(name);
    if (pt == p12_tensors.end() || pt->second.shape != shape) { err = "Packed tensor shape mismatch: " + name; return false; }
    const TensorRef& t = pt->second;
    if (shape.size() == 1) {
        if (t.bytes != size_t(shape[0]) * 2) {
            err = t.bytes == size_t(-1) ? "Invalid packed region: " + name + ".raw" : "Invalid packed norm";
            return false;
        }
        out = t;
        out.data = p12.data + p12_data_start + t.raw_off;
        return true;
    }
    if (t.table_bytes == size_t(-1)) { err = "Invalid packed region: " + name; return false; }
    if (numel % 128 || t.table_bytes != size_t(numel / 128) * 4) { err = "Invalid packed block table"; return false; }
    const uint32_t* table = reinterpret_cast<const uint32_t*>(p12.data + p12_data_start + t.table_off);
    if (!validate_chain(table, size_t(numel / 128), t.data_bytes)) { err = "Packed block out of range: " + name; return false; }
    out = t;
    out.data = p12.data + p12_data_start;
    return true;
}

}  // namespace plamo
