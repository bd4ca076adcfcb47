// model_format.cpp — canonical tensor table, safetensors header parsing and the
// synthetic checkpoint writer.  Host code only.
#include "model_format.h"
#include "../host/config.h"
#include "../../include/qwen_b200.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <map>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace qb {

namespace {

std::vector<TensorSpec> build_table() {
    std::vector<TensorSpec> t;
    auto add = [&](const std::string& n, std::vector<int64_t> s) {
        TensorSpec x; x.name = n; x.shape = s;
        size_t e = 1; for (auto d : s) e *= (size_t)d;
        x.bytes = e * 2; t.push_back(x);
    };
    add("lm_head.weight", {VOCAB_SIZE, DIM});
    add("model.embed_tokens.weight", {VOCAB_SIZE, DIM});
    add("model.norm.weight", {DIM});
    for (int l = 0; l < N_LAYERS; l++) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        add(p + "input_layernorm.weight", {DIM});
        add(p + "mlp.down_proj.weight", {DIM, HIDDEN_DIM});
        add(p + "mlp.gate_proj.weight", {HIDDEN_DIM, DIM});
        add(p + "mlp.up_proj.weight", {HIDDEN_DIM, DIM});
        add(p + "post_attention_layernorm.weight", {DIM});
        add(p + "self_attn.k_norm.weight", {HEAD_DIM});
        add(p + "self_attn.k_proj.weight", {KV_DIM, DIM});
        add(p + "self_attn.o_proj.weight", {DIM, Q_DIM});
        add(p + "self_attn.q_norm.weight", {HEAD_DIM});
        add(p + "self_attn.q_proj.weight", {Q_DIM, DIM});
        add(p + "self_attn.v_proj.weight", {KV_DIM, DIM});
    }
    // safetensors writers store tensors sorted by name (byte-wise); the data
    // section is then packed in that order.
    std::sort(t.begin(), t.end(), [](const TensorSpec& a, const TensorSpec& b) { return a.name < b.name; });
    size_t off = 0;
    for (auto& x : t) { x.offset = off; off += x.bytes; }
    return t;
}

struct Json {   // just enough JSON for a safetensors header
    const char* s; size_t n, i = 0;
    void ws() { while (i < n && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) i++; }
    bool ch(char c) { ws(); if (i < n && s[i] == c) { i++; return true; } return false; }
    bool peek(char c) { ws(); return i < n && s[i] == c; }
    bool str(std::string& o) {
        ws(); if (i >= n || s[i] != '"') return false; i++; o.clear();
        while (i < n && s[i] != '"') { if (s[i] == '\\') { if (++i >= n) return false; } o.push_back(s[i++]); }
        if (i >= n) return false; i++; return true;
    }
    bool num(int64_t& v) {
        ws(); size_t j = i; bool neg = false; if (j < n && s[j] == '-') { neg = true; j++; }
        if (j >= n || s[j] < '0' || s[j] > '9') return false;
        int64_t x = 0; while (j < n && s[j] >= '0' && s[j] <= '9') { x = x * 10 + (s[j] - '0'); j++; }
        i = j; v = neg ? -x : x; return true;
    }
    bool skip() {
        ws(); if (i >= n) return false;
        if (s[i] == '"') { std::string t; return str(t); }
        if (s[i] == '{' || s[i] == '[') {
            const char close = s[i] == '{' ? '}' : ']'; i++;
            if (ch(close)) return true;
            for (;;) {
                if (close == '}') { std::string k; if (!str(k) || !ch(':')) return false; }
                if (!skip()) return false;
                if (ch(',')) continue;
                return ch(close);
            }
        }
        while (i < n && s[i] != ',' && s[i] != '}' && s[i] != ']') i++;
        return true;
    }
};

uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

inline uint16_t f2bf(float f) {
    uint32_t u; memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

}  // namespace

const std::vector<TensorSpec>& canonical_table() {
    static const std::vector<TensorSpec> t = build_table();
    return t;
}

size_t canonical_total_bytes() {
    const auto& t = canonical_table();
    return t.back().offset + t.back().bytes;
}

int canonical_index(const std::string& name) {
    static const std::map<std::string, int> m = [] {
        std::map<std::string, int> r; const auto& t = canonical_table();
        for (size_t i = 0; i < t.size(); i++) r[t[i].name] = (int)i;
        return r;
    }();
    auto it = m.find(name);
    return it == m.end() ? -1 : it->second;
}

LayerIndex layer_index(int l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    LayerIndex x;
    x.in_ln = canonical_index(p + "input_layernorm.weight");
    x.down = canonical_index(p + "mlp.down_proj.weight");
    x.gate = canonical_index(p + "mlp.gate_proj.weight");
    x.up = canonical_index(p + "mlp.up_proj.weight");
    x.post_ln = canonical_index(p + "post_attention_layernorm.weight");
    x.k_norm = canonical_index(p + "self_attn.k_norm.weight");
    x.k_proj = canonical_index(p + "self_attn.k_proj.weight");
    x.o_proj = canonical_index(p + "self_attn.o_proj.weight");
    x.q_norm = canonical_index(p + "self_attn.q_norm.weight");
    x.q_proj = canonical_index(p + "self_attn.q_proj.weight");
    x.v_proj = canonical_index(p + "self_attn.v_proj.weight");
    return x;
}
int embed_index() { return canonical_index("model.embed_tokens.weight"); }
int lm_head_index() { return canonical_index("lm_head.weight"); }
int final_norm_index() { return canonical_index("model.norm.weight"); }

const std::vector<int>& blob_order() {
    static const std::vector<int> o = [] {
        std::vector<int> v = {embed_index(), lm_head_index(), final_norm_index()};
        for (int l = 0; l < N_LAYERS; l++) {
            const LayerIndex x = layer_index(l);
            for (int i : {x.q_proj, x.k_proj, x.v_proj, x.o_proj, x.q_norm, x.k_norm, x.gate, x.up, x.down, x.in_ln, x.post_ln}) v.push_back(i);
        }
        return v;
    }();
    return o;
}

namespace {

// A blob has no header: its size is exactly the sum of the tensors, and its
// first 8 bytes do not announce a safetensors JSON header that fits the file.
bool looks_like_blob(int fd, size_t bytes) {
    if (bytes != canonical_total_bytes()) return false;
    uint64_t hl = 0;
    char c = 0;
    if (pread(fd, &hl, 8, 0) != 8) return false;
    if (hl == 0 || hl > (100u << 20) || 8 + hl > bytes) return true;
    if (pread(fd, &c, 1, 8) != 1) return false;
    return c != '{';
}

void map_blob(const std::string& path, size_t bytes, CheckpointMap& out) {
    const auto& table = canonical_table();
    out.file_offset.assign(table.size(), 0);
    size_t off = 0;
    for (int i : blob_order()) { out.file_offset[i] = off; off += table[i].bytes; }
    out.file_bytes = bytes;
    out.data_start = 0;
    out.blob = true;
    out.source = path;
    out.canonical_order = false;
}

std::string sibling_blob(const std::string& path) {
    const size_t p = path.find_last_of('/');
    return (p == std::string::npos ? std::string(".") : path.substr(0, p)) + "/weights_qwen600.bin";
}

}  // namespace

int parse_checkpoint(const std::string& path, CheckpointMap& out, std::string& err) {
    const auto& table = canonical_table();
    out = CheckpointMap{};
    out.source = path;
    int fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) { err = "cannot open checkpoint: " + path; return QWEN_E_IO; }
    struct stat st;
    if (fstat(fd, &st) != 0) { close(fd); err = "cannot stat checkpoint: " + path; return QWEN_E_IO; }
    out.file_bytes = (size_t)st.st_size;
    if (looks_like_blob(fd, out.file_bytes)) {
        close(fd);
        map_blob(path, out.file_bytes, out);
        return QWEN_OK;
    }
    uint64_t hl = 0;
    if (out.file_bytes < 8 || pread(fd, &hl, 8, 0) != 8) { close(fd); err = "checkpoint shorter than its 8-byte header length"; return QWEN_E_FORMAT; }
    if (hl == 0 || hl > (100u << 20) || 8 + hl > out.file_bytes) {
        close(fd); err = "safetensors header length " + std::to_string(hl) + " does not fit the file"; return QWEN_E_FORMAT;
    }
    std::string js(hl, '\0');
    if (pread(fd, &js[0], hl, 8) != (ssize_t)hl) { close(fd); err = "short read of safetensors header"; return QWEN_E_IO; }
    close(fd);
    out.data_start = 8 + hl;
    const size_t data_bytes = out.file_bytes - out.data_start;

    out.file_offset.assign(table.size(), (size_t)-1);
    std::vector<std::pair<size_t, size_t>> ranges;
    Json J{js.data(), js.size()};
    if (!J.ch('{')) { err = "safetensors header is not a JSON object"; return QWEN_E_FORMAT; }
    if (!J.ch('}')) {
        for (;;) {
            std::string name;
            if (!J.str(name) || !J.ch(':')) { err = "malformed safetensors header"; return QWEN_E_FORMAT; }
            if (name == "__metadata__") { if (!J.skip()) { err = "malformed __metadata__"; return QWEN_E_FORMAT; } }
            else {
                if (!J.ch('{')) { err = "malformed entry for " + name; return QWEN_E_FORMAT; }
                std::string dtype; std::vector<int64_t> shape, offs;
                if (!J.ch('}')) {
                    for (;;) {
                        std::string key;
                        if (!J.str(key) || !J.ch(':')) { err = "malformed entry for " + name; return QWEN_E_FORMAT; }
                        if (key == "dtype") { if (!J.str(dtype)) { err = "bad dtype for " + name; return QWEN_E_FORMAT; } }
                        else if (key == "shape" || key == "data_offsets") {
                            std::vector<int64_t>& v = key == "shape" ? shape : offs;
                            if (!J.ch('[')) { err = "bad " + key + " for " + name; return QWEN_E_FORMAT; }
                            if (!J.ch(']')) for (;;) {
                                int64_t x; if (!J.num(x)) { err = "bad " + key + " for " + name; return QWEN_E_FORMAT; }
                                v.push_back(x);
                                if (J.ch(',')) continue;
                                if (J.ch(']')) break;
                                err = "bad " + key + " for " + name; return QWEN_E_FORMAT;
                            }
                        } else if (!J.skip()) { err = "malformed entry for " + name; return QWEN_E_FORMAT; }
                        if (J.ch(',')) continue;
                        if (J.ch('}')) break;
                        err = "malformed entry for " + name; return QWEN_E_FORMAT;
                    }
                }
                const int idx = canonical_index(name);
                if (idx < 0) { err = "unexpected tensor in checkpoint: " + name; return QWEN_E_FORMAT; }
                const TensorSpec& ts = table[idx];
                if (dtype != "BF16") { err = name + ": dtype " + dtype + ", expected BF16"; return QWEN_E_FORMAT; }
                if (shape != ts.shape) { err = name + ": shape does not match the model"; return QWEN_E_FORMAT; }
                if (offs.size() != 2 || offs[0] < 0 || offs[1] < offs[0] || (size_t)(offs[1] - offs[0]) != ts.bytes) {
                    err = name + ": data_offsets do not match its size"; return QWEN_E_FORMAT;
                }
                if ((size_t)offs[1] > data_bytes) { err = name + ": data runs past the end of the file (truncated checkpoint?)"; return QWEN_E_FORMAT; }
                if (out.file_offset[idx] != (size_t)-1) { err = "duplicate tensor " + name; return QWEN_E_FORMAT; }
                out.file_offset[idx] = out.data_start + (size_t)offs[0];
                ranges.push_back({(size_t)offs[0], (size_t)offs[1]});
            }
            if (J.ch(',')) continue;
            if (J.ch('}')) break;
            err = "malformed safetensors header"; return QWEN_E_FORMAT;
        }
    }
    for (size_t i = 0; i < table.size(); i++)
        if (out.file_offset[i] == (size_t)-1) { err = "missing tensor " + table[i].name; return QWEN_E_FORMAT; }
    std::sort(ranges.begin(), ranges.end());
    for (size_t i = 1; i < ranges.size(); i++)
        if (ranges[i].first < ranges[i - 1].second) { err = "overlapping tensors in checkpoint"; return QWEN_E_FORMAT; }
    out.canonical_order = true;
    for (size_t i = 0; i < table.size(); i++)
        if (out.file_offset[i] != out.data_start + table[i].offset) { out.canonical_order = false; break; }
    // the reference's preference for an ordered blob beside the checkpoint
    const std::string sib = sibling_blob(path);
    struct stat sb;
    if (stat(sib.c_str(), &sb) == 0 && S_ISREG(sb.st_mode) && (size_t)sb.st_size == canonical_total_bytes()) {
        const int bfd = open(sib.c_str(), O_RDONLY);
        if (bfd >= 0) {
            const bool ok = looks_like_blob(bfd, (size_t)sb.st_size);
            close(bfd);
            if (ok) map_blob(sib, (size_t)sb.st_size, out);
        }
    }
    return QWEN_OK;
}

int write_blob(const std::string& safetensors_path, const std::string& out_path, std::string& err) {
    CheckpointMap m;
    int rc = parse_checkpoint(safetensors_path, m, err);
    if (rc != QWEN_OK) return rc;
    const auto& table = canonical_table();
    const int in = open(m.source.c_str(), O_RDONLY);
    if (in < 0) { err = "cannot open " + m.source; return QWEN_E_IO; }
    const std::string tmp = out_path + ".partial";
    const int out = open(tmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC, 0644);
    if (out < 0) { close(in); err = "cannot create " + tmp; return QWEN_E_IO; }
    std::vector<char> buf((size_t)16 << 20);
    rc = QWEN_OK;
    for (int i : blob_order()) {
        size_t done = 0;
        while (done < table[i].bytes && rc == QWEN_OK) {
            const size_t n = std::min(buf.size(), table[i].bytes - done);
            if (pread(in, buf.data(), n, (off_t)(m.file_offset[i] + done)) != (ssize_t)n) { err = "short read of " + table[i].name; rc = QWEN_E_IO; break; }
            if (write(out, buf.data(), n) != (ssize_t)n) { err = "short write to " + tmp; rc = QWEN_E_IO; break; }
            done += n;
        }
        if (rc != QWEN_OK) break;
    }
    close(in);
    if (close(out) != 0 && rc == QWEN_OK) { err = "cannot close " + tmp; rc = QWEN_E_IO; }
    if (rc == QWEN_OK && rename(tmp.c_str(), out_path.c_str()) != 0) { err = "cannot rename " + tmp; rc = QWEN_E_IO; }
    if (rc != QWEN_OK) unlink(tmp.c_str());
    return rc;
}

int write_synthetic(const std::string& path, uint64_t seed, std::string& err) {
    const auto& table = canonical_table();
    std::string js = "{\"__metadata__\":{\"format\":\"pt\",\"generator\":\"qwen_b200 synthetic N(0,0.02) seed " +
                     std::to_string(seed) + "\"}";
    for (const auto& t : table) {
        js += ",\"" + t.name + "\":{\"dtype\":\"BF16\",\"shape\":[";
        for (size_t k = 0; k < t.shape.size(); k++) js += (k ? "," : "") + std::to_string(t.shape[k]);
        js += "],\"data_offsets\":[" + std::to_string(t.offset) + "," + std::to_string(t.offset + t.bytes) + "]}";
    }
    js += "}";
    while ((8 + js.size()) % 256) js.push_back(' ');   // keep the data section 256-byte aligned
    const uint64_t hl = js.size();
    const size_t total = 8 + hl + canonical_total_bytes();

    const std::string tmp = path + ".partial";
    int fd = open(tmp.c_str(), O_RDWR | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) { err = "cannot create " + tmp; return QWEN_E_IO; }
    if (ftruncate(fd, (off_t)total) != 0) { close(fd); err = "cannot size " + tmp; return QWEN_E_IO; }
    char* m = (char*)mmap(nullptr, total, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    close(fd);
    if (m == MAP_FAILED) { err = "cannot map " + tmp; return QWEN_E_IO; }
    memcpy(m, &hl, 8);
    memcpy(m + 8, js.data(), hl);
    char* data = m + 8 + hl;

    const int emb = embed_index(), lm = lm_head_index();
    for (size_t ti = 0; ti < table.size(); ti++) {
        const TensorSpec& t = table[ti];
        if ((int)ti == lm) continue;   // written as a copy of the embedding below
        uint16_t* dst = (uint16_t*)(data + t.offset);
        const int64_t n = (int64_t)(t.bytes / 2);
        if (t.shape.size() == 1) {     // every 1-D tensor is an RMSNorm / QK-norm gain
            for (int64_t i = 0; i < n; i++) dst[i] = 0x3F80;   // 1.0
            continue;
        }
        // Tensor key: the seed mixed with the tensor's name hash (FNV-1a), so a
        // tensor's values do not depend on its position in the table.
        uint64_t h = 1469598103934665603ull;
        for (char c : t.name) { h ^= (uint8_t)c; h *= 1099511628211ull; }
        const uint64_t key = splitmix64(seed ^ splitmix64(h));
        // Element pair (2i, 2i+1) <- Box-Muller on two 53-bit uniforms drawn from
        // splitmix64(key + 2i) and splitmix64(key + 2i + 1).
        #pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < n / 2; i++) {
            const uint64_t a = splitmix64(key + 2 * (uint64_t)i), b = splitmix64(key + 2 * (uint64_t)i + 1);
            const double u1 = ((double)(a >> 11) + 0.5) * (1.0 / 9007199254740992.0);
            const double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
            const double r = sqrt(-2.0 * log(u1)), th = 6.283185307179586 * u2;
            dst[2 * i] = f2bf((float)(0.02 * r * cos(th)));
            dst[2 * i + 1] = f2bf((float)(0.02 * r * sin(th)));
        }
    }
    memcpy(data + table[lm].offset, data + table[emb].offset, table[emb].bytes);
    if (msync(m, total, MS_SYNC) != 0) { munmap(m, total); err = "msync failed for " + tmp; return QWEN_E_IO; }
    munmap(m, total);
    if (rename(tmp.c_str(), path.c_str()) != 0) { err = "cannot rename " + tmp + " to " + path; return QWEN_E_IO; }
    return QWEN_OK;
}

}  // namespace qb
