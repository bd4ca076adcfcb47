// oracle.cpp — CPU restatement of the reference decode math.
//
// TEST INFRASTRUCTURE ONLY.  Nothing in the product (the package's C-ABI
// library, its host headers or its kernels) links, loads or calls this file.
// Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
// arm use it, and only as the checker or as the timed CPU baseline.
//
// What it restates (reference = Ramshankar07/qwen600-ROCm-inference):
//   forward(token, pos)            qwen_model.cuh:772-851
//     embedding row copy           qwen_model.cuh:783-784
//     RMSNorm                      qwen_model.cuh:118-173  (fp32 sum of squares,
//                                  r = rsqrt(ss/DIM + eps), y = (x*r)*w)
//     Q/K/V projections            qwen_model.cuh:796-800  (W row-major [out][in])
//     per-head QK-norm             qwen_model.cuh:195-247
//     NeoX RoPE, pairs (j, j+64)   qwen_model.cuh:316-365
//     attention scores / softmax / weighted V
//                                  qwen_model.cuh:551-614, 384-481
//     O projection + residual      qwen_model.cuh:813      (cuBLAS beta = 1)
//     gate/up + SwiGLU             qwen_model.cuh:823-828, 673-689
//     down projection + residual   qwen_model.cuh:831
//     final norm + LM head         qwen_model.cuh:839-845
//   sample()                       sampler.h:27-175 (xorshift64*, argmax,
//                                  Hoare quickselect, temperature softmax,
//                                  top-p cut, inverse-CDF draw)
//
// Numeric modes:
//   ORACLE_FP32 (0)   every intermediate is an fp32 value (dot products and
//                     sums accumulate in double, then round to float); the only
//                     bf16 rounding is the KV cache, whose storage type in the
//                     reference is bf16 (qwen_model.cuh:44-45).
//   ORACLE_BF16 (1)   rounds to bf16 (round-to-nearest-even) at exactly the
//                     points where the reference CUDA path stores bf16.
//   ORACLE_FP32_KV (2) like mode 0 but the KV cache also holds fp32 (no bf16
//                     rounding anywhere): the pure-fp32 model.
//
// The RoPE angle is computed the way the reference writes it
// (qwen_model.cuh:331-334): freq = 1/powf(theta, 2j/128) and angle = pos*freq,
// both in fp32, then sincosf.
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <cmath>
#include <string>
#include <vector>
#include <map>
#include <algorithm>
#include <functional>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

constexpr int DIM = 1024, HIDDEN = 3072, LAYERS = 28, NH = 16, NKV = 8, HD = 128;
constexpr int QD = NH * HD, KVD = NKV * HD, VOCAB = 151936;
constexpr float THETA = 1000000.0f, EPS = 1e-6f;

inline float bf2f(uint16_t h) { uint32_t u = (uint32_t)h << 16; float f; memcpy(&f, &u, 4); return f; }
inline uint16_t f2bf(float f) {
    uint32_t u; memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // quiet NaN
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
inline float rbf(float f) { return bf2f(f2bf(f)); }

// Minimal safetensors header reader: name -> (byte offset in data section, bytes).
struct TensorLoc { size_t off = 0, bytes = 0; std::string dtype; std::vector<int64_t> shape; };

bool parse_header(const char* js, size_t n, std::map<std::string, TensorLoc>& out) {
    size_t i = 0;
    auto ws = [&]() { while (i < n && (js[i] == ' ' || js[i] == '\n' || js[i] == '\t' || js[i] == '\r')) i++; };
    auto str = [&](std::string& s) -> bool {
        ws(); if (i >= n || js[i] != '"') return false; i++; s.clear();
        while (i < n && js[i] != '"') { if (js[i] == '\\' && i + 1 < n) i++; s.push_back(js[i++]); }
        if (i >= n) return false; i++; return true;
    };
    auto num = [&](int64_t& v) -> bool {
        ws(); char* e = nullptr; v = strtoll(js + i, &e, 10); if (e == js + i) return false; i = e - js; return true;
    };
    std::function<bool()> skip = [&]() -> bool {   // skip any JSON value
        ws(); if (i >= n) return false;
        if (js[i] == '"') { std::string s; return str(s); }
        if (js[i] == '{' || js[i] == '[') {
            char close = js[i] == '{' ? '}' : ']'; i++; ws();
            if (i < n && js[i] == close) { i++; return true; }
            while (true) {
                if (close == '}') { std::string k; if (!str(k)) return false; ws(); if (js[i] != ':') return false; i++; }
                if (!skip()) return false; ws();
                if (js[i] == ',') { i++; continue; }
                if (js[i] == close) { i++; return true; }
                return false;
            }
        }
        while (i < n && js[i] != ',' && js[i] != '}' && js[i] != ']') i++;
        return true;
    };
    ws(); if (i >= n || js[i] != '{') return false; i++;
    while (true) {
        ws(); if (i < n && js[i] == '}') return true;
        std::string name; if (!str(name)) return false; ws(); if (js[i] != ':') return false; i++; ws();
        if (name == "__metadata__") { if (!skip()) return false; }
        else {
            if (js[i] != '{') return false; i++;
            TensorLoc t; int64_t a = -1, b = -1;
            while (true) {
                ws(); if (js[i] == '}') { i++; break; }
                std::string key; if (!str(key)) return false; ws(); if (js[i] != ':') return false; i++; ws();
                if (key == "dtype") { if (!str(t.dtype)) return false; }
                else if (key == "shape" || key == "data_offsets") {
                    if (js[i] != '[') return false; i++;
                    std::vector<int64_t> v;
                    while (true) { ws(); if (js[i] == ']') { i++; break; } int64_t x; if (!num(x)) return false; v.push_back(x); ws(); if (js[i] == ',') i++; }
                    if (key == "shape") t.shape = v; else { if (v.size() != 2) return false; a = v[0]; b = v[1]; }
                } else if (!skip()) return false;
                ws(); if (js[i] == ',') i++;
            }
            if (a < 0 || b < a) return false;
            t.off = (size_t)a; t.bytes = (size_t)(b - a); out[name] = t;
        }
        ws(); if (js[i] == ',') { i++; continue; }
        if (js[i] == '}') return true;
        return false;
    }
}

struct Layer {
    const uint16_t *in_ln, *post_ln, *wq, *wk, *wv, *wo, *qn, *kn, *wg, *wu, *wd;
};

struct Oracle {
    int mode = 0, max_seq = 0;
    char* map = nullptr; size_t map_bytes = 0;
    const uint16_t *embed = nullptr, *lm = nullptr, *final_ln = nullptr;
    Layer layer[LAYERS];
    std::vector<float> kc, vc;        // [layer][max_seq][KVD] (bf16-valued unless mode 2)
    int float_accum = 0;              // perturbation: single float accumulator in matvec
    int ref_softmax = 0;              // reproduce the reference's softmax reduction (see ref_softmax_rows)
    float* dump = nullptr;            // optional: residual after each layer [LAYERS][DIM]
    float* dump_qkv = nullptr;        // optional: raw q|k|v projections [LAYERS][QD+2*KVD]
};

// y[i] = sum_j W[i][j] * x[j], W bf16 [n][k] row-major; double accumulation
// (g_float_accum: one float accumulator instead, used only to measure how the
// model responds to round-off-sized perturbations).
static int g_float_accum = 0;
void matvec(const uint16_t* W, const float* x, float* y, int n, int k) {
    if (g_float_accum) {
        #pragma omp parallel for schedule(static)
        for (int i = 0; i < n; i++) {
            const uint16_t* w = W + (size_t)i * k; float a = 0.f;
            for (int j = 0; j < k; j++) a += bf2f(w[j]) * x[j];
            y[i] = a;
        }
        return;
    }
    #pragma omp parallel for schedule(static)
    for (int i = 0; i < n; i++) {
        const uint16_t* w = W + (size_t)i * k;
        double acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < k; j += 8)
            for (int e = 0; e < 8; e++) acc[e] += (double)bf2f(w[j + e]) * (double)x[j + e];
        y[i] = (float)(((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7])));
    }
}

// RMSNorm (qwen_model.cuh:133-171).  fp32 mode: double sum, float result.
// bf16 mode: fp32 sum, r = 1/sqrtf(fmaf(ss, 1/DIM, eps)), output rounded to bf16.
void rmsnorm(const float* x, const uint16_t* w, float* y, int n, int mode) {
    if (mode == 0) {
        double ss = 0; for (int j = 0; j < n; j++) ss += (double)x[j] * x[j];
        float r = (float)(1.0 / sqrt(ss / n + (double)EPS));
        for (int j = 0; j < n; j++) y[j] = (x[j] * r) * bf2f(w[j]);
    } else {
        float ss = 0; for (int j = 0; j < n; j++) ss = fmaf(x[j], x[j], ss);
        float r = 1.0f / sqrtf(fmaf(ss, 1.0f / (float)n, EPS));
        for (int j = 0; j < n; j++) y[j] = rbf((x[j] * r) * bf2f(w[j]));
    }
}

// The reference's softmax over len = pos + 1 scores (qwen_model.cuh:486-545):
// len <= 32 runs one thread per head (softmax_kernel_simple, :452-481); longer
// rows run softmax_kernel_optimized (:384-449) with block_size = min(1024, len)
// threads whose shared-memory tree reductions (:412-419, :433-440) halve
// `s` from block_size / 2 and so drop partial results whenever block_size is
// not a power of two.  This restates that arithmetic, dropped terms included,
// so the oracle can be compared with the reference's own output.
void ref_softmax_row(float* sc, int len) {
    if (len <= 32) {
        float m = -INFINITY; for (int i = 0; i < len; i++) m = std::max(m, sc[i]);
        float sum = 0.f; for (int i = 0; i < len; i++) { sc[i] = expf(sc[i] - m); sum += sc[i]; }
        const float inv = 1.0f / sum; for (int i = 0; i < len; i++) sc[i] *= inv;
        return;
    }
    const int bs = std::min(1024, len);
    std::vector<float> part(bs);
    for (int t = 0; t < bs; t++) { float m = -INFINITY; for (int i = t; i < len; i += bs) if (sc[i] > m) m = sc[i]; part[t] = m; }
    for (int st = bs / 2; st > 0; st >>= 1) for (int t = 0; t < st; t++) if (part[t + st] > part[t]) part[t] = part[t + st];
    const float m = part[0];
    for (int t = 0; t < bs; t++) { float a = 0.f; for (int i = t; i < len; i += bs) { sc[i] = expf(sc[i] - m); a += sc[i]; } part[t] = a; }
    for (int st = bs / 2; st > 0; st >>= 1) for (int t = 0; t < st; t++) part[t] += part[t + st];
    const float inv = 1.0f / part[0];
    for (int i = 0; i < len; i++) sc[i] *= inv;
}

}  // namespace

extern "C" {

// cos/sin of the RoPE angle for (pos, j), j in [0, 64) — qwen_model.cuh:331-334.
void oracle_rope_cs(int pos, int j, float* c, float* s) {
    float freq = 1.0f / powf(THETA, (float)(j * 2) / (float)HD);
    float val = (float)pos * freq;
    sincosf(val, s, c);
}

int oracle_open(const char* path, int mode, int max_seq, void** out) {
    *out = nullptr;
    if (max_seq <= 0 || max_seq > 8192 || mode < 0 || mode > 2) return -1;
    int fd = open(path, O_RDONLY); if (fd < 0) return -2;
    struct stat st; if (fstat(fd, &st) != 0) { close(fd); return -2; }
    uint64_t hl = 0; if (pread(fd, &hl, 8, 0) != 8 || 8 + hl > (uint64_t)st.st_size) { close(fd); return -3; }
    char* m = (char*)mmap(nullptr, st.st_size, PROT_READ, MAP_PRIVATE, fd, 0); close(fd);
    if (m == MAP_FAILED) return -2;
    std::map<std::string, TensorLoc> t;
    if (!parse_header(m + 8, hl, t)) { munmap(m, st.st_size); return -4; }
    const char* data = m + 8 + hl; size_t data_bytes = st.st_size - 8 - hl;
    auto get = [&](const std::string& name, size_t bytes) -> const uint16_t* {
        auto it = t.find(name);
        if (it == t.end() || it->second.bytes != bytes || it->second.off + bytes > data_bytes || it->second.dtype != "BF16") return nullptr;
        return (const uint16_t*)(data + it->second.off);
    };
    Oracle* o = new Oracle(); o->mode = mode; o->max_seq = max_seq; o->map = m; o->map_bytes = st.st_size;
    bool ok = true;
    ok &= (o->embed = get("model.embed_tokens.weight", (size_t)VOCAB * DIM * 2)) != nullptr;
    ok &= (o->lm = get("lm_head.weight", (size_t)VOCAB * DIM * 2)) != nullptr;
    ok &= (o->final_ln = get("model.norm.weight", DIM * 2)) != nullptr;
    for (int l = 0; l < LAYERS && ok; l++) {
        std::string p = "model.layers." + std::to_string(l) + ".";
        Layer& L = o->layer[l];
        ok &= (L.in_ln = get(p + "input_layernorm.weight", DIM * 2)) != nullptr;
        ok &= (L.post_ln = get(p + "post_attention_layernorm.weight", DIM * 2)) != nullptr;
        ok &= (L.wq = get(p + "self_attn.q_proj.weight", (size_t)QD * DIM * 2)) != nullptr;
        ok &= (L.wk = get(p + "self_attn.k_proj.weight", (size_t)KVD * DIM * 2)) != nullptr;
        ok &= (L.wv = get(p + "self_attn.v_proj.weight", (size_t)KVD * DIM * 2)) != nullptr;
        ok &= (L.wo = get(p + "self_attn.o_proj.weight", (size_t)DIM * QD * 2)) != nullptr;
        ok &= (L.qn = get(p + "self_attn.q_norm.weight", HD * 2)) != nullptr;
        ok &= (L.kn = get(p + "self_attn.k_norm.weight", HD * 2)) != nullptr;
        ok &= (L.wg = get(p + "mlp.gate_proj.weight", (size_t)HIDDEN * DIM * 2)) != nullptr;
        ok &= (L.wu = get(p + "mlp.up_proj.weight", (size_t)HIDDEN * DIM * 2)) != nullptr;
        ok &= (L.wd = get(p + "mlp.down_proj.weight", (size_t)DIM * HIDDEN * 2)) != nullptr;
    }
    if (!ok) { munmap(m, st.st_size); delete o; return -5; }
    o->kc.assign((size_t)LAYERS * max_seq * KVD, 0);
    o->vc.assign((size_t)LAYERS * max_seq * KVD, 0);
    *out = o;
    return 0;
}

void oracle_close(void* h) {
    Oracle* o = (Oracle*)h; if (!o) return;
    munmap(o->map, o->map_bytes); delete o;
}

void oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int oracle_get_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

// Record the residual stream after every layer into dump[LAYERS][DIM] (NULL = off).
void oracle_set_dump(void* h, float* dump) { ((Oracle*)h)->dump = dump; }
// Fill K/V cache positions [0, n) with seeded N(0, 1) values rounded to bf16:
// lets a timing run decode at context n without computing n prompt positions
// first (the per-token arithmetic is the same; the cache contents differ).
int oracle_fill_kv(void* h, int n, unsigned long long seed) {
    Oracle* o = (Oracle*)h;
    if (!o || n < 0 || n > o->max_seq) return -1;
    for (int l = 0; l < LAYERS; l++)
        for (int t = 0; t < n; t++)
            for (int j = 0; j < KVD; j++) {
                unsigned long long z = seed + ((unsigned long long)((l * o->max_seq + t) * KVD + j) << 1);
                for (int r = 0; r < 2; r++) {
                    z += 0x9E3779B97F4A7C15ull;
                    unsigned long long y = z;
                    y = (y ^ (y >> 30)) * 0xBF58476D1CE4E5B9ull; y = (y ^ (y >> 27)) * 0x94D049BB133111EBull; y ^= y >> 31;
                    const float u = ((float)(y >> 40) + 0.5f) / 16777216.0f - 0.5f;   // uniform, variance 1/12
                    const float v = rbf(u * 3.4641016f);
                    (r == 0 ? o->kc : o->vc)[((size_t)l * o->max_seq + t) * KVD + j] = v;
                }
            }
    return 0;
}

void oracle_set_dump_qkv(void* h, float* dump) { ((Oracle*)h)->dump_qkv = dump; }
void oracle_set_float_accum(void* h, int on) { ((Oracle*)h)->float_accum = on; }
// bf16 mode only: use the reference's softmax reduction (ref_softmax_row).
void oracle_set_ref_softmax(void* h, int on) { ((Oracle*)h)->ref_softmax = on; }

// One decode position (qwen_model.cuh:772-851).  Positions must arrive in order
// 0..pos, as in the reference.  logits: VOCAB floats.  xfinal (optional): the
// normed final hidden state (DIM floats).
int oracle_forward(void* h, int token, int pos, float* logits, float* xfinal) {
    Oracle* o = (Oracle*)h;
    if (!o || token < 0 || token >= VOCAB || pos < 0 || pos >= o->max_seq) return -1;
    const int mode = o->mode == 1 ? 1 : 0;      // mode 2 computes like mode 0
    const bool kv_fp32 = o->mode == 2;
    g_float_accum = o->float_accum;
    std::vector<float> x(DIM), xb(DIM), q(QD), k(KVD), v(KVD), att(QD), hb(HIDDEN), hb2(HIDDEN), tmp(DIM);
    for (int j = 0; j < DIM; j++) x[j] = bf2f(o->embed[(size_t)token * DIM + j]);
    float cs[HD / 2], sn[HD / 2];
    for (int j = 0; j < HD / 2; j++) oracle_rope_cs(pos, j, &cs[j], &sn[j]);
    const int L = pos + 1;

    for (int l = 0; l < LAYERS; l++) {
        const Layer& W = o->layer[l];
        rmsnorm(x.data(), W.in_ln, xb.data(), DIM, mode);
        matvec(W.wq, xb.data(), q.data(), QD, DIM);
        matvec(W.wk, xb.data(), k.data(), KVD, DIM);
        matvec(W.wv, xb.data(), v.data(), KVD, DIM);
        if (o->dump_qkv) {
            float* d = o->dump_qkv + (size_t)l * (QD + 2 * KVD);
            memcpy(d, q.data(), QD * 4); memcpy(d + QD, k.data(), KVD * 4); memcpy(d + QD + KVD, v.data(), KVD * 4);
        }
        if (mode == 1) { for (auto& a : q) a = rbf(a); for (auto& a : k) a = rbf(a); for (auto& a : v) a = rbf(a); }
        // QK-norm (per head) then RoPE
        auto headnorm = [&](float* vec, const uint16_t* g) {
            if (mode == 0) {
                double ss = 0; for (int d = 0; d < HD; d++) ss += (double)vec[d] * vec[d];
                float r = (float)(1.0 / sqrt(ss / HD + (double)EPS));
                for (int d = 0; d < HD; d++) vec[d] = (vec[d] * r) * bf2f(g[d]);
            } else {
                float ss = 0; for (int d = 0; d < HD; d++) ss += vec[d] * vec[d];
                float r = 1.0f / sqrtf(ss * (1.0f / HD) + EPS);
                for (int d = 0; d < HD; d++) vec[d] = rbf((vec[d] * r) * bf2f(g[d]));
            }
        };
        auto rope = [&](float* vec) {
            for (int j = 0; j < HD / 2; j++) {
                float a = vec[j], b = vec[j + HD / 2];
                float ra = a * cs[j] - b * sn[j], rb = a * sn[j] + b * cs[j];
                if (mode == 1) { ra = rbf(ra); rb = rbf(rb); }
                vec[j] = ra; vec[j + HD / 2] = rb;
            }
        };
        for (int hh = 0; hh < NH; hh++) { headnorm(&q[hh * HD], W.qn); rope(&q[hh * HD]); }
        for (int hh = 0; hh < NKV; hh++) { headnorm(&k[hh * HD], W.kn); rope(&k[hh * HD]); }
        float* kc = &o->kc[((size_t)l * o->max_seq + pos) * KVD];
        float* vc = &o->vc[((size_t)l * o->max_seq + pos) * KVD];
        for (int j = 0; j < KVD; j++) { kc[j] = kv_fp32 ? k[j] : rbf(k[j]); vc[j] = kv_fp32 ? v[j] : rbf(v[j]); }
        // attention: 16 query heads, kv head = h / 2
        const float* Kl = &o->kc[(size_t)l * o->max_seq * KVD];
        const float* Vl = &o->vc[(size_t)l * o->max_seq * KVD];
        #pragma omp parallel for schedule(static)
        for (int hh = 0; hh < NH; hh++) {
            const int g = hh / (NH / NKV);
            const float* qh = &q[hh * HD];
            std::vector<float> s(L);
            for (int t = 0; t < L; t++) {
                const float* kt = Kl + (size_t)t * KVD + g * HD;
                float sc;
                if (mode == 0) { double a = 0; for (int d = 0; d < HD; d++) a += (double)qh[d] * kt[d]; sc = (float)a; }
                else { float a = 0; for (int d = 0; d < HD; d++) a = fmaf(qh[d], kt[d], a); sc = a; }
                s[t] = sc / sqrtf((float)HD);
            }
            float m = -INFINITY; for (int t = 0; t < L; t++) m = std::max(m, s[t]);
            if (mode == 0) {
                double sum = 0; for (int t = 0; t < L; t++) { s[t] = (float)exp((double)s[t] - m); sum += s[t]; }
                for (int t = 0; t < L; t++) s[t] = (float)(s[t] / sum);
                for (int d = 0; d < HD; d++) {
                    double a = 0; for (int t = 0; t < L; t++) a += (double)s[t] * Vl[(size_t)t * KVD + g * HD + d];
                    att[hh * HD + d] = (float)a;
                }
            } else {
                if (o->ref_softmax) ref_softmax_row(s.data(), L);
                else {
                    float sum = 0; for (int t = 0; t < L; t++) { s[t] = expf(s[t] - m); sum += s[t]; }
                    float inv = 1.0f / sum; for (int t = 0; t < L; t++) s[t] *= inv;
                }
                for (int d = 0; d < HD; d++) {
                    float a = 0; for (int t = 0; t < L; t++) a = fmaf(s[t], Vl[(size_t)t * KVD + g * HD + d], a);
                    att[hh * HD + d] = rbf(a);
                }
            }
        }
        // O projection with residual (beta = 1)
        matvec(W.wo, att.data(), tmp.data(), DIM, QD);
        for (int j = 0; j < DIM; j++) x[j] = mode == 0 ? x[j] + tmp[j] : rbf(tmp[j] + x[j]);
        // MLP
        rmsnorm(x.data(), W.post_ln, xb.data(), DIM, mode);
        matvec(W.wg, xb.data(), hb.data(), HIDDEN, DIM);
        matvec(W.wu, xb.data(), hb2.data(), HIDDEN, DIM);
        for (int j = 0; j < HIDDEN; j++) {
            float gt = hb[j], up = hb2[j];
            if (mode == 1) { gt = rbf(gt); up = rbf(up); }
            float sv = mode == 0 ? (float)((double)gt / (1.0 + exp(-(double)gt))) : gt * (1.0f / (1.0f + expf(-gt)));
            hb[j] = mode == 0 ? sv * up : rbf(sv * up);
        }
        matvec(W.wd, hb.data(), tmp.data(), DIM, HIDDEN);
        for (int j = 0; j < DIM; j++) x[j] = mode == 0 ? x[j] + tmp[j] : rbf(tmp[j] + x[j]);
        if (o->dump) memcpy(o->dump + (size_t)l * DIM, x.data(), DIM * sizeof(float));
    }
    rmsnorm(x.data(), o->final_ln, xb.data(), DIM, mode);
    if (xfinal) memcpy(xfinal, xb.data(), DIM * sizeof(float));
    if (logits) {
        matvec(o->lm, xb.data(), logits, VOCAB, DIM);
        if (mode == 1) for (int i = 0; i < VOCAB; i++) logits[i] = rbf(logits[i]);
    }
    return 0;
}

// Plain bf16 GEMV y = bf16(W x) with double accumulation (the isolated GEMV
// sweep's math: bf16 in, fp32-or-better accumulate, bf16 out).
void oracle_gemv_bf16(const uint16_t* W, const uint16_t* x, uint16_t* y, int n, int k) {
    std::vector<float> xf(k); for (int j = 0; j < k; j++) xf[j] = bf2f(x[j]);
    std::vector<float> yf(n); matvec(W, xf.data(), yf.data(), n, k);
    for (int i = 0; i < n; i++) y[i] = f2bf(yf[i]);
}

// ---------------------------------------------------------------------------
// Sampler (sampler.h:27-175), restated.
// ---------------------------------------------------------------------------
struct PI { float p; int i; };

static unsigned int xs_u32(unsigned long long* s) {       // xorshift64* (sampler.h:27-32)
    *s ^= *s >> 12; *s ^= *s << 25; *s ^= *s >> 27;
    return (unsigned int)((*s * 0x2545F4914F6CDD1DULL) >> 32);
}
static float xs_f32(unsigned long long* s) { return (xs_u32(s) >> 8) / 16777216.0f; }   // sampler.h:34-38

unsigned int oracle_random_u32(unsigned long long* s) { return xs_u32(s); }
float oracle_random_f32(unsigned long long* s) { return xs_f32(s); }

// Hoare's FIND (quickselect), the partition scheme of sampler.h:54-79: after it
// the k largest entries occupy [0, k) in partition order.
static void hoare_select(PI* a, int n, int k) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const float pv = a[k].p;
        int i = lo, j = hi;
        do {
            while (a[i].p > pv) i++;
            while (a[j].p < pv) j--;
            if (i <= j) { PI t = a[i]; a[i] = a[j]; a[j] = t; i++; j--; }
        } while (i <= j);
        if (j < k) lo = i;
        if (i > k) hi = j;
    }
}
static int desc_cmp(const void* x, const void* y) {      // sampler.h:41-51
    float a = ((const PI*)x)->p, b = ((const PI*)y)->p;
    return a > b ? -1 : (a < b ? 1 : 0);
}

// order_mode 0: candidates are scanned in the reference's order (quickselect
// order when top-p is off, qsort order when on).  order_mode 1: candidates are
// scanned by descending probability, ties by ascending index (the device
// sampler's documented order).
int oracle_sample(const float* logits, int n, float temperature, float topp, int top_k,
                  unsigned long long* rng, int order_mode) {
    if (top_k == 0) top_k = n;                                   // sampler.h:109
    if (temperature == 0.0f || top_k == 1) {                     // sampler.h:125-128, 82-97
        int mi = 0; float mp = logits[0];
        for (int i = 1; i < n; i++) if (logits[i] > mp) { mi = i; mp = logits[i]; }
        return mi;
    }
    std::vector<PI> pi(n);
    for (int i = 0; i < n; i++) { pi[i].p = logits[i]; pi[i].i = i; }
    int nc = top_k < n ? top_k : n;
    // With nc == n the reference's quick_select reads its pivot one past the end
    // (sampler.h:63 with k = n) and does not terminate; every entry is a
    // candidate then, kept in index order.
    if (nc < n) hoare_select(pi.data(), n, nc);
    if (order_mode == 1) {
        std::sort(pi.begin(), pi.begin() + nc, [](const PI& a, const PI& b) { return a.p > b.p || (a.p == b.p && a.i < b.i); });
    }
    float mx = pi[0].p; for (int i = 1; i < nc; i++) if (pi[i].p > mx) mx = pi[i].p;
    float sum = 0.0f;
    for (int i = 0; i < nc; i++) { float e = expf((pi[i].p - mx) / temperature); pi[i].p = e; sum += e; }
    for (int i = 0; i < nc; i++) pi[i].p /= sum;
    if (topp > 0.0f && topp < 1.0f) {
        if (order_mode == 0) qsort(pi.data(), nc, sizeof(PI), desc_cmp);
        float cum = 0.0f; int last = nc - 1;
        for (int i = 0; i < nc; i++) { cum += pi[i].p; if (cum > topp) { last = i; break; } }
        nc = last + 1; sum = cum;
    }
    float coin = xs_f32(rng) * sum;
    float cdf = 0.0f;
    for (int i = 0; i < nc; i++) { cdf += pi[i].p; if (coin < cdf) return pi[i].i; }
    return pi[nc - 1].i;
}

// ---------------------------------------------------------------------------
// Synthetic checkpoint writer, so that bench.py's reference arm (the timed CPU
// baseline) obtains its weights without the product library.  It writes the
// same safetensors file as the library's qwen_write_synthetic_checkpoint (a
// CPU test compares the two byte for byte): tensors in byte-sorted name order
// packed from offset 0 (the layout of the reference's TENSOR_METADATA,
// static_loader.h:80-400), every matrix N(0, 0.02) in bf16 by Box-Muller on
// splitmix64 uniforms keyed on the seed and the tensor name (FNV-1a), every
// 1-D gain 1.0, lm_head a copy of the embedding (tied weights).
// ---------------------------------------------------------------------------
static uint64_t sm64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

int oracle_write_synthetic(const char* path, unsigned long long seed) {
    struct T { std::string name; std::vector<int64_t> shape; size_t bytes = 0, off = 0; };
    std::vector<T> t;
    auto add = [&](const std::string& n, std::vector<int64_t> sh) {
        T x; x.name = n; x.shape = sh; size_t e = 1; for (auto d : sh) e *= (size_t)d; x.bytes = 2 * e; t.push_back(x);
    };
    add("lm_head.weight", {VOCAB, DIM});
    add("model.embed_tokens.weight", {VOCAB, DIM});
    add("model.norm.weight", {DIM});
    for (int l = 0; l < LAYERS; l++) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        add(p + "input_layernorm.weight", {DIM});
        add(p + "mlp.down_proj.weight", {DIM, HIDDEN});
        add(p + "mlp.gate_proj.weight", {HIDDEN, DIM});
        add(p + "mlp.up_proj.weight", {HIDDEN, DIM});
        add(p + "post_attention_layernorm.weight", {DIM});
        add(p + "self_attn.k_norm.weight", {HD});
        add(p + "self_attn.k_proj.weight", {KVD, DIM});
        add(p + "self_attn.o_proj.weight", {DIM, QD});
        add(p + "self_attn.q_norm.weight", {HD});
        add(p + "self_attn.q_proj.weight", {QD, DIM});
        add(p + "self_attn.v_proj.weight", {KVD, DIM});
    }
    std::sort(t.begin(), t.end(), [](const T& a, const T& b) { return a.name < b.name; });
    size_t total = 0;
    for (auto& x : t) { x.off = total; total += x.bytes; }
    std::string js = "{\"__metadata__\":{\"format\":\"pt\",\"generator\":\"qwen_b200 synthetic N(0,0.02) seed " + std::to_string(seed) + "\"}";
    for (const auto& x : t) {
        js += ",\"" + x.name + "\":{\"dtype\":\"BF16\",\"shape\":[";
        for (size_t k = 0; k < x.shape.size(); k++) js += (k ? "," : "") + std::to_string(x.shape[k]);
        js += "],\"data_offsets\":[" + std::to_string(x.off) + "," + std::to_string(x.off + x.bytes) + "]}";
    }
    js += "}";
    while ((8 + js.size()) % 256) js.push_back(' ');
    const uint64_t hl = js.size();
    const size_t file_bytes = 8 + hl + total;
    const std::string tmp = std::string(path) + ".oracle-partial";
    int fd = open(tmp.c_str(), O_RDWR | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) return -1;
    if (ftruncate(fd, (off_t)file_bytes) != 0) { close(fd); return -1; }
    char* m = (char*)mmap(nullptr, file_bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    close(fd);
    if (m == MAP_FAILED) return -1;
    memcpy(m, &hl, 8);
    memcpy(m + 8, js.data(), hl);
    char* data = m + 8 + hl;
    size_t emb_off = 0, lm_off = 0, emb_bytes = 0;
    for (const auto& x : t) {
        if (x.name == "model.embed_tokens.weight") { emb_off = x.off; emb_bytes = x.bytes; }
        if (x.name == "lm_head.weight") { lm_off = x.off; continue; }
        uint16_t* dst = (uint16_t*)(data + x.off);
        const int64_t n = (int64_t)(x.bytes / 2);
        if (x.shape.size() == 1) { for (int64_t i = 0; i < n; i++) dst[i] = 0x3F80; continue; }
        uint64_t h = 1469598103934665603ull;
        for (char ch : x.name) { h ^= (uint8_t)ch; h *= 1099511628211ull; }
        const uint64_t key = sm64(seed ^ sm64(h));
        #pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < n / 2; i++) {
            const uint64_t a = sm64(key + 2 * (uint64_t)i), b = sm64(key + 2 * (uint64_t)i + 1);
            const double u1 = ((double)(a >> 11) + 0.5) * (1.0 / 9007199254740992.0);
            const double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
            const double r = sqrt(-2.0 * log(u1)), th = 6.283185307179586 * u2;
            dst[2 * i] = f2bf((float)(0.02 * r * cos(th)));
            dst[2 * i + 1] = f2bf((float)(0.02 * r * sin(th)));
        }
    }
    memcpy(data + lm_off, data + emb_off, emb_bytes);
    const int ok = msync(m, file_bytes, MS_SYNC) == 0;
    munmap(m, file_bytes);
    if (!ok || rename(tmp.c_str(), path) != 0) return -1;
    return 0;
}

}  // extern "C"
